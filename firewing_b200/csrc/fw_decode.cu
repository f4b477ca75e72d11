// fw_decode.cu -- decode-width (T <= 256) sparse-MoE block kernels for sm_100a.
//
// Pipeline per layer (one stream, programmatic dependent launch between
// kernels):
//   k_rows_dot       router logits [T][E] (+ shared-gate logit) -- exact GEMV
//   k_route_permute  f32 softmax, top-k, renormalised scores, sigmoid gate,
//                    per-expert pair lists (one CTA)
//   k_experts        (fw_experts.cu) gate_up + SwiGLU and down + route-weight
//                    scale for every active expert and the shared expert
//   k_combine        ascending-expert bf16 accumulation + gated shared add
//
// Every GEMV reproduces the reference's f32 reduction order exactly
// (src/expert.rs:514-552): a row's 32 partial sums are held 8 per lane by
// 4 lanes, each walking the 32-column blocks in order, then reduced with the
// reference tree (fw::reduce_partials).  Rows are streamed once per CTA with
// 16-byte read-only loads; activations sit in shared memory as f32.
#include <algorithm>
#include <cfloat>
#include <cstdint>

#include "fw_common.cuh"
#include "fw_kernels.h"

namespace fw {
namespace {

constexpr int kTG = 8;  // tokens per pass over a weight row

// ---------------------------------------------------------------------------
// Exact GEMV core: this lane's 4-lane group owns one row; NT tokens.
// xs: shared f32 activations [NT][xs_stride]; cols % 32 == 0.
// Result (valid in lane q == 0 of the group) is the f32 dot per token.
template <int NT>
__device__ __forceinline__ void group_row_dot(const uint16_t* __restrict__ row_ptr,
                                              const float* __restrict__ xs, int xs_stride,
                                              int cols, int q, float (&out)[kTG]) {
  float acc[NT][8];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[t][i] = 0.0f;
  const int nb = cols >> 5;
  const uint16_t* p = row_ptr + q * 8;
  const float* xq = xs + q * 8;
  constexpr int U = 8;
  int b = 0;
  for (; b + U <= nb; b += U) {
    uint4 w[U];
#pragma unroll
    for (int u = 0; u < U; ++u) w[u] = ldg_stream(p + (b + u) * 32);
#pragma unroll
    for (int u = 0; u < U; ++u) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const float* xr = xq + t * xs_stride + (b + u) * 32;
        fma8(w[u], *reinterpret_cast<const float4*>(xr), *reinterpret_cast<const float4*>(xr + 4),
             acc[t]);
      }
    }
  }
  for (; b < nb; ++b) {
    const uint4 w = ldg_stream(p + b * 32);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float* xr = xq + t * xs_stride + b * 32;
      fma8(w, *reinterpret_cast<const float4*>(xr), *reinterpret_cast<const float4*>(xr + 4),
           acc[t]);
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) out[t] = reduce_partials(acc[t]);
}

__device__ __forceinline__ void dispatch_row_dot(int nt, const uint16_t* row_ptr, const float* xs,
                                                 int xs_stride, int cols, int q,
                                                 float (&out)[kTG]) {
  if (nt <= 1)
    group_row_dot<1>(row_ptr, xs, xs_stride, cols, q, out);
  else if (nt <= 2)
    group_row_dot<2>(row_ptr, xs, xs_stride, cols, q, out);
  else if (nt <= 4)
    group_row_dot<4>(row_ptr, xs, xs_stride, cols, q, out);
  else
    group_row_dot<8>(row_ptr, xs, xs_stride, cols, q, out);
}

__device__ __forceinline__ int round_nt(int nt) { return nt <= 1 ? 1 : nt <= 2 ? 2 : nt <= 4 ? 4 : 8; }

// Stage `nt` bf16 rows (row r at src_row(r)) of `cols` values into shared f32,
// zero-filling rows nt..round_nt(nt)-1.
template <typename RowFn>
__device__ __forceinline__ void stage_rows_f32(float* xs, int cols, int nt, RowFn src_row) {
  const int nt_pad = round_nt(nt);
  const int per_row = cols >> 3;
  for (int i = threadIdx.x; i < nt_pad * per_row; i += blockDim.x) {
    const int r = i / per_row, c = (i - r * per_row) * 8;
    float4 a, b;
    if (r < nt) {
      const uint4 v = *reinterpret_cast<const uint4*>(src_row(r) + c);
      a = make_float4(lo_bf16(v.x), hi_bf16(v.x), lo_bf16(v.y), hi_bf16(v.y));
      b = make_float4(lo_bf16(v.z), hi_bf16(v.z), lo_bf16(v.w), hi_bf16(v.w));
    } else {
      a = b = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    *reinterpret_cast<float4*>(xs + r * cols + c) = a;
    *reinterpret_cast<float4*>(xs + r * cols + c + 4) = b;
  }
}

// ---------------------------------------------------------------------------
// out[t][r] = bf16(dot(W[r], x[t])) for r < rows (linear_bf16,
// src/expert.rs:554-560), optional bias (f32, re-rounded), and an optional
// extra row (the shared-expert gate vector) written to extra_out[t].
struct RowsDotArgs {
  const uint16_t* w;
  int rows, cols, T;
  const uint16_t* x;  // [T][cols]
  uint16_t* out;      // [T][rows]
  const float* bias;  // [rows] or null
  const uint16_t* extra_row;  // [cols] or null
  uint16_t* extra_out;        // [T]
};

constexpr int kRowsPerDotCta = 16;  // 2 warps x 8 rows

__global__ void __launch_bounds__(64) k_rows_dot(RowsDotArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ float xs[];
  const int t0 = blockIdx.y * kTG;
  const int nt = min(kTG, a.T - t0);
  if (nt <= 0) return;
  stage_rows_f32(xs, a.cols, nt, [&](int r) { return a.x + static_cast<size_t>(t0 + r) * a.cols; });
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int total_rows = a.rows + (a.extra_row != nullptr ? 1 : 0);
  const int row = blockIdx.x * kRowsPerDotCta + warp * 8 + g;
  const bool valid = row < total_rows;
  const uint16_t* row_ptr = (row < a.rows) ? a.w + static_cast<size_t>(row) * a.cols
                                           : (valid ? a.extra_row : a.w);
  float val[kTG];
  dispatch_row_dot(nt, row_ptr, xs, a.cols, a.cols, q, val);
  if (q == 0 && valid) {
    for (int t = 0; t < nt; ++t) {
      uint16_t v = f32_to_bf16(val[t]);
      if (row < a.rows) {
        if (a.bias != nullptr) v = f32_to_bf16(bf16_to_f32(v) + a.bias[row]);
        a.out[static_cast<size_t>(t0 + t) * a.rows + row] = v;
      } else {
        a.extra_out[t0 + t] = v;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Router logits for the block: rows = the E router rows plus the shared-expert
// gate vector as row E; grid = (row groups of kRouterRows, token groups of
// 8).  A CTA bulk-copies its rows into shared memory -- issued before the
// grid-dependency wait, since weights do not depend on the previous kernel --
// and its tokens' contiguous [8][H] activation tile after it.  Warp w owns
// row w; lane j owns partial j (columns j, j+32, ... in order,
// src/expert.rs:514-552) for the 8 tokens, reading both operands as bf16
// from shared memory (conflict-free: a warp reads 64 contiguous bytes).
constexpr int kRouterRows = 8;    // rows (= warps) per CTA
constexpr int kRouterTokens = 8;  // tokens per CTA

struct RouterArgs {
  const uint16_t* wpm;        // [E+1][H] partial-major copy of w and extra_row, or null
  const uint16_t* w;          // [E][H]
  const uint16_t* extra_row;  // [H] shared-expert gate vector
  const float* bias;          // [E] or null
  const uint16_t* x;          // [T][H]
  uint16_t* logits;           // [T][E]
  uint16_t* extra_out;        // [T]
  int E, H, T;
  int* err;
};

// Reference tree over the 32 lanes' partials; result valid in lane 0.
__device__ __forceinline__ float warp_reduce_ref(float p) {
  p += __shfl_down_sync(0xffffffffu, p, 16);
  p += __shfl_down_sync(0xffffffffu, p, 8);
  p += __shfl_down_sync(0xffffffffu, p, 4);
  const float q = p + __shfl_down_sync(0xffffffffu, p, 1);  // lanes 0, 2: (0+1), (2+3)
  return q + __shfl_down_sync(0xffffffffu, q, 2);
}

__global__ void __launch_bounds__(kRouterRows * 32) k_router(RouterArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint16_t* rows = reinterpret_cast<uint16_t*>(smem);                                   // [kRouterRows][H]
  uint16_t* xt = rows + kRouterRows * a.H;                                              // [kRouterTokens][H]
  uint64_t* bars = reinterpret_cast<uint64_t*>(xt + kRouterTokens * a.H);              // [2]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kRouterRows;
  const int nrows = min(kRouterRows, a.E + 1 - row0);
  const int t0 = blockIdx.y * kRouterTokens;
  const int nt = min(kRouterTokens, a.T - t0);
  const uint32_t row_bytes = static_cast<uint32_t>(a.H) * 2;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bars[0], row_bytes * nrows);
    const uint64_t policy = l2_evict_first_policy();
    for (int r = 0; r < nrows; ++r) {
      const int row = row0 + r;
      const uint16_t* src = row < a.E ? a.w + static_cast<size_t>(row) * a.H : a.extra_row;
      bulk_g2s(rows + r * a.H, src, row_bytes, &bars[0], policy);
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bars[1], row_bytes * nt);
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(xt)),
        "l"(a.x + static_cast<size_t>(t0) * a.H), "r"(row_bytes * nt), "r"(smem_u32(&bars[1]))
        : "memory");
  }
  __syncthreads();  // barrier initialisation visible to all threads
  const bool ok = mbar_wait_bounded(&bars[0], 0, 2000000000ull) && mbar_wait_bounded(&bars[1], 0, 2000000000ull);
  if (!ok) {
    if (lane == 0) set_error(a.err, kErrTimeout);
    return;
  }
  if (warp >= nrows) return;
  const uint16_t* wr = rows + warp * a.H + lane;
  const uint16_t* xr = xt + lane;
  float acc[kRouterTokens];
#pragma unroll
  for (int t = 0; t < kRouterTokens; ++t) acc[t] = 0.0f;
  const int nb = a.H >> 5;
#pragma unroll 4
  for (int b = 0; b < nb; ++b) {
    const float wv = bf16_to_f32(wr[b * 32]);
#pragma unroll
    for (int t = 0; t < kRouterTokens; ++t)
      if (t < nt) acc[t] = fmaf(wv, bf16_to_f32(xr[t * a.H + b * 32]), acc[t]);
  }
  const int row = row0 + warp;
#pragma unroll
  for (int t = 0; t < kRouterTokens; ++t) {
    const float dot = warp_reduce_ref(acc[t]);
    if (lane == 0 && t < nt) {
      uint16_t v = f32_to_bf16(dot);
      if (row < a.E) {
        // build-defined extension: f32 logit bias, re-rounded to bf16
        if (a.bias != nullptr) v = f32_to_bf16(bf16_to_f32(v) + a.bias[row]);
        a.logits[static_cast<size_t>(t0 + t) * a.E + row] = v;
      } else {
        a.extra_out[t0 + t] = v;
      }
    }
  }
}


// The router on the partial-major copy of the router rows (element
// (row, j, i) = row[j + 32 i]; row E the shared gate vector), for H a
// multiple of 256 (launched for single-token forwards).  A CTA of 4
// warps covers 4 * RW rows x TT tokens; warp w rows RW*w..RW*w+RW-1 of the
// tile.  With RW = 1 the E + 1 rows spread over ~130 CTAs, so each SM
// copies and reduces only 16 KB of router weights.  The CTA's rows are copied into
// shared memory with cp.async before the grid-dependency wait (they do not
// depend on the previous kernel), the tokens after it; both tiles are laid
// out partial-major with lane blocks padded to an odd number of 16-byte
// chunks, so a quarter-warp's 16-byte reads hit distinct banks.  Lane j owns
// partial j: its columns j, j+32, ... come as chunks of 8 in column order,
// each added with 8 sequential mixed-precision FMAs -- the reference
// schedule exactly -- then its tree.
constexpr int kPmWarps = 4;

__host__ __device__ inline int pm_stride(int H) {
  const int nch = H / 256;
  return nch + 1 + (nch & 1);
}

__device__ __forceinline__ void cp_async16_dec(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

template <int TT, int RW>
__device__ __forceinline__ void router_pm_body(const RouterArgs& a) {
  constexpr int kPmRows = kPmWarps * RW;
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = a.H >> 8, S = pm_stride(a.H), per = a.H >> 5;
  uint4* ws = reinterpret_cast<uint4*>(smem);  // [kPmRows][32 lane blocks][S chunks]
  uint4* xs = ws + kPmRows * 32 * S;            // [TT][32 lane blocks][S chunks]
  const int rbase = blockIdx.x * kPmRows;
  const int nrows = min(kPmRows, a.E + 1 - rbase);
  const int row0 = rbase + warp * RW;
  const int t0 = blockIdx.y * TT;
  const int nt = min(TT, a.T - t0);
  for (int g = threadIdx.x; g < nrows * 32 * nch; g += blockDim.x) {
    const int r = g / (32 * nch), rem = g - r * 32 * nch, j = rem / nch, q = rem - j * nch;
    cp_async16_dec(ws + (r * 32 + j) * S + q, a.wpm + static_cast<size_t>(rbase + r) * a.H + j * per + q * 8);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  pdl_wait();  // the token rows may be the previous kernel's output
  pdl_launch_dependents();
  // Token chunk (t, j, q): columns j + 32 (8q + e), e = 0..7, gathered with
  // 2-byte loads (coalesced over j) into one 16-byte shared store.
  for (int g = threadIdx.x; g < TT * 32 * nch; g += blockDim.x) {
    const int t = g / (32 * nch), rem = g - t * 32 * nch, q = rem >> 5, j = rem & 31;
    uint32_t v[4] = {0u, 0u, 0u, 0u};
    if (t < nt) {
      const uint16_t* src = a.x + static_cast<size_t>(t0 + t) * a.H + 256 * q + j;
#pragma unroll
      for (int e = 0; e < 4; ++e)
        v[e] = static_cast<uint32_t>(src[64 * e]) | (static_cast<uint32_t>(src[64 * e + 32]) << 16);
    }
    xs[(t * 32 + j) * S + q] = make_uint4(v[0], v[1], v[2], v[3]);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  const uint4* wr[RW];
#pragma unroll
  for (int r = 0; r < RW; ++r) {
    const int lr = min(warp * RW + r, nrows - 1);  // rows past E repeat the last and are not stored
    wr[r] = ws + (lr * 32 + lane) * S;
  }
  float acc[RW][TT];
#pragma unroll
  for (int r = 0; r < RW; ++r)
#pragma unroll
    for (int t = 0; t < TT; ++t) acc[r][t] = 0.0f;
  for (int q = 0; q < nch; ++q) {
    uint4 w[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) w[r] = wr[r][q];
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      const uint4 xv = xs[(t * 32 + lane) * S + q];
#pragma unroll
      for (int r = 0; r < RW; ++r) {
        acc[r][t] = fma_seq2(w[r].x, xv.x, acc[r][t]);
        acc[r][t] = fma_seq2(w[r].y, xv.y, acc[r][t]);
        acc[r][t] = fma_seq2(w[r].z, xv.z, acc[r][t]);
        acc[r][t] = fma_seq2(w[r].w, xv.w, acc[r][t]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RW; ++r) {
    const int row = row0 + r;
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      const float dot = warp_reduce_ref(acc[r][t]);
      if (lane == 0 && t < nt && row <= a.E) {
        uint16_t v = f32_to_bf16(dot);
        if (row < a.E) {
          // build-defined extension: f32 logit bias, re-rounded to bf16
          if (a.bias != nullptr) v = f32_to_bf16(bf16_to_f32(v) + a.bias[row]);
          a.logits[static_cast<size_t>(t0 + t) * a.E + row] = v;
        } else {
          a.extra_out[t0 + t] = v;
        }
      }
    }
  }
}

template <int TT, int RW>
__global__ void __launch_bounds__(kPmWarps * 32) k_router_pm(RouterArgs a) {
  router_pm_body<TT, RW>(a);
}

// ---------------------------------------------------------------------------
// Route (src/decoder_layer.rs:278-307) + permute.  One CTA per token, one
// thread per expert.  The CTA that finishes last (atomic ticket) builds the
// expert schedule for the expert kernel.
struct RouteArgs {
  const uint16_t* logits;  // [T][E]
  int T, E, K;
  int32_t* idx;            // [T][K] selection in top-k order
  uint16_t* score;         // [T][K] bf16 renormalised scores
  int* err;
  // Block-only extras (null when routing standalone)
  const uint16_t* sh_logit;  // [T]
  const uint16_t* sig_lut;
  uint16_t* sh_sig;          // [T]
  int32_t* sorted_slot;      // [T][K]
  int32_t* sched;            // schedule words (see fw_kernels.h)
  int* up_done;              // [E+1] expert-kernel slot counters to zero
  int tgp, qpr, qps, ops;    // expert-kernel pass size, quads/octets per slot
  int* ticket;               // CTA completion counter (zero between calls)
  int* pair_count;           // [E] prefill path: per-expert pair counts to add into (or null)
  // Schedule scope: routed experts e with e % ep_world == ep_rank (expert
  // parallelism: this GPU's experts), and the shared expert over sh_T tokens.
  int ep_rank, ep_world, sh_T;
};

// f32 total-order key with the index folded in (higher logit, then lower
// index, wins), as src/router.rs:241-247 orders the selection.
__device__ __forceinline__ float key_value(uint32_t key) {
  const uint32_t k16 = key >> 16;
  const uint32_t bits = (k16 & 0x8000u) ? (k16 & 0x7fffu) : (~k16 & 0xffffu);
  return bf16_to_f32(bits);
}

// Block-wide exclusive scan of two values per thread (blockDim.x <= 1024);
// wsum holds 64 ints.  Returns exclusive prefixes, totals via *tot_a/b.
__device__ __forceinline__ void block_scan2(int va, int vb, int& ea, int& eb, int* wsum, int& tot_a, int& tot_b) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  int ia = va, ib = vb;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ya = __shfl_up_sync(0xffffffffu, ia, o);
    const int yb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) {
      ia += ya;
      ib += yb;
    }
  }
  __syncthreads();
  if (lane == 31) {
    wsum[warp] = ia;
    wsum[32 + warp] = ib;
  }
  __syncthreads();
  if (warp == 0) {
    const int sa0 = lane < nw ? wsum[lane] : 0, sb0 = lane < nw ? wsum[32 + lane] : 0;
    int sa = sa0, sb = sb0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ya = __shfl_up_sync(0xffffffffu, sa, o);
      const int yb = __shfl_up_sync(0xffffffffu, sb, o);
      if (lane >= o) {
        sa += ya;
        sb += yb;
      }
    }
    wsum[lane] = sa - sa0;
    wsum[32 + lane] = sb - sb0;
    if (lane == 31) {
      wsum[64] = sa;
      wsum[65] = sb;
    }
  }
  __syncthreads();
  ea = wsum[warp] + ia - va;
  eb = wsum[32 + warp] + ib - vb;
  tot_a = wsum[64];
  tot_b = wsum[65];
  __syncthreads();
}

// The expert schedule (see fw_kernels.h) from all T*K selections.
__device__ void build_schedule(const RouteArgs& a, unsigned char* smem) {
  const int E = a.E, K = a.K, T = a.T, P = T * K;
  const int W = (T + 63) >> 6;  // 64-bit token masks per expert
  int32_t* pidx = reinterpret_cast<int32_t*>(smem);
  unsigned long long* mask = reinterpret_cast<unsigned long long*>(pidx + ((P + 1) & ~1));
  int* cnt = reinterpret_cast<int*>(mask + static_cast<size_t>(E) * W);
  int* poff = cnt + E;
  int* wsum = poff + E;  // 66 ints
  for (int p = threadIdx.x; p < P; p += blockDim.x) pidx[p] = __ldcg(a.idx + p);
  for (int i = threadIdx.x; i < E * W; i += blockDim.x) mask[i] = 0ull;
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  for (int i = threadIdx.x; i <= E; i += blockDim.x) a.up_done[i] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const int e = pidx[p];
    if (e % a.ep_world != a.ep_rank) continue;  // another GPU's expert
    const int t = p / K;
    atomicAdd(&cnt[e], 1);
    atomicOr(&mask[e * W + (t >> 6)], 1ull << (t & 63));
  }
  __syncthreads();
  int32_t* active = a.sched + 1;
  int32_t* offsets = a.sched + 1 + E;
  int32_t* pairs = a.sched + 2 + 2 * E;
  int32_t* up_pref = pairs + P;
  int32_t* dn_pref = up_pref + E + 2;
  // thread e owns expert e (blockDim.x >= E)
  const int e = threadIdx.x;
  const int c = e < E ? cnt[e] : 0;
  const int f = c > 0 ? 1 : 0;
  int slot, off, n_act, n_pairs;
  block_scan2(f, c, slot, off, wsum, n_act, n_pairs);
  if (e < E) {
    poff[e] = off;
    if (f) {
      active[slot] = e;
      offsets[slot] = off;
    }
  }
  if (threadIdx.x == 0) {
    a.sched[0] = n_act;
    offsets[n_act] = n_pairs;
  }
  // Cost prefixes for the expert kernel.  A slot of n tokens has
  // ceil(n / tgp) token passes of qpr quads (up) and ops octets (down).  A
  // unit of a pass with nt tokens costs 4 + pad(nt) in the up phase and
  // 4 + 4 pad(nt) in the down phase (pad = 1, 2, 4, 8: the tokens the
  // kernel computes): both weigh the unit's bytes against its FMAs and
  // reductions, which a down unit (one stage) pays per stage.
  const int nfull = f ? c / a.tgp : 0, rem = f ? c % a.tgp : 0;
  const int pad = rem <= 1 ? rem : rem <= 2 ? 2 : rem <= 4 ? 4 : 8;
  const int pcu = nfull * (4 + a.tgp) + (rem ? 4 + pad : 0);
  const int pcd = nfull * (4 + 4 * a.tgp) + (rem ? 4 + 4 * pad : 0);
  int pu, pd, tu, td;
  block_scan2(pcu * a.qpr, pcd * a.ops, pu, pd, wsum, tu, td);
  if (e < E && f) {
    up_pref[slot] = pu;
    dn_pref[slot] = pd;
  }
  if (threadIdx.x == 0) {
    const int sfull = a.sh_T / a.tgp, srem = a.sh_T % a.tgp;
    const int spad = srem <= 1 ? srem : srem <= 2 ? 2 : srem <= 4 ? 4 : 8;
    const int spcu = sfull * (4 + a.tgp) + (srem ? 4 + spad : 0);
    const int spcd = sfull * (4 + 4 * a.tgp) + (srem ? 4 + 4 * spad : 0);
    up_pref[n_act] = tu;
    up_pref[n_act + 1] = tu + spcu * a.qps;
    dn_pref[n_act] = td;
    dn_pref[n_act + 1] = td + spcd * a.ops;
  }
  __syncthreads();
  // Stable fill: a pair's rank in its expert's list is the number of earlier
  // tokens that selected the same expert (an expert appears once per token).
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const int ex_id = pidx[p];
    if (ex_id % a.ep_world != a.ep_rank) continue;
    const int t = p / K;
    const unsigned long long* m = mask + ex_id * W;
    int rank = 0;
    for (int wd = 0; wd < (t >> 6); ++wd) rank += __popcll(m[wd]);
    rank += __popcll(m[t >> 6] & ((1ull << (t & 63)) - 1ull));
    pairs[poff[ex_id] + rank] = p;
  }
}

// One token on one GPU: the schedule follows from the K selected ids alone
// (each slot holds one pair), so one warp writes the same words
// build_schedule would, without its block-wide scans over E experts: slot =
// rank of the id among the selection, pair = its top-k position, every slot
// (and the shared expert's) costing one 1-token pass.  `my` is lane k's
// selected id (k < K).
__device__ void single_token_schedule(const RouteArgs& a, int my, int lane) {
  const int E = a.E, Kk = a.K;
  int32_t* active = a.sched + 1;
  int32_t* offsets = a.sched + 1 + E;
  int32_t* pairs = a.sched + 2 + 2 * E;
  int32_t* up_pref = pairs + Kk;
  int32_t* dn_pref = up_pref + E + 2;
  int rank = 0;
  for (int k = 0; k < Kk; ++k) rank += (__shfl_sync(0xffffffffu, my, k) < my) ? 1 : 0;
  // a 1-token pass: 4 + pad(1) up, 4 + 4 pad(1) down (as build_schedule)
  const int cu = 5 * a.qpr, cd = 8 * a.ops;
  if (lane < Kk) {
    active[rank] = my;
    offsets[rank] = rank;
    pairs[rank] = lane;
    up_pref[rank] = rank * cu;
    dn_pref[rank] = rank * cd;
  }
  if (lane == 0) {
    a.sched[0] = Kk;
    offsets[Kk] = Kk;
    up_pref[Kk] = Kk * cu;
    up_pref[Kk + 1] = Kk * cu + 5 * a.qps;
    dn_pref[Kk] = Kk * cd;
    dn_pref[Kk + 1] = Kk * cd + cd;
  }
  for (int i = lane; i <= Kk; i += 32) a.up_done[i] = 0;
}

__global__ void __launch_bounds__(1024) k_route(RouteArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int E = a.E, K = a.K;
  const int t = blockIdx.x;
  const int e = threadIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  float* ex = reinterpret_cast<float*>(smem);                          // [E + 4]
  uint32_t* cand = reinterpret_cast<uint32_t*>(ex + E + 4);            // [nw * K]
  int* sel = reinterpret_cast<int*>(cand + nw * K);                    // [K]
  int* flag = sel + 32;                                                // [4]
  pdl_wait();
  pdl_launch_dependents();
  uint32_t key = 0;
  bool nan = false;
  if (e < E) {
    const uint32_t b = a.logits[static_cast<size_t>(t) * E + e];
    nan = ((b & 0x7f80u) == 0x7f80u) && ((b & 0x007fu) != 0u);
    key = (total_key(b) << 16) | static_cast<uint32_t>(0xffff - e);
  }
  if (__syncthreads_or(nan)) {
    // src/decoder_layer.rs:279-281 rejects NaN logits: flag it and emit a
    // placeholder selection so the rest of the pipeline stays in bounds.
    if (threadIdx.x == 0) set_error(a.err, kErrNanLogits);
    if (threadIdx.x < K) {
      a.idx[static_cast<size_t>(t) * K + threadIdx.x] = threadIdx.x;
      a.score[static_cast<size_t>(t) * K + threadIdx.x] = 0;
      if (a.sorted_slot) a.sorted_slot[static_cast<size_t>(t) * K + threadIdx.x] = threadIdx.x;
      if (a.pair_count) atomicAdd(&a.pair_count[threadIdx.x], 1);
    }
    if (a.sh_sig != nullptr && threadIdx.x == 0) a.sh_sig[t] = 0;
  } else {
    // The shared-expert gate lookup has no dependency on the selection.
    if (a.sh_sig != nullptr && threadIdx.x == 32) a.sh_sig[t] = a.sig_lut[a.sh_logit[t]];
    // Top-K per warp (K rounds of a warp max), then warp 0 merges.
    bool taken = false;
    for (int k = 0; k < K; ++k) {
      const uint32_t m = __reduce_max_sync(0xffffffffu, taken ? 0u : key);
      if (!taken && key == m && m != 0u) taken = true;
      if (lane == 0) cand[warp * K + k] = m;
    }
    __syncthreads();
    if (warp == 0) {
      // Each warp's K candidates are in descending order: merge the nw lists
      // as a tournament, lane w holding the head of warp w's list.  Keys
      // are unique (the expert id is folded in), so one lane advances.
      int head = 0;
      uint32_t v = lane < nw ? cand[lane * K] : 0u;
      for (int k = 0; k < K; ++k) {
        const uint32_t m = __reduce_max_sync(0xffffffffu, v);
        if (v == m && m != 0u) {
          ++head;
          v = head < K ? cand[lane * K + head] : 0u;
        }
        if (lane == 0) {
          sel[k] = 0xffff - static_cast<int>(m & 0xffffu);
          if (k == 0) ex[E + 1] = key_value(m);  // the largest logit
        }
      }
    }
    __syncthreads();
    // Softmax with the maximum subtracted (src/decoder_layer.rs:289-297);
    // exp is correctly rounded (f64, then f32).
    const float maximum = ex[E + 1];
    if (e < E) ex[e] = static_cast<float>(exp(static_cast<double>(__fsub_rn(key_value(key), maximum))));
    __syncthreads();
    if (threadIdx.x == 0) {
      // Rust's f32 Sum: start at -0.0, add in index order.
      float den = -0.0f;
      const float4* ex4 = reinterpret_cast<const float4*>(ex);
      for (int i = 0; i < (E >> 2); ++i) {
        const float4 v = ex4[i];
        den = __fadd_rn(den, v.x);
        den = __fadd_rn(den, v.y);
        den = __fadd_rn(den, v.z);
        den = __fadd_rn(den, v.w);
      }
      ex[E] = den;
    }
    __syncthreads();
    if (warp == 0) {
      const float den = ex[E];
      const int my = lane < K ? sel[lane] : 0;
      const float pk = lane < K ? __fdiv_rn(ex[my], den) : 0.0f;
      float ssum = -0.0f;  // selected_sum in top-k order
      for (int k = 0; k < K; ++k) ssum = __fadd_rn(ssum, __shfl_sync(0xffffffffu, pk, k));
      int rank = 0;  // slot order by ascending expert id (src/decoder_layer.rs:428-429)
      for (int k = 0; k < K; ++k) rank += (__shfl_sync(0xffffffffu, my, k) < my) ? 1 : 0;
      if (lane < K) {
        a.idx[static_cast<size_t>(t) * K + lane] = my;
        a.score[static_cast<size_t>(t) * K + lane] = f32_to_bf16(__fdiv_rn(pk, ssum));
        if (a.sorted_slot != nullptr) a.sorted_slot[static_cast<size_t>(t) * K + rank] = lane;
        if (a.pair_count != nullptr) atomicAdd(&a.pair_count[my], 1);
      }
    }
  }
  if (a.sched == nullptr) return;
  if (a.T == 1 && a.ep_world == 1) {
    if (warp == 0) single_token_schedule(a, lane < a.K ? a.idx[lane] : 0, lane);  // this lane's own write above
    return;
  }
  // The last CTA to finish builds the schedule from every token's selection
  // (a single-token launch is its own last CTA: no ticket).
  __syncthreads();
  if (gridDim.x > 1) {
    if (threadIdx.x == 0) {
      __threadfence();
      flag[0] = (atomicAdd(a.ticket, 1) == a.T - 1) ? 1 : 0;
    }
    __syncthreads();
    const bool last = flag[0] != 0;
    __syncthreads();  // every thread has read the flag before the schedule reuses smem
    if (!last) return;
    __threadfence();
  }
  build_schedule(a, smem);
  if (gridDim.x > 1 && threadIdx.x == 0) *a.ticket = 0;  // ready for the next forward
}

constexpr int kRouteWarps = 16;

// Route of token t by one warp (the arithmetic of k_route, in its order):
// writes idx / score / sorted_slot / sh_sig for t, adds its selections into
// cnt (shared memory, or null), and returns lane k's selected id (k < K).
// ex: E floats of this warp's shared memory.  Logit loads bypass L1 (the
// fused router writes them from other SMs).
template <int NS>
__device__ __forceinline__ int route_warp_token(const RouteArgs& a, int t, float* ex, int* cnt, int lane) {
  const int E = a.E, K = a.K, ne = E >> 5;
  const uint16_t* lr = a.logits + static_cast<size_t>(t) * E;
  uint32_t key[NS];
  bool nan = false;
#pragma unroll
  for (int i = 0; i < NS; ++i) {
    key[i] = 0u;
    if (i < ne) {
      const int e = lane + 32 * i;
      const uint32_t b = __ldcg(lr + e);
      nan |= ((b & 0x7f80u) == 0x7f80u) && ((b & 0x007fu) != 0u);
      key[i] = (total_key(b) << 16) | static_cast<uint32_t>(0xffff - e);
    }
  }
  if (__any_sync(0xffffffffu, nan)) {
    // src/decoder_layer.rs:279-281 rejects NaN logits (see k_route)
    if (lane == 0) set_error(a.err, kErrNanLogits);
    if (lane < K) {
      a.idx[static_cast<size_t>(t) * K + lane] = lane;
      a.score[static_cast<size_t>(t) * K + lane] = 0;
      if (a.sorted_slot) a.sorted_slot[static_cast<size_t>(t) * K + lane] = lane;
      if (cnt != nullptr) atomicAdd(&cnt[lane], 1);
    }
    if (a.sh_sig != nullptr && lane == 0) a.sh_sig[t] = 0;
    return lane < K ? lane : 0;
  }
  if (a.sh_sig != nullptr && lane == 0) a.sh_sig[t] = a.sig_lut[__ldcg(a.sh_logit + t)];
  // top-K: K rounds of a warp max over each lane's best untaken key
  uint32_t taken = 0u, top = 0u;
  int mysel = 0;
  for (int k = 0; k < K; ++k) {
    uint32_t best = 0u;
    int bi = -1;
#pragma unroll
    for (int i = 0; i < NS; ++i)
      if (i < ne && !((taken >> i) & 1u) && key[i] > best) {
        best = key[i];
        bi = i;
      }
    const uint32_t m = __reduce_max_sync(0xffffffffu, best);
    if (best == m && bi >= 0) taken |= 1u << bi;  // keys are unique: one lane
    if (k == 0) top = m;
    if (lane == k) mysel = 0xffff - static_cast<int>(m & 0xffffu);
  }
  // softmax with the maximum subtracted (src/decoder_layer.rs:289-297);
  // exp correctly rounded (f64, then f32)
  const float maximum = key_value(top);
#pragma unroll
  for (int i = 0; i < NS; ++i)
    if (i < ne) ex[lane + 32 * i] = static_cast<float>(exp(static_cast<double>(__fsub_rn(key_value(key[i]), maximum))));
  __syncwarp();
  float den = -0.0f;  // Rust's f32 Sum: -0.0, then index order
  if (lane == 0) {
    const float4* ex4 = reinterpret_cast<const float4*>(ex);
    for (int i = 0; i < (E >> 2); ++i) {
      const float4 v = ex4[i];
      den = __fadd_rn(den, v.x);
      den = __fadd_rn(den, v.y);
      den = __fadd_rn(den, v.z);
      den = __fadd_rn(den, v.w);
    }
  }
  den = __shfl_sync(0xffffffffu, den, 0);
  const float pk = lane < K ? __fdiv_rn(ex[mysel], den) : 0.0f;
  float ssum = -0.0f;  // selected_sum in top-k order
  for (int k = 0; k < K; ++k) ssum = __fadd_rn(ssum, __shfl_sync(0xffffffffu, pk, k));
  int rank = 0;  // slot order by ascending expert id (src/decoder_layer.rs:428-429)
  for (int k = 0; k < K; ++k) rank += (__shfl_sync(0xffffffffu, mysel, k) < mysel) ? 1 : 0;
  if (lane < K) {
    a.idx[static_cast<size_t>(t) * K + lane] = mysel;
    a.score[static_cast<size_t>(t) * K + lane] = f32_to_bf16(__fdiv_rn(pk, ssum));
    if (a.sorted_slot != nullptr) a.sorted_slot[static_cast<size_t>(t) * K + rank] = lane;
    if (cnt != nullptr) atomicAdd(&cnt[mysel], 1);
  }
  return mysel;
}

// Route for prefill widths (thousands of tokens): one warp per token
// (route_warp_token), so selections and scores are bit-identical to
// k_route's.  16 tokens per CTA instead of one CTA per token, and the pair
// counts are summed per CTA before one global atomic per expert (a hot
// expert's counter would otherwise take one atomic per token).
template <int NS>
__global__ void __launch_bounds__(kRouteWarps * 32) k_route_warp(RouteArgs a) {
  extern __shared__ __align__(16) float rw_smem[];
  const int E = a.E;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* ex = rw_smem + static_cast<size_t>(warp) * E;                                // [E] this warp's exp terms
  int* cnt = reinterpret_cast<int*>(rw_smem + static_cast<size_t>(kRouteWarps) * E);  // [E] this CTA's pair counts
  pdl_wait();
  pdl_launch_dependents();
  if (a.pair_count != nullptr)
    for (int i = threadIdx.x; i < E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  const int t = blockIdx.x * kRouteWarps + warp;
  if (t < a.T) route_warp_token<NS>(a, t, ex, a.pair_count != nullptr ? cnt : nullptr, lane);
  if (a.pair_count == nullptr) return;
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x)
    if (cnt[i] != 0) atomicAdd(&a.pair_count[i], cnt[i]);
}



// Expert parallelism: the schedule of this GPU's experts over every rank's
// tokens (a.idx holds the gathered selections), built by one CTA.
__global__ void __launch_bounds__(1024) k_schedule(RouteArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  pdl_wait();
  pdl_launch_dependents();
  build_schedule(a, smem);
}

// ---------------------------------------------------------------------------
// Combine (src/decoder_layer.rs:475-545, 532-537): per token, the K weighted
// rows are added into a bf16 accumulator in ascending expert id, rounding
// after every add, then the gated shared row is added.
struct CombineArgs {
  int H, K, T;
  const int32_t* sorted_slot;
  // Weighted row of token t's top-k position k: t*K + k, or with expert
  // parallelism ((idx[t][k] % ep_world) * T + t) * K + k (rows arrive per
  // source GPU, T tokens each).
  const int32_t* idx;
  int ep_world;
  const int32_t* row_of;  // if set: the row of (t, k) is row_of[t * K + k]
  const uint16_t* weighted;
  const uint16_t* gated_sh;
  uint16_t* y;
  HcPost hc;  // hyper-connection injection (hc.out null: none)
  // Expert parallelism over peer memory: the rows arrived in this rank's
  // window (k_ep_wait_done ran first); skip when the forward failed.
  const int* err;
};

// Expert parallelism over peer memory: one thread waits (bounded) until
// every rank has set its done flag in this rank's window, i.e. every
// weighted row of this rank's tokens has landed; the combine follows in
// stream order.
struct EpWaitArgs {
  EpPeers p;
  int* err;
};
__global__ void k_ep_wait_done(EpWaitArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) ep_wait_flags(a.p, kEpFlagDone, a.err);
}

// One CTA per token, 8 columns per thread: the slot order, then the
// weighted rows in groups of G (all loads of a group in flight before its
// adds), then the shared row.  The adds run in ascending expert id, as the
// reference accumulates.  Row indices are 32-bit: with 64-bit ones the
// kernel needed more than 64 registers.  G = 8 for wide forwards; with
// G = K every row and the shared row travel together (two memory latencies
// per thread instead of four), which needs 96 registers: at config 2 it
// measured 0.100 ms against 0.088 ms for G = 8 (fewer CTAs per SM), so it
// is kept for the narrow forwards whose CTAs all fit on the GPU at once.
template <int G>
__global__ void __launch_bounds__(512, G > 8 ? 1 : 2) k_combine(CombineArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  if (a.err != nullptr && ld_volatile_int(a.err) != 0) return;
  const int t = blockIdx.x;
  const int c = threadIdx.x * 8;
  if (c >= a.H) return;
  uint32_t acc[4];  // 8 bf16 sums, two per word
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = 0;  // bf16(0.0) pairs
  const int32_t* ss = a.sorted_slot + static_cast<size_t>(t) * a.K;
  uint4 sv = make_uint4(0u, 0u, 0u, 0u);
  for (int n0 = 0; n0 < a.K; n0 += G) {
    int sl[G];
#pragma unroll
    for (int i = 0; i < G; ++i) sl[i] = n0 + i < a.K ? ss[n0 + i] : 0;
    uint32_t row[G];  // weighted row index (< 2^31: T * K * ep_world rows)
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const int src =
          (a.idx != nullptr && n0 + i < a.K) ? a.idx[static_cast<size_t>(t) * a.K + sl[i]] % a.ep_world : 0;
      row[i] = a.row_of != nullptr ? static_cast<uint32_t>(n0 + i < a.K ? a.row_of[static_cast<size_t>(t) * a.K + sl[i]] : 0)
                                   : static_cast<uint32_t>((src * a.T + t) * a.K + sl[i]);
    }
    uint4 v[G];
#pragma unroll
    for (int i = 0; i < G; ++i)
      if (n0 + i < a.K) v[i] = *reinterpret_cast<const uint4*>(a.weighted + static_cast<size_t>(row[i]) * a.H + c);
    if constexpr (G > 8)  // one group: the shared row travels with it
      if (n0 + G >= a.K) sv = *reinterpret_cast<const uint4*>(a.gated_sh + static_cast<size_t>(t) * a.H + c);
#pragma unroll
    for (int i = 0; i < G; ++i) {
      if (n0 + i < a.K) {
        acc[0] = add_bf16x2(acc[0], v[i].x);
        acc[1] = add_bf16x2(acc[1], v[i].y);
        acc[2] = add_bf16x2(acc[2], v[i].z);
        acc[3] = add_bf16x2(acc[3], v[i].w);
      }
    }
  }
  if constexpr (G <= 8) sv = *reinterpret_cast<const uint4*>(a.gated_sh + static_cast<size_t>(t) * a.H + c);
  const uint32_t o[4] = {add_bf16x2(acc[0], sv.x), add_bf16x2(acc[1], sv.y), add_bf16x2(acc[2], sv.z),
                         add_bf16x2(acc[3], sv.w)};
  *reinterpret_cast<uint4*>(a.y + static_cast<size_t>(t) * a.H + c) = make_uint4(o[0], o[1], o[2], o[3]);
  if (a.hc.out == nullptr) return;
  // Hyper-connection injection (src/decoder_layer.rs:587-607):
  // out[g*H + c] = add_bf16(post[g*H + c], bf16(moe[c] * w[g])).
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const float wg = bf16_to_f32(a.hc.inj_w[static_cast<size_t>(t) * 4 + g]);
    const size_t off = static_cast<size_t>(t) * 4 * a.H + static_cast<size_t>(g) * a.H + c;
    const uint4 pv = *reinterpret_cast<const uint4*>(a.hc.post + off);
    const uint32_t pw[4] = {pv.x, pv.y, pv.z, pv.w};
    uint32_t r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t pl = f32_to_bf16(__fmul_rn(lo_bf16(o[i]), wg));
      const uint32_t ph = f32_to_bf16(__fmul_rn(hi_bf16(o[i]), wg));
      const uint32_t l = f32_to_bf16(__fadd_rn(lo_bf16(pw[i]), bf16_to_f32(pl)));
      const uint32_t h = f32_to_bf16(__fadd_rn(hi_bf16(pw[i]), bf16_to_f32(ph)));
      r[i] = l | (h << 16);
    }
    *reinterpret_cast<uint4*>(a.hc.out + off) = make_uint4(r[0], r[1], r[2], r[3]);
  }
}

// ---------------------------------------------------------------------------
// out = add_bf16(a, b) elementwise (src/expert.rs:578); n even elements
// go two per step, an odd tail alone.
__global__ void k_add_bf16(const uint16_t* a, const uint16_t* b, long long n, uint16_t* out) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; 2 * i < n; i += stride) {
    if (2 * i + 1 < n) {
      const uint32_t x = static_cast<uint32_t>(a[2 * i]) | (static_cast<uint32_t>(a[2 * i + 1]) << 16);
      const uint32_t y = static_cast<uint32_t>(b[2 * i]) | (static_cast<uint32_t>(b[2 * i + 1]) << 16);
      const uint32_t r = add_bf16x2(x, y);
      out[2 * i] = static_cast<uint16_t>(r & 0xffffu);
      out[2 * i + 1] = static_cast<uint16_t>(r >> 16);
    } else {
      out[2 * i] = static_cast<uint16_t>(add_bf16x2(a[2 * i], b[2 * i]) & 0xffffu);
    }
  }
}

__global__ void k_swiglu(const uint16_t* gate, const uint16_t* up, long long n,
                         const uint16_t* lut, uint16_t* out) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float silu = bf16_to_f32(lut[gate[i]]);
    out[i] = f32_to_bf16(silu * bf16_to_f32(up[i]));
  }
}

// ---------------------------------------------------------------------------
// Synthetic weights: element i of tensor (seed, id) is SplitMix64 output i of
// the keyed stream, as four 16-bit uniforms summed (Irwin-Hall, n = 4),
// times an f32 scale, rounded to bf16 -- the same bits as the CPU generator.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void k_synth(uint64_t key, uint64_t start, uint64_t count, float scale, uint16_t* out) {
  const uint64_t gamma = 0x9E3779B97F4A7C15ull;
  const uint64_t n8 = count / 8;
  for (uint64_t j = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; j < n8;
       j += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    uint32_t packed[4];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      uint32_t two = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint64_t idx = start + j * 8 + i + h;
        const uint64_t r = mix64(key + (idx + 1) * gamma);
        const int32_t s = static_cast<int32_t>(r & 0xffffu) + static_cast<int32_t>((r >> 16) & 0xffffu) +
                          static_cast<int32_t>((r >> 32) & 0xffffu) + static_cast<int32_t>(r >> 48) -
                          131070;
        two |= static_cast<uint32_t>(f32_to_bf16(__fmul_rn(static_cast<float>(s), scale))) << (16 * h);
      }
      packed[i / 2] = two;
    }
    *reinterpret_cast<uint4*>(out + j * 8) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
  // tail (count % 8)
  const uint64_t tail0 = n8 * 8;
  for (uint64_t i = tail0 + blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t r = mix64(key + (start + i + 1) * gamma);
    const int32_t s = static_cast<int32_t>(r & 0xffffu) + static_cast<int32_t>((r >> 16) & 0xffffu) +
                      static_cast<int32_t>((r >> 32) & 0xffffu) + static_cast<int32_t>(r >> 48) - 131070;
    out[i] = f32_to_bf16(__fmul_rn(static_cast<float>(s), scale));
  }
}

template <typename Kern, typename Arg>
cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, const Arg& arg) {
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, arg);
}

size_t route_smem(int E, int T, int K, bool schedule) {
  const int nw = (E + 31) / 32;
  size_t b = sizeof(float) * (E + 4) + sizeof(uint32_t) * nw * K + sizeof(int) * 36;
  if (schedule) {
    const int P = T * K;
    const int W = (T + 63) / 64;
    const size_t s = sizeof(int32_t) * ((P + 1) & ~1) + sizeof(unsigned long long) * static_cast<size_t>(E) * W +
                     sizeof(int) * (2 * E + 66);
    b = b > s ? b : s;
  }
  return (b + 15) & ~size_t(15);
}

cudaError_t launch_route_kernel(const RouteArgs& a, cudaStream_t st) {
  const int threads = (a.E + 31) / 32 * 32;
  return launch_pdl(k_route, dim3(a.T), dim3(threads), route_smem(a.E, a.T, a.K, a.sched != nullptr), st, a);
}

}  // namespace

cudaError_t launch_linear(const uint16_t* w, const uint16_t* x, int rows, int cols, int T,
                          uint16_t* y, cudaStream_t st) {
  RowsDotArgs a{w, rows, cols, T, x, y, nullptr, nullptr, nullptr};
  const dim3 grid((rows + kRowsPerDotCta - 1) / kRowsPerDotCta, (T + kTG - 1) / kTG);
  return launch_pdl(k_rows_dot, grid, dim3(64), sizeof(float) * kTG * cols, st, a);
}

cudaError_t launch_route(const uint16_t* logits, int T, int E, int K, int32_t* idx,
                         uint16_t* score, int* err, cudaStream_t st) {
  RouteArgs a{logits, T, E, K, idx, score, err, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
              0, 0, 0, 0, nullptr, nullptr, 0, 1, T};
  return launch_route_kernel(a, st);
}

cudaError_t launch_add_bf16(const uint16_t* a, const uint16_t* b, long long n, uint16_t* out, cudaStream_t st) {
  const long long pairs = (n + 1) / 2;
  const long long blocks = (pairs + 255) / 256;
  const int grid = static_cast<int>(blocks < 4096 ? (blocks > 0 ? blocks : 1) : 4096);
  k_add_bf16<<<grid, 256, 0, st>>>(a, b, n, out);
  return cudaGetLastError();
}

cudaError_t launch_swiglu(const uint16_t* gate, const uint16_t* up, long long n,
                          const uint16_t* silu_lut, uint16_t* out, cudaStream_t st) {
  const long long blocks = (n + 255) / 256;
  const int grid = static_cast<int>(blocks < 4096 ? (blocks > 0 ? blocks : 1) : 4096);
  k_swiglu<<<grid, 256, 0, st>>>(gate, up, n, silu_lut, out);
  return cudaGetLastError();
}

cudaError_t launch_synth(uint64_t key, uint32_t /*tensor*/, uint64_t start, uint64_t count,
                         float scale, uint16_t* out, cudaStream_t st) {
  if (count == 0) return cudaSuccess;
  k_synth<<<148 * 8, 256, 0, st>>>(key, start, count, scale, out);
  return cudaGetLastError();
}

cudaError_t launch_router(const Shape& s, const LayerWeights& w, const Scratch& sc, const uint16_t* x, int T,
                          cudaStream_t st) {
  RouterArgs a{w.router_pm, w.router, w.sh_gate_w, w.bias, x, sc.logits, sc.sh_logit, s.E, s.H, T, sc.err};
  // One token: the partial-major router, one row per warp on ~130 CTAs
  // (with 16 rows per CTA it measured 18.5 k -> 19.4 k token-layers/s against
  // k_router).  At T = 4 the same kernel measured 5 % slower than k_router,
  // so wider forwards keep k_router.
  if (T == 1 && w.router_pm != nullptr && s.H % 256 == 0) {
    constexpr int kRows = kPmWarps;  // RW = 1
    const int rows = (s.E + 1 + kRows - 1) / kRows;
    const size_t smem = static_cast<size_t>(kRows + 1) * 32 * pm_stride(s.H) * 16;
    return launch_pdl(k_router_pm<1, 1>, dim3(rows, 1), dim3(kPmWarps * 32), smem, st, a);
  }
  const size_t smem = static_cast<size_t>(kRouterRows + kRouterTokens) * s.H * 2 + 16;
  const dim3 grid((s.E + 1 + kRouterRows - 1) / kRouterRows, (T + kRouterTokens - 1) / kRouterTokens);
  return launch_pdl(k_router, grid, dim3(kRouterRows * 32), smem, st, a);
}

cudaError_t launch_route_block(const Shape& s, const Luts& luts, const Scratch& sc, int T, int32_t* topk_idx,
                               uint16_t* topk_score, bool schedule, int* pair_count, cudaStream_t st) {
  RouteArgs a{sc.logits, T, s.E, s.K, topk_idx, topk_score, sc.err,
              sc.sh_logit, luts.sigmoid, sc.sh_sig, sc.sorted_slot, schedule ? sc.sched : nullptr, sc.up_done,
              experts_tokens_per_pass(s), s.I / 4, s.Is / 4, s.H / 8, sc.ticket, pair_count, 0, 1, T};
  return launch_route_kernel(a, st);
}

cudaError_t launch_route_prefill(const Shape& s, const Luts& luts, const Scratch& sc, int T, int32_t* topk_idx,
                                 uint16_t* topk_score, int* pair_count, cudaStream_t st) {
  RouteArgs a{sc.logits, T, s.E, s.K, topk_idx, topk_score, sc.err,
              sc.sh_logit, luts.sigmoid, sc.sh_sig, sc.sorted_slot, nullptr, sc.up_done,
              experts_tokens_per_pass(s), s.I / 4, s.Is / 4, s.H / 8, sc.ticket, pair_count, 0, 1, T};
  const size_t smem = sizeof(float) * static_cast<size_t>(kRouteWarps + 1) * s.E;
  const dim3 grid((T + kRouteWarps - 1) / kRouteWarps), block(kRouteWarps * 32);
  return s.E <= 512 ? launch_pdl(k_route_warp<16>, grid, block, smem, st, a)
                    : launch_pdl(k_route_warp<32>, grid, block, smem, st, a);
}

cudaError_t launch_ep_schedule(const Shape& s, const Scratch& sc, const int32_t* idx_all, int T, int ep_rank,
                               int ep_world, int sh_T, cudaStream_t st) {
  RouteArgs a{nullptr, T, s.E, s.K, const_cast<int32_t*>(idx_all), nullptr, sc.err,
              nullptr, nullptr, nullptr, nullptr, sc.sched, sc.up_done,
              experts_tokens_per_pass(s), s.I / 4, s.Is / 4, s.H / 8, nullptr, nullptr, ep_rank, ep_world, sh_T};
  const int threads = (s.E + 31) / 32 * 32;
  return launch_pdl(k_schedule, dim3(1), dim3(threads), route_smem(s.E, T, s.K, true), st, a);
}

cudaError_t launch_combine(const Shape& s, const Scratch& sc, int T, uint16_t* y, cudaStream_t st,
                           const int32_t* ep_idx, int ep_world, const uint16_t* ep_rows, const int32_t* row_of,
                           const HcPost* hc, const EpPeers* wait) {
  CombineArgs a{s.H, s.K, T, sc.sorted_slot, ep_idx, ep_world > 0 ? ep_world : 1, row_of,
                ep_rows != nullptr ? ep_rows : sc.weighted, sc.gated_sh, y, hc != nullptr ? *hc : HcPost{},
                wait != nullptr ? sc.err : nullptr};
  if (wait != nullptr) {
    const cudaError_t e = launch_pdl(k_ep_wait_done, dim3(1), dim3(32), 0, st, EpWaitArgs{*wait, sc.err});
    if (e != cudaSuccess) return e;
  }
  // top-10 forwards of at most two CTAs per SM: every row in one load group
  DeviceAttrs da;
  const int sms = current_device_attrs(&da) == cudaSuccess ? da.sms : 148;
  if (s.K == 10 && T <= 2 * sms)
    return launch_pdl(k_combine<10>, dim3(T), dim3(s.H / 8), 0, st, a);
  return launch_pdl(k_combine<8>, dim3(T), dim3(s.H / 8), 0, st, a);
}

cudaError_t launch_block(const Shape& s, const LayerWeights& w, const Luts& luts, const Scratch& sc,
                         const uint16_t* x, int T, uint16_t* y, int32_t* topk_idx,
                         uint16_t* topk_score, cudaStream_t st, cudaEvent_t* ev, const HcPost* hc) {
  if (T <= 0) return cudaSuccess;
  cudaError_t e;
  auto mark = [&](int i) { return ev != nullptr ? cudaEventRecord(ev[i], st) : cudaSuccess; };
  if ((e = mark(0)) != cudaSuccess) return e;
  // 1. router logits + shared-gate logit
  e = launch_router(s, w, sc, x, T, st);
  if (e != cudaSuccess || (e = mark(1)) != cudaSuccess) return e;
  // 2. route + expert schedule (the dispatch stage is empty on one GPU)
  e = launch_route_block(s, luts, sc, T, topk_idx, topk_score, true, nullptr, st);
  if (e != cudaSuccess || (e = mark(2)) != cudaSuccess || (e = mark(3)) != cudaSuccess) return e;
  // 3. experts: gate_up + SwiGLU, then down + scale (one persistent kernel)
  e = launch_experts(s, w, luts, sc, x, T, topk_score, st, x, T);
  if (e != cudaSuccess || (e = mark(4)) != cudaSuccess) return e;
  // 4. combine
  e = launch_combine(s, sc, T, y, st, nullptr, 0, nullptr, nullptr, hc);
  if (e == cudaSuccess) e = mark(5);
  return e;
}

}  // namespace fw
