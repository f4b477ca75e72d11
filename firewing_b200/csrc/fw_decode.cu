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
// Route (src/decoder_layer.rs:278-307) + permute.  One CTA of 32 warps; warp w
// routes tokens w, w+32, ...  Then the CTA builds the expert schedule.
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
};

constexpr int kRouteWarps = 32;

// Lane `lane` holds experts lane + 32*i, i < NPER, as total-order keys with
// the index folded in (higher key = higher logit, then lower index).  The
// bf16 value is recoverable from the key, so no second array is needed.
__device__ __forceinline__ float key_value(uint32_t key) {
  const uint32_t k16 = key >> 16;
  const uint32_t bits = (k16 & 0x8000u) ? (k16 & 0x7fffu) : (~k16 & 0xffffu);
  return bf16_to_f32(bits);
}

template <int NPER>
__device__ void route_token(const RouteArgs& a, int t, float* ex, int32_t* pidx) {
  const int lane = threadIdx.x & 31;
  const int E = a.E, K = a.K;
  const int nper = E >> 5;
  const uint16_t* lg = a.logits + static_cast<size_t>(t) * E;
  uint32_t key[NPER];
  bool nan = false;
#pragma unroll
  for (int i = 0; i < NPER; ++i) {
    key[i] = 0;
    if (i < nper) {
      const int e = lane + 32 * i;
      const uint32_t b = lg[e];
      nan |= ((b & 0x7f80u) == 0x7f80u) && ((b & 0x007fu) != 0u);
      key[i] = (total_key(b) << 16) | static_cast<uint32_t>(0xffff - e);
    }
  }
  if (__any_sync(0xffffffffu, nan)) {
    // src/decoder_layer.rs:279-281 rejects NaN logits; flag and emit a
    // placeholder selection so the rest of the pipeline stays in bounds.
    if (lane == 0) set_error(a.err, kErrNanLogits);
    for (int k = lane; k < K; k += 32) {
      a.idx[static_cast<size_t>(t) * K + k] = k;
      a.score[static_cast<size_t>(t) * K + k] = 0;
      if (pidx) pidx[t * K + k] = k;
      if (a.sorted_slot) a.sorted_slot[static_cast<size_t>(t) * K + k] = k;
    }
    if (a.sh_sig != nullptr && lane == 0) a.sh_sig[t] = 0;
    return;
  }
  // Top-K: K rounds of a warp-wide max over (total-order key, -index)
  // (selection order of src/router.rs:241-247).
  uint32_t taken = 0;
  int sel_mine = -1;  // lane k keeps the k-th selection
  for (int k = 0; k < K; ++k) {
    uint32_t best = 0;
#pragma unroll
    for (int i = 0; i < NPER; ++i)
      if (i < nper && !((taken >> i) & 1u)) best = max(best, key[i]);
    const uint32_t wbest = __reduce_max_sync(0xffffffffu, best);
    const int e = 0xffff - static_cast<int>(wbest & 0xffffu);
    if ((e & 31) == lane) taken |= 1u << (e >> 5);
    if (lane == k) sel_mine = e;
  }
  // Softmax over all experts with the maximum subtracted
  // (src/decoder_layer.rs:289-297); exp is correctly rounded (f64 then f32).
  const int top1 = __shfl_sync(0xffffffffu, sel_mine, 0);
  const float maximum = bf16_to_f32(lg[top1]);
#pragma unroll
  for (int i = 0; i < NPER; ++i)
    if (i < nper)
      ex[lane + 32 * i] =
          static_cast<float>(exp(static_cast<double>(__fsub_rn(key_value(key[i]), maximum))));
  __syncwarp();
  if (lane == 0) {
    float den = -0.0f;  // Rust's f32 Sum: start at -0.0, add in index order
    for (int e = 0; e < E; ++e) den = __fadd_rn(den, ex[e]);
    ex[E] = den;
  }
  __syncwarp();
  const float den = ex[E];
  // p_k = e_k / den; selected_sum in top-k order; score = bf16(p_k / sum).
  float p_mine = 0.0f;
  if (lane < K) p_mine = __fdiv_rn(ex[sel_mine], den);
  float ssum = -0.0f;
  for (int k = 0; k < K; ++k) ssum = __fadd_rn(ssum, __shfl_sync(0xffffffffu, p_mine, k));
  if (lane < K) {
    a.idx[static_cast<size_t>(t) * K + lane] = sel_mine;
    a.score[static_cast<size_t>(t) * K + lane] = f32_to_bf16(__fdiv_rn(p_mine, ssum));
    if (pidx) pidx[t * K + lane] = sel_mine;
  }
  if (a.sorted_slot != nullptr) {
    // Slot order by ascending expert id (src/decoder_layer.rs:428-429).
    int rank = 0;
    for (int k = 0; k < K; ++k) {
      const int other = __shfl_sync(0xffffffffu, sel_mine, k);
      rank += (other < sel_mine) ? 1 : 0;
    }
    if (lane < K) a.sorted_slot[static_cast<size_t>(t) * K + rank] = lane;
  }
  if (a.sh_sig != nullptr && lane == 0) a.sh_sig[t] = a.sig_lut[a.sh_logit[t]];
  __syncwarp();
}

template <int NPER>
__global__ void __launch_bounds__(1024) k_route_permute(RouteArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int E = a.E, K = a.K, T = a.T;
  const int warp = threadIdx.x >> 5;
  float* ex = reinterpret_cast<float*>(smem_raw) + warp * (E + 4);
  int32_t* pidx = reinterpret_cast<int32_t*>(smem_raw + sizeof(float) * kRouteWarps * (E + 4));
  for (int t = warp; t < T; t += kRouteWarps) route_token<NPER>(a, t, ex, a.sched ? pidx : nullptr);
  if (a.sched == nullptr) return;
  __syncthreads();

  // ---- permute: expert schedule for the expert kernel ----
  const int P = T * K;
  const int W = (T + 63) >> 6;  // 64-bit token masks per expert
  unsigned long long* mask = reinterpret_cast<unsigned long long*>(pidx + ((P + 3) & ~3));
  int* cnt = reinterpret_cast<int*>(mask + static_cast<size_t>(E) * W);
  int* poff = cnt + E;
  int* wsum = poff + E;  // [32] warp totals of flags, [32] of counts
  for (int i = threadIdx.x; i < E * W; i += blockDim.x) mask[i] = 0ull;
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const int e = pidx[p];
    const int t = p / K;
    atomicAdd(&cnt[e], 1);
    atomicOr(&mask[e * W + (t >> 6)], 1ull << (t & 63));
  }
  __syncthreads();
  // Block-wide exclusive scans over experts (E <= 1024 = blockDim).
  const int e = threadIdx.x;
  const int lane = threadIdx.x & 31;
  const int c = (e < E) ? cnt[e] : 0;
  const int f = c > 0 ? 1 : 0;
  int ic = c, iflag = f;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int yc = __shfl_up_sync(0xffffffffu, ic, o);
    const int yf = __shfl_up_sync(0xffffffffu, iflag, o);
    if (lane >= o) {
      ic += yc;
      iflag += yf;
    }
  }
  if (lane == 31) {
    wsum[warp] = iflag;
    wsum[32 + warp] = ic;
  }
  __syncthreads();
  if (warp == 0) {
    int vf = wsum[lane], vc = wsum[32 + lane];
    int sf = vf, sc = vc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int yf = __shfl_up_sync(0xffffffffu, sf, o);
      const int yc = __shfl_up_sync(0xffffffffu, sc, o);
      if (lane >= o) {
        sf += yf;
        sc += yc;
      }
    }
    wsum[lane] = sf - vf;  // exclusive warp prefix
    wsum[32 + lane] = sc - vc;
  }
  __syncthreads();
  int32_t* active = a.sched + 1;
  int32_t* offsets = a.sched + 1 + E;
  int32_t* pairs = a.sched + 2 + 2 * E;
  if (a.up_done != nullptr)
    for (int i = threadIdx.x; i <= E; i += blockDim.x) a.up_done[i] = 0;
  const int my_slot = wsum[warp] + iflag - f;  // this expert's slot (if active)
  if (e < E) {
    const int off = wsum[32 + warp] + ic - c;
    poff[e] = off;
    if (f) {
      active[my_slot] = e;
      offsets[my_slot] = off;
    }
    if (e == E - 1) {
      a.sched[0] = my_slot + f;
      offsets[my_slot + f] = off + c;
    }
  }
  __syncthreads();
  // Cost prefixes for the expert kernel.  A slot of n tokens has
  // ceil(n / tgp) token passes of qpr quads (up) and ops octets (down); a
  // unit of a pass with nt tokens costs 4 + pad(nt) (pad = 1, 2, 4, 8: the
  // tokens the kernel computes), weighing bytes and FMAs.
  {
    const int nfull = f ? c / a.tgp : 0, rem = f ? c % a.tgp : 0;
    const int pad = rem <= 1 ? rem : rem <= 2 ? 2 : rem <= 4 ? 4 : 8;
    const int pc = nfull * (4 + a.tgp) + (rem ? 4 + pad : 0);  // per-unit-row cost of the slot
    const int vu = pc * a.qpr, vd = pc * a.ops;
    int iu = vu, id = vd;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int yu = __shfl_up_sync(0xffffffffu, iu, o);
      const int yd = __shfl_up_sync(0xffffffffu, id, o);
      if (lane >= o) {
        iu += yu;
        id += yd;
      }
    }
    __syncthreads();  // wsum reuse
    if (lane == 31) {
      wsum[warp] = iu;
      wsum[32 + warp] = id;
    }
    __syncthreads();
    if (warp == 0) {
      const int su0 = wsum[lane], sd0 = wsum[32 + lane];
      int su = su0, sd = sd0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int yu = __shfl_up_sync(0xffffffffu, su, o);
        const int yd = __shfl_up_sync(0xffffffffu, sd, o);
        if (lane >= o) {
          su += yu;
          sd += yd;
        }
      }
      wsum[lane] = su - su0;
      wsum[32 + lane] = sd - sd0;
    }
    __syncthreads();
    int32_t* up_pref = pairs + P;
    int32_t* dn_pref = up_pref + E + 2;
    if (e < E && f) {
      up_pref[my_slot] = wsum[warp] + iu - vu;
      dn_pref[my_slot] = wsum[32 + warp] + id - vd;
    }
    if (e == E - 1) {
      const int n_act = my_slot + f;
      const int sfull = T / a.tgp, srem = T % a.tgp;
      const int spad = srem <= 1 ? srem : srem <= 2 ? 2 : srem <= 4 ? 4 : 8;
      const int spc = sfull * (4 + a.tgp) + (srem ? 4 + spad : 0);
      const int tu = wsum[warp] + iu, td = wsum[32 + warp] + id;
      up_pref[n_act] = tu;
      up_pref[n_act + 1] = tu + spc * a.qps;
      dn_pref[n_act] = td;
      dn_pref[n_act + 1] = td + spc * a.ops;
    }
  }
  // Stable fill: a pair's rank in its expert's list is the number of earlier
  // tokens that selected the same expert (an expert appears once per token).
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const int ex_id = pidx[p];
    const int t = p / K;
    const unsigned long long* m = mask + ex_id * W;
    int rank = 0;
    for (int wd = 0; wd < (t >> 6); ++wd) rank += __popcll(m[wd]);
    rank += __popcll(m[t >> 6] & ((1ull << (t & 63)) - 1ull));
    pairs[poff[ex_id] + rank] = p;
  }
}

// ---------------------------------------------------------------------------
// Combine (src/decoder_layer.rs:475-545, 532-537): per token, the K weighted
// rows are added into a bf16 accumulator in ascending expert id, rounding
// after every add, then the gated shared row is added.
struct CombineArgs {
  int H, K, T;
  const int32_t* sorted_slot;
  const uint16_t* weighted;
  const uint16_t* gated_sh;
  uint16_t* y;
};

__global__ void k_combine(CombineArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x;
  const int c = threadIdx.x * 8;
  if (c >= a.H) return;
  uint32_t acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0;  // bf16(0.0)
  for (int n = 0; n < a.K; ++n) {
    const int slot = a.sorted_slot[static_cast<size_t>(t) * a.K + n];
    const size_t p = static_cast<size_t>(t) * a.K + slot;
    const uint4 v = *reinterpret_cast<const uint4*>(a.weighted + p * a.H + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[2 * i] = f32_to_bf16(bf16_to_f32(acc[2 * i]) + lo_bf16(w[i]));
      acc[2 * i + 1] = f32_to_bf16(bf16_to_f32(acc[2 * i + 1]) + hi_bf16(w[i]));
    }
  }
  const uint4 sv = *reinterpret_cast<const uint4*>(a.gated_sh + static_cast<size_t>(t) * a.H + c);
  const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t l = f32_to_bf16(bf16_to_f32(acc[2 * i]) + lo_bf16(sw[i]));
    const uint32_t h = f32_to_bf16(bf16_to_f32(acc[2 * i + 1]) + hi_bf16(sw[i]));
    o[i] = l | (h << 16);
  }
  *reinterpret_cast<uint4*>(a.y + static_cast<size_t>(t) * a.H + c) = make_uint4(o[0], o[1], o[2], o[3]);
}

// ---------------------------------------------------------------------------
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

cudaError_t launch_route_kernel(const RouteArgs& a, size_t smem, cudaStream_t st) {
  const int nper = a.E / 32;
  if (nper <= 4) return launch_pdl(k_route_permute<4>, dim3(1), dim3(1024), smem, st, a);
  if (nper <= 8) return launch_pdl(k_route_permute<8>, dim3(1), dim3(1024), smem, st, a);
  if (nper <= 16) return launch_pdl(k_route_permute<16>, dim3(1), dim3(1024), smem, st, a);
  return launch_pdl(k_route_permute<32>, dim3(1), dim3(1024), smem, st, a);
}

size_t route_smem(int E, int T, int K, bool permute) {
  size_t b = sizeof(float) * kRouteWarps * (E + 4);
  if (permute) {
    const int P = T * K;
    const int W = (T + 63) / 64;
    b += sizeof(int32_t) * ((P + 3) & ~3) + sizeof(unsigned long long) * static_cast<size_t>(E) * W +
         sizeof(int) * (2 * E + 64);
  }
  return b;
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
              0, 0, 0, 0};
  return launch_route_kernel(a, route_smem(E, T, K, false), st);
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

cudaError_t launch_block(const Shape& s, const LayerWeights& w, const Luts& luts, const Scratch& sc,
                         const uint16_t* x, int T, uint16_t* y, int32_t* topk_idx,
                         uint16_t* topk_score, cudaStream_t st, cudaEvent_t* ev) {
  if (T <= 0) return cudaSuccess;
  cudaError_t e;
  auto mark = [&](int i) { return ev != nullptr ? cudaEventRecord(ev[i], st) : cudaSuccess; };
  if ((e = mark(0)) != cudaSuccess) return e;
  // 1. router logits + shared-gate logit
  {
    RowsDotArgs a{w.router, s.E, s.H, T, x, sc.logits, w.bias, w.sh_gate_w, sc.sh_logit};
    const dim3 grid((s.E + 1 + kRowsPerDotCta - 1) / kRowsPerDotCta, (T + kTG - 1) / kTG);
    e = launch_pdl(k_rows_dot, grid, dim3(64), sizeof(float) * kTG * s.H, st, a);
    if (e != cudaSuccess || (e = mark(1)) != cudaSuccess) return e;
  }
  // 2. route + permute
  {
    RouteArgs a{sc.logits, T, s.E, s.K, topk_idx, topk_score, sc.err,
                sc.sh_logit, luts.sigmoid, sc.sh_sig, sc.sorted_slot, sc.sched, sc.up_done,
                experts_tokens_per_pass(s), s.I / 4, s.Is / 4, s.H / 8};
    e = launch_route_kernel(a, route_smem(s.E, T, s.K, true), st);
    if (e != cudaSuccess || (e = mark(2)) != cudaSuccess) return e;
  }
  // 3. experts: gate_up + SwiGLU, then down + scale (one persistent kernel)
  e = launch_experts(s, w, luts, sc, x, T, topk_score, st);
  if (e != cudaSuccess || (e = mark(3)) != cudaSuccess) return e;
  // 4. combine
  {
    CombineArgs a{s.H, s.K, T, sc.sorted_slot, sc.weighted, sc.gated_sh, y};
    e = launch_pdl(k_combine, dim3(T), dim3(s.H / 8), 0, st, a);
    if (e == cudaSuccess) e = mark(4);
  }
  return e;
}

}  // namespace fw
