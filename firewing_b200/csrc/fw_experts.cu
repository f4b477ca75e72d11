// fw_experts.cu -- persistent expert kernel for the decode path (sm_100a).
//
// One CTA per SM.  The work of a layer is two row spaces:
//   up   : for every schedule slot (active routed experts in ascending id,
//          then the shared expert) its gate/up row pairs, in "quads" of 4
//          gate rows + the 4 matching up rows;
//   down : for every slot its H down rows, in "octets" of 8 rows.
// Each CTA takes one contiguous, equal-sized range of each space, so the
// bytes streamed per SM are balanced whatever the routing.  Inside a CTA,
// 8 warps take the quads (octets) of the range round-robin.
//
// Every warp owns a 4-stage shared-memory ring.  Lane 0 runs ahead of the
// warp's own consumption and issues one bulk async copy per weight row
// (cp.async.bulk, completion counted on the stage's mbarrier; never
// multicast), so up to 3 stages x 4 KB per warp are in flight regardless of
// occupancy.  A stage is 8 rows x up to 256 columns.  Rows are padded by
// 16 bytes in shared memory so the 8 lanes of a quarter-warp, which read the
// same columns of 8 different rows, hit 8 distinct bank groups.
//
// Lane mapping (exact reference reduction, src/expert.rs:514-552): lane l
// owns row r = l & 7 and partials 8q..8q+7, q = l >> 3; it walks the
// 32-column blocks of its row in order, one 16-byte shared load per block,
// and fw::reduce_partials_strided applies the reference tree.
//
// The down rows of a slot need all of that slot's SwiGLU rows: the CTA that
// finishes its share of a slot's quads adds them to up_done[slot]
// (release); a CTA about to stage a slot's activations for its down rows
// waits (acquire, bounded) until the count is complete.  Up work never
// waits, and all CTAs are co-resident (cooperative launch), so the waits
// always end.
#include <cstdint>

#include "fw_common.cuh"
#include "fw_kernels.h"

namespace fw {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRing = 4;                                 // stages per warp ring
constexpr int kMaxChunk = 256;                        // columns per stage
constexpr int kStageBytes = 8 * (kMaxChunk * 2 + 16);  // 4224
constexpr int kTGP = 4;                                // tokens per pass
constexpr uint64_t kWaitNs = 2000000000ull;            // bounded waits: 2 s
constexpr uint64_t kDrainNs = 200000000ull;            // drain after abort: 0.2 s

struct ExpertsArgs {
  int H, I, Is, E, K, T;
  const uint16_t* x;        // [T][H]
  const uint16_t* gate_up;  // [E_local][2I][H]
  const uint16_t* down;     // [E_local][H][I]
  const uint16_t* sh_gate;  // [Is][H]
  const uint16_t* sh_up;    // [Is][H]
  const uint16_t* sh_down;  // [H][Is]
  int expert_base;
  const uint16_t* silu_lut;
  const int32_t* sched;
  const uint16_t* pair_score;  // [T*K]
  const uint16_t* sh_sig;      // [T]
  uint16_t* act;               // [T*K][I]
  uint16_t* act_sh;            // [T][Is]
  uint16_t* weighted;          // [T*K][H]
  uint16_t* gated_sh;          // [T][H]
  int* up_done;                // [E+1], zeroed by the route kernel
  int* err;
};

__device__ __forceinline__ int chunk_cols(int k) {
  for (int c = kMaxChunk; c >= 32; c -= 32)
    if (k % c == 0) return c;
  return 32;
}

// Geometry of one launch, identical in every thread.
struct Geo {
  int n_active;    // routed slots; the shared expert is slot n_active
  int qpr, qps;    // quads per routed / shared slot
  int ops;         // octets per slot (H / 8)
  int up_lo, up_hi;  // this CTA's quad range
  int dn_lo, dn_hi;  // this CTA's octet range
  int cu;          // up chunk columns
  int cdr, cds;    // down chunk columns (routed / shared)
};

__device__ __forceinline__ int slot_qbase(const Geo& g, int s) { return s * g.qpr; }
__device__ __forceinline__ int slot_nq(const Geo& g, int s) { return s < g.n_active ? g.qpr : g.qps; }
__device__ __forceinline__ int slot_tokens(const ExpertsArgs& a, const Geo& g, int s) {
  return s < g.n_active ? a.sched[1 + a.E + s + 1] - a.sched[1 + a.E + s] : a.T;
}
// first slot of a phase's range, and one past the last
__device__ __forceinline__ void phase_slots(const Geo& g, int phase, int& s0, int& s1) {
  if (phase == 0) {
    if (g.up_lo >= g.up_hi) {
      s0 = s1 = 0;
      return;
    }
    const int routed_q = g.n_active * g.qpr;
    s0 = g.up_lo < routed_q ? g.up_lo / g.qpr : g.n_active;
    s1 = (g.up_hi - 1) < routed_q ? (g.up_hi - 1) / g.qpr + 1 : g.n_active + 1;
  } else {
    if (g.dn_lo >= g.dn_hi) {
      s0 = s1 = 0;
      return;
    }
    s0 = g.dn_lo / g.ops;
    s1 = (g.dn_hi - 1) / g.ops + 1;
  }
}
__device__ __forceinline__ void slot_items(const Geo& g, int phase, int s, int& lo, int& hi) {
  if (phase == 0) {
    const int b = slot_qbase(g, s);
    lo = max(g.up_lo, b);
    hi = min(g.up_hi, b + slot_nq(g, s));
  } else {
    const int b = s * g.ops;
    lo = max(g.dn_lo, b);
    hi = min(g.dn_hi, b + g.ops);
  }
}
__device__ __forceinline__ int slot_chunks(const ExpertsArgs& a, const Geo& g, int phase, int s) {
  if (phase == 0) return a.H / g.cu;
  return s < g.n_active ? a.I / g.cdr : a.Is / g.cds;
}

// Issue-side cursor over this warp's stage sequence:
// phase -> slot -> token pass -> item (warp-strided) -> chunk.
struct Cursor {
  int phase, slot, s_end, tg, ntg, item, lo, hi, chunk, nchunks;
};

__device__ void cursor_enter_slot(Cursor& c, const ExpertsArgs& a, const Geo& g, int warp) {
  slot_items(g, c.phase, c.slot, c.lo, c.hi);
  c.tg = 0;
  c.ntg = (slot_tokens(a, g, c.slot) + kTGP - 1) / kTGP;
  c.item = c.lo + warp;
  c.chunk = 0;
  c.nchunks = slot_chunks(a, g, c.phase, c.slot);
}

// Move forward until the cursor names a stage, or phase == 2 (done).
__device__ void cursor_normalize(Cursor& c, const ExpertsArgs& a, const Geo& g, int warp) {
  while (c.phase < 2) {
    if (c.slot < c.s_end && c.item < c.hi) return;
    if (c.slot < c.s_end) {
      if (++c.tg < c.ntg) {
        c.item = c.lo + warp;
        c.chunk = 0;
        continue;
      }
      ++c.slot;
      if (c.slot < c.s_end) {
        cursor_enter_slot(c, a, g, warp);
        continue;
      }
    }
    // next phase
    ++c.phase;
    if (c.phase < 2) {
      phase_slots(g, c.phase, c.slot, c.s_end);
      if (c.slot < c.s_end) cursor_enter_slot(c, a, g, warp);
    }
  }
}

__device__ void cursor_begin(Cursor& c, const ExpertsArgs& a, const Geo& g, int warp) {
  c.phase = 0;
  phase_slots(g, 0, c.slot, c.s_end);
  if (c.slot < c.s_end) cursor_enter_slot(c, a, g, warp);
  cursor_normalize(c, a, g, warp);
}

__device__ void cursor_next(Cursor& c, const ExpertsArgs& a, const Geo& g, int warp) {
  if (++c.chunk == c.nchunks) {
    c.chunk = 0;
    c.item += kWarps;
  }
  cursor_normalize(c, a, g, warp);
}

// Lane 0: issue the 8 row copies of the stage the cursor names into `buf`.
__device__ void issue_stage(const Cursor& c, const ExpertsArgs& a, const Geo& g, unsigned char* buf,
                            uint64_t* bar, uint64_t policy) {
  if (c.phase == 0) {
    const int lq = c.item - slot_qbase(g, c.slot);
    const uint16_t *gate_base, *up_base;
    if (c.slot < g.n_active) {
      const int e = a.sched[1 + c.slot] - a.expert_base;
      gate_base = a.gate_up + static_cast<size_t>(e) * 2 * a.I * a.H;
      up_base = gate_base + static_cast<size_t>(a.I) * a.H;
    } else {
      gate_base = a.sh_gate;
      up_base = a.sh_up;
    }
    const int cols = g.cu, pitch = cols * 2 + 16;
    const uint32_t bytes = cols * 2;
    mbar_arrive_expect_tx(bar, 8 * bytes);
    const size_t col0 = static_cast<size_t>(c.chunk) * cols;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const uint16_t* base = r < 4 ? gate_base : up_base;
      const size_t row = static_cast<size_t>(4 * lq + (r & 3));
      bulk_g2s(buf + r * pitch, base + row * a.H + col0, bytes, bar, policy);
    }
  } else {
    const int lo8 = c.item - c.slot * g.ops;
    const bool routed = c.slot < g.n_active;
    const int kd = routed ? a.I : a.Is;
    const int cols = routed ? g.cdr : g.cds, pitch = cols * 2 + 16;
    const uint16_t* base = routed ? a.down + static_cast<size_t>(a.sched[1 + c.slot] - a.expert_base) *
                                                 a.H * a.I
                                  : a.sh_down;
    const uint32_t bytes = cols * 2;
    mbar_arrive_expect_tx(bar, 8 * bytes);
    const size_t col0 = static_cast<size_t>(c.chunk) * cols;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const size_t row = static_cast<size_t>(8 * lo8 + r);
      bulk_g2s(buf + r * pitch, base + row * kd + col0, bytes, bar, policy);
    }
  }
}

// Accumulate one stage: 8 rows x `cols` columns starting at column col0,
// NT tokens of f32 activations (row stride xstride) in shared memory.
template <int NT>
__device__ __forceinline__ void stage_fma(const unsigned char* buf, int pitch, int cols, const float* xs,
                                          int xstride, int col0, int r, int q, float (&acc)[kTGP][8]) {
  const uint16_t* wrow = reinterpret_cast<const uint16_t*>(buf + r * pitch) + q * 8;
  const float* xq = xs + col0 + q * 8;
  const int nb = cols >> 5;
#pragma unroll 4
  for (int b = 0; b < nb; ++b) {
    const uint4 w = *reinterpret_cast<const uint4*>(wrow + b * 32);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float* xr = xq + t * xstride + b * 32;
      fma8(w, *reinterpret_cast<const float4*>(xr), *reinterpret_cast<const float4*>(xr + 4), acc[t]);
    }
  }
}

__device__ __forceinline__ void stage_fma_nt(int nt, const unsigned char* buf, int pitch, int cols,
                                             const float* xs, int xstride, int col0, int r, int q,
                                             float (&acc)[kTGP][8]) {
  if (nt == 1)
    stage_fma<1>(buf, pitch, cols, xs, xstride, col0, r, q, acc);
  else if (nt == 2)
    stage_fma<2>(buf, pitch, cols, xs, xstride, col0, r, q, acc);
  else if (nt == 3)
    stage_fma<3>(buf, pitch, cols, xs, xstride, col0, r, q, acc);
  else
    stage_fma<4>(buf, pitch, cols, xs, xstride, col0, r, q, acc);
}

__global__ void __launch_bounds__(kThreads, 1) k_experts(ExpertsArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* ring = smem;                                                    // [warps][stages][4224]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWarps * kRing * kStageBytes);  // [warps][stages]
  int* s_abort = reinterpret_cast<int*>(bars + kWarps * kRing);
  float* xs = reinterpret_cast<float*>(smem + kWarps * kRing * kStageBytes + 512);  // [kTGP][xstride]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane & 7, q = lane >> 3;
  unsigned char* my_ring = ring + warp * kRing * kStageBytes;
  uint64_t* my_bars = bars + warp * kRing;

  if (threadIdx.x == 0) *s_abort = 0;
  if (lane == 0) {
    for (int i = 0; i < kRing; ++i) mbar_init(&my_bars[i], 1);
  }
  fence_mbar_init();

  pdl_wait();  // the schedule comes from the route kernel
  pdl_launch_dependents();

  Geo g;
  g.n_active = a.sched[0];
  g.qpr = a.I / 4;
  g.qps = a.Is / 4;
  g.ops = a.H / 8;
  g.cu = chunk_cols(a.H);
  g.cdr = chunk_cols(a.I);
  g.cds = chunk_cols(a.Is);
  {
    const long long Q = static_cast<long long>(g.n_active) * g.qpr + g.qps;
    const long long O = static_cast<long long>(g.n_active + 1) * g.ops;
    const long long G = gridDim.x, c = blockIdx.x;
    g.up_lo = static_cast<int>(Q * c / G);
    g.up_hi = static_cast<int>(Q * (c + 1) / G);
    g.dn_lo = static_cast<int>(O * c / G);
    g.dn_hi = static_cast<int>(O * (c + 1) / G);
  }
  __syncthreads();  // barrier init visible to all warps

  const uint64_t policy = l2_evict_first_policy();
  Cursor ic;  // issue cursor (meaningful in lane 0)
  int issued = 0;
  if (lane == 0) {
    cursor_begin(ic, a, g, warp);
    for (int i = 0; i < kRing && ic.phase < 2; ++i) {
      issue_stage(ic, a, g, my_ring + i * kStageBytes, &my_bars[i], policy);
      ++issued;
      cursor_next(ic, a, g, warp);
    }
  }
  int consumed = 0;
  const int xstride_up = a.H;
  bool aborted = false;

  for (int phase = 0; phase < 2 && !aborted; ++phase) {
    int s0, s1;
    phase_slots(g, phase, s0, s1);
    for (int s = s0; s < s1 && !aborted; ++s) {
      const bool routed = s < g.n_active;
      const int ntok = slot_tokens(a, g, s);
      const int p0 = routed ? a.sched[1 + a.E + s] : 0;
      const int32_t* pairs = a.sched + 2 + 2 * a.E + p0;
      int lo, hi;
      slot_items(g, phase, s, lo, hi);
      const int nchunks = slot_chunks(a, g, phase, s);
      const int cols = phase == 0 ? g.cu : (routed ? g.cdr : g.cds);
      const int pitch = cols * 2 + 16;
      const int kd = phase == 0 ? a.H : (routed ? a.I : a.Is);
      if (phase == 1) {
        // All SwiGLU rows of this slot must be complete (bounded wait).
        if (threadIdx.x == 0) {
          const int target = slot_nq(g, s);
          if (ld_acquire_gpu(&a.up_done[s]) < target) {
            const uint64_t t0 = global_ns();
            while (ld_acquire_gpu(&a.up_done[s]) < target) {
              if (global_ns() - t0 > kWaitNs) {
                set_error(a.err, kErrTimeout);
                *s_abort = 1;
                break;
              }
              __nanosleep(256);
            }
          }
        }
        __syncthreads();
        if (*reinterpret_cast<volatile int*>(s_abort)) {
          aborted = true;
          break;
        }
      }
      for (int tg = 0; tg * kTGP < ntok && !aborted; ++tg) {
        const int nt = min(kTGP, ntok - tg * kTGP);
        __syncthreads();  // previous pass finished reading xs
        // Stage the pass's activations as f32 (rows nt..kTGP-1 zero).
        {
          const int per_row = kd >> 3;
          for (int i = threadIdx.x; i < kTGP * per_row; i += kThreads) {
            const int t = i / per_row, c8 = (i - t * per_row) * 8;
            float4 lo4 = make_float4(0.f, 0.f, 0.f, 0.f), hi4 = lo4;
            if (t < nt) {
              uint4 v;
              if (phase == 0) {
                const int tok = routed ? pairs[tg * kTGP + t] / a.K : tg * kTGP + t;
                v = *reinterpret_cast<const uint4*>(a.x + static_cast<size_t>(tok) * a.H + c8);
              } else if (routed) {
                v = ld_cg_u4(a.act + static_cast<size_t>(pairs[tg * kTGP + t]) * a.I + c8);
              } else {
                v = ld_cg_u4(a.act_sh + static_cast<size_t>(tg * kTGP + t) * a.Is + c8);
              }
              lo4 = make_float4(lo_bf16(v.x), hi_bf16(v.x), lo_bf16(v.y), hi_bf16(v.y));
              hi4 = make_float4(lo_bf16(v.z), hi_bf16(v.z), lo_bf16(v.w), hi_bf16(v.w));
            }
            *reinterpret_cast<float4*>(xs + t * kd + c8) = lo4;
            *reinterpret_cast<float4*>(xs + t * kd + c8 + 4) = hi4;
          }
        }
        __syncthreads();
        for (int item = lo + warp; item < hi; item += kWarps) {
          float acc[kTGP][8];
#pragma unroll
          for (int t = 0; t < kTGP; ++t)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[t][i] = 0.0f;
          for (int ch = 0; ch < nchunks; ++ch) {
            const int slot_i = consumed % kRing;
            if (!mbar_wait_bounded(&my_bars[slot_i], (consumed / kRing) & 1, kWaitNs)) {
              if (lane == 0) set_error(a.err, kErrTimeout);
              *reinterpret_cast<volatile int*>(s_abort) = 1;
              aborted = true;
              break;
            }
            stage_fma_nt(nt, my_ring + slot_i * kStageBytes, pitch, cols, xs, kd, ch * cols, r, q, acc);
            ++consumed;
            __syncwarp();
            if (lane == 0 && ic.phase < 2) {
              fence_proxy_async_smem();
              const int j = issued % kRing;
              issue_stage(ic, a, g, my_ring + j * kStageBytes, &my_bars[j], policy);
              ++issued;
              cursor_next(ic, a, g, warp);
            }
          }
          if (aborted) break;
          // Epilogue: reference reduction tree, then the bf16 boundaries.
          float val[kTGP];
#pragma unroll
          for (int t = 0; t < kTGP; ++t) val[t] = reduce_partials_strided(acc[t]);
          if (phase == 0) {
            const int lq = item - slot_qbase(g, s);
#pragma unroll
            for (int t = 0; t < kTGP; ++t) {
              const uint32_t vb = f32_to_bf16(val[t]);
              const uint32_t ub = __shfl_down_sync(0xffffffffu, vb, 4);
              if (lane < 4 && t < nt) {
                // swiglu_bf16 (src/expert.rs:562-571): bf16(silu) from the table
                const uint16_t out = f32_to_bf16(bf16_to_f32(a.silu_lut[vb]) * bf16_to_f32(ub));
                const int row = 4 * lq + lane;
                if (routed)
                  a.act[static_cast<size_t>(pairs[tg * kTGP + t]) * a.I + row] = out;
                else
                  a.act_sh[static_cast<size_t>(tg * kTGP + t) * a.Is + row] = out;
              }
            }
          } else if (lane < 8) {
            const int h = 8 * (item - s * g.ops) + lane;
            for (int t = 0; t < nt; ++t) {
              const float d = bf16_to_f32(f32_to_bf16(val[t]));
              if (routed) {
                // bf16(down * route weight) (src/expert.rs:748-751)
                const int p = pairs[tg * kTGP + t];
                a.weighted[static_cast<size_t>(p) * a.H + h] = f32_to_bf16(d * bf16_to_f32(a.pair_score[p]));
              } else {
                // bf16(sigmoid * down) (src/expert.rs:1144-1147)
                const int tok = tg * kTGP + t;
                a.gated_sh[static_cast<size_t>(tok) * a.H + h] = f32_to_bf16(d * bf16_to_f32(a.sh_sig[tok]));
              }
            }
          }
        }
      }
      if (phase == 0 && !aborted) {
        __syncthreads();  // every warp's SwiGLU rows of this slot are stored
        if (threadIdx.x == 0 && hi > lo) {
          __threadfence();
          atomicAdd(&a.up_done[s], hi - lo);
        }
      }
    }
  }
  if (aborted && lane == 0) {
    // Let this warp's copies in flight land before the CTA's shared memory
    // is released (bounded).
    for (int k = consumed; k < issued; ++k) mbar_wait_bounded(&my_bars[k % kRing], (k / kRing) & 1, kDrainNs);
  }
}

int g_num_sms = 0;

}  // namespace

size_t experts_smem_bytes(const Shape& s) {
  const int kmax = max(s.H, max(s.I, s.Is));
  return static_cast<size_t>(kWarps) * kRing * kStageBytes + 512 + static_cast<size_t>(kTGP) * kmax * 4;
}

cudaError_t launch_experts(const Shape& s, const LayerWeights& w, const Luts& luts, const Scratch& sc,
                           const uint16_t* x, int T, const uint16_t* topk_score, cudaStream_t st) {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
  }
  const size_t smem = experts_smem_bytes(s);
  cudaError_t e = cudaFuncSetAttribute(k_experts, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  ExpertsArgs a{s.H, s.I, s.Is, s.E, s.K, T, x, w.gate_up, w.down, w.sh_gate, w.sh_up, w.sh_down,
                w.expert_base, luts.silu, sc.sched, topk_score, sc.sh_sig, sc.act, sc.act_sh,
                sc.weighted, sc.gated_sh, sc.up_done, sc.err};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g_num_sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, k_experts, a);
}

}  // namespace fw
