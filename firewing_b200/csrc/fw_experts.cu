// fw_experts.cu -- persistent expert kernel for the decode path (sm_100a).
//
// One CTA per SM (cooperative launch, so all CTAs are co-resident).  A
// layer's expert work is two unit spaces, each ordered slot-major (slots =
// active routed experts in ascending id, then the shared expert at slot
// n_active):
//   up   : unit = (slot, token pass, quad); a quad is 4 gate rows + the 4
//          matching up rows of the slot's gate_up weights;
//   down : unit = (slot, token pass, octet); an octet is 8 down rows.
// A token pass covers up to `tgp` of the slot's tokens (their activations
// sit in shared memory as f32).  Units all stream the same bytes, so each
// CTA takes one contiguous, equal-sized unit range: a slot with many tokens
// (the shared expert, a hot expert) spreads its passes over several SMs.
//
// Inside a CTA the units of a pass go round-robin to 8 warps.  Every warp
// owns a 2-stage shared-memory ring.  A stage is 8 rows x up to 512 columns
// (1 KB per row).  After consuming a stage the warp refills it: lane 0 posts
// the expected bytes on the stage's mbarrier and lanes 0..7 each issue one
// row's bulk async copy (cp.async.bulk, never multicast).  Rows are padded
// by 16 bytes so the 8 lanes of a quarter-warp, which read the same columns
// of 8 different rows, hit 8 distinct bank groups.  Activations sit in
// shared memory as bf16 and meet the weights in sm_100 mixed-precision FMAs
// (bf16 operands, f32 accumulator: fw::fma8_bf16).
//
// Exact reduction (src/expert.rs:514-552): lane l owns row r = l & 7 and
// partials 8q..8q+7, q = l >> 3; it walks the 32-column blocks of its row
// in order with one 16-byte shared load per block, and
// fw::reduce_partials_strided applies the reference tree.
//
// The down rows of a slot need all of that slot's SwiGLU rows: a CTA adds
// the up units it finished for a slot to up_done[slot] (release); a CTA
// waits (acquire, bounded) for the slot's full unit count before staging
// its activations.  Up work never waits, so the waits always end.
#include <cstdint>

#include "fw_common.cuh"
#include "fw_kernels.h"

namespace fw {
namespace {

constexpr int kWarps = 8;                     // warps per CTA (one ring each)
constexpr int kThreads = kWarps * 32;
// Ring per warp: 2 stages; tiled stages are exactly 8 KB, padded
// reference-layout stages 8 rows of 1040 bytes.
template <bool kTiled> struct RingCfg {
  static constexpr int kRing = 2;                                     // stages per warp ring
  static constexpr int kStageBytes = kTiled ? 8192 : 8 * (512 * 2 + 16);  // 8192 / 8320
};
constexpr int kMaxTGP = 8;                        // tokens per pass (upper bound)
constexpr int kSmemMeta = 512;                    // mbarriers, abort flag, token table
constexpr uint64_t kWaitNs = 2000000000ull;       // bounded waits: 2 s
constexpr uint64_t kDrainNs = 200000000ull;       // drain after abort: 0.2 s

struct ExpertsArgs {
  int H, I, Is, E, K, T, tgp;
  const uint16_t* x;        // [T][H]
  const uint16_t* gate_up;  // [E_local][2I][H]
  const uint16_t* down;     // [E_local][H][I]
  const uint16_t* sh_gate;  // [Is][H]
  const uint16_t* sh_up;    // [Is][H]
  const uint16_t* sh_down;  // [H][Is]
  int ep_world;             // bank index of expert e: e / ep_world
  const uint16_t* silu_lut;
  const int32_t* sched;
  const uint16_t* pair_score;  // [T*K]
  const uint16_t* sh_sig;      // [T]
  uint16_t* act;               // [T*K][2I] gate | up rows (bf16), SwiGLU applied when staged
  uint16_t* act_sh;            // [T][2Is]
  uint16_t* weighted;          // [T*K][H]
  uint16_t* gated_sh;          // [T][H]
  int* up_done;                // [E+1], zeroed by the route kernel
  int* err;
  const uint16_t* sh_x;        // [sh_T][H] the shared expert's token rows
  int sh_T;
  // Bound of the waits on up_done (ns), and a count added to every up_done
  // target (0; a test makes it unreachable to exercise the bounded wait).
  unsigned long long wait_ns;
  int stall;
  // Expert parallelism over peer memory (ep.world > 0): routed rows go to
  // their owner's window (ep_recv_row) instead of `weighted`, and the
  // kernel's last CTA sets this rank's done flag in every window.
  EpPeers ep;
  // L2 prefetch once a CTA's units are done (see Scratch::prefetch)
  const void* pf[3];
  unsigned long long pf_bytes[3];
};

// This CTA's share of the prefetch ranges (thread 0; 16-byte aligned
// ranges of 16-byte multiples), in pieces of at most 64 KB.
__device__ __forceinline__ void prefetch_share(const ExpertsArgs& a) {
  if (threadIdx.x != 0) return;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    if (a.pf[i] == nullptr || a.pf_bytes[i] == 0) continue;
    const unsigned long long share = ((a.pf_bytes[i] + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
    const unsigned long long b0 = share * blockIdx.x;
    const unsigned long long end = min(b0 + share, a.pf_bytes[i]);
    for (unsigned long long o = b0; o < end; o += 65536)
      bulk_prefetch_l2(static_cast<const unsigned char*>(a.pf[i]) + o, static_cast<uint32_t>(min(65536ull, end - o)));
  }
}

// Destination of pair `pair`'s weighted row: `weighted`, or under expert
// parallelism over peer memory (kEp) the owner's window.
template <bool kEp>
__device__ __forceinline__ uint16_t* routed_row(const ExpertsArgs& a, int pair) {
  if constexpr (kEp) return ep_recv_row(a.ep, pair);
  return a.weighted + static_cast<size_t>(pair) * a.H;
}

// Per-launch constants, identical in every thread of a CTA.
struct Ctx {
  const ExpertsArgs* a;
  int n_active;
  const int32_t* up_pref;  // [n_active + 2] cost prefix per slot (shared memory)
  const int32_t* dn_pref;
  const int32_t* offs;     // [n_active + 1] pair offsets per slot (shared memory)
  const int32_t* act_ids;  // [n_active] expert id per slot (shared memory)
  int lo[2], hi[2];        // this CTA's unit range per phase
  int qpr, qps, ops;       // quads per routed / shared slot, octets per slot
  int cu, cdr, cds;        // chunk columns: up, down routed, down shared
};

__device__ __forceinline__ const int32_t* pref(const Ctx& c, int phase) { return phase ? c.dn_pref : c.up_pref; }
__device__ __forceinline__ int units_per_pass(const Ctx& c, int phase, int s) {
  return phase ? c.ops : (s < c.n_active ? c.qpr : c.qps);
}
__device__ __forceinline__ int n_chunks(const Ctx& c, int phase, int s) {
  if (phase == 0) return c.a->H / c.cu;
  return s < c.n_active ? c.a->I / c.cdr : c.a->Is / c.cds;
}
__device__ __forceinline__ int chunk_width(const Ctx& c, int phase, int s) {
  return phase == 0 ? c.cu : (s < c.n_active ? c.cdr : c.cds);
}

// A pass = (phase, slot, token pass) restricted to this CTA: items qa..qb-1
// (local quad / octet indices of the slot).  CTAs split each phase's COST
// space, where a unit of a pass with nt tokens costs unit_cost(phase, nt)
// (the route kernel's prefix); a unit belongs to the CTA whose range holds
// its start.
struct Pass {
  int phase, s, tg, qa, qb;
};

__device__ __forceinline__ int pad_tokens(int nt) { return nt <= 1 ? nt : nt <= 2 ? 2 : nt <= 4 ? 4 : 8; }
// Cost of one unit of a pass with nt tokens (must match the route kernel).
__device__ __forceinline__ int unit_cost(int phase, int nt) { return 4 + (phase ? 4 : 1) * pad_tokens(nt); }

__device__ __forceinline__ int slot_tokens(const Ctx& c, int s) {
  const ExpertsArgs& a = *c.a;
  return s < c.n_active ? c.offs[s + 1] - c.offs[s] : a.sh_T;
}

// Slot whose cost range contains u (binary search over the prefix).
__device__ int slot_of(const int32_t* p, int n_slots, int u) {
  int lo = 0, hi = n_slots - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p[mid] <= u) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ int ceil_div_pos(int a, int b) { return a <= 0 ? 0 : (a + b - 1) / b; }

// From pass (s, tg) onwards, find the first pass with units in this CTA's
// range; false when the range is exhausted.
__device__ bool settle_pass(const Ctx& c, int phase, int s, int tg, Pass& p) {
  const int32_t* pr = pref(c, phase);
  const int lo = c.lo[phase], hi = c.hi[phase];
  const int tgp = c.a->tgp;
  while (s <= c.n_active) {
    const int ntok = slot_tokens(c, s);
    const int ntg = (ntok + tgp - 1) / tgp;
    const int n = units_per_pass(c, phase, s);
    for (; tg < ntg; ++tg) {
      const int base = pr[s] + tg * n * unit_cost(phase, tgp);
      if (base >= hi) return false;
      const int nt = min(tgp, ntok - tg * tgp);
      const int u = unit_cost(phase, nt);
      const int i0 = ceil_div_pos(lo - base, u);
      const int i1 = min(n, ceil_div_pos(hi - base, u));
      if (i0 < i1) {
        p = Pass{phase, s, tg, i0, i1};
        return true;
      }
    }
    ++s;
    tg = 0;
  }
  return false;
}

__device__ bool first_pass(const Ctx& c, int phase, Pass& p) {
  const int lo = c.lo[phase], hi = c.hi[phase];
  if (lo >= hi) return false;
  const int32_t* pr = pref(c, phase);
  const int s = slot_of(pr, c.n_active + 1, lo);
  const int n = units_per_pass(c, phase, s);
  const int tg = (lo - pr[s]) / (n * unit_cost(phase, c.a->tgp));
  return settle_pass(c, phase, s, tg, p);
}

__device__ bool next_pass(const Ctx& c, Pass& p) {
  Pass q;
  if (!settle_pass(c, p.phase, p.s, p.tg + 1, q)) return false;
  p = q;
  return true;
}

// Issue-side cursor over this warp's stages (uniform across the warp).
struct Cursor {
  Pass p;
  bool live;
  int item, chunk, nchunks, cols;
  const uint16_t* row0;  // up: gate base; down: down base
  const uint16_t* row1;  // up: up base
};

__device__ void cursor_slot(Cursor& k, const Ctx& c) {
  const ExpertsArgs& a = *c.a;
  const int s = k.p.s;
  k.nchunks = n_chunks(c, k.p.phase, s);
  k.cols = chunk_width(c, k.p.phase, s);
  if (k.p.phase == 0) {
    if (s < c.n_active) {
      k.row0 = a.gate_up + static_cast<size_t>(c.act_ids[s] / a.ep_world) * 2 * a.I * a.H;
      k.row1 = k.row0 + static_cast<size_t>(a.I) * a.H;
    } else {
      k.row0 = a.sh_gate;  // tiled: the shared gate/up tiles
      k.row1 = a.sh_up;
    }
  } else {
    k.row0 = s < c.n_active ? a.down + static_cast<size_t>(c.act_ids[s] / a.ep_world) * a.H * a.I
                            : a.sh_down;
    k.row1 = nullptr;
  }
}

// Advance to the first pass with an item for this warp (or end).
__device__ void cursor_settle(Cursor& k, const Ctx& c, int warp) {
  while (k.live && k.item >= k.p.qb) {
    const int s_prev = k.p.s, ph_prev = k.p.phase;
    if (!next_pass(c, k.p)) {
      if (k.p.phase == 0 && first_pass(c, 1, k.p)) {
        // continue in the down phase
      } else {
        k.live = false;
        return;
      }
    }
    k.item = k.p.qa + warp;
    k.chunk = 0;
    if (k.p.s != s_prev || k.p.phase != ph_prev) cursor_slot(k, c);
  }
}

__device__ void cursor_begin(Cursor& k, const Ctx& c, int warp) {
  k.live = first_pass(c, 0, k.p) || first_pass(c, 1, k.p);
  if (!k.live) return;
  k.item = k.p.qa + warp;
  k.chunk = 0;
  cursor_slot(k, c);
  cursor_settle(k, c, warp);
}

__device__ __forceinline__ void cursor_next(Cursor& k, const Ctx& c, int warp) {
  if (++k.chunk == k.nchunks) {
    k.chunk = 0;
    k.item += kWarps;
    cursor_settle(k, c, warp);
  }
}

// Whole warp: refill `buf` with the stage the cursor names.  Reference
// layout: lane 0 posts the byte count, lanes 0..7 copy one padded row each.
// Tiled layout: the stage is one contiguous tile, a single copy.
template <bool kTiled>
__device__ __forceinline__ void issue_stage(const Cursor& k, const Ctx& c, unsigned char* buf, uint64_t* bar,
                                            uint64_t policy, int lane) {
  const ExpertsArgs& a = *c.a;
  fence_proxy_async_smem();
  if (kTiled) {
    if (lane == 0) {
      const uint32_t bytes = 8u * k.cols * 2;
      mbar_arrive_expect_tx(bar, bytes);
      const size_t tile = static_cast<size_t>(k.item) * k.nchunks + k.chunk;
      bulk_g2s(buf, k.row0 + tile * 8 * k.cols, bytes, bar, policy);
    }
    return;
  }
  const int pitch = k.cols * 2 + 16;
  const uint32_t bytes = k.cols * 2;
  if (lane == 0) mbar_arrive_expect_tx(bar, 8 * bytes);
  __syncwarp();
  if (lane < 8) {
    const uint16_t* src;
    if (k.p.phase == 0) {
      const size_t row = static_cast<size_t>(4 * k.item + (lane & 3));
      src = (lane < 4 ? k.row0 : k.row1) + row * a.H;
    } else {
      const int kd = k.p.s < c.n_active ? a.I : a.Is;
      src = k.row0 + static_cast<size_t>(8 * k.item + lane) * kd;
    }
    bulk_g2s(buf + lane * pitch, src + static_cast<size_t>(k.chunk) * k.cols, bytes, bar, policy);
  }
}

// Accumulate one stage: 8 rows x `cols` columns from column col0, NT tokens
// of bf16 activations (row stride xstride elements) in shared memory.
// Reference layout: rows padded to cols*2+16 bytes.  Tiled layout: 1 KB
// segments of 8 rows x 64 columns, row r at byte r*128 of a segment, its
// 16-byte chunk j at chunk position j ^ r.
template <int NT, bool kTiled>
__device__ __forceinline__ void stage_fma(const unsigned char* buf, int cols, const uint16_t* xs, int xstride,
                                          int col0, int r, int q, float (&acc)[kMaxTGP][8]) {
  const unsigned char* wrow = buf + r * (kTiled ? 128 : cols * 2 + 16);
  const uint16_t* xq = xs + col0 + q * 8;
  const int nb = cols >> 5;
#pragma unroll 4
  for (int b = 0; b < nb; ++b) {
    const int off = kTiled ? ((b >> 1) * 1024 + (((4 * (b & 1) + q) ^ r) << 4)) : (4 * b + q) * 16;
    const uint4 w = *reinterpret_cast<const uint4*>(wrow + off);
#pragma unroll
    for (int t = 0; t < NT; ++t)
      fma8_bf16(w, *reinterpret_cast<const uint4*>(xq + t * xstride + b * 32), acc[t]);
  }
}

// Per-pass token table in shared memory: tok_row[t] is the pair id (routed)
// or token id (shared) of the pass's token t; tok_scale[t] its route weight
// (routed) or sigmoid gate (shared) as f32.
template <int NT, bool kEp>
__device__ __forceinline__ void epilogue(const Ctx& c, const Pass& p, int item, int nt, float (&acc)[kMaxTGP][8],
                                         int lane, const int* tok_row, const float* tok_scale) {
  const ExpertsArgs& a = *c.a;
  const bool routed = p.s < c.n_active;
  float val[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) val[t] = reduce_partials_strided(acc[t]);
  if (p.phase == 0) {
    // Gate and up rows as bf16 (linear_bf16); SwiGLU is applied when the
    // down phase stages them.
    if (lane < 8) {
      const int row = 4 * item + (lane & 3);
      const int half = routed ? a.I : a.Is;
      const int col = lane < 4 ? row : half + row;
      uint16_t* base = routed ? a.act : a.act_sh;
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < nt) base[static_cast<size_t>(tok_row[t]) * 2 * half + col] = f32_to_bf16(val[t]);
    }
  } else if (lane < 8) {
    const int h = 8 * item + lane;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t < nt) {
        const float d = bf16_to_f32(f32_to_bf16(val[t]));
        // routed: bf16(down * route weight) (src/expert.rs:748-751);
        // shared: bf16(sigmoid * down) (src/expert.rs:1144-1147)
        uint16_t* dst = routed ? routed_row<kEp>(a, tok_row[t]) : a.gated_sh + static_cast<size_t>(tok_row[t]) * a.H;
        dst[h] = f32_to_bf16(d * tok_scale[t]);
      }
    }
  }
}

template <int NT, bool kTiled, bool kEp>
__device__ __forceinline__ bool run_items(const Ctx& c, const Pass& p, int nt, const uint16_t* xs, int xstride,
                                          unsigned char* my_ring, uint64_t* my_bars, Cursor& k, int& consumed,
                                          uint64_t policy, int warp, int lane, int* s_abort, const int* tok_row,
                                          const float* tok_scale) {
  constexpr int kRing = RingCfg<kTiled>::kRing, kStageBytes = RingCfg<kTiled>::kStageBytes;
  const int r = lane & 7, q = lane >> 3;
  const int nch = n_chunks(c, p.phase, p.s);
  const int cols = chunk_width(c, p.phase, p.s);
  for (int item = p.qa + warp; item < p.qb; item += kWarps) {
    float acc[kMaxTGP][8];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[t][i] = 0.0f;
    for (int ch = 0; ch < nch; ++ch) {
      const int j = consumed % kRing;
      if (!mbar_wait_bounded(&my_bars[j], (consumed / kRing) & 1, kWaitNs)) {
        if (lane == 0) set_error(c.a->err, kErrTimeout);
        *reinterpret_cast<volatile int*>(s_abort) = 1;
        return false;
      }
      stage_fma<NT, kTiled>(my_ring + j * kStageBytes, cols, xs, xstride, ch * cols, r, q, acc);
      ++consumed;
      __syncwarp();
      if (k.live) {
        issue_stage<kTiled>(k, c, my_ring + j * kStageBytes, &my_bars[j], policy, lane);
        cursor_next(k, c, warp);
      }
    }
    epilogue<NT, kEp>(c, p, item, nt, acc, lane, tok_row, tok_scale);
  }
  return true;
}

template <bool kTiled, bool kEp>
__global__ void __launch_bounds__(kThreads, 1) k_experts(const __grid_constant__ ExpertsArgs a) {
  constexpr int kRing = RingCfg<kTiled>::kRing, kStageBytes = RingCfg<kTiled>::kStageBytes;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* ring = smem;                                                         // [warps][kRing][stage]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWarps * kRing * kStageBytes);  // [warps][kRing]
  int* s_abort = reinterpret_cast<int*>(bars + kWarps * kRing);
  int* tok_row = s_abort + 4;                                    // [kMaxTGP]
  float* tok_scale = reinterpret_cast<float*>(tok_row + kMaxTGP);  // [kMaxTGP]
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + kWarps * kRing * kStageBytes + kSmemMeta);  // [tgp][kd] bf16

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned char* my_ring = ring + warp * kRing * kStageBytes;
  uint64_t* my_bars = bars + warp * kRing;
  if (threadIdx.x == 0) *s_abort = 0;
  if (lane == 0)
    for (int i = 0; i < kRing; ++i) mbar_init(&my_bars[i], 1);
  fence_mbar_init();

  pdl_wait();  // the schedule comes from the route kernel
  pdl_launch_dependents();
  // Under expert parallelism a failed dispatch leaves the schedule stale:
  // compute nothing, but still signal (with the failure) so peers stop waiting.
  const bool skip = kEp && ld_volatile_int(a.err) != 0;

  Ctx c;
  c.a = &a;
  c.n_active = a.sched[0];
  {
    // The schedule's slot tables, once, into shared memory: every cursor step
    // and pass boundary reads them.
    int32_t* t = reinterpret_cast<int32_t*>(xs + static_cast<size_t>(a.tgp) * max(a.H, max(a.I, a.Is)));
    const int n = c.n_active;
    const int32_t* g_act = a.sched + 1;
    const int32_t* g_off = a.sched + 1 + a.E;
    const int32_t* g_up = a.sched + 2 + 2 * a.E + a.T * a.K;
    const int32_t* g_dn = g_up + (a.E + 2);
    int32_t* s_up = t;
    int32_t* s_dn = t + (a.E + 2);
    int32_t* s_off = t + 2 * (a.E + 2);
    int32_t* s_act = s_off + (a.E + 2);
    for (int i = threadIdx.x; i < n + 2; i += kThreads) {
      s_up[i] = g_up[i];
      s_dn[i] = g_dn[i];
      if (i <= n) s_off[i] = g_off[i];
      if (i < n) s_act[i] = g_act[i];
    }
    c.up_pref = s_up;
    c.dn_pref = s_dn;
    c.offs = s_off;
    c.act_ids = s_act;
    __syncthreads();
  }
  c.qpr = a.I / 4;
  c.qps = a.Is / 4;
  c.ops = a.H / 8;
  c.cu = chunk_cols(a.H);
  c.cdr = chunk_cols(a.I);
  c.cds = chunk_cols(a.Is);
  {
    const long long G = gridDim.x, b = blockIdx.x;
    const long long U = c.up_pref[c.n_active + 1], D = c.dn_pref[c.n_active + 1];
    c.lo[0] = static_cast<int>(U * b / G);
    c.hi[0] = static_cast<int>(U * (b + 1) / G);
    c.lo[1] = static_cast<int>(D * b / G);
    c.hi[1] = static_cast<int>(D * (b + 1) / G);
  }
  __syncthreads();  // barrier init visible to all warps

  const uint64_t policy = l2_evict_first_policy();
  Cursor k;
  cursor_begin(k, c, warp);
  for (int i = 0; i < kRing && k.live && !skip; ++i) {
    issue_stage<kTiled>(k, c, my_ring + i * kStageBytes, &my_bars[i], policy, lane);
    cursor_next(k, c, warp);
  }
  int consumed = 0;
  bool aborted = false;

  for (int phase = 0; phase < 2 && !aborted && !skip; ++phase) {
    Pass p;
    bool ok = first_pass(c, phase, p);
    int cur_s = -1, cur_units = 0;
    while (ok && !aborted) {
      const bool routed = p.s < c.n_active;
      if (phase == 0 && p.s != cur_s && cur_s >= 0) {
        // every gate/up row of the previous slot's units is stored
        __syncthreads();
        if (threadIdx.x == 0) {
          __threadfence();
          atomicAdd(&a.up_done[cur_s], cur_units);
        }
        cur_units = 0;
      }
      if (phase == 1 && p.s != cur_s) {
        // all of this slot's up units must be complete (bounded wait)
        if (threadIdx.x == 0) {
          const int target =
              ((slot_tokens(c, p.s) + a.tgp - 1) / a.tgp) * units_per_pass(c, 0, p.s) + a.stall;
          if (ld_acquire_gpu(&a.up_done[p.s]) < target) {
            const uint64_t t0 = global_ns();
            while (ld_acquire_gpu(&a.up_done[p.s]) < target) {
              if (global_ns() - t0 > a.wait_ns) {
                set_error(a.err, kErrTimeout);
                *s_abort = 1;
                break;
              }
              __nanosleep(128);
            }
          }
        }
        __syncthreads();
        if (*reinterpret_cast<volatile int*>(s_abort)) {
          aborted = true;
          break;
        }
      }
      cur_s = p.s;
      cur_units += p.qb - p.qa;
      const int ntok = slot_tokens(c, p.s);
      const int t0 = p.tg * a.tgp;
      const int nt = min(a.tgp, ntok - t0);
      const int kd = phase == 0 ? a.H : (routed ? a.I : a.Is);
      const int32_t* pairs = a.sched + 2 + 2 * a.E + (routed ? c.offs[p.s] : 0);
      const int nt_pad = nt <= 1 ? 1 : nt <= 2 ? 2 : nt <= 4 ? 4 : 8;
      __syncthreads();  // the previous pass finished reading xs and the token table
      if (threadIdx.x < nt) {
        const int t = threadIdx.x;
        if (routed) {
          const int pr = pairs[t0 + t];
          tok_row[t] = pr;
          tok_scale[t] = bf16_to_f32(a.pair_score[pr]);
        } else {
          tok_row[t] = t0 + t;
          tok_scale[t] = bf16_to_f32(a.sh_sig[t0 + t]);
        }
      }
      {
        // Stage the pass's activations as f32 (rows nt..nt_pad-1 zero).  Up:
        // the tokens' inputs.  Down: swiglu_bf16 (src/expert.rs:562-571) of
        // the stored gate/up rows, bf16(bf16(silu(g)) * u), silu from the table.
        const int per_row = kd >> 3;
        for (int i = threadIdx.x; i < nt_pad * per_row; i += kThreads) {
          const int t = i / per_row, c8 = (i - t * per_row) * 8;
          uint4 out = make_uint4(0u, 0u, 0u, 0u);
          if (t < nt) {
            if (phase == 0) {
              const uint16_t* xr = routed ? a.x + static_cast<size_t>(pairs[t0 + t] / a.K) * a.H
                                          : a.sh_x + static_cast<size_t>(t0 + t) * a.H;
              out = *reinterpret_cast<const uint4*>(xr + c8);
            } else {
              const uint16_t* row = routed ? a.act + static_cast<size_t>(pairs[t0 + t]) * 2 * a.I
                                           : a.act_sh + static_cast<size_t>(t0 + t) * 2 * a.Is;
              const uint4 g = ld_cg_u4(row + c8);
              const uint4 u = ld_cg_u4(row + kd + c8);
              const uint32_t gg[4] = {g.x, g.y, g.z, g.w}, uu[4] = {u.x, u.y, u.z, u.w};
              uint16_t sl[8];
#pragma unroll
              for (int e2 = 0; e2 < 4; ++e2) {
                sl[2 * e2] = a.silu_lut[gg[e2] & 0xffffu];
                sl[2 * e2 + 1] = a.silu_lut[gg[e2] >> 16];
              }
              uint32_t o[4];
#pragma unroll
              for (int e2 = 0; e2 < 4; ++e2) {
                const uint32_t lo = f32_to_bf16(bf16_to_f32(sl[2 * e2]) * lo_bf16(uu[e2]));
                const uint32_t hi = f32_to_bf16(bf16_to_f32(sl[2 * e2 + 1]) * hi_bf16(uu[e2]));
                o[e2] = lo | (hi << 16);
              }
              out = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
          *reinterpret_cast<uint4*>(xs + t * kd + c8) = out;
        }
      }
      __syncthreads();
      bool good;
      if (nt_pad == 1)
        good = run_items<1, kTiled, kEp>(c, p, nt, xs, kd, my_ring, my_bars, k, consumed, policy, warp, lane, s_abort,
                               tok_row, tok_scale);
      else if (nt_pad == 2)
        good = run_items<2, kTiled, kEp>(c, p, nt, xs, kd, my_ring, my_bars, k, consumed, policy, warp, lane, s_abort,
                               tok_row, tok_scale);
      else if (nt_pad == 4)
        good = run_items<4, kTiled, kEp>(c, p, nt, xs, kd, my_ring, my_bars, k, consumed, policy, warp, lane, s_abort,
                               tok_row, tok_scale);
      else
        good = run_items<8, kTiled, kEp>(c, p, nt, xs, kd, my_ring, my_bars, k, consumed, policy, warp, lane, s_abort,
                               tok_row, tok_scale);
      if (!good) {
        aborted = true;
        break;
      }
      ok = next_pass(c, p);
    }
    if (phase == 0 && !aborted && cur_s >= 0) {
      __syncthreads();
      if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(&a.up_done[cur_s], cur_units);
      }
    }
  }
  if (aborted && lane == 0) {
    // Stages this warp issued but did not consume: let them land before the
    // CTA's shared memory is released (bounded).
    for (int i = 0; i < kRing; ++i) {
      const int kk = consumed + i;
      if (!mbar_wait_bounded(&my_bars[kk % kRing], (kk / kRing) & 1, kDrainNs)) break;
    }
  }
  prefetch_share(a);
  if constexpr (kEp) ep_signal(a.ep, kEpFlagDone, a.ep.ticket + 1, a.err);
}

// ---- small widths: one producer warp, a CTA-wide ring ----------------------
//
// At a few tokens the FMA work per stage is small and the kernel above is
// bound by its structure: 8 per-warp rings of 2 stages hold whole 4-stage up
// units, so at ~9.5 up units per CTA half the warps idle while the others
// stream a second unit, and every pass boundary is a CTA barrier.  This
// variant (tiled layout, T <= kSmallMaxT) keeps the same schedule, cost
// space and CTA ranges but splits loading from arithmetic:
//   - warp 7 walks the CTA's stage sequence -- its up units, then its down
//     units -- and streams every stage into a CTA-wide ring of R stages
//     (about 200 KB at T = 1) with one bulk copy each, gated by the ring's
//     empty barriers, so the bytes in flight do not depend on how the units
//     fall on warps.  Lanes 0..7 issue 8 consecutive stages per step: one
//     lane issuing alone spent ~0.2 us of instructions per stage;
//   - warps 0..6 take the CTA's units round-robin, each unit's stages in
//     order, with no CTA barriers: the up activations are all T token rows,
//     staged once; the down activations (SwiGLU of the slot's gate/up rows)
//     go to a per-warp buffer after a per-warp bounded wait on up_done.
// A unit's FMA chain, reduction and epilogue are those of the kernel above.
// Deadlock freedom: all up stages precede all down stages in the producer's
// order, and R exceeds a unit's stage count, so every up unit of every CTA
// completes without waiting on a down unit; down units wait only on up
// units.  Every wait is bounded and also ends when another warp aborted.

constexpr int kSmallMaxT = 4;      // widths served by the small-width kernel (measured: T = 8 is faster on the kernel above)
constexpr int kSmallSlot = 8192;   // ring slot: one tiled stage (8 rows x <= 512 columns)
constexpr int kSmallMaxR = 32;     // ring slots at most
// "Full" barriers are indexed by stage mod kSmallFull, independently of the
// ring slot (stage mod R).  Stages are issued in steps of 8, in order across
// steps; F = the first stage of the current step (all below it issued).  A
// consumer waits on stage g only after its previous unit is consumed, so
// g < F + 8 + 7 units x 8 stages; every stage below F - R is consumed.  With
// kSmallFull >= R + 64 the barrier's previous use (stage g - kSmallFull) has
// landed whenever g is waited on, and its next use (g + kSmallFull) cannot
// be issued before g is consumed, so the parity names the right phase.
constexpr int kSmallFull = 128;
constexpr int kIssueLanes = 8;     // producer lanes issuing one stage each per step
constexpr unsigned kIssueMask = 0xffu;
constexpr int kSmallWarps = 7;     // consumer warps; warp 7 is the producer (8 warps keep 255 registers)
constexpr int kSmallThreads = (kSmallWarps + 1) * 32;

struct SmallLayout {
  size_t bars, meta, tables, pairs, toks, xs, wact, total;
  int nx, ntmax, kdmax;
};

__host__ __device__ inline size_t align128(size_t v) { return (v + 127) & ~static_cast<size_t>(127); }

// Shared-memory plan of a CTA with R ring slots: ring, full/empty barriers,
// abort flag, schedule tables, pair tables, per-warp token tables, the token
// rows (x, then the shared expert's rows when they are a separate buffer),
// per-warp down activations.
__host__ __device__ inline SmallLayout small_layout(int H, int I, int Is, int E, int K, int T, int sh_T,
                                                    bool sh_separate, int tgp, int R) {
  SmallLayout L{};
  L.nx = T + (sh_separate ? sh_T : 0);
  L.ntmax = T < tgp ? (T > 0 ? T : 1) : tgp;
  L.kdmax = I > Is ? I : Is;
  L.bars = static_cast<size_t>(R) * kSmallSlot;
  L.meta = L.bars + align128(static_cast<size_t>(kSmallFull + R) * 8);
  L.tables = L.meta + 128;
  L.pairs = L.tables + align128(static_cast<size_t>(4) * (E + 2) * 4);
  L.toks = L.pairs + align128(static_cast<size_t>(2 * T * K + sh_T) * 4);
  L.xs = L.toks + align128(static_cast<size_t>(3) * kSmallWarps * kMaxTGP * 4);
  L.wact = L.xs + align128(static_cast<size_t>(L.nx) * H * 2);
  L.total = L.wact + align128(static_cast<size_t>(kSmallWarps) * L.ntmax * L.kdmax * 2);
  return L;
}

// Ring slots for a small-width launch: the most that fit, at least twice a
// unit's stage count (and 12); 0 when the width is not served.
inline int small_ring_slots(const Shape& s, int T, int sh_T, bool sh_separate, int tgp, size_t smem_max) {
  if (T < 1 || T > kSmallMaxT) return 0;
  const int nch = max(s.H / chunk_cols(s.H), max(s.I / chunk_cols(s.I), s.Is / chunk_cols(s.Is)));
  const int r_min = max(12, 2 * nch + 2);
  if (nch > 8) return 0;  // the full-barrier bound assumes units of at most 8 stages
  for (int R = kSmallMaxR; R >= r_min; --R)
    if (small_layout(s.H, s.I, s.Is, s.E, s.K, T, sh_T, sh_separate, tgp, R).total <= smem_max) return R;
  return 0;
}

// Bounded wait on a ring barrier that also ends when another warp aborted.
__device__ __forceinline__ bool ring_wait(uint64_t* bar, uint32_t parity, volatile int* s_abort, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*s_abort) return false;
    if (global_ns() - t0 > kWaitNs) {
      set_error(err, kErrTimeout);
      *s_abort = 1;
      return false;
    }
  }
}

// Accumulate one tiled stage against NT token rows given by pointer (the
// stage's column chunk starts at col0 of each row).
template <int NT>
__device__ __forceinline__ void stage_fma_rows(const unsigned char* buf, int cols, const uint16_t* const (&xr)[NT],
                                               int col0, int r, int q, float (&acc)[kMaxTGP][8]) {
  const unsigned char* wrow = buf + r * 128;
  const int nb = cols >> 5;
#pragma unroll 4
  for (int b = 0; b < nb; ++b) {
    const int off = (b >> 1) * 1024 + (((4 * (b & 1) + q) ^ r) << 4);
    const uint4 w = *reinterpret_cast<const uint4*>(wrow + off);
#pragma unroll
    for (int t = 0; t < NT; ++t)
      fma8_bf16(w, *reinterpret_cast<const uint4*>(xr[t] + col0 + b * 32 + q * 8), acc[t]);
  }
}

// One unit (all of its stages, starting at ring stage g) for NT padded tokens.
template <int NT>
__device__ __forceinline__ bool small_unit(const Ctx& c, const Pass& p, int item, int nt, const uint16_t* const (&rows)[kMaxTGP],
                                           unsigned char* ring, uint64_t* full, uint64_t* empty, int R, int g,
                                           int lane, volatile int* s_abort, const int* tok_row,
                                           const float* tok_scale) {
  const int r = lane & 7, q = lane >> 3;
  const int nch = n_chunks(c, p.phase, p.s), cols = chunk_width(c, p.phase, p.s);
  const uint16_t* xr[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) xr[t] = rows[t];
  float acc[kMaxTGP][8];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[t][i] = 0.0f;
  for (int ch = 0; ch < nch; ++ch, ++g) {
    const int slot = g % R;
    const bool ok = ring_wait(&full[g % kSmallFull], (g / kSmallFull) & 1, s_abort, c.a->err);
    if (!__all_sync(0xffffffffu, ok)) return false;
    stage_fma_rows<NT>(ring + static_cast<size_t>(slot) * kSmallSlot, cols, xr, ch * cols, r, q, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  epilogue<NT, false>(c, p, item, nt, acc, lane, tok_row, tok_scale);
  return true;
}

// Publish n stored up units of slot s: the warp's stores, then a release
// (fence + add) by lane 0.
__device__ __forceinline__ void flush_up(int* up_done, int s, int n, int lane) {
  __syncwarp();
  if (lane == 0 && n > 0) {
    __threadfence();
    atomicAdd(&up_done[s], n);
  }
}

__global__ void __launch_bounds__(kSmallThreads, 1) k_experts_small(const __grid_constant__ ExpertsArgs a, int R) {
  extern __shared__ __align__(128) unsigned char smem[];
  const bool sh_sep = a.sh_x != a.x;
  const SmallLayout L = small_layout(a.H, a.I, a.Is, a.E, a.K, a.T, a.sh_T, sh_sep, a.tgp, R);
  unsigned char* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);  // [kSmallFull]
  uint64_t* empty = full + kSmallFull;                           // [R]
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L.meta);
  int32_t* tables = reinterpret_cast<int32_t*>(smem + L.tables);
  int32_t* s_pairs = reinterpret_cast<int32_t*>(smem + L.pairs);
  float* s_pscore = reinterpret_cast<float*>(s_pairs + a.T * a.K);
  float* s_shsig = s_pscore + a.T * a.K;
  int* toks = reinterpret_cast<int*>(smem + L.toks);
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + L.xs);
  uint16_t* wact = reinterpret_cast<uint16_t*>(smem + L.wact);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    *s_abort = 0;
    for (int i = 0; i < kSmallFull; ++i) mbar_init(&full[i], 1);
    for (int i = 0; i < R; ++i) mbar_init(&empty[i], 1);
  }
  fence_mbar_init();

  pdl_wait();  // the schedule comes from the route kernel
  pdl_launch_dependents();

  Ctx c;
  c.a = &a;
  c.n_active = a.sched[0];
  {
    const int n = c.n_active;
    const int32_t* g_act = a.sched + 1;
    const int32_t* g_off = a.sched + 1 + a.E;
    const int32_t* g_pairs = a.sched + 2 + 2 * a.E;
    const int32_t* g_up = g_pairs + a.T * a.K;
    const int32_t* g_dn = g_up + (a.E + 2);
    int32_t* s_up = tables;
    int32_t* s_dn = tables + (a.E + 2);
    int32_t* s_off = tables + 2 * (a.E + 2);
    int32_t* s_act = s_off + (a.E + 2);
    for (int i = threadIdx.x; i < n + 2; i += kSmallThreads) {
      s_up[i] = g_up[i];
      s_dn[i] = g_dn[i];
      if (i <= n) s_off[i] = g_off[i];
      if (i < n) s_act[i] = g_act[i];
    }
    for (int i = threadIdx.x; i < a.T * a.K; i += kSmallThreads) {
      s_pairs[i] = g_pairs[i];
      s_pscore[i] = bf16_to_f32(a.pair_score[i]);
    }
    for (int i = threadIdx.x; i < a.sh_T; i += kSmallThreads) s_shsig[i] = bf16_to_f32(a.sh_sig[i]);
    // every token row the up units read: x, then the shared expert's rows
    // when they are a separate buffer
    const int per_row = a.H >> 3;
    for (int i = threadIdx.x; i < L.nx * per_row; i += kSmallThreads) {
      const int t = i / per_row, c8 = (i - t * per_row) * 8;
      const uint16_t* src = t < a.T ? a.x + static_cast<size_t>(t) * a.H : a.sh_x + static_cast<size_t>(t - a.T) * a.H;
      *reinterpret_cast<uint4*>(xs + static_cast<size_t>(t) * a.H + c8) = *reinterpret_cast<const uint4*>(src + c8);
    }
    c.up_pref = s_up;
    c.dn_pref = s_dn;
    c.offs = s_off;
    c.act_ids = s_act;
  }
  c.qpr = a.I / 4;
  c.qps = a.Is / 4;
  c.ops = a.H / 8;
  c.cu = chunk_cols(a.H);
  c.cdr = chunk_cols(a.I);
  c.cds = chunk_cols(a.Is);
  __syncthreads();  // tables, rows and barrier init visible to all warps
  {
    const long long G = gridDim.x, b = blockIdx.x;
    const long long U = c.up_pref[c.n_active + 1], D = c.dn_pref[c.n_active + 1];
    c.lo[0] = static_cast<int>(U * b / G);
    c.hi[0] = static_cast<int>(U * (b + 1) / G);
    c.lo[1] = static_cast<int>(D * b / G);
    c.hi[1] = static_cast<int>(D * (b + 1) / G);
  }

  // Producer: lanes 0..7 issue 8 consecutive stages per step (one copy
  // each), so one step's instruction stream serves 8 stages.  Lane j's slot
  // was last used by stage g - R, issued in an earlier step (R > 8).
  int issued = 0;           // stages issued in complete steps (uniform over the issuing lanes)
  unsigned tail_mask = 0u;  // after an abort: lanes of the last step that issued
  if (warp == kSmallWarps) {
    if (lane < kIssueLanes) {
      const uint64_t policy = l2_evict_first_policy();
      bool stop = false;
      for (int phase = 0; phase < 2 && !stop; ++phase) {
        Pass p;
        bool ok = first_pass(c, phase, p);
        while (ok && !stop) {
          Cursor k;
          k.p = p;
          cursor_slot(k, c);
          const int n = (p.qb - p.qa) * k.nchunks;  // stages of this pass
          const uint32_t bytes = 8u * k.cols * 2;
          for (int o0 = 0; o0 < n; o0 += kIssueLanes) {
            const int o = o0 + lane, gs = issued + lane;
            bool good = true, sent = false;
            if (o < n) {
              const int slot = gs % R;
              if (gs >= R) good = ring_wait(&empty[slot], ((gs / R) - 1) & 1, s_abort, a.err);
              if (good) {
                fence_proxy_async_smem();
                uint64_t* fb = &full[gs % kSmallFull];
                mbar_arrive_expect_tx(fb, bytes);
                const int item = p.qa + o / k.nchunks, ch = o % k.nchunks;
                const size_t tile = static_cast<size_t>(item) * k.nchunks + ch;
                bulk_g2s(ring + static_cast<size_t>(slot) * kSmallSlot, k.row0 + tile * 8 * k.cols, bytes, fb,
                         policy);
                sent = true;
              }
            }
            if (__any_sync(kIssueMask, !good)) {
              tail_mask = __ballot_sync(kIssueMask, sent);
              stop = true;
              break;
            }
            issued += min(kIssueLanes, n - o0);
          }
          ok = next_pass(c, p);
        }
      }
    }
  } else {
    int* tok_row = toks + warp * kMaxTGP;
    float* tok_scale = reinterpret_cast<float*>(toks + (kSmallWarps + warp) * kMaxTGP);
    int* tok_x = toks + (2 * kSmallWarps + warp) * kMaxTGP;
    uint16_t* my_act = wact + static_cast<size_t>(warp) * L.ntmax * L.kdmax;
    int g = 0, u = 0;
    int cur_phase = -1, cur_s = -1, cur_tg = -1;
    int nt = 0, nt_pad = 1, kd = 0;
    const uint16_t* rows[kMaxTGP];
    int pend_s = -1, pend_n = 0;  // up units stored but not yet counted in up_done
    bool aborted = false;
    for (int phase = 0; phase < 2 && !aborted; ++phase) {
      Pass p;
      bool ok = first_pass(c, phase, p);
      while (ok && !aborted) {
        const int nch = n_chunks(c, phase, p.s);
        for (int item = p.qa; item < p.qb; ++item, ++u, g += nch) {
          if (u % kSmallWarps != warp) continue;
          if (phase != cur_phase || p.s != cur_s || p.tg != cur_tg) {
            // this warp enters a new pass: its token table and activations
            const bool routed = p.s < c.n_active;
            const int t0 = p.tg * a.tgp;
            nt = min(a.tgp, slot_tokens(c, p.s) - t0);
            nt_pad = pad_tokens(nt);
            kd = phase == 0 ? a.H : (routed ? a.I : a.Is);
            __syncwarp();  // the previous pass's readers of the table and buffer are done
            if (lane < nt) {
              if (routed) {
                const int pr = s_pairs[c.offs[p.s] + t0 + lane];
                tok_row[lane] = pr;
                tok_scale[lane] = s_pscore[pr];
                tok_x[lane] = pr / a.K;
              } else {
                tok_row[lane] = t0 + lane;
                tok_scale[lane] = s_shsig[t0 + lane];
                tok_x[lane] = (sh_sep ? a.T : 0) + t0 + lane;
              }
            }
            if (phase == 1) {
              // all of the slot's up units are stored (bounded wait)
              const int target =
                  ((slot_tokens(c, p.s) + a.tgp - 1) / a.tgp) * units_per_pass(c, 0, p.s) + a.stall;
              int good = 1;
              if (lane == 0 && ld_acquire_gpu(&a.up_done[p.s]) < target) {
                const uint64_t w0 = global_ns();
                while (ld_acquire_gpu(&a.up_done[p.s]) < target) {
                  if (*s_abort) {
                    good = 0;
                    break;
                  }
                  if (global_ns() - w0 > a.wait_ns) {
                    set_error(a.err, kErrTimeout);
                    *s_abort = 1;
                    good = 0;
                    break;
                  }
                  __nanosleep(64);
                }
              }
              if (!__shfl_sync(0xffffffffu, good, 0)) {
                aborted = true;
                break;
              }
              (void)ld_acquire_gpu(&a.up_done[p.s]);  // every lane: acquire before reading the rows
              // SwiGLU (src/expert.rs:562-571) of the stored gate/up rows,
              // bf16(bf16(silu(g)) * u), silu from the table
              const int per_row = kd >> 3;
              for (int i = lane; i < nt * per_row; i += 32) {
                const int t = i / per_row, c8 = (i - t * per_row) * 8;
                const uint16_t* row = routed ? a.act + static_cast<size_t>(s_pairs[c.offs[p.s] + t0 + t]) * 2 * a.I
                                             : a.act_sh + static_cast<size_t>(t0 + t) * 2 * a.Is;
                const uint4 gv = ld_cg_u4(row + c8);
                const uint4 uv = ld_cg_u4(row + kd + c8);
                const uint32_t gg[4] = {gv.x, gv.y, gv.z, gv.w}, uu[4] = {uv.x, uv.y, uv.z, uv.w};
                uint32_t o[4];
#pragma unroll
                for (int e2 = 0; e2 < 4; ++e2) {
                  const uint32_t sl0 = a.silu_lut[gg[e2] & 0xffffu], sl1 = a.silu_lut[gg[e2] >> 16];
                  const uint32_t lo = f32_to_bf16(bf16_to_f32(sl0) * lo_bf16(uu[e2]));
                  const uint32_t hi = f32_to_bf16(bf16_to_f32(sl1) * hi_bf16(uu[e2]));
                  o[e2] = lo | (hi << 16);
                }
                *reinterpret_cast<uint4*>(my_act + static_cast<size_t>(t) * kd + c8) = make_uint4(o[0], o[1], o[2], o[3]);
              }
            }
            __syncwarp();
#pragma unroll
            for (int t = 0; t < kMaxTGP; ++t) {
              const int tt = t < nt ? t : 0;  // padded tokens read token 0's row (results unused)
              rows[t] = phase == 0 ? xs + static_cast<size_t>(tok_x[tt]) * a.H : my_act + static_cast<size_t>(tt) * kd;
            }
            cur_phase = phase;
            cur_s = p.s;
            cur_tg = p.tg;
          }
          bool good;
          if (nt_pad == 1)
            good = small_unit<1>(c, p, item, nt, rows, ring, full, empty, R, g, lane, s_abort, tok_row,
                                 tok_scale);
          else if (nt_pad == 2)
            good = small_unit<2>(c, p, item, nt, rows, ring, full, empty, R, g, lane, s_abort, tok_row,
                                 tok_scale);
          else if (nt_pad == 4)
            good = small_unit<4>(c, p, item, nt, rows, ring, full, empty, R, g, lane, s_abort, tok_row,
                                 tok_scale);
          else
            good = small_unit<8>(c, p, item, nt, rows, ring, full, empty, R, g, lane, s_abort, tok_row,
                                 tok_scale);
          if (!good) {
            aborted = true;
            break;
          }
          if (phase == 0) {
            // this unit's gate/up rows are stored: count it for the slot
            // (published when the warp moves to another slot)
            if (p.s != pend_s) {
              flush_up(a.up_done, pend_s, pend_n, lane);
              pend_s = p.s;
              pend_n = 0;
            }
            ++pend_n;
          }
        }
        if (aborted) break;
        ok = next_pass(c, p);
      }
      if (phase == 0) {
        // before any down unit can wait on these counts
        flush_up(a.up_done, pend_s, pend_n, lane);
        pend_s = -1;
        pend_n = 0;
      }
    }
  }
  __syncthreads();
  if (warp == kSmallWarps && lane == 0) {
    // Copies still in flight (after an abort): let them land before the
    // CTA's shared memory is released (bounded).  Stages below issued - R
    // were consumed (their slots were reused); the last step's lanes that
    // issued are in tail_mask.
    for (int i = issued > R ? issued - R : 0; i < issued + kIssueLanes; ++i) {
      if (i >= issued && !((tail_mask >> (i - issued)) & 1u)) continue;
      if (!mbar_wait_bounded(&full[i % kSmallFull], (i / kSmallFull) & 1, kDrainNs)) break;
    }
  }
  prefetch_share(a);
}

}  // namespace

// Both layouts use the same tokens per pass (the route kernel's cost
// prefixes depend on it): 8 when the padded 2-stage ring leaves room.
int experts_tokens_per_pass(const Shape& s) {
  const int kmax = max(s.H, max(s.I, s.Is));
  const size_t ring = static_cast<size_t>(kWarps) * 2 * (8 * (512 * 2 + 16)) + kSmemMeta;
  return ring + static_cast<size_t>(8) * kmax * 2 + static_cast<size_t>(4) * (s.E + 2) * 4 <= 220 * 1024 ? 8 : 4;
}

static size_t ring_bytes(bool tiled) {
  return tiled ? static_cast<size_t>(kWarps) * RingCfg<true>::kRing * RingCfg<true>::kStageBytes
               : static_cast<size_t>(kWarps) * RingCfg<false>::kRing * RingCfg<false>::kStageBytes;
}

size_t experts_smem_bytes(const Shape& s, bool tiled) {
  const int kmax = max(s.H, max(s.I, s.Is));
  // ring, meta, activations, then the slot tables (4 x (E + 2) ints)
  return ring_bytes(tiled) + kSmemMeta + static_cast<size_t>(experts_tokens_per_pass(s)) * kmax * 2 +
         static_cast<size_t>(4) * (s.E + 2) * 4;
}

cudaError_t launch_experts(const Shape& s, const LayerWeights& w, const Luts& luts, const Scratch& sc,
                           const uint16_t* x, int T, const uint16_t* topk_score, cudaStream_t st,
                           const uint16_t* sh_x, int sh_T, const EpPeers* ep) {
  DeviceAttrs dev;
  if (const cudaError_t e = current_device_attrs(&dev); e != cudaSuccess) return e;
  const int tgp = experts_tokens_per_pass(s);
  ExpertsArgs a{s.H, s.I, s.Is, s.E, s.K, T, tgp, x, w.gate_up, w.down, w.sh_gate,
                w.sh_up, w.sh_down, w.ep_world, luts.silu, sc.sched, topk_score, sc.sh_sig, sc.act,
                sc.act_sh, sc.weighted, sc.gated_sh, sc.up_done, sc.err, sh_x, sh_T,
                sc.wait_ns, sc.stall, ep != nullptr ? *ep : EpPeers{},
                {sc.prefetch[0], sc.prefetch[1], sc.prefetch[2]},
                {sc.prefetch_bytes[0], sc.prefetch_bytes[1], sc.prefetch_bytes[2]}};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(dev.sms);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  // Small widths on one GPU.  Under expert parallelism (the shared expert's
  // rows in their own buffer) the kernel above keeps the path: the small
  // kernel's separate-rows case has not run on two GPUs.
  const int R = w.tiled && sh_x == x ? small_ring_slots(s, T, sh_T, false, tgp, static_cast<size_t>(dev.smem_optin)) : 0;
  if (R > 0) {
    const size_t smem = small_layout(s.H, s.I, s.Is, s.E, s.K, T, sh_T, false, tgp, R).total;
    cudaError_t e = cudaFuncSetAttribute(k_experts_small, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cfg.blockDim = dim3(kSmallThreads);
    cfg.dynamicSmemBytes = smem;
    return cudaLaunchKernelEx(&cfg, k_experts_small, a, R);
  }
  const size_t smem = experts_smem_bytes(s, w.tiled);
  const bool ep_peers = ep != nullptr && ep->world > 0;
  auto kern = w.tiled ? (ep_peers ? k_experts<true, true> : k_experts<true, false>)
                      : (ep_peers ? k_experts<false, true> : k_experts<false, false>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace fw
