// fw_prefill.cu -- the sparse-MoE block for prefill token counts on the
// sm_100 tensor cores.
//
// The decode path (fw_experts.cu) streams every selected expert's weights
// once per forward and reproduces the reference dot schedule on the CUDA
// cores; that is the right design while a token group is a few tokens.  With
// thousands of tokens (T = 8192: ~160 tokens per expert on average, several
// thousand for a hot expert) the block is a grouped GEMM and belongs on the
// tensor cores:
//
//   router (tensor-core logits + exact repair of those that can be
//           selected, k_router_tc / k_router_fix) -> route (+ pair counts)
//   -> k_pf_offsets (one CTA: pair offsets, work-unit prefixes)
//   -> k_pf_scatter (pairs grouped by expert; token rows copied into the
//                    grouped input xg [pairs][H])
//   -> k_gemm<up>:   per expert, [2I x H] gate/up rows x its xg rows,
//                    SwiGLU in the epilogue -> act [pairs][I] (bf16)
//   -> k_gemm<down>: per expert, [H x I] down rows x act rows, route weight
//                    (or the shared sigmoid gate) in the epilogue ->
//                    weighted [T*K][H] (bf16)
//   -> combine (shared with decode: ascending expert id, bf16 after each add)
//
// The shared expert is one more slot whose token list is all T tokens.
//
// GEMM kernel (k_gemm): persistent, one CTA per SM, 11 warps.
//   warp 0  producer: TMA loads of the weight tile (4-D map over the tiled
//           bank: 128 rows x 64 columns = 16 KB, already in the 128-byte
//           swizzled K-major operand layout) into a 4-stage ring.
//   warp 1  producer: TMA loads of the token tile (contiguous rows, 128-byte
//           swizzle) into a 4-stage ring, as the binary decomposition of the
//           tile's rows into boxes of 256, 128, 64, 32 and 16 rows (one copy
//           for a whole chunk: the number of copies per stage, not their
//           bytes, was the limit with 16-row boxes).
//   warp 2  MMA issuer: tcgen05.mma kind::f16 (bf16 x bf16 -> f32),
//           M = 128 weight rows, N = the unit's tokens rounded up to 16
//           (<= 256), K = 64 per stage as 4 instructions; accumulators in
//           TMEM, double-buffered (2 x 256 columns); tcgen05.commit frees
//           ring stages and hands finished accumulators to the epilogue.
//   warps 3-10 epilogue, two sets of four: tcgen05.ld of the accumulator
//           (warp w reads TMEM lanes 32*(w%4)..+31; the sets take alternate
//           32-column groups), bf16 rounding points of the reference, stores.
// Work unit = (slot, 256-token chunk, 128-row tile); units are numbered
// slot-major and dealt round-robin to the CTAs.
//
// Numerics: every product is exact and accumulated in f32 by the tensor
// core in its own order, so outputs differ from the reference's 32-partial
// schedule by f32 rounding before each bf16 rounding point (within the
// block tolerance, max-abs 2e-2 / rel-L2 1e-3).  Every logit that can be
// selected is recomputed exactly, so expert selection matches the
// reference's bit for bit.
//
// Every wait is bounded (2 s of globaltimer); on expiry the CTA records
// kErrTimeout, stops issuing, lets its copies and MMAs drain (bounded), frees
// its TMEM and exits.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include <cudaTypedefs.h>

#include "fw_common.cuh"
#include "fw_kernels.h"

namespace fw {
namespace {

// Ring depths and the token chunk are build-time settings (defaults below),
// so tile and pipeline sweeps can build variants without editing the code.
#ifndef FW_PF_RING_A
#define FW_PF_RING_A 4
#endif
#ifndef FW_PF_RING_B
#define FW_PF_RING_B 4
#endif
#ifndef FW_PF_BN
#define FW_PF_BN 256
#endif
constexpr int kBM = 128;        // weight rows per tile (MMA M)
constexpr int kBK = 64;         // columns per ring stage (one 128-byte swizzle atom)
constexpr int kBN = FW_PF_BN;   // tokens per work unit (MMA N, max)
constexpr int kRingA = FW_PF_RING_A;  // weight-tile ring stages
constexpr int kRingB = FW_PF_RING_B;  // token-tile ring stages
static_assert(kBN == 256, "token chunk of 256 (pairs need the upper half of the token slot)");
// The two rings advance together, one weight tile and one token tile per
// stage, so they share their barriers: a stage is full when both producers
// have posted it and both copies have landed, and one commit frees both.
static_assert(kRingA == kRingB, "the weight and token rings share their barriers");
constexpr int kRing = kRingA;
constexpr int kABytes = kBM * kBK * 2;   // 16 KB
constexpr int kBBytes = kBN * kBK * 2;   // 32 KB
constexpr int kPairTileOff = kBBytes / 2;  // second weight tile of a pair: upper half of the token slot
constexpr int kPairCols = 128;             // its accumulator: TMEM columns 128.. of the buffer
static_assert(kBBytes / 2 >= kABytes, "a pair's second weight tile fits beside a half-width token tile");
constexpr int kStageBytes = 32 * kBM * 2;  // epilogue staging per set: 32 tokens x 128 rows, bf16
constexpr int kEpiSets = 2;                // epilogue warp sets (4 warps each, alternate column groups)
constexpr int kEpiWarp0 = 3;               // warps 0, 1: producers; 2: MMA; 3..: epilogue
constexpr int kGemmThreads = 32 * kEpiWarp0 + kEpiSets * 128;
constexpr int kAccCols = 256;   // TMEM columns per accumulator buffer
constexpr uint64_t kWaitNs = 2000000000ull;

// ---- tcgen05 / TMA wrappers -------------------------------------------------

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory operand descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (sm_100 descriptor version 1).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3fffu) | (1ull << 16) | (static_cast<uint64_t>(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

// Instruction descriptor: kind::f16, bf16 A and B (K-major), f32 D, M x N.
__device__ __forceinline__ uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 32 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Named barrier 1 + set over one epilogue set's four warps (128 threads).
__device__ __forceinline__ void epi_sync(int set) { asm volatile("bar.sync %0, 128;" ::"r"(1 + set) : "memory"); }
// Same barrier with an OR over the set's 128 threads: keeps a set's
// decisions uniform, so none of its warps can leave while the others wait
// at epi_sync.
__device__ __forceinline__ bool epi_any(int set, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, %2, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(1 + set)
      : "memory");
  return r != 0;
}


// ---- packed bf16 epilogue arithmetic --------------------------------------------
// bf16 bits with NaN as 0x7fc0 (the canonical pattern of f32_to_bf16).
__device__ __forceinline__ uint32_t nanfix_bf16x2(uint32_t r) {
  uint32_t lo = r & 0xffffu, hi = r >> 16;
  lo = (lo & 0x7fffu) > 0x7f80u ? 0x7fc0u : lo;
  hi = (hi & 0x7fffu) > 0x7f80u ? 0x7fc0u : hi;
  return lo | (hi << 16);
}
// {bf16(lo), bf16(hi)} round to nearest even, one instruction for the pair.
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return nanfix_bf16x2(r);
}
// a * b per bf16 half, one rounding (a bf16 x bf16 product is exact in f32
// outside the f32 subnormal range, so this equals f32_to_bf16 of the f32
// product there).
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return nanfix_bf16x2(r);
}

// ---- work units ---------------------------------------------------------------

struct GemmArgs {
  int phase;               // 0: gate/up + SwiGLU; 1: down + scale
  int E, T, K, H, I, Is;
  int kb_r, kb_s;          // 64-column stages per unit (routed, shared)
  int mt_r, mt_s;          // 128-row tiles per chunk (routed, shared)
  int groups_r;            // 8-row groups per routed expert matrix
  // K-blocked token operands ([K/64][rows][64]): rows per 64-column block of
  // the routed operand (xg / act: pair capacity) and of the shared one
  // (act_sh: token capacity); b_blocked_s = 0 when the shared up operand is
  // the row-major input x.
  int rows_r, rows_s, b_blocked_s;
  // Expert parallelism: destination row of pair t*K+k's weighted output in
  // the packed send buffer (null: row t*K+k of `weighted`).
  const int32_t* send_pos;
  const int* offset;       // [E+1] grouped pair offsets
  // [2][E+2] unit prefixes of this phase (slot E = shared): compute-heavy
  // slots (more than kPairMax tokens), then weight-streaming ones; the two
  // classes are interleaved in the unit order (decode_unit)
  const int* prefix;
  const int32_t* pair_tk;  // [pairs] t*K + k
  const uint16_t* score;   // [T*K] route weights (bf16)
  const uint16_t* sh_sig;  // [T] shared gate (bf16)
  const uint16_t* silu;    // [65536] bf16(silu(g)) table
  uint16_t* act;           // [pairs][I]
  uint16_t* act_sh;        // [T][Is]
  uint16_t* weighted;      // [T*K][H]
  uint16_t* gated_sh;      // [T][H]
  int* err;
  // Expert parallelism over peer memory (ep.world > 0): nothing is computed
  // when this rank's forward already failed; the down phase stores routed
  // rows in their owner's window (ep_recv_row) and its last CTA sets this
  // rank's done flag in every window.
  EpPeers ep;
};

// Token chunks of at most kPairMax tokens (every expert with few tokens,
// and the last chunk of a busy one) take their weight tiles two at a time:
// one unit streams the chunk's token tile once against two 128-row weight
// tiles (the second lands in the unused upper half of the stage's token
// slot) and accumulates into two TMEM column ranges, so each stage carries
// twice the tensor work for one token load and one commit.
constexpr int kPairMax = kBN / 2;

// Work units of one phase for a slot of `count` token rows and `mt` 128-row
// tiles: full chunks take one unit per tile, a last chunk of at most
// kPairMax tokens one per pair of tiles.
__host__ __device__ inline int slot_units(int count, int mt) {
  if (count <= 0) return 0;
  const int chunks = (count + kBN - 1) / kBN;
  const int last = count - (chunks - 1) * kBN;
  return (chunks - 1) * mt + (last <= kPairMax ? (mt + 1) / 2 : mt);
}

struct Unit {
  int slot, m, n0, nvalid, bn, kblocks;
  int np;  // weight tiles of the unit: m and, when 2, m + 1
  bool routed;
};

// Unit u of this phase; s_prefix ([2][E+2]) / s_offset are the
// shared-memory copies.  The units of compute-heavy slots (more than
// kPairMax tokens: full 256-token chunks, tensor-bound) and of
// weight-streaming slots (HBM-bound) are interleaved in proportion to their
// counts, so that at any time some SMs stream weights while others compute:
// with a skewed router the busy experts have the low ids, and slot order
// alone would run all the tensor-bound units first and all the HBM-bound
// ones after them.  Unit u is compute-heavy unit floor(u * Uh / U) when that
// value steps at u, else weight-streaming unit u - floor(u * Uh / U).
__device__ __forceinline__ Unit decode_unit(const GemmArgs& a, const int* s_prefix, const int* s_offset, int u) {
  const int* ph = s_prefix;
  const int* pt = s_prefix + a.E + 2;
  const long long uh = ph[a.E + 1], ut = pt[a.E + 1];
  const int hk = static_cast<int>(static_cast<long long>(u) * uh / (uh + ut));
  const int hk1 = static_cast<int>(static_cast<long long>(u + 1) * uh / (uh + ut));
  const bool heavy = hk1 > hk;
  const int idx = heavy ? hk : u - hk;
  const int* pre = heavy ? ph : pt;
  int lo = 0, hi = a.E;  // largest slot s with pre[s] <= idx (it has units of this class)
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (pre[mid] <= idx) lo = mid;
    else hi = mid - 1;
  }
  Unit w;
  w.slot = lo;
  w.routed = lo < a.E;
  const int mt = w.routed ? a.mt_r : a.mt_s;
  const int local = idx - pre[lo];
  const int count = w.routed ? s_offset[lo + 1] - s_offset[lo] : a.T;
  const int chunks = (count + kBN - 1) / kBN;
  const int full = (chunks - 1) * mt;  // units of the chunks before the last
  int chunk;
  if (local < full) {
    chunk = local / mt;
    w.m = local - chunk * mt;
    w.np = 1;
  } else {
    chunk = chunks - 1;
    const int i = local - full;
    if (count - chunk * kBN <= kPairMax) {
      w.m = 2 * i;
      w.np = min(2, mt - w.m);
    } else {
      w.m = i;
      w.np = 1;
    }
  }
  w.n0 = (w.routed ? s_offset[lo] : 0) + chunk * kBN;
  w.nvalid = min(kBN, count - chunk * kBN);
  w.bn = (w.nvalid + 15) & ~15;
  w.kblocks = w.routed ? a.kb_r : a.kb_s;
  return w;
}

struct __align__(8) GemmSmemTail {
  uint64_t full[kRing];   // both producers arrive (with their bytes)
  uint64_t empty[kRing];  // one tcgen05.commit frees the weight and the token slot
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void raise_abort(GemmSmemTail* t, int* err) {
  set_error(err, kErrTimeout);
  *reinterpret_cast<volatile int*>(&t->abort) = 1;
}
__device__ __forceinline__ bool aborted(GemmSmemTail* t) { return *reinterpret_cast<volatile int*>(&t->abort) != 0; }

// One producer warp feeding a ring of `depth` stages: per stage, lane 0
// waits for the slot (bounded) and posts the byte count, then `issue`
// (called by the whole warp) starts the copies.  Returns the number of
// stages issued; on exit the copies still in flight have landed (bounded).
template <typename Issue, typename Bytes>
__device__ __forceinline__ void produce(const GemmArgs& a, const int* s_prefix, const int* s_offset, int total,
                                        GemmSmemTail* tail, uint64_t* full, uint64_t* empty, int depth, int lane,
                                        Bytes bytes_of, Issue issue) {
  int it = 0;
  bool ok = true;
  for (int u = blockIdx.x; ok && u < total; u += gridDim.x) {
    if (__any_sync(0xffffffffu, aborted(tail))) break;  // warp-uniform
    const Unit w = decode_unit(a, s_prefix, s_offset, u);
    const uint32_t bytes = bytes_of(w, u);
    for (int kb = 0; kb < w.kblocks; ++kb, ++it) {
      const int st = it % depth;
      const uint32_t ph = (it / depth) & 1;
      bool got = true;
      if (lane == 0) {
        got = mbar_wait_bounded(&empty[st], ph ^ 1u, kWaitNs);
        if (got) mbar_arrive_expect_tx(&full[st], bytes);
        else raise_abort(tail, a.err);
      }
      got = __shfl_sync(0xffffffffu, got, 0) != 0;  // lane 0 waited; the warp follows it
      if (!got) {
        ok = false;
        break;
      }
      issue(w, kb, st, &full[st]);
    }
  }
  // Let the copies already issued land before the CTA can exit.
  if (lane == 0) {
    const int first = it > depth ? it - depth : 0;
    for (int j = first; j < it; ++j)
      if (!mbar_wait_bounded(&full[j % depth], (j / depth) & 1, kWaitNs)) raise_abort(tail, a.err);
  }
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm(const __grid_constant__ CUtensorMap map_a_r, const __grid_constant__ CUtensorMap map_a_s,
           const __grid_constant__ TokenMaps map_b_r, const __grid_constant__ TokenMaps map_b_s, GemmArgs a) {
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment for the swizzled operand tiles.
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  unsigned char* ring_a = smem;                         // [kRingA][16 KB]
  unsigned char* ring_b = smem + kRingA * kABytes;      // [kRingB][32 KB]
  uint16_t* s_stage = reinterpret_cast<uint16_t*>(ring_b + kRingB * kBBytes);  // [sets][32][128] epilogue staging
  GemmSmemTail* tail = reinterpret_cast<GemmSmemTail*>(ring_b + kRingB * kBBytes + kEpiSets * kStageBytes);
  int* s_prefix = reinterpret_cast<int*>(tail + 1);     // [2][E+2]
  int* s_offset = s_prefix + 2 * (a.E + 2);             // [E+1]
  // [kBN] epilogue: destination row per column (8-byte aligned)
  uint16_t** s_col_dst = reinterpret_cast<uint16_t**>((reinterpret_cast<uintptr_t>(s_offset + a.E + 1) + 7) & ~uintptr_t(7));
  float* s_col_scale = reinterpret_cast<float*>(s_col_dst + kBN);  // [kBN] epilogue: scale per column
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&tail->full[i], 2);
      mbar_init(&tail->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tail->acc_full[i], 1);
      mbar_init(&tail->acc_empty[i], 4 * kEpiSets);
    }
    mbar_init(&tail->mma_done, 1);
    tail->abort = 0;
    fence_mbar_init();
  }
  pdl_wait();
  pdl_launch_dependents();
  if (warp == 0) {
    // 512 TMEM columns: two 256-column accumulators (one CTA per SM).
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tail->tmem_base)),
                 "r"(2 * kAccCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  for (int i = threadIdx.x; i < 2 * (a.E + 2); i += blockDim.x) s_prefix[i] = a.prefix[i];
  for (int i = threadIdx.x; i < a.E + 1; i += blockDim.x) s_offset[i] = a.offset[i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tail->tmem_base;
  const int total =
      (a.ep.world > 0 && ld_volatile_int(a.err) != 0) ? 0 : s_prefix[a.E + 1] + s_prefix[2 * (a.E + 2) - 1];

  if (warp == 0) {
    // ---------------- weight-tile producer ----------------
    const uint64_t policy = l2_evict_first_policy();
    produce(
        a, s_prefix, s_offset, total, tail, tail->full, tail->empty, kRing, lane,
        [&](const Unit& w, int) { return static_cast<uint32_t>(w.np * kABytes); },
        [&](const Unit& w, int kb, int st, uint64_t* bar) {
          const int grp0 = (w.routed ? w.slot * a.groups_r : 0) + w.m * (kBM / 8);
          const CUtensorMap* ma = w.routed ? &map_a_r : &map_a_s;
          if (lane == 0) {
            tma_load_4d(ring_a + st * kABytes, ma, 0, 0, kb, grp0, bar, policy);
            // second tile of a pair: the upper half of the stage's token slot
            if (w.np == 2) tma_load_4d(ring_b + st * kBBytes + kPairTileOff, ma, 0, 0, kb, grp0 + kBM / 8, bar, policy);
          }
        });
  } else if (warp == 1) {
    // ---------------- token-tile producer ----------------
    produce(
        a, s_prefix, s_offset, total, tail, tail->full, tail->empty, kRing, lane,
        [&](const Unit& w, int) { return static_cast<uint32_t>(w.bn * kBK * 2); },
        [&](const Unit& w, int kb, int st, uint64_t* bar) {
          unsigned char* sb = ring_b + st * kBBytes;
          const TokenMaps* mb = w.routed ? &map_b_r : &map_b_s;
          // K-blocked operands: block kb's rows n0.. are one contiguous run.
          const bool blocked = w.routed || a.b_blocked_s;
          const int c0 = blocked ? 0 : kb * kBK;
          const int r0 = (blocked ? kb * (w.routed ? a.rows_r : a.rows_s) : 0) + w.n0;
          // bn (a multiple of 16, <= 256) as boxes of 256, 128, ..., 16 rows
          if (lane == 0) {
            int j = 0;
#pragma unroll
            for (int b = kTokenBoxes - 1; b >= 0; --b)
              if (w.bn & (16 << b)) {
                tma_load_2d(sb + j * 128, &mb->box[b], c0, r0 + j, bar);
                j += 16 << b;
              }
          }
        });
  } else if (warp == 2) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int ia = 0, ai = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < total; u += gridDim.x, ++ai) {
        if (aborted(tail)) break;
        const Unit w = decode_unit(a, s_prefix, s_offset, u);
        const int buf = ai & 1;
        const uint32_t aph = (ai >> 1) & 1;
        if (!mbar_wait_bounded(&tail->acc_empty[buf], aph ^ 1u, kWaitNs)) {
          raise_abort(tail, a.err);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * kAccCols;
        const uint32_t idesc = idesc_bf16(kBM, w.bn);
        const bool pair = w.np == 2;
        for (int kb = 0; kb < w.kblocks; ++kb, ++ia) {
          const int sa_i = ia % kRing, sb_i = sa_i;
          if (!mbar_wait_bounded(&tail->full[sa_i], (ia / kRing) & 1, kWaitNs)) {
            raise_abort(tail, a.err);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(ring_a + sa_i * kABytes);
          const uint32_t sb = smem_u32(ring_b + sb_i * kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            umma_bf16(d, sw128_desc(sa + k * 32), sw128_desc(sb + k * 32), idesc, (kb | k) != 0 ? 1u : 0u);
            if (pair)
              umma_bf16(d + kPairCols, sw128_desc(sb + kPairTileOff + k * 32), sw128_desc(sb + k * 32), idesc,
                        (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&tail->empty[sa_i]);
        }
        if (ok) umma_commit(&tail->acc_full[buf]);
      }
      // Every MMA this thread issued has completed once mma_done flips.
      umma_commit(&tail->mma_done);
      if (!mbar_wait_bounded(&tail->mma_done, 0, kWaitNs)) raise_abort(tail, a.err);
    }
  } else {
    // ---------------- epilogue (warps 3..10) ----------------
    // Two sets of four warps (one warp per TMEM lane quarter in each set);
    // set s handles the 32-column groups s, s+2, ...  Per group: tcgen05.ld,
    // the reference's rounding points, the bf16 results into the set's
    // shared staging tile, then 16-byte stores of whole output rows by the
    // set's 128 threads.
    const int ew = warp - kEpiWarp0;
    const int set = ew >> 2;
    const int q = warp & 3;             // TMEM lane quarter this warp may read
    const int row = q * 32 + lane;      // accumulator row (weight row within the tile)
    const int et = (ew & 3) * 32 + lane;  // 0..127 within the set
    uint16_t* stage = s_stage + set * (kStageBytes / 2);
    int ai = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++ai) {
      // Decisions stay uniform over the set's 128 threads (tcgen05.ld is
      // warp-collective; epi_sync waits for all four warps of the set).
      if (epi_any(set, aborted(tail))) break;
      const Unit w = decode_unit(a, s_prefix, s_offset, u);
      const int buf = ai & 1;
      const uint32_t aph = (ai >> 1) & 1;
      if (a.phase == 1) {
        // Column tables (this set's groups): destination row and f32 scale.
        for (int j = et; j < w.nvalid; j += 128) {
          if (((j >> 5) & 1) != set) continue;
          if (w.routed) {
            const int tk = a.pair_tk[w.n0 + j];
            s_col_dst[j] = a.ep.world > 0 ? ep_recv_row(a.ep, tk)
                                          : a.weighted + static_cast<size_t>(a.send_pos != nullptr ? a.send_pos[tk] : tk) * a.H;
            s_col_scale[j] = bf16_to_f32(a.score[tk]);
          } else {
            s_col_dst[j] = a.gated_sh + static_cast<size_t>(w.n0 + j) * a.H;
            s_col_scale[j] = bf16_to_f32(a.sh_sig[w.n0 + j]);
          }
        }
      }
      const bool got = mbar_wait_bounded(&tail->acc_full[buf], aph, kWaitNs);
      if (epi_any(set, !got)) {  // also orders the table writes above before their use
        if (et == 0) raise_abort(tail, a.err);
        break;
      }
      tc_fence_after();
      const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * kAccCols;
      // A pair's second tile sits kPairCols columns further in the buffer.
      for (int jt = 0; jt < w.np; ++jt) {
      const int mo = w.m + jt;  // the 128-row tile these columns belong to
      for (int c0 = 32 * set; c0 < w.bn; c0 += 32 * kEpiSets) {
        uint32_t v[32];
        tmem_ld32(tbase + jt * kPairCols + c0, v);
        if (a.phase == 0) {
          // Rows alternate 4 gate / 4 up per 8-row group; lanes with
          // (row & 7) < 4 own a gate row and take the matching up value
          // from lane + 4.  swiglu_bf16 (src/expert.rs:562-571) on the bf16
          // outputs of linear_bf16: bf16(bf16(silu(g)) * u).
          uint32_t gb[16], ub[16];  // bf16 pairs: columns j, j+1
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float g0 = __uint_as_float(v[j]), g1 = __uint_as_float(v[j + 1]);
            const float u0 = __shfl_down_sync(0xffffffffu, g0, 4), u1 = __shfl_down_sync(0xffffffffu, g1, 4);
            gb[j / 2] = cvt_bf16x2(g0, g1);
            ub[j / 2] = cvt_bf16x2(u0, u1);
          }
          if ((lane & 7) < 4) {
            const int il = 16 * q + 4 * (lane >> 3) + (lane & 3);  // intermediate within the tile
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const uint32_t s2 = static_cast<uint32_t>(a.silu[gb[j / 2] & 0xffffu]) |
                                  (static_cast<uint32_t>(a.silu[gb[j / 2] >> 16]) << 16);
              const uint32_t p2 = mul_bf16x2(s2, ub[j / 2]);
              stage[j * 64 + il] = static_cast<uint16_t>(p2 & 0xffffu);
              stage[(j + 1) * 64 + il] = static_cast<uint16_t>(p2 >> 16);
            }
          }
        } else {
          // routed: bf16(bf16(down) * route weight) (src/expert.rs:748-751);
          // shared: bf16(sigmoid * bf16(down)) (src/expert.rs:1144-1147)
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const uint32_t d2 = cvt_bf16x2(__uint_as_float(v[j]), __uint_as_float(v[j + 1]));
            const uint32_t s2 = __float_as_uint(s_col_scale[c0 + j]) >> 16 |
                                (__float_as_uint(s_col_scale[c0 + j + 1]) & 0xffff0000u);
            const uint32_t p2 = mul_bf16x2(d2, s2);
            stage[j * 128 + row] = static_cast<uint16_t>(p2 & 0xffffu);
            stage[(j + 1) * 128 + row] = static_cast<uint16_t>(p2 >> 16);
          }
        }
        epi_sync(set);
        const int rows_here = min(32, w.nvalid - c0);
        if (a.phase == 0) {
          // [32 tokens][64 intermediates] = rows of K-block m of act
          // ([I/64][rows][64]): 8 chunks of 16 bytes per token.
          uint16_t* dst = (w.routed ? a.act : a.act_sh) +
                          static_cast<size_t>(mo) * (w.routed ? a.rows_r : a.rows_s) * 64;
          for (int ch = et; ch < rows_here * 8; ch += 128) {
            const int r = ch >> 3, c = ch & 7;
            *reinterpret_cast<uint4*>(dst + static_cast<size_t>(w.n0 + c0 + r) * 64 + c * 8) =
                *reinterpret_cast<const uint4*>(stage + r * 64 + c * 8);
          }
        } else {
          // [32 tokens][128 output rows]: 16 chunks of 16 bytes per token
          // (under expert parallelism, routed rows go over NVLink).
          for (int ch = et; ch < rows_here * 16; ch += 128) {
            const int r = ch >> 4, c = ch & 15;
            *reinterpret_cast<uint4*>(s_col_dst[c0 + r] + mo * kBM + c * 8) =
                *reinterpret_cast<const uint4*>(stage + r * 128 + c * 8);
          }
        }
        epi_sync(set);
      }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tail->acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kAccCols) : "memory");
  if (a.phase == 1 && a.ep.world > 0) ep_signal(a.ep, kEpFlagDone, a.ep.ticket + 1, a.err);
}

// ---- router for prefill widths ---------------------------------------------------
//
// Expert selection has to be the reference's, and only the logits near a
// token's top-k boundary decide it.  So the router runs in two kernels:
//   k_router_tc   every (token, expert) logit on the tensor cores, f32
//                 accumulation ([T][E] `approx`), 128 router rows x 256
//                 tokens per CTA;
//   k_router_fix  one warp per token: an interval holding the reference's
//                 biased bf16 logit of each expert, from approx -+ delta with
//                 delta = 2^-10 * |w_e|_2 * |x_t|_2.  Experts whose upper end
//                 reaches the k-th largest lower end are the only ones that
//                 can be selected; their logits are recomputed with the
//                 reference's dot schedule (src/expert.rs:514-552).  The other
//                 logits keep the rounded approximation, within one bf16 step
//                 of the reference's, and enter only the softmax denominator.
//                 The shared gate logit is always recomputed.
// The bound: the reference's dot (32 partials of H/32 products, then a
// 5-level tree) is within (H/32 + 5) * 2^-24 * S of the exact dot, where
// S = sum |w_i x_i| <= |w|_2 |x|_2 (Cauchy-Schwarz); the tensor core adds
// exact bf16 products into an f32 accumulator in H/16 steps, within
// (H/16) * 17 * 2^-24 * S even if each step truncated all 17 aligned terms
// to 24 bits.  At H = 4096 the two add up to 2^-11.8 * S, so 2^-10 leaves a
// factor of three.  Rounding to bf16 and adding the bias are monotone, so
// the interval's ends give the lowest and highest possible bf16 logit.  An
// expert whose highest possible logit is below the k-th largest lowest one
// is beaten strictly by k others: the top-k (with its tie rule, decided by
// k_route on the repaired logits) only ever compares exact logits.
constexpr int kRcN = 256;                     // tokens per CTA (MMA N)
constexpr int kRcStages = 4;
constexpr int kRcBBytes = kRcN * kBK * 2;     // 32 KB token tile
constexpr int kFixWarps = 4;                  // tokens per k_router_fix CTA
constexpr float kDotBound = 0x1p-10f;         // delta / (|w| |x|)
constexpr float kNormSlack = 1.00390625f;     // 1 + 2^-8: f32 sum of <= 2^15 squares, rounded up
constexpr float kNormFloor = 0x1p-60f;        // norms below this are raised to it
constexpr float kFiniteMax = 0x1p120f;        // larger |approx| or delta: no interval, recompute

struct __align__(8) RcTail {
  uint64_t full[kRcStages];
  uint64_t empty[kRcStages];
  uint64_t acc_full;
  uint32_t tmem_base;
};

size_t router_tc_smem() { return 1024 + static_cast<size_t>(kRcStages) * (kABytes + kRcBBytes) + sizeof(RcTail); }

struct RouterTcArgs {
  int E, T, H;
  int bn;          // token rows per tile: min(256, T rounded up to 16)
  float* approx;   // [T][E]
  int* err;
};

// Warp 0 lane 0 loads (TMA, 128-byte swizzle: router rows m0.. and token
// rows n0.., 64 columns per stage), warp 1 lane 0 issues the MMAs
// (M = 128 router rows, N = bn tokens, K = 16 per instruction) into one
// TMEM accumulator; then warp w stores TMEM lanes 32w.. (router rows) as
// f32 logits, 32 tokens per tcgen05.ld, each a coalesced 128-byte row run.
__global__ void __launch_bounds__(128, 1)
    k_router_tc(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                RouterTcArgs a) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  unsigned char* ring_a = smem;
  unsigned char* ring_b = smem + kRcStages * kABytes;
  RcTail* tail = reinterpret_cast<RcTail*>(ring_b + kRcStages * kRcBBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mtiles = (a.E + kBM - 1) / kBM;
  const int m0 = (blockIdx.x % mtiles) * kBM, n0 = (blockIdx.x / mtiles) * a.bn;
  const int nkb = a.H / kBK;
  const uint32_t stage_bytes = kABytes + a.bn * kBK * 2;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kRcStages; ++i) {
      mbar_init(&tail->full[i], 1);
      mbar_init(&tail->empty[i], 1);
    }
    mbar_init(&tail->acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tail->tmem_base)),
                 "r"(kRcN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tail->tmem_base;
  // The token rows may be the previous kernel's output.
  pdl_wait();
  pdl_launch_dependents();
  bool ok = true;
  if (warp == 0 && lane == 0) {
    int issued = 0;
    for (int kb = 0; kb < nkb; ++kb) {
      const int st = kb % kRcStages;
      if (!mbar_wait_bounded(&tail->empty[st], ((kb / kRcStages) & 1) ^ 1u, kWaitNs)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(&tail->full[st], stage_bytes);
      tma_load_2d(ring_a + st * kABytes, &map_w, kb * kBK, m0, &tail->full[st]);
      tma_load_2d(ring_b + st * kRcBBytes, &map_x, kb * kBK, n0, &tail->full[st]);
      ++issued;
    }
    // Copies in flight land before the CTA can exit.
    for (int j = issued > kRcStages ? issued - kRcStages : 0; j < issued; ++j)
      if (!mbar_wait_bounded(&tail->full[j % kRcStages], (j / kRcStages) & 1, kWaitNs)) ok = false;
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = idesc_bf16(kBM, a.bn);
    for (int kb = 0; kb < nkb; ++kb) {
      const int st = kb % kRcStages;
      if (!mbar_wait_bounded(&tail->full[st], (kb / kRcStages) & 1, kWaitNs)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sa = smem_u32(ring_a + st * kABytes), sb = smem_u32(ring_b + st * kRcBBytes);
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k)
        umma_bf16(tmem, sw128_desc(sa + k * 32), sw128_desc(sb + k * 32), idesc, (kb | k) != 0 ? 1u : 0u);
      umma_commit(&tail->empty[st]);
    }
    // Arrives once every MMA issued above has completed (after a failure too).
    umma_commit(&tail->acc_full);
  }
  if (!ok) set_error(a.err, kErrTimeout);
  __syncwarp();
  const bool got = mbar_wait_bounded(&tail->acc_full, 0, kWaitNs);
  if (!__all_sync(0xffffffffu, got)) {
    if (lane == 0) set_error(a.err, kErrTimeout);
  } else {
    tc_fence_after();
    const int e = m0 + 32 * warp + lane;
    for (int c0 = 0; c0 < a.bn && n0 + c0 < a.T; c0 += 32) {
      uint32_t v[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * warp) << 16) + c0, v);
      if (e < a.E) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int t = n0 + c0 + j;
          if (t < a.T) a.approx[static_cast<size_t>(t) * a.E + e] = __uint_as_float(v[j]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kRcN) : "memory");
}

struct RouterFixArgs {
  const uint16_t* wpm;        // [E+1][H] router rows and the shared gate vector, partial-major
  const float* bias;          // [E] or null
  const float* wnorm;         // [E] upper bounds of the router rows' 2-norms
  const float* approx;        // [T][E]
  const uint16_t* x;          // [T][H]
  uint16_t* logits;           // [T][E]
  uint16_t* extra_out;        // [T]
  int E, H, T, K;
};

// Lane blocks of a staged row are padded to an odd number of 16-byte
// chunks, so the 16-byte loads of eight consecutive lanes hit distinct banks.
__host__ __device__ inline int fix_stride(int H) {
  const int nch = H / 256;
  return nch + 1 + (nch & 1);
}
size_t router_fix_smem(int H, int E) {
  return static_cast<size_t>(kFixWarps) * (2 * 32 * 16 * static_cast<size_t>(fix_stride(H)) + 2 * E);
}

// bf16 logit with the build's optional f32 bias, re-rounded (as k_router).
__device__ __forceinline__ uint16_t biased_logit(float v, const float* bias, int e) {
  uint16_t b = f32_to_bf16(v);
  if (bias != nullptr) b = f32_to_bf16(bf16_to_f32(b) + bias[e]);
  return b;
}

// Upper bound of |v|_2 from an f32 sum of squares of at most 2^15 terms.
__device__ __forceinline__ float norm_bound(float sum_sq) {
  return fmaxf(__fsqrt_ru(__fmul_ru(sum_sq, kNormSlack)), kNormFloor);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_prev() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }


// One warp per token (see the section comment).  Lane j holds the token's
// columns j, j+32, ... (PX bf16 pairs at most: H <= 64 * PX) in registers,
// and the interval keys of experts j, j+32, ... (NS slots: E <= 32 * NS).
// Candidate rows come from the partial-major copy (lane j's columns
// contiguous), staged with cp.async, the next row in flight while the
// current dot runs.
template <int PX, int NS>
__global__ void __launch_bounds__(32 * kFixWarps) k_router_fix(RouterFixArgs a) {
  extern __shared__ __align__(16) unsigned char fix_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = a.H >> 8;  // 16-byte chunks (8 columns) per lane
  const int S = fix_stride(a.H);
  uint4* wbase = reinterpret_cast<uint4*>(fix_smem) + static_cast<size_t>(warp) * 2 * 32 * S;
  uint16_t* cand = reinterpret_cast<uint16_t*>(reinterpret_cast<uint4*>(fix_smem) + kFixWarps * 2 * 32 * S) +
                   static_cast<size_t>(warp) * a.E;
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x * kFixWarps + warp;
  if (t >= a.T) return;

  // Token columns j + 32i, paired (i, i+1), and an upper bound of |x|_2.
  const uint16_t* xr = a.x + static_cast<size_t>(t) * a.H + lane;
  const int pairs = a.H >> 6;
  uint32_t xv[PX];
  float ss = 0.0f;
#pragma unroll
  for (int p = 0; p < PX; ++p) {
    xv[p] = 0u;
    if (p < pairs) {
      const uint32_t lo = xr[64 * p], hi = xr[64 * p + 32];
      xv[p] = lo | (hi << 16);
      const float fl = bf16_to_f32(lo), fh = bf16_to_f32(hi);
      ss = __fmaf_rn(fl, fl, ss);
      ss = __fmaf_rn(fh, fh, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float xn = norm_bound(ss);

  // Interval keys (the total order of bf16 the route kernel ranks by) of
  // every expert; the rounded approximation is written for each bounded one.
  const float* ar = a.approx + static_cast<size_t>(t) * a.E;
  uint16_t* lr = a.logits + static_cast<size_t>(t) * a.E;
  const int ne = a.E >> 5;
  uint32_t lohi[NS];  // (lowest key << 16) | highest key
#pragma unroll
  for (int i = 0; i < NS; ++i) {
    lohi[i] = 0u;
    if (i < ne) {
      const int e = lane + 32 * i;
      const float av = ar[e];
      const float d = __fmul_ru(__fmul_ru(a.wnorm[e], xn), kDotBound);
      uint32_t lo = 0u, hi = 0xffffu;  // unbounded: always a candidate
      if (fabsf(av) <= kFiniteMax && d <= kFiniteMax) {
        lo = total_key(biased_logit(__fsub_rd(av, d), a.bias, e));
        hi = total_key(biased_logit(__fadd_ru(av, d), a.bias, e));
        lr[e] = biased_logit(av, a.bias, e);
      }
      lohi[i] = (lo << 16) | hi;
    }
  }
  // tau = the K-th largest lowest key (bitwise search over the 16-bit keys).
  uint32_t tau = 0u;
  for (int b = 15; b >= 0; --b) {
    const uint32_t c = (tau | (1u << b)) << 16;
    unsigned n = 0;
#pragma unroll
    for (int i = 0; i < NS; ++i) n += (i < ne && lohi[i] >= c) ? 1u : 0u;
    if (static_cast<int>(__reduce_add_sync(0xffffffffu, n)) >= a.K) tau |= 1u << b;
  }
  int nc = 0;
#pragma unroll
  for (int i = 0; i < NS; ++i) {
    const bool c = i < ne && (lohi[i] & 0xffffu) >= tau;
    const uint32_t m = __ballot_sync(0xffffffffu, c);
    if (c) cand[nc + __popc(m & ((1u << lane) - 1u))] = static_cast<uint16_t>(lane + 32 * i);
    nc += __popc(m);
  }
  __syncwarp();  // candidate list and the approximations above before the exact writes

  // Rows 0..nc-1: the candidates; row nc: the shared gate vector (row E).
  // Global chunk g of a row (lane block g / nch, chunk g % nch) goes to
  // padded position (g / nch) * S + g % nch.
  int blk0 = lane / nch, rem0 = lane - blk0 * nch;
  const int step_blk = 32 / nch, step_rem = 32 - step_blk * nch;
  auto fetch = [&](int j, uint4* buf) {
    const uint4* src = reinterpret_cast<const uint4*>(a.wpm + static_cast<size_t>(j < nc ? cand[j] : a.E) * a.H);
    int blk = blk0, rem = rem0;
    for (int g = lane; g < 32 * nch; g += 32) {
      cp_async16(buf + blk * S + rem, src + g);
      blk += step_blk;
      rem += step_rem;
      if (rem >= nch) {
        rem -= nch;
        ++blk;
      }
    }
    cp_async_commit();
  };
  fetch(0, wbase);
  for (int j = 0; j <= nc; ++j) {
    uint4* cur = wbase + (j & 1) * 32 * S;
    if (j < nc) fetch(j + 1, wbase + ((j + 1) & 1) * 32 * S);
    else cp_async_commit();  // an empty group keeps "all but the newest" meaning row j
    cp_async_wait_prev();
    __syncwarp();  // every lane's part of row j has landed
    // The reference dot: lane j sums its columns in order, then the tree
    // +16, +8, +4, (0+1)+(2+3) (src/expert.rs:514-552).
    const uint4* wl = cur + lane * S;
    float acc = 0.0f;
#pragma unroll
    for (int q = 0; q < PX / 4; ++q) {
      if (q < nch) {
        const uint4 w4 = wl[q];
        acc = fma_seq2(w4.x, xv[4 * q], acc);
        acc = fma_seq2(w4.y, xv[4 * q + 1], acc);
        acc = fma_seq2(w4.z, xv[4 * q + 2], acc);
        acc = fma_seq2(w4.w, xv[4 * q + 3], acc);
      }
    }
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 16));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 8));
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
    const float qs = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));  // lanes 0, 2: (0+1), (2+3)
    const float dot = __fadd_rn(qs, __shfl_down_sync(0xffffffffu, qs, 2));
    if (lane == 0) {
      if (j < nc) lr[cand[j]] = biased_logit(dot, a.bias, cand[j]);
      else a.extra_out[t] = f32_to_bf16(dot);
    }
    __syncwarp();  // row j read by every lane before its buffer is refilled
  }
}

// Per layer, for the prefill router: an upper bound of each router row's
// 2-norm (one warp per row), and the partial-major copy of the router rows
// plus the shared gate vector: element (row, j, i) = row[j + 32 i].
__global__ void k_router_tables(const uint16_t* w, const uint16_t* extra_row, int E, int H, float* norms,
                                uint16_t* pm) {
  const long long n = static_cast<long long>(E + 1) * H;
  const int per = H / 32;
  for (long long o = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; o < n;
       o += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(o / H), r = static_cast<int>(o - static_cast<long long>(row) * H);
    const int j = r / per, i = r - j * per;
    pm[o] = (row < E ? w + static_cast<size_t>(row) * H : extra_row)[j + 32 * i];
  }
  const int e = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (e >= E) return;
  const uint16_t* rw = w + static_cast<size_t>(e) * H;
  float ss = 0.0f;
  for (int c = lane; c < H; c += 32) {
    const float v = bf16_to_f32(rw[c]);
    ss = __fmaf_rn(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) norms[e] = norm_bound(ss);
}

// ---- grouping kernels -----------------------------------------------------------

struct OffsetsArgs {
  int E, T, mt_up_r, mt_up_s, mt_dn;
  int* count;    // [E], zeroed here for the next forward
  int* fill;     // [E], zeroed here
  int* offset;   // [E+1]
  int* prefix;   // [2 phases][2 classes][E+2], see GemmArgs::prefix
};

// One CTA of blockDim.x >= E threads (thread e = expert e): exclusive scans
// of the pair counts and, per phase, of the units of compute-heavy slots and
// of weight-streaming slots.
__global__ void k_pf_offsets(OffsetsArgs a) {
  constexpr int kScans = 5;  // pairs, up heavy, up streaming, down heavy, down streaming
  __shared__ int wsum[kScans][32];
  pdl_wait();
  pdl_launch_dependents();
  const int e = threadIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  const int c = e < a.E ? a.count[e] : 0;
  const bool heavy = c > kPairMax;
  const int up = slot_units(c, a.mt_up_r), dn = slot_units(c, a.mt_dn);
  int v[kScans] = {c, heavy ? up : 0, heavy ? 0 : up, heavy ? dn : 0, heavy ? 0 : dn};
  int incl[kScans];
#pragma unroll
  for (int i = 0; i < kScans; ++i) {
    int x = v[i];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    incl[i] = x;
    if (lane == 31) wsum[i][warp] = x;
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int i = 0; i < kScans; ++i) {
      int x = lane < nw ? wsum[i][lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      wsum[i][lane] = x;  // inclusive warp totals
    }
  }
  __syncthreads();
  const int P = a.E + 2;
  if (e < a.E) {
    a.offset[e] = incl[0] - v[0] + (warp > 0 ? wsum[0][warp - 1] : 0);
#pragma unroll
    for (int i = 1; i < kScans; ++i) a.prefix[(i - 1) * P + e] = incl[i] - v[i] + (warp > 0 ? wsum[i][warp - 1] : 0);
    a.count[e] = 0;
    a.fill[e] = 0;
  }
  if (e == 0) {
    // slot E: the shared expert over T tokens
    const bool sh_heavy = a.T > kPairMax;
    const int sh[4] = {sh_heavy ? slot_units(a.T, a.mt_up_s) : 0, sh_heavy ? 0 : slot_units(a.T, a.mt_up_s),
                       sh_heavy ? slot_units(a.T, a.mt_dn) : 0, sh_heavy ? 0 : slot_units(a.T, a.mt_dn)};
    a.offset[a.E] = wsum[0][nw - 1];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tot = wsum[i + 1][nw - 1];
      a.prefix[i * P + a.E] = tot;
      a.prefix[i * P + a.E + 1] = tot + sh[i];
    }
  }
}

// Pairs grouped by expert: every (token, top-k position) whose expert e has
// e % world == rank (this GPU's experts under expert parallelism; all of
// them otherwise) gets a slot in its expert's group (bank e / world), and the
// token's input row is copied to that slot of the grouped input, so the
// gate/up GEMM reads each expert's token rows of a 64-column block as one
// contiguous run.  One warp per token: lane k takes top-k position k, and
// the row is read once and stored to each of the token's slots.  A CTA
// counts its pairs per expert in shared memory and reserves each expert's
// range with one global atomic (under a skewed router thousands of pairs
// select one expert).
constexpr int kScatterTokens = 8;
size_t scatter_smem(int banks) { return sizeof(int) * static_cast<size_t>(banks); }

__global__ void __launch_bounds__(kScatterTokens * 32) k_pf_scatter(const int32_t* idx, int TK, int K, int E, int H,
                                                                    int rank, int world, const int* offset, int* fill,
                                                                    int32_t* pair_tk, const uint16_t* x, uint16_t* xg,
                                                                    long long xg_rows, int* err) {
  extern __shared__ int s_cnt[];  // [E / world]: this CTA's pairs per bank, then their base in the group
  const int nb = E / world;
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kScatterTokens + warp;
  const bool live = t < TK / K;
  for (int i = threadIdx.x; i < nb; i += blockDim.x) s_cnt[i] = 0;
  __syncthreads();
  int bank = -1, lr = 0;
  if (live && lane < K) {
    const int e = idx[t * K + lane];
    if (e < 0 || e >= E) {
      set_error(err, kErrBadIndex);
    } else if (e % world == rank) {
      bank = e / world;
      lr = atomicAdd(&s_cnt[bank], 1);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nb; i += blockDim.x) {
    const int c = s_cnt[i];
    if (c > 0) s_cnt[i] = atomicAdd(&fill[i], c);
  }
  __syncthreads();
  int slot = -1;
  if (bank >= 0) {
    slot = offset[bank] + s_cnt[bank] + lr;
    pair_tk[slot] = t * K + lane;
  }
  const unsigned have = __ballot_sync(0xffffffffu, slot >= 0);
  if (!live || have == 0) return;
  // xg is K-blocked, [H/64][xg_rows][64]: 16-byte chunk c of the row goes
  // to block c / 8, row slot, chunk c % 8.  Eight chunks in flight per lane.
  const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H);
  const int nch = H / 8;
  for (int c0 = lane; c0 < nch; c0 += 8 * 32) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (c0 + 32 * u < nch) v[u] = src[c0 + 32 * u];
    unsigned rest = have;
    while (rest != 0) {
      const int k = __ffs(rest) - 1;
      rest &= rest - 1;
      const long long row = __shfl_sync(0xffffffffu, slot, k);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + 32 * u;
        if (c < nch)
          *reinterpret_cast<uint4*>(xg + ((static_cast<long long>(c >> 3) * xg_rows + row) * 64 + (c & 7) * 8)) = v[u];
      }
    }
  }
}

// Expert parallelism: per-expert pair counts of this GPU's experts over
// every rank's gathered selections.
__global__ void k_ep_count(const int32_t* idx, int n, int rank, int world, int ecount, int* count) {
  pdl_wait();
  pdl_launch_dependents();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int e = idx[i];
    if (e >= 0 && e % world == rank && e / world < ecount) atomicAdd(&count[e / world], 1);
  }
}

// Expert parallelism: packed positions of weighted rows.  Entry i of idx
// (a top-k id) belongs to group g with flag f:
//   send mode: g = i / group_len (the token owner), f = (idx % world == me);
//   recv mode: g = idx % world (the GPU that computed the row), f = 1.
// pos[i] = offset[g] + (flagged entries of group g before i), else -1;
// count[g], offset[g] (exclusive over g).  Entries in index order keep each
// group's rows in (token, k) order on both sides.  One CTA of 1024 threads.
__global__ void __launch_bounds__(1024) k_ep_positions(const int32_t* idx, int n, int group_len, int me, int world,
                                                        int recv_mode, int32_t* pos, int* count,
                                                        int* offset) {
  __shared__ int part[kEpMaxWorld][1025];
  __shared__ int tot[kEpMaxWorld], off[kEpMaxWorld];
  pdl_wait();
  pdl_launch_dependents();
  const int tid = threadIdx.x, nt = blockDim.x;
  const int per = (n + nt - 1) / nt, i0 = tid * per, i1 = min(n, i0 + per);
  auto key = [&](int i) {
    const int owner = idx[i] % world;
    if (recv_mode) return owner;
    return owner == me ? i / group_len : -1;
  };
  int c[kEpMaxWorld];
#pragma unroll
  for (int g = 0; g < kEpMaxWorld; ++g) c[g] = 0;
  for (int i = i0; i < i1; ++i) {
    const int k = key(i);
#pragma unroll
    for (int g = 0; g < kEpMaxWorld; ++g) c[g] += (k == g) ? 1 : 0;
  }
  for (int g = 0; g < world; ++g) part[g][tid] = c[g];
  __syncthreads();
  // exclusive scan over threads, one group per warp (world <= 8 <= warps)
  const int warp = tid >> 5, lane = tid & 31;
  if (warp < world) {
    int run = 0;
    for (int b = 0; b < nt; b += 32) {
      const int v = b + lane < nt ? part[warp][b + lane] : 0;
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (b + lane < nt) part[warp][b + lane] = run + x - v;
      run += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0) tot[warp] = run;
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int g = 0; g < world; ++g) {
      off[g] = acc;
      count[g] = tot[g];
      offset[g] = acc;
      acc += tot[g];
    }
  }
  __syncthreads();
  int cur[kEpMaxWorld];
#pragma unroll
  for (int g = 0; g < kEpMaxWorld; ++g) cur[g] = g < world ? off[g] + part[g][tid] : 0;
  for (int i = i0; i < i1; ++i) {
    const int k = key(i);
    int p = -1;
#pragma unroll
    for (int g = 0; g < kEpMaxWorld; ++g)
      if (k == g) p = cur[g]++;
    pos[i] = p;
  }
}

template <typename Kern, typename... Args>
cudaError_t launch_pdl_ex(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
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
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

size_t gemm_smem_bytes(int E) {
  return 1024 + static_cast<size_t>(kRingA) * kABytes + static_cast<size_t>(kRingB) * kBBytes +
         kEpiSets * kStageBytes + sizeof(GemmSmemTail) + sizeof(int) * (3 * static_cast<size_t>(E) + 5) + 8 +
         (sizeof(uint16_t*) + sizeof(float)) * kBN;
}

// ---- tensor maps (host) --------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Tiled bank of `mats` matrices of `rows` x K: 4-D view (64 columns, 8 rows,
// K/64 segments, 8-row groups), box = one 128-row x 64-column operand tile.
bool weight_map(CUtensorMap* m, const uint16_t* base, int K, long long rows_total) {
  const auto fn = encode_fn();
  if (fn == nullptr || base == nullptr) return false;
  const cuuint64_t dims[4] = {64, 8, static_cast<cuuint64_t>(K / 64), static_cast<cuuint64_t>(rows_total / 8)};
  const cuuint64_t strides[3] = {128, 1024, static_cast<cuuint64_t>(K) * 16};
  const cuuint32_t box[4] = {64, 8, 1, kBM / 8};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<uint16_t*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Row-major [rows][cols] bf16 matrix, boxes of 64 columns x box_rows rows,
// 128-byte swizzle (the K-major operand layout of the token tiles).
bool rows_map(CUtensorMap* m, const uint16_t* base, int cols, long long rows, int box_rows) {
  const auto fn = encode_fn();
  if (fn == nullptr || base == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The five token-tile boxes of a row-major [rows][cols] operand.
bool token_maps(TokenMaps* m, const uint16_t* base, int cols, long long rows) {
  for (int b = 0; b < kTokenBoxes; ++b)
    if (!rows_map(&m->box[b], base, cols, rows, 16 << b)) return false;
  return true;
}

// SMs of the current device (148 on B200), read once per device.
int sm_count() {
  DeviceAttrs a;
  return current_device_attrs(&a) == cudaSuccess ? a.sms : 148;
}

}  // namespace

bool prefill_supported(const Shape& s) {
  return s.H % 256 == 0 && (2 * s.I) % kBM == 0 && (2 * s.Is) % kBM == 0 && s.E <= 1024;
}

bool make_prefill_weight_maps(const Shape& s, const LayerWeights& w, PrefillWeightMaps* out) {
  if (!w.tiled || !prefill_supported(s)) return false;
  const long long E = w.expert_count;
  return weight_map(&out->gate_up, w.gate_up, s.H, E * 2 * s.I) && weight_map(&out->down, w.down, s.I, E * s.H) &&
         weight_map(&out->sh_gate_up, w.sh_gate, s.H, 2LL * s.Is) && weight_map(&out->sh_down, w.sh_down, s.Is, s.H) &&
         rows_map(&out->router, w.router, s.H, s.E, kBM);
}

bool make_prefill_scratch_maps(const Shape& s, const Scratch& sc, PrefillScratchMaps* out) {
  if (!prefill_supported(s)) return false;
  // K-blocked [K/64][rows][64] operands as 64-column row-major views.
  const long long P = sc.pair_cap, M = sc.max_T;
  return token_maps(&out->xg, sc.xg, 64, (s.H / 64) * P) && token_maps(&out->act, sc.act, 64, (s.I / 64) * P) &&
         token_maps(&out->act_sh, sc.act_sh, 64, (s.Is / 64) * M);
}

cudaError_t launch_router_tables(const uint16_t* w, const uint16_t* extra_row, int E, int H, float* norms,
                                 uint16_t* pm, cudaStream_t st) {
  if (H % 256 != 0) return cudaErrorInvalidValue;
  const long long n = static_cast<long long>(E + 1) * H;
  const int blocks = static_cast<int>(std::max<long long>((E + 7) / 8, std::min<long long>((n + 255) / 256, 4096)));
  k_router_tables<<<blocks, 256, 0, st>>>(w, extra_row, E, H, norms, pm);
  return cudaGetLastError();
}

template <int PX>
cudaError_t launch_router_fix_px(const RouterFixArgs& fa, cudaStream_t st) {
  const dim3 grid((fa.T + kFixWarps - 1) / kFixWarps), block(32 * kFixWarps);
  const size_t smem = router_fix_smem(fa.H, fa.E);
  return fa.E <= 512 ? launch_pdl_ex(k_router_fix<PX, 16>, grid, block, smem, st, fa)
                     : launch_pdl_ex(k_router_fix<PX, 32>, grid, block, smem, st, fa);
}

cudaError_t launch_router_fix(const RouterFixArgs& fa, cudaStream_t st) {
  const int pairs = fa.H / 64;
  if (pairs <= 16) return launch_router_fix_px<16>(fa, st);
  if (pairs <= 32) return launch_router_fix_px<32>(fa, st);
  if (pairs <= 48) return launch_router_fix_px<48>(fa, st);
  return launch_router_fix_px<64>(fa, st);
}

cudaError_t launch_prefill_front(const Shape& s, const LayerWeights& w, const PrefillWeightMaps& wm,
                                 const Luts& luts, const Scratch& sc, const uint16_t* x, int T, int32_t* topk_idx,
                                 uint16_t* topk_score, bool count_pairs, cudaStream_t st, cudaEvent_t mid) {
  if (w.router_norm == nullptr || w.router_pm == nullptr || sc.router_approx == nullptr) return cudaErrorInvalidValue;
  cudaError_t e;
  if (count_pairs && (e = cudaMemsetAsync(sc.pair_count, 0, sizeof(int) * s.E, st)) != cudaSuccess) return e;
  // Tensor-core logits, then the exact repair of the ones that can be selected.
  const int bn = T < kRcN ? (T + 15) & ~15 : kRcN;
  CUtensorMap x_rows;
  if (!rows_map(&x_rows, x, s.H, T, bn)) return cudaErrorInvalidValue;
  const RouterTcArgs ta{s.E, T, s.H, bn, sc.router_approx, sc.err};
  const int mtiles = (s.E + kBM - 1) / kBM;
  if ((e = launch_pdl_ex(k_router_tc, dim3(mtiles * ((T + bn - 1) / bn)), dim3(128), router_tc_smem(), st, wm.router,
                         x_rows, ta)) != cudaSuccess)
    return e;
  const RouterFixArgs fa{w.router_pm, w.bias, w.router_norm, sc.router_approx, x, sc.logits, sc.sh_logit,
                         s.E, s.H, T, s.K};
  if ((e = launch_router_fix(fa, st)) != cudaSuccess) return e;
  if (mid != nullptr && (e = cudaEventRecord(mid, st)) != cudaSuccess) return e;
  return launch_route_prefill(s, luts, sc, T, topk_idx, topk_score, count_pairs ? sc.pair_count : nullptr, st);
}

cudaError_t launch_prefill_offsets(const Shape& s, const Scratch& sc, int ecount, int sh_T, cudaStream_t st) {
  OffsetsArgs oa{ecount, sh_T, 2 * s.I / kBM, 2 * s.Is / kBM, s.H / kBM, sc.pair_count, sc.pair_fill, sc.pair_offset,
                 sc.unit_prefix};
  return launch_pdl_ex(k_pf_offsets, dim3(1), dim3((ecount + 31) / 32 * 32), 0, st, oa);
}

cudaError_t launch_prefill_group(const Shape& s, const Scratch& sc, const int32_t* idx, int n_pairs,
                                 const uint16_t* x_src, int ep_rank, int ep_world, int ecount, int sh_T,
                                 bool count_here, cudaStream_t st) {
  cudaError_t e;
  if (count_here) {
    if ((e = cudaMemsetAsync(sc.pair_count, 0, sizeof(int) * ecount, st)) != cudaSuccess) return e;
    const int blocks = std::min(4 * sm_count(), (n_pairs + 255) / 256 > 0 ? (n_pairs + 255) / 256 : 1);
    if ((e = launch_pdl_ex(k_ep_count, dim3(blocks), dim3(256), 0, st, idx, n_pairs, ep_rank, ep_world, ecount,
                           sc.pair_count)) !=
        cudaSuccess)
      return e;
  }
  if ((e = launch_prefill_offsets(s, sc, ecount, sh_T, st)) != cudaSuccess) return e;
  if (s.K > 32) return cudaErrorInvalidValue;
  const int tokens = (n_pairs + s.K - 1) / s.K;
  return launch_pdl_ex(k_pf_scatter, dim3((tokens + kScatterTokens - 1) / kScatterTokens), dim3(kScatterTokens * 32),
                       scatter_smem(ecount), st, idx, n_pairs, s.K, s.E, s.H, ep_rank,
                       ep_world, static_cast<const int*>(sc.pair_offset), sc.pair_fill, sc.pair_tk, x_src, sc.xg,
                       static_cast<long long>(sc.pair_cap), sc.err);
}

cudaError_t launch_prefill_gemms(const Shape& s, const PrefillWeightMaps& wm, const PrefillScratchMaps& smaps,
                                 const Luts& luts, const Scratch& sc, const uint16_t* x_own, int T_own, int ecount,
                                 const uint16_t* score, const int32_t* send_pos, uint16_t* out_rows,
                                 cudaStream_t st, const EpPeers* ep) {
  // Per-forward map of this rank's input rows (the shared expert's token tiles).
  TokenMaps x_rows;
  if (!token_maps(&x_rows, x_own, s.H, T_own)) return cudaErrorInvalidValue;
  cudaError_t e;
  const size_t smem = gemm_smem_bytes(ecount);
  const dim3 grid(sm_count()), block(kGemmThreads);
  GemmArgs g{};
  auto launch = [&](const CUtensorMap& ma_r, const CUtensorMap& ma_s, const TokenMaps& mb_r, const TokenMaps& mb_s) {
    return launch_pdl_ex(k_gemm, grid, block, smem, st, ma_r, ma_s, mb_r, mb_s, g);
  };
  g.E = ecount;
  g.T = T_own;
  g.K = s.K;
  g.H = s.H;
  g.I = s.I;
  g.Is = s.Is;
  g.offset = sc.pair_offset;
  g.pair_tk = sc.pair_tk;
  g.score = score;
  g.sh_sig = sc.sh_sig;
  g.silu = luts.silu;
  g.act = sc.act;
  g.act_sh = sc.act_sh;
  g.weighted = out_rows;
  g.gated_sh = sc.gated_sh;
  g.err = sc.err;
  g.send_pos = send_pos;
  if (ep != nullptr) g.ep = *ep;
  g.rows_r = sc.pair_cap;
  g.rows_s = sc.max_T;
  // gate/up + SwiGLU
  g.phase = 0;
  g.kb_r = s.H / kBK;
  g.kb_s = s.H / kBK;
  g.mt_r = 2 * s.I / kBM;
  g.mt_s = 2 * s.Is / kBM;
  g.groups_r = 2 * s.I / 8;
  g.b_blocked_s = 0;  // shared up: the row-major input
  g.prefix = sc.unit_prefix;
  if ((e = launch(wm.gate_up, wm.sh_gate_up, smaps.xg, x_rows)) != cudaSuccess) return e;
  // down + route weight / shared gate
  g.phase = 1;
  g.kb_r = s.I / kBK;
  g.kb_s = s.Is / kBK;
  g.mt_r = s.H / kBM;
  g.mt_s = s.H / kBM;
  g.groups_r = s.H / 8;
  g.b_blocked_s = 1;  // shared down: K-blocked act_sh
  g.prefix = sc.unit_prefix + 2 * (ecount + 2);
  return launch(wm.down, wm.sh_down, smaps.act, smaps.act_sh);
}

cudaError_t launch_ep_positions(const int32_t* idx, int n, int group_len, int me, int world, bool recv,
                                int32_t* pos, int* count, int* offset, cudaStream_t st) {
  if (world > kEpMaxWorld) return cudaErrorInvalidValue;
  return launch_pdl_ex(k_ep_positions, dim3(1), dim3(1024), 0, st, idx, n, group_len, me, world, recv ? 1 : 0,
                       pos, count, offset);
}

cudaError_t launch_prefill(const Shape& s, const LayerWeights& w, const PrefillWeightMaps& wm,
                           const PrefillScratchMaps& smaps, const Luts& luts, const Scratch& sc, const uint16_t* x,
                           int T, uint16_t* y, int32_t* topk_idx, uint16_t* topk_score, cudaStream_t st,
                           cudaEvent_t* ev, const HcPost* hc) {
  if (T <= 0) return cudaSuccess;
  cudaError_t e;
  auto mark = [&](int i) { return ev != nullptr ? cudaEventRecord(ev[i], st) : cudaSuccess; };
  if ((e = mark(0)) != cudaSuccess) return e;
  if ((e = launch_prefill_front(s, w, wm, luts, sc, x, T, topk_idx, topk_score, true, st,
                                ev != nullptr ? ev[1] : nullptr)) != cudaSuccess)
    return e;
  if ((e = mark(2)) != cudaSuccess) return e;
  if ((e = launch_prefill_group(s, sc, topk_idx, T * s.K, x, 0, 1, s.E, T, false, st)) != cudaSuccess) return e;
  if ((e = mark(3)) != cudaSuccess) return e;
  if ((e = launch_prefill_gemms(s, wm, smaps, luts, sc, x, T, s.E, topk_score, nullptr, sc.weighted, st)) !=
      cudaSuccess)
    return e;
  if ((e = mark(4)) != cudaSuccess) return e;
  if ((e = launch_combine(s, sc, T, y, st, nullptr, 0, nullptr, nullptr, hc)) != cudaSuccess) return e;
  return mark(5);
}

}  // namespace fw
