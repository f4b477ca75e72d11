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
//   router (exact, shared with decode) -> route (+ per-expert pair counts)
//   -> k_pf_offsets (one CTA: pair offsets, work-unit prefixes)
//   -> k_pf_scatter (pairs grouped by expert)
//   -> k_gemm<up>:   per expert, [2I x H] gate/up rows x gathered token rows,
//                    SwiGLU in the epilogue -> act [pairs][I] (bf16)
//   -> k_gemm<down>: per expert, [H x I] down rows x act rows, route weight
//                    (or the shared sigmoid gate) in the epilogue ->
//                    weighted [T*K][H] (bf16)
//   -> combine (shared with decode: ascending expert id, bf16 after each add)
//
// The shared expert is one more slot whose token list is all T tokens.
//
// GEMM kernel (k_gemm): persistent, one CTA per SM, 6 warps.
//   warp 0  producer: TMA loads of the weight tile (4-D map over the tiled
//           bank: 128 rows x 64 columns = 16 KB, already in the 128-byte
//           swizzled K-major operand layout) and of the token tile (routed
//           up: tile::gather4 of x rows by token id; otherwise 16-row boxes
//           of contiguous rows, 128-byte swizzle) into a 4-stage ring.
//   warp 1  MMA issuer: tcgen05.mma kind::f16 (bf16 x bf16 -> f32),
//           M = 128 weight rows, N = the unit's tokens rounded up to 16
//           (<= 256), K = 64 per stage as 4 instructions; accumulators in
//           TMEM, double-buffered (2 x 256 columns); tcgen05.commit frees
//           ring stages and hands finished accumulators to the epilogue.
//   warps 2-5 epilogue: tcgen05.ld of the accumulator (warp w reads TMEM
//           lanes 32*(w%4)..+31), bf16 rounding points of the reference,
//           stores.
// Work unit = (slot, 256-token chunk, 128-row tile); units are numbered
// slot-major and dealt round-robin to the CTAs.
//
// Numerics: every product is exact and accumulated in f32 by the tensor
// core in its own order, so outputs differ from the reference's 32-partial
// schedule by f32 rounding before each bf16 rounding point (within the
// block tolerance, max-abs 2e-2 / rel-L2 1e-3).  The router stays exact, so
// expert selection matches the reference bit for bit.
//
// Every wait is bounded (2 s of globaltimer); on expiry the CTA records
// kErrTimeout, stops issuing, lets its copies and MMAs drain (bounded), frees
// its TMEM and exits.
#include <cstdint>
#include <cstdio>
#include <mutex>

#include <cudaTypedefs.h>

#include "fw_common.cuh"
#include "fw_kernels.h"

namespace fw {
namespace {

constexpr int kBM = 128;        // weight rows per tile (MMA M)
constexpr int kBK = 64;         // columns per ring stage (one 128-byte swizzle atom)
constexpr int kBN = 256;        // tokens per work unit (MMA N, max)
constexpr int kRing = 4;        // ring stages
constexpr int kABytes = kBM * kBK * 2;   // 16 KB
constexpr int kBBytes = kBN * kBK * 2;   // 32 KB
constexpr int kGemmThreads = 192;
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

// Four rows (r0..r3) of a 2-D map whose box is 64 columns x 1 row.
__device__ __forceinline__ void tma_gather4(void* dst, const CUtensorMap* map, int col, int r0, int r1, int r2,
                                            int r3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(col), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(smem_u32(bar))
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

// ---- work units ---------------------------------------------------------------

struct GemmArgs {
  int phase;               // 0: gate/up + SwiGLU; 1: down + scale
  int E, T, K, H, I, Is;
  int kb_r, kb_s;          // 64-column stages per unit (routed, shared)
  int mt_r, mt_s;          // 128-row tiles per chunk (routed, shared)
  int groups_r;            // 8-row groups per routed expert matrix
  const int* offset;       // [E+1] grouped pair offsets
  const int* prefix;       // [E+2] unit prefix of this phase (slot E = shared)
  const int32_t* pair_tk;  // [pairs] t*K + k
  const uint16_t* score;   // [T*K] route weights (bf16)
  const uint16_t* sh_sig;  // [T] shared gate (bf16)
  const uint16_t* silu;    // [65536] bf16(silu(g)) table
  uint16_t* act;           // [pairs][I]
  uint16_t* act_sh;        // [T][Is]
  uint16_t* weighted;      // [T*K][H]
  uint16_t* gated_sh;      // [T][H]
  int* err;
};

struct Unit {
  int slot, m, n0, nvalid, bn, kblocks;
  bool routed;
};

// Unit u of this phase; s_prefix / s_offset are the shared-memory copies.
__device__ __forceinline__ Unit decode_unit(const GemmArgs& a, const int* s_prefix, const int* s_offset, int u) {
  int lo = 0, hi = a.E;  // largest slot s with prefix[s] <= u
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_prefix[mid] <= u) lo = mid;
    else hi = mid - 1;
  }
  Unit w;
  w.slot = lo;
  w.routed = lo < a.E;
  const int mt = w.routed ? a.mt_r : a.mt_s;
  const int local = u - s_prefix[lo];
  const int chunk = local / mt;
  w.m = local - chunk * mt;
  const int count = w.routed ? s_offset[lo + 1] - s_offset[lo] : a.T;
  w.n0 = (w.routed ? s_offset[lo] : 0) + chunk * kBN;
  w.nvalid = min(kBN, count - chunk * kBN);
  w.bn = (w.nvalid + 15) & ~15;
  w.kblocks = w.routed ? a.kb_r : a.kb_s;
  return w;
}

struct __align__(8) GemmSmemTail {
  uint64_t full[kRing];
  uint64_t empty[kRing];
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

__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm(const __grid_constant__ CUtensorMap map_a_r, const __grid_constant__ CUtensorMap map_a_s,
           const __grid_constant__ CUtensorMap map_b_r, const __grid_constant__ CUtensorMap map_b_s, GemmArgs a) {
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment for the swizzled operand tiles.
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  unsigned char* ring_a = smem;                         // [kRing][16 KB]
  unsigned char* ring_b = smem + kRing * kABytes;       // [kRing][32 KB]
  GemmSmemTail* tail = reinterpret_cast<GemmSmemTail*>(ring_b + kRing * kBBytes);
  int* s_tok = reinterpret_cast<int*>(tail + 1);        // [kBN] producer's gather rows
  int* s_prefix = s_tok + kBN;                          // [E+2]
  int* s_offset = s_prefix + a.E + 2;                   // [E+1]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&tail->full[i], 1);
      mbar_init(&tail->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tail->acc_full[i], 1);
      mbar_init(&tail->acc_empty[i], 4);
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
  for (int i = threadIdx.x; i < a.E + 2; i += blockDim.x) s_prefix[i] = a.prefix[i];
  for (int i = threadIdx.x; i < a.E + 1; i += blockDim.x) s_offset[i] = a.offset[i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tail->tmem_base;
  const int total = s_prefix[a.E + 1];

  if (warp == 0) {
    // ---------------- producer ----------------
    const uint64_t policy = l2_evict_first_policy();
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < total; u += gridDim.x) {
      if (__any_sync(0xffffffffu, aborted(tail))) break;  // warp-uniform
      const Unit w = decode_unit(a, s_prefix, s_offset, u);
      const bool gather = a.phase == 0 && w.routed;
      if (gather) {
        __syncwarp();
        for (int j = lane; j < w.bn; j += 32) s_tok[j] = a.pair_tk[w.n0 + min(j, w.nvalid - 1)] / a.K;
        __syncwarp();
      }
      const int grp0 = (w.routed ? w.slot * a.groups_r : 0) + w.m * (kBM / 8);
      const CUtensorMap* ma = w.routed ? &map_a_r : &map_a_s;
      const CUtensorMap* mb = w.routed ? &map_b_r : &map_b_s;
      const uint32_t bytes = kABytes + w.bn * kBK * 2;
      for (int kb = 0; kb < w.kblocks; ++kb, ++it) {
        const int st = it % kRing;
        const uint32_t ph = (it / kRing) & 1;
        bool got = true;
        if (lane == 0) {
          got = mbar_wait_bounded(&tail->empty[st], ph ^ 1u, kWaitNs);
          if (got) mbar_arrive_expect_tx(&tail->full[st], bytes);
          else raise_abort(tail, a.err);
        }
        got = __shfl_sync(0xffffffffu, got, 0) != 0;  // lane 0 waited; the warp follows it
        if (!got) {
          ok = false;
          break;
        }
        unsigned char* sa = ring_a + st * kABytes;
        unsigned char* sb = ring_b + st * kBBytes;
        if (lane == 0) tma_load_4d(sa, ma, 0, 0, kb, grp0, &tail->full[st], policy);
        if (gather) {
          for (int j = lane * 4; j < w.bn; j += 128)
            tma_gather4(sb + j * 128, mb, kb * kBK, s_tok[j], s_tok[j + 1], s_tok[j + 2], s_tok[j + 3],
                        &tail->full[st]);
        } else {
          for (int j = lane * 16; j < w.bn; j += 512) tma_load_2d(sb + j * 128, mb, kb * kBK, w.n0 + j, &tail->full[st]);
        }
      }
    }
    // Let the copies already issued land before the CTA can exit.
    if (lane == 0) {
      const int first = it > kRing ? it - kRing : 0;
      for (int j = first; j < it; ++j)
        if (!mbar_wait_bounded(&tail->full[j % kRing], (j / kRing) & 1, kWaitNs)) raise_abort(tail, a.err);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int it = 0, ai = 0;
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
        for (int kb = 0; kb < w.kblocks; ++kb, ++it) {
          const int st = it % kRing;
          const uint32_t ph = (it / kRing) & 1;
          if (!mbar_wait_bounded(&tail->full[st], ph, kWaitNs)) {
            raise_abort(tail, a.err);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(ring_a + st * kABytes);
          const uint32_t sb = smem_u32(ring_b + st * kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_bf16(d, sw128_desc(sa + k * 32), sw128_desc(sb + k * 32), idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&tail->empty[st]);
        }
        if (ok) umma_commit(&tail->acc_full[buf]);
      }
      // Every MMA this thread issued has completed once mma_done flips.
      umma_commit(&tail->mma_done);
      if (!mbar_wait_bounded(&tail->mma_done, 0, kWaitNs)) raise_abort(tail, a.err);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    const int row = q * 32 + lane;  // accumulator row (weight row within the tile)
    int ai = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++ai) {
      // Decisions stay warp-uniform: tcgen05.ld below is warp-collective.
      if (__any_sync(0xffffffffu, aborted(tail))) break;
      const Unit w = decode_unit(a, s_prefix, s_offset, u);
      const int buf = ai & 1;
      const uint32_t aph = (ai >> 1) & 1;
      const bool got = mbar_wait_bounded(&tail->acc_full[buf], aph, kWaitNs);
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0) raise_abort(tail, a.err);
        break;
      }
      tc_fence_after();
      const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * kAccCols;
      if (a.phase == 0) {
        // Rows alternate 4 gate / 4 up per 8-row group: intermediate
        // 4 * group + (row & 3); lanes with (row & 7) < 4 own the gate value
        // and fetch the matching up value from lane + 4.
        const bool gate_lane = (lane & 7) < 4;
        const int inter = 4 * (w.m * (kBM / 8) + (row >> 3)) + (lane & 3);
        uint16_t* dst = w.routed ? a.act : a.act_sh;
        const int width = w.routed ? a.I : a.Is;
        for (int c0 = 0; c0 < w.bn; c0 += 32) {
          uint32_t v[32];
          tmem_ld32(tbase + c0, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float g = __uint_as_float(v[j]);
            const float up = __shfl_down_sync(0xffffffffu, g, 4);
            const int n = c0 + j;
            if (gate_lane && n < w.nvalid) {
              // swiglu_bf16 (src/expert.rs:562-571) on the bf16 gate / up
              // outputs of linear_bf16: bf16(bf16(silu(g)) * u).
              const uint16_t gb = f32_to_bf16(g);
              const float s = bf16_to_f32(a.silu[gb]);
              const float ub = bf16_to_f32(f32_to_bf16(up));
              dst[static_cast<size_t>(w.n0 + n) * width + inter] = f32_to_bf16(s * ub);
            }
          }
        }
      } else {
        const int h = w.m * kBM + row;
        for (int c0 = 0; c0 < w.bn; c0 += 32) {
          uint32_t v[32];
          tmem_ld32(tbase + c0, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = c0 + j;
            if (n < w.nvalid) {
              const float d = bf16_to_f32(f32_to_bf16(__uint_as_float(v[j])));
              if (w.routed) {
                // bf16(down * route weight) (src/expert.rs:748-751)
                const int tk = a.pair_tk[w.n0 + n];
                a.weighted[static_cast<size_t>(tk) * a.H + h] = f32_to_bf16(d * bf16_to_f32(a.score[tk]));
              } else {
                // bf16(sigmoid * down) (src/expert.rs:1144-1147)
                const int t = w.n0 + n;
                a.gated_sh[static_cast<size_t>(t) * a.H + h] = f32_to_bf16(d * bf16_to_f32(a.sh_sig[t]));
              }
            }
          }
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
}

// ---- grouping kernels -----------------------------------------------------------

struct OffsetsArgs {
  int E, T, mt_up_r, mt_up_s, mt_dn;
  int* count;    // [E], zeroed here for the next forward
  int* fill;     // [E], zeroed here
  int* offset;   // [E+1]
  int* prefix;   // [2][E+2]
};

// One CTA of blockDim.x >= E threads (thread e = expert e).
__global__ void k_pf_offsets(OffsetsArgs a) {
  __shared__ int wsum[3][32];
  pdl_wait();
  pdl_launch_dependents();
  const int e = threadIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  const int c = e < a.E ? a.count[e] : 0;
  const int chunks = (c + kBN - 1) / kBN;
  int v[3] = {c, chunks * a.mt_up_r, chunks * a.mt_dn};
  int incl[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
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
    for (int i = 0; i < 3; ++i) {
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
  int excl[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) excl[i] = incl[i] - v[i] + (warp > 0 ? wsum[i][warp - 1] : 0);
  if (e < a.E) {
    a.offset[e] = excl[0];
    a.prefix[e] = excl[1];
    a.prefix[a.E + 2 + e] = excl[2];
    a.count[e] = 0;
    a.fill[e] = 0;
  }
  if (e == 0) {
    const int pairs = wsum[0][nw - 1], up = wsum[1][nw - 1], dn = wsum[2][nw - 1];
    const int sh_chunks = (a.T + kBN - 1) / kBN;
    a.offset[a.E] = pairs;
    a.prefix[a.E] = up;
    a.prefix[a.E + 1] = up + sh_chunks * a.mt_up_s;
    a.prefix[a.E + 2 + a.E] = dn;
    a.prefix[a.E + 2 + a.E + 1] = dn + sh_chunks * a.mt_dn;
  }
}

// One thread per (token, top-k position): its slot in its expert's group.
__global__ void k_pf_scatter(const int32_t* idx, int TK, int E, const int* offset, int* fill, int32_t* pair_tk,
                             int* err) {
  pdl_wait();
  pdl_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= TK) return;
  const int e = idx[i];
  if (e < 0 || e >= E) {
    set_error(err, kErrBadIndex);
    return;
  }
  pair_tk[offset[e] + atomicAdd(&fill[e], 1)] = i;
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
  return 1024 + static_cast<size_t>(kRing) * (kABytes + kBBytes) + sizeof(GemmSmemTail) +
         sizeof(int) * (kBN + 2 * static_cast<size_t>(E) + 3);
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

int sm_count() {
  static std::once_flag once;
  static int n = 148;
  std::call_once(once, [] {
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
      n = v;
  });
  return n;
}

}  // namespace

bool prefill_supported(const Shape& s) {
  return s.H % kBM == 0 && (2 * s.I) % kBM == 0 && (2 * s.Is) % kBM == 0 && s.E <= 1024;
}

bool make_prefill_weight_maps(const Shape& s, const LayerWeights& w, PrefillWeightMaps* out) {
  if (!w.tiled || !prefill_supported(s)) return false;
  const long long E = w.expert_count;
  return weight_map(&out->gate_up, w.gate_up, s.H, E * 2 * s.I) && weight_map(&out->down, w.down, s.I, E * s.H) &&
         weight_map(&out->sh_gate_up, w.sh_gate, s.H, 2LL * s.Is) && weight_map(&out->sh_down, w.sh_down, s.Is, s.H);
}

bool make_prefill_scratch_maps(const Shape& s, const Scratch& sc, PrefillScratchMaps* out) {
  if (!prefill_supported(s)) return false;
  return rows_map(&out->act, sc.act, s.I, static_cast<long long>(sc.max_T) * s.K, 16) &&
         rows_map(&out->act_sh, sc.act_sh, s.Is, sc.max_T, 16);
}

cudaError_t launch_prefill(const Shape& s, const LayerWeights& w, const PrefillWeightMaps& wm,
                           const PrefillScratchMaps& smaps, const Luts& luts, const Scratch& sc, const uint16_t* x,
                           int T, uint16_t* y, int32_t* topk_idx, uint16_t* topk_score, cudaStream_t st,
                           cudaEvent_t* ev) {
  if (T <= 0) return cudaSuccess;
  cudaError_t e;
  auto mark = [&](int i) { return ev != nullptr ? cudaEventRecord(ev[i], st) : cudaSuccess; };
  // Per-forward maps of the input rows: gathered (routed up) and plain
  // 16-row boxes (shared up).
  CUtensorMap x_gather, x_rows;
  if (!rows_map(&x_gather, x, s.H, T, 1) || !rows_map(&x_rows, x, s.H, T, 16)) return cudaErrorInvalidValue;
  if ((e = mark(0)) != cudaSuccess) return e;
  if ((e = cudaMemsetAsync(sc.pair_count, 0, sizeof(int) * s.E, st)) != cudaSuccess) return e;
  if ((e = launch_router(s, w, sc, x, T, st)) != cudaSuccess || (e = mark(1)) != cudaSuccess) return e;
  if ((e = launch_route_block(s, luts, sc, T, topk_idx, topk_score, false, sc.pair_count, st)) != cudaSuccess)
    return e;
  {
    OffsetsArgs oa{s.E, T, 2 * s.I / kBM, 2 * s.Is / kBM, s.H / kBM, sc.pair_count, sc.pair_fill, sc.pair_offset,
                   sc.unit_prefix};
    const int threads = (s.E + 31) / 32 * 32;
    if ((e = launch_pdl_ex(k_pf_offsets, dim3(1), dim3(threads), 0, st, oa)) != cudaSuccess) return e;
    const int TK = T * s.K;
    if ((e = launch_pdl_ex(k_pf_scatter, dim3((TK + 255) / 256), dim3(256), 0, st,
                           static_cast<const int32_t*>(topk_idx), TK, s.E, static_cast<const int*>(sc.pair_offset),
                           sc.pair_fill, sc.pair_tk, sc.err)) != cudaSuccess)
      return e;
  }
  if ((e = mark(2)) != cudaSuccess) return e;
  const size_t smem = gemm_smem_bytes(s.E);
  const dim3 grid(sm_count()), block(kGemmThreads);
  GemmArgs g{};
  g.E = s.E;
  g.T = T;
  g.K = s.K;
  g.H = s.H;
  g.I = s.I;
  g.Is = s.Is;
  g.offset = sc.pair_offset;
  g.pair_tk = sc.pair_tk;
  g.score = topk_score;
  g.sh_sig = sc.sh_sig;
  g.silu = luts.silu;
  g.act = sc.act;
  g.act_sh = sc.act_sh;
  g.weighted = sc.weighted;
  g.gated_sh = sc.gated_sh;
  g.err = sc.err;
  // gate/up + SwiGLU
  g.phase = 0;
  g.kb_r = s.H / kBK;
  g.kb_s = s.H / kBK;
  g.mt_r = 2 * s.I / kBM;
  g.mt_s = 2 * s.Is / kBM;
  g.groups_r = 2 * s.I / 8;
  g.prefix = sc.unit_prefix;
  if ((e = launch_pdl_ex(k_gemm, grid, block, smem, st, wm.gate_up, wm.sh_gate_up, x_gather, x_rows, g)) !=
      cudaSuccess)
    return e;
  // down + route weight / shared gate
  g.phase = 1;
  g.kb_r = s.I / kBK;
  g.kb_s = s.Is / kBK;
  g.mt_r = s.H / kBM;
  g.mt_s = s.H / kBM;
  g.groups_r = s.H / 8;
  g.prefix = sc.unit_prefix + s.E + 2;
  if ((e = launch_pdl_ex(k_gemm, grid, block, smem, st, wm.down, wm.sh_down, smaps.act, smaps.act_sh, g)) !=
      cudaSuccess)
    return e;
  if ((e = mark(3)) != cudaSuccess) return e;
  if ((e = launch_combine(s, sc, T, y, st)) != cudaSuccess) return e;
  return mark(4);
}

}  // namespace fw
