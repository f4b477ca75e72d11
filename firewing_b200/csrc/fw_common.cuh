// fw_common.cuh -- device helpers shared by the sparse-MoE kernels (sm_100a).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "fw_kernels.h"

namespace fw {

__device__ __forceinline__ void set_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// bf16 <-> f32 with the reference's arithmetic (src/expert.rs:315-322):
// round-to-nearest-even by an integer add.  One deviation, for NaN only: GPU
// arithmetic returns the canonical NaN 0x7fffffff, which that integer add
// would carry into -0.0, whereas the reference's CPU propagates the input
// NaN's payload (0x7fc00000) and the add keeps it a NaN.  A NaN therefore
// rounds to the quiet NaN 0x7fc0, so NaN inputs still reach route()'s NaN
// rejection (src/decoder_layer.rs:279-281).
__device__ __forceinline__ float bf16_to_f32(uint32_t bits16) { return __uint_as_float(bits16 << 16); }
__device__ __forceinline__ uint16_t f32_to_bf16(float v) {
  const uint32_t b = __float_as_uint(v);
  if ((b & 0x7fffffffu) > 0x7f800000u) return 0x7fc0u;
  return static_cast<uint16_t>((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
}
// a + b per bf16 half (low and high), rounded once to bf16 with round to
// nearest even, NaN results as 0x7fc0: bit-identical to
// f32_to_bf16(bf16_to_f32(a) + bf16_to_f32(b)) per half (the reference's
// add_bf16, src/expert.rs:578).  For two bf16 operands the f32 sum is exact
// unless their exponents differ by 16 or more; the smaller operand is then
// below 2^-15 of the larger, under half a bf16 step, and both roundings give
// the larger operand.
__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  uint32_t lo = r & 0xffffu, hi = r >> 16;
  lo = (lo & 0x7fffu) > 0x7f80u ? 0x7fc0u : lo;
  hi = (hi & 0x7fffu) > 0x7f80u ? 0x7fc0u : hi;
  return lo | (hi << 16);
}
// acc += lo(w) * lo(x), then acc += hi(w) * hi(x): mixed-precision FMAs
// (bf16 operands, f32 accumulator); an exact bf16 product and one rounding
// per add, as the reference's multiply then add.
__device__ __forceinline__ float fma_seq2(uint32_t w, uint32_t x, float acc) {
  asm("{\n\t.reg .b16 w0, w1, x0, x1;\n\t"
      "mov.b32 {w0, w1}, %1;\n\t"
      "mov.b32 {x0, x1}, %2;\n\t"
      "fma.rn.f32.bf16 %0, w0, x0, %0;\n\t"
      "fma.rn.f32.bf16 %0, w1, x1, %0;\n\t}"
      : "+f"(acc)
      : "r"(w), "r"(x));
  return acc;
}

// Two packed bf16 values (little-endian: element 0 in the low half).
__device__ __forceinline__ float lo_bf16(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf16(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// f32 total order (Rust f32::total_cmp) on bf16 bits: larger key = larger
// value, -0 < +0.  Used with ascending-index tie-break (src/router.rs:241-247).
__device__ __forceinline__ uint32_t total_key(uint32_t bits16) {
  return (bits16 & 0x8000u) ? (~bits16 & 0xffffu) : (bits16 | 0x8000u);
}

// Streaming 16-byte weight load: read-only path, no L1 allocation.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Programmatic dependent launch (PDL): wait for the preceding grid's
// results / let the next grid start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// One 32-column block of the reference dot schedule for a lane that owns
// partials 8q..8q+7 (q = lane & 3): acc[i] += w[i] * x[i] for the 8
// consecutive columns it loaded.  A bf16 x bf16 product is exact in f32
// (16 significant bits), so fmaf(w, x, acc) rounds exactly like the
// reference's rounded multiply followed by a rounded add, for every product
// that neither underflows below 2^-126 nor overflows.
__device__ __forceinline__ void fma8(const uint4 w, const float4 xa, const float4 xb, float* acc) {
  acc[0] = fmaf(lo_bf16(w.x), xa.x, acc[0]);
  acc[1] = fmaf(hi_bf16(w.x), xa.y, acc[1]);
  acc[2] = fmaf(lo_bf16(w.y), xa.z, acc[2]);
  acc[3] = fmaf(hi_bf16(w.y), xa.w, acc[3]);
  acc[4] = fmaf(lo_bf16(w.z), xb.x, acc[4]);
  acc[5] = fmaf(hi_bf16(w.z), xb.y, acc[5]);
  acc[6] = fmaf(lo_bf16(w.w), xb.z, acc[6]);
  acc[7] = fmaf(hi_bf16(w.w), xb.w, acc[7]);
}

// Finish the reference reduction tree (src/expert.rs:530-540) for a
// 4-lane group holding the 32 partials as 8 per lane: partial j = 8q + i.
//   +16: j += j+16  -> lanes q<2 take lanes q+2
//   +8 : j += j+8   -> lane q=0 takes lane q=1
//   +4 : j += j+4   -> within lane 0: i += i+4
//   (0+1)+(2+3)
// Every lane of the group must call it; the result is valid in lane q = 0.
__device__ __forceinline__ float reduce_partials(float* p) {
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i] += __shfl_down_sync(0xffffffffu, p[i], 2, 4);
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i] += __shfl_down_sync(0xffffffffu, p[i], 1, 4);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] += p[i + 4];
  return (p[0] + p[1]) + (p[2] + p[3]);
}

}  // namespace fw

namespace fw {

// ---- shared-memory async copies (bulk copy engine) and mbarriers ----------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for an mbarrier phase, giving up after `limit_ns` (returns false).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > limit_ns) return false;
  }
}

// L2 policy for weights that are read exactly once per forward.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Global -> shared bulk copy (no multicast); completes `bytes` on `bar`.
// dst and src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Bulk prefetch of global memory into L2 (no shared-memory destination).
// src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) writes to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint4 ld_cg_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Reduction tree for a row whose 32 partials are held 8 per lane by lanes
// r, r+8, r+16, r+24 (q = lane >> 3 selects partials 8q..8q+7):
//   +16 -> q<2 take q+2 (lane+16); +8 -> q=0 takes q=1 (lane+8);
//   +4 within the lane; then (0+1)+(2+3).  Valid in lanes 0..7.
__device__ __forceinline__ float reduce_partials_strided(float* p) {
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i] += __shfl_down_sync(0xffffffffu, p[i], 16);
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i] += __shfl_down_sync(0xffffffffu, p[i], 8);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] += p[i + 4];
  return (p[0] + p[1]) + (p[2] + p[3]);
}

}  // namespace fw

namespace fw {

// acc[i] += w[i] * x[i] for 8 bf16 pairs, with the sm_100 mixed-precision
// FMA (bf16 operands, f32 accumulator): the bf16 x bf16 product is exact in
// f32 and the add is rounded once -- the reference's rounded multiply
// followed by a rounded add, for every product in the normal f32 range.
__device__ __forceinline__ void fma8_bf16(const uint4 w, const uint4 x, float* acc) {
  asm("{\n\t"
      ".reg .b16 w0, w1, w2, w3, w4, w5, w6, w7, x0, x1, x2, x3, x4, x5, x6, x7;\n\t"
      "mov.b32 {w0, w1}, %8;\n\t"
      "mov.b32 {w2, w3}, %9;\n\t"
      "mov.b32 {w4, w5}, %10;\n\t"
      "mov.b32 {w6, w7}, %11;\n\t"
      "mov.b32 {x0, x1}, %12;\n\t"
      "mov.b32 {x2, x3}, %13;\n\t"
      "mov.b32 {x4, x5}, %14;\n\t"
      "mov.b32 {x6, x7}, %15;\n\t"
      "fma.rn.f32.bf16 %0, w0, x0, %0;\n\t"
      "fma.rn.f32.bf16 %1, w1, x1, %1;\n\t"
      "fma.rn.f32.bf16 %2, w2, x2, %2;\n\t"
      "fma.rn.f32.bf16 %3, w3, x3, %3;\n\t"
      "fma.rn.f32.bf16 %4, w4, x4, %4;\n\t"
      "fma.rn.f32.bf16 %5, w5, x5, %5;\n\t"
      "fma.rn.f32.bf16 %6, w6, x6, %6;\n\t"
      "fma.rn.f32.bf16 %7, w7, x7, %7;\n\t"
      "}"
      : "+f"(acc[0]), "+f"(acc[1]), "+f"(acc[2]), "+f"(acc[3]), "+f"(acc[4]), "+f"(acc[5]), "+f"(acc[6]),
        "+f"(acc[7])
      : "r"(w.x), "r"(w.y), "r"(w.z), "r"(w.w), "r"(x.x), "r"(x.y), "r"(x.z), "r"(x.w));
}

}  // namespace fw

namespace fw {

// ---- expert parallelism over NVLink peer memory (see EpPeers) -------------------

__device__ __forceinline__ void st_release_sys_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_volatile_int(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// Flag `kind` that rank `writer` sets in rank `owner`'s window.
__device__ __forceinline__ unsigned* ep_flag(const EpPeers& p, int owner, int kind, int writer) {
  return reinterpret_cast<unsigned*>(p.win[owner] + kind * 128) + writer;
}

// Where the weighted row of pair g*K + k goes: row t*K + k of the receive
// area of the rank that owns token g (rank g / t_local, its token t), in
// that rank's window.
// (pair < world * t_local * K <= 8 * 16384 * 32: 32-bit arithmetic.)
__device__ __forceinline__ uint16_t* ep_recv_row(const EpPeers& p, int pair) {
  const int g = pair / p.K;
  const int k = pair - g * p.K;
  const int owner = g / p.t_local;
  const int t = g - owner * p.t_local;
  return reinterpret_cast<uint16_t*>(p.win[owner] + p.off_recv) + static_cast<size_t>(t * p.K + k) * p.H;
}

// Called by one thread: wait (bounded by p.wait_ns) until every rank has set
// its flag `kind` in this rank's window for forward p.seq.  Returns false
// after recording kErrTimeout (a rank never set it), kErrPeer (a rank
// reported a failure in this forward), or when this rank's status word
// already holds an error (its forward failed earlier; nothing more waits).
__device__ __forceinline__ bool ep_wait_flags(const EpPeers& p, int kind, int* err) {
  const unsigned* f = reinterpret_cast<const unsigned*>(p.win[p.rank] + kind * 128);
  uint64_t t0 = 0;
  bool timing = false;
  for (int w = 0; w < p.world; ++w) {
    unsigned v;
    while (((v = ld_acquire_sys_u32(f + w)) >> 1) < p.seq) {
      if (ld_volatile_int(err) != 0) return false;
      if (!timing) {
        t0 = global_ns();
        timing = true;
      } else if (global_ns() - t0 > p.wait_ns) {
        set_error(err, kErrTimeout);
        return false;
      }
      __nanosleep(100);
    }
    if ((v >> 1) == p.seq && (v & 1u) != 0) {
      set_error(err, kErrPeer);
      return false;
    }
  }
  return ld_volatile_int(err) == 0;
}

// Called by every thread of every CTA at the very end of a kernel whose
// writes other ranks will read (rows in their windows, or this rank's
// window they read from): the last CTA to finish sets flag `kind` to
// 2*seq (+1 when this rank's status word holds an error) in every rank's
// window.  Each CTA fences its writes at system scope before it counts
// itself in; the last one fences again after seeing every count, so every
// CTA's writes precede the flags a peer acquires.
__device__ __forceinline__ void ep_signal(const EpPeers& p, int kind, int* ticket, const int* err) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned ctas = gridDim.x * gridDim.y * gridDim.z;
    if (static_cast<unsigned>(atomicAdd(ticket, 1)) == ctas - 1) {
      __threadfence_system();
      const unsigned v = 2u * p.seq + (ld_volatile_int(err) != 0 ? 1u : 0u);
      for (int w = 0; w < p.world; ++w) st_release_sys_u32(ep_flag(p, w, kind, p.rank), v);
      atomicExch(ticket, 0);
    }
  }
}

}  // namespace fw
