// fw_layout.cu -- the tiled expert layout: synthetic generation into it and
// re-layout from the reference layout (see TiledSpec in fw_kernels.h).
#include <cstdint>
#include <mutex>

#include "fw_common.cuh"
#include "fw_kernels.h"

namespace fw {
namespace {

__device__ __forceinline__ uint64_t mix64_dev(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Source (0 / 1) and reference index of tiled element d.
__device__ __forceinline__ void tiled_source(const TiledSpec& s, long long d, int& src, long long& ref) {
  const long long ml = d / s.mat_elems;
  const long long dl = d - ml * s.mat_elems;
  const long long m = ml * s.m_stride + s.m0;
  const long long seg = dl >> 9;  // 512 elements per 8 x 64 segment
  const int w = static_cast<int>(dl & 511);
  const int r = w >> 6, pc = w & 63;
  const int nseg = s.K >> 6;
  const long long g = seg / nseg;
  const int col = static_cast<int>(seg - g * nseg) * 64 + ((((pc >> 3) ^ r) << 3) | (pc & 7));
  if (s.kind == 0) {
    const long long row = 4 * g + (r & 3);
    if (s.half > 0) {
      src = 0;
      ref = m * s.src_mat_elems + (row + (r < 4 ? 0 : s.half)) * s.K + col;
    } else {
      src = r < 4 ? 0 : 1;
      ref = m * s.src_mat_elems + row * s.K + col;
    }
  } else {
    src = 0;
    ref = m * s.src_mat_elems + (8 * g + r) * s.K + col;
  }
}

__global__ void k_synth_tiled(TiledSpec s, long long total, uint64_t key0, uint64_t key1, float scale,
                              uint16_t* out) {
  const uint64_t gamma = 0x9E3779B97F4A7C15ull;
  for (long long d = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; d < total;
       d += static_cast<long long>(gridDim.x) * blockDim.x) {
    int src;
    long long ref;
    tiled_source(s, d, src, ref);
    const uint64_t h = mix64_dev((src == 0 ? key0 : key1) + (static_cast<uint64_t>(ref) + 1) * gamma);
    const int32_t v = static_cast<int32_t>(h & 0xffffu) + static_cast<int32_t>((h >> 16) & 0xffffu) +
                      static_cast<int32_t>((h >> 32) & 0xffffu) + static_cast<int32_t>(h >> 48) - 131070;
    out[d] = f32_to_bf16(__fmul_rn(static_cast<float>(v), scale));
  }
}

__global__ void k_relayout(TiledSpec s, long long d0, long long count, long long src_base, const uint16_t* src0,
                           const uint16_t* src1, uint16_t* out) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long d = d0 + i;
    int src;
    long long ref;
    tiled_source(s, d, src, ref);
    out[d] = (src == 0 ? src0 : src1)[ref - src_base];
  }
}

}  // namespace

cudaError_t launch_synth_tiled(const TiledSpec& spec, long long n_mats, uint64_t key0, uint64_t key1, float scale,
                               uint16_t* out, cudaStream_t st) {
  const long long total = n_mats * spec.mat_elems;
  if (total <= 0) return cudaSuccess;
  k_synth_tiled<<<148 * 8, 256, 0, st>>>(spec, total, key0, key1, scale, out);
  return cudaGetLastError();
}

cudaError_t launch_relayout(const TiledSpec& spec, long long m0, long long n, const uint16_t* src0,
                            const uint16_t* src1, uint16_t* out, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  // The sources hold matrices m0.. only: shift reference indices by m0's.
  k_relayout<<<148 * 8, 256, 0, st>>>(spec, m0 * spec.mat_elems, n * spec.mat_elems, m0 * spec.src_mat_elems,
                                      src0, src1, out);
  return cudaGetLastError();
}

cudaError_t current_device_attrs(DeviceAttrs* out) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static DeviceAttrs cache[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  DeviceAttrs& a = cache[dev];
  if (a.sms == 0) {
    DeviceAttrs v;
    if ((e = cudaDeviceGetAttribute(&v.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&v.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
      return e;
    if (v.sms <= 0) return cudaErrorInvalidDevice;
    a = v;
  }
  *out = a;
  return cudaSuccess;
}

}  // namespace fw
