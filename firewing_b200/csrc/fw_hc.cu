// fw_hc.cu -- the hyper-connection caller on either side of the block
// (src/hyper_connection.rs:412-490, src/decoder_layer.rs:451-458, 587-607).
//
// Before the block, per token, from the attention output post [4H] (four
// streams of H):
//   normed  = grouped_rms(post, hc_norm)          k_hc_norm
//   down    = linear_bf16(mix_down [LR][4H], normed)   k_hc_gemv
//   down    = bf16(silu(bf16(down / 4)))            k_hc_silu
//   up      = linear_bf16(mix_up [4H][LR], down)   k_hc_gemv
//   mixed   = bf16(mean over streams of bf16(sigmoid(up) * normed))   k_hc_mix
//   inject  = linear_bf16(inject [4][4H], normed)  k_hc_gemv
//   w       = bf16(2 * sigmoid(bf16(inject / 4)))   k_hc_mix
// `mixed` is the block input.  After the block the combine writes
// out[g*H + c] = bf16(post[g*H + c] + bf16(moe[c] * w[g])) in its epilogue
// (HcPost in fw_kernels.h), so the block output never round-trips.
//
// Every rounding point is the reference's: the square-sum cascade of
// grouped_rms in its exact order, the 32-partial dot schedule, sigmoid and
// SiLU from the host-built tables.
#include <cstdint>

#include "fw_common.cuh"
#include "fw_kernels.h"

namespace fw {
namespace {

// One warp per (token, stream): PyTorch's contiguous f32 square-sum cascade
// (src/hyper_connection.rs:211-283; 4 lanes x 4 interleaved registers x 4
// levels) with lane 4*r + l owning accumulator chain (register r, lane l),
// then inverse = 1 / sqrt(sum / H + eps) and bf16(v * inverse * (1 + w)).
// H must be a multiple of 16 (no leftover vectors or tail elements).
__global__ void k_hc_norm(const uint16_t* post, const uint16_t* norm_w, int H, float eps, uint16_t* normed) {
  const int tg = blockIdx.x;  // token * 4 + stream
  const int g = tg & 3;
  const int lane = threadIdx.x;
  const uint16_t* in = post + static_cast<size_t>(tg) * H;
  const int r = (lane >> 2) & 3, l = lane & 3;
  const int cascade = H / 16;
  int ceil_log2 = 0;
  for (int v = cascade - 1; v > 0; v >>= 1) ++ceil_log2;
  if (cascade <= 1) ceil_log2 = 0;
  const int power = (ceil_log2 / 4) > 4 ? (ceil_log2 / 4) : 4;
  const int step = 1 << power, mask = step - 1;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // levels 0..3 of this chain
  auto sq = [&](int index) {
    const float v = bf16_to_f32(in[(index * 4 + r) * 4 + l]);
    return __fmul_rn(v, v);
  };
  int index = 0;
  while (index + step <= cascade) {
    for (int s = 0; s < step; ++s, ++index) acc[0] = __fadd_rn(acc[0], sq(index));
    for (int level = 1; level < 4; ++level) {
      acc[level] = __fadd_rn(acc[level], acc[level - 1]);
      acc[level - 1] = 0.0f;
      if (index & (mask << (level * power))) break;
    }
  }
  for (; index < cascade; ++index) acc[0] = __fadd_rn(acc[0], sq(index));
  for (int level = 1; level < 4; ++level) acc[0] = __fadd_rn(acc[0], acc[level]);
  // registers 1..3 into register 0, per lane, in order
  float c0 = acc[0];
  const float c1 = __shfl_down_sync(0xffffffffu, c0, 4);
  const float c2 = __shfl_down_sync(0xffffffffu, c0, 8);
  const float c3 = __shfl_down_sync(0xffffffffu, c0, 12);
  c0 = __fadd_rn(__fadd_rn(__fadd_rn(c0, c1), c2), c3);  // valid in lanes 0..3
  const float a1 = __shfl_sync(0xffffffffu, c0, 1), a2 = __shfl_sync(0xffffffffu, c0, 2),
              a3 = __shfl_sync(0xffffffffu, c0, 3);
  float sum = 0.0f;
  sum = __fadd_rn(sum, c0);
  sum = __fadd_rn(sum, a1);
  sum = __fadd_rn(sum, a2);
  sum = __fadd_rn(sum, a3);
  sum = __shfl_sync(0xffffffffu, sum, 0);
  const float inverse = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, static_cast<float>(H)), eps)));
  const uint16_t* w = norm_w + static_cast<size_t>(g) * H;
  uint16_t* out = normed + static_cast<size_t>(tg) * H;
  for (int i = lane; i < H; i += 32) {
    const float gain = __fadd_rn(1.0f, bf16_to_f32(w[i]));
    out[i] = f32_to_bf16(__fmul_rn(__fmul_rn(bf16_to_f32(in[i]), inverse), gain));
  }
}

// linear_bf16 (src/expert.rs:554-560) with the reference dot schedule: one
// warp per (row, token), lane j sums columns j, j+32, ... in order; the
// tree +16, +8, +4, (0+1)+(2+3).  cols % 32 == 0.
__global__ void k_hc_gemv(const uint16_t* w, const uint16_t* x, int rows, int cols, int T, uint16_t* y) {
  const long long wi = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wi >= static_cast<long long>(rows) * T) return;
  const int row = static_cast<int>(wi % rows), t = static_cast<int>(wi / rows);
  const uint16_t* wr = w + static_cast<size_t>(row) * cols + lane;
  const uint16_t* xr = x + static_cast<size_t>(t) * cols + lane;
  float acc = 0.0f;
  for (int b = 0; b < cols; b += 32) acc = fmaf(bf16_to_f32(wr[b]), bf16_to_f32(xr[b]), acc);
  acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 16));
  acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 8));
  acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
  const float q = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));  // lanes 0, 2: (0+1), (2+3)
  const float dot = __fadd_rn(q, __shfl_down_sync(0xffffffffu, q, 2));
  if (lane == 0) y[static_cast<size_t>(t) * rows + row] = f32_to_bf16(dot);
}

// mix_down -> bf16(silu(bf16(v / 4))) in place (SiLU from the table).
__global__ void k_hc_silu(uint16_t* v, long long n, const uint16_t* silu) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    v[i] = silu[f32_to_bf16(__fdiv_rn(bf16_to_f32(v[i]), 4.0f))];
}

// mixed[t][c] = bf16(((((0 + p0) + p1) + p2) + p3) / 4) with
// p_g = bf16(sigmoid(up[g*H + c]) * normed[g*H + c]); and the injection
// weights w[t][g] = bf16(2 * sigmoid(bf16(inject[t][g] / 4))).
__global__ void k_hc_mix(const uint16_t* up, const uint16_t* normed, const uint16_t* inject, int H, int T,
                         const uint16_t* sigmoid, uint16_t* mixed, uint16_t* inj_w) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i < 4LL * T) {
    const uint16_t s = sigmoid[f32_to_bf16(__fdiv_rn(bf16_to_f32(inject[i]), 4.0f))];
    inj_w[i] = f32_to_bf16(__fmul_rn(2.0f, bf16_to_f32(s)));
  }
  if (i >= static_cast<long long>(T) * H) return;
  const long long t = i / H, c = i - t * H;
  float sum = 0.0f;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const size_t k = static_cast<size_t>(t) * 4 * H + static_cast<size_t>(g) * H + c;
    const float p = bf16_to_f32(f32_to_bf16(__fmul_rn(bf16_to_f32(sigmoid[up[k]]), bf16_to_f32(normed[k]))));
    sum = __fadd_rn(sum, p);
  }
  mixed[i] = f32_to_bf16(__fdiv_rn(sum, 4.0f));
}

int blocks_for(long long n, int per) {
  const long long b = (n + per - 1) / per;
  return static_cast<int>(b < 1 ? 1 : (b > 65535LL * 16 ? 65535LL * 16 : b));
}

}  // namespace

cudaError_t launch_hc_pre(const HcWeights& w, const HcScratch& hs, const Luts& luts, const uint16_t* post, int H,
                          int T, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  const int HH = 4 * H, LR = w.lowrank;
  k_hc_norm<<<4 * T, 32, 0, st>>>(post, w.norm, H, 1.0e-6f, hs.normed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  auto gemv = [&](const uint16_t* mat, const uint16_t* x, int rows, int cols, uint16_t* y) {
    const long long warps = static_cast<long long>(rows) * T;
    k_hc_gemv<<<blocks_for(warps * 32, 256), 256, 0, st>>>(mat, x, rows, cols, T, y);
    return cudaGetLastError();
  };
  if ((e = gemv(w.mix_down, hs.normed, LR, HH, hs.down)) != cudaSuccess) return e;
  k_hc_silu<<<blocks_for(static_cast<long long>(T) * LR, 256), 256, 0, st>>>(hs.down, static_cast<long long>(T) * LR,
                                                                             luts.silu);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if ((e = gemv(w.mix_up, hs.down, HH, LR, hs.up)) != cudaSuccess) return e;
  if ((e = gemv(w.inject, hs.normed, 4, HH, hs.inject)) != cudaSuccess) return e;
  k_hc_mix<<<blocks_for(static_cast<long long>(T) * H, 256), 256, 0, st>>>(hs.up, hs.normed, hs.inject, H, T,
                                                                           luts.sigmoid, hs.mixed, hs.inj_w);
  return cudaGetLastError();
}

}  // namespace fw
