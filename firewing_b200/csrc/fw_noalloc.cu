// fw_noalloc.cu -- the sparse-MoE block forward without any device allocation.
//
// fw_moe_forward is built around a handle that cudaMallocs its weights and
// per-forward scratch.  Some callers cannot do that: a host framework whose
// caching allocator has already reserved the GPU's memory (any further
// cudaMalloc fails), or a latency-critical loop that must not call
// cudaMalloc/cudaFree because they synchronise the device.  For them,
// fw_moe_forward_noalloc runs the same block with caller-owned weights,
// inputs and outputs, and takes its scratch from a fixed area compiled into
// this library:
//   - g_scratch, a file-scope __device__ array of kNoAllocScratchBytes (8 MiB);
//     every GPU that loads the library holds it until the process exits;
//   - the two 65,536-entry bf16 tables (SiLU, sigmoid), also file-scope.
// The first call on a device (with that device current) looks up the
// arrays' device addresses with cudaGetSymbolAddress and uploads the tables;
// make that first call before any stream capture.  All calls share the one
// scratch area and leave their contents in it, so calls that overlap on the
// GPU (two streams, two host threads) race; this entry point is synchronous
// on its stream to keep back-to-back calls ordered.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include <cuda_runtime.h>

#include "fw_kernels.h"
#include "fwmoe.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_scratch[kNoAllocScratchBytes];
__device__ __align__(256) uint16_t g_silu_table[65536];
__device__ __align__(256) uint16_t g_sigmoid_table[65536];

struct DeviceState {
  bool ready = false;
  unsigned char* scratch = nullptr;  // device address of g_scratch
  uint16_t* silu = nullptr;
  uint16_t* sigmoid = nullptr;
};

std::mutex g_setup_mu;
DeviceState g_state[kMaxDevices];
// Host copies of the tables: static storage, so set-up allocates nothing.
uint16_t g_host_silu[65536];
uint16_t g_host_sigmoid[65536];
bool g_host_tables_ready = false;

uint16_t to_bf16(float v) {
  uint32_t b;
  std::memcpy(&b, &v, sizeof b);
  return static_cast<uint16_t>((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
}
float from_bf16(uint16_t v) {
  const uint32_t b = static_cast<uint32_t>(v) << 16;
  float f;
  std::memcpy(&f, &b, sizeof f);
  return f;
}

int cuda_fail(const char* what, cudaError_t e) {
  char msg[256];
  std::snprintf(msg, sizeof msg, "fw_moe_forward_noalloc: %s: %s", what, cudaGetErrorString(e));
  return fw::record_error(FW_ECUDA, msg);
}

// Once per device, with that device current.
int setup_device(int dev, DeviceState** out) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  DeviceState& st = g_state[dev];
  if (!st.ready) {
    if (!g_host_tables_ready) {
      // bf16(silu(g)) and sigmoid_bf16(g) for every bf16 pattern, with the
      // host libm, as the reference builds its table (src/metal_moe.rs:385-392).
      for (uint32_t bits = 0; bits < 65536u; ++bits) {
        const float g = from_bf16(static_cast<uint16_t>(bits));
        g_host_silu[bits] = to_bf16(g / (1.0f + std::exp(-g)));
        g_host_sigmoid[bits] = to_bf16(1.0f / (1.0f + std::exp(-g)));
      }
      g_host_tables_ready = true;
    }
    cudaError_t e;
    void* p = nullptr;
    // In host code the array names are host-side stand-ins; the device
    // addresses come from the runtime.
    if ((e = cudaGetSymbolAddress(&p, g_scratch)) != cudaSuccess) return cuda_fail("scratch address", e);
    st.scratch = static_cast<unsigned char*>(p);
    if ((e = cudaGetSymbolAddress(&p, g_silu_table)) != cudaSuccess) return cuda_fail("silu table address", e);
    st.silu = static_cast<uint16_t*>(p);
    if ((e = cudaGetSymbolAddress(&p, g_sigmoid_table)) != cudaSuccess)
      return cuda_fail("sigmoid table address", e);
    st.sigmoid = static_cast<uint16_t*>(p);
    if ((e = cudaMemcpyAsync(st.silu, g_host_silu, sizeof g_host_silu, cudaMemcpyHostToDevice,
                             cudaStreamLegacy)) != cudaSuccess)
      return cuda_fail("silu table upload", e);
    if ((e = cudaMemcpyAsync(st.sigmoid, g_host_sigmoid, sizeof g_host_sigmoid, cudaMemcpyHostToDevice,
                             cudaStreamLegacy)) != cudaSuccess)
      return cuda_fail("sigmoid table upload", e);
    // landed before any stream reads them (pageable copies may return early)
    if ((e = cudaStreamSynchronize(cudaStreamLegacy)) != cudaSuccess) return cuda_fail("table upload", e);
    st.ready = true;
  }
  *out = &st;
  return FW_OK;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Lay the forward's scratch out in `base` (or only size it when base is
// null).  Returns the bytes needed.
size_t carve(const fw::Shape& s, int T, bool need_idx, bool need_score, unsigned char* base,
             fw::Scratch* sc, int32_t** idx, uint16_t** score) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    unsigned char* p = base ? base + off : nullptr;
    off = align256(off + bytes);
    return p;
  };
  const size_t E = s.E, K = s.K, H = s.H, I = s.I, Is = s.Is, M = T;
  sc->max_T = T;
  sc->logits = reinterpret_cast<uint16_t*>(take(M * E * 2));
  sc->sh_logit = reinterpret_cast<uint16_t*>(take(M * 2));
  sc->sh_sig = reinterpret_cast<uint16_t*>(take(M * 2));
  sc->sorted_slot = reinterpret_cast<int32_t*>(take(M * K * 4));
  sc->sched = reinterpret_cast<int32_t*>(take(fw::sched_words(s.E, T, s.K) * 4));
  sc->act = reinterpret_cast<uint16_t*>(take(M * K * 2 * I * 2));
  sc->act_sh = reinterpret_cast<uint16_t*>(take(M * 2 * Is * 2));
  sc->weighted = reinterpret_cast<uint16_t*>(take(M * K * H * 2));
  sc->gated_sh = reinterpret_cast<uint16_t*>(take(M * H * 2));
  sc->up_done = reinterpret_cast<int*>(take((E + 1) * 4));
  sc->ticket = reinterpret_cast<int*>(take(sizeof(int)));
  sc->err = reinterpret_cast<int*>(take(sizeof(int)));
  *idx = need_idx ? reinterpret_cast<int32_t*>(take(M * K * 4)) : nullptr;
  *score = need_score ? reinterpret_cast<uint16_t*>(take(M * K * 2)) : nullptr;
  return off;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace

extern "C" int fw_moe_forward_noalloc(const fw_moe_config* config, const fw_moe_weights* weights,
                                      const uint16_t* x, int32_t tokens, uint16_t* y,
                                      int32_t* topk_idx, uint16_t* topk_scores, void* stream) {
  if (config == nullptr || weights == nullptr)
    return fw::record_error(FW_EINVAL, "fw_moe_forward_noalloc: config / weights is null");
  const fw_moe_config& c = *config;
  if (c.hidden <= 0 || c.hidden % 64 != 0 || c.hidden > 4096 || c.intermediate <= 0 ||
      c.intermediate % 64 != 0 || c.shared_intermediate <= 0 || c.shared_intermediate % 64 != 0 ||
      c.intermediate > 4096 || c.shared_intermediate > 4096 ||
      c.experts <= 0 || c.experts % 32 != 0 || c.experts > 1024 || c.top_k < 1 || c.top_k > 32 ||
      c.top_k > c.experts)
    return fw::record_error(FW_EINVAL, "fw_moe_forward_noalloc: unsupported block shape");
  if (tokens < 0 || tokens > 256)
    return fw::record_error(FW_EINVAL, "fw_moe_forward_noalloc: tokens must be in [0, 256]");
  if (tokens == 0) return FW_OK;
  const fw_moe_weights& w = *weights;
  if (!w.router || !w.gate_up || !w.down || !w.shared_gate || !w.shared_up || !w.shared_down ||
      !w.shared_gate_w || !x || !y)
    return fw::record_error(FW_EINVAL, "fw_moe_forward_noalloc: a weight / x / y pointer is null");
  if (!aligned(x, 16) || !aligned(y, 16) || !aligned(w.router, 16) || !aligned(w.gate_up, 16) ||
      !aligned(w.down, 16) || !aligned(w.shared_gate, 16) || !aligned(w.shared_up, 16) ||
      !aligned(w.shared_down, 16) || !aligned(w.shared_gate_w, 16) || !aligned(topk_idx, 4) ||
      !aligned(topk_scores, 4))
    return fw::record_error(FW_EINVAL, "fw_moe_forward_noalloc: buffers must be 16-byte aligned");
  const fw::Shape s{c.hidden, c.intermediate, c.shared_intermediate, c.experts, c.top_k};
  fw::Scratch sc;
  int32_t* idx_scratch = nullptr;
  uint16_t* score_scratch = nullptr;
  const size_t need =
      carve(s, tokens, topk_idx == nullptr, topk_scores == nullptr, nullptr, &sc, &idx_scratch, &score_scratch);
  if (need > kNoAllocScratchBytes) {
    char msg[256];
    std::snprintf(msg, sizeof msg,
                  "fw_moe_forward_noalloc: this shape and token count need %zu bytes of scratch; "
                  "the static area holds %zu",
                  need, kNoAllocScratchBytes);
    return fw::record_error(FW_EINVAL, msg);
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices) return fw::record_error(FW_EINVAL, "fw_moe_forward_noalloc: device id");
  DeviceState* st = nullptr;
  const int rc = setup_device(dev, &st);
  if (rc != FW_OK) return rc;
  carve(s, tokens, topk_idx == nullptr, topk_scores == nullptr, st->scratch, &sc, &idx_scratch,
        &score_scratch);
  fw::LayerWeights lw;
  lw.router = w.router;
  lw.gate_up = w.gate_up;
  lw.down = w.down;
  lw.sh_gate = w.shared_gate;
  lw.sh_up = w.shared_up;
  lw.sh_down = w.shared_down;
  lw.sh_gate_w = w.shared_gate_w;
  lw.bias = w.logit_bias;
  lw.expert_count = c.experts;
  const fw::Luts luts{st->silu, st->sigmoid};
  const cudaStream_t cs = static_cast<cudaStream_t>(stream);
  // The status word and the route kernel's completion ticket must start at
  // zero; every other scratch byte is written before it is read in the call.
  if ((e = cudaMemsetAsync(sc.err, 0, sizeof(int), cs)) != cudaSuccess) return cuda_fail("status reset", e);
  if ((e = cudaMemsetAsync(sc.ticket, 0, sizeof(int), cs)) != cudaSuccess) return cuda_fail("ticket reset", e);
  e = fw::launch_block(s, lw, luts, sc, x, tokens, y, topk_idx ? topk_idx : idx_scratch,
                       topk_scores ? topk_scores : score_scratch, cs);
  if (e != cudaSuccess) return cuda_fail("launch", e);
  if ((e = cudaStreamSynchronize(cs)) != cudaSuccess) return cuda_fail("stream sync", e);
  int code = 0;
  if ((e = cudaMemcpy(&code, sc.err, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
    return cuda_fail("status read", e);
  if (code == fw::kErrNanLogits)
    return fw::record_error(FW_ENAN, "fw_moe_forward_noalloc: router received NaN logits");
  if (code != fw::kErrNone) return fw::record_error(FW_ECUDA, "fw_moe_forward_noalloc: device status");
  return FW_OK;
}
