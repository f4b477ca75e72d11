// fw_api.cu -- the C ABI of include/fwmoe.h.
//
// Host-side runtime around the kernels: handle lifetime, device weight
// ownership, scratch sizing, the bf16 SiLU/sigmoid tables, status mapping.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "fw_kernels.h"
#include "fwmoe.h"

namespace {

// The last failure's message, per thread, in a fixed buffer (recording an
// error never allocates).
thread_local char g_last_error[512] = "";

int fail(int code, const char* msg) {
  std::snprintf(g_last_error, sizeof g_last_error, "%s", msg);
  return code;
}
int fail(int code, const char* what, const char* detail) {
  std::snprintf(g_last_error, sizeof g_last_error, "%s: %s", what, detail);
  return code;
}
int fail(int code, const std::string& msg) { return fail(code, msg.c_str()); }

#define FW_CUDA(call)                                                                    \
  do {                                                                                   \
    const cudaError_t e_ = (call);                                                       \
    if (e_ != cudaSuccess)                                                               \
      return fail(e_ == cudaErrorMemoryAllocation ? FW_ENOMEM : FW_ECUDA, #call,         \
                  cudaGetErrorString(e_));                                               \
  } while (0)

// Host -> device copy that has landed when it returns.  A plain cudaMemcpy
// from pageable memory may return once the bytes are staged, before the DMA
// has written the destination, and it runs on the legacy default stream,
// which a non-blocking stream does not wait for: a kernel launched there next
// could read the destination early.  Copying on the consumer's stream and
// synchronising that stream closes both gaps (cudaStreamLegacy where the
// consumer's stream is not known yet).
cudaError_t upload(void* dst, const void* src, size_t bytes, cudaStream_t st) {
  const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, st);
  return e != cudaSuccess ? e : cudaStreamSynchronize(st);
}
// Zero fill with the same guarantee (cudaMemset on device memory is
// asynchronous with respect to the host).
cudaError_t zero_fill(void* dst, size_t bytes, cudaStream_t st) {
  const cudaError_t e = cudaMemsetAsync(dst, 0, bytes, st);
  return e != cudaSuccess ? e : cudaStreamSynchronize(st);
}

// bf16 helpers with the reference arithmetic (src/expert.rs:315-322).
uint16_t host_to_bf16(float v) {
  uint32_t b;
  std::memcpy(&b, &v, sizeof b);
  return static_cast<uint16_t>((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
}
float host_from_bf16(uint16_t v) {
  const uint32_t b = static_cast<uint32_t>(v) << 16;
  float f;
  std::memcpy(&f, &b, sizeof f);
  return f;
}

// The two 65,536-entry tables, built with the host libm exactly as the
// reference builds its SiLU table (src/metal_moe.rs:385-392) and as
// sigmoid_bf16 rounds (src/expert.rs:573-576).
void build_tables(std::vector<uint16_t>& silu, std::vector<uint16_t>& sigmoid) {
  silu.resize(65536);
  sigmoid.resize(65536);
  for (uint32_t bits = 0; bits < 65536u; ++bits) {
    const float g = host_from_bf16(static_cast<uint16_t>(bits));
    silu[bits] = host_to_bf16(g / (1.0f + std::exp(-g)));
    sigmoid[bits] = host_to_bf16(1.0f / (1.0f + std::exp(-g)));
  }
}

// Per-device tables and status word for the handle-free primitives.
struct DeviceCommon {
  uint16_t* silu = nullptr;
  uint16_t* sigmoid = nullptr;
  int* err = nullptr;
};
std::mutex g_common_mu;
std::map<int, DeviceCommon> g_common;

int device_common(int device, DeviceCommon** out) {
  std::lock_guard<std::mutex> lock(g_common_mu);
  auto it = g_common.find(device);
  if (it == g_common.end()) {
    std::vector<uint16_t> silu, sig;
    build_tables(silu, sig);
    DeviceCommon c;
    FW_CUDA(cudaMalloc(&c.silu, 65536 * sizeof(uint16_t)));
    FW_CUDA(cudaMalloc(&c.sigmoid, 65536 * sizeof(uint16_t)));
    FW_CUDA(cudaMalloc(&c.err, sizeof(int)));
    FW_CUDA(upload(c.silu, silu.data(), 65536 * sizeof(uint16_t), cudaStreamLegacy));
    FW_CUDA(upload(c.sigmoid, sig.data(), 65536 * sizeof(uint16_t), cudaStreamLegacy));
    FW_CUDA(zero_fill(c.err, sizeof(int), cudaStreamLegacy));
    it = g_common.emplace(device, c).first;
  }
  *out = &it->second;
  return FW_OK;
}

int map_device_error(int code) {
  switch (code) {
    case fw::kErrNone: return FW_OK;
    case fw::kErrNanLogits: return fail(FW_ENAN, "router received NaN logits");
    case fw::kErrTimeout: return fail(FW_ETIMEOUT, "a bounded device wait timed out");
    case fw::kErrBadIndex: return fail(FW_EINVAL, "expert index out of range on device");
    case fw::kErrCapacity: return fail(FW_EINVAL, "token/expert pairs exceeded scratch capacity");
    case fw::kErrPeer: return fail(FW_ENCCL, "an expert-parallel peer reported a failure in this forward");
    default: return fail(FW_ECUDA, "unknown device status " + std::to_string(code));
  }
}

// SplitMix64 keyed stream (Steele, Lea, Flood 2014); the device kernel
// applies the same finaliser per element.
uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
constexpr uint64_t kGamma = 0x9E3779B97F4A7C15ull;
uint64_t synth_key(uint64_t seed, uint32_t tensor) {
  return mix64(mix64(seed + kGamma) + static_cast<uint64_t>(tensor) * kGamma + kGamma);
}
float synth_scale(float std_dev) {
  const double sd = std::sqrt((65536.0 * 65536.0 - 1.0) / 3.0);
  return static_cast<float>(static_cast<double>(std_dev) / sd);
}

struct OwnedLayer {
  fw::LayerWeights w;
  std::vector<void*> owned;
  bool loaded = false;
  bool prefill = false;           // tensor maps below are valid
  fw::PrefillWeightMaps maps{};   // the tiled banks as tensor-core operands
  fw::HcWeights hc{};             // hyper-connection weights (fw_moe_load_hc)
  std::vector<void*> hc_owned;
};

}  // namespace

namespace fw {
int record_error(int code, const char* msg) { return fail(code, msg); }
}  // namespace fw

// Widest forward the decode kernels take; wider ones use the prefill path.
constexpr int kDecodeMaxTokens = 256;
// Default width from which a shape with a prefill path takes it.  Measured on
// one B200 at config 0 (8 layers, uniform router, token-layers/s decode ->
// tensor-core path): T = 64: 165 k -> 154 k; T = 96: 199 k -> 205 k;
// T = 128: 221 k -> 254 k; T = 192: 250 k -> 360 k; T = 256: 272 k -> 468 k.
// Two tokens per expert (T * K / E) is where the CUDA-core dot products stop
// hiding under the weight stream.
// Under expert parallelism the same default applies to the total over the
// ranks: the config-1 stack at 2 x 64 tokens measured 314 k token-layers/s
// on the decode path and 380 k on the tensor-core path.
constexpr int kPrefillDefaultMin = 96;
constexpr int kMaxTokens = 16384;

struct fw_moe {
  fw_moe_config cfg{};
  int device = 0;
  fw::Shape shape{};
  std::vector<OwnedLayer> layers;
  fw::Luts luts{};
  uint16_t* silu = nullptr;
  uint16_t* sigmoid = nullptr;
  fw::Scratch sc{};
  std::vector<void*> scratch_owned;
  uint16_t* x_dev = nullptr;
  uint16_t* y_dev = nullptr;
  int32_t* idx_dev = nullptr;
  uint16_t* score_dev = nullptr;
  cudaStream_t stream = nullptr;
  uint64_t bytes = 0;
  bool profile = false;
  cudaEvent_t stage_ev[fw::kStages + 1] = {};
  bool prefill_ok = false;            // shape supported and scratch maps built
  fw::PrefillScratchMaps pf_maps{};
  int prefill_min_tokens = kDecodeMaxTokens + 1;  // forwards this wide or wider take the prefill path
  // The last forward (fw_moe_last_union): 0 none, 1 decode (expert schedule),
  // 2 prefill (grouped pair offsets over `last_experts` bank experts).
  int last_path = 0, last_experts = 0;
  cudaStream_t last_stream = nullptr;
  // Expert parallelism (fw_moe_ep_init): this rank's expert range, the NCCL
  // communicator and the exchange buffers (world * max_tokens tokens).
  fw::EpComm* ep = nullptr;
  int ep_rank = 0, ep_world = 1;
  uint16_t* ep_x_all = nullptr;      // [world*M][H] gathered token rows
  int32_t* ep_idx_all = nullptr;     // [world*M][K] gathered top-k ids
  uint16_t* ep_score_all = nullptr;  // [world*M][K] gathered route weights
  uint16_t* ep_recv = nullptr;       // weighted rows of this rank's tokens, per source
  int ep_decode_max = 0;             // widest forward the expert-parallel decode path takes
  // expert-parallel prefill: packed exchange positions and counts
  int32_t* ep_send_pos = nullptr;    // [world*M*K]
  int32_t* ep_recv_pos = nullptr;    // [M*K]
  int* ep_counts = nullptr;          // device [4][world]: send rows, send offsets, recv rows, recv offsets
  int* ep_counts_host = nullptr;     // pinned copy
  cudaEvent_t ep_counts_ev = nullptr;
  // Expert parallelism over NVLink peer memory (the default transport).
  int ep_transport = FW_EP_TRANSPORT_P2P;
  fw::P2pComm* p2p = nullptr;
  unsigned ep_seq = 0;               // forwards issued under expert parallelism (same on every rank)
  int stall_next = 0;                // fw_moe_test_stall: the next forward's expert kernel stalls
  // hyper-connection caller (allocated by the first fw_moe_load_hc)
  fw::HcScratch hs{};
  int hs_lowrank = 0;                // LR the scratch holds
  uint16_t* hc_moe = nullptr;        // [M][H] block output inside a hyper-connection forward
  uint16_t* hc_post_dev = nullptr;   // [M][4H] staging for fw_moe_forward_hc (host buffers)
  uint16_t* hc_out_dev = nullptr;    // [M][4H]
};

namespace fw {
HandlePlace handle_place(const fw_moe* h) { return HandlePlace{h->device, h->ep_rank, h->ep_world}; }
}  // namespace fw


namespace {

template <typename T>
int alloc(fw_moe* h, T** p, size_t count, std::vector<void*>& owned) {
  void* v = nullptr;
  FW_CUDA(cudaMalloc(&v, count * sizeof(T) > 0 ? count * sizeof(T) : 16));
  owned.push_back(v);
  h->bytes += count * sizeof(T);
  *p = static_cast<T*>(v);
  return FW_OK;
}

#define FW_TRY(call)            \
  do {                          \
    const int rc_ = (call);     \
    if (rc_ != FW_OK) return rc_; \
  } while (0)

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

int check_config(const fw_moe_config* c) {
  if (c == nullptr) return fail(FW_EINVAL, "config is null");
  if (c->hidden <= 0 || c->hidden % 64 != 0 || c->hidden > 4096)
    return fail(FW_EINVAL, "hidden must be a positive multiple of 64, at most 4096");
  if (c->intermediate <= 0 || c->intermediate % 64 != 0 || c->shared_intermediate <= 0 ||
      c->shared_intermediate % 64 != 0 || c->intermediate > 4096 || c->shared_intermediate > 4096)
    return fail(FW_EINVAL, "intermediate sizes must be positive multiples of 64, at most 4096");
  if (c->experts <= 0 || c->experts % 32 != 0 || c->experts > 1024)
    return fail(FW_EINVAL, "experts must be a multiple of 32, at most 1024");
  if (c->top_k < 1 || c->top_k > 32 || c->top_k > c->experts)
    return fail(FW_EINVAL, "top_k must be in [1, min(32, experts)]");
  if (c->max_tokens < 1 || c->max_tokens > kMaxTokens)
    return fail(FW_EINVAL, "max_tokens must be in [1, 16384]");
  if (c->max_tokens > kDecodeMaxTokens &&
      !fw::prefill_supported(fw::Shape{c->hidden, c->intermediate, c->shared_intermediate, c->experts, c->top_k}))
    return fail(FW_EINVAL, "max_tokens above 256 needs hidden a multiple of 256 and 2*intermediate sizes multiples of 128");
  if (c->layers < 1) return fail(FW_EINVAL, "layers must be >= 1");
  // shared memory of the GEMV stages: 8 tokens x cols x f32
  if (8ull * c->hidden * 4 > 200 * 1024) return fail(FW_EINVAL, "hidden too large for staging");
  return FW_OK;
}

int check_handle(const fw_moe* h, int32_t layer) {
  if (h == nullptr) return fail(FW_EINVAL, "handle is null");
  if (layer < 0 || layer >= h->cfg.layers) return fail(FW_EINVAL, "layer out of range");
  if (!h->layers[layer].loaded) return fail(FW_EINVAL, "layer not loaded");
  return FW_OK;
}

// Experts this handle holds: all of them, or under expert parallelism those
// e with e % world == rank (bank index e / world).  Interleaving spreads a
// skewed router's hot low-id experts over the GPUs.
int held_experts(const fw_moe* h) { return h->cfg.experts / h->ep_world; }

// The router's per-layer tables (row-norm bounds for the prefill router,
// the partial-major copy both routers read), stream-ordered after the router
// weights and the shared gate vector; hidden sizes that are not a multiple
// of 256 use the other decode router and have no prefill path.
int router_tables(fw_moe* h, OwnedLayer& L) {
  if (h->cfg.hidden % 256 != 0) return FW_OK;  // the decode router's 16-byte chunks and the prefill path need it
  const size_t E = h->cfg.experts, H = h->cfg.hidden;
  float* norms = nullptr;
  uint16_t* pm = nullptr;
  FW_TRY(alloc(h, &norms, E, L.owned));
  FW_TRY(alloc(h, &pm, (E + 1) * H, L.owned));
  FW_CUDA(fw::launch_router_tables(L.w.router, L.w.sh_gate_w, static_cast<int>(E), static_cast<int>(H), norms, pm,
                                   h->stream));
  L.w.router_norm = norms;
  L.w.router_pm = pm;
  return FW_OK;
}

int free_layer(OwnedLayer& L) {
  for (void* p : L.owned) cudaFree(p);
  L.owned.clear();
  L.w = fw::LayerWeights{};
  L.loaded = false;
  return FW_OK;
}

}  // namespace

namespace {

// Stage events of a forward (kStages + 1 of them), or null.
struct Marks {
  cudaEvent_t* ev;
  cudaStream_t st;
  cudaError_t operator()(int i) const { return ev != nullptr ? cudaEventRecord(ev[i], st) : cudaSuccess; }
};

// The next layer's weights that do not depend on its input (router rows in
// the partial-major copy its router reads, shared expert tiles), for the
// decode expert kernel to prefetch into L2 when its work is done: decode
// forwards usually run the layers in order.
void prefetch_next(const fw_moe* h, int layer, fw::Scratch* sc) {
  if (layer + 1 >= h->cfg.layers) return;
  const OwnedLayer& n = h->layers[layer + 1];
  if (!n.loaded || !n.w.tiled) return;
  const unsigned long long H = h->cfg.hidden, E = h->cfg.experts, Is = h->cfg.shared_intermediate;
  sc->prefetch[0] = n.w.router_pm != nullptr ? static_cast<const void*>(n.w.router_pm) : n.w.router;
  sc->prefetch_bytes[0] = (n.w.router_pm != nullptr ? E + 1 : E) * H * 2;
  sc->prefetch[1] = n.w.sh_gate;  // tiled gate/up
  sc->prefetch_bytes[1] = 2 * Is * H * 2;
  sc->prefetch[2] = n.w.sh_down;
  sc->prefetch_bytes[2] = H * Is * 2;
}

// The expert kernel's stall count for this forward (fw_moe_test_stall).
int take_stall(fw_moe* h) {
  const int v = h->stall_next;
  h->stall_next = 0;
  return v;
}

// One layer under expert parallelism over NCCL, stream-ordered (see
// fw_ep.cu): local router and route, dispatch (all-gather), this rank's
// experts over every rank's tokens plus the shared expert over its own,
// combine exchange, then the ascending-id sum of its own tokens' rows.
int ep_forward_nccl(fw_moe* h, const OwnedLayer& L, const uint16_t* x, int T_l, uint16_t* y, int32_t* idx,
                    uint16_t* score, cudaStream_t cs, cudaEvent_t* ev, const fw::HcPost* hc) {
  const fw::Shape& s = h->shape;
  const int N = h->ep_world, T = N * T_l;
  cudaError_t e = cudaSuccess;
  const Marks mark{ev, cs};
  auto cuda_failed = [&](const char* what) { return fail(FW_ECUDA, what, cudaGetErrorString(e)); };
  if ((e = mark(0)) != cudaSuccess) return cuda_failed("event");
  if ((e = fw::launch_router(s, L.w, h->sc, x, T_l, cs)) != cudaSuccess) return cuda_failed("router launch");
  if ((e = mark(1)) != cudaSuccess) return cuda_failed("event");
  if ((e = fw::launch_route_block(s, h->luts, h->sc, T_l, idx, score, false, nullptr, cs)) != cudaSuccess)
    return cuda_failed("route launch");
  if ((e = mark(2)) != cudaSuccess) return cuda_failed("event");
  const char* m = fw::ep_dispatch(h->ep, x, h->ep_x_all, static_cast<size_t>(T_l) * s.H, idx, h->ep_idx_all,
                                  score, h->ep_score_all, static_cast<size_t>(T_l) * s.K, cs);
  if (m != nullptr) return fail(FW_ENCCL, m);
  if ((e = fw::launch_ep_schedule(s, h->sc, h->ep_idx_all, T, h->ep_rank, N, T_l, cs)) != cudaSuccess)
    return cuda_failed("schedule launch");
  if ((e = mark(3)) != cudaSuccess) return cuda_failed("event");
  fw::Scratch sc = h->sc;
  sc.stall = take_stall(h);
  if ((e = fw::launch_experts(s, L.w, h->luts, sc, h->ep_x_all, T, h->ep_score_all, cs, x, T_l)) != cudaSuccess)
    return cuda_failed("expert kernel launch");
  if ((e = mark(4)) != cudaSuccess) return cuda_failed("event");
  m = fw::ep_combine_exchange(h->ep, h->sc.weighted, h->ep_recv, static_cast<size_t>(T_l) * s.K * s.H, cs);
  if (m != nullptr) return fail(FW_ENCCL, m);
  if ((e = fw::launch_combine(s, h->sc, T_l, y, cs, idx, N, h->ep_recv, nullptr, hc)) != cudaSuccess)
    return cuda_failed("combine launch");
  if ((e = mark(5)) != cudaSuccess) return cuda_failed("event");
  return FW_OK;
}

// One layer of the prefill path under expert parallelism over NCCL: local
// router and route, dispatch (all-gather), this rank's experts grouped over
// every rank's pairs and run as the tensor-core GEMMs (plus the shared
// expert over its own tokens), the weighted rows packed per destination in
// (token, k) order, a row-sized exchange (counts read on the host while the
// GEMMs run), then the owner's ascending-id sum.
int ep_prefill_forward_nccl(fw_moe* h, const OwnedLayer& L, const uint16_t* x, int T_l, uint16_t* y, int32_t* idx,
                            uint16_t* score, cudaStream_t cs, cudaEvent_t* ev, const fw::HcPost* hc) {
  const fw::Shape& s = h->shape;
  const int N = h->ep_world, T = N * T_l;
  const int count = held_experts(h);
  cudaError_t e = cudaSuccess;
  const Marks mark{ev, cs};
  auto cuda_failed = [&](const char* what) { return fail(FW_ECUDA, what, cudaGetErrorString(e)); };
  if ((e = mark(0)) != cudaSuccess) return cuda_failed("event");
  if ((e = fw::launch_prefill_front(s, L.w, L.maps, h->luts, h->sc, x, T_l, idx, score, false, cs,
                                    ev != nullptr ? ev[1] : nullptr)) != cudaSuccess)
    return cuda_failed("router / route launch");
  if ((e = mark(2)) != cudaSuccess) return cuda_failed("event");
  const char* m = fw::ep_dispatch(h->ep, x, h->ep_x_all, static_cast<size_t>(T_l) * s.H, idx, h->ep_idx_all,
                                  score, h->ep_score_all, static_cast<size_t>(T_l) * s.K, cs);
  if (m != nullptr) return fail(FW_ENCCL, m);
  if ((e = fw::launch_prefill_group(s, h->sc, h->ep_idx_all, T * s.K, h->ep_x_all, h->ep_rank, N, count, T_l, true,
                                    cs)) !=
      cudaSuccess)
    return cuda_failed("grouping launch");
  int* cnt = h->ep_counts;
  if ((e = fw::launch_ep_positions(h->ep_idx_all, T * s.K, T_l * s.K, h->ep_rank, N, false, h->ep_send_pos,
                                   cnt, cnt + N, cs)) != cudaSuccess ||
      (e = fw::launch_ep_positions(idx, T_l * s.K, T_l * s.K, h->ep_rank, N, true, h->ep_recv_pos, cnt + 2 * N,
                                   cnt + 3 * N, cs)) != cudaSuccess)
    return cuda_failed("exchange positions launch");
  if ((e = cudaMemcpyAsync(h->ep_counts_host, cnt, 4 * N * sizeof(int), cudaMemcpyDeviceToHost, cs)) != cudaSuccess ||
      (e = cudaEventRecord(h->ep_counts_ev, cs)) != cudaSuccess)
    return cuda_failed("exchange counts");
  if ((e = mark(3)) != cudaSuccess) return cuda_failed("event");
  if ((e = fw::launch_prefill_gemms(s, L.maps, h->pf_maps, h->luts, h->sc, x, T_l, count, h->ep_score_all,
                                    h->ep_send_pos, h->sc.weighted, cs)) != cudaSuccess)
    return cuda_failed("GEMM launch");
  if ((e = mark(4)) != cudaSuccess) return cuda_failed("event");
  // The GEMMs keep running while the host reads the exchange sizes.
  if ((e = cudaEventSynchronize(h->ep_counts_ev)) != cudaSuccess) return cuda_failed("exchange counts");
  const int* hc_ = h->ep_counts_host;
  m = fw::ep_exchange_rows(h->ep, h->sc.weighted, hc_, hc_ + N, h->ep_recv, hc_ + 2 * N, hc_ + 3 * N,
                           static_cast<size_t>(s.H), cs);
  if (m != nullptr) return fail(FW_ENCCL, m);
  if ((e = fw::launch_combine(s, h->sc, T_l, y, cs, nullptr, 0, h->ep_recv, h->ep_recv_pos, hc)) != cudaSuccess)
    return cuda_failed("combine launch");
  if ((e = mark(5)) != cudaSuccess) return cuda_failed("event");
  return FW_OK;
}

// One layer under expert parallelism over NVLink peer memory (fw_p2p.cu),
// decode widths: router and route of this rank's tokens; publish them in
// its window; pull every rank's selections and the token rows this rank's
// experts need (bounded wait on the peers' pub flags); schedule; the
// decode expert kernel, whose epilogue stores each weighted row in its
// owner's window and whose last CTA sets this rank's done flags; the
// combine (bounded wait on every done flag) over this rank's window.
int ep_forward_p2p(fw_moe* h, const OwnedLayer& L, const uint16_t* x, int T_l, uint16_t* y, int32_t* idx,
                   uint16_t* score, cudaStream_t cs, cudaEvent_t* ev, const fw::HcPost* hc) {
  const fw::Shape& s = h->shape;
  const int N = h->ep_world, T = N * T_l;
  const fw::EpPeers P = fw::p2p_peers(h->p2p, T_l, ++h->ep_seq, h->sc.wait_ns);
  cudaError_t e = cudaSuccess;
  const Marks mark{ev, cs};
  auto cuda_failed = [&](const char* what) { return fail(FW_ECUDA, what, cudaGetErrorString(e)); };
  if ((e = mark(0)) != cudaSuccess) return cuda_failed("event");
  if ((e = fw::launch_router(s, L.w, h->sc, x, T_l, cs)) != cudaSuccess) return cuda_failed("router launch");
  if ((e = mark(1)) != cudaSuccess) return cuda_failed("event");
  if ((e = fw::launch_route_block(s, h->luts, h->sc, T_l, idx, score, false, nullptr, cs)) != cudaSuccess ||
      (e = fw::launch_ep_publish(P, x, idx, score, h->sc.err, cs)) != cudaSuccess)
    return cuda_failed("route / publish launch");
  if ((e = mark(2)) != cudaSuccess) return cuda_failed("event");
  if ((e = fw::launch_ep_pull(P, s.E, h->ep_idx_all, h->ep_score_all, h->ep_x_all, h->sc.err, cs)) != cudaSuccess ||
      (e = fw::launch_ep_schedule(s, h->sc, h->ep_idx_all, T, h->ep_rank, N, T_l, cs)) != cudaSuccess)
    return cuda_failed("dispatch launch");
  if ((e = mark(3)) != cudaSuccess) return cuda_failed("event");
  fw::Scratch sc = h->sc;
  sc.stall = take_stall(h);
  if ((e = fw::launch_experts(s, L.w, h->luts, sc, h->ep_x_all, T, h->ep_score_all, cs, x, T_l, &P)) != cudaSuccess)
    return cuda_failed("expert kernel launch");
  if ((e = mark(4)) != cudaSuccess) return cuda_failed("event");
  if ((e = fw::launch_combine(s, h->sc, T_l, y, cs, nullptr, 0, fw::p2p_recv(h->p2p), nullptr, hc, &P)) !=
      cudaSuccess)
    return cuda_failed("combine launch");
  if ((e = mark(5)) != cudaSuccess) return cuda_failed("event");
  return FW_OK;
}

// The same over peer memory at prefill widths: router and route, publish;
// every rank's selections and this rank's pair counts (bounded wait on the
// pub flags); pair offsets; the grouped input, each needed token row read
// once from its owner's window; the tensor-core GEMMs, whose down epilogue
// stores each weighted row in its owner's window (the transfer overlaps the
// GEMM) and whose last CTA sets the done flags; the combine.  No host
// synchronisation.
int ep_prefill_forward_p2p(fw_moe* h, const OwnedLayer& L, const uint16_t* x, int T_l, uint16_t* y, int32_t* idx,
                           uint16_t* score, cudaStream_t cs, cudaEvent_t* ev, const fw::HcPost* hc) {
  const fw::Shape& s = h->shape;
  const int count = held_experts(h);
  const fw::EpPeers P = fw::p2p_peers(h->p2p, T_l, ++h->ep_seq, h->sc.wait_ns);
  cudaError_t e = cudaSuccess;
  const Marks mark{ev, cs};
  auto cuda_failed = [&](const char* what) { return fail(FW_ECUDA, what, cudaGetErrorString(e)); };
  if ((e = mark(0)) != cudaSuccess) return cuda_failed("event");
  if ((e = fw::launch_prefill_front(s, L.w, L.maps, h->luts, h->sc, x, T_l, idx, score, false, cs,
                                    ev != nullptr ? ev[1] : nullptr)) != cudaSuccess ||
      (e = fw::launch_ep_publish(P, x, idx, score, h->sc.err, cs)) != cudaSuccess)
    return cuda_failed("router / route / publish launch");
  if ((e = mark(2)) != cudaSuccess) return cuda_failed("event");
  if ((e = cudaMemsetAsync(h->sc.pair_count, 0, sizeof(int) * count, cs)) != cudaSuccess ||
      (e = fw::launch_ep_ids(P, s.E, h->ep_idx_all, h->ep_score_all, h->sc.pair_count, h->sc.err, cs)) !=
          cudaSuccess ||
      (e = fw::launch_prefill_offsets(s, h->sc, count, T_l, cs)) != cudaSuccess ||
      (e = fw::launch_ep_scatter(P, count, h->ep_idx_all, h->sc.pair_offset, h->sc.pair_fill, h->sc.pair_tk,
                                 h->sc.xg, h->sc.pair_cap, h->sc.err, cs)) != cudaSuccess)
    return cuda_failed("dispatch launch");
  if ((e = mark(3)) != cudaSuccess) return cuda_failed("event");
  if ((e = fw::launch_prefill_gemms(s, L.maps, h->pf_maps, h->luts, h->sc, x, T_l, count, h->ep_score_all, nullptr,
                                    h->sc.weighted, cs, &P)) != cudaSuccess)
    return cuda_failed("GEMM launch");
  if ((e = mark(4)) != cudaSuccess) return cuda_failed("event");
  if ((e = fw::launch_combine(s, h->sc, T_l, y, cs, nullptr, 0, fw::p2p_recv(h->p2p), nullptr, hc, &P)) !=
      cudaSuccess)
    return cuda_failed("combine launch");
  if ((e = mark(5)) != cudaSuccess) return cuda_failed("event");
  return FW_OK;
}

// Whole block under expert parallelism (either transport, either path).
int ep_block(fw_moe* h, const OwnedLayer& L, const uint16_t* x, int T_l, uint16_t* y, int32_t* idx, uint16_t* score,
             cudaStream_t cs, cudaEvent_t* ev, const fw::HcPost* hc, bool* prefill) {
  // The experts of a rank see every rank's tokens: the width that decides
  // the path is the total over the ranks.
  *prefill = T_l > h->ep_decode_max ||
             (L.prefill && static_cast<int64_t>(T_l) * h->ep_world >= h->prefill_min_tokens);
  if (*prefill && !L.prefill) return fail(FW_EINVAL, "this many tokens need the prefill path, which this handle's shape lacks");
  if (h->p2p != nullptr)
    return *prefill ? ep_prefill_forward_p2p(h, L, x, T_l, y, idx, score, cs, ev, hc)
                    : ep_forward_p2p(h, L, x, T_l, y, idx, score, cs, ev, hc);
  if (*prefill && h->ep_send_pos == nullptr)
    return fail(FW_EINVAL, "this many tokens need the prefill path, which this handle's shape lacks");
  return *prefill ? ep_prefill_forward_nccl(h, L, x, T_l, y, idx, score, cs, ev, hc)
                  : ep_forward_nccl(h, L, x, T_l, y, idx, score, cs, ev, hc);
}

// Replace a scratch buffer owned by the handle with one of `count` elements.
template <typename T>
int regrow(fw_moe* h, T** p, size_t count) {
  auto& o = h->scratch_owned;
  for (size_t i = 0; i < o.size(); ++i)
    if (o[i] == static_cast<void*>(*p)) {
      cudaFree(o[i]);
      o.erase(o.begin() + static_cast<long>(i));
      break;
    }
  *p = nullptr;
  return alloc(h, p, count, o);
}

}  // namespace

extern "C" {

int fw_ep_unique_id(uint8_t id[128]) {
  if (id == nullptr) return fail(FW_EINVAL, "id is null");
  const char* m = fw::ep_unique_id(id);
  return m == nullptr ? FW_OK : fail(FW_ENCCL, m);
}

int fw_moe_ep_set_transport(fw_moe* h, int32_t transport) {
  if (h == nullptr) return fail(FW_EINVAL, "handle is null");
  if (transport != FW_EP_TRANSPORT_P2P && transport != FW_EP_TRANSPORT_NCCL)
    return fail(FW_EINVAL, "unknown expert-parallel transport");
  if (h->ep != nullptr || h->p2p != nullptr) return fail(FW_EINVAL, "expert parallelism is already initialised");
  h->ep_transport = transport;
  return FW_OK;
}

int fw_moe_ep_init(fw_moe* h, int32_t rank, int32_t world, const uint8_t id[128]) {
  if (h == nullptr || id == nullptr) return fail(FW_EINVAL, "handle / id is null");
  if (h->ep != nullptr || h->p2p != nullptr) return fail(FW_EINVAL, "expert parallelism is already initialised");
  if (world < 2 || world > 8 || rank < 0 || rank >= world)
    return fail(FW_EINVAL, "need 2 <= world <= 8 and 0 <= rank < world");
  if (h->cfg.experts % world != 0) return fail(FW_EINVAL, "experts must divide evenly over the ranks");
  for (const auto& L : h->layers)
    if (L.loaded) return fail(FW_EINVAL, "initialise expert parallelism before loading layers");
  FW_CUDA(cudaSetDevice(h->device));
  const bool p2p = h->ep_transport == FW_EP_TRANSPORT_P2P;
  const size_t M = h->cfg.max_tokens, W = static_cast<size_t>(world);
  // Decode width under expert parallelism: the schedule spans every rank's
  // tokens and is built by one CTA (at most 1024 tokens in total).
  const size_t Md = std::min<size_t>(std::min<size_t>(M, kDecodeMaxTokens), 1024 / W);
  // Prefill buffers whenever the shape has the path: fw_moe_set_prefill_min_tokens
  // can send any width there.
  const bool prefill = h->prefill_ok;
  const size_t K = h->cfg.top_k, H = h->cfg.hidden, I = h->cfg.intermediate, E = h->cfg.experts;
  fw::Scratch& s = h->sc;
  // Schedule and activations cover every rank's tokens; the rest of the
  // scratch stays per rank.  Over NCCL the outgoing weighted rows do too;
  // over peer memory they go straight to their owners' windows.
  const size_t Gd = W * Md, Gp = prefill ? W * M : 0;
  FW_TRY(regrow(h, &s.sched, fw::sched_words(static_cast<int>(E), static_cast<int>(Gd), static_cast<int>(K))));
  FW_TRY(regrow(h, &s.act, std::max(Gd * K * 2 * I, Gp * K * I)));
  if (!p2p) FW_TRY(regrow(h, &s.weighted, std::max(Gd * K * H, Gp * K * H)));
  // Gathered rows: decode widths only over peer memory (prefill rows go
  // straight from the owners' windows into the grouped input).
  FW_TRY(alloc(h, &h->ep_x_all, (p2p ? Gd : W * M) * H, h->scratch_owned));
  FW_TRY(alloc(h, &h->ep_idx_all, W * M * K, h->scratch_owned));
  FW_TRY(alloc(h, &h->ep_score_all, W * M * K, h->scratch_owned));
  if (!p2p) FW_TRY(alloc(h, &h->ep_recv, std::max(Gd * K * H, prefill ? M * K * H : 0), h->scratch_owned));
  if (prefill) {
    FW_TRY(regrow(h, &s.pair_tk, Gp * K));
    FW_TRY(regrow(h, &s.xg, Gp * K * H));
    s.pair_cap = static_cast<long long>(Gp * K);
    if (!p2p) {
      FW_TRY(alloc(h, &h->ep_send_pos, Gp * K, h->scratch_owned));
      FW_TRY(alloc(h, &h->ep_recv_pos, M * K, h->scratch_owned));
      FW_TRY(alloc(h, &h->ep_counts, 4 * W, h->scratch_owned));
      FW_CUDA(cudaMallocHost(&h->ep_counts_host, 4 * W * sizeof(int)));
      FW_CUDA(cudaEventCreateWithFlags(&h->ep_counts_ev, cudaEventDisableTiming));
    }
  }
  // act / xg moved: re-encode the scratch tensor maps
  if (h->prefill_ok && !fw::make_prefill_scratch_maps(h->shape, s, &h->pf_maps))
    return fail(FW_ECUDA, "prefill tensor maps could not be encoded");
  if (p2p) {
    fw::P2pComm* c = nullptr;
    const char* m = fw::p2p_init(h->device, rank, world, id, static_cast<int>(M), static_cast<int>(H),
                                 static_cast<int>(K), &c);
    if (m != nullptr) return fail(FW_ENCCL, m);
    h->p2p = c;
    h->bytes += fw::p2p_window_bytes(c);
  } else {
    fw::EpComm* c = nullptr;
    const char* m = fw::ep_comm_init(rank, world, id, &c);
    if (m != nullptr) return fail(FW_ENCCL, m);
    h->ep = c;
  }
  h->ep_rank = rank;
  h->ep_world = world;
  h->ep_decode_max = static_cast<int>(Md);
  return FW_OK;
}

int fw_moe_set_wait_limit(fw_moe* h, uint64_t nanoseconds) {
  if (h == nullptr) return fail(FW_EINVAL, "handle is null");
  if (nanoseconds < 1000000ull || nanoseconds > 60000000000ull)
    return fail(FW_EINVAL, "the wait limit must be between 1 ms and 60 s");
  h->sc.wait_ns = nanoseconds;
  return FW_OK;
}

int fw_moe_test_stall(fw_moe* h) {
  if (h == nullptr) return fail(FW_EINVAL, "handle is null");
  h->stall_next = 1 << 30;
  return FW_OK;
}

const char* fw_last_error(void) { return g_last_error; }

int fw_moe_create(const fw_moe_config* config, int device, fw_moe** out) {
  if (out == nullptr) return fail(FW_EINVAL, "out is null");
  *out = nullptr;
  FW_TRY(check_config(config));
  int ndev = 0;
  FW_CUDA(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return fail(FW_EINVAL, "device out of range");
  FW_CUDA(cudaSetDevice(device));
  fw_moe* h = new fw_moe();
  h->cfg = *config;
  h->device = device;
  h->shape = fw::Shape{config->hidden, config->intermediate, config->shared_intermediate,
                       config->experts, config->top_k};
  h->layers.resize(config->layers);
  const int M = config->max_tokens, K = config->top_k, E = config->experts;
  const int H = config->hidden, I = config->intermediate, Is = config->shared_intermediate;
  auto& o = h->scratch_owned;
  int rc = FW_OK;
  do {
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) {
      rc = fail(FW_ECUDA, "stream creation failed");
      break;
    }
    std::vector<uint16_t> silu, sig;
    build_tables(silu, sig);
    if ((rc = alloc(h, &h->silu, 65536, o)) != FW_OK) break;
    if ((rc = alloc(h, &h->sigmoid, 65536, o)) != FW_OK) break;
    if (upload(h->silu, silu.data(), 65536 * 2, h->stream) != cudaSuccess ||
        upload(h->sigmoid, sig.data(), 65536 * 2, h->stream) != cudaSuccess) {
      rc = fail(FW_ECUDA, "table upload failed");
      break;
    }
    h->luts = fw::Luts{h->silu, h->sigmoid};
    fw::Scratch& s = h->sc;
    s.max_T = M;
    if ((rc = alloc(h, &s.logits, static_cast<size_t>(M) * E, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.sh_logit, M, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.sh_sig, M, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.sorted_slot, static_cast<size_t>(M) * K, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.sched, fw::sched_words(E, M, K), o)) != FW_OK) break;
    if ((rc = alloc(h, &s.act, static_cast<size_t>(M) * K * 2 * I, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.act_sh, static_cast<size_t>(M) * 2 * Is, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.weighted, static_cast<size_t>(M) * K * H, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.gated_sh, static_cast<size_t>(M) * H, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.up_done, static_cast<size_t>(E) + 1, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.ticket, 1, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.err, 1, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.pair_count, E, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.pair_fill, E, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.pair_offset, static_cast<size_t>(E) + 1, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.unit_prefix, 4 * (static_cast<size_t>(E) + 2), o)) != FW_OK) break;
    if ((rc = alloc(h, &s.pair_tk, static_cast<size_t>(M) * K, o)) != FW_OK) break;
    if ((rc = alloc(h, &s.xg, static_cast<size_t>(M) * K * H, o)) != FW_OK) break;
    s.pair_cap = static_cast<long long>(M) * K;
    if (fw::prefill_supported(h->shape) &&
        (rc = alloc(h, &s.router_approx, static_cast<size_t>(M) * E, o)) != FW_OK)
      break;
    if ((rc = alloc(h, &h->x_dev, static_cast<size_t>(M) * H, o)) != FW_OK) break;
    if ((rc = alloc(h, &h->y_dev, static_cast<size_t>(M) * H, o)) != FW_OK) break;
    if ((rc = alloc(h, &h->idx_dev, static_cast<size_t>(M) * K, o)) != FW_OK) break;
    if ((rc = alloc(h, &h->score_dev, static_cast<size_t>(M) * K, o)) != FW_OK) break;
    if (zero_fill(s.err, sizeof(int), h->stream) != cudaSuccess ||
        zero_fill(s.ticket, sizeof(int), h->stream) != cudaSuccess ||
        zero_fill(s.pair_count, sizeof(int) * E, h->stream) != cudaSuccess ||
        zero_fill(s.pair_fill, sizeof(int) * E, h->stream) != cudaSuccess) {
      rc = fail(FW_ECUDA, "status reset failed");
      break;
    }
    h->prefill_ok = fw::prefill_supported(h->shape) && fw::make_prefill_scratch_maps(h->shape, s, &h->pf_maps);
    if (h->prefill_ok) h->prefill_min_tokens = kPrefillDefaultMin;
    if (M > kDecodeMaxTokens && !h->prefill_ok) {
      rc = fail(FW_ECUDA, "prefill tensor maps could not be encoded");
      break;
    }
  } while (false);
  if (rc != FW_OK) {
    fw_moe_destroy(h);
    return rc;
  }
  *out = h;
  return FW_OK;
}

int fw_moe_get_config(const fw_moe* h, fw_moe_config* out) {
  if (h == nullptr || out == nullptr) return fail(FW_EINVAL, "null argument");
  *out = h->cfg;
  return FW_OK;
}

int fw_moe_destroy(fw_moe* h) {
  if (h == nullptr) return FW_OK;
  cudaSetDevice(h->device);
  if (h->ep != nullptr && h->stream) {
    // a collective a peer never joined must not hold the teardown
    cudaError_t ce = cudaSuccess;
    fw::ep_bounded_sync(h->ep, h->stream, 2 * h->sc.wait_ns, &ce);
  }
  fw::ep_comm_destroy(h->ep);
  if (h->stream) cudaStreamSynchronize(h->stream);
  fw::p2p_destroy(h->p2p);
  if (h->ep_counts_host) cudaFreeHost(h->ep_counts_host);
  if (h->ep_counts_ev) cudaEventDestroy(h->ep_counts_ev);
  for (auto& L : h->layers) {
    free_layer(L);
    for (void* p : L.hc_owned) cudaFree(p);
  }
  for (void* p : h->scratch_owned) cudaFree(p);
  if (h->stream) cudaStreamDestroy(h->stream);
  for (auto& ev : h->stage_ev)
    if (ev) cudaEventDestroy(ev);
  delete h;
  return FW_OK;
}

int fw_moe_load_layer(fw_moe* h, int32_t layer, const uint16_t* router, const uint16_t* gate_up,
                      const uint16_t* down, const uint16_t* shared_gate, const uint16_t* shared_up,
                      const uint16_t* shared_down, const uint16_t* shared_gate_w,
                      const float* logit_bias) {
  if (h == nullptr) return fail(FW_EINVAL, "handle is null");
  if (layer < 0 || layer >= h->cfg.layers) return fail(FW_EINVAL, "layer out of range");
  if (!router || !gate_up || !down || !shared_gate || !shared_up || !shared_down || !shared_gate_w)
    return fail(FW_EINVAL, "a weight pointer is null");
  FW_CUDA(cudaSetDevice(h->device));
  OwnedLayer& L = h->layers[layer];
  free_layer(L);
  const size_t H = h->cfg.hidden, I = h->cfg.intermediate, Is = h->cfg.shared_intermediate;
  const size_t E = h->cfg.experts;
  // Router and shared gate vector keep the reference layout.
  struct Item {
    const void* src;
    size_t count;
    const uint16_t** dst;
  } items[] = {
      {router, E * H, &L.w.router},
      {shared_gate_w, H, &L.w.sh_gate_w},
  };
  for (auto& it : items) {
    uint16_t* d = nullptr;
    const int rc = alloc(h, &d, it.count, L.owned);
    if (rc != FW_OK) {
      free_layer(L);
      return rc;
    }
    const cudaError_t e = upload(d, it.src, it.count * 2, h->stream);
    if (e != cudaSuccess) {
      free_layer(L);
      return fail(FW_ECUDA, "weight copy", cudaGetErrorString(e));
    }
    *it.dst = d;
  }
  if (int rc = router_tables(h, L); rc != FW_OK) {
    free_layer(L);
    return rc;
  }
  const int ecount = held_experts(h), world = h->ep_world, rank = h->ep_rank;
  // Expert banks (this handle's experts) and the shared expert go to the
  // tiled layout through a bounded temporary buffer, a few experts at a time
  // (one at a time when the held experts are interleaved in the source).
  struct Tiled {
    fw::TiledSpec spec;
    long long n_mats;
    const uint16_t* src0;
    const uint16_t* src1;
    const uint16_t** dst;
    bool expert_bank;  // source holds every expert; this handle takes its own
  } tiled[] = {
      {{0, static_cast<int>(H), static_cast<int>(I), static_cast<long long>(2 * I * H),
        static_cast<long long>(2 * I * H)},
       ecount, gate_up, nullptr, &L.w.gate_up, true},
      {{1, static_cast<int>(I), 0, static_cast<long long>(H * I), static_cast<long long>(H * I)},
       ecount, down, nullptr, &L.w.down, true},
      {{0, static_cast<int>(H), 0, static_cast<long long>(2 * Is * H), static_cast<long long>(Is * H)}, 1,
       shared_gate, shared_up, &L.w.sh_gate, false},
      {{1, static_cast<int>(Is), 0, static_cast<long long>(H * Is), static_cast<long long>(H * Is)}, 1,
       shared_down, nullptr, &L.w.sh_down, false},
  };
  for (auto& t : tiled) {
    const bool strided = t.expert_bank && world > 1;
    uint16_t* d = nullptr;
    int rc = alloc(h, &d, static_cast<size_t>(t.n_mats * t.spec.mat_elems), L.owned);
    if (rc != FW_OK) {
      free_layer(L);
      return rc;
    }
    const size_t src_elems = static_cast<size_t>(t.spec.src_mat_elems);
    const size_t per_chunk = std::max<size_t>(1, (size_t(256) << 20) / (src_elems * 2 * (t.src1 ? 2 : 1)));
    const size_t chunk = strided ? 1 : std::min<size_t>(per_chunk, static_cast<size_t>(t.n_mats));
    uint16_t* tmp = nullptr;
    cudaError_t e = cudaMalloc(&tmp, chunk * src_elems * 2 * (t.src1 ? 2 : 1));
    for (size_t m0 = 0; e == cudaSuccess && m0 < static_cast<size_t>(t.n_mats); m0 += chunk) {
      const size_t n = std::min(chunk, static_cast<size_t>(t.n_mats) - m0);
      const size_t sm = strided ? m0 * world + rank : m0;  // source matrix of local matrix m0
      // copies and re-layout in order on the handle's stream
      e = cudaMemcpyAsync(tmp, t.src0 + sm * src_elems, n * src_elems * 2, cudaMemcpyDefault, h->stream);
      if (e == cudaSuccess && t.src1)
        e = cudaMemcpyAsync(tmp + n * src_elems, t.src1 + m0 * src_elems, n * src_elems * 2, cudaMemcpyDefault,
                            h->stream);
      if (e == cudaSuccess)
        e = fw::launch_relayout(t.spec, static_cast<long long>(m0), static_cast<long long>(n), tmp,
                                t.src1 ? tmp + n * src_elems : nullptr, d, h->stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
    }
    if (tmp) cudaFree(tmp);
    if (e != cudaSuccess) {
      free_layer(L);
      return fail(e == cudaErrorMemoryAllocation ? FW_ENOMEM : FW_ECUDA, "expert re-layout",
                  cudaGetErrorString(e));
    }
    *t.dst = d;
  }
  L.w.sh_up = L.w.sh_gate;  // tiled: the gate/up tiles hold both
  L.w.tiled = true;
  if (logit_bias != nullptr) {
    float* d = nullptr;
    const int rc = alloc(h, &d, E, L.owned);
    if (rc != FW_OK) {
      free_layer(L);
      return rc;
    }
    if (upload(d, logit_bias, E * 4, h->stream) != cudaSuccess) {
      free_layer(L);
      return fail(FW_ECUDA, "bias copy failed");
    }
    L.w.bias = d;
  }
  L.w.ep_rank = rank;
  L.w.ep_world = world;
  L.w.expert_count = ecount;
  L.prefill = h->prefill_ok && fw::make_prefill_weight_maps(h->shape, L.w, &L.maps);
  L.loaded = true;
  return FW_OK;
}

int fw_moe_load_expert(fw_moe* h, int32_t layer, int32_t expert, const uint16_t* gate_up, const uint16_t* down) {
  FW_TRY(check_handle(h, layer));
  if (expert < 0 || expert >= h->cfg.experts) return fail(FW_EINVAL, "expert out of range");
  if (gate_up == nullptr || down == nullptr) return fail(FW_EINVAL, "gate_up / down is null");
  if (expert % h->ep_world != h->ep_rank) return fail(FW_EINVAL, "expert is held by another rank");
  FW_CUDA(cudaSetDevice(h->device));
  OwnedLayer& L = h->layers[layer];
  const size_t H = h->cfg.hidden, I = h->cfg.intermediate;
  const long long bank = expert / h->ep_world;  // bank index of the expert on this GPU
  const fw::TiledSpec gu{0, static_cast<int>(H), static_cast<int>(I), static_cast<long long>(2 * I * H),
                         static_cast<long long>(2 * I * H)};
  const fw::TiledSpec dn{1, static_cast<int>(I), 0, static_cast<long long>(H * I), static_cast<long long>(H * I)};
  uint16_t* tmp = nullptr;
  cudaError_t e = cudaMalloc(&tmp, 3 * H * I * 2);
  if (e == cudaSuccess) e = cudaMemcpyAsync(tmp, gate_up, 2 * I * H * 2, cudaMemcpyDefault, h->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(tmp + 2 * I * H, down, H * I * 2, cudaMemcpyDefault, h->stream);
  // the banks are this handle's own buffers
  if (e == cudaSuccess) e = fw::launch_relayout(gu, bank, 1, tmp, nullptr, const_cast<uint16_t*>(L.w.gate_up), h->stream);
  if (e == cudaSuccess)
    e = fw::launch_relayout(dn, bank, 1, tmp + 2 * I * H, nullptr, const_cast<uint16_t*>(L.w.down), h->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
  if (tmp) cudaFree(tmp);
  if (e != cudaSuccess)
    return fail(e == cudaErrorMemoryAllocation ? FW_ENOMEM : FW_ECUDA, "expert load", cudaGetErrorString(e));
  return FW_OK;
}

int fw_moe_synth_layer(fw_moe* h, int32_t layer, uint64_t seed, float std_dev, int32_t zipf_bias) {
  if (h == nullptr) return fail(FW_EINVAL, "handle is null");
  if (layer < 0 || layer >= h->cfg.layers) return fail(FW_EINVAL, "layer out of range");
  if (!(std_dev > 0.0f)) return fail(FW_EINVAL, "std must be positive");
  FW_CUDA(cudaSetDevice(h->device));
  OwnedLayer& L = h->layers[layer];
  free_layer(L);
  const size_t H = h->cfg.hidden, I = h->cfg.intermediate, Is = h->cfg.shared_intermediate;
  const size_t E = h->cfg.experts;
  const float scale = synth_scale(std_dev);
  // Router and shared gate vector: reference layout.
  struct Item {
    uint32_t id;
    size_t count;
    const uint16_t** dst;
  } items[] = {
      {0, E * H, &L.w.router},
      {6, H, &L.w.sh_gate_w},
  };
  for (auto& it : items) {
    uint16_t* d = nullptr;
    const int rc = alloc(h, &d, it.count, L.owned);
    if (rc != FW_OK) {
      free_layer(L);
      return rc;
    }
    const cudaError_t e = fw::launch_synth(synth_key(seed, it.id), it.id, 0, it.count, scale, d, h->stream);
    if (e != cudaSuccess) {
      free_layer(L);
      return fail(FW_ECUDA, "synth launch", cudaGetErrorString(e));
    }
    *it.dst = d;
  }
  if (int rc = router_tables(h, L); rc != FW_OK) {
    free_layer(L);
    return rc;
  }
  const int ecount = held_experts(h);
  // Expert banks (this handle's experts) and the shared expert: generated
  // straight into the tiled layout (element values are those of their
  // reference indices).
  struct Tiled {
    fw::TiledSpec spec;
    long long n_mats;
    uint32_t id0, id1;
    const uint16_t** dst;
  } tiled[] = {
      {{0, static_cast<int>(H), static_cast<int>(I), static_cast<long long>(2 * I * H),
        static_cast<long long>(2 * I * H)},
       ecount, 1, 1, &L.w.gate_up},
      {{1, static_cast<int>(I), 0, static_cast<long long>(H * I), static_cast<long long>(H * I)},
       ecount, 2, 2, &L.w.down},
      {{0, static_cast<int>(H), 0, static_cast<long long>(2 * Is * H), static_cast<long long>(Is * H)}, 1, 3, 4,
       &L.w.sh_gate},
      {{1, static_cast<int>(Is), 0, static_cast<long long>(H * Is), static_cast<long long>(H * Is)}, 1, 5, 5,
       &L.w.sh_down},
  };
  for (int b = 0; b < 2; ++b) {  // generator values of the held experts' global indices
    tiled[b].spec.m0 = h->ep_rank;
    tiled[b].spec.m_stride = h->ep_world;
  }
  for (auto& t : tiled) {
    uint16_t* d = nullptr;
    const int rc = alloc(h, &d, static_cast<size_t>(t.n_mats * t.spec.mat_elems), L.owned);
    if (rc != FW_OK) {
      free_layer(L);
      return rc;
    }
    const cudaError_t e = fw::launch_synth_tiled(t.spec, t.n_mats, synth_key(seed, t.id0), synth_key(seed, t.id1),
                                                 scale, d, h->stream);
    if (e != cudaSuccess) {
      free_layer(L);
      return fail(FW_ECUDA, "synth launch", cudaGetErrorString(e));
    }
    *t.dst = d;
  }
  L.w.sh_up = L.w.sh_gate;
  L.w.tiled = true;
  if (zipf_bias) {
    std::vector<float> bias(E);
    for (size_t e = 0; e < E; ++e)
      bias[e] = static_cast<float>(0.5 * std::log(std::pow(static_cast<double>(e + 1), -1.1)));
    float* d = nullptr;
    const int rc = alloc(h, &d, E, L.owned);
    if (rc != FW_OK) {
      free_layer(L);
      return rc;
    }
    if (upload(d, bias.data(), E * 4, h->stream) != cudaSuccess) {
      free_layer(L);
      return fail(FW_ECUDA, "bias copy failed");
    }
    L.w.bias = d;
  }
  const cudaError_t e = cudaStreamSynchronize(h->stream);
  if (e != cudaSuccess) {
    free_layer(L);
    return fail(FW_ECUDA, std::string("synth: ") + cudaGetErrorString(e));
  }
  L.w.ep_rank = h->ep_rank;
  L.w.ep_world = h->ep_world;
  L.w.expert_count = ecount;
  L.prefill = h->prefill_ok && fw::make_prefill_weight_maps(h->shape, L.w, &L.maps);
  L.loaded = true;
  return FW_OK;
}

namespace {
// Remember which path the forward took, for fw_moe_last_union.
void note_forward(fw_moe* h, bool prefill, cudaStream_t st) {
  h->last_path = prefill ? 2 : 1;
  h->last_experts = held_experts(h);
  h->last_stream = st;
}
}  // namespace

int fw_moe_forward_async(fw_moe* h, int32_t layer, const uint16_t* x, int32_t tokens, uint16_t* y,
                         int32_t* topk_idx, uint16_t* topk_scores, void* stream) {
  FW_TRY(check_handle(h, layer));
  if (tokens < 0 || tokens > h->cfg.max_tokens) return fail(FW_EINVAL, "tokens out of range");
  if (tokens == 0) return FW_OK;
  if (x == nullptr || y == nullptr) return fail(FW_EINVAL, "x / y is null");
  if (!aligned16(x) || !aligned16(y)) return fail(FW_EINVAL, "x / y must be 16-byte aligned");
  if (!aligned4(topk_idx) || !aligned4(topk_scores))
    return fail(FW_EINVAL, "topk buffers must be 4-byte aligned");
  FW_CUDA(cudaSetDevice(h->device));
  const OwnedLayer& L = h->layers[layer];
  int32_t* idx = topk_idx ? topk_idx : h->idx_dev;
  uint16_t* sc = topk_scores ? topk_scores : h->score_dev;
  const cudaStream_t cs = static_cast<cudaStream_t>(stream);
  cudaEvent_t* ev = h->profile ? h->stage_ev : nullptr;
  if (h->ep != nullptr || h->p2p != nullptr) {
    if (fw::ep_comm_aborted(h->ep)) return fail(FW_ENCCL, "the communicator was aborted after a failure");
    bool ep_prefill = false;
    const int rc = ep_block(h, L, x, tokens, y, idx, sc, cs, ev, nullptr, &ep_prefill);
    if (rc == FW_OK) note_forward(h, ep_prefill, cs);
    return rc;
  }
  const bool prefill = tokens > kDecodeMaxTokens || tokens >= h->prefill_min_tokens;
  if (prefill && !L.prefill) return fail(FW_EINVAL, "this layer has no prefill tensor maps");
  fw::Scratch scr = h->sc;
  scr.stall = take_stall(h);
  // measured: +1 % at T = 64, neutral at T = 1, -2 % at T = 4
  if (!prefill && tokens > 4) prefetch_next(h, layer, &scr);
  const cudaError_t e =
      prefill ? fw::launch_prefill(h->shape, L.w, L.maps, h->pf_maps, h->luts, scr, x, tokens, y, idx, sc, cs, ev)
              : fw::launch_block(h->shape, L.w, h->luts, scr, x, tokens, y, idx, sc, cs, ev);
  if (e != cudaSuccess) return fail(FW_ECUDA, std::string("launch: ") + cudaGetErrorString(e));
  note_forward(h, prefill, cs);
  return FW_OK;
}

int fw_moe_last_path(fw_moe* h, int32_t* path) {
  if (h == nullptr || path == nullptr) return fail(FW_EINVAL, "null argument");
  if (h->last_path == 0) return fail(FW_EINVAL, "no forward has run on this handle");
  *path = h->last_path == 2 ? FW_PATH_PREFILL : FW_PATH_DECODE;
  return FW_OK;
}

int fw_moe_last_union(fw_moe* h, int32_t* distinct_experts, uint64_t* weight_bytes) {
  if (h == nullptr || distinct_experts == nullptr || weight_bytes == nullptr)
    return fail(FW_EINVAL, "null argument");
  if (h->last_path == 0) return fail(FW_EINVAL, "no forward has run on this handle");
  FW_CUDA(cudaSetDevice(h->device));
  FW_CUDA(cudaStreamSynchronize(h->last_stream));
  int n = 0;
  if (h->last_path == 1) {
    FW_CUDA(cudaMemcpy(&n, h->sc.sched, sizeof(int), cudaMemcpyDeviceToHost));  // n_active
  } else {
    std::vector<int> off(static_cast<size_t>(h->last_experts) + 1);
    FW_CUDA(cudaMemcpy(off.data(), h->sc.pair_offset, off.size() * sizeof(int), cudaMemcpyDeviceToHost));
    for (int e = 0; e < h->last_experts; ++e) n += off[e + 1] > off[e] ? 1 : 0;
  }
  const uint64_t H = h->cfg.hidden, I = h->cfg.intermediate, Is = h->cfg.shared_intermediate;
  const uint64_t E = h->cfg.experts;
  *distinct_experts = n;
  *weight_bytes = 2 * (E * H + H + 3 * H * Is + static_cast<uint64_t>(n) * 3 * H * I);
  return FW_OK;
}

int fw_moe_set_prefill_min_tokens(fw_moe* h, int32_t min_tokens) {
  if (h == nullptr) return fail(FW_EINVAL, "handle is null");
  if (min_tokens < 1) return fail(FW_EINVAL, "min_tokens must be >= 1");
  if (min_tokens <= kDecodeMaxTokens && !h->prefill_ok)
    return fail(FW_EINVAL, "this block shape has no prefill path");
  h->prefill_min_tokens = min_tokens;
  return FW_OK;
}

int fw_moe_sync(fw_moe* h, void* stream) {
  if (h == nullptr) return fail(FW_EINVAL, "handle is null");
  FW_CUDA(cudaSetDevice(h->device));
  if (h->ep != nullptr) {
    // Over NCCL a missing peer would hold the stream forever: wait at most
    // the handle's wait limit (twice: the kernels' own waits come first).
    cudaError_t ce = cudaSuccess;
    switch (fw::ep_bounded_sync(h->ep, static_cast<cudaStream_t>(stream), 2 * h->sc.wait_ns, &ce)) {
      case 0: break;
      case 1: return fail(FW_ETIMEOUT, "an expert-parallel collective did not complete within the wait limit "
                                       "(communicator aborted; destroy the handle)");
      case 2: return fail(FW_ENCCL, "the NCCL communicator reported an error (aborted; destroy the handle)");
      default: return fail(FW_ECUDA, "stream", cudaGetErrorString(ce));
    }
  }
  FW_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  int code = 0;
  FW_CUDA(cudaMemcpy(&code, h->sc.err, sizeof(int), cudaMemcpyDeviceToHost));
  if (code != 0) {
    FW_CUDA(zero_fill(h->sc.err, sizeof(int), h->stream));
    return map_device_error(code);
  }
  if (h->ep != nullptr) {
    const char* m = fw::ep_async_error(h->ep);
    if (m != nullptr) return fail(FW_ENCCL, m);
  }
  return FW_OK;
}

int fw_moe_forward(fw_moe* h, int32_t layer, const uint16_t* x, int32_t tokens, uint16_t* y,
                   int32_t* topk_idx, uint16_t* topk_scores) {
  FW_TRY(check_handle(h, layer));
  if (tokens < 0 || tokens > h->cfg.max_tokens) return fail(FW_EINVAL, "tokens out of range");
  if (tokens == 0) return FW_OK;
  if (x == nullptr || y == nullptr) return fail(FW_EINVAL, "x / y is null");
  FW_CUDA(cudaSetDevice(h->device));
  const size_t H = h->cfg.hidden, K = h->cfg.top_k;
  FW_CUDA(cudaMemcpyAsync(h->x_dev, x, tokens * H * 2, cudaMemcpyDefault, h->stream));
  FW_TRY(fw_moe_forward_async(h, layer, h->x_dev, tokens, h->y_dev, h->idx_dev, h->score_dev,
                              h->stream));
  FW_CUDA(cudaMemcpyAsync(y, h->y_dev, tokens * H * 2, cudaMemcpyDefault, h->stream));
  if (topk_idx)
    FW_CUDA(cudaMemcpyAsync(topk_idx, h->idx_dev, tokens * K * 4, cudaMemcpyDefault, h->stream));
  if (topk_scores)
    FW_CUDA(cudaMemcpyAsync(topk_scores, h->score_dev, tokens * K * 2, cudaMemcpyDefault, h->stream));
  return fw_moe_sync(h, h->stream);
}

int fw_moe_load_hc(fw_moe* h, int32_t layer, int32_t lowrank, const uint16_t* hc_norm, const uint16_t* mix_down,
                   const uint16_t* mix_up, const uint16_t* inject) {
  if (h == nullptr) return fail(FW_EINVAL, "handle is null");
  if (layer < 0 || layer >= h->cfg.layers) return fail(FW_EINVAL, "layer out of range");
  if (lowrank <= 0 || lowrank % 32 != 0 || lowrank > 4096)
    return fail(FW_EINVAL, "lowrank must be a positive multiple of 32, at most 4096");
  if (!hc_norm || !mix_down || !mix_up || !inject) return fail(FW_EINVAL, "a hyper-connection weight is null");
  if (h->cfg.hidden % 16 != 0) return fail(FW_EINVAL, "hidden must be a multiple of 16");
  FW_CUDA(cudaSetDevice(h->device));
  const size_t H = h->cfg.hidden, HH = 4 * H, LR = lowrank, M = h->cfg.max_tokens;
  if (h->hs_lowrank < lowrank) {
    // scratch for the largest lowrank seen (the other buffers once)
    fw::HcScratch& s = h->hs;
    if (h->hs_lowrank == 0) {
      FW_TRY(alloc(h, &s.normed, M * HH, h->scratch_owned));
      FW_TRY(alloc(h, &s.up, M * HH, h->scratch_owned));
      FW_TRY(alloc(h, &s.inject, M * 4, h->scratch_owned));
      FW_TRY(alloc(h, &s.mixed, M * H, h->scratch_owned));
      FW_TRY(alloc(h, &s.inj_w, M * 4, h->scratch_owned));
      FW_TRY(alloc(h, &h->hc_moe, M * H, h->scratch_owned));
      FW_TRY(alloc(h, &h->hc_post_dev, M * HH, h->scratch_owned));
      FW_TRY(alloc(h, &h->hc_out_dev, M * HH, h->scratch_owned));
      FW_TRY(alloc(h, &s.down, M * LR, h->scratch_owned));
    } else {
      FW_TRY(regrow(h, &s.down, M * LR));
    }
    h->hs_lowrank = lowrank;
  }
  OwnedLayer& L = h->layers[layer];
  for (void* p : L.hc_owned) cudaFree(p);
  L.hc_owned.clear();
  L.hc = fw::HcWeights{};
  struct Item {
    const uint16_t* src;
    size_t count;
    const uint16_t** dst;
  } items[] = {{hc_norm, HH, &L.hc.norm}, {mix_down, LR * HH, &L.hc.mix_down}, {mix_up, HH * LR, &L.hc.mix_up},
               {inject, 4 * HH, &L.hc.inject}};
  for (auto& it : items) {
    uint16_t* d = nullptr;
    const int rc = alloc(h, &d, it.count, L.hc_owned);
    if (rc != FW_OK) return rc;
    FW_CUDA(upload(d, it.src, it.count * 2, h->stream));
    *it.dst = d;
  }
  L.hc.lowrank = lowrank;
  return FW_OK;
}

int fw_moe_forward_hc_async(fw_moe* h, int32_t layer, const uint16_t* post, int32_t tokens, uint16_t* out,
                            int32_t* topk_idx, uint16_t* topk_scores, void* stream) {
  FW_TRY(check_handle(h, layer));
  const OwnedLayer& L = h->layers[layer];
  if (L.hc.lowrank == 0) return fail(FW_EINVAL, "layer has no hyper-connection weights (fw_moe_load_hc)");
  if (tokens < 0 || tokens > h->cfg.max_tokens) return fail(FW_EINVAL, "tokens out of range");
  if (tokens == 0) return FW_OK;
  if (post == nullptr || out == nullptr) return fail(FW_EINVAL, "post / out is null");
  if (!aligned16(post) || !aligned16(out)) return fail(FW_EINVAL, "post / out must be 16-byte aligned");
  if (!aligned4(topk_idx) || !aligned4(topk_scores))
    return fail(FW_EINVAL, "topk buffers must be 4-byte aligned");
  FW_CUDA(cudaSetDevice(h->device));
  const cudaStream_t cs = static_cast<cudaStream_t>(stream);
  cudaError_t e = fw::launch_hc_pre(L.hc, h->hs, h->luts, post, h->cfg.hidden, tokens, cs);
  if (e != cudaSuccess) return fail(FW_ECUDA, std::string("hyper-connection launch: ") + cudaGetErrorString(e));
  int32_t* idx = topk_idx ? topk_idx : h->idx_dev;
  uint16_t* sc = topk_scores ? topk_scores : h->score_dev;
  const fw::HcPost hp{post, h->hs.inj_w, out};
  cudaEvent_t* ev = h->profile ? h->stage_ev : nullptr;
  if (h->ep != nullptr || h->p2p != nullptr) {
    // The hyper-connection stages are per token (this rank's); the block in
    // between is expert-parallel and its combine applies the injection.
    bool ep_prefill = false;
    const int rc = ep_block(h, L, h->hs.mixed, tokens, h->hc_moe, idx, sc, cs, ev, &hp, &ep_prefill);
    if (rc == FW_OK) note_forward(h, ep_prefill, cs);
    return rc;
  }
  const bool prefill = tokens > kDecodeMaxTokens || tokens >= h->prefill_min_tokens;
  if (prefill && !L.prefill) return fail(FW_EINVAL, "this layer has no prefill tensor maps");
  e = prefill ? fw::launch_prefill(h->shape, L.w, L.maps, h->pf_maps, h->luts, h->sc, h->hs.mixed, tokens, h->hc_moe,
                                   idx, sc, cs, ev, &hp)
              : fw::launch_block(h->shape, L.w, h->luts, h->sc, h->hs.mixed, tokens, h->hc_moe, idx, sc, cs, ev,
                                 &hp);
  if (e != cudaSuccess) return fail(FW_ECUDA, std::string("launch: ") + cudaGetErrorString(e));
  note_forward(h, prefill, cs);
  return FW_OK;
}

int fw_moe_forward_hc(fw_moe* h, int32_t layer, const uint16_t* post, int32_t tokens, uint16_t* out,
                      int32_t* topk_idx, uint16_t* topk_scores) {
  FW_TRY(check_handle(h, layer));
  if (tokens < 0 || tokens > h->cfg.max_tokens) return fail(FW_EINVAL, "tokens out of range");
  if (tokens == 0) return FW_OK;
  if (post == nullptr || out == nullptr) return fail(FW_EINVAL, "post / out is null");
  if (h->hc_post_dev == nullptr) return fail(FW_EINVAL, "no hyper-connection weights loaded (fw_moe_load_hc)");
  FW_CUDA(cudaSetDevice(h->device));
  const size_t HH = 4 * static_cast<size_t>(h->cfg.hidden), K = h->cfg.top_k;
  FW_CUDA(cudaMemcpyAsync(h->hc_post_dev, post, tokens * HH * 2, cudaMemcpyDefault, h->stream));
  FW_TRY(fw_moe_forward_hc_async(h, layer, h->hc_post_dev, tokens, h->hc_out_dev, h->idx_dev, h->score_dev,
                                 h->stream));
  FW_CUDA(cudaMemcpyAsync(out, h->hc_out_dev, tokens * HH * 2, cudaMemcpyDefault, h->stream));
  if (topk_idx)
    FW_CUDA(cudaMemcpyAsync(topk_idx, h->idx_dev, tokens * K * 4, cudaMemcpyDefault, h->stream));
  if (topk_scores)
    FW_CUDA(cudaMemcpyAsync(topk_scores, h->score_dev, tokens * K * 2, cudaMemcpyDefault, h->stream));
  return fw_moe_sync(h, h->stream);
}

int fw_moe_profile(fw_moe* h, int32_t enable) {
  if (h == nullptr) return fail(FW_EINVAL, "handle is null");
  FW_CUDA(cudaSetDevice(h->device));
  if (enable) {
    for (auto& ev : h->stage_ev)
      if (!ev) FW_CUDA(cudaEventCreate(&ev));
  }
  h->profile = enable != 0;
  return FW_OK;
}

int fw_moe_profile_read(fw_moe* h, float* stage_ms, int32_t n) {
  if (h == nullptr || stage_ms == nullptr || n < fw::kStages) return fail(FW_EINVAL, "bad argument");
  if (!h->profile) return fail(FW_EINVAL, "profiling is off");
  FW_CUDA(cudaSetDevice(h->device));
  FW_CUDA(cudaEventSynchronize(h->stage_ev[fw::kStages]));
  for (int i = 0; i < fw::kStages; ++i)
    FW_CUDA(cudaEventElapsedTime(&stage_ms[i], h->stage_ev[i], h->stage_ev[i + 1]));
  for (int i = fw::kStages; i < n; ++i) stage_ms[i] = 0.0f;
  return FW_OK;
}

int fw_moe_memory(const fw_moe* h, uint64_t* bytes) {
  if (h == nullptr || bytes == nullptr) return fail(FW_EINVAL, "null argument");
  *bytes = h->bytes;
  return FW_OK;
}

int fw_linear_bf16(const uint16_t* w, const uint16_t* x, int32_t rows, int32_t cols, int32_t tokens,
                   uint16_t* y, void* stream) {
  if (!w || !x || !y) return fail(FW_EINVAL, "null argument");
  if (rows <= 0 || tokens <= 0 || cols <= 0 || cols % 32 != 0 || 8ull * cols * 4 > 200 * 1024)
    return fail(FW_EINVAL, "rows/tokens must be positive; cols a multiple of 32, at most 6400");
  if (!aligned16(w) || !aligned16(x)) return fail(FW_EINVAL, "w / x must be 16-byte aligned");
  const cudaError_t e = fw::launch_linear(w, x, rows, cols, tokens, y, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(FW_ECUDA, std::string("linear: ") + cudaGetErrorString(e));
  return FW_OK;
}

int fw_swiglu_bf16(const uint16_t* gate, const uint16_t* up, int64_t n, uint16_t* out, void* stream) {
  if (!gate || !up || !out || n < 0) return fail(FW_EINVAL, "bad argument");
  if (n == 0) return FW_OK;
  int dev = 0;
  FW_CUDA(cudaGetDevice(&dev));
  DeviceCommon* c = nullptr;
  FW_TRY(device_common(dev, &c));
  const cudaError_t e = fw::launch_swiglu(gate, up, n, c->silu, out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(FW_ECUDA, std::string("swiglu: ") + cudaGetErrorString(e));
  return FW_OK;
}

int fw_add_bf16(const uint16_t* a, const uint16_t* b, int64_t n, uint16_t* out, void* stream) {
  if (!a || !b || !out || n < 0) return fail(FW_EINVAL, "bad argument");
  if (n == 0) return FW_OK;
  const cudaError_t e = fw::launch_add_bf16(a, b, n, out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(FW_ECUDA, std::string("add: ") + cudaGetErrorString(e));
  return FW_OK;
}

int fw_route_bf16(const uint16_t* logits, int32_t tokens, int32_t experts, int32_t top_k,
                  int32_t* indices, uint16_t* scores, void* stream) {
  if (!logits || !indices || !scores) return fail(FW_EINVAL, "null argument");
  if (tokens < 0 || experts <= 0 || experts % 32 != 0 || experts > 1024 || top_k < 1 ||
      top_k > 32 || top_k > experts)
    return fail(FW_EINVAL, "bad route shape");
  if (tokens == 0) return FW_OK;
  int dev = 0;
  FW_CUDA(cudaGetDevice(&dev));
  DeviceCommon* c = nullptr;
  FW_TRY(device_common(dev, &c));
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = fw::launch_route(logits, tokens, experts, top_k, indices, scores, c->err, st);
  if (e != cudaSuccess) return fail(FW_ECUDA, std::string("route: ") + cudaGetErrorString(e));
  FW_CUDA(cudaStreamSynchronize(st));
  int code = 0;
  FW_CUDA(cudaMemcpy(&code, c->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (code != 0) {
    FW_CUDA(zero_fill(c->err, sizeof(int), st));
    return map_device_error(code);
  }
  return FW_OK;
}

bool firewing_cuda_topk_bf16(const uint16_t* values, size_t count, size_t k, size_t* indices) {
  if (values == nullptr || indices == nullptr || k == 0 || k > count || count % 32 != 0 ||
      count > 1024 || k > 32)
    return false;
  uint16_t* dv = nullptr;
  int32_t* di = nullptr;
  uint16_t* ds = nullptr;
  bool ok = cudaMalloc(&dv, count * 2) == cudaSuccess && cudaMalloc(&di, k * 4) == cudaSuccess &&
            cudaMalloc(&ds, k * 2) == cudaSuccess &&
            upload(dv, values, count * 2, cudaStreamLegacy) == cudaSuccess;
  std::vector<int32_t> idx(k);
  if (ok) {
    ok = fw_route_bf16(dv, 1, static_cast<int32_t>(count), static_cast<int32_t>(k), di, ds, nullptr) ==
             FW_OK &&
         cudaMemcpy(idx.data(), di, k * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
  }
  cudaFree(dv);
  cudaFree(di);
  cudaFree(ds);
  if (!ok) return false;
  for (size_t i = 0; i < k; ++i) indices[i] = static_cast<size_t>(idx[i]);
  return true;
}

}  // extern "C"
