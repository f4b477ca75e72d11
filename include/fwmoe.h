/*
 * fwmoe.h -- C ABI of the B200 (sm_100a) sparse-MoE block library.
 *
 * Drop-in GPU backend for the sparse-MoE block of x3haloed/firewing (Rust
 * crate).  Plain C types only: pointers, sizes, status codes.  Every entry
 * point cites the reference interface it replaces (paths relative to the
 * firewing source tree).
 *
 * Conventions (mirroring the reference's fail-closed `Result<_, String>`):
 *   - every function returns an int status: FW_OK (0) or a negative FW_E*;
 *     fw_last_error() returns a thread-local message for the last failure;
 *   - tensors are bf16 bit patterns (uint16_t), row-major, little-endian, in
 *     the reference's layout (src/expert.rs:362-512);
 *   - a handle is not thread-safe and owns one device; calls made with it
 *     switch the calling thread's current CUDA device to that device;
 *   - `stream` arguments are cudaStream_t values passed as void*
 *     (NULL = the legacy default stream).
 *
 * Numerics: every GEMV keeps the reference's f32 reduction order
 * (src/expert.rs:514-552) and every bf16 rounding point, so outputs are
 * bit-identical to the reference CPU path except for the router softmax,
 * whose exp is correctly rounded where the host libm's expf may be one ulp
 * off; a renormalised score can then differ by one bf16 ulp.  Products must
 * stay inside the normal f32 range (|w*x| >= 2^-126 or zero) for the
 * bit-exact claim; outside it results stay within one f32 rounding.
 */
#ifndef FWMOE_H
#define FWMOE_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FW_OK 0
#define FW_EINVAL (-1)   /* bad argument, shape or state */
#define FW_ECUDA (-2)    /* a CUDA call failed */
#define FW_ENCCL (-3)    /* a collective failed (expert parallelism) */
#define FW_ETIMEOUT (-4) /* a bounded device wait gave up */
#define FW_ENOMEM (-5)   /* device allocation failed */
#define FW_ENAN (-6)     /* router logits contained NaN (src/decoder_layer.rs:279) */

typedef struct fw_moe fw_moe;

/* Block configuration.  The reference hard-codes these
 * (src/decoder_layer.rs:14-17, 40-42; src/metal_moe.rs:15-21).
 * Constraints: hidden, intermediate and shared_intermediate multiples of
 * 64, at most 4096; experts % 32 == 0 and <= 1024;
 * 1 <= top_k <= min(32, experts); 1 <= max_tokens <= 16384, and above 256
 * only when hidden is a multiple of 256 and 2*intermediate and
 * 2*shared_intermediate are multiples of 128 (the prefill path's tiles). */
typedef struct fw_moe_config {
    int32_t hidden;              /* H */
    int32_t intermediate;        /* I of a routed expert */
    int32_t shared_intermediate; /* Is of the shared expert */
    int32_t experts;             /* E routed experts */
    int32_t top_k;               /* K */
    int32_t max_tokens;          /* largest T passed to a forward */
    int32_t layers;              /* resident layers (each loaded separately) */
} fw_moe_config;

/* Thread-local description of the last failure ("" if none). */
const char* fw_last_error(void);

/* Create a block runner on `device`: allocates scratch and builds the bf16
 * SiLU / sigmoid tables on the host, as ExactResidentTop10Runner::install
 * does (src/metal_moe.rs:95-223, 385-392, 399-421). */
int fw_moe_create(const fw_moe_config* config, int device, fw_moe** out);
int fw_moe_destroy(fw_moe* handle);
/* The configuration the handle was created with. */
int fw_moe_get_config(const fw_moe* handle, fw_moe_config* out);

/* Copy one layer's weights (host or device pointers) into memory the handle
 * owns.  Layouts: router [E][H] (model.layers.N.mlp.gate.weight);
 * gate_up [E][2I][H] (experts.gate_up_proj, gate rows first); down [E][H][I]
 * (experts.down_proj); shared_gate, shared_up [Is][H]; shared_down [H][Is];
 * shared_gate_w [1][H] (shared_expert_gate.weight); logit_bias [E] f32 or
 * NULL.  Replaces the reference's per-call weight reads
 * (src/expert.rs:362-512) and buffer install (src/metal_moe.rs:162-207). */
int fw_moe_load_layer(fw_moe* handle, int32_t layer, const uint16_t* router,
                      const uint16_t* gate_up, const uint16_t* down,
                      const uint16_t* shared_gate, const uint16_t* shared_up,
                      const uint16_t* shared_down, const uint16_t* shared_gate_w,
                      const float* logit_bias);

/* Fill one layer with seeded synthetic weights generated on the device
 * (no reference counterpart: the benchmark configurations use synthetic
 * weights).  Element i of tensor id (router 0, gate_up 1, down 2,
 * shared_gate 3, shared_up 4, shared_down 5, shared_gate_w 6) is output i of
 * a SplitMix64 stream keyed by (seed, id), as an Irwin-Hall(4) sum of 16-bit
 * uniforms scaled to standard deviation `std`, rounded to bf16.  zipf_bias
 * != 0 installs logit_bias[e] = 0.5*ln((e+1)^-1.1). */
int fw_moe_synth_layer(fw_moe* handle, int32_t layer, uint64_t seed, float std,
                       int32_t zipf_bias);

/* Whole sparse-MoE block for `tokens` tokens, synchronous, HOST buffers:
 * x [T][H] -> y [T][H] = routed top-k mixture + sigmoid-gated shared expert;
 * topk_idx [T][K] / topk_scores [T][K] (may be NULL) receive the selection in
 * top-k order and the renormalised bf16 scores.  Replaces the in-layer block
 * body (src/decoder_layer.rs:460-586) and ExactResidentTop10Runner::
 * execute_exact (src/metal_moe.rs:423-441).  Returns FW_ENAN when a token's
 * router logits contain NaN, like route() (src/decoder_layer.rs:278-281). */
int fw_moe_forward(fw_moe* handle, int32_t layer, const uint16_t* x, int32_t tokens,
                   uint16_t* y, int32_t* topk_idx, uint16_t* topk_scores);

/* Same, DEVICE buffers, stream-ordered and asynchronous.  topk_idx /
 * topk_scores may be NULL.  Device-side failures (NaN logits) are reported by
 * the next fw_moe_sync on the handle. */
int fw_moe_forward_async(fw_moe* handle, int32_t layer, const uint16_t* x, int32_t tokens,
                         uint16_t* y, int32_t* topk_idx, uint16_t* topk_scores,
                         void* stream);

/* The hyper-connection caller on either side of the block
 * (src/hyper_connection.rs:412-490, src/decoder_layer.rs:451-458, 587-607).
 * fw_moe_load_hc copies one layer's weights (host or device pointers):
 * hc_norm [4H], input_mix_weight_down [lowrank][4H], input_mix_weight_up
 * [4H][lowrank], block_inject_weight [4][4H]; lowrank a multiple of 32.
 * fw_moe_forward_hc maps the attention output post [T][4H] (four residual
 * streams) to the layer output [T][4H]:
 *   - grouped RMS norm, the low-rank input mix and the injection weights
 *     give the block input mixed [T][H];
 *   - the block runs on it;
 *   - out[g*H + c] = bf16(post[g*H + c] + bf16(moe[c] * w[g])), fused into
 *     the combine.
 * Every rounding point is the reference's, so decode-width outputs are bit
 * for bit the reference's.  Host buffers (forward_hc) or device buffers
 * (forward_hc_async, stream-ordered).  Under expert parallelism the
 * hyper-connection stages run on each rank's own tokens and the block in
 * between is expert-parallel; the call is then collective like
 * fw_moe_forward. */
int fw_moe_load_hc(fw_moe* handle, int32_t layer, int32_t lowrank, const uint16_t* hc_norm,
                   const uint16_t* mix_down, const uint16_t* mix_up, const uint16_t* inject);
int fw_moe_forward_hc(fw_moe* handle, int32_t layer, const uint16_t* post, int32_t tokens,
                      uint16_t* out, int32_t* topk_idx, uint16_t* topk_scores);
int fw_moe_forward_hc_async(fw_moe* handle, int32_t layer, const uint16_t* post, int32_t tokens,
                            uint16_t* out, int32_t* topk_idx, uint16_t* topk_scores, void* stream);

/* Forwards of at least `min_tokens` tokens (and every forward wider than
 * 256 tokens) run the prefill path: the expert FFNs as grouped bf16 GEMMs on
 * the tensor cores (f32 accumulation in the tensor core's own order, outputs
 * within the block tolerance of the reference, selection exact).  Narrower
 * forwards run the decode path, which reproduces the reference's dot
 * schedule bit for bit.  Under expert parallelism the width compared is the
 * total over the ranks (tokens x world), since each rank's experts see every
 * rank's tokens.  Default 96 for a shape with a prefill path (from about
 * two tokens per expert the tensor cores are faster; measured at config 0:
 * 205 k against 199 k token-layers/s at T = 96, 468 k against 272 k at
 * T = 256; two GPUs at 64 tokens each: 380 k against 314 k), 257 for a
 * shape without one.  No reference counterpart: the reference has one path
 * for every width (src/decoder_layer.rs:460-586).  FW_EINVAL when
 * min_tokens <= 256 and the shape has no prefill path. */
int fw_moe_set_prefill_min_tokens(fw_moe* handle, int32_t min_tokens);

/* Which path the handle's last forward took: FW_PATH_DECODE (bit-exact
 * dot schedule) or FW_PATH_PREFILL (tensor cores, block tolerance).
 * FW_EINVAL before the first forward.  No reference counterpart. */
#define FW_PATH_DECODE 1
#define FW_PATH_PREFILL 2
int fw_moe_last_path(fw_moe* handle, int32_t* path);

/* Expert parallelism over the GPUs of one node (no reference counterpart:
 * the reference runs the block on one device).  Rank r of `world` holds the
 * routed experts e with e % world == r of every layer, at bank index
 * e / world (interleaved, so a skewed router's hot low ids spread over the
 * ranks; router, shared expert and bias replicated), and brings its own
 * tokens to each forward.  fw_moe_load_layer takes the full checkpoint banks
 * and keeps this rank's experts.
 * Per layer:
 *   - router and route run on the rank's own tokens;
 *   - dispatch: this rank's experts get the token rows that selected them;
 *   - this rank's experts run over those tokens (and the shared expert over
 *     its own tokens);
 *   - combine: each token's weighted rows return to its owner, which sums
 *     them in ascending expert id.
 * Two transports (fw_moe_ep_set_transport, before fw_moe_ep_init):
 *   FW_EP_TRANSPORT_P2P (default): NVLink peer memory.  Every rank's
 *     exchange window is mapped by every rank; dispatch pulls each needed
 *     token row once per destination GPU, the expert kernels' epilogues
 *     store the weighted rows straight into the owners' windows (the
 *     transfer overlaps the expert GEMMs), and flags with bounded waits
 *     order the steps; nothing waits on the host.  The ranks' processes find
 *     each other through abstract Unix sockets named after `id`.
 *   FW_EP_TRANSPORT_NCCL: all-gathers for the dispatch and grouped
 *     send/recv for the combine over NCCL (libnccl.so.2, loaded at run
 *     time); the prefill path waits once on the host for the exchange sizes.
 * The decode path (widths up to min(256, 1024 / world) tokens per rank) is
 * bit-identical to one GPU.  Wider forwards take the prefill path's
 * tensor-core GEMMs; their outputs are within the block tolerance.
 *   fw_ep_unique_id: a communicator id; make it on one rank and hand the
 *     128 bytes to every rank (any host transport).
 *   fw_moe_ep_init: on every rank, collectively, after fw_moe_create and
 *     before any layer is loaded.  Needs 2 <= world <= 8 and
 *     experts % world == 0.  Afterwards every forward on the handle is
 *     collective: all ranks call it for the same layer with the same token
 *     count, in the same order.  FW_ENCCL on transport errors, and from the
 *     next fw_moe_sync when a peer reported a failure; FW_ETIMEOUT when a
 *     peer did not take part in a forward within the wait limit
 *     (fw_moe_set_wait_limit).  A handle whose expert-parallel forward failed
 *     stays failed (the ranks no longer agree on the forward count):
 *     destroy it on every rank. */
#define FW_EP_TRANSPORT_P2P 0
#define FW_EP_TRANSPORT_NCCL 1
int fw_moe_ep_set_transport(fw_moe* handle, int32_t transport);
int fw_ep_unique_id(uint8_t id[128]);
int fw_moe_ep_init(fw_moe* handle, int32_t rank, int32_t world, const uint8_t id[128]);

/* Weights from a safetensors checkpoint (no reference counterpart as a C
 * call: the reference reads the same tensors with read_expert_slice /
 * read_tensor_2d, src/expert.rs:362-512, and its mapped checkpoint catalog,
 * src/checkpoint_catalog.rs:146-443).  `checkpoint` is a directory holding
 * model.safetensors.index.json and its shards, or one .safetensors file;
 * shards are memory-mapped and validated as the reference validates them
 * (header length, dtypes, shapes, offsets, overlaps, index consistency).
 *   fw_moe_load_layer_safetensors: the block's tensors under `prefix`
 *     (e.g. "model.language_model.layers.0.mlp"): gate.weight [E][H],
 *     experts.gate_up_proj [E][2I][H], experts.down_proj [E][H][I],
 *     shared_expert.{gate,up}_proj.weight [Is][H],
 *     shared_expert.down_proj.weight [H][Is], shared_expert_gate.weight
 *     [1][H]; all BF16.  Under expert parallelism only this rank's experts
 *     are copied to the device.
 *   fw_moe_load_hc_safetensors: the hyper-connection tensors under `prefix`
 *     (e.g. "model.language_model.layers.0.mlp_hyper_connection"):
 *     hc_norm.weight [4H], input_mix_weight_down.weight [LR][4H],
 *     input_mix_weight_up.weight [4H][LR], block_inject_weight.weight
 *     [4][4H]; LR from the checkpoint.
 *   fw_safetensors_tensor_info: handle-free; validates one file and reports a
 *     tensor's dtype, shape (rank <= 8) and payload range.
 * FW_EINVAL with a message naming the tensor on any mismatch. */
int fw_moe_load_layer_safetensors(fw_moe* handle, int32_t layer, const char* checkpoint, const char* prefix);
int fw_moe_load_hc_safetensors(fw_moe* handle, int32_t layer, const char* checkpoint, const char* prefix);
int fw_safetensors_tensor_info(const char* file, const char* tensor, char dtype[16], int64_t shape[8],
                               int32_t* rank, uint64_t* offset, uint64_t* bytes);

/* Replace one routed expert of a loaded layer: gate_up [2I][H] and down
 * [H][I] in the reference layout, host or device pointers (the reference
 * streams experts one at a time into its resident buffers,
 * src/metal_moe.rs:162-207; src/compressed_overlap.rs).  Synchronous; not
 * concurrent with a forward of the same layer.  Under expert parallelism
 * only experts this rank holds (FW_EINVAL otherwise). */
int fw_moe_load_expert(fw_moe* handle, int32_t layer, int32_t expert, const uint16_t* gate_up,
                       const uint16_t* down);

/* Compressed expert containers, the reference's streamed-expert format
 * (tools/build_sequential_shuffle_container.py, read by
 * src/compressed_overlap.rs): one independent zstd frame per (layer, expert)
 * at a page-aligned offset of `container_file`, listed by a JSON manifest
 * (records {layer, expert, offset, compressed_bytes, physical_bytes,
 * frame_sha256, source_sha256}); a frame decompresses to the expert's
 * gate_up then down bytes, shuffled (even bytes, then odd bytes).
 *   fw_moe_load_expert_container: every record of `container_layer` into
 *     layer `layer` of the handle (experts held by this rank); the host
 *     decompresses (libzstd, loaded at run time, several frames at once),
 *     the GPU un-shuffles and re-lays the expert out.  verify != 0 checks
 *     both SHA-256 digests.  *loaded = experts replaced.
 *   fw_codec_container_check: handle-free; validates the manifest and
 *     decodes (and with verify, hashes) the records of `layer` (all when
 *     layer < 0) for experts of source_bytes_per_expert bytes.
 * FW_EINVAL on any format, size or hash mismatch. */
int fw_moe_load_expert_container(fw_moe* handle, int32_t layer, const char* manifest, int32_t container_layer,
                                 int32_t verify, int32_t* loaded);
int fw_codec_container_check(const char* manifest, int32_t layer, uint64_t source_bytes_per_expert,
                             int32_t verify, int32_t* records);

/* The expert union of the last forward on the handle (synchronises its
 * stream): the distinct routed experts it streamed on this GPU (U), and the
 * weight bytes it read: router, shared gate, shared expert and those U
 * experts once each, however many of the forward's tokens selected them.
 * With speculative decoding, a verify forward over the proposal positions
 * reads U experts for T tokens; the caller divides its accepted tokens (A)
 * by U as the reference's A / U accounting does (docs/ARCHITECTURE.md:93-96,
 * src/mtp_transaction.rs:182-212).  FW_EINVAL before the first forward. */
int fw_moe_last_union(fw_moe* handle, int32_t* distinct_experts, uint64_t* weight_bytes);

/* Wait for `stream`, then report and clear device-side status. */
int fw_moe_sync(fw_moe* handle, void* stream);

/* Bound of the handle's device-side waits on other CTAs' work and on
 * expert-parallel peers, in nanoseconds (1 ms .. 60 s; default 2 s).  A wait
 * that runs out ends its kernel early with FW_ETIMEOUT reported by
 * fw_moe_sync, instead of hanging the device.  No reference counterpart: the
 * reference's device transactions fail closed on a command buffer error
 * (src/metal_moe.rs:259-264, 353-358). */
int fw_moe_set_wait_limit(fw_moe* handle, uint64_t nanoseconds);

/* Test hook (no reference counterpart): the next forward on the handle makes
 * the expert kernel's wait for its gate/up units unreachable, so that wait
 * runs out after the wait limit and the forward reports FW_ETIMEOUT; the
 * forward after it is normal again. */
int fw_moe_test_stall(fw_moe* handle);

/* Per-stage timing, for roofline measurement (the reference times its phases
 * with host intervals, src/metal_moe.rs:473-477, 590-606).  While enabled,
 * every forward records CUDA events around its five stages, which
 * serialises them; fw_moe_profile_read waits for the last forward and
 * returns the five durations in milliseconds (n >= 5):
 *   router logits; route (and, under expert parallelism, publishing this
 *   rank's tokens); dispatch (grouping pairs by expert, and under expert
 *   parallelism bringing every rank's selections and the needed rows);
 *   experts (gate_up + SwiGLU, down + scale); combine (under expert
 *   parallelism including the wait for the slowest peer's rows). */
int fw_moe_profile(fw_moe* handle, int32_t enable);
int fw_moe_profile_read(fw_moe* handle, float* stage_ms, int32_t n);

/* Device bytes the handle holds (weights + scratch). */
int fw_moe_memory(const fw_moe* handle, uint64_t* bytes);

/* Device pointers to one layer's weights, in the layouts of
 * fw_moe_load_layer (logit_bias may be NULL). */
typedef struct fw_moe_weights {
    const uint16_t* router;
    const uint16_t* gate_up;
    const uint16_t* down;
    const uint16_t* shared_gate;
    const uint16_t* shared_up;
    const uint16_t* shared_down;
    const uint16_t* shared_gate_w;
    const float* logit_bias;
} fw_moe_weights;

/* The whole block, like fw_moe_forward_async, for callers that cannot
 * allocate device memory (no counterpart in the reference): a framework whose
 * caching allocator already holds the GPU's memory, or a latency-critical
 * loop that must not call cudaMalloc/cudaFree, which synchronise the device.
 * It allocates nothing: weights, x [T][H], y [T][H], topk_idx [T][K] and
 * topk_scores [T][K] are the caller's DEVICE buffers on the current device
 * (topk buffers may be NULL), and the scratch lives in an 8 MiB array
 * compiled into the library, which every GPU that loads the library holds
 * until exit.  Only the shape fields of `config` are read.  Shapes whose
 * scratch exceeds 8 MiB are rejected with FW_EINVAL (config 0, H=2048 with
 * K=10, fits up to T=121).  The weights stay in the reference layout, so
 * this path always runs the generic decode expert kernel: at T <= 4 it is
 * slower than fw_moe_forward, whose handle re-lays the banks out for the
 * small-width kernel.  The first call on a device sets up that device
 * (looks up the array's device address, uploads the SiLU/sigmoid tables):
 * make it before any stream capture.  Calls share the scratch array, so
 * calls that overlap on the GPU race; each call is synchronous on `stream`.
 * Returns FW_ENAN on NaN router logits, like fw_moe_forward. */
int fw_moe_forward_noalloc(const fw_moe_config* config, const fw_moe_weights* weights,
                           const uint16_t* x, int32_t tokens, uint16_t* y, int32_t* topk_idx,
                           uint16_t* topk_scores, void* stream);

/* ---- primitives over DEVICE buffers (the reference crate's functions) ---- */

/* y[t][r] = bf16(dot(w[r], x[t])) with the reference reduction order:
 * linear_bf16 (src/expert.rs:554-560) for `tokens` input vectors.
 * cols % 32 == 0. */
int fw_linear_bf16(const uint16_t* w, const uint16_t* x, int32_t rows, int32_t cols,
                   int32_t tokens, uint16_t* y, void* stream);

/* out[i] = bf16(bf16(silu(gate[i])) * up[i]): swiglu_bf16
 * (src/expert.rs:562-571) via the host-built table of
 * src/metal_moe.rs:385-392. */
int fw_swiglu_bf16(const uint16_t* gate, const uint16_t* up, int64_t n, uint16_t* out,
                   void* stream);
/* out[i] = add_bf16(a[i], b[i]) (src/expert.rs:578): bf16 round to nearest
 * even of the f32 sum, NaN as 0x7fc0; device pointers, stream-ordered. */
int fw_add_bf16(const uint16_t* a, const uint16_t* b, int64_t n, uint16_t* out, void* stream);

/* In-layer route for `tokens` logit rows [T][experts]: top-k (logit
 * descending, ties by ascending index, src/router.rs:241-247), f32 softmax,
 * renormalised bf16 scores: route (src/decoder_layer.rs:278-307).
 * experts % 32 == 0, <= 1024.  Synchronous; FW_ENAN on NaN logits. */
int fw_route_bf16(const uint16_t* logits, int32_t tokens, int32_t experts, int32_t top_k,
                  int32_t* indices, uint16_t* scores, void* stream);

/* Drop-in for the reference's only C ABI on the path,
 * `bool firewing_torch_topk_bf16(const uint16_t*, size_t, size_t, size_t*)`
 * (native/topk_shim.cpp:18-44, bound at src/decoder_layer.rs:19-39): HOST
 * buffers, runs on the current device.  false on null pointers, k == 0,
 * k > count, count % 32 != 0 or count > 1024.  Ties are ordered by
 * ascending index (the shim's order among equal values depends on the C++
 * library). */
bool firewing_cuda_topk_bf16(const uint16_t* values, size_t count, size_t k, size_t* indices);

#ifdef __cplusplus
}
#endif
#endif /* FWMOE_H */
