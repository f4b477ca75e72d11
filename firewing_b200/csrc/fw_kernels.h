// fw_kernels.h -- host-side launch interface of the sparse-MoE kernels.
// Internal to libfwmoe; the public C ABI is include/fwmoe.h.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

struct fw_moe;  // the C ABI handle (include/fwmoe.h)

namespace fw {

// Device-side status codes written to the per-handle error word (first
// writer wins).  The host maps them to FW_E* return codes.
enum DeviceError : int {
  kErrNone = 0,
  kErrNanLogits = 1,   // a router logit was NaN (src/decoder_layer.rs:279)
  kErrTimeout = 2,     // a bounded wait on an mbarrier / flag gave up
  kErrBadIndex = 3,    // an expert id outside [0, E) reached a kernel
  kErrCapacity = 4,    // more (token, expert) pairs than the scratch holds
  kErrPeer = 5,        // an expert-parallel peer reported a failure in this forward
};

// ---- expert parallelism over NVLink peer memory (fw_p2p.cu) -----------------
constexpr int kEpMaxWorld = 8;
// Every rank owns one exchange window (same layout on every rank), and every
// window is mapped into every rank's address space:
//   [0, 32)      uint32 pub[world]:  pub[w] = 2*seq (+1 on failure) once rank
//                                    w's tokens of forward `seq` are in its window
//   [128, 160)   uint32 done[world]: done[w] likewise once rank w has written
//                                    every weighted row it computed for this
//                                    rank's tokens of forward `seq`
//   off_x        [M][H] bf16   this rank's token rows of the current forward
//   off_idx      [M][K] int32  their top-k ids
//   off_score    [M][K] bf16   their route weights
//   off_recv     [M][K][H] bf16 weighted rows of this rank's tokens, row t*K+k
//                               written by the rank that holds expert idx[t][k]
// A flag is written with a release store at system scope and read with
// acquire loads; every wait on one is bounded.
struct EpPeers {
  unsigned char* win[kEpMaxWorld] = {};  // window of rank r in this rank's address space
  int rank = 0, world = 0;               // world == 0: expert parallelism over peer memory is off
  int t_local = 0;                       // tokens per rank in this forward
  int K = 0, H = 0;
  long long off_x = 0, off_idx = 0, off_score = 0, off_recv = 0;
  unsigned seq = 0;                      // forward sequence number (same on every rank)
  unsigned long long wait_ns = 0;        // bound of every wait on a peer
  int* ticket = nullptr;                 // [2] CTA completion counters of the signalling kernels (kept at 0)
};
constexpr int kEpFlagPub = 0, kEpFlagDone = 1;


// Block shape.  All counts in elements.
struct Shape {
  int H;   // hidden
  int I;   // routed expert intermediate
  int Is;  // shared expert intermediate
  int E;   // routed experts
  int K;   // top-k
};

// One layer's device weights, reference layout (src/expert.rs:362-512):
//   router [E][H], gate_up [E][2I][H] (gate rows then up rows),
//   down [E][H][I], shared gate/up [Is][H], shared down [H][Is],
//   shared gate vector [H], optional f32 logit bias [E].
struct LayerWeights {
  const uint16_t* router = nullptr;
  const uint16_t* gate_up = nullptr;
  const uint16_t* down = nullptr;
  const uint16_t* sh_gate = nullptr;
  const uint16_t* sh_up = nullptr;
  const uint16_t* sh_down = nullptr;
  const uint16_t* sh_gate_w = nullptr;
  const float* bias = nullptr;
  // [E] upper bounds of the router rows' 2-norms (prefill router, see
  // launch_router_norms); null without a prefill path.
  const float* router_norm = nullptr;
  // [E+1][H] router rows and the shared gate vector in partial-major order
  // (element (row, j, i) = row[j + 32 i]) for the prefill router's exact
  // repair; null without a prefill path.
  const uint16_t* router_pm = nullptr;
  // Experts held: e with e % ep_world == ep_rank, bank index e / ep_world
  // (expert parallelism interleaves the experts over the GPUs; one GPU
  // holds all of them at their own index).
  int ep_rank = 0, ep_world = 1;
  int expert_count = 0;  // experts held
  // Expert banks in the tiled layout (see TiledSpec) instead of the
  // reference layout; sh_gate then holds the shared gate/up tiles and sh_up
  // is unused.
  bool tiled = false;
};

// Columns per expert-kernel stage for a matrix of k columns (k a multiple
// of 64): the largest multiple of 64 that divides k, at most 512.
__host__ __device__ inline int chunk_cols(int k) {
  for (int c = 512; c >= 64; c -= 64)
    if (k % c == 0) return c;
  return 64;
}

// Tiled expert layout.  A matrix of R x K (reference, row-major) is stored
// as 8-row groups; a group is K/64 segments of 8 rows x 64 columns (1 KB),
// segment-contiguous along K, groups in row order, matrices (experts) in
// order.  Inside a segment, row r occupies bytes r*128 .. r*128+127 and its
// 16-byte chunk j (columns 8j..8j+7) sits at chunk position j ^ r.  Paired
// groups (kind 0) hold the 4 gate rows 4g..4g+3 then the 4 matching up rows
// of a gate_up bank; plain groups (kind 1) hold rows 8g..8g+7.
//   - The decode expert kernel's stage is chunk_cols(K)/64 consecutive
//     segments of one group: one bulk copy, read conflict-free.
//   - A segment is exactly the 128-byte-swizzled K-major operand atom of the
//     sm_100 tensor cores, so a 4-D tensor map (64 columns, 8 rows, K/64
//     segments, groups) brings 16 groups = 128 rows x 64 columns into shared
//     memory in that operand layout with no swizzle of its own.
struct TiledSpec {
  int kind;                // 0: paired gate/up rows, 1: plain rows
  int K;                   // columns
  int half;                // kind 0, one source: up rows start at row `half` of it; 0: two sources
  long long mat_elems;     // elements per matrix (expert) in the tiled buffer
  long long src_mat_elems; // elements per matrix in the reference source
  long long m0 = 0;        // synthetic generation: global index of the bank's matrix 0 ...
  long long m_stride = 1;  // ... and of matrix j: m0 + j * m_stride (interleaved expert placement)
};

// Scratch for one forward of up to max_T tokens (device memory).
struct Scratch {
  uint16_t* logits = nullptr;    // [T][E]
  uint16_t* sh_logit = nullptr;  // [T]
  uint16_t* sh_sig = nullptr;    // [T]
  int32_t* sorted_slot = nullptr;  // [T][K] slots in ascending expert order
  int32_t* sched = nullptr;      // schedule words, see sched_* helpers
  uint16_t* act = nullptr;       // decode: [T*K][2I] gate | up rows (SwiGLU applied on staging);
                                 // prefill: SwiGLU rows K-blocked, [I/64][T*K][64]
  uint16_t* act_sh = nullptr;    // decode: [T][2Is]; prefill: [Is/64][T][64]
  uint16_t* weighted = nullptr;  // [T*K][H]
  uint16_t* gated_sh = nullptr;  // [T][H]
  int* up_done = nullptr;        // [E+1] per-slot SwiGLU completion counters
  int* ticket = nullptr;         // route-kernel completion counter (kept at 0)
  int* err = nullptr;            // device status word
  int max_T = 0;
  // Prefill path (expert-grouped tensor-core GEMMs), see launch_prefill.
  int* pair_count = nullptr;     // [E] pairs per expert (zeroed per forward)
  int* pair_fill = nullptr;      // [E] scatter cursors
  int* pair_offset = nullptr;    // [E+1] first pair of each expert in grouped order
  int* unit_prefix = nullptr;    // [2 phases][2 classes][E+2] GEMM work-unit prefixes per slot (see fw_prefill.cu)
  int32_t* pair_tk = nullptr;    // [T*K] grouped pairs: t*K + top-k position
  uint16_t* xg = nullptr;        // input rows in grouped pair order, K-blocked: [H/64][pair_cap][64]
  long long pair_cap = 0;        // pair rows of xg / act / pair_tk (max_T * K; more under expert parallelism)
  float* router_approx = nullptr;  // [T][E] tensor-core router logits (prefill), before the exact repair
  // Bound of the expert kernels' waits on other CTAs and on peers (ns), and
  // a count added to the expert kernel's up_done targets (0; a test sets it
  // to make that bounded wait expire).
  unsigned long long wait_ns = 2000000000ull;
  int stall = 0;
  // Decode forwards: device ranges the expert kernel's CTAs prefetch into L2
  // when their work is done (the next layer's router rows and shared expert,
  // which do not depend on its input); null / 0 for none.
  const void* prefetch[3] = {};
  unsigned long long prefetch_bytes[3] = {};
};

// Schedule layout inside Scratch::sched (int32 words), written by the route
// kernel for a forward of T tokens:
//   [0]                         n_active
//   [1 .. 1+E)                  active expert ids, ascending (slot order)
//   [1+E .. 2+2E)               pair offsets per slot (n_active+1 used)
//   [2+2E .. 2+2E+T*K)          pair ids grouped by slot, tokens ascending
//   [2+2E+T*K .. +E+2)          expert-kernel up-cost prefix per slot
//   [.. +E+2)                   expert-kernel down-cost prefix per slot
// (slot n_active is the shared expert; prefixes have n_active+2 entries)
inline size_t sched_words(int E, int max_T, int K) {
  return 2 + 2 * static_cast<size_t>(E) + static_cast<size_t>(max_T) * K + 2 * (static_cast<size_t>(E) + 2);
}

// Lookup tables built on the host (bf16(silu(g)) and bf16(sigmoid(g)) for
// every bf16 bit pattern, src/metal_moe.rs:385-392).
struct Luts {
  const uint16_t* silu = nullptr;
  const uint16_t* sigmoid = nullptr;
};

// ---- hyper-connection caller (fw_hc.cu) -------------------------------------
struct HcWeights {
  const uint16_t* norm = nullptr;      // [4H] hc_norm
  const uint16_t* mix_down = nullptr;  // [LR][4H] input_mix_weight_down
  const uint16_t* mix_up = nullptr;    // [4H][LR] input_mix_weight_up
  const uint16_t* inject = nullptr;    // [4][4H] block_inject_weight
  int lowrank = 0;                     // LR (multiple of 32)
};
struct HcScratch {
  uint16_t* normed = nullptr;  // [T][4H]
  uint16_t* down = nullptr;    // [T][LR]
  uint16_t* up = nullptr;      // [T][4H]
  uint16_t* inject = nullptr;  // [T][4]
  uint16_t* mixed = nullptr;   // [T][H] the block input
  uint16_t* inj_w = nullptr;   // [T][4] injection weights
};
// The injection after the block, done in the combine's epilogue:
// out[t][g*H + c] = bf16(post[t][g*H + c] + bf16(y[t][c] * inj_w[t][g])).
struct HcPost {
  const uint16_t* post = nullptr;   // [T][4H] attention output (the residual streams)
  const uint16_t* inj_w = nullptr;  // [T][4]
  uint16_t* out = nullptr;          // [T][4H] layer output
};
// Everything before the block: post [T][4H] -> hs.mixed [T][H], hs.inj_w.
cudaError_t launch_hc_pre(const HcWeights& w, const HcScratch& hs, const Luts& luts, const uint16_t* post, int H,
                          int T, cudaStream_t st);

// Pipeline stages of one block forward (for per-stage timing): router
// logits; route (and, under expert parallelism, publishing this rank's
// tokens); dispatch (grouping the pairs by expert, and bringing every rank's
// selections and the needed token rows under expert parallelism); the expert
// FFNs; the combine (under expert parallelism including the wait for the
// peers' rows).
enum Stage : int { kStageRouter = 0, kStageRoute, kStageDispatch, kStageExperts, kStageCombine, kStages };

// Whole decode-path block for T tokens, stream-ordered.  When stage_events is
// non-null, kStages + 1 events are recorded around the stages.
cudaError_t launch_block(const Shape& s, const LayerWeights& w, const Luts& luts,
                         const Scratch& sc, const uint16_t* x, int T, uint16_t* y,
                         int32_t* topk_idx, uint16_t* topk_score, cudaStream_t st,
                         cudaEvent_t* stage_events = nullptr, const HcPost* hc = nullptr);

// The persistent expert kernel (gate_up + SwiGLU and down + scale for every
// active expert and the shared expert); dynamic shared memory it needs.
size_t experts_smem_bytes(const Shape& s, bool tiled);
// Tokens the expert kernel stages per pass (8, or 4 for wide hidden sizes).
int experts_tokens_per_pass(const Shape& s);
// x / T: the routed pairs' token rows (all ranks' tokens under expert
// parallelism); sh_x / sh_T: the tokens of the shared expert (this rank's).
// ep: expert parallelism over peer memory (routed rows to their owners'
// windows, done flags at the end), or null.
cudaError_t launch_experts(const Shape& s, const LayerWeights& w, const Luts& luts, const Scratch& sc,
                           const uint16_t* x, int T, const uint16_t* topk_score, cudaStream_t st,
                           const uint16_t* sh_x, int sh_T, const EpPeers* ep = nullptr);

// Primitives (the reference crate's functions over device buffers).
cudaError_t launch_linear(const uint16_t* w, const uint16_t* x, int rows, int cols, int T,
                          uint16_t* y, cudaStream_t st);
cudaError_t launch_route(const uint16_t* logits, int T, int E, int K, int32_t* idx,
                         uint16_t* score, int* err, cudaStream_t st);
// out = add_bf16(a, b) elementwise, n elements (src/expert.rs:578).
cudaError_t launch_add_bf16(const uint16_t* a, const uint16_t* b, long long n, uint16_t* out, cudaStream_t st);
cudaError_t launch_swiglu(const uint16_t* gate, const uint16_t* up, long long n,
                          const uint16_t* silu_lut, uint16_t* out, cudaStream_t st);

// ---- prefill path (fw_prefill.cu) ----------------------------------------
// Tensor maps of one layer's tiled banks for the tensor-core GEMMs.
struct PrefillWeightMaps {
  CUtensorMap gate_up;     // routed gate/up bank, 128-row x 64-column boxes
  CUtensorMap down;        // routed down bank
  CUtensorMap sh_gate_up;  // shared expert gate/up
  CUtensorMap sh_down;     // shared expert down
  CUtensorMap router;      // router [E][H] (reference layout), 128-row x 64-column boxes
};
// Tensor maps of the fixed scratch (activations between the two GEMMs).
// Token-tile maps of one operand: boxes of 16, 32, 64, 128 and 256 rows
// (64 columns, 128-byte swizzle); a tile of n rows (a multiple of 16) is
// loaded as the binary decomposition of n, at most five copies.
constexpr int kTokenBoxes = 5;
struct TokenMaps {
  CUtensorMap box[kTokenBoxes];
};
struct PrefillScratchMaps {
  TokenMaps xg;      // [H/64][pair_cap][64] grouped input rows
  TokenMaps act;     // [I/64][pair_cap][64] grouped SwiGLU rows
  TokenMaps act_sh;  // [Is/64][T][64] shared expert SwiGLU rows
};
// Whether the prefill kernels support this shape (H a multiple of 256, 2I
// and 2Is multiples of 128).
bool prefill_supported(const Shape& s);
// Encode the maps (host only; false on failure).
bool make_prefill_weight_maps(const Shape& s, const LayerWeights& w, PrefillWeightMaps* out);
bool make_prefill_scratch_maps(const Shape& s, const Scratch& sc, PrefillScratchMaps* out);
// Whole block for T tokens through the prefill kernels: router, route with
// pair counts, expert grouping, gate_up GEMM (+SwiGLU), down GEMM (+route
// weight / shared gate), combine.  Stage events as launch_block.
cudaError_t launch_prefill(const Shape& s, const LayerWeights& w, const PrefillWeightMaps& wm,
                           const PrefillScratchMaps& sm, const Luts& luts, const Scratch& sc, const uint16_t* x,
                           int T, uint16_t* y, int32_t* topk_idx, uint16_t* topk_score, cudaStream_t st,
                           cudaEvent_t* stage_events = nullptr, const HcPost* hc = nullptr);
// Prefill stages, composed by launch_prefill (one GPU) and by the
// expert-parallel prefill forward (fw_api.cu):
//   front: router + route of T tokens (pair counts when count_pairs);
//   group: pairs of idx [n_pairs] whose expert e has e % ep_world == ep_rank,
//          grouped by bank index e / ep_world (ecount of them), their rows
//          (x_src: row i / K) into xg; counts computed here when count_here;
//          shared expert over sh_T tokens;
//   gemms: gate/up and down GEMMs; weighted rows to out_rows at row t*K+k,
//          or at send_pos[t*K+k] when send_pos is given.
// mid (or null): an event recorded between the router logits and the route.
cudaError_t launch_prefill_front(const Shape& s, const LayerWeights& w, const PrefillWeightMaps& wm,
                                 const Luts& luts, const Scratch& sc, const uint16_t* x, int T, int32_t* topk_idx,
                                 uint16_t* topk_score, bool count_pairs, cudaStream_t st, cudaEvent_t mid = nullptr);
// Per-layer tables of the prefill router (H a multiple of 256): upper
// bounds of the router rows' 2-norms [E] and the partial-major copy of the
// router rows plus the shared gate vector [E+1][H].
cudaError_t launch_router_tables(const uint16_t* w, const uint16_t* extra_row, int E, int H, float* norms,
                                 uint16_t* pm, cudaStream_t st);
// Pair offsets and GEMM work-unit prefixes from the pair counts of ecount
// bank experts (one CTA); counts and scatter cursors are zeroed for the next
// forward.
cudaError_t launch_prefill_offsets(const Shape& s, const Scratch& sc, int ecount, int sh_T, cudaStream_t st);
cudaError_t launch_prefill_group(const Shape& s, const Scratch& sc, const int32_t* idx, int n_pairs,
                                 const uint16_t* x_src, int ep_rank, int ep_world, int ecount, int sh_T,
                                 bool count_here, cudaStream_t st);
// ep: expert parallelism over peer memory (routed rows to their owners'
// windows, done flags after the down GEMM), or null.
cudaError_t launch_prefill_gemms(const Shape& s, const PrefillWeightMaps& wm, const PrefillScratchMaps& smaps,
                                 const Luts& luts, const Scratch& sc, const uint16_t* x_own, int T_own, int ecount,
                                 const uint16_t* score, const int32_t* send_pos, uint16_t* out_rows,
                                 cudaStream_t st, const EpPeers* ep = nullptr);
// Packed positions of weighted rows for the expert-parallel exchange (see
// k_ep_positions): send side over the gathered ids (group = token owner),
// receive side over this rank's ids (group = computing GPU).
cudaError_t launch_ep_positions(const int32_t* idx, int n, int group_len, int me, int world, bool recv,
                                int32_t* pos, int* count, int* offset, cudaStream_t st);

// Stages shared with the decode path (fw_decode.cu).
cudaError_t launch_router(const Shape& s, const LayerWeights& w, const Scratch& sc, const uint16_t* x, int T,
                          cudaStream_t st);
cudaError_t launch_route_block(const Shape& s, const Luts& luts, const Scratch& sc, int T, int32_t* topk_idx,
                               uint16_t* topk_score, bool schedule, int* pair_count, cudaStream_t st);
// Route of a prefill-width forward: one warp per token, selections and
// scores bit-identical to launch_route_block's, pair counts added into
// pair_count (or null); no schedule.
cudaError_t launch_route_prefill(const Shape& s, const Luts& luts, const Scratch& sc, int T, int32_t* topk_idx,
                                 uint16_t* topk_score, int* pair_count, cudaStream_t st);
// ep_idx / ep_world / ep_rows: expert parallelism (rows per source GPU,
// see CombineArgs); null / 0 / null on one GPU.
// row_of: explicit row of every (t, k) in ep_rows (expert-parallel prefill).
// hc: the hyper-connection injection, fused into the epilogue (or null).
// wait: expert parallelism over peer memory: wait (bounded) for every
// rank's done flag before reading the rows (or null).
cudaError_t launch_combine(const Shape& s, const Scratch& sc, int T, uint16_t* y, cudaStream_t st,
                           const int32_t* ep_idx = nullptr, int ep_world = 0, const uint16_t* ep_rows = nullptr,
                           const int32_t* row_of = nullptr, const HcPost* hc = nullptr,
                           const EpPeers* wait = nullptr);
// Expert parallelism: schedule of this rank's experts (e % ep_world ==
// ep_rank) over the gathered selections idx_all [T][K], shared expert over
// sh_T tokens.
cudaError_t launch_ep_schedule(const Shape& s, const Scratch& sc, const int32_t* idx_all, int T, int ep_rank,
                               int ep_world, int sh_T, cudaStream_t st);

// ---- expert parallelism (fw_ep.cu): NCCL, loaded at run time ---------------
// Each returns null on success, else a message.
struct EpComm;
const char* ep_unique_id(unsigned char out[128]);
const char* ep_comm_init(int rank, int world, const unsigned char id[128], EpComm** out);
void ep_comm_destroy(EpComm* c);
// All-gather of every rank's token rows (x_elems each), top-k ids and route
// weights (k_elems each), one NCCL group on `st`.
const char* ep_dispatch(EpComm* c, const uint16_t* x, uint16_t* x_all, size_t x_elems, const int32_t* idx,
                        int32_t* idx_all, const uint16_t* score, uint16_t* score_all, size_t k_elems,
                        cudaStream_t st);
// Block p of `send` (block_elems bf16) to rank p, block p of `recv` from rank p.
const char* ep_combine_exchange(EpComm* c, const uint16_t* send, uint16_t* recv, size_t block_elems,
                                cudaStream_t st);
const char* ep_async_error(EpComm* c);
// Bounded wait for the stream with NCCL failure handling (see fw_ep.cu):
// 0 done, 1 timeout (communicator aborted), 2 NCCL error (aborted),
// 3 CUDA error (*cuda_err).
int ep_bounded_sync(EpComm* c, cudaStream_t st, unsigned long long limit_ns, cudaError_t* cuda_err);
bool ep_comm_aborted(const EpComm* c);
// Row-sized exchange: rows_send[p] rows of `row_elems` bf16 from send at
// row off_send[p] to rank p; rows_recv[p] rows from rank p into recv at
// row off_recv[p] (counts on the host).
const char* ep_exchange_rows(EpComm* c, const uint16_t* send, const int* rows_send, const int* off_send,
                             uint16_t* recv, const int* rows_recv, const int* off_recv, size_t row_elems,
                             cudaStream_t st);

// ---- expert parallelism over peer memory (fw_p2p.cu) ------------------------
struct P2pComm;
// Create this rank's exchange window (for forwards of up to max_tokens
// tokens per rank) and map every rank's; collective over the world ranks'
// processes (they find each other by the 128-byte id).  Null or a message.
const char* p2p_init(int device, int rank, int world, const unsigned char id[128], int max_tokens, int H, int K,
                     P2pComm** out);
void p2p_destroy(P2pComm* c);
size_t p2p_window_bytes(const P2pComm* c);
EpPeers p2p_peers(const P2pComm* c, int t_local, unsigned seq, unsigned long long wait_ns);
uint16_t* p2p_recv(const P2pComm* c);  // this rank's receive area, [max_tokens][K][H]
// Copy this rank's tokens (rows, ids, route weights) into its window and set
// its pub flags.
cudaError_t launch_ep_publish(const EpPeers& p, const uint16_t* x, const int32_t* idx, const uint16_t* score, int* err,
                              cudaStream_t st);
// Decode widths: every rank's ids and weights into idx_all / score_all
// [world*t_local][K], and the rows of tokens with one of this rank's
// experts into x_all [world*t_local][H].
cudaError_t launch_ep_pull(const EpPeers& p, int E, int32_t* idx_all, uint16_t* score_all, uint16_t* x_all, int* err,
                           cudaStream_t st);
// Prefill widths: every rank's ids and weights, and pair counts of this
// rank's experts (count zeroed by the caller) ...
cudaError_t launch_ep_ids(const EpPeers& p, int E, int32_t* idx_all, uint16_t* score_all, int* count, int* err,
                          cudaStream_t st);
// ... then, after the pair offsets, the grouped input rows, each token row
// read once from its owner's window.
cudaError_t launch_ep_scatter(const EpPeers& p, int banks, const int32_t* idx_all, const int* offset, int* fill,
                              int32_t* pair_tk, uint16_t* xg, long long xg_rows, int* err, cudaStream_t st);

// Store a failure message for fw_last_error() (fixed buffer, no allocation);
// returns `code`.
int record_error(int code, const char* msg);

// Attributes of the calling thread's current device, read once per device
// (a process may drive handles on several devices from several threads).
struct DeviceAttrs {
  int sms = 0;         // multiprocessors
  int smem_optin = 0;  // opt-in shared memory per block, bytes
};
cudaError_t current_device_attrs(DeviceAttrs* out);
// Where a handle lives: its device and, under expert parallelism, its rank
// and world (rank 0 of 1 otherwise).
struct HandlePlace {
  int device, rank, world;
};
HandlePlace handle_place(const fw_moe* h);

// Seeded synthetic weights written straight into the tiled layout: element
// d takes the generator value of its reference index under stream
// keys[source] (the same bits fw_moe_synth_layer gives in reference layout).
cudaError_t launch_synth_tiled(const TiledSpec& spec, long long n_mats, uint64_t key0, uint64_t key1, float scale,
                               uint16_t* out, cudaStream_t st);
// Reference-layout matrices [m0, m0 + n) (src0 / src1 hold exactly those
// matrices) into the tiled buffer out (whole tensor).
cudaError_t launch_relayout(const TiledSpec& spec, long long m0, long long n, const uint16_t* src0,
                            const uint16_t* src1, uint16_t* out, cudaStream_t st);

// Seeded synthetic bf16 tensor (identical bits to the CPU generator);
// key = SplitMix64 stream key of (seed, tensor id).
cudaError_t launch_synth(uint64_t key, uint32_t tensor, uint64_t start, uint64_t count,
                         float scale, uint16_t* out, cudaStream_t st);

}  // namespace fw
