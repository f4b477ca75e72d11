/*
 * fw_oracle.h -- CPU oracle for the sparse-MoE block.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * crate's CPU arithmetic for the sparse-MoE block (x3haloed/firewing,
 * src/expert.rs, src/decoder_layer.rs, src/router.rs).  It is the checker the
 * parity tests, smoke() and bench.py's CPU-baseline leg compare the CUDA path
 * against.  Nothing in the product (firewing_b200/, include/) links it.
 *
 * Parity pins: the reference's own known-answer tests (expert.rs:1226-1293,
 * router.rs:415-433, decoder_layer.rs:666-689, metal_moe.rs:668-680) and the
 * plaintext parts of its committed fixtures are replayed against this code by
 * tests/test_oracle_golden.py.
 *
 * Build: see oracle/Makefile (gcc -O3 -ffp-contract=off, no fast-math: the
 * reference is Rust, which never contracts a*b+c into an FMA).
 */
#ifndef FW_ORACLE_H
#define FW_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- bf16 scalar helpers (src/expert.rs:315-322, src/router.rs:126-133) ---- */
uint16_t fwo_to_bf16(float value);
float fwo_from_bf16(uint16_t value);

/* ---- reductions (src/expert.rs:514-560) ---- */
float fwo_dot_bf16(const uint16_t* left, const uint16_t* right, size_t n);
/* Forward scalar sum, as the verifier-variant router uses (src/router.rs:229-236). */
float fwo_dot_forward(const uint16_t* left, const uint16_t* right, size_t n);
void fwo_linear_bf16(const uint16_t* weight, const uint16_t* input, size_t rows,
                     size_t columns, uint16_t* out);

/* ---- elementwise (src/expert.rs:562-580) ---- */
void fwo_swiglu_bf16(const uint16_t* gate, const uint16_t* up, size_t n, uint16_t* out);
uint16_t fwo_sigmoid_bf16(uint16_t value);
uint16_t fwo_add_bf16(uint16_t left, uint16_t right);
/* 65,536-entry tables indexed by bf16 bits (src/metal_moe.rs:385-392). */
void fwo_build_silu_lut(uint16_t* lut);
void fwo_build_sigmoid_lut(uint16_t* lut);

/* ---- routing (src/decoder_layer.rs:278-322, src/router.rs:241-247) ---- */
/* Top-k by (value desc under f32 total order, index asc).  Returns 0 on
 * success, -1 on null pointers, k == 0 or k > count (native/topk_shim.cpp:22). */
int fwo_topk_bf16(const uint16_t* values, size_t count, size_t k, int32_t* indices);
/* The in-layer route: NaN reject, top-k, f32 softmax, renormalised bf16
 * scores.  Returns 0, or -1 when a logit is NaN / arguments are invalid. */
int fwo_route(const uint16_t* logits, size_t experts, size_t k, int32_t* indices,
              uint16_t* scores);
int fwo_equivalent_topk_order(const int32_t* expected, const int32_t* actual, size_t k,
                              const uint16_t* logits);

/* ---- whole block ---- */
typedef struct {
    int32_t hidden;              /* H */
    int32_t intermediate;        /* I, routed expert */
    int32_t shared_intermediate; /* Is */
    int32_t experts;             /* E */
    int32_t top_k;               /* K */
} fwo_shape;

typedef struct {
    const uint16_t* router;          /* [E][H] */
    const uint16_t* const* gate_up;  /* E pointers to [2I][H]; NULL = not resident */
    const uint16_t* const* down;     /* E pointers to [H][I] */
    const uint16_t* shared_gate;     /* [Is][H] */
    const uint16_t* shared_up;       /* [Is][H] */
    const uint16_t* shared_down;     /* [H][Is] */
    const uint16_t* shared_gate_w;   /* [1][H] */
    const float* logit_bias;         /* [E] or NULL (build-defined extension) */
} fwo_layer;

typedef struct {
    uint16_t* logits;        /* [T][E] bf16 router logits (after bias), or NULL */
    uint16_t* routed;        /* [T][H] routed mixture, or NULL */
    uint16_t* gated_shared;  /* [T][H] sigmoid-gated shared expert, or NULL */
} fwo_taps;

/* Router stage only: logits -> (indices, scores) for T tokens. */
int fwo_router(const fwo_shape* shape, const fwo_layer* layer, const uint16_t* x,
               int32_t tokens, int32_t* indices, uint16_t* scores, uint16_t* logits);

/* Whole block for T tokens (each token independent, like the reference's
 * per-token loop at src/decoder_layer3.rs:382-561).  threads > 1 spreads
 * tokens over OpenMP threads; results do not depend on it.
 * Returns 0, -1 (invalid / NaN logits) or -2 (a selected expert has no
 * resident weights). */
int fwo_block(const fwo_shape* shape, const fwo_layer* layer, const uint16_t* x,
              int32_t tokens, uint16_t* y, int32_t* indices, uint16_t* scores,
              const fwo_taps* taps, int32_t threads);

/* ---- seeded synthetic data (shared definition with the CUDA generator) ---- */
uint64_t fwo_splitmix64_key(uint64_t seed, uint32_t tensor);
/* Element i of a tensor: SplitMix64 output i of the stream keyed by
 * (seed, tensor), summed as four 16-bit uniforms (Irwin-Hall, n=4), scaled
 * by an f32 factor and rounded to bf16.  Pure integer arithmetic plus one
 * IEEE f32 multiply, so CPU and GPU produce identical bits. */
float fwo_synth_scale(float std);
void fwo_synth_bf16(uint64_t seed, uint32_t tensor, uint64_t start, size_t count,
                    float scale, uint16_t* out);
/* Inputs: Irwin-Hall N(0,1) stand-in per row, RMS-normalised in f64
 * (x / sqrt(mean(x^2) + 1e-6)), then bf16. */
void fwo_synth_input(uint64_t seed, int32_t rows, int32_t hidden, uint16_t* out);
/* Zipf-like router bias 0.5*ln(rank^-1.1), rank = e + 1, as f32. */
void fwo_zipf_bias(int32_t experts, float* out);

/* ---- deterministic fixture input (src/expert.rs:341-360) ---- */
typedef struct {
    int64_t multiplier, add, modulus, center, divisor;
    uint64_t sparse_stride;
} fwo_input_spec;
int fwo_make_hidden(size_t size, const fwo_input_spec* spec, uint16_t* out);

/* ---- hyper-connection caller of the block (src/hyper_connection.rs,
 *      src/decoder_layer.rs:451-458, 587-607) ---- */
/* PyTorch's contiguous f32 inner square-sum cascade
 * (src/hyper_connection.rs:211-283). */
float fwo_inner_square_sum(const float* values, size_t n);
/* grouped_rms (src/hyper_connection.rs:285-303): per group of `hidden`,
 * bf16(v * (1/sqrt(sum/hidden + eps)) * (1 + w)). */
void fwo_grouped_rms(const uint16_t* input, const uint16_t* weight, size_t hidden, size_t groups, float eps,
                     uint16_t* out);
/* four_stream_mean (src/hyper_connection.rs:305-307): sequential from 0.0. */
float fwo_four_stream_mean(const float values[4]);
/* run_hyper_connection (src/hyper_connection.rs:412-490) for one token:
 * input [4H] -> mixed [H] (the block input) and injection weights [4];
 * normed [4H] optional (NULL to skip). */
typedef struct {
    const uint16_t* norm;      /* [4H] hc_norm */
    const uint16_t* mix_down;  /* [LR][4H] input_mix_weight_down */
    const uint16_t* mix_up;    /* [4H][LR] input_mix_weight_up */
    const uint16_t* inject;    /* [4][4H] block_inject_weight */
} fwo_hc_layer;
void fwo_hc_pre(const uint16_t* input, const fwo_hc_layer* layer, size_t hidden, size_t lowrank,
                uint16_t* mixed, uint16_t* injection_weights, uint16_t* normed);
/* The injection after the block (src/decoder_layer.rs:587-607):
 * out[g*H + c] = add_bf16(post[g*H + c], bf16(moe[c] * w[g])). */
void fwo_hc_post(const uint16_t* post, const uint16_t* moe, const uint16_t* injection_weights, size_t hidden,
                 uint16_t* out);

#ifdef __cplusplus
}
#endif
#endif
