/*
 * fw_oracle.c -- CPU oracle for the sparse-MoE block (TEST INFRASTRUCTURE ONLY).
 *
 * A plain-C restatement of the reference crate's CPU arithmetic, used only by
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as the
 * checker.  Every function cites the reference file:line it restates
 * (paths relative to the x3haloed/firewing source tree).
 *
 * Compile with -ffp-contract=off and without fast-math: the reference is
 * Rust, whose `a += b * c` is a rounded multiply followed by a rounded add.
 *
 * Parity status: pinned against the reference's own known-answer tests and
 * the plaintext parts of its committed fixtures (tests/test_oracle_golden.py).
 * The real-weight SHA-256 captures need the 360 GB checkpoint and do not pin
 * here.  exp() is the host libm expf, standing in for Rust's f32::exp.
 */
#include "fw_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* src/expert.rs:315-318 -- RNE by integer add, no NaN/Inf guard. */
uint16_t fwo_to_bf16(float value) {
    uint32_t bits;
    memcpy(&bits, &value, sizeof bits);
    return (uint16_t)((bits + (0x7fffu + ((bits >> 16) & 1u))) >> 16);
}

/* src/expert.rs:320-322 */
float fwo_from_bf16(uint16_t value) {
    uint32_t bits = (uint32_t)value << 16;
    float out;
    memcpy(&out, &bits, sizeof out);
    return out;
}

/* src/expert.rs:514-552 -- PyTorch aarch64 BF16 dot schedule: eight
 * four-lane accumulators over 32-wide blocks, tree +4/+2/+1 over registers,
 * (l0+l1)+(l2+l3), then an 8-wide tail and a scalar tail. */
float fwo_dot_bf16(const uint16_t* left, const uint16_t* right, size_t n) {
    /* acc[4*reg + lane] is the reference's accumulators[reg][lane]: partial
     * j sums the products of columns j, j+32, j+64, ... in order.  The flat
     * layout lets the compiler keep the 32 independent partials in vector
     * registers without changing any rounding. */
    float acc[32];
    for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
    const size_t complete_blocks = n / 32 * 32;
    for (size_t block = 0; block < complete_blocks; block += 32) {
        const uint16_t* l = left + block;
        const uint16_t* r = right + block;
        for (int j = 0; j < 32; ++j) {
            uint32_t lb = (uint32_t)l[j] << 16, rb = (uint32_t)r[j] << 16;
            float lf, rf;
            memcpy(&lf, &lb, sizeof lf);
            memcpy(&rf, &rb, sizeof rf);
            acc[j] += lf * rf;
        }
    }
    /* tree over registers: offset 4, 2, 1 (register r += register r+offset) */
    static const int offsets[3] = {4, 2, 1};
    for (int o = 0; o < 3; ++o) {
        const int offset = offsets[o];
        for (int reg = 0; reg < offset; ++reg) {
            for (int lane = 0; lane < 4; ++lane) acc[4 * reg + lane] += acc[4 * (offset + reg) + lane];
        }
    }
    float reduced = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    const size_t complete_vectors = n / 8 * 8;
    float tail[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (size_t block = complete_blocks; block < complete_vectors; block += 8) {
        for (int lane = 0; lane < 4; ++lane) {
            tail[lane] += fwo_from_bf16(left[block + lane]) * fwo_from_bf16(right[block + lane]);
            tail[lane] +=
                fwo_from_bf16(left[block + 4 + lane]) * fwo_from_bf16(right[block + 4 + lane]);
        }
    }
    reduced += (tail[0] + tail[1]) + (tail[2] + tail[3]);
    for (size_t index = complete_vectors; index < n; ++index) {
        reduced += fwo_from_bf16(left[index]) * fwo_from_bf16(right[index]);
    }
    return reduced;
}

/* src/router.rs:229-236 (forward fold; only used by the known-answer test
 * at src/expert.rs:1246-1263 that shows the two orders differ). */
float fwo_dot_forward(const uint16_t* left, const uint16_t* right, size_t n) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) sum = sum + fwo_from_bf16(left[i]) * fwo_from_bf16(right[i]);
    return sum;
}

/* src/expert.rs:554-560 */
void fwo_linear_bf16(const uint16_t* weight, const uint16_t* input, size_t rows,
                     size_t columns, uint16_t* out) {
    for (size_t r = 0; r < rows; ++r) out[r] = fwo_to_bf16(fwo_dot_bf16(weight + r * columns, input, columns));
}

/* src/expert.rs:562-571 -- silu rounded to bf16 before the multiply. */
void fwo_swiglu_bf16(const uint16_t* gate, const uint16_t* up, size_t n, uint16_t* out) {
    for (size_t i = 0; i < n; ++i) {
        const float g = fwo_from_bf16(gate[i]);
        const float silu = fwo_from_bf16(fwo_to_bf16(g / (1.0f + expf(-g))));
        out[i] = fwo_to_bf16(silu * fwo_from_bf16(up[i]));
    }
}

/* src/expert.rs:573-576 */
uint16_t fwo_sigmoid_bf16(uint16_t value) {
    const float v = fwo_from_bf16(value);
    return fwo_to_bf16(1.0f / (1.0f + expf(-v)));
}

/* src/expert.rs:578-580 */
uint16_t fwo_add_bf16(uint16_t left, uint16_t right) {
    return fwo_to_bf16(fwo_from_bf16(left) + fwo_from_bf16(right));
}

/* src/metal_moe.rs:385-392 -- bf16(silu(g)) for every bf16 bit pattern. */
void fwo_build_silu_lut(uint16_t* lut) {
    for (uint32_t bits = 0; bits < 65536u; ++bits) {
        const float g = fwo_from_bf16((uint16_t)bits);
        lut[bits] = fwo_to_bf16(g / (1.0f + expf(-g)));
    }
}

/* sigmoid_bf16 (src/expert.rs:573-576) tabulated the same way. */
void fwo_build_sigmoid_lut(uint16_t* lut) {
    for (uint32_t bits = 0; bits < 65536u; ++bits) lut[bits] = fwo_sigmoid_bf16((uint16_t)bits);
}

/* f32 total order (Rust f32::total_cmp) restricted to bf16 bit patterns:
 * unsigned key, larger key = larger value, -0 < +0. */
static inline uint32_t total_key(uint16_t bits) {
    return (bits & 0x8000u) ? (uint32_t)(~bits & 0xffffu) : (uint32_t)(bits | 0x8000u);
}

/* Selection order of src/router.rs:241-247: logit descending under
 * total_cmp, ties by ascending index.  Error convention of
 * native/topk_shim.cpp:22-24. */
int fwo_topk_bf16(const uint16_t* values, size_t count, size_t k, int32_t* indices) {
    if (values == NULL || indices == NULL || k == 0 || k > count) return -1;
    /* Partial selection sort: k passes, each taking the best remaining. */
    unsigned char* taken = (unsigned char*)calloc(count, 1);
    if (taken == NULL) return -1;
    for (size_t slot = 0; slot < k; ++slot) {
        size_t best = (size_t)-1;
        uint32_t best_key = 0;
        for (size_t i = 0; i < count; ++i) {
            if (taken[i]) continue;
            const uint32_t key = total_key(values[i]);
            if (best == (size_t)-1 || key > best_key) {
                best = i;
                best_key = key;
            }
        }
        taken[best] = 1;
        indices[slot] = (int32_t)best;
    }
    free(taken);
    return 0;
}

/* src/decoder_layer.rs:278-307 */
int fwo_route(const uint16_t* logits, size_t experts, size_t k, int32_t* indices,
              uint16_t* scores) {
    if (logits == NULL || indices == NULL || scores == NULL || experts == 0) return -1;
    for (size_t e = 0; e < experts; ++e) {
        if (isnan(fwo_from_bf16(logits[e]))) return -1;
    }
    if (fwo_topk_bf16(logits, experts, k, indices) != 0) return -1;
    float* probabilities = (float*)malloc(experts * sizeof(float));
    if (probabilities == NULL) return -1;
    float maximum = -INFINITY;
    for (size_t e = 0; e < experts; ++e) maximum = fmaxf(maximum, fwo_from_bf16(logits[e]));
    float denominator = -0.0f;
    for (size_t e = 0; e < experts; ++e) {
        probabilities[e] = expf(fwo_from_bf16(logits[e]) - maximum);
        denominator = denominator + probabilities[e];
    }
    for (size_t e = 0; e < experts; ++e) probabilities[e] = probabilities[e] / denominator;
    float selected_sum = -0.0f;
    for (size_t s = 0; s < k; ++s) selected_sum = selected_sum + probabilities[indices[s]];
    for (size_t s = 0; s < k; ++s) scores[s] = fwo_to_bf16(probabilities[indices[s]] / selected_sum);
    free(probabilities);
    return 0;
}

/* src/decoder_layer.rs:309-322 -- same set, position-wise equal logits. */
int fwo_equivalent_topk_order(const int32_t* expected, const int32_t* actual, size_t k,
                              const uint16_t* logits) {
    for (size_t i = 0; i < k; ++i) {
        if (logits[expected[i]] != logits[actual[i]]) return 0;
    }
    /* set equality: every expected index appears in actual (k is small). */
    for (size_t i = 0; i < k; ++i) {
        int found = 0;
        for (size_t j = 0; j < k; ++j) found |= (expected[i] == actual[j]);
        if (!found) return 0;
    }
    for (size_t i = 0; i < k; ++i) {
        int found = 0;
        for (size_t j = 0; j < k; ++j) found |= (actual[i] == expected[j]);
        if (!found) return 0;
    }
    return 1;
}

static void router_logits_one(const fwo_shape* s, const fwo_layer* l, const uint16_t* x,
                              uint16_t* logits) {
    const size_t H = (size_t)s->hidden;
    /* src/decoder_layer.rs:460 -- logits via linear_bf16 (PyTorch topology). */
    fwo_linear_bf16(l->router, x, (size_t)s->experts, H, logits);
    if (l->logit_bias != NULL) {
        /* Build-defined extension (no reference counterpart): the Zipf-like
         * bias is added in f32 to the bf16 logit and re-rounded to bf16. */
        for (int32_t e = 0; e < s->experts; ++e)
            logits[e] = fwo_to_bf16(fwo_from_bf16(logits[e]) + l->logit_bias[e]);
    }
}

int fwo_router(const fwo_shape* s, const fwo_layer* l, const uint16_t* x, int32_t tokens,
               int32_t* indices, uint16_t* scores, uint16_t* logits) {
    if (s == NULL || l == NULL || x == NULL || tokens < 0) return -1;
    uint16_t* scratch = (uint16_t*)malloc((size_t)s->experts * sizeof(uint16_t));
    if (scratch == NULL) return -1;
    int rc = 0;
    for (int32_t t = 0; t < tokens && rc == 0; ++t) {
        uint16_t* lg = logits ? logits + (size_t)t * s->experts : scratch;
        router_logits_one(s, l, x + (size_t)t * s->hidden, lg);
        rc = fwo_route(lg, (size_t)s->experts, (size_t)s->top_k, indices + (size_t)t * s->top_k,
                       scores + (size_t)t * s->top_k);
    }
    free(scratch);
    return rc;
}

/* One token through the block: src/decoder_layer.rs:460-586 (route, routed
 * experts in ascending id with a bf16 accumulator rounded after every add,
 * shared expert with sigmoid gate, final bf16 add). */
static int block_one(const fwo_shape* s, const fwo_layer* l, const uint16_t* x, uint16_t* y,
                     int32_t* indices, uint16_t* scores, uint16_t* logits_tap,
                     uint16_t* routed_tap, uint16_t* shared_tap) {
    const size_t H = (size_t)s->hidden, I = (size_t)s->intermediate;
    const size_t Is = (size_t)s->shared_intermediate, E = (size_t)s->experts;
    const size_t K = (size_t)s->top_k;
    size_t big = 2 * I > 2 * Is ? 2 * I : 2 * Is;
    if (H > big) big = H;
    uint16_t* logits = (uint16_t*)malloc(E * sizeof(uint16_t));
    uint16_t* gate_up = (uint16_t*)malloc(big * sizeof(uint16_t));
    uint16_t* act = (uint16_t*)malloc(big * sizeof(uint16_t));
    uint16_t* down = (uint16_t*)malloc(H * sizeof(uint16_t));
    uint16_t* routed = (uint16_t*)malloc(H * sizeof(uint16_t));
    uint16_t* sh_up = (uint16_t*)malloc(big * sizeof(uint16_t));
    int32_t* order = (int32_t*)malloc(K * sizeof(int32_t));
    int rc = 0;
    if (!logits || !gate_up || !act || !down || !routed || !sh_up || !order) {
        rc = -1;
        goto done;
    }
    router_logits_one(s, l, x, logits);
    if (logits_tap) memcpy(logits_tap, logits, E * sizeof(uint16_t));
    if (fwo_route(logits, E, K, indices, scores) != 0) {
        rc = -1;
        goto done;
    }
    /* Execution order: ascending expert id (src/decoder_layer.rs:428-429,
     * tools/generate_mixture_fixture.py:63). */
    for (size_t i = 0; i < K; ++i) order[i] = (int32_t)i;
    for (size_t i = 1; i < K; ++i) {
        int32_t v = order[i];
        size_t j = i;
        while (j > 0 && indices[order[j - 1]] > indices[v]) {
            order[j] = order[j - 1];
            --j;
        }
        order[j] = v;
    }
    for (size_t h = 0; h < H; ++h) routed[h] = fwo_to_bf16(0.0f);
    for (size_t n = 0; n < K; ++n) {
        const int32_t slot = order[n];
        const int32_t e = indices[slot];
        const uint16_t* wgu = l->gate_up[e];
        const uint16_t* wd = l->down[e];
        if (wgu == NULL || wd == NULL) {
            rc = -2;
            goto done;
        }
        /* src/expert.rs:734-751 */
        fwo_linear_bf16(wgu, x, 2 * I, H, gate_up);
        fwo_swiglu_bf16(gate_up, gate_up + I, I, act);
        fwo_linear_bf16(wd, act, H, I, down);
        const float w = fwo_from_bf16(scores[slot]);
        for (size_t h = 0; h < H; ++h) {
            const uint16_t weighted = fwo_to_bf16(fwo_from_bf16(down[h]) * w);
            routed[h] = fwo_add_bf16(routed[h], weighted);
        }
    }
    if (routed_tap) memcpy(routed_tap, routed, H * sizeof(uint16_t));
    /* Shared expert: src/expert.rs:1138-1153, src/decoder_layer.rs:548-586. */
    fwo_linear_bf16(l->shared_gate, x, Is, H, gate_up);
    fwo_linear_bf16(l->shared_up, x, Is, H, sh_up);
    fwo_swiglu_bf16(gate_up, sh_up, Is, act);
    fwo_linear_bf16(l->shared_down, act, H, Is, down);
    uint16_t gate_logit;
    fwo_linear_bf16(l->shared_gate_w, x, 1, H, &gate_logit);
    const float sig = fwo_from_bf16(fwo_sigmoid_bf16(gate_logit));
    for (size_t h = 0; h < H; ++h) {
        const uint16_t gated = fwo_to_bf16(fwo_from_bf16(down[h]) * sig);
        if (shared_tap) shared_tap[h] = gated;
        y[h] = fwo_add_bf16(routed[h], gated);
    }
done:
    free(logits);
    free(gate_up);
    free(act);
    free(down);
    free(routed);
    free(sh_up);
    free(order);
    return rc;
}

typedef struct {
    const fwo_shape* s;
    const fwo_layer* l;
    const uint16_t* x;
    uint16_t* y;
    int32_t* indices;
    uint16_t* scores;
    const fwo_taps* taps;
    int32_t tokens;
    int32_t first, stride; /* tokens first, first+stride, ... */
    int rc;
} block_job;

static void* block_worker(void* arg) {
    block_job* j = (block_job*)arg;
    const size_t H = (size_t)j->s->hidden, E = (size_t)j->s->experts, K = (size_t)j->s->top_k;
    const fwo_taps* taps = j->taps;
    j->rc = 0;
    for (int32_t t = j->first; t < j->tokens; t += j->stride) {
        const int r = block_one(j->s, j->l, j->x + (size_t)t * H, j->y + (size_t)t * H,
                                j->indices + (size_t)t * K, j->scores + (size_t)t * K,
                                taps && taps->logits ? taps->logits + (size_t)t * E : NULL,
                                taps && taps->routed ? taps->routed + (size_t)t * H : NULL,
                                taps && taps->gated_shared ? taps->gated_shared + (size_t)t * H : NULL);
        if (r < j->rc) j->rc = r;
    }
    return NULL;
}

int fwo_block(const fwo_shape* s, const fwo_layer* l, const uint16_t* x, int32_t tokens,
              uint16_t* y, int32_t* indices, uint16_t* scores, const fwo_taps* taps,
              int32_t threads) {
    if (s == NULL || l == NULL || x == NULL || y == NULL || indices == NULL || scores == NULL ||
        tokens < 0 || s->hidden <= 0 || s->intermediate <= 0 || s->shared_intermediate <= 0 ||
        s->experts <= 0 || s->top_k <= 0 || s->top_k > s->experts)
        return -1;
    if (threads < 1) threads = 1;
    if (threads > tokens) threads = tokens > 0 ? tokens : 1;
    if (threads > 256) threads = 256;
    block_job jobs[256];
    pthread_t tids[256];
    for (int32_t i = 0; i < threads; ++i) {
        block_job j = {s, l, x, y, indices, scores, taps, tokens, i, threads, 0};
        jobs[i] = j;
    }
    /* Tokens are independent, so the split does not change any result. */
    int spawned = 1;
    for (int32_t i = 1; i < threads; ++i) {
        if (pthread_create(&tids[i], NULL, block_worker, &jobs[i]) != 0) break;
        ++spawned;
    }
    /* Threads that failed to start leave their tokens to the calling thread. */
    for (int32_t i = spawned; i < threads; ++i) {
        jobs[i].first = i;
        block_worker(&jobs[i]);
    }
    block_worker(&jobs[0]);
    for (int32_t i = 1; i < spawned; ++i) pthread_join(tids[i], NULL);
    int rc = 0;
    for (int32_t i = 0; i < threads; ++i) rc = jobs[i].rc < rc ? jobs[i].rc : rc;
    return rc;
}

/* ---- seeded synthetic data ---- */

/* SplitMix64 finaliser (Steele, Lea, Flood, "Fast splittable pseudorandom
 * number generators", OOPSLA 2014). */
static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static const uint64_t kGamma = 0x9E3779B97F4A7C15ull;

uint64_t fwo_splitmix64_key(uint64_t seed, uint32_t tensor) {
    return mix64(mix64(seed + kGamma) + (uint64_t)tensor * kGamma + kGamma);
}

/* Irwin-Hall(4) over 16-bit uniforms: mean 0, sd sqrt((65536^2-1)/3). */
float fwo_synth_scale(float std) {
    const double sd = sqrt((65536.0 * 65536.0 - 1.0) / 3.0);
    return (float)((double)std / sd);
}

static inline int32_t irwin_hall4(uint64_t h) {
    return (int32_t)(h & 0xffffu) + (int32_t)((h >> 16) & 0xffffu) +
           (int32_t)((h >> 32) & 0xffffu) + (int32_t)(h >> 48) - 131070;
}

void fwo_synth_bf16(uint64_t seed, uint32_t tensor, uint64_t start, size_t count, float scale,
                    uint16_t* out) {
    const uint64_t key = fwo_splitmix64_key(seed, tensor);
    for (size_t i = 0; i < count; ++i) {
        const uint64_t h = mix64(key + (start + i + 1) * kGamma);
        const float v = (float)irwin_hall4(h) * scale;
        out[i] = fwo_to_bf16(v);
    }
}

void fwo_synth_input(uint64_t seed, int32_t rows, int32_t hidden, uint16_t* out) {
    const float scale = fwo_synth_scale(1.0f);
    float* row = (float*)malloc((size_t)hidden * sizeof(float));
    if (row == NULL) return;
    const uint64_t key = fwo_splitmix64_key(seed, 0x1000u);
    for (int32_t r = 0; r < rows; ++r) {
        double sq = 0.0;
        for (int32_t c = 0; c < hidden; ++c) {
            const uint64_t idx = (uint64_t)r * (uint64_t)hidden + (uint64_t)c;
            const uint64_t h = mix64(key + (idx + 1) * kGamma);
            row[c] = (float)irwin_hall4(h) * scale;
            sq += (double)row[c] * (double)row[c];
        }
        const double inv = 1.0 / sqrt(sq / (double)hidden + 1e-6);
        for (int32_t c = 0; c < hidden; ++c)
            out[(size_t)r * hidden + c] = fwo_to_bf16((float)((double)row[c] * inv));
    }
    free(row);
}

void fwo_zipf_bias(int32_t experts, float* out) {
    for (int32_t e = 0; e < experts; ++e) out[e] = (float)(0.5 * log(pow((double)(e + 1), -1.1)));
}

/* src/expert.rs:341-360 */
int fwo_make_hidden(size_t size, const fwo_input_spec* spec, uint16_t* out) {
    if (spec == NULL || out == NULL || spec->modulus <= 0 || spec->divisor <= 0 ||
        spec->sparse_stride == 0)
        return -1;
    for (size_t index = 0; index < size; ++index) {
        const int64_t affine = (int64_t)index * spec->multiplier + spec->add;
        int64_t rem = affine % spec->modulus;
        if (rem < 0) rem += spec->modulus; /* rem_euclid */
        const int64_t raw = rem - spec->center;
        const float value =
            (index % spec->sparse_stride == 0) ? (float)raw / (float)spec->divisor : 0.0f;
        out[index] = fwo_to_bf16(value);
    }
    return 0;
}

/* ---- hyper-connection caller -------------------------------------------- */

/* src/hyper_connection.rs:211-283: four lanes x four interleaved registers
 * x four cascade levels of f32 accumulators, each square rounded before its
 * add (no fused multiply-add). */
float fwo_inner_square_sum(const float* values, size_t n) {
    enum { LANES = 4, INTERLEAVE = 4, LEVELS = 4 };
    const size_t vector_count = n / LANES;
    const size_t cascade_size = vector_count / INTERLEAVE;
    size_t ceil_log2 = 0;
    if (cascade_size > 1) {
        size_t v = cascade_size - 1;
        while (v) { ++ceil_log2; v >>= 1; }
    }
    const size_t level_power = (ceil_log2 / LEVELS) > 4 ? (ceil_log2 / LEVELS) : 4;
    const size_t level_step = (size_t)1 << level_power;
    const size_t level_mask = level_step - 1;
    float acc[LEVELS][INTERLEAVE][LANES];
    memset(acc, 0, sizeof acc);
    size_t index = 0;
    while (index + level_step <= cascade_size) {
        for (size_t s = 0; s < level_step; ++s) {
            for (int r = 0; r < INTERLEAVE; ++r) {
                const size_t base = (index * INTERLEAVE + r) * LANES;
                for (int l = 0; l < LANES; ++l) {
                    const float sq = values[base + l] * values[base + l];
                    acc[0][r][l] = acc[0][r][l] + sq;
                }
            }
            ++index;
        }
        for (int level = 1; level < LEVELS; ++level) {
            for (int r = 0; r < INTERLEAVE; ++r)
                for (int l = 0; l < LANES; ++l) {
                    acc[level][r][l] = acc[level][r][l] + acc[level - 1][r][l];
                    acc[level - 1][r][l] = 0.0f;
                }
            if (index & (level_mask << (level * level_power))) break;
        }
    }
    while (index < cascade_size) {
        for (int r = 0; r < INTERLEAVE; ++r) {
            const size_t base = (index * INTERLEAVE + r) * LANES;
            for (int l = 0; l < LANES; ++l) {
                const float sq = values[base + l] * values[base + l];
                acc[0][r][l] = acc[0][r][l] + sq;
            }
        }
        ++index;
    }
    for (int level = 1; level < LEVELS; ++level)
        for (int r = 0; r < INTERLEAVE; ++r)
            for (int l = 0; l < LANES; ++l) acc[0][r][l] = acc[0][r][l] + acc[level][r][l];
    for (size_t vec = cascade_size * INTERLEAVE; vec < vector_count; ++vec)
        for (int l = 0; l < LANES; ++l) {
            const float v = values[vec * LANES + l];
            const float sq = v * v;
            acc[0][0][l] = acc[0][0][l] + sq;
        }
    for (int r = 1; r < INTERLEAVE; ++r)
        for (int l = 0; l < LANES; ++l) acc[0][0][l] = acc[0][0][l] + acc[0][r][l];
    float result = 0.0f;
    for (size_t i = vector_count * LANES; i < n; ++i) {
        const float sq = values[i] * values[i];
        result = result + sq;
    }
    for (int l = 0; l < LANES; ++l) result = result + acc[0][0][l];
    return result;
}

/* src/hyper_connection.rs:285-303 */
void fwo_grouped_rms(const uint16_t* input, const uint16_t* weight, size_t hidden, size_t groups, float eps,
                     uint16_t* out) {
    float* f = (float*)malloc(hidden * sizeof(float));
    for (size_t g = 0; g < groups; ++g) {
        const uint16_t* in = input + g * hidden;
        for (size_t i = 0; i < hidden; ++i) f[i] = fwo_from_bf16(in[i]);
        const float mean = fwo_inner_square_sum(f, hidden) / (float)hidden;
        const float inverse = 1.0f / sqrtf(mean + eps);
        for (size_t i = 0; i < hidden; ++i) {
            const float scaled = f[i] * inverse;
            const float gain = 1.0f + fwo_from_bf16(weight[g * hidden + i]);
            out[g * hidden + i] = fwo_to_bf16(scaled * gain);
        }
    }
    free(f);
}

/* src/hyper_connection.rs:305-307 */
float fwo_four_stream_mean(const float values[4]) {
    float sum = 0.0f;
    for (int i = 0; i < 4; ++i) sum = sum + values[i];
    return sum / 4.0f;
}

/* src/hyper_connection.rs:309-317 -- silu rounded to bf16. */
static uint16_t silu_bf16(uint16_t v16) {
    const float v = fwo_from_bf16(v16);
    return fwo_to_bf16(v / (1.0f + expf(-v)));
}

/* src/hyper_connection.rs:412-490 */
void fwo_hc_pre(const uint16_t* input, const fwo_hc_layer* layer, size_t hidden, size_t lowrank,
                uint16_t* mixed, uint16_t* injection_weights, uint16_t* normed_out) {
    const size_t HH = 4 * hidden;
    uint16_t* normed = (uint16_t*)malloc(HH * 2);
    uint16_t* down = (uint16_t*)malloc(lowrank * 2);
    uint16_t* up = (uint16_t*)malloc(HH * 2);
    fwo_grouped_rms(input, layer->norm, hidden, 4, 1.0e-6f, normed);
    fwo_linear_bf16(layer->mix_down, normed, lowrank, HH, down);
    for (size_t i = 0; i < lowrank; ++i) down[i] = silu_bf16(fwo_to_bf16(fwo_from_bf16(down[i]) / 4.0f));
    fwo_linear_bf16(layer->mix_up, down, HH, lowrank, up);
    for (size_t c = 0; c < hidden; ++c) {
        float p[4];
        for (int g = 0; g < 4; ++g) {
            const size_t i = g * hidden + c;
            p[g] = fwo_from_bf16(fwo_to_bf16(fwo_from_bf16(fwo_sigmoid_bf16(up[i])) * fwo_from_bf16(normed[i])));
        }
        mixed[c] = fwo_to_bf16(fwo_four_stream_mean(p));
    }
    uint16_t inj[4];
    fwo_linear_bf16(layer->inject, normed, 4, HH, inj);
    for (int g = 0; g < 4; ++g) {
        const uint16_t scaled = fwo_to_bf16(fwo_from_bf16(inj[g]) / 4.0f);
        injection_weights[g] = fwo_to_bf16(2.0f * fwo_from_bf16(fwo_sigmoid_bf16(scaled)));
    }
    if (normed_out) memcpy(normed_out, normed, HH * 2);
    free(normed);
    free(down);
    free(up);
}

/* src/decoder_layer.rs:587-607 */
void fwo_hc_post(const uint16_t* post, const uint16_t* moe, const uint16_t* injection_weights, size_t hidden,
                 uint16_t* out) {
    for (int g = 0; g < 4; ++g)
        for (size_t c = 0; c < hidden; ++c) {
            const uint16_t prod = fwo_to_bf16(fwo_from_bf16(moe[c]) * fwo_from_bf16(injection_weights[g]));
            out[g * hidden + c] = fwo_add_bf16(post[g * hidden + c], prod);
        }
}
