/*
 * att1_oracle.h - CPU restatement of ATT-1's q4/q8 decode path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the
 * B200 kernels: tests, the smoke entry point and the CPU-baseline leg of the
 * bench may load it; the product path (libatt1_b200.so) never links it.
 *
 * Every function restates one reference function with the same operation
 * order, so that results are bit-identical to the reference built with the
 * same compiler flags (pinned by tests against oracle/_ref, which is compiled
 * from the reference sources). Citations are file:line inside ATT-1.
 *
 * Extensions over the reference (each equivalent to a reference computation):
 *   - grouped-query attention: query head h reads KV head h / (H / Hkv).
 *     The reference expands GQA K/V rows into full MHA
 *     (compiler/convert_llama_to_att1.py:288-326); q4/q8 quantise per row, so
 *     expanded rows are byte-identical and give the same arithmetic.
 *   - eps / theta per model instead of the hard-coded 1e-6 / 10000
 *     (src/infer.c:721-722); the block functions already take them
 *     (include/att1_transformer_block.h:10-17).
 *   - batch: B independent sequences, each its own decode state.
 *   - a seeded synthetic weight generator shared bit-for-bit with the GPU.
 */
#ifndef ATT1_ORACLE_H
#define ATT1_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- quantisers (src/quant.c) -------------------------------------------- */
int or_q4_quantize(const float *w, size_t rows, size_t cols, uint32_t group,
                   uint8_t *packed, float *scales);
int or_q8_quantize(const float *w, size_t rows, size_t cols,
                   int8_t *values, float *scales);

/* ---- matmuls (src/quant.c:340-393, src/matmul_q8.c:3-40) ------------------ */
int or_matmul_q4(float *dst, const float *lhs, size_t lhs_rows, size_t cols,
                 const uint8_t *packed, const float *scales, size_t rows,
                 uint32_t group, int threads);
int or_matmul_q8(float *dst, const float *lhs, size_t lhs_rows, size_t cols,
                 const int8_t *values, const float *scales, size_t rows,
                 int threads);

/* ---- f32 ops (src/norm.c, src/rope.c, src/ffn.c, src/sampler.c) ---------- */
int or_rmsnorm(float *dst, const float *src, const float *weight, size_t n,
               float eps);
int or_softmax(float *v, size_t n);
int or_rope(float *v, size_t n, size_t pos, float theta);
int or_swiglu(float *dst, const float *gate, const float *up, size_t n);
int or_argmax(const float *logits, size_t n, uint32_t *out);

/* ---- seeded synthetic data ------------------------------------------------ */
/* Approximately N(0, std): Irwin-Hall sum of twelve 16-bit uniforms taken from
 * three splitmix64 draws of (seed, tensor_id, index). Exact integer sum, one
 * f32 multiply: identical bits on any IEEE-754 machine. */
void or_synth_normal(uint64_t seed, uint64_t tensor_id, uint64_t first,
                     size_t count, float std, float *out);
/* Same values, generated on `threads` threads. */
void or_synth_normal_mt(uint64_t seed, uint64_t tensor_id, uint64_t first, size_t count, float std,
                        float *out, int threads);
uint32_t or_synth_token(uint64_t seed, uint64_t index, uint32_t vocab);
uint64_t or_splitmix64(uint64_t x);

/* ---- decoder -------------------------------------------------------------- */
enum { OR_Q4 = 4, OR_Q8 = 8 };

typedef struct or_config {
    uint32_t vocab, n_layers, n_heads, n_kv_heads, d_model, d_ff, max_seq;
    uint32_t group;        /* q4 group size */
    uint32_t dtype;        /* OR_Q4 or OR_Q8 */
    float eps;             /* block RMSNorm eps */
    float final_eps;       /* output RMSNorm eps */
    float theta;           /* RoPE base */
} or_config;

typedef struct or_model or_model;
typedef struct or_state or_state;

/* Tensor ids of the synthetic generator (shared with the GPU generator). */
enum {
    OR_T_ATTN_NORM = 0, OR_T_WQ = 1, OR_T_WK = 2, OR_T_WV = 3, OR_T_WO = 4,
    OR_T_FFN_NORM = 5, OR_T_GATE = 6, OR_T_UP = 7, OR_T_DOWN = 8,
    OR_T_PER_LAYER = 16
};
#define OR_T_EMBED       0x7F000000ull
#define OR_T_OUTPUT_NORM 0x7F000001ull
#define OR_T_OUTPUT      0x7F000002ull

/* Build a synthetic model: matrices N(0, 0.02), norms 1.0. */
or_model *or_model_synth(const or_config *cfg, uint64_t seed, int threads);
void or_model_free(or_model *m);
const or_config *or_model_config(const or_model *m);
/* Borrowed views of one quantised matrix: kind 0..8 as OR_T_*, layer ignored
 * for the output matrix (kind = 9). */
int or_model_q4_view(const or_model *m, uint32_t layer, uint32_t kind,
                     const uint8_t **packed, const float **scales,
                     size_t *rows, size_t *cols);
int or_model_q8_view(const or_model *m, uint32_t layer, uint32_t kind,
                     const int8_t **values, const float **scales,
                     size_t *rows, size_t *cols);
const float *or_model_f32_view(const or_model *m, uint32_t layer, uint32_t kind);

or_state *or_state_create(const or_model *m);
void or_state_free(or_state *s);
size_t or_state_position(const or_state *s);
/* One decode step (src/infer.c:656-880). logits may be NULL. */
int or_decode(const or_model *m, or_state *s, uint32_t token, float *logits,
              uint32_t *out_token, int threads);
/* Test set-up (no reference counterpart): K/V rows [0, count) of one layer
 * from [count][n_kv_heads][head_dim] arrays, and the position the next decode
 * takes, so a test can start deep in a context without decoding its prefix. */
int or_state_import_kv(const or_model *m, or_state *s, uint32_t layer, size_t count,
                       const float *keys, const float *values);
int or_state_seek(const or_model *m, or_state *s, size_t position);
/* KV views for checks: layer l, [max_seq][n_kv_heads][head_dim]. */
const float *or_state_keys(const or_state *s, uint32_t layer);
const float *or_state_values(const or_state *s, uint32_t layer);

#ifdef __cplusplus
}
#endif
#endif
