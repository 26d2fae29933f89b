/*
 * b2_kernels.h - thin C ABI over the sm_100a kernels of the decode path.
 *
 * Every entry point takes device pointers, sizes and a CUDA stream (passed as
 * void *), launches asynchronously and returns 0 or a negative att1_status_t
 * code (argument errors are detected on the host before any launch). Kernels
 * report run-time faults (a timed-out wait, a non-finite input) by OR-ing
 * B2_ERR_* bits into a caller-supplied device error word.
 *
 * The host C11 library (att1_infer_*, att1_backend_*) is the only intended
 * caller; these functions are exported so that tests and other hosts can
 * drive single kernels.
 */
#ifndef B2_KERNELS_H
#define B2_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* run-time error bits written into the device error word */
#define B2_ERR_TIMEOUT     0x1  /* a bounded wait gave up */
#define B2_ERR_NONFINITE   0x2  /* non-finite GEMV input vector */
#define B2_ERR_POSITION    0x4  /* position outside the KV capacity */
#define B2_ERR_NAN_LOGITS  0x8  /* NaN in logits (greedy sampler rejects) */
#define B2_ERR_TOKEN       0x10 /* token id outside the vocabulary */

/* ---- quantised weights in device layout ---------------------------------- */
/*
 * q4 "unit" layout: a matrix [rows][cols] is cut into 16-row tiles and
 * 64-column group pairs (two q4 groups of 32). Each (tile, pair) unit is 640
 * contiguous bytes, units ordered tile-major (a tile's column pairs are
 * contiguous): unit(tile, pair) = tile * pairs + pair. Inside a unit:
 *   bytes [0,512):  32 lanes x 16 B; lane l = 4*r + t (r = row in tile mod 8)
 *                   holds words {row r g0, row r+8 g0, row r g1, row r+8 g1};
 *                   byte i of a word = nibble(col 4t+i) | nibble(col 16+4t+i)<<4
 *                   (cols relative to the group), the same 4-bit two's
 *                   complement values as the reference's packed bytes.
 *   bytes [512,640): 8 x float4 {s(r,g0), s(r,g1), s(r+8,g0), s(r+8,g1)}.
 * Padding rows/columns hold zero nibbles and zero scales. The mapping is a
 * permutation of the reference's nibbles (b2_q4_unpack inverts it).
 *
 * q8 unit layout: (16-row tile, 32-column block) units of 512 bytes in the
 * same tile-major order, lane l
 * holds 16 int8 {row r k 4t..4t+3, row r+8 k 4t.., row r k 16+4t.., row r+8
 * k 16+4t..}; one f32 scale per row in a separate array [tiles*16].
 */
#define B2_Q4_UNIT_BYTES 640u
#define B2_Q8_UNIT_BYTES 512u

enum b2_row_map {
    B2_ROWS_PLAIN = 0,   /* device row i = source row i */
    B2_ROWS_GATEUP = 1   /* tile t: rows 0..7 = gate rows 8t.., rows 8..15 = up rows 8t.. */
};

typedef struct b2_qweight {
    const void *data;        /* device units */
    const float *row_scale;  /* q8: device [tiles*16]; q4: NULL */
    uint32_t format;         /* 4 or 8 */
    uint32_t rows, cols;     /* logical device rows (2*F for gate/up) and columns */
    uint32_t tiles;          /* ceil(rows / 16) */
    uint32_t kunits;         /* q4: ceil(cols / 64); q8: ceil(cols / 32) */
} b2_qweight;

size_t b2_q4_bytes(uint32_t rows, uint32_t cols);
size_t b2_q8_bytes(uint32_t rows, uint32_t cols);        /* units only */

/* Reference layout (packed [rows][cols/2] + scales [rows][cols/group]) ->
 * units, written at `tile_offset` tiles into dst. group in {32, 64, 128}.
 * map = B2_ROWS_GATEUP takes src (gate) and src2 (up), each [rows/2][cols]. */
int b2_q4_pack(void *dst, uint32_t tile_offset, uint32_t dst_rows, uint32_t cols,
               const uint8_t *packed, const float *scales,
               const uint8_t *packed2, const float *scales2,
               uint32_t group, int map, void *stream);
/* Units -> reference layout (group 32) of source `which` (0, or 1 = up for
 * B2_ROWS_GATEUP) with `rows` source rows. */
int b2_q4_unpack(uint8_t *packed, float *scales, const void *src, uint32_t tile_offset,
                 uint32_t rows, uint32_t cols, int map, int which, void *stream);
/* Generate N(0, std) weights for tensor (seed, tensor_id) [rows][cols] and
 * quantise them exactly as the reference q4 quantiser (group 32) directly
 * into units. GATEUP: tensor_id = gate, tensor_id2 = up, each [dst_rows/2]. */
int b2_q4_synth(void *dst, uint32_t tile_offset, uint32_t dst_rows, uint32_t cols,
                uint64_t seed, uint64_t tensor_id, uint64_t tensor_id2, float std,
                int map, void *stream);

/* A shard of a generated tensor (tensor parallelism): device row i takes
 * source row src_row0 + i (of each source for GATEUP) and device column j
 * source column src_col0 + j of rows src_cols long. q4 groups stay the
 * reference's 32-column groups (src_col0 % 32 == 0); a q8 row keeps the
 * scale of its whole source row. */
int b2_q4_synth_part(void *dst, uint32_t tile_offset, uint32_t dst_rows, uint32_t cols,
                     uint64_t seed, uint64_t tensor_id, uint64_t tensor_id2, float std, int map,
                     uint32_t src_row0, uint32_t src_col0, uint32_t src_cols, void *stream);
int b2_q8_synth_part(void *dst, float *row_scale, uint32_t tile_offset, uint32_t dst_rows,
                     uint32_t cols, uint64_t seed, uint64_t tensor_id, uint64_t tensor_id2,
                     float std, int map, uint32_t src_row0, uint32_t src_col0, uint32_t src_cols,
                     void *stream);

int b2_q8_pack(void *dst, float *row_scale, uint32_t tile_offset, uint32_t dst_rows,
               uint32_t cols, const int8_t *values, const float *scales,
               const int8_t *values2, const float *scales2, int map, void *stream);
int b2_q8_unpack(int8_t *values, float *scales, const void *src, const float *row_scale,
                 uint32_t tile_offset, uint32_t rows, uint32_t cols, int map, int which,
                 void *stream);
int b2_q8_synth(void *dst, float *row_scale, uint32_t tile_offset, uint32_t dst_rows,
                uint32_t cols, uint64_t seed, uint64_t tensor_id, uint64_t tensor_id2,
                float std, int map, void *stream);

/* Quantise an f32 device matrix per output row by the reference q8 rule
 * (src/quant.c:61-116) into units. transposed = 1 reads w as [cols][rows]
 * (the reference's [in][out] f32 layout, src/infer.c:196-233). */
int b2_q8_quantize_f32(void *dst, float *row_scale, uint32_t tile_offset, uint32_t dst_rows,
                       uint32_t cols, const float *w, const float *w2, int transposed, int map,
                       void *stream);
/* f32 GEMM for the "cuda" backend: dst[rows][cols] = lhs[rows][inner] * rhs[inner][cols]. */
int b2_matmul_f32(float *dst, const float *lhs, const float *rhs, uint32_t rows, uint32_t cols,
                  uint32_t inner, void *stream);

/* dst[m][rows] = lhs[m][cols] * W^T with W in the reference layout (q4:
 * packed [rows][cols/2] + scales [rows][cols/group]; q8: values [rows][cols] +
 * scales [rows]), in the reference's own operation order (att1_matmul_q4xf32,
 * src/quant.c:340-393; att1_matmul_q8xf32, src/matmul_q8.c:3-40: groups and
 * columns in order, sum += x * (q * scale) without contraction), so results
 * equal the reference's bit for bit. One thread per output: the backend
 * vtable uses them for shapes the unit-layout GEMV does not tile (q4 group 16,
 * columns not a multiple of 32); decode uses b2_gemv. */
int b2_matmul_q4_ordered(float *dst, const float *lhs, uint32_t m, uint32_t cols, const uint8_t *packed,
                         const float *scales, uint32_t rows, uint32_t group, void *stream);
int b2_matmul_q8_ordered(float *dst, const float *lhs, uint32_t m, uint32_t cols, const int8_t *values,
                         const float *scales, uint32_t rows, void *stream);

/* f32 tensor of N(0, std) values (bit-identical to the oracle generator). */
int b2_synth_f32(float *dst, size_t count, uint64_t seed, uint64_t tensor_id, float std,
                 void *stream);
int b2_fill_f32(float *dst, size_t count, float value, void *stream);

/* ---- GEMV: y[b][r] = sum_c W[r][c] * prologue(x)[b][c], fused epilogue ---- */
enum b2_epilogue {
    B2_EPI_STORE = 0,   /* out[b][r] = y */
    B2_EPI_RESID = 1,   /* out[b][r] = resid[b][r] + y */
    B2_EPI_QKV = 2,     /* q rows -> out (RoPE); k rows -> K cache (RoPE); v rows -> V cache */
    B2_EPI_SWIGLU = 3,  /* gate/up rows -> out[b][j] = silu(gate) * up */
    B2_EPI_LOGITS = 4,  /* out[b][r] = y and greedy argmax key per item */
    B2_EPI_PUSH = 5     /* tensor parallel: y to every rank's exchange slot (b2_tp) */
};

/* ---- tensor parallelism: partial results exchanged over peer memory ------- */
/*
 * Each rank owns one exchange region (b2_tp_region_bytes) in its device
 * memory that every rank can store to (NVLink peer access or CUDA IPC
 * mappings). Layout: flags [points+1][B2_TP_MAX] u64 | argmax keys
 * [B2_TP_MAX][B2_TP_MAX_ITEMS] u64 | slots [points][B2_TP_MAX][slot_floats] f32 | logits
 * slots [B2_TP_MAX][logit_floats] f32. Rank s contributes to point p by
 * storing into slot (p, s) of every rank and then setting flag (p, s) of
 * every rank to the step epoch + 1; a consumer waits for all flags of p and
 * adds the slots in rank order, so every rank computes the same sum. Point
 * `points` is the logits all-gather (rank s's vocabulary rows in logits slot
 * s, its argmax key in keys[s]).
 */
#define B2_TP_MAX 8
#define B2_TP_NONE 0xFFFFFFFFu
#define B2_TP_MAX_ITEMS 64        /* argmax keys per rank in an exchange region */

typedef struct b2_tp {
    uint32_t rank, world;         /* world 0 or 1: no exchange */
    uint8_t *peer[B2_TP_MAX];     /* every rank's region as mapped on this device; peer[rank] = own */
    uint32_t points;              /* regular exchange points in the region */
    uint32_t slot_floats;         /* floats per regular slot (batch * d_model) */
    uint32_t logit_floats;        /* floats per logits slot (batch * local vocab rows) */
    const uint32_t *epoch;        /* device step counter, equal on every rank (b2_step_end_tp advances it) */
    int32_t *done;                /* device completion counter of this kernel: zero, left zero */
    uint32_t out_point;           /* B2_EPI_PUSH: point this GEMV contributes to (LOGITS: the logits point) */
    uint32_t in_point;            /* prologue input x = in_resid + sum over ranks of slot (in_point, r); or B2_TP_NONE */
    const float *in_resid;        /* [batch][cols] residual added by that prologue */
    float *in_out;                /* [batch][cols]: the prologue stores the summed input here, may be NULL */
    uint32_t row_offset;          /* LOGITS: vocabulary id of local row 0 */
    uint32_t wait_polls;          /* polls of a flag before a wait gives up (B2_ERR_TIMEOUT); 0 = 2^24 */
} b2_tp;

size_t b2_tp_region_bytes(uint32_t points, uint32_t slot_floats, uint32_t logit_floats);

/* The same exchange for the tensor-core GEMM route, as kernels of their own:
 * b2_tp_push writes this rank's partial x[n] into its slot of `point` in every
 * rank's region and publishes the point; b2_tp_sum waits (bounded) until every
 * rank has and writes out = resid + sum of the ranks' slots in rank order
 * (out may equal resid); b2_tp_push_logits writes logits [batch][rows] and the
 * argmax keys into every rank's logits slot and publishes point tp->points,
 * for b2_step_end_tp. n is at most tp->slot_floats, a multiple of 4. No
 * counterpart in the reference, whose decode runs on one CPU process. */
int b2_tp_push(const float *x, uint32_t n, const b2_tp *tp, uint32_t point, void *stream);
int b2_tp_sum(const float *resid, float *out, uint32_t n, const b2_tp *tp, uint32_t point, int32_t *err,
              void *stream);
int b2_tp_push_logits(const float *logits, uint32_t batch, uint32_t rows, const unsigned long long *argmax,
                      const b2_tp *tp, void *stream);

typedef struct b2_kv_layout {
    float *k_pool, *v_pool;       /* page pools of one layer */
    const int32_t *page_table;    /* [batch][pages_per_seq] physical page ids */
    uint32_t page_tokens;         /* tokens per page */
    uint32_t pages_per_seq;
    uint32_t n_kv_heads, head_dim;/* page = [n_kv_heads][page_tokens][head_dim] f32: a head's
                                     tokens contiguous (32 KB runs at 64 tokens x 128 dims) */
} b2_kv_layout;

typedef struct b2_gemv_args {
    b2_qweight w;
    uint32_t batch;               /* 1..16 */
    const float *x;               /* [batch][x_stride] */
    uint32_t x_stride;
    const float *norm_w;          /* RMSNorm gains [cols] (prologue), NULL = none */
    float eps;
    int epilogue;                 /* b2_epilogue */
    float *out;                   /* [batch][out_stride] */
    uint32_t out_stride;
    const float *resid;           /* B2_EPI_RESID */
    /* B2_EPI_QKV */
    uint32_t q_rows, kv_rows;     /* rows [0,q_rows) q, [q_rows, q_rows+kv_rows) k, rest v */
    const float *rope_freq;       /* [head_dim/2], freq[i] = 1/powf(theta, 2i/head_dim) */
    const int32_t *positions;     /* [batch] position of the token being decoded */
    b2_kv_layout kv;
    /* B2_EPI_LOGITS */
    unsigned long long *argmax;   /* [batch] packed (ordered value, ~index) keys */
    /* scratch and counters (b2_gemv_scratch_bytes / b2_gemv_counters_len):
     * reserved; a CTA owns whole tiles, so partial sums stay in shared memory.
     * Counters are zeroed once by the caller and left zero. */
    void *scratch;
    size_t scratch_bytes;
    int32_t *counters;
    uint32_t counters_len;
    int32_t *err;                 /* device error word */
    int pdl;                      /* launch with programmatic dependent launch */
    int grid;                     /* 0 = one CTA per SM */
    b2_tp tp;                     /* tensor parallel exchange (zero = none) */
} b2_gemv_args;

size_t b2_gemv_scratch_bytes(const b2_gemv_args *a);
uint32_t b2_gemv_counters_len(const b2_gemv_args *a);
int b2_gemv(const b2_gemv_args *a, void *stream);


/* ---- single-query attention over the paged KV cache (split over positions) */
typedef struct b2_attn_args {
    uint32_t batch, n_heads, n_kv_heads, head_dim;
    const float *q;               /* [batch][n_heads*head_dim] (RoPE applied) */
    b2_kv_layout kv;
    const int32_t *positions;     /* [batch]: attend positions 0..pos inclusive */
    uint32_t max_ctx;             /* capacity bound used to size the grid */
    float *ctx;                   /* [batch][n_heads*head_dim] */
    void *scratch;                /* chunk partials (any contents) */
    size_t scratch_bytes;
    int32_t *counters;            /* zeroed once by the caller, left zero */
    uint32_t counters_len;
    int32_t *err;
    int pdl;
} b2_attn_args;

size_t b2_attn_scratch_bytes(const b2_attn_args *a);
uint32_t b2_attn_counters_len(const b2_attn_args *a);
int b2_attn(const b2_attn_args *a, void *stream);

/* b2_attn for callers that cannot allocate device memory where they run it:
 * code inside a memory pool or arena it does not own, code that must not
 * synchronise the device (cudaMalloc / cudaFree can), or a host whose
 * allocator is closed to plugins. It has no counterpart in the reference.
 * The split partials and counters come from one fixed array of
 * B2_NOALLOC_SCRATCH_BYTES in device memory (held by every GPU that loads the
 * library until exit); a->scratch and a->counters are ignored, everything
 * else is as for b2_attn, and calls b2_attn would reject are rejected before
 * the array is touched. Plans that need more than the array return
 * ATT1_ERR_UNSUPPORTED (-9). All calls on a device share the array: calls that
 * overlap on the GPU race and must be ordered by the caller. The first call
 * on each device looks up the array's address and should come before any
 * stream capture on that device. Allocates nothing. */
#define B2_NOALLOC_SCRATCH_BYTES (4u << 20)
int b2_attn_noalloc(const b2_attn_args *a, void *stream);

/* ---- per-token step kernels ------------------------------------------------ */
/* x[b] = embed[tokens[b]]; argmax keys reset. Validates token ids. */
int b2_step_begin(const float *embed, uint32_t vocab, uint32_t d_model, const uint32_t *tokens,
                  uint32_t batch, float *x, unsigned long long *argmax, int32_t *err,
                  int pdl, void *stream);
/* tokens[b] = argmax index; positions[b] += 1. */
int b2_step_end(const unsigned long long *argmax, uint32_t batch, uint32_t *tokens,
                int32_t *positions, int32_t *err, int pdl, void *stream);
/* Step end over argmax keys gathered from `world` ranks ([world][batch], e.g.
 * by an all-gather): the largest key per item is the greedy token (keys carry
 * global vocabulary ids); positions advance. */
int b2_step_end_keys(const unsigned long long *keys, uint32_t world, uint32_t batch, uint32_t *tokens,
                     int32_t *positions, int32_t *err, int pdl, void *stream);
/* Tensor parallel step end: waits for every rank's logits flag, takes the
 * largest argmax key over the ranks (the global greedy token), advances the
 * positions and the epoch (tp->epoch is written through a cast). */
int b2_step_end_tp(const b2_tp *tp, uint32_t batch, uint32_t *tokens, int32_t *positions, int32_t *err,
                   int pdl, void *stream);
/* Top-k / temperature sampling after b2_step_end (which has advanced the
 * positions): for item b, the top_k largest logits[b*stride + 0..vocab) by
 * (value desc, id asc), weights w_i = expf((l_i - l_0) / temperature) summed
 * in that order into s, u = (r >> 40) * 2^-24 with
 * r = splitmix64(splitmix64(seed) ^ (b << 32 | positions[b])), and tokens[b]
 * = the first i whose running sum exceeds u * s (the last if none). When the
 * largest logit is +inf the weights are 1 for the +inf entries and 0 for the
 * rest; when it is -inf (all top_k are -inf) the token is the first ranked. The
 * reference declares att1_sampler_config (include/att1_sampler.h:7-10) but
 * samples greedily only (src/sampler.c:5-34); top_k 1 reproduces that. */
#define B2_MAX_TOP_K 256
int b2_sample_topk(const float *logits, uint32_t batch, uint32_t vocab, uint32_t stride, uint32_t top_k,
                   float temperature, unsigned long long seed, const int32_t *positions, uint32_t *tokens,
                   int pdl, void *stream);
/* The same draw over logits split in vocab / shard_rows shards (the
 * tensor-parallel all-gather: one per rank): logit (b, v) at
 * logits[(v / shard_rows) * shard_stride + b * item_stride + v % shard_rows]. */
int b2_sample_topk_sharded(const float *logits, uint32_t batch, uint32_t vocab, uint32_t shard_rows,
                           size_t shard_stride, uint32_t item_stride, uint32_t top_k, float temperature,
                           unsigned long long seed, const int32_t *positions, uint32_t *tokens, int pdl,
                           void *stream);

/* ---- the whole decode step as one persistent launch ------------------------ */
/*
 * One cooperative launch (one CTA per SM) runs the step of b2_step_begin, the
 * per-layer b2_gemv / b2_attn sequence, the lm_head and b2_step_end, with a
 * grid barrier between dependent operations; the weight stream of every
 * GEMV is read ahead across those barriers. Numerically it is the same
 * kernels' arithmetic. The plan owns its scratch, counters and the barrier
 * words; the arguments' scratch, counters, grid and pdl fields are ignored.
 */
typedef struct b2_decode_layer {
    b2_gemv_args qkv, wo, gu, down;  /* as for b2_gemv */
    b2_attn_args attn;               /* as for b2_attn */
} b2_decode_layer;

typedef struct b2_decode_args {
    uint32_t n_layers, batch;
    const b2_decode_layer *layers;   /* host array [n_layers], read at plan creation */
    b2_gemv_args out;                /* lm_head, B2_EPI_LOGITS */
    const float *embed;              /* device [vocab][d_model] */
    uint32_t vocab, d_model;
    const uint32_t *tokens_in;       /* device [batch]: this step's tokens */
    uint32_t *tokens_out;            /* device [batch]: greedy next tokens (may equal tokens_in) */
    int32_t *positions;              /* device [batch]: advanced by one per step */
    unsigned long long *argmax;      /* device [batch]: argmax keys (scratch) */
    float *x;                        /* device [batch][d_model]: the residual stream */
    int32_t *err;                    /* device error word */
} b2_decode_args;

typedef struct b2_decode_plan b2_decode_plan;
/* Checks every operation as its own entry point does, plans one shared-memory
 * carve-up for the step and uploads the operation list (allocates device memory). */
int b2_decode_plan_create(const b2_decode_args *a, b2_decode_plan **out);
/* One decode step: one launch on `stream`. */
int b2_decode_step(b2_decode_plan *p, void *stream);
/* Zeroes the barrier words and counters (after a step that reported an error). */
int b2_decode_reset(b2_decode_plan *p, void *stream);
void b2_decode_plan_destroy(b2_decode_plan *p);

/* ---- dequant GEMM on the tensor cores (prefill, large decode batches) ---- */
/*
 * out[n][o] (= resid[n][o] +) sum_k x[n][k] * W[o][k] for n < m rows of x,
 * W in the unit layout above. Replaces att1_matmul_q4xf32 / _q8xf32
 * (src/quant.c:340-393, src/matmul_q8.c:3-40) when many rows of x share one
 * pass over W (tcgen05.mma, bf16 hi/lo operand splits, f32 accumulation).
 * x is first prepared by b2_gemm_prep (optional RMSNorm of each row with
 * norm_w, as src/norm.c:5-34, then the split into the MMA operand layout)
 * into a buffer of b2_gemm_xs_bytes(m, cols). When the k range is split over
 * CTAs the partial sums need scratch of b2_gemm_scratch_bytes(args).
 */
typedef struct b2_gemm_args {
    b2_qweight w;
    const void *xs;        /* device, b2_gemm_prep output for m rows, w.cols columns */
    uint32_t m;            /* rows of x (tokens) */
    uint32_t epilogue;     /* B2_EPI_STORE or B2_EPI_RESID */
    float *out;            /* device [m][out_stride] */
    uint32_t out_stride;
    const float *resid;    /* B2_EPI_RESID: device [m][out_stride] (may equal out) */
    void *scratch;         /* device, b2_gemm_scratch_bytes */
    size_t scratch_bytes;
    uint32_t splits;       /* k splits; 0 = choose */
    int32_t *err;          /* device error word (timeouts) */
    int pdl;
} b2_gemm_args;

size_t b2_gemm_xs_bytes(uint32_t m, uint32_t cols);
int b2_gemm_prep(const float *x, uint32_t x_stride, uint32_t m, uint32_t cols, const float *norm_w, float eps,
                 void *xs, int32_t *err, void *stream);
size_t b2_gemm_scratch_bytes(const b2_gemm_args *a);
int b2_gemm(const b2_gemm_args *a, void *stream);

/* The GEMV epilogues (QKV: RoPE + KV append; SWIGLU over interleaved gate/up
 * rows; LOGITS: greedy argmax keys) applied to a dense [m][rows] result y,
 * e.g. of b2_gemm. Row n of y is item n: positions[n] and page-table row n. */
typedef struct b2_rows_args {
    uint32_t epilogue;             /* B2_EPI_QKV, B2_EPI_SWIGLU or B2_EPI_LOGITS */
    uint32_t m;                    /* rows of y */
    const float *y;                /* device [m][y_stride] */
    uint32_t y_stride, rows;       /* rows: logical device rows of the weight (q|k|v, gate/up, vocab) */
    float *out;                    /* QKV: q [m][out_stride]; SWIGLU: [m][out_stride]; LOGITS: copy or NULL */
    uint32_t out_stride;
    uint32_t q_rows, kv_rows;      /* QKV */
    const float *rope_freq;
    const int32_t *positions;      /* [m] */
    b2_kv_layout kv;
    unsigned long long *argmax;    /* LOGITS: [m] keys, max-combined (reset by b2_step_begin) */
    uint32_t row_offset;           /* LOGITS: global id of row 0 */
    int32_t *err;
    int pdl;
} b2_rows_args;
int b2_rows_epilogue(const b2_rows_args *a, void *stream);

/* ---- element ops (backend vtable on device buffers) ---------------------- */
int b2_rmsnorm(float *dst, const float *src, const float *w, uint32_t n, float eps, void *stream);
int b2_softmax(float *v, uint32_t n, void *stream);
int b2_rope(float *v, uint32_t n, uint32_t pos, float theta, void *stream);
int b2_swiglu(float *dst, const float *gate, const float *up, uint32_t n, void *stream);
int b2_argmax(const float *v, uint32_t n, unsigned long long *key, void *stream);

/* device properties used for launch shapes */
int b2_sm_count(void);

#ifdef __cplusplus
}
#endif
#endif
