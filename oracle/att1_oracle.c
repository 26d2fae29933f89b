/*
 * att1_oracle.c - CPU restatement of ATT-1's q4/q8 decode path.
 *
 * TEST INFRASTRUCTURE ONLY (see att1_oracle.h). Each function states the
 * reference function it follows (file:line inside ATT-1) and keeps its
 * floating-point operation order, so that results are bit-identical to the
 * reference compiled with the same flags (-O2 -ffp-contract=off).
 */
#include "att1_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ======================================================================== */
/* Quantisers                                                               */
/* ======================================================================== */

static int q4_group_ok(uint32_t g)
{
    /* src/quant.c:120-125: power of two in [16, 128] */
    return g >= 16u && g <= 128u && (g & (g - 1u)) == 0u;
}

/* src/quant.c:297-338 -> :199-226 (quantize_group), :127-146 (group_scale),
 * :148-174 (pack_group). scale = max|x| / 7 (1 if all zero),
 * q = clamp(lroundf(x / scale), -7, 7), low nibble = even element. */
int or_q4_quantize(const float *w, size_t rows, size_t cols, uint32_t group,
                   uint8_t *packed, float *scales)
{
    size_t r, g, i;
    size_t ng;

    if (w == NULL || packed == NULL || scales == NULL || rows == 0 ||
        cols == 0 || !q4_group_ok(group) || (cols & 1u) || cols % group) {
        return -1;
    }
    ng = cols / group;
    for (r = 0; r < rows; r++) {
        for (g = 0; g < ng; g++) {
            const float *src = w + r * cols + g * group;
            uint8_t *dst = packed + r * (cols / 2) + g * (group / 2);
            float max_abs = 0.0f;
            float scale;
            int8_t q[128];

            for (i = 0; i < group; i++) {
                const float a = fabsf(src[i]);
                if (!isfinite(src[i])) {
                    return -1;
                }
                if (a > max_abs) {
                    max_abs = a;
                }
            }
            scale = (max_abs > 0.0f) ? (max_abs / 7.0f) : 1.0f;
            for (i = 0; i < group; i++) {
                long v = lroundf(src[i] / scale);
                if (v > 7) v = 7;
                if (v < -7) v = -7;
                q[i] = (int8_t)v;
            }
            for (i = 0; i < group; i += 2) {
                dst[i / 2] = (uint8_t)(((uint8_t)q[i] & 0x0Fu) |
                                       (((uint8_t)q[i + 1] & 0x0Fu) << 4));
            }
            scales[r * ng + g] = scale;
        }
    }
    return 0;
}

/* src/quant.c:61-116: per-row scale = max|row| / 127 (1 if all zero),
 * q = clamp(lroundf(x / scale), -127, 127). */
int or_q8_quantize(const float *w, size_t rows, size_t cols,
                   int8_t *values, float *scales)
{
    size_t r, c;

    if (w == NULL || values == NULL || scales == NULL || rows == 0 || cols == 0) {
        return -1;
    }
    for (r = 0; r < rows; r++) {
        float max_abs = 0.0f;
        float scale = 1.0f;
        for (c = 0; c < cols; c++) {
            const float v = w[r * cols + c];
            const float a = fabsf(v);
            if (!isfinite(v)) {
                return -1;
            }
            if (a > max_abs) {
                max_abs = a;
            }
        }
        if (max_abs > 0.0f) {
            scale = max_abs / 127.0f;
        }
        scales[r] = scale;
        for (c = 0; c < cols; c++) {
            long q = lroundf(w[r * cols + c] / scale);
            if (q > 127) q = 127;
            if (q < -127) q = -127;
            values[r * cols + c] = (int8_t)q;
        }
    }
    return 0;
}

/* ======================================================================== */
/* Matmuls, row-sliced over threads (each output row keeps the reference's   */
/* sequential accumulation, so the result does not depend on thread count)  */
/* ======================================================================== */

typedef struct mm_job {
    float *dst;
    const float *lhs;
    size_t lhs_rows, cols, rows;
    const uint8_t *packed;
    const int8_t *values;
    const float *scales;
    uint32_t group;
    size_t r0, r1;
} mm_job;

/* src/quant.c:340-393: sum += lhs[j] * ((float)q * scale), groups in order,
 * elements in order within a group (unpack :176-197 sign-extends nibbles). */
static void mm_q4_rows(const mm_job *j)
{
    const size_t ng = j->cols / j->group;
    size_t b, r, g, k;

    for (b = 0; b < j->lhs_rows; b++) {
        const float *x = j->lhs + b * j->cols;
        for (r = j->r0; r < j->r1; r++) {
            float sum = 0.0f;
            for (g = 0; g < ng; g++) {
                const uint8_t *p = j->packed + r * (j->cols / 2) + g * (j->group / 2);
                const float scale = j->scales[r * ng + g];
                const float *xa = x + g * j->group;
                for (k = 0; k < j->group; k += 2) {
                    const uint8_t byte = p[k / 2];
                    const uint8_t lo = byte & 0x0Fu;
                    const uint8_t hi = (byte >> 4) & 0x0Fu;
                    const int8_t qlo = (lo & 0x08u) ? (int8_t)(lo | 0xF0u) : (int8_t)lo;
                    const int8_t qhi = (hi & 0x08u) ? (int8_t)(hi | 0xF0u) : (int8_t)hi;
                    sum += xa[k] * ((float)qlo * scale);
                    sum += xa[k + 1] * ((float)qhi * scale);
                }
            }
            j->dst[b * j->rows + r] = sum;
        }
    }
}

/* src/matmul_q8.c:3-40: sum += lhs[c] * ((float)q * row_scale). */
static void mm_q8_rows(const mm_job *j)
{
    size_t b, r, c;

    for (b = 0; b < j->lhs_rows; b++) {
        const float *x = j->lhs + b * j->cols;
        for (r = j->r0; r < j->r1; r++) {
            const float scale = j->scales[r];
            const int8_t *q = j->values + r * j->cols;
            float sum = 0.0f;
            for (c = 0; c < j->cols; c++) {
                sum += x[c] * ((float)q[c] * scale);
            }
            j->dst[b * j->rows + r] = sum;
        }
    }
}

static void *mm_thread(void *arg)
{
    const mm_job *j = (const mm_job *)arg;
    if (j->packed != NULL) {
        mm_q4_rows(j);
    } else {
        mm_q8_rows(j);
    }
    return NULL;
}

static int mm_run(mm_job *base, int threads)
{
    mm_job jobs[256];
    pthread_t tid[256];
    int started[256];
    int n, t;

    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if ((size_t)threads > base->rows) threads = (int)base->rows;
    n = threads;
    if (n == 1) {
        base->r0 = 0;
        base->r1 = base->rows;
        mm_thread(base);
        return 0;
    }
    for (t = 0; t < n; t++) {
        jobs[t] = *base;
        jobs[t].r0 = base->rows * (size_t)t / (size_t)n;
        jobs[t].r1 = base->rows * (size_t)(t + 1) / (size_t)n;
        started[t] = (pthread_create(&tid[t], NULL, mm_thread, &jobs[t]) == 0);
        if (!started[t]) {
            mm_thread(&jobs[t]);
        }
    }
    for (t = 0; t < n; t++) {
        if (started[t]) {
            pthread_join(tid[t], NULL);
        }
    }
    return 0;
}

int or_matmul_q4(float *dst, const float *lhs, size_t lhs_rows, size_t cols,
                 const uint8_t *packed, const float *scales, size_t rows,
                 uint32_t group, int threads)
{
    mm_job j;

    if (dst == NULL || lhs == NULL || packed == NULL || scales == NULL ||
        lhs_rows == 0 || cols == 0 || rows == 0 || !q4_group_ok(group) ||
        cols % group) {
        return -1;
    }
    memset(&j, 0, sizeof(j));
    j.dst = dst; j.lhs = lhs; j.lhs_rows = lhs_rows; j.cols = cols;
    j.rows = rows; j.packed = packed; j.scales = scales; j.group = group;
    return mm_run(&j, threads);
}

int or_matmul_q8(float *dst, const float *lhs, size_t lhs_rows, size_t cols,
                 const int8_t *values, const float *scales, size_t rows,
                 int threads)
{
    mm_job j;

    if (dst == NULL || lhs == NULL || values == NULL || scales == NULL ||
        lhs_rows == 0 || cols == 0 || rows == 0) {
        return -1;
    }
    memset(&j, 0, sizeof(j));
    j.dst = dst; j.lhs = lhs; j.lhs_rows = lhs_rows; j.cols = cols;
    j.rows = rows; j.values = values; j.scales = scales;
    return mm_run(&j, threads);
}

/* ======================================================================== */
/* f32 ops                                                                  */
/* ======================================================================== */

/* src/norm.c:5-34: scale = 1 / sqrtf(sum(x^2)/n + eps); y = x * scale * w. */
int or_rmsnorm(float *dst, const float *src, const float *weight, size_t n,
               float eps)
{
    float ss = 0.0f;
    float scale;
    size_t i;

    if (dst == NULL || src == NULL || weight == NULL || n == 0 || eps <= 0.0f) {
        return -1;
    }
    for (i = 0; i < n; i++) {
        ss += src[i] * src[i];
    }
    scale = 1.0f / sqrtf((ss / (float)n) + eps);
    for (i = 0; i < n; i++) {
        dst[i] = src[i] * scale * weight[i];
    }
    return 0;
}

/* src/norm.c:36-71: max-subtract, expf, sum, divide. */
int or_softmax(float *v, size_t n)
{
    float mx, sum = 0.0f;
    size_t i;

    if (v == NULL || n == 0) {
        return -1;
    }
    mx = v[0];
    for (i = 1; i < n; i++) {
        if (v[i] > mx) mx = v[i];
    }
    for (i = 0; i < n; i++) {
        v[i] = expf(v[i] - mx);
        sum += v[i];
    }
    if (sum == 0.0f) {
        return -1;
    }
    for (i = 0; i < n; i++) {
        v[i] /= sum;
    }
    return 0;
}

/* src/rope.c:5-34: interleaved pairs (i, i+1), i even;
 * angle = pos * (1 / powf(theta, i / n)). */
int or_rope(float *v, size_t n, size_t pos, float theta)
{
    size_t i;

    if (v == NULL || n == 0 || (n % 2u) != 0 || theta <= 0.0f) {
        return -1;
    }
    for (i = 0; i < n; i += 2) {
        const float exponent = (float)i / (float)n;
        const float freq = 1.0f / powf(theta, exponent);
        const float angle = (float)pos * freq;
        const float c = cosf(angle);
        const float s = sinf(angle);
        const float x0 = v[i];
        const float x1 = v[i + 1];
        v[i] = (x0 * c) - (x1 * s);
        v[i + 1] = (x0 * s) + (x1 * c);
    }
    return 0;
}

/* src/ffn.c:5-30: silu(g) = g / (1 + expf(-g)); y = silu(g) * up. */
int or_swiglu(float *dst, const float *gate, const float *up, size_t n)
{
    size_t i;

    if (dst == NULL || gate == NULL || up == NULL || n == 0) {
        return -1;
    }
    for (i = 0; i < n; i++) {
        const float g = gate[i];
        dst[i] = (g / (1.0f + expf(-g))) * up[i];
    }
    return 0;
}

/* src/sampler.c:5-34: NaN anywhere -> error; lowest index wins ties. */
int or_argmax(const float *logits, size_t n, uint32_t *out)
{
    size_t i, best = 0;

    if (logits == NULL || out == NULL || n == 0) {
        return -1;
    }
    for (i = 0; i < n; i++) {
        if (isnan(logits[i])) {
            return -1;
        }
    }
    for (i = 1; i < n; i++) {
        if (logits[i] > logits[best]) {
            best = i;
        }
    }
    *out = (uint32_t)best;
    return 0;
}

/* ======================================================================== */
/* Synthetic data                                                           */
/* ======================================================================== */

uint64_t or_splitmix64(uint64_t x)
{
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint64_t synth_key(uint64_t seed, uint64_t tensor_id)
{
    return or_splitmix64(or_splitmix64(seed) ^ (tensor_id * 0xD1B54A32D192ED03ull));
}

static uint32_t sum16x4(uint64_t r)
{
    return (uint32_t)(r & 0xFFFFu) + (uint32_t)((r >> 16) & 0xFFFFu) +
           (uint32_t)((r >> 32) & 0xFFFFu) + (uint32_t)(r >> 48);
}

void or_synth_normal(uint64_t seed, uint64_t tensor_id, uint64_t first,
                     size_t count, float std, float *out)
{
    const uint64_t key = synth_key(seed, tensor_id);
    const float c = std * (1.0f / 131072.0f);
    size_t i;

    for (i = 0; i < count; i++) {
        const uint64_t e = first + i;
        const uint32_t s = sum16x4(or_splitmix64(key + 3u * e)) +
                           sum16x4(or_splitmix64(key + 3u * e + 1u)) +
                           sum16x4(or_splitmix64(key + 3u * e + 2u));
        /* 12 uniforms on [0, 65535]: mean 393210, sd ~65536 */
        out[i] = (float)((int32_t)(2u * s) - 786420) * c;
    }
}

typedef struct synth_job {
    uint64_t seed, tid, first;
    size_t count;
    float std;
    float *out;
} synth_job;

static void *synth_thread(void *arg)
{
    const synth_job *j = (const synth_job *)arg;
    or_synth_normal(j->seed, j->tid, j->first, j->count, j->std, j->out);
    return NULL;
}

void or_synth_normal_mt(uint64_t seed, uint64_t tensor_id, uint64_t first, size_t count, float std,
                        float *out, int threads)
{
    synth_job jobs[64];
    pthread_t tid[64];
    int started[64];
    int n = threads < 1 ? 1 : (threads > 64 ? 64 : threads), t;
    if (count < 65536 || n == 1) {
        or_synth_normal(seed, tensor_id, first, count, std, out);
        return;
    }
    for (t = 0; t < n; t++) {
        const size_t a = count * (size_t)t / (size_t)n, b = count * (size_t)(t + 1) / (size_t)n;
        jobs[t].seed = seed; jobs[t].tid = tensor_id; jobs[t].first = first + a;
        jobs[t].count = b - a; jobs[t].std = std; jobs[t].out = out + a;
        started[t] = pthread_create(&tid[t], NULL, synth_thread, &jobs[t]) == 0;
        if (!started[t]) synth_thread(&jobs[t]);
    }
    for (t = 0; t < n; t++)
        if (started[t]) pthread_join(tid[t], NULL);
}

uint32_t or_synth_token(uint64_t seed, uint64_t index, uint32_t vocab)
{
    const uint64_t r = or_splitmix64(synth_key(seed, 0x70000000ull) + index);
    return (uint32_t)((r >> 32) % vocab);
}

/* ======================================================================== */
/* Decoder                                                                  */
/* ======================================================================== */

typedef struct or_mat {
    size_t rows, cols;
    uint8_t *packed;   /* q4 */
    int8_t *values;    /* q8 */
    float *scales;
} or_mat;

typedef struct or_layer {
    float *attn_norm, *ffn_norm;
    or_mat w[9]; /* indexed by OR_T_*; slots 0 and 5 unused */
} or_layer;

struct or_model {
    or_config cfg;
    uint32_t head_dim;
    float *embed;
    float *out_norm;
    or_layer *layers;
    or_mat output;
};

struct or_state {
    size_t pos;
    size_t n_layers;
    float **keys, **values;     /* per layer [max_seq][Hkv][hd] */
    float *x, *xn, *q, *k, *v, *ctx, *att, *h1, *gate, *up, *hs, *tmp, *scores;
};

/* Rows quantise independently (per row, or per group inside a row), so a
 * matrix is cut into row ranges quantised on their own threads; the bytes are
 * those of one call over the whole matrix. */
typedef struct quant_job {
    const float *w;
    size_t rows, cols;
    uint32_t group, dtype;
    uint8_t *packed;
    int8_t *values;
    float *scales;
    int rc;
} quant_job;

static void *quant_thread(void *arg)
{
    quant_job *j = arg;
    j->rc = j->dtype == OR_Q4 ? or_q4_quantize(j->w, j->rows, j->cols, j->group, j->packed, j->scales)
                              : or_q8_quantize(j->w, j->rows, j->cols, j->values, j->scales);
    return NULL;
}

static int quantize_mt(const float *w, size_t rows, size_t cols, const or_config *cfg, or_mat *m, int threads)
{
    quant_job jobs[64];
    pthread_t tid[64];
    int started[64];
    size_t per, r0;
    int t, n, rc = 0;
    if (threads < 1) threads = 1;
    if (threads > 64) threads = 64;
    if ((size_t)threads > rows) threads = (int)rows;
    per = (rows + (size_t)threads - 1) / (size_t)threads;
    for (n = 0, r0 = 0; r0 < rows; n++, r0 += per) {
        const size_t r = rows - r0 < per ? rows - r0 : per;
        quant_job *j = &jobs[n];
        j->w = w + r0 * cols;
        j->rows = r;
        j->cols = cols;
        j->group = cfg->group;
        j->dtype = cfg->dtype;
        j->packed = m->packed ? m->packed + r0 * cols / 2 : NULL;
        j->values = m->values ? m->values + r0 * cols : NULL;
        j->scales = cfg->dtype == OR_Q4 ? m->scales + r0 * (cols / cfg->group) : m->scales + r0;
        j->rc = -1;
    }
    for (t = 0; t < n; t++) started[t] = pthread_create(&tid[t], NULL, quant_thread, &jobs[t]) == 0;
    for (t = 0; t < n; t++) {
        if (started[t]) pthread_join(tid[t], NULL);
        else quant_thread(&jobs[t]);
        if (jobs[t].rc != 0) rc = -1;
    }
    return rc;
}

static int mat_build(or_mat *m, const or_config *cfg, uint64_t seed,
                     uint64_t tid, size_t rows, size_t cols, int threads)
{
    float *w = malloc(rows * cols * sizeof(float));
    int rc;
    if (w == NULL) {
        return -1;
    }
    or_synth_normal_mt(seed, tid, 0, rows * cols, 0.02f, w, threads);
    m->rows = rows;
    m->cols = cols;
    if (cfg->dtype == OR_Q4) {
        m->packed = malloc(rows * cols / 2);
        m->scales = malloc(rows * (cols / cfg->group) * sizeof(float));
        rc = (m->packed && m->scales) ? quantize_mt(w, rows, cols, cfg, m, threads) : -1;
    } else {
        m->values = malloc(rows * cols);
        m->scales = malloc(rows * sizeof(float));
        rc = (m->values && m->scales) ? quantize_mt(w, rows, cols, cfg, m, threads) : -1;
    }
    free(w);
    return rc;
}

static void mat_free(or_mat *m)
{
    free(m->packed);
    free(m->values);
    free(m->scales);
    memset(m, 0, sizeof(*m));
}

static float *ones(size_t n)
{
    float *p = malloc(n * sizeof(float));
    size_t i;
    if (p != NULL) {
        for (i = 0; i < n; i++) p[i] = 1.0f;
    }
    return p;
}

or_model *or_model_synth(const or_config *cfg, uint64_t seed, int threads)
{
    or_model *m;
    uint32_t l;
    size_t d, hd, qd, kvd, f;

    if (cfg == NULL || cfg->n_heads == 0 || cfg->n_kv_heads == 0 ||
        cfg->d_model % cfg->n_heads || cfg->n_heads % cfg->n_kv_heads ||
        (cfg->dtype != OR_Q4 && cfg->dtype != OR_Q8)) {
        return NULL;
    }
    m = calloc(1, sizeof(*m));
    if (m == NULL) return NULL;
    m->cfg = *cfg;
    d = cfg->d_model;
    hd = d / cfg->n_heads;
    m->head_dim = (uint32_t)hd;
    qd = hd * cfg->n_heads;
    kvd = hd * cfg->n_kv_heads;
    f = cfg->d_ff;
    m->embed = malloc((size_t)cfg->vocab * d * sizeof(float));
    m->out_norm = ones(d);
    m->layers = calloc(cfg->n_layers, sizeof(or_layer));
    if (!m->embed || !m->out_norm || !m->layers) goto fail;
    or_synth_normal_mt(seed, OR_T_EMBED, 0, (size_t)cfg->vocab * d, 0.02f, m->embed, threads);
    for (l = 0; l < cfg->n_layers; l++) {
        or_layer *L = &m->layers[l];
        const uint64_t base = (uint64_t)l * OR_T_PER_LAYER;
        L->attn_norm = ones(d);
        L->ffn_norm = ones(d);
        if (!L->attn_norm || !L->ffn_norm) goto fail;
        if (mat_build(&L->w[OR_T_WQ], cfg, seed, base + OR_T_WQ, qd, d, threads) ||
            mat_build(&L->w[OR_T_WK], cfg, seed, base + OR_T_WK, kvd, d, threads) ||
            mat_build(&L->w[OR_T_WV], cfg, seed, base + OR_T_WV, kvd, d, threads) ||
            mat_build(&L->w[OR_T_WO], cfg, seed, base + OR_T_WO, d, qd, threads) ||
            mat_build(&L->w[OR_T_GATE], cfg, seed, base + OR_T_GATE, f, d, threads) ||
            mat_build(&L->w[OR_T_UP], cfg, seed, base + OR_T_UP, f, d, threads) ||
            mat_build(&L->w[OR_T_DOWN], cfg, seed, base + OR_T_DOWN, d, f, threads)) {
            goto fail;
        }
    }
    if (mat_build(&m->output, cfg, seed, OR_T_OUTPUT, cfg->vocab, d, threads)) goto fail;
    return m;
fail:
    or_model_free(m);
    return NULL;
}

void or_model_free(or_model *m)
{
    uint32_t l;
    int k;
    if (m == NULL) return;
    if (m->layers != NULL) {
        for (l = 0; l < m->cfg.n_layers; l++) {
            free(m->layers[l].attn_norm);
            free(m->layers[l].ffn_norm);
            for (k = 0; k < 9; k++) mat_free(&m->layers[l].w[k]);
        }
    }
    free(m->layers);
    free(m->embed);
    free(m->out_norm);
    mat_free(&m->output);
    free(m);
}

const or_config *or_model_config(const or_model *m)
{
    return m ? &m->cfg : NULL;
}

static const or_mat *model_mat(const or_model *m, uint32_t layer, uint32_t kind)
{
    if (m == NULL) return NULL;
    if (kind == 9) return &m->output;
    if (layer >= m->cfg.n_layers || kind >= 9 || kind == OR_T_ATTN_NORM ||
        kind == OR_T_FFN_NORM) {
        return NULL;
    }
    return &m->layers[layer].w[kind];
}

int or_model_q4_view(const or_model *m, uint32_t layer, uint32_t kind,
                     const uint8_t **packed, const float **scales,
                     size_t *rows, size_t *cols)
{
    const or_mat *w = model_mat(m, layer, kind);
    if (w == NULL || w->packed == NULL) return -1;
    *packed = w->packed; *scales = w->scales; *rows = w->rows; *cols = w->cols;
    return 0;
}

int or_model_q8_view(const or_model *m, uint32_t layer, uint32_t kind,
                     const int8_t **values, const float **scales,
                     size_t *rows, size_t *cols)
{
    const or_mat *w = model_mat(m, layer, kind);
    if (w == NULL || w->values == NULL) return -1;
    *values = w->values; *scales = w->scales; *rows = w->rows; *cols = w->cols;
    return 0;
}

const float *or_model_f32_view(const or_model *m, uint32_t layer, uint32_t kind)
{
    if (m == NULL) return NULL;
    if (kind == OR_T_EMBED) return m->embed;
    if (kind == OR_T_OUTPUT_NORM) return m->out_norm;
    if (layer >= m->cfg.n_layers) return NULL;
    if (kind == OR_T_ATTN_NORM) return m->layers[layer].attn_norm;
    if (kind == OR_T_FFN_NORM) return m->layers[layer].ffn_norm;
    return NULL;
}

or_state *or_state_create(const or_model *m)
{
    or_state *s;
    const or_config *c;
    size_t kvd, qd, l;
    if (m == NULL) return NULL;
    c = &m->cfg;
    s = calloc(1, sizeof(*s));
    if (s == NULL) return NULL;
    kvd = (size_t)m->head_dim * c->n_kv_heads;
    qd = (size_t)m->head_dim * c->n_heads;
    s->keys = calloc(c->n_layers, sizeof(float *));
    s->values = calloc(c->n_layers, sizeof(float *));
    if (!s->keys || !s->values) goto fail;
    s->n_layers = c->n_layers;
    for (l = 0; l < c->n_layers; l++) {
        s->keys[l] = calloc((size_t)c->max_seq * kvd, sizeof(float));
        s->values[l] = calloc((size_t)c->max_seq * kvd, sizeof(float));
        if (!s->keys[l] || !s->values[l]) goto fail;
    }
    s->x = calloc(c->d_model, sizeof(float));
    s->xn = calloc(c->d_model, sizeof(float));
    s->q = calloc(qd, sizeof(float));
    s->k = calloc(kvd, sizeof(float));
    s->v = calloc(kvd, sizeof(float));
    s->ctx = calloc(qd, sizeof(float));
    s->att = calloc(c->d_model, sizeof(float));
    s->h1 = calloc(c->d_model, sizeof(float));
    s->gate = calloc(c->d_ff, sizeof(float));
    s->up = calloc(c->d_ff, sizeof(float));
    s->hs = calloc(c->d_ff, sizeof(float));
    s->tmp = calloc(c->d_model, sizeof(float));
    s->scores = calloc(c->max_seq, sizeof(float));
    if (!s->x || !s->xn || !s->q || !s->k || !s->v || !s->ctx || !s->att ||
        !s->h1 || !s->gate || !s->up || !s->hs || !s->tmp || !s->scores) goto fail;
    return s;
fail:
    s->pos = 0;
    or_state_free(s);
    return NULL;
}

void or_state_free(or_state *s)
{
    size_t l;
    if (s == NULL) return;
    for (l = 0; l < s->n_layers; l++) {
        if (s->keys) free(s->keys[l]);
        if (s->values) free(s->values[l]);
    }
    free(s->keys); free(s->values);
    free(s->x); free(s->xn); free(s->q); free(s->k); free(s->v); free(s->ctx);
    free(s->att); free(s->h1); free(s->gate); free(s->up); free(s->hs);
    free(s->tmp); free(s->scores);
    free(s);
}

size_t or_state_position(const or_state *s)
{
    return s ? s->pos : 0;
}

const float *or_state_keys(const or_state *s, uint32_t layer)
{
    return s ? s->keys[layer] : NULL;
}

const float *or_state_values(const or_state *s, uint32_t layer)
{
    return s ? s->values[layer] : NULL;
}

/* Test set-up, no reference counterpart: write K/V rows [0, count) of one layer
 * ([count][Hkv][hd], the layer's own layout) and continue at a position, so a
 * parity test can start deep in the context without decoding its prefix. */
int or_state_import_kv(const or_model *m, or_state *s, uint32_t layer, size_t count,
                       const float *keys, const float *values)
{
    size_t kvd;
    if (m == NULL || s == NULL || keys == NULL || values == NULL || layer >= m->cfg.n_layers ||
        count > m->cfg.max_seq)
        return -1;
    kvd = (size_t)m->head_dim * m->cfg.n_kv_heads;
    memcpy(s->keys[layer], keys, count * kvd * sizeof(float));
    memcpy(s->values[layer], values, count * kvd * sizeof(float));
    return 0;
}

int or_state_seek(const or_model *m, or_state *s, size_t position)
{
    if (m == NULL || s == NULL || position >= m->cfg.max_seq) return -1;
    s->pos = position;
    return 0;
}

static int mat_apply(const or_model *m, const or_mat *w, float *dst,
                     const float *x, int threads)
{
    if (m->cfg.dtype == OR_Q4) {
        return or_matmul_q4(dst, x, 1, w->cols, w->packed, w->scales, w->rows,
                            m->cfg.group, threads);
    }
    return or_matmul_q8(dst, x, 1, w->cols, w->values, w->scales, w->rows,
                        threads);
}

/* src/infer.c:656-880 with the block of src/transformer_block.c:417-557 and
 * the attention of src/attention.c:435-556 (GQA head mapping, see header). */
int or_decode(const or_model *m, or_state *s, uint32_t token, float *logits,
              uint32_t *out_token, int threads)
{
    const or_config *c;
    size_t d, hd, H, Hkv, grp, kvd, i, h, p, l;
    float inv_sqrt;
    float *lg;
    int rc;

    if (m == NULL || s == NULL) return -1;
    c = &m->cfg;
    if (token >= c->vocab || s->pos >= c->max_seq) return -1;
    d = c->d_model;
    hd = m->head_dim;
    H = c->n_heads;
    Hkv = c->n_kv_heads;
    grp = H / Hkv;
    kvd = hd * Hkv;

    /* infer.c:713-715 embedding row copy */
    memcpy(s->x, m->embed + (size_t)token * d, d * sizeof(float));

    for (l = 0; l < c->n_layers; l++) {
        const or_layer *L = &m->layers[l];
        float *K = s->keys[l];
        float *V = s->values[l];

        /* transformer_block.c:478 pre-attention RMSNorm */
        if (or_rmsnorm(s->xn, s->x, L->attn_norm, d, c->eps)) return -1;
        /* attention.c:490-498 projections */
        if (mat_apply(m, &L->w[OR_T_WQ], s->q, s->xn, threads) ||
            mat_apply(m, &L->w[OR_T_WK], s->k, s->xn, threads) ||
            mat_apply(m, &L->w[OR_T_WV], s->v, s->xn, threads)) return -1;
        /* attention.c:72-106 RoPE per head on q and k */
        for (h = 0; h < H; h++) {
            if (or_rope(s->q + h * hd, hd, s->pos, c->theta)) return -1;
        }
        for (h = 0; h < Hkv; h++) {
            if (or_rope(s->k + h * hd, hd, s->pos, c->theta)) return -1;
        }
        /* kv_cache.c:76-114 append at [pos][head][hd] */
        memcpy(K + s->pos * kvd, s->k, kvd * sizeof(float));
        memcpy(V + s->pos * kvd, s->v, kvd * sizeof(float));
        /* attention.c:508-541 per-head scores, softmax, context */
        memset(s->ctx, 0, H * hd * sizeof(float));
        inv_sqrt = 1.0f / sqrtf((float)hd);
        for (h = 0; h < H; h++) {
            const float *qh = s->q + h * hd;
            float *ch = s->ctx + h * hd;
            const size_t kvh = h / grp;
            for (p = 0; p <= s->pos; p++) {
                const float *kh = K + p * kvd + kvh * hd;
                float dot = 0.0f;
                for (i = 0; i < hd; i++) dot += qh[i] * kh[i];
                s->scores[p] = dot * inv_sqrt;
            }
            if (or_softmax(s->scores, s->pos + 1)) return -1;
            for (p = 0; p <= s->pos; p++) {
                const float *vh = V + p * kvd + kvh * hd;
                for (i = 0; i < hd; i++) ch[i] += s->scores[p] * vh[i];
            }
        }
        if (mat_apply(m, &L->w[OR_T_WO], s->att, s->ctx, threads)) return -1;
        /* transformer_block.c:507 residual */
        for (i = 0; i < d; i++) s->h1[i] = s->x[i] + s->att[i];
        if (or_rmsnorm(s->xn, s->h1, L->ffn_norm, d, c->eps)) return -1;
        if (mat_apply(m, &L->w[OR_T_GATE], s->gate, s->xn, threads) ||
            mat_apply(m, &L->w[OR_T_UP], s->up, s->xn, threads)) return -1;
        if (or_swiglu(s->hs, s->gate, s->up, c->d_ff)) return -1;
        if (mat_apply(m, &L->w[OR_T_DOWN], s->tmp, s->hs, threads)) return -1;
        /* transformer_block.c:544 residual */
        for (i = 0; i < d; i++) s->x[i] = s->h1[i] + s->tmp[i];
    }
    /* infer.c:818-836 final norm + lm_head */
    if (or_rmsnorm(s->xn, s->x, m->out_norm, d, c->final_eps)) return -1;
    lg = logits;
    if (lg == NULL) {
        lg = malloc((size_t)c->vocab * sizeof(float));
        if (lg == NULL) return -1;
    }
    rc = mat_apply(m, &m->output, lg, s->xn, threads);
    if (rc == 0 && out_token != NULL) {
        rc = or_argmax(lg, c->vocab, out_token);
    }
    if (lg != logits) free(lg);
    if (rc == 0) s->pos++;
    return rc;
}
