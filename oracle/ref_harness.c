/*
 * ref_harness.c - drives the REFERENCE implementation (compiled from the
 * ATT-1 sources by oracle/Makefile into oracle/_ref/) on the seeded synthetic
 * models, to pin the oracle restatement and to time the reference CPU path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing of the reference is re-implemented here:
 * quantisation, blocks, norm, matmuls and the sampler are the reference's own
 * functions. The harness supplies:
 *   - weights from the shared seeded generator (or_synth_normal), quantised by
 *     att1_quantize_q4_per_group / att1_quantize_q8_per_row (src/quant.c);
 *   - GQA expanded to the reference's MHA layout (as the reference converter
 *     does, compiler/convert_llama_to_att1.py:288-326);
 *   - the per-layer loop of src/infer.c:724-836 with eps/theta taken from the
 *     model config (the block takes them, include/att1_transformer_block.h);
 *   - a "cpu-q4"/"cpu-q8" named backend whose matmul op splits output rows
 *     over threads and calls the reference matmul on each row slice (each
 *     row keeps its sequential accumulation, so results are unchanged).
 */
#include "att1_backend.h"
#include "att1_kv_cache.h"
#include "att1_math.h"
#include "att1_quant.h"
#include "att1_sampler.h"
#include "att1_transformer_block.h"

#include "att1_oracle.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

typedef struct rh_layer {
    float *attn_norm, *ffn_norm;
    att1_q4_matrix q4[9];
    att1_q8_matrix q8[9];
} rh_layer;

typedef struct rh_model {
    or_config cfg;
    uint32_t head_dim;
    float *embed, *out_norm;
    rh_layer *layers;
    att1_q4_matrix q4_out;
    att1_q8_matrix q8_out;
    int threads;
    att1_backend backend;
    att1_backend_ops ops;
    const att1_backend_ops *base_ops;
    att1_backend *base;
} rh_model;

typedef struct rh_state {
    size_t pos;
    att1_kv_cache *kv;
    float *x, *next, *norm;
} rh_state;

/* ---- threaded matmul ops ------------------------------------------------- */

typedef struct rh_job {
    float *dst;
    const float *lhs;
    size_t lhs_rows, lhs_cols, total_rows;
    att1_q4_matrix q4;
    att1_q8_matrix q8;
    int is_q4;
    float *tmp;
    size_t r0;
    int rc;
} rh_job;

static void *rh_job_run(void *arg)
{
    rh_job *j = (rh_job *)arg;
    if (j->is_q4) {
        j->rc = att1_matmul_q4xf32(j->tmp, j->lhs, j->lhs_rows, j->lhs_cols, &j->q4);
    } else {
        j->rc = att1_matmul_q8xf32(j->tmp, j->lhs, j->lhs_rows, j->lhs_cols, &j->q8);
    }
    return NULL;
}

static int rh_threaded(rh_model *m, float *dst, const float *lhs, size_t lhs_rows,
                       size_t lhs_cols, const att1_q4_matrix *q4,
                       const att1_q8_matrix *q8)
{
    const size_t rows = q4 ? q4->rows : q8->rows;
    int n = m->threads < 1 ? 1 : (m->threads > 64 ? 64 : m->threads);
    rh_job jobs[64];
    pthread_t tid[64];
    int started[64];
    int t, rc = 0;
    size_t b, r;

    if ((size_t)n > rows) n = (int)rows;
    if (n == 1) {
        return q4 ? att1_matmul_q4xf32(dst, lhs, lhs_rows, lhs_cols, q4)
                  : att1_matmul_q8xf32(dst, lhs, lhs_rows, lhs_cols, q8);
    }
    for (t = 0; t < n; t++) {
        const size_t r0 = rows * (size_t)t / (size_t)n;
        const size_t r1 = rows * (size_t)(t + 1) / (size_t)n;
        rh_job *j = &jobs[t];
        memset(j, 0, sizeof(*j));
        j->lhs = lhs; j->lhs_rows = lhs_rows; j->lhs_cols = lhs_cols;
        j->r0 = r0; j->is_q4 = (q4 != NULL);
        if (q4) {
            const size_t ng = q4->cols / q4->group_size;
            j->q4 = *q4;
            j->q4.rows = r1 - r0;
            j->q4.packed = q4->packed + r0 * (q4->cols / 2);
            j->q4.scales = q4->scales + r0 * ng;
        } else {
            j->q8 = *q8;
            j->q8.rows = r1 - r0;
            j->q8.values = q8->values + r0 * q8->cols;
            j->q8.scales = q8->scales + r0;
        }
        j->tmp = malloc(lhs_rows * (r1 - r0) * sizeof(float));
        if (j->tmp == NULL) return -1;
        started[t] = (pthread_create(&tid[t], NULL, rh_job_run, j) == 0);
        if (!started[t]) {
            rh_job_run(j);
        }
    }
    for (t = 0; t < n; t++) {
        rh_job *j = &jobs[t];
        const size_t nr = (t + 1 < n) ? (jobs[t + 1].r0 - j->r0) : (rows - j->r0);
        if (started[t]) pthread_join(tid[t], NULL);
        if (j->rc != 0) rc = -1;
        for (b = 0; b < lhs_rows; b++) {
            for (r = 0; r < nr; r++) {
                dst[b * rows + j->r0 + r] = j->tmp[b * nr + r];
            }
        }
        free(j->tmp);
    }
    return rc;
}

static int rh_op_q4(att1_backend *be, float *dst, const float *lhs,
                    size_t lhs_rows, size_t lhs_cols, const att1_q4_matrix *w)
{
    return rh_threaded((rh_model *)be->user_data, dst, lhs, lhs_rows, lhs_cols, w, NULL);
}

static int rh_op_q8(att1_backend *be, float *dst, const float *lhs,
                    size_t lhs_rows, size_t lhs_cols, const att1_q8_matrix *w)
{
    return rh_threaded((rh_model *)be->user_data, dst, lhs, lhs_rows, lhs_cols, NULL, w);
}

/* ---- model --------------------------------------------------------------- */

static float *rh_ones(size_t n)
{
    float *p = malloc(n * sizeof(float));
    size_t i;
    if (p) for (i = 0; i < n; i++) p[i] = 1.0f;
    return p;
}

/* Generate the [rows][cols] GQA matrix, expand rows by rep (row r of the
 * result is row (r / (rep * hd)) * hd + r % hd of the source when rep > 1),
 * quantise with the reference quantiser. */
static int rh_mat(rh_model *m, uint64_t seed, uint64_t tid, size_t rows,
                  size_t cols, size_t rep, att1_q4_matrix *q4, att1_q8_matrix *q8)
{
    const size_t hd = m->head_dim;
    const size_t out_rows = rows * rep;
    float *w = malloc(rows * cols * sizeof(float));
    float *e = NULL;
    int rc;
    size_t r;

    if (w == NULL) return -1;
    or_synth_normal_mt(seed, tid, 0, rows * cols, 0.02f, w, m->threads);
    if (rep > 1) {
        e = malloc(out_rows * cols * sizeof(float));
        if (e == NULL) { free(w); return -1; }
        for (r = 0; r < out_rows; r++) {
            const size_t head = r / hd, i = r % hd;
            const size_t src = (head / rep) * hd + i;
            memcpy(e + r * cols, w + src * cols, cols * sizeof(float));
        }
    }
    if (m->cfg.dtype == OR_Q4) {
        rc = att1_quantize_q4_per_group(q4, e ? e : w, out_rows, cols, m->cfg.group);
    } else {
        rc = att1_quantize_q8_per_row(q8, e ? e : w, out_rows, cols);
    }
    free(w);
    free(e);
    return rc;
}

void rh_model_free(rh_model *m);

rh_model *rh_model_synth(const or_config *cfg, uint64_t seed, int threads)
{
    rh_model *m;
    size_t d, f, hd, rep;
    uint32_t l;
    att1_status_t st;

    if (cfg == NULL || cfg->n_heads == 0 || cfg->n_kv_heads == 0 ||
        cfg->d_model % cfg->n_heads || cfg->n_heads % cfg->n_kv_heads) {
        return NULL;
    }
    m = calloc(1, sizeof(*m));
    if (m == NULL) return NULL;
    m->cfg = *cfg;
    m->threads = threads;
    d = cfg->d_model;
    f = cfg->d_ff;
    hd = d / cfg->n_heads;
    m->head_dim = (uint32_t)hd;
    rep = cfg->n_heads / cfg->n_kv_heads;
    m->embed = malloc((size_t)cfg->vocab * d * sizeof(float));
    m->out_norm = rh_ones(d);
    m->layers = calloc(cfg->n_layers, sizeof(rh_layer));
    if (!m->embed || !m->out_norm || !m->layers) goto fail;
    or_synth_normal_mt(seed, OR_T_EMBED, 0, (size_t)cfg->vocab * d, 0.02f, m->embed, threads);
    for (l = 0; l < cfg->n_layers; l++) {
        rh_layer *L = &m->layers[l];
        const uint64_t b = (uint64_t)l * OR_T_PER_LAYER;
        L->attn_norm = rh_ones(d);
        L->ffn_norm = rh_ones(d);
        if (!L->attn_norm || !L->ffn_norm) goto fail;
        if (rh_mat(m, seed, b + OR_T_WQ, d, d, 1, &L->q4[OR_T_WQ], &L->q8[OR_T_WQ]) ||
            rh_mat(m, seed, b + OR_T_WK, hd * cfg->n_kv_heads, d, rep, &L->q4[OR_T_WK], &L->q8[OR_T_WK]) ||
            rh_mat(m, seed, b + OR_T_WV, hd * cfg->n_kv_heads, d, rep, &L->q4[OR_T_WV], &L->q8[OR_T_WV]) ||
            rh_mat(m, seed, b + OR_T_WO, d, d, 1, &L->q4[OR_T_WO], &L->q8[OR_T_WO]) ||
            rh_mat(m, seed, b + OR_T_GATE, f, d, 1, &L->q4[OR_T_GATE], &L->q8[OR_T_GATE]) ||
            rh_mat(m, seed, b + OR_T_UP, f, d, 1, &L->q4[OR_T_UP], &L->q8[OR_T_UP]) ||
            rh_mat(m, seed, b + OR_T_DOWN, d, f, 1, &L->q4[OR_T_DOWN], &L->q8[OR_T_DOWN])) {
            goto fail;
        }
    }
    if (rh_mat(m, seed, OR_T_OUTPUT, cfg->vocab, d, 1, &m->q4_out, &m->q8_out)) goto fail;

    st = (cfg->dtype == OR_Q4) ? att1_backend_cpu_q4_create(&m->base)
                               : att1_backend_cpu_q8_create(&m->base);
    if (st != ATT1_OK) goto fail;
    m->ops = *m->base->ops;
    if (cfg->dtype == OR_Q4) {
        m->ops.matmul_q4xf32 = rh_op_q4;
    } else {
        m->ops.matmul_q8xf32 = rh_op_q8;
    }
    m->backend.ops = &m->ops;
    m->backend.user_data = m;
    return m;
fail:
    rh_model_free(m);
    return NULL;
}

void rh_model_free(rh_model *m)
{
    uint32_t l;
    int k;
    if (m == NULL) return;
    if (m->layers) {
        for (l = 0; l < m->cfg.n_layers; l++) {
            free(m->layers[l].attn_norm);
            free(m->layers[l].ffn_norm);
            for (k = 0; k < 9; k++) {
                att1_q4_matrix_free(&m->layers[l].q4[k]);
                att1_q8_matrix_free(&m->layers[l].q8[k]);
            }
        }
    }
    free(m->layers);
    free(m->embed);
    free(m->out_norm);
    att1_q4_matrix_free(&m->q4_out);
    att1_q8_matrix_free(&m->q8_out);
    if (m->base) att1_backend_destroy(m->base);
    free(m);
}

void rh_model_set_threads(rh_model *m, int threads)
{
    if (m) m->threads = threads;
}

/* Borrowed packed bytes / scales of a matrix (kind as OR_T_*, 9 = output). */
int rh_model_q4_view(const rh_model *m, uint32_t layer, uint32_t kind,
                     const uint8_t **packed, const float **scales,
                     size_t *rows, size_t *cols)
{
    const att1_q4_matrix *w;
    if (m == NULL) return -1;
    if (kind == 9) w = &m->q4_out;
    else if (layer < m->cfg.n_layers && kind < 9) w = &m->layers[layer].q4[kind];
    else return -1;
    if (w->packed == NULL) return -1;
    *packed = w->packed; *scales = w->scales; *rows = w->rows; *cols = w->cols;
    return 0;
}

rh_state *rh_state_create(const rh_model *m)
{
    rh_state *s;
    uint32_t l;
    if (m == NULL) return NULL;
    s = calloc(1, sizeof(*s));
    if (s == NULL) return NULL;
    s->kv = calloc(m->cfg.n_layers, sizeof(att1_kv_cache));
    s->x = calloc(m->cfg.d_model, sizeof(float));
    s->next = calloc(m->cfg.d_model, sizeof(float));
    s->norm = calloc(m->cfg.d_model, sizeof(float));
    if (!s->kv || !s->x || !s->next || !s->norm) return NULL;
    for (l = 0; l < m->cfg.n_layers; l++) {
        if (att1_kv_cache_init(&s->kv[l], m->cfg.max_seq, m->cfg.n_heads,
                               m->head_dim) != ATT1_OK) {
            return NULL;
        }
    }
    return s;
}

void rh_state_free(const rh_model *m, rh_state *s)
{
    uint32_t l;
    if (s == NULL) return;
    if (s->kv && m) {
        for (l = 0; l < m->cfg.n_layers; l++) att1_kv_cache_free(&s->kv[l]);
    }
    free(s->kv); free(s->x); free(s->next); free(s->norm);
    free(s);
}

/* Fill every layer's cache with `length` positions of seeded values, as if
 * that many tokens had been decoded (used only to time attention at depth). */
int rh_state_fill(const rh_model *m, rh_state *s, size_t length, uint64_t seed)
{
    uint32_t l;
    if (m == NULL || s == NULL || length > m->cfg.max_seq) return -1;
    for (l = 0; l < m->cfg.n_layers; l++) {
        const size_t n = length * m->cfg.n_heads * m->head_dim;
        or_synth_normal(seed, 0x60000000ull + 2u * l, 0, n, 1.0f, s->kv[l].keys);
        or_synth_normal(seed, 0x60000001ull + 2u * l, 0, n, 1.0f, s->kv[l].values);
        s->kv[l].length = length;
    }
    s->pos = length;
    return 0;
}

/* One decode step: src/infer.c:713-880 with the reference block functions. */
int rh_decode(rh_model *m, rh_state *s, uint32_t token, float *logits,
              uint32_t *out_token)
{
    att1_transformer_block_config bc;
    const size_t d = m->cfg.d_model;
    uint32_t l;
    int rc;

    if (token >= m->cfg.vocab || s->pos >= m->cfg.max_seq) return -1;
    memcpy(s->x, m->embed + (size_t)token * d, d * sizeof(float));
    bc.model_dim = d;
    bc.num_heads = m->cfg.n_heads;
    bc.head_dim = m->head_dim;
    bc.ffn_dim = m->cfg.d_ff;
    bc.rms_epsilon = m->cfg.eps;
    bc.rope_theta = m->cfg.theta;
    for (l = 0; l < m->cfg.n_layers; l++) {
        rh_layer *L = &m->layers[l];
        if (m->cfg.dtype == OR_Q4) {
            att1_transformer_block_q4_weights w;
            w.attention_norm = L->attn_norm; w.ffn_norm = L->ffn_norm;
            w.wq = &L->q4[OR_T_WQ]; w.wk = &L->q4[OR_T_WK]; w.wv = &L->q4[OR_T_WV];
            w.wo = &L->q4[OR_T_WO]; w.w_gate = &L->q4[OR_T_GATE];
            w.w_up = &L->q4[OR_T_UP]; w.w_down = &L->q4[OR_T_DOWN];
            rc = att1_transformer_block_forward_backend_q4(
                s->next, &s->kv[l], s->x, &w, &bc, s->pos, &m->backend);
        } else {
            att1_transformer_block_q8_weights w;
            w.attention_norm = L->attn_norm; w.ffn_norm = L->ffn_norm;
            w.wq = &L->q8[OR_T_WQ]; w.wk = &L->q8[OR_T_WK]; w.wv = &L->q8[OR_T_WV];
            w.wo = &L->q8[OR_T_WO]; w.w_gate = &L->q8[OR_T_GATE];
            w.w_up = &L->q8[OR_T_UP]; w.w_down = &L->q8[OR_T_DOWN];
            rc = att1_transformer_block_forward_backend_q8(
                s->next, &s->kv[l], s->x, &w, &bc, s->pos, &m->backend);
        }
        if (rc != 0) return -1;
        memcpy(s->x, s->next, d * sizeof(float));
    }
    if (att1_rmsnorm_f32(s->norm, s->x, m->out_norm, d, m->cfg.final_eps) != 0) return -1;
    if (m->cfg.dtype == OR_Q4) {
        rc = rh_op_q4(&m->backend, logits, s->norm, 1, d, &m->q4_out);
    } else {
        rc = rh_op_q8(&m->backend, logits, s->norm, 1, d, &m->q8_out);
    }
    if (rc != 0) return -1;
    if (out_token != NULL && att1_sampler_greedy_f32(logits, m->cfg.vocab, out_token) != 0) {
        return -1;
    }
    s->pos++;
    return 0;
}

/* Direct passthroughs to the reference quantiser/matmul for element tests. */
int rh_quantize_q4(const float *w, size_t rows, size_t cols, uint32_t group,
                   uint8_t *packed, float *scales)
{
    att1_q4_matrix m;
    const size_t ng = cols / (group ? group : 1);
    if (att1_quantize_q4_per_group(&m, w, rows, cols, group) != 0) return -1;
    memcpy(packed, m.packed, rows * cols / 2);
    memcpy(scales, m.scales, rows * ng * sizeof(float));
    att1_q4_matrix_free(&m);
    return 0;
}

int rh_quantize_q8(const float *w, size_t rows, size_t cols, int8_t *values,
                   float *scales)
{
    att1_q8_matrix m;
    if (att1_quantize_q8_per_row(&m, w, rows, cols) != 0) return -1;
    memcpy(values, m.values, rows * cols);
    memcpy(scales, m.scales, rows * sizeof(float));
    att1_q8_matrix_free(&m);
    return 0;
}

int rh_matmul_q4(float *dst, const float *lhs, size_t lhs_rows, size_t cols,
                 uint8_t *packed, float *scales, size_t rows, uint32_t group)
{
    att1_q4_matrix m;
    m.rows = rows; m.cols = cols; m.group_size = group;
    m.packed = packed; m.scales = scales;
    return att1_matmul_q4xf32(dst, lhs, lhs_rows, cols, &m);
}

int rh_matmul_q8(float *dst, const float *lhs, size_t lhs_rows, size_t cols,
                 int8_t *values, float *scales, size_t rows)
{
    att1_q8_matrix m;
    m.rows = rows; m.cols = cols; m.values = values; m.scales = scales;
    return att1_matmul_q8xf32(dst, lhs, lhs_rows, cols, &m);
}

int rh_pack_group(const int8_t *src, uint32_t group, uint8_t *dst)
{
    return att1_q4_pack_group(src, group, dst);
}

int rh_unpack_group(const uint8_t *src, uint32_t group, int8_t *dst)
{
    return att1_q4_unpack_group(src, group, dst);
}

int rh_quantize_group(const float *src, uint32_t group, uint8_t *dst, float *scale)
{
    return att1_q4_quantize_group(src, group, dst, scale);
}

int rh_rmsnorm(float *dst, const float *src, const float *w, size_t n, float eps)
{
    return att1_rmsnorm_f32(dst, src, w, n, eps);
}

int rh_softmax(float *v, size_t n) { return att1_softmax_f32(v, n); }

int rh_rope(float *v, size_t n, size_t pos, float theta)
{
    return att1_rope_f32(v, n, pos, theta);
}

int rh_swiglu(float *dst, const float *g, const float *u, size_t n)
{
    return att1_swiglu_f32(dst, g, u, n);
}

int rh_argmax(const float *v, size_t n, uint32_t *out)
{
    return att1_sampler_greedy_f32(v, n, out);
}
