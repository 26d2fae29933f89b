/*
 * att1_infer.c - device-resident decode behind the ATT-1 model API.
 *
 * Implements include/att1_infer.h and include/att1_b200.h: the decode step of
 * ATT-1's src/infer.c:656-880 (embedding, n_layers pre-norm blocks of
 * src/transformer_block.c:417-557, final RMSNorm, lm_head, greedy sampler)
 * as a fixed sequence of sm_100a kernels per token:
 *
 *   step_begin                 x = embed[token]
 *   per layer:
 *     gemv QKV  (RMSNorm prologue; RoPE + KV-page append epilogue)
 *     attn      (single query over the KV pages, GQA)
 *     gemv WO   (residual epilogue)             h = x + Wo ctx
 *     gemv GU   (RMSNorm prologue; SwiGLU epilogue over interleaved gate/up)
 *     gemv DOWN (residual epilogue)             x = h + Wd s
 *   gemv OUT  (RMSNorm prologue; logits + argmax key epilogue)
 *   step_end                   token = argmax, position += 1
 *
 * The sequence is captured once as a CUDA graph with programmatic dependent
 * launch edges and replayed per token; positions and tokens stay on the
 * device, so a step needs only the token id in and the next id out.
 */
#define _POSIX_C_SOURCE 200809L
#include "att1_infer.h"
#include "att1_b200.h"
#include "b2_host.h"

#include <float.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct dev_layer {
    float *attn_norm, *ffn_norm;
    b2_dev_mat qkv, wo, gu, down;
    b2_gemv_args a_qkv, a_wo, a_gu, a_down;
    b2_attn_args a_attn;
} dev_layer;

struct att1_infer {
    att1_b200_config cfg;
    uint32_t head_dim, batch, q_rows, kv_rows;
    /* tensor parallelism: this rank's shard (tp_world 1: the whole model) */
    uint32_t tp_rank, tp_world;
    uint32_t hq, hkv, ffl, vl, v_off;  /* query / KV heads, FFN rows, vocabulary rows and first id */
    uint8_t *tp_region;                /* this rank's exchange region */
    size_t tp_region_bytes;
    uint8_t *tp_peer[B2_TP_MAX];       /* every rank's region as mapped here */
    int tp_opened[B2_TP_MAX];          /* mapped through CUDA IPC (closed at release) */
    uint32_t *tp_epoch;
    int32_t *tp_done;
    int tp_ready;
    uint32_t tp_wait_polls;            /* bound of every exchange wait (0: the kernels' default) */
    /* the exchange through an NCCL communicator instead of peer memory
     * (att1_b200_infer_tp_connect_nccl): ncclComm_t, gathered argmax keys [world][batch] */
    void *nccl_comm;
    unsigned long long *nccl_keys;
    b2_tp tp_base;                     /* exchange description shared by the step's kernels */
    int device;
    cudaStream_t stream;
    dev_layer *layers;
    float *embed, *out_norm, *rope_freq;
    b2_dev_mat output;
    b2_gemv_args a_out;
    float *k_pool, *v_pool;
    size_t layer_pool_elems;
    int32_t *page_table;
    uint32_t page_tokens, pages_per_seq;
    float *x, *h1, *q, *ctx, *hs, *logits;
    uint32_t *tokens_d;
    int32_t *pos_d;
    unsigned long long *argmax_d;
    int32_t *err_d;
    void *scratch;
    size_t scratch_bytes;
    int32_t *counters;
    uint32_t counters_len;
    uint32_t *tokens_h, *out_h;
    int32_t *err_h;
    float *logits_h;
    int logits_valid;
    size_t position;
    int use_graph, use_pdl, use_persistent;
    /* KV in the sessions of a KV-MMU (att1_b200_infer_use_kv_mmu): item b is the
     * session in slot mmu_slot0 + b; NULL: the context's own page pools */
    att1_kv_mmu *mmu;
    uint64_t mmu_sid0;
    size_t mmu_slot0;
    /* decode through the tensor-core GEMM (batches the GEMVs cannot hold) */
    int use_dense;
    size_t graph_nodes; /* operations in the captured step graph (0: not captured) */
    /* sampling: top_k <= 1 greedy; else b2_sample_topk after the step end */
    uint32_t top_k;
    float temperature;
    uint64_t sample_seed;
    float *y_qkv, *y_gu, *y_part;
    void *xs, *gscratch;
    size_t xs_bytes, gscratch_bytes;
    /* prompt prefill buffers for up to pf_cap tokens (allocated on first use) */
    uint32_t pf_cap;
    float *pf_x, *pf_h, *pf_q, *pf_ctx, *pf_hs, *pf_yqkv, *pf_ygu;
    uint32_t *pf_tok;
    int32_t *pf_pos, *pf_pt, *pf_counters;
    int32_t *pf_mpt; /* KV-MMU session: its rows of every layer, [layer][pf_cap][pages_per_seq] */
    size_t pf_mpt_elems;
    unsigned long long *pf_keys;
    void *pf_xs, *pf_gscratch, *pf_ascratch;
    size_t pf_xs_bytes, pf_gscratch_bytes, pf_ascratch_bytes;
    uint32_t pf_counters_len;
    int step_pending;
    uint64_t trace_t0;
    cudaGraphExec_t exec;
    int graph_failed;
    b2_decode_plan *plan;
    att1_backend *backend;
    att1_trace_t *trace;
    const att1_model *model;
    size_t device_bytes;
};

static att1_status_t dense_alloc(att1_infer_t *inf);

/* ---- allocation ------------------------------------------------------------ */

static att1_status_t dalloc(att1_infer_t *inf, void **p, size_t bytes)
{
    cudaError_t e;
    *p = NULL;
    if (bytes == 0) bytes = 256;
    e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) {
        *p = NULL;
        return b2_cuda_status(e);
    }
    inf->device_bytes += bytes;
    e = cudaMemsetAsync(*p, 0, bytes, inf->stream);
    return b2_cuda_status(e);
}

static void dfree(void *p)
{
    if (p != NULL) cudaFree(p);
}

static att1_status_t mat_alloc(att1_infer_t *inf, b2_dev_mat *m, uint32_t fmt, uint32_t rows, uint32_t cols)
{
    att1_status_t st;
    memset(m, 0, sizeof(*m));
    m->w.format = fmt;
    m->w.rows = rows;
    m->w.cols = cols;
    m->w.tiles = (rows + 15) / 16;
    m->w.kunits = fmt == 4 ? (cols + 63) / 64 : (cols + 31) / 32;
    st = dalloc(inf, &m->data, fmt == 4 ? b2_q4_bytes(rows, cols) : b2_q8_bytes(rows, cols));
    if (st != ATT1_OK) return st;
    if (fmt == 8) {
        st = dalloc(inf, (void **)&m->row_scale, (size_t)m->w.tiles * 16 * sizeof(float));
        if (st != ATT1_OK) return st;
    }
    m->w.data = m->data;
    m->w.row_scale = m->row_scale;
    return ATT1_OK;
}

static void mat_free(b2_dev_mat *m)
{
    dfree(m->data);
    dfree(m->row_scale);
    memset(m, 0, sizeof(*m));
}

static void free_prefill(att1_infer_t *inf)
{
    dfree(inf->pf_x);
    dfree(inf->pf_h);
    dfree(inf->pf_q);
    dfree(inf->pf_ctx);
    dfree(inf->pf_hs);
    dfree(inf->pf_yqkv);
    dfree(inf->pf_ygu);
    dfree(inf->pf_tok);
    dfree(inf->pf_pos);
    dfree(inf->pf_pt);
    dfree(inf->pf_mpt);
    dfree(inf->pf_counters);
    dfree(inf->pf_keys);
    dfree(inf->pf_xs);
    dfree(inf->pf_gscratch);
    dfree(inf->pf_ascratch);
    inf->pf_mpt = NULL;
    inf->pf_mpt_elems = 0;
    inf->pf_cap = 0;
}

static void release(att1_infer_t *inf)
{
    uint32_t l;
    if (inf == NULL) return;
    cudaSetDevice(inf->device);
    if (inf->stream) cudaStreamSynchronize(inf->stream);
    if (inf->exec) cudaGraphExecDestroy(inf->exec);
    if (inf->plan) b2_decode_plan_destroy(inf->plan);
    if (inf->layers) {
        for (l = 0; l < inf->cfg.n_layers; l++) {
            dev_layer *L = &inf->layers[l];
            dfree(L->attn_norm);
            dfree(L->ffn_norm);
            mat_free(&L->qkv);
            mat_free(&L->wo);
            mat_free(&L->gu);
            mat_free(&L->down);
        }
        free(inf->layers);
    }
    mat_free(&inf->output);
    dfree(inf->embed);
    dfree(inf->out_norm);
    dfree(inf->rope_freq);
    dfree(inf->k_pool);
    dfree(inf->v_pool);
    dfree(inf->page_table);
    dfree(inf->x);
    dfree(inf->h1);
    dfree(inf->q);
    dfree(inf->ctx);
    dfree(inf->hs);
    dfree(inf->logits);
    dfree(inf->tokens_d);
    dfree(inf->pos_d);
    dfree(inf->argmax_d);
    dfree(inf->err_d);
    dfree(inf->scratch);
    dfree(inf->counters);
    dfree(inf->y_qkv);
    dfree(inf->y_gu);
    dfree(inf->y_part);
    dfree(inf->xs);
    dfree(inf->gscratch);
    free_prefill(inf);
    if (inf->tokens_h) cudaFreeHost(inf->tokens_h);
    if (inf->out_h) cudaFreeHost(inf->out_h);
    if (inf->err_h) cudaFreeHost(inf->err_h);
    if (inf->logits_h) cudaFreeHost(inf->logits_h);
    if (inf->backend) att1_backend_destroy(inf->backend);
    for (l = 0; l < B2_TP_MAX; l++)
        if (inf->tp_opened[l]) cudaIpcCloseMemHandle(inf->tp_peer[l]);
    if (inf->nccl_comm) b2_nccl_comm_destroy(inf->nccl_comm);
    dfree(inf->nccl_keys);
    dfree(inf->tp_region);
    dfree(inf->tp_epoch);
    dfree(inf->tp_done);
    if (inf->stream) cudaStreamDestroy(inf->stream);
    free(inf);
}

/* ---- configuration checks ---------------------------------------------------------- */

static att1_status_t check_config(const att1_b200_config *c, uint32_t batch)
{
    uint32_t hd;
    if (c == NULL || batch == 0 || batch > ATT1_B200_MAX_BATCH) return ATT1_ERR_INVALID_ARG;
    if (c->vocab == 0 || c->n_layers == 0 || c->n_heads == 0 || c->n_kv_heads == 0 || c->d_model == 0 ||
        c->d_ff == 0 || c->max_seq == 0)
        return ATT1_ERR_INVALID_ARG;
    if (c->dtype != 4 && c->dtype != 8) return ATT1_ERR_INVALID_ARG;
    if (!(c->eps > 0.0f) || !(c->final_eps > 0.0f) || !(c->theta > 0.0f)) return ATT1_ERR_INVALID_ARG;
    if (c->d_model % c->n_heads || c->n_heads % c->n_kv_heads) return ATT1_ERR_SHAPE;
    hd = c->d_model / c->n_heads;
    /* device layout limits: 16-row tiles per head, 32-column groups */
    if (hd % 16 || hd > 128 || c->n_heads / c->n_kv_heads > 8) return ATT1_ERR_UNSUPPORTED;
    if (c->d_model % 32 || c->d_ff % 32) return ATT1_ERR_UNSUPPORTED;
    if (c->dtype == 4 && c->group != 32 && c->group != 0) return ATT1_ERR_UNSUPPORTED;
    return ATT1_OK;
}

/* ---- kernel arguments ------------------------------------------------------------------ */

static void gemv_base(att1_infer_t *inf, b2_gemv_args *a, const b2_dev_mat *m)
{
    memset(a, 0, sizeof(*a));
    a->w = m->w;
    a->batch = inf->batch;
    a->err = inf->err_d;
    a->pdl = inf->use_pdl;
}

static b2_kv_layout kv_layout(att1_infer_t *inf, uint32_t layer)
{
    b2_kv_layout kv;
    if (inf->mmu != NULL && att1_b200_kv_mmu_layout(inf->mmu, inf->mmu_sid0, layer, &kv) == ATT1_OK) return kv;
    kv.k_pool = inf->k_pool + (size_t)layer * inf->layer_pool_elems;
    kv.v_pool = inf->v_pool + (size_t)layer * inf->layer_pool_elems;
    kv.page_table = inf->page_table;
    kv.page_tokens = inf->page_tokens;
    kv.pages_per_seq = inf->pages_per_seq;
    kv.n_kv_heads = inf->hkv;
    kv.head_dim = inf->head_dim;
    return kv;
}

/* The persistent single-launch step over the same arguments. A shape the
 * persistent kernel cannot hold (shared memory) keeps the per-kernel sequence. */
static att1_status_t build_plan(att1_infer_t *inf)
{
    const att1_b200_config *c = &inf->cfg;
    b2_decode_layer *ls;
    b2_decode_args da;
    uint32_t l;
    int rc;
    if (inf->plan) {
        cudaStreamSynchronize(inf->stream);
        b2_decode_plan_destroy(inf->plan);
        inf->plan = NULL;
    }
    if (inf->tp_world > 1) return ATT1_OK; /* the persistent step has no exchange */
    ls = calloc(c->n_layers, sizeof(*ls));
    if (ls == NULL) return ATT1_ERR_OOM;
    for (l = 0; l < c->n_layers; l++) {
        ls[l].qkv = inf->layers[l].a_qkv;
        ls[l].wo = inf->layers[l].a_wo;
        ls[l].gu = inf->layers[l].a_gu;
        ls[l].down = inf->layers[l].a_down;
        ls[l].attn = inf->layers[l].a_attn;
    }
    memset(&da, 0, sizeof(da));
    da.n_layers = c->n_layers;
    da.batch = inf->batch;
    da.layers = ls;
    da.out = inf->a_out;
    da.embed = inf->embed;
    da.vocab = c->vocab;
    da.d_model = c->d_model;
    da.tokens_in = inf->tokens_d;
    da.tokens_out = inf->tokens_d;
    da.positions = inf->pos_d;
    da.argmax = inf->argmax_d;
    da.x = inf->x;
    da.err = inf->err_d;
    rc = b2_decode_plan_create(&da, &inf->plan);
    free(ls);
    if (rc == -2) return ATT1_ERR_OOM;
    if (rc != 0) inf->plan = NULL;
    return ATT1_OK;
}

/* Tensor parallelism (Megatron split, as proposed for ATT-1's shard
 * metadata): QKV and gate/up hold this rank's heads / FFN rows, WO and down
 * this rank's input columns; their partial outputs go to every rank's
 * exchange slot (B2_EPI_PUSH) and the next GEMV's prologue adds the ranks'
 * partials and the residual (x + WO, h1 + down) in rank order, so every rank
 * carries the same residual stream. The lm_head holds this rank's vocabulary
 * rows; logits and argmax keys are all-gathered and b2_step_end_tp takes the
 * global greedy token. Exchange points: 2l = WO of layer l, 2l+1 = down of
 * layer l, 2L = logits. */
static void tp_wire(att1_infer_t *inf)
{
    const att1_b200_config *c = &inf->cfg;
    b2_tp t;
    uint32_t l, s;
    memset(&t, 0, sizeof(t));
    t.rank = inf->tp_rank;
    t.world = inf->tp_world;
    for (s = 0; s < inf->tp_world; s++) t.peer[s] = inf->tp_peer[s];
    t.points = 2 * c->n_layers;
    t.slot_floats = inf->batch * c->d_model;
    t.logit_floats = inf->batch * inf->vl;
    t.epoch = inf->tp_epoch;
    t.done = inf->tp_done;
    t.wait_polls = inf->tp_wait_polls;
    t.in_point = B2_TP_NONE;
    t.out_point = B2_TP_NONE;
    inf->tp_base = t;
    for (l = 0; l < c->n_layers; l++) {
        dev_layer *L = &inf->layers[l];
        L->a_wo.tp = t;
        L->a_wo.epilogue = B2_EPI_PUSH;
        L->a_wo.resid = NULL;
        L->a_wo.tp.out_point = 2 * l;
        L->a_gu.tp = t;
        L->a_gu.tp.in_point = 2 * l;
        L->a_gu.tp.in_resid = inf->x;
        L->a_gu.tp.in_out = inf->h1;
        L->a_down.tp = t;
        L->a_down.epilogue = B2_EPI_PUSH;
        L->a_down.resid = NULL;
        L->a_down.tp.out_point = 2 * l + 1;
        if (l > 0) {
            L->a_qkv.tp = t;
            L->a_qkv.tp.in_point = 2 * l - 1;
            L->a_qkv.tp.in_resid = inf->h1;
            L->a_qkv.tp.in_out = inf->x;
        }
    }
    inf->a_out.tp = t;
    inf->a_out.tp.out_point = t.points;
    inf->a_out.tp.in_point = 2 * c->n_layers - 1;
    inf->a_out.tp.in_resid = inf->h1;
    inf->a_out.tp.row_offset = inf->v_off;
    inf->tp_base.out_point = t.points;
}

/* The comparison arm (att1_b200_infer_tp_connect_nccl): the one-GPU wiring
 * with partial sums. WO and down add the residual on rank 0 only, so the sum
 * of every rank's output (ncclAllReduce after each) is the residual plus all
 * partials; the lm_head keeps this rank's vocabulary rows and global ids for
 * its argmax keys, gathered after it. */
static void nccl_wire(att1_infer_t *inf)
{
    const att1_b200_config *c = &inf->cfg;
    uint32_t l;
    for (l = 0; l < c->n_layers; l++) {
        dev_layer *L = &inf->layers[l];
        if (inf->tp_rank != 0) {
            L->a_wo.epilogue = B2_EPI_STORE;
            L->a_wo.resid = NULL;
            L->a_down.epilogue = B2_EPI_STORE;
            L->a_down.resid = NULL;
        }
    }
    inf->a_out.tp.row_offset = inf->v_off;
}

static att1_status_t build_args(att1_infer_t *inf)
{
    const att1_b200_config *c = &inf->cfg;
    size_t need = 0, s;
    uint32_t l;
    att1_status_t st;

    for (l = 0; l < c->n_layers; l++) {
        dev_layer *L = &inf->layers[l];
        b2_gemv_args *a;

        a = &L->a_qkv;
        gemv_base(inf, a, &L->qkv);
        a->x = inf->x;
        a->x_stride = c->d_model;
        a->norm_w = L->attn_norm;
        a->eps = c->eps;
        a->epilogue = B2_EPI_QKV;
        a->out = inf->q;
        a->out_stride = inf->q_rows;
        a->q_rows = inf->q_rows;
        a->kv_rows = inf->kv_rows;
        a->rope_freq = inf->rope_freq;
        a->positions = inf->pos_d;
        a->kv = kv_layout(inf, l);

        memset(&L->a_attn, 0, sizeof(L->a_attn));
        L->a_attn.batch = inf->batch;
        L->a_attn.n_heads = inf->hq;
        L->a_attn.n_kv_heads = inf->hkv;
        L->a_attn.head_dim = inf->head_dim;
        L->a_attn.q = inf->q;
        L->a_attn.kv = kv_layout(inf, l);
        L->a_attn.positions = inf->pos_d;
        L->a_attn.max_ctx = c->max_seq;
        L->a_attn.ctx = inf->ctx;
        L->a_attn.err = inf->err_d;
        L->a_attn.pdl = inf->use_pdl;

        a = &L->a_wo;
        gemv_base(inf, a, &L->wo);
        a->x = inf->ctx;
        a->x_stride = inf->q_rows;
        a->epilogue = B2_EPI_RESID;
        a->resid = inf->x;
        a->out = inf->h1;
        a->out_stride = c->d_model;

        a = &L->a_gu;
        gemv_base(inf, a, &L->gu);
        a->x = inf->h1;
        a->x_stride = c->d_model;
        a->norm_w = L->ffn_norm;
        a->eps = c->eps;
        a->epilogue = B2_EPI_SWIGLU;
        a->out = inf->hs;
        a->out_stride = inf->ffl;

        a = &L->a_down;
        gemv_base(inf, a, &L->down);
        a->x = inf->hs;
        a->x_stride = inf->ffl;
        a->epilogue = B2_EPI_RESID;
        a->resid = inf->h1;
        a->out = inf->x;
        a->out_stride = c->d_model;
    }
    {
        b2_gemv_args *a = &inf->a_out;
        gemv_base(inf, a, &inf->output);
        a->x = inf->x;
        a->x_stride = c->d_model;
        a->norm_w = inf->out_norm;
        a->eps = c->final_eps;
        a->epilogue = B2_EPI_LOGITS;
        a->out = inf->logits;
        a->out_stride = inf->vl;
        a->argmax = inf->argmax_d;
    }
    if (inf->tp_world > 1) {
        if (inf->nccl_comm != NULL) nccl_wire(inf);
        else tp_wire(inf);
    }
    /* One partial-sum region and one counter array serve every kernel: they
     * run one after another and each leaves its counters at zero. */
    inf->use_dense = inf->batch > 16;
    {
        uint32_t cmax = 0, cl;
        for (l = 0; l < c->n_layers; l++) {
            dev_layer *L = &inf->layers[l];
            b2_gemv_args *g[4] = {&L->a_qkv, &L->a_wo, &L->a_gu, &L->a_down};
            int k;
            for (k = 0; k < 4; k++) {
                if ((s = b2_gemv_scratch_bytes(g[k])) > need) need = s;
                if (s == 0) inf->use_dense = 1; /* x's digit planes do not fit on chip */
                if ((cl = b2_gemv_counters_len(g[k])) > cmax) cmax = cl;
            }
            if ((s = b2_attn_scratch_bytes(&L->a_attn)) > need) need = s;
            if ((cl = b2_attn_counters_len(&L->a_attn)) > cmax) cmax = cl;
        }
        if ((s = b2_gemv_scratch_bytes(&inf->a_out)) > need) need = s;
        if (s == 0) inf->use_dense = 1;
        if ((cl = b2_gemv_counters_len(&inf->a_out)) > cmax) cmax = cl;
        dfree(inf->scratch);
        dfree(inf->counters);
        inf->scratch = NULL;
        inf->counters = NULL;
        if ((st = dalloc(inf, &inf->scratch, need)) != ATT1_OK) return st;
        if ((st = dalloc(inf, (void **)&inf->counters, (size_t)cmax * sizeof(int32_t))) != ATT1_OK) return st;
        inf->scratch_bytes = need;
        inf->counters_len = cmax;
    }
    for (l = 0; l < c->n_layers; l++) {
        dev_layer *L = &inf->layers[l];
        b2_gemv_args *g[4] = {&L->a_qkv, &L->a_wo, &L->a_gu, &L->a_down};
        int k;
        for (k = 0; k < 4; k++) {
            g[k]->scratch = inf->scratch;
            g[k]->scratch_bytes = need;
            g[k]->counters = inf->counters;
            g[k]->counters_len = inf->counters_len;
        }
        L->a_attn.scratch = inf->scratch;
        L->a_attn.scratch_bytes = need;
        L->a_attn.counters = inf->counters;
        L->a_attn.counters_len = inf->counters_len;
    }
    inf->a_out.scratch = inf->scratch;
    inf->a_out.scratch_bytes = need;
    inf->a_out.counters = inf->counters;
    inf->a_out.counters_len = inf->counters_len;
    if (inf->use_dense) return dense_alloc(inf);
    return build_plan(inf);
}

static void set_pdl(att1_infer_t *inf, int pdl)
{
    uint32_t l;
    for (l = 0; l < inf->cfg.n_layers; l++) {
        dev_layer *L = &inf->layers[l];
        L->a_qkv.pdl = L->a_wo.pdl = L->a_gu.pdl = L->a_down.pdl = L->a_attn.pdl = pdl;
    }
    inf->a_out.pdl = pdl;
    inf->use_pdl = pdl;
}

/* ---- buffers common to both creation paths ------------------------------------------------------ */

static att1_status_t alloc_common(att1_infer_t *inf)
{
    const att1_b200_config *c = &inf->cfg;
    const uint32_t B = inf->batch;
    att1_status_t st;
    uint32_t i, b;
    int32_t *pt;
    float *freq;
    size_t pages;
    cudaError_t e;

    inf->page_tokens = c->max_seq < 64 ? c->max_seq : 64;
    inf->pages_per_seq = (c->max_seq + inf->page_tokens - 1) / inf->page_tokens;
    pages = (size_t)B * inf->pages_per_seq;
    inf->layer_pool_elems = pages * inf->page_tokens * inf->hkv * inf->head_dim;
    if ((st = dalloc(inf, (void **)&inf->k_pool, inf->layer_pool_elems * c->n_layers * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->v_pool, inf->layer_pool_elems * c->n_layers * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->page_table, pages * sizeof(int32_t))) ||
        (st = dalloc(inf, (void **)&inf->rope_freq, (inf->head_dim / 2) * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->x, (size_t)B * c->d_model * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->h1, (size_t)B * c->d_model * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->q, (size_t)B * inf->q_rows * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->ctx, (size_t)B * inf->q_rows * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->hs, (size_t)B * inf->ffl * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->logits, (size_t)B * inf->vl * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->tokens_d, ATT1_B200_MAX_BATCH * sizeof(uint32_t))) ||
        (st = dalloc(inf, (void **)&inf->pos_d, ATT1_B200_MAX_BATCH * sizeof(int32_t))) ||
        (st = dalloc(inf, (void **)&inf->argmax_d, ATT1_B200_MAX_BATCH * sizeof(unsigned long long))) ||
        (st = dalloc(inf, (void **)&inf->err_d, sizeof(int32_t))))
        return st;
    /* page table: sequence b owns pages [b*pages_per_seq, (b+1)*pages_per_seq) */
    pt = malloc(pages * sizeof(int32_t));
    freq = malloc((inf->head_dim / 2) * sizeof(float));
    if (pt == NULL || freq == NULL) {
        free(pt);
        free(freq);
        return ATT1_ERR_OOM;
    }
    for (b = 0; b < B; b++)
        for (i = 0; i < inf->pages_per_seq; i++) pt[(size_t)b * inf->pages_per_seq + i] = (int32_t)(b * inf->pages_per_seq + i);
    /* src/rope.c:21-22: freq of pair i/2 = 1 / powf(theta, i / head_dim), host libm */
    for (i = 0; i < inf->head_dim / 2; i++) freq[i] = 1.0f / powf(c->theta, (float)(2 * i) / (float)inf->head_dim);
    /* on the context's stream, after dalloc's zero fill of the same buffers: a
     * plain cudaMemcpy runs on the legacy stream, which does not wait for a
     * non-blocking stream, so the fill could land after the table */
    e = cudaMemcpyAsync(inf->page_table, pt, pages * sizeof(int32_t), cudaMemcpyHostToDevice, inf->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(inf->rope_freq, freq, (inf->head_dim / 2) * sizeof(float), cudaMemcpyHostToDevice,
                            inf->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(inf->stream);
    free(pt);
    free(freq);
    if (e != cudaSuccess) return b2_cuda_status(e);
    if (cudaMallocHost((void **)&inf->tokens_h, ATT1_B200_MAX_BATCH * sizeof(uint32_t)) != cudaSuccess ||
        cudaMallocHost((void **)&inf->out_h, ATT1_B200_MAX_BATCH * sizeof(uint32_t)) != cudaSuccess ||
        cudaMallocHost((void **)&inf->err_h, sizeof(int32_t)) != cudaSuccess ||
        cudaMallocHost((void **)&inf->logits_h, (size_t)B * c->vocab * sizeof(float)) != cudaSuccess)
        return ATT1_ERR_OOM;
    if (inf->tp_world > 1) {
        inf->tp_region_bytes = b2_tp_region_bytes(2 * c->n_layers, B * c->d_model, B * inf->vl);
        if ((st = dalloc(inf, (void **)&inf->tp_region, inf->tp_region_bytes)) ||
            (st = dalloc(inf, (void **)&inf->tp_epoch, sizeof(uint32_t))) ||
            (st = dalloc(inf, (void **)&inf->tp_done, sizeof(int32_t))))
            return st;
        inf->tp_peer[inf->tp_rank] = inf->tp_region;
    }
    return ATT1_OK;
}

static att1_status_t new_context(const att1_b200_config *cfg, uint32_t batch, uint32_t rank, uint32_t world,
                                 att1_infer_t **out)
{
    att1_infer_t *inf;
    uint32_t hd;
    att1_status_t st = check_config(cfg, batch);
    if (st != ATT1_OK) return st;
    if (world == 0 || world > B2_TP_MAX || rank >= world) return ATT1_ERR_INVALID_ARG;
    hd = cfg->d_model / cfg->n_heads;
    if (world > 1) {
        /* whole heads, whole 32-column groups and a whole 16-row gate/up tile per rank */
        if (cfg->n_heads % world || cfg->n_kv_heads % world || cfg->d_ff % world || cfg->vocab % world)
            return ATT1_ERR_SHAPE;
        if ((cfg->n_heads / world) * hd % 32 || (cfg->d_ff / world) % 32) return ATT1_ERR_UNSUPPORTED;
    }
    inf = calloc(1, sizeof(*inf));
    if (inf == NULL) return ATT1_ERR_OOM;
    inf->cfg = *cfg;
    if (inf->cfg.group == 0) inf->cfg.group = 32;
    inf->batch = batch;
    inf->tp_rank = rank;
    inf->tp_world = world;
    inf->hq = cfg->n_heads / world;
    inf->hkv = cfg->n_kv_heads / world;
    inf->ffl = cfg->d_ff / world;
    inf->vl = cfg->vocab / world;
    inf->v_off = rank * inf->vl;
    inf->tp_ready = world == 1;
    inf->head_dim = hd;
    inf->q_rows = inf->hq * hd;
    inf->kv_rows = inf->hkv * hd;
    inf->use_graph = 1;
    inf->use_pdl = 1;
    inf->use_persistent = 0;
    if (cudaGetDevice(&inf->device) != cudaSuccess ||
        cudaStreamCreateWithFlags(&inf->stream, cudaStreamNonBlocking) != cudaSuccess) {
        free(inf);
        return ATT1_ERR_UNSUPPORTED;
    }
    inf->layers = calloc(cfg->n_layers, sizeof(dev_layer));
    if (inf->layers == NULL) {
        release(inf);
        return ATT1_ERR_OOM;
    }
    *out = inf;
    return ATT1_OK;
}

static att1_status_t alloc_weights(att1_infer_t *inf, uint32_t fmt)
{
    const att1_b200_config *c = &inf->cfg;
    att1_status_t st;
    uint32_t l;
    for (l = 0; l < c->n_layers; l++) {
        dev_layer *L = &inf->layers[l];
        if ((st = mat_alloc(inf, &L->qkv, fmt, inf->q_rows + 2 * inf->kv_rows, c->d_model)) ||
            (st = mat_alloc(inf, &L->wo, fmt, c->d_model, inf->q_rows)) ||
            (st = mat_alloc(inf, &L->gu, fmt, 2 * inf->ffl, c->d_model)) ||
            (st = mat_alloc(inf, &L->down, fmt, c->d_model, inf->ffl)) ||
            (st = dalloc(inf, (void **)&L->attn_norm, c->d_model * sizeof(float))) ||
            (st = dalloc(inf, (void **)&L->ffn_norm, c->d_model * sizeof(float))))
            return st;
    }
    if ((st = mat_alloc(inf, &inf->output, fmt, inf->vl, c->d_model)) ||
        (st = dalloc(inf, (void **)&inf->embed, (size_t)c->vocab * c->d_model * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->out_norm, c->d_model * sizeof(float))))
        return st;
    return ATT1_OK;
}

static void free_weights(att1_infer_t *inf)
{
    uint32_t l;
    for (l = 0; l < inf->cfg.n_layers; l++) {
        mat_free(&inf->layers[l].qkv);
        mat_free(&inf->layers[l].wo);
        mat_free(&inf->layers[l].gu);
        mat_free(&inf->layers[l].down);
    }
    mat_free(&inf->output);
}

static att1_status_t finish_create(att1_infer_t *inf)
{
    att1_status_t st = build_args(inf);
    cudaError_t e;
    if (st != ATT1_OK) return st;
    e = cudaStreamSynchronize(inf->stream);
    if (e == cudaSuccess) e = cudaGetLastError();
    return b2_cuda_status(e);
}

/* ---- synthetic model -------------------------------------------------------------------------------- */

#define T_PER_LAYER 16u
#define T_EMBED 0x7F000000ull
#define T_OUTPUT 0x7F000002ull

/* rows [row0, row0 + rows) x columns [col0, col0 + cols) of a source tensor
 * with src_cols columns */
static int synth_mat(att1_infer_t *inf, b2_dev_mat *m, uint32_t tile_off, uint32_t rows, uint32_t cols,
                     uint64_t seed, uint64_t tid, uint64_t tid2, int map, uint32_t row0, uint32_t col0,
                     uint32_t src_cols)
{
    if (m->w.format == 4)
        return b2_q4_synth_part(m->data, tile_off, rows, cols, seed, tid, tid2, 0.02f, map, row0, col0, src_cols,
                                inf->stream);
    return b2_q8_synth_part(m->data, m->row_scale, tile_off, rows, cols, seed, tid, tid2, 0.02f, map, row0, col0,
                            src_cols, inf->stream);
}

static att1_status_t create_synth(const att1_b200_config *cfg, uint64_t seed, uint32_t batch, uint32_t rank,
                                  uint32_t world, att1_infer_t **out_infer)
{
    att1_infer_t *inf = NULL;
    att1_status_t st;
    uint32_t l;
    int rc = 0;

    if (out_infer == NULL) return ATT1_ERR_INVALID_ARG;
    *out_infer = NULL;
    st = new_context(cfg, batch, rank, world, &inf);
    if (st != ATT1_OK) return st;
    if ((st = alloc_weights(inf, cfg->dtype)) || (st = alloc_common(inf))) goto fail;
    for (l = 0; l < cfg->n_layers && rc == 0; l++) {
        dev_layer *L = &inf->layers[l];
        const uint64_t b = (uint64_t)l * T_PER_LAYER;
        const uint32_t d = cfg->d_model, qr = inf->q_rows, kr = inf->kv_rows, fl = inf->ffl, r = rank;
        rc |= synth_mat(inf, &L->qkv, 0, qr, d, seed, b + ATT1_B200_WQ, 0, B2_ROWS_PLAIN, r * qr, 0, d);
        rc |= synth_mat(inf, &L->qkv, qr / 16, kr, d, seed, b + ATT1_B200_WK, 0, B2_ROWS_PLAIN, r * kr, 0, d);
        rc |= synth_mat(inf, &L->qkv, (qr + kr) / 16, kr, d, seed, b + ATT1_B200_WV, 0, B2_ROWS_PLAIN, r * kr, 0, d);
        rc |= synth_mat(inf, &L->wo, 0, d, qr, seed, b + ATT1_B200_WO, 0, B2_ROWS_PLAIN, 0, r * qr, world * qr);
        rc |= synth_mat(inf, &L->gu, 0, 2 * fl, d, seed, b + ATT1_B200_GATE, b + ATT1_B200_UP, B2_ROWS_GATEUP, r * fl,
                        0, d);
        rc |= synth_mat(inf, &L->down, 0, d, fl, seed, b + ATT1_B200_DOWN, 0, B2_ROWS_PLAIN, 0, r * fl, world * fl);
        rc |= b2_fill_f32(L->attn_norm, cfg->d_model, 1.0f, inf->stream);
        rc |= b2_fill_f32(L->ffn_norm, cfg->d_model, 1.0f, inf->stream);
    }
    rc |= synth_mat(inf, &inf->output, 0, inf->vl, cfg->d_model, seed, T_OUTPUT, 0, B2_ROWS_PLAIN, inf->v_off, 0,
                    cfg->d_model);
    rc |= b2_synth_f32(inf->embed, (size_t)cfg->vocab * cfg->d_model, seed, T_EMBED, 0.02f, inf->stream);
    rc |= b2_fill_f32(inf->out_norm, cfg->d_model, 1.0f, inf->stream);
    if (rc != 0) {
        st = ATT1_ERR_STATE;
        goto fail;
    }
    /* a tensor-parallel rank is finished when it is connected to its peers */
    if (world > 1) {
        cudaError_t e = cudaStreamSynchronize(inf->stream);
        if (e == cudaSuccess) e = cudaGetLastError();
        if ((st = b2_cuda_status(e)) != ATT1_OK) goto fail;
    } else if ((st = finish_create(inf)) != ATT1_OK) {
        goto fail;
    }
    *out_infer = inf;
    return ATT1_OK;
fail:
    release(inf);
    return st;
}

att1_status_t att1_b200_infer_create_synth(const att1_b200_config *cfg, uint64_t seed, uint32_t batch,
                                           att1_infer_t **out_infer)
{
    return create_synth(cfg, seed, batch, 0, 1, out_infer);
}

att1_status_t att1_b200_infer_create_synth_tp(const att1_b200_config *cfg, uint64_t seed, uint32_t batch,
                                              uint32_t rank, uint32_t world, att1_infer_t **out_infer)
{
    if (world < 2) return ATT1_ERR_INVALID_ARG;
    return create_synth(cfg, seed, batch, rank, world, out_infer);
}

att1_status_t att1_b200_infer_tp_handle(const att1_infer_t *infer, void *handle)
{
    cudaIpcMemHandle_t h;
    if (infer == NULL || handle == NULL || infer->tp_world < 2) return ATT1_ERR_INVALID_ARG;
    if (cudaIpcGetMemHandle(&h, infer->tp_region) != cudaSuccess) return ATT1_ERR_UNSUPPORTED;
    memcpy(handle, &h, sizeof(h));
    return ATT1_OK;
}

static att1_status_t tp_finish(att1_infer_t *inf)
{
    att1_status_t st;
    cudaError_t e;
    if ((st = build_args(inf)) != ATT1_OK) return st;
    e = cudaStreamSynchronize(inf->stream);
    if (e == cudaSuccess) e = cudaGetLastError();
    if ((st = b2_cuda_status(e)) != ATT1_OK) return st;
    inf->tp_ready = 1;
    return ATT1_OK;
}

att1_status_t att1_b200_infer_tp_connect(att1_infer_t *infer, const void *handles)
{
    uint32_t s;
    if (infer == NULL || handles == NULL || infer->tp_world < 2 || infer->tp_ready) return ATT1_ERR_INVALID_ARG;
    for (s = 0; s < infer->tp_world; s++) {
        cudaIpcMemHandle_t h;
        void *p = NULL;
        if (s == infer->tp_rank) continue;
        memcpy(&h, (const uint8_t *)handles + (size_t)s * ATT1_B200_TP_HANDLE_BYTES, sizeof(h));
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            return ATT1_ERR_UNSUPPORTED;
        }
        infer->tp_peer[s] = p;
        infer->tp_opened[s] = 1;
    }
    return tp_finish(infer);
}

att1_status_t att1_b200_infer_tp_disconnect(att1_infer_t *infer)
{
    uint32_t s;
    if (infer == NULL || infer->tp_world < 2) return ATT1_ERR_INVALID_ARG;
    cudaSetDevice(infer->device);
    cudaStreamSynchronize(infer->stream);
    for (s = 0; s < B2_TP_MAX; s++) {
        if (infer->tp_opened[s]) cudaIpcCloseMemHandle(infer->tp_peer[s]);
        infer->tp_opened[s] = 0;
        if (s != infer->tp_rank) infer->tp_peer[s] = NULL;
    }
    infer->tp_ready = 0;
    return ATT1_OK;
}

att1_status_t att1_b200_nccl_unique_id(void *id)
{
    if (id == NULL) return ATT1_ERR_INVALID_ARG;
    if (!b2_nccl_available()) return ATT1_ERR_UNSUPPORTED;
    return b2_nccl_unique_id(id) == 0 ? ATT1_OK : ATT1_ERR_STATE;
}

att1_status_t att1_b200_infer_tp_connect_nccl(att1_infer_t *infer, const void *id)
{
    att1_status_t st;
    if (infer == NULL || id == NULL || infer->tp_world < 2 || infer->tp_ready) return ATT1_ERR_INVALID_ARG;
    if (!b2_nccl_available() || infer->batch > 16 || infer->use_dense) return ATT1_ERR_UNSUPPORTED;
    if (cudaSetDevice(infer->device) != cudaSuccess) return ATT1_ERR_STATE;
    if ((st = dalloc(infer, (void **)&infer->nccl_keys,
                     (size_t)infer->tp_world * infer->batch * sizeof(unsigned long long))) != ATT1_OK)
        return st;
    if (b2_nccl_comm_init(&infer->nccl_comm, (int)infer->tp_world, id, (int)infer->tp_rank) != 0) {
        infer->nccl_comm = NULL;
        return ATT1_ERR_STATE;
    }
    infer->tp_peer[infer->tp_rank] = infer->tp_region;
    if ((st = tp_finish(infer)) != ATT1_OK) return st;
    if (infer->use_dense) return ATT1_ERR_UNSUPPORTED; /* the plan put this batch on the tensor-core route */
    return ATT1_OK;
}

att1_status_t att1_b200_infer_tp_set_wait(att1_infer_t *infer, uint32_t polls)
{
    if (infer == NULL || infer->tp_world < 2) return ATT1_ERR_INVALID_ARG;
    if (infer->step_pending) return ATT1_ERR_STATE;
    cudaSetDevice(infer->device);
    cudaStreamSynchronize(infer->stream);
    if (infer->exec) { /* the graph holds the kernels' parameters: capture again */
        cudaGraphExecDestroy(infer->exec);
        infer->exec = NULL;
    }
    infer->tp_wait_polls = polls;
    if (!infer->tp_ready) return ATT1_OK; /* wired at connect */
    return build_args(infer);
}

/* The exchange region holds flags that carry a step epoch: a rank whose step
 * failed (a timed-out wait) may have published points of that step that the
 * others never consumed. Zeroing every rank's flags and epochs, with no rank
 * stepping, puts all of them back at epoch 0 together. */
att1_status_t att1_b200_infer_tp_reset(att1_infer_t *infer)
{
    const att1_b200_config *c;
    size_t flag_bytes;
    if (infer == NULL || infer->tp_world < 2) return ATT1_ERR_INVALID_ARG;
    if (infer->step_pending) return ATT1_ERR_STATE;
    c = &infer->cfg;
    cudaSetDevice(infer->device);
    flag_bytes = ((size_t)(2 * c->n_layers + 1) * B2_TP_MAX + B2_TP_MAX * B2_TP_MAX_ITEMS) * sizeof(uint64_t);
    if (cudaStreamSynchronize(infer->stream) != cudaSuccess ||
        cudaMemsetAsync(infer->tp_region, 0, flag_bytes, infer->stream) != cudaSuccess ||
        cudaMemsetAsync(infer->tp_epoch, 0, sizeof(uint32_t), infer->stream) != cudaSuccess ||
        cudaMemsetAsync(infer->tp_done, 0, sizeof(int32_t), infer->stream) != cudaSuccess ||
        cudaMemsetAsync(infer->err_d, 0, sizeof(int32_t), infer->stream) != cudaSuccess ||
        cudaStreamSynchronize(infer->stream) != cudaSuccess)
        return ATT1_ERR_STATE;
    return ATT1_OK;
}

att1_status_t att1_b200_infer_tp_connect_local(att1_infer_t *const *infers, uint32_t world)
{
    uint32_t r, s;
    att1_status_t st;
    if (infers == NULL || world < 2 || world > B2_TP_MAX) return ATT1_ERR_INVALID_ARG;
    for (r = 0; r < world; r++)
        if (infers[r] == NULL || infers[r]->tp_world != world || infers[r]->tp_rank != r || infers[r]->tp_ready)
            return ATT1_ERR_INVALID_ARG;
    for (r = 0; r < world; r++) {
        int dev = infers[r]->device;
        if (cudaSetDevice(dev) != cudaSuccess) return ATT1_ERR_STATE;
        for (s = 0; s < world; s++) {
            int ok = 0;
            if (infers[s]->device == dev) continue;
            if (cudaDeviceCanAccessPeer(&ok, dev, infers[s]->device) != cudaSuccess || !ok) return ATT1_ERR_UNSUPPORTED;
            if (cudaDeviceEnablePeerAccess(infers[s]->device, 0) != cudaSuccess) {
                if (cudaGetLastError() != cudaErrorPeerAccessAlreadyEnabled) return ATT1_ERR_UNSUPPORTED;
            }
        }
        for (s = 0; s < world; s++) infers[r]->tp_peer[s] = infers[s]->tp_region;
    }
    for (r = 0; r < world; r++) {
        if (cudaSetDevice(infers[r]->device) != cudaSuccess) return ATT1_ERR_STATE;
        if ((st = tp_finish(infers[r])) != ATT1_OK) return st;
    }
    return ATT1_OK;
}

/* ---- model from a .att1 file ------------------------------------------------------------------------ */

static const att1_model_tensor *find_tensor(const att1_model *m, uint32_t layer, const char *suffix)
{
    char name[ATT1_MODEL_NAME_SIZE];
    if (layer == UINT32_MAX) return att1_model_find_tensor(m, suffix);
    if (snprintf(name, sizeof(name), "layers.%u.%s", layer, suffix) >= (int)sizeof(name)) return NULL;
    return att1_model_find_tensor(m, name);
}

static int is_shape(const att1_model_tensor *t, uint32_t dtype, uint32_t nd, uint64_t d0, uint64_t d1)
{
    return t != NULL && t->dtype == dtype && t->ndims == nd && t->shape[0] == d0 && (nd < 2 || t->shape[1] == d1);
}

/* Upload a host tensor payload to a temporary device buffer. */
static att1_status_t upload_tmp(att1_infer_t *inf, const att1_model_tensor *t, void **dev)
{
    cudaError_t e = cudaMalloc(dev, t->nbytes);
    if (e != cudaSuccess) return b2_cuda_status(e);
    e = cudaMemcpyAsync(*dev, t->data, t->nbytes, cudaMemcpyHostToDevice, inf->stream);
    return b2_cuda_status(e);
}

static uint32_t q4_group_of(const att1_model_tensor *t)
{
    uint32_t g = t->flags & 0xFFu;
    return g == 0 ? 32u : g;
}

/* q4 tensors (rows x cols each) -> units at tile_off, optionally interleaved. */
static att1_status_t load_q4(att1_infer_t *inf, b2_dev_mat *m, uint32_t tile_off, const att1_model_tensor *t0,
                             const att1_model_tensor *t1)
{
    void *d0 = NULL, *d1 = NULL;
    att1_status_t st;
    const uint32_t rows = (uint32_t)t0->shape[0], cols = (uint32_t)t0->shape[1];
    const size_t pb = (size_t)rows * cols / 2;
    int rc;
    if ((st = upload_tmp(inf, t0, &d0)) != ATT1_OK) goto out;
    if (t1 != NULL && (st = upload_tmp(inf, t1, &d1)) != ATT1_OK) goto out;
    rc = b2_q4_pack(m->data, tile_off, t1 ? 2 * rows : rows, cols, (const uint8_t *)d0,
                    (const float *)((const uint8_t *)d0 + pb), (const uint8_t *)d1,
                    d1 ? (const float *)((const uint8_t *)d1 + pb) : NULL, q4_group_of(t0),
                    t1 ? B2_ROWS_GATEUP : B2_ROWS_PLAIN, inf->stream);
    st = rc == 0 ? ATT1_OK : (rc == -1 ? ATT1_ERR_UNSUPPORTED : ATT1_ERR_STATE);
    if (st == ATT1_OK) st = b2_cuda_status(cudaStreamSynchronize(inf->stream));
out:
    if (d0) cudaFree(d0);
    if (d1) cudaFree(d1);
    return st;
}

/* q8 from file: q8 tensors [out][in], or f32 tensors [in][out] quantised
 * per output row on the device (src/infer.c:196-233, 337-433). */
static att1_status_t load_q8(att1_infer_t *inf, b2_dev_mat *m, uint32_t tile_off, const att1_model_tensor *t0,
                             const att1_model_tensor *t1)
{
    void *d0 = NULL, *d1 = NULL;
    att1_status_t st;
    int rc;
    if ((st = upload_tmp(inf, t0, &d0)) != ATT1_OK) goto out;
    if (t1 != NULL && (st = upload_tmp(inf, t1, &d1)) != ATT1_OK) goto out;
    if (t0->dtype == ATT1_MODEL_DTYPE_Q8) {
        const uint32_t rows = (uint32_t)t0->shape[0], cols = (uint32_t)t0->shape[1];
        const size_t vb = (size_t)rows * cols;
        rc = b2_q8_pack(m->data, m->row_scale, tile_off, t1 ? 2 * rows : rows, cols, (const int8_t *)d0,
                        (const float *)((const uint8_t *)d0 + vb), (const int8_t *)d1,
                        d1 ? (const float *)((const uint8_t *)d1 + vb) : NULL, t1 ? B2_ROWS_GATEUP : B2_ROWS_PLAIN,
                        inf->stream);
    } else {
        const uint32_t in = (uint32_t)t0->shape[0], outr = (uint32_t)t0->shape[1];
        rc = b2_q8_quantize_f32(m->data, m->row_scale, tile_off, t1 ? 2 * outr : outr, in, (const float *)d0,
                                (const float *)d1, 1, t1 ? B2_ROWS_GATEUP : B2_ROWS_PLAIN, inf->stream);
    }
    st = rc == 0 ? ATT1_OK : ATT1_ERR_STATE;
    if (st == ATT1_OK) st = b2_cuda_status(cudaStreamSynchronize(inf->stream));
out:
    if (d0) cudaFree(d0);
    if (d1) cudaFree(d1);
    return st;
}

static att1_status_t upload_f32(att1_infer_t *inf, float *dst, const att1_model_tensor *t)
{
    return b2_cuda_status(cudaMemcpyAsync(dst, t->data, t->nbytes, cudaMemcpyHostToDevice, inf->stream));
}

/* ---- tensor-parallel shards of file tensors --------------------------------------------------- */

/* Host copy of rows [r0, r0 + nr) x columns [c0, c0 + nc) of a q4 or q8 file
 * tensor, in the tensor's own layout (q4: packed nibbles then group scales;
 * q8: int8 values then one scale per row, the whole source row's), described
 * by `view`. Shards keep whole q4 groups, so the bytes equal those of the
 * reference's quantisation of the full matrix. */
static att1_status_t slice_quant(const att1_model_tensor *t, uint64_t r0, uint64_t nr, uint64_t c0, uint64_t nc,
                                 att1_model_tensor *view, uint8_t **buf)
{
    const uint64_t cols = t->shape[1];
    const uint8_t *src = (const uint8_t *)t->data;
    uint8_t *out;
    uint64_t r;
    *buf = NULL;
    *view = *t;
    if (t->dtype == ATT1_MODEL_DTYPE_Q4) {
        const uint64_t g = q4_group_of(t), rows = t->shape[0];
        const float *sc = (const float *)(src + rows * cols / 2);
        float *os;
        if (c0 % g || nc % g) return ATT1_ERR_UNSUPPORTED;
        out = malloc(nr * nc / 2 + nr * (nc / g) * sizeof(float));
        if (out == NULL) return ATT1_ERR_OOM;
        for (r = 0; r < nr; r++) memcpy(out + r * nc / 2, src + (r0 + r) * cols / 2 + c0 / 2, nc / 2);
        os = (float *)(out + nr * nc / 2);
        for (r = 0; r < nr; r++)
            memcpy(os + r * (nc / g), sc + (r0 + r) * (cols / g) + c0 / g, (nc / g) * sizeof(float));
        view->nbytes = nr * nc / 2 + nr * (nc / g) * sizeof(float);
    } else {
        const uint64_t rows = t->shape[0];
        const float *sc = (const float *)(src + rows * cols);
        out = malloc(nr * nc + nr * sizeof(float));
        if (out == NULL) return ATT1_ERR_OOM;
        for (r = 0; r < nr; r++) memcpy(out + r * nc, src + (r0 + r) * cols + c0, nc);
        memcpy(out + nr * nc, sc + r0, nr * sizeof(float));
        view->nbytes = nr * nc + nr * sizeof(float);
    }
    view->shape[0] = nr;
    view->shape[1] = nc;
    view->data = out;
    *buf = out;
    return ATT1_OK;
}

/* Host copy of output columns [o0, o0 + no) of an f32 tensor stored [in][out]. */
static att1_status_t slice_f32_out(const att1_model_tensor *t, uint64_t o0, uint64_t no, att1_model_tensor *view,
                                   uint8_t **buf)
{
    const uint64_t in = t->shape[0], outd = t->shape[1];
    const float *src = (const float *)t->data;
    float *out = malloc(in * no * sizeof(float));
    uint64_t i;
    *buf = (uint8_t *)out;
    if (out == NULL) return ATT1_ERR_OOM;
    for (i = 0; i < in; i++) memcpy(out + i * no, src + i * outd + o0, no * sizeof(float));
    *view = *t;
    view->shape[1] = no;
    view->nbytes = in * no * sizeof(float);
    view->data = out;
    return ATT1_OK;
}

/* q8 from an f32 [in][out] tensor, input rows [i0, i0 + ni) of every output
 * row: the whole matrix is quantised on the device (each row's scale from all
 * of its inputs, src/quant.c:61-116) and this shard's 32-column units copied. */
static att1_status_t load_q8_f32_cols(att1_infer_t *inf, b2_dev_mat *m, const att1_model_tensor *t, uint64_t i0,
                                      uint64_t ni)
{
    const uint32_t in = (uint32_t)t->shape[0], outr = (uint32_t)t->shape[1], tiles = (outr + 15) / 16;
    const size_t ku_all = in / 32, ku0 = i0 / 32, nku = ni / 32;
    void *d0 = NULL, *units = NULL;
    float *rs = NULL;
    att1_status_t st;
    cudaError_t e;
    if (in % 32 || i0 % 32 || ni % 32) return ATT1_ERR_UNSUPPORTED;
    if ((st = upload_tmp(inf, t, &d0)) != ATT1_OK) goto out;
    if ((e = cudaMalloc(&units, b2_q8_bytes(outr, in))) != cudaSuccess ||
        (e = cudaMalloc((void **)&rs, (size_t)tiles * 16 * sizeof(float))) != cudaSuccess) {
        st = b2_cuda_status(e);
        goto out;
    }
    if (b2_q8_quantize_f32(units, rs, 0, outr, in, (const float *)d0, NULL, 1, B2_ROWS_PLAIN, inf->stream) != 0) {
        st = ATT1_ERR_STATE;
        goto out;
    }
    e = cudaMemcpy2DAsync(m->data, nku * B2_Q8_UNIT_BYTES, (const uint8_t *)units + ku0 * B2_Q8_UNIT_BYTES,
                          ku_all * B2_Q8_UNIT_BYTES, nku * B2_Q8_UNIT_BYTES, tiles, cudaMemcpyDeviceToDevice,
                          inf->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->row_scale, rs, (size_t)tiles * 16 * sizeof(float), cudaMemcpyDeviceToDevice,
                            inf->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(inf->stream);
    st = b2_cuda_status(e);
out:
    if (d0) cudaFree(d0);
    if (units) cudaFree(units);
    if (rs) cudaFree(rs);
    return st;
}

/* One matrix (or the gate/up pair) of this rank: rows [r0, r0 + nr) when
 * `by_rows`, else input columns [r0, r0 + nr); the whole tensor at world 1. */
static att1_status_t load_shard(att1_infer_t *inf, uint32_t fmt, b2_dev_mat *m, uint32_t tile_off,
                                const att1_model_tensor *t0, const att1_model_tensor *t1, int by_rows, uint64_t r0,
                                uint64_t nr)
{
    att1_model_tensor v0, v1;
    uint8_t *b0 = NULL, *b1 = NULL;
    att1_status_t st;
    const int f32 = t0->dtype == ATT1_MODEL_DTYPE_F32;
    if (inf->tp_world == 1) return (fmt == 4 ? load_q4 : load_q8)(inf, m, tile_off, t0, t1);
    if (f32 && !by_rows) {
        if (t1 != NULL) return ATT1_ERR_UNSUPPORTED;
        return load_q8_f32_cols(inf, m, t0, r0, nr);
    }
    if (f32) {
        st = slice_f32_out(t0, r0, nr, &v0, &b0);
        if (st == ATT1_OK && t1 != NULL) st = slice_f32_out(t1, r0, nr, &v1, &b1);
    } else if (by_rows) {
        st = slice_quant(t0, r0, nr, 0, t0->shape[1], &v0, &b0);
        if (st == ATT1_OK && t1 != NULL) st = slice_quant(t1, r0, nr, 0, t1->shape[1], &v1, &b1);
    } else {
        st = slice_quant(t0, 0, t0->shape[0], r0, nr, &v0, &b0);
    }
    if (st == ATT1_OK) st = (fmt == 4 ? load_q4 : load_q8)(inf, m, tile_off, &v0, t1 ? &v1 : NULL);
    free(b0);
    free(b1);
    return st;
}

/* Validate (src/model_view.c:221-366) and upload one precision's weights
 * (this rank's shard under tensor parallelism). */
/* check_only: validate every tensor the precision needs and load nothing, so a
 * precision switch that the file cannot serve leaves the context as it was. */
static att1_status_t load_model_weights(att1_infer_t *inf, const att1_model *m, uint32_t fmt, int check_only)
{
    const att1_model_config *mc = &m->config;
    const uint64_t d = mc->d_model, f = mc->d_ff, V = mc->vocab_size;
    const att1_model_tensor *emb = find_tensor(m, UINT32_MAX, "tok_embeddings.weight");
    const att1_model_tensor *onorm = find_tensor(m, UINT32_MAX, "output_norm.weight");
    const att1_model_tensor *outw = find_tensor(m, UINT32_MAX, "output.weight");
    const int file_q8 = outw != NULL && outw->dtype == ATT1_MODEL_DTYPE_Q8;
    att1_status_t st;
    uint32_t l;

    if (emb == NULL || onorm == NULL || outw == NULL) return ATT1_ERR_NOT_FOUND;
    if (!is_shape(emb, ATT1_MODEL_DTYPE_F32, 2, V, d) || !is_shape(onorm, ATT1_MODEL_DTYPE_F32, 1, d, 1))
        return ATT1_ERR_SHAPE;
    if (fmt == 4 && !is_shape(outw, ATT1_MODEL_DTYPE_Q4, 2, V, d)) return ATT1_ERR_SHAPE;
    if (fmt == 8 && !(file_q8 ? is_shape(outw, ATT1_MODEL_DTYPE_Q8, 2, V, d)
                              : is_shape(outw, ATT1_MODEL_DTYPE_F32, 2, d, V)))
        return ATT1_ERR_SHAPE;
    for (l = 0; l < mc->n_layers; l++) {
        const att1_model_tensor *an = find_tensor(m, l, "attention_norm.weight");
        const att1_model_tensor *fn = find_tensor(m, l, "ffn_norm.weight");
        const char *names[7] = {"attention.wq.weight", "attention.wk.weight", "attention.wv.weight",
                                "attention.wo.weight", "ffn.w_gate.weight",   "ffn.w_up.weight",
                                "ffn.w_down.weight"};
        const att1_model_tensor *t[7];
        int k;
        if (an == NULL || fn == NULL) return ATT1_ERR_NOT_FOUND;
        if (!is_shape(an, ATT1_MODEL_DTYPE_F32, 1, d, 1) || !is_shape(fn, ATT1_MODEL_DTYPE_F32, 1, d, 1))
            return ATT1_ERR_SHAPE;
        for (k = 0; k < 7; k++) {
            /* [out][in] for q4/q8 tensors, [in][out] for f32 */
            const uint64_t out_d = (k >= 4 && k <= 5) ? f : d, in_d = (k == 6) ? f : d;
            t[k] = find_tensor(m, l, names[k]);
            if (t[k] == NULL) return ATT1_ERR_NOT_FOUND;
            if (fmt == 4 && !is_shape(t[k], ATT1_MODEL_DTYPE_Q4, 2, out_d, in_d)) return ATT1_ERR_SHAPE;
            if (fmt == 8 && !(file_q8 ? is_shape(t[k], ATT1_MODEL_DTYPE_Q8, 2, out_d, in_d)
                                      : is_shape(t[k], ATT1_MODEL_DTYPE_F32, 2, in_d, out_d)))
                return ATT1_ERR_SHAPE;
        }
        if (!check_only) {
            dev_layer *L = &inf->layers[l];
            const uint64_t r = inf->tp_rank, qr = inf->q_rows, kr = inf->kv_rows, fl = inf->ffl;
            if ((st = load_shard(inf, fmt, &L->qkv, 0, t[0], NULL, 1, r * qr, qr)) ||
                (st = load_shard(inf, fmt, &L->qkv, inf->q_rows / 16, t[1], NULL, 1, r * kr, kr)) ||
                (st = load_shard(inf, fmt, &L->qkv, (inf->q_rows + inf->kv_rows) / 16, t[2], NULL, 1, r * kr, kr)) ||
                (st = load_shard(inf, fmt, &L->wo, 0, t[3], NULL, 0, r * qr, qr)) ||
                (st = load_shard(inf, fmt, &L->gu, 0, t[4], t[5], 1, r * fl, fl)) ||
                (st = load_shard(inf, fmt, &L->down, 0, t[6], NULL, 0, r * fl, fl)) ||
                (st = upload_f32(inf, L->attn_norm, an)) || (st = upload_f32(inf, L->ffn_norm, fn)))
                return st;
        }
    }
    if (check_only) return ATT1_OK;
    if ((st = load_shard(inf, fmt, &inf->output, 0, outw, NULL, 1, inf->v_off, inf->vl)) ||
        (st = upload_f32(inf, inf->embed, emb)) || (st = upload_f32(inf, inf->out_norm, onorm)))
        return st;
    return b2_cuda_status(cudaStreamSynchronize(inf->stream));
}

static att1_status_t create_model(const att1_model *model, uint32_t dtype, float eps, float final_eps, float theta,
                                  uint32_t rank, uint32_t world, att1_infer_t **out_infer)
{
    att1_b200_config c;
    att1_infer_t *inf = NULL;
    att1_status_t st;
    if (out_infer == NULL) return ATT1_ERR_INVALID_ARG;
    *out_infer = NULL;
    if (model == NULL) return ATT1_ERR_INVALID_ARG;
    memset(&c, 0, sizeof(c));
    c.vocab = model->config.vocab_size;
    c.n_layers = model->config.n_layers;
    c.n_heads = model->config.n_heads;
    c.n_kv_heads = model->config.n_heads;
    c.d_model = model->config.d_model;
    c.d_ff = model->config.d_ff;
    c.max_seq = model->config.max_seq_len;
    c.group = 32;
    c.dtype = dtype;
    c.eps = eps;
    c.final_eps = final_eps;
    c.theta = theta;
    if (c.vocab == 0 || c.n_layers == 0 || c.n_heads == 0 || c.d_model == 0 || c.d_ff == 0 || c.max_seq == 0 ||
        c.d_model % c.n_heads || ((c.d_model / c.n_heads) % 2))
        return ATT1_ERR_INVALID_ARG;
    st = new_context(&c, 1, rank, world, &inf);
    if (st != ATT1_OK) return st;
    inf->model = model;
    if ((st = alloc_weights(inf, dtype)) || (st = alloc_common(inf)) || (st = load_model_weights(inf, model, dtype, 0)))
        goto fail;
    /* a tensor-parallel rank is finished when it is connected to its peers */
    if (world > 1) {
        cudaError_t e = cudaStreamSynchronize(inf->stream);
        if (e == cudaSuccess) e = cudaGetLastError();
        st = b2_cuda_status(e);
    } else {
        st = finish_create(inf);
    }
    if (st != ATT1_OK) goto fail;
    *out_infer = inf;
    return ATT1_OK;
fail:
    release(inf);
    return st;
}

att1_status_t att1_b200_infer_create_model(const att1_model *model, uint32_t dtype, float eps, float final_eps,
                                           float theta, att1_infer_t **out_infer)
{
    return create_model(model, dtype, eps, final_eps, theta, 0, 1, out_infer);
}

att1_status_t att1_b200_infer_create_model_tp(const att1_model *model, uint32_t dtype, float eps, float final_eps,
                                              float theta, uint32_t rank, uint32_t world, att1_infer_t **out_infer)
{
    return create_model(model, dtype, eps, final_eps, theta, rank, world, out_infer);
}

att1_status_t att1_infer_create_q4(const att1_model *model, att1_infer_t **out_infer)
{
    /* src/infer.c:721-722 and :823: eps 1e-6, theta 10000 for file models */
    att1_status_t st = att1_b200_infer_create_model(model, 4, 0.000001f, 0.000001f, 10000.0f, out_infer);
    if (st == ATT1_OK && att1_backend_cuda_q4_create(&(*out_infer)->backend) != ATT1_OK) {
        att1_infer_destroy(*out_infer);
        *out_infer = NULL;
        return ATT1_ERR_STATE;
    }
    return st;
}

att1_status_t att1_infer_create(const att1_model *model, att1_infer_t **out_infer)
{
    att1_status_t st = att1_b200_infer_create_model(model, 8, 0.000001f, 0.000001f, 10000.0f, out_infer);
    if (st == ATT1_OK && att1_backend_cuda_q8_create(&(*out_infer)->backend) != ATT1_OK) {
        att1_infer_destroy(*out_infer);
        *out_infer = NULL;
        return ATT1_ERR_STATE;
    }
    return st;
}

void att1_infer_destroy(att1_infer_t *infer)
{
    release(infer);
}

uint32_t att1_b200_infer_batch(const att1_infer_t *infer)
{
    return infer ? infer->batch : 0;
}

size_t att1_b200_infer_device_bytes(const att1_infer_t *infer)
{
    return infer ? infer->device_bytes : 0;
}

void *att1_b200_infer_stream(const att1_infer_t *infer)
{
    return infer ? (void *)infer->stream : NULL;
}

/* ---- the decode step ------------------------------------------------------------------------------------- */

/* ---- the tensor-core route: GEMM + row epilogues ------------------------------------------------ */

/* Buffers of one pass of m rows (a decode batch, or a prompt chunk). */
typedef struct dense_bufs {
    uint32_t m;
    float *x, *h, *q, *ctx, *hs, *y_qkv, *y_gu, *y_part; /* y_part: a rank's partial [m][d] (tensor parallel) */
    const int32_t *positions, *page_table; /* page_table: NULL = each layer's own (kv_layout) */
    size_t pt_layer_stride;                /* int32 elements from one layer's page_table rows to the next's */
    void *xs, *gscratch, *ascratch;
    size_t xs_bytes, gscratch_bytes, ascratch_bytes;
    int32_t *acounters;
    uint32_t acounters_len;
} dense_bufs;

static void gemm_init(att1_infer_t *inf, b2_gemm_args *g, const b2_dev_mat *w, const dense_bufs *b)
{
    memset(g, 0, sizeof(*g));
    g->w = w->w;
    g->xs = b->xs;
    g->m = b->m;
    g->scratch = b->gscratch;
    g->scratch_bytes = b->gscratch_bytes;
    g->err = inf->err_d;
    g->pdl = inf->use_pdl;
}

/* x (optionally RMS-normed) times W^T: prep + GEMM (+ split reduction). */
static int dense_gemm(att1_infer_t *inf, const dense_bufs *b, const b2_dev_mat *w, const float *x, uint32_t x_stride,
                      const float *norm_w, float eps, uint32_t epilogue, float *out, uint32_t out_stride,
                      const float *resid, cudaStream_t st)
{
    b2_gemm_args g;
    int rc = b2_gemm_prep(x, x_stride, b->m, w->w.cols, norm_w, eps, b->xs, inf->err_d, st);
    if (rc != 0) return rc;
    gemm_init(inf, &g, w, b);
    g.epilogue = epilogue;
    g.out = out;
    g.out_stride = out_stride;
    g.resid = resid;
    return b2_gemm(&g, st);
}

/* One transformer block (src/transformer_block.c:417-557) over b->m rows. */
static int dense_layer(att1_infer_t *inf, uint32_t l, const dense_bufs *b, cudaStream_t st)
{
    const att1_b200_config *c = &inf->cfg;
    dev_layer *L = &inf->layers[l];
    const uint32_t d = c->d_model, qkv = inf->q_rows + 2 * inf->kv_rows;
    b2_rows_args r;
    b2_attn_args at;
    int rc = dense_gemm(inf, b, &L->qkv, b->x, d, L->attn_norm, c->eps, B2_EPI_STORE, b->y_qkv, qkv, NULL, st);
    if (rc != 0) return rc;
    memset(&r, 0, sizeof(r));
    r.epilogue = B2_EPI_QKV;
    r.m = b->m;
    r.y = b->y_qkv;
    r.y_stride = qkv;
    r.rows = qkv;
    r.out = b->q;
    r.out_stride = inf->q_rows;
    r.q_rows = inf->q_rows;
    r.kv_rows = inf->kv_rows;
    r.rope_freq = inf->rope_freq;
    r.positions = b->positions;
    r.kv = kv_layout(inf, l);
    if (b->page_table != NULL) r.kv.page_table = b->page_table + (size_t)l * b->pt_layer_stride;
    r.err = inf->err_d;
    r.pdl = inf->use_pdl;
    if ((rc = b2_rows_epilogue(&r, st)) != 0) return rc;
    at = L->a_attn;
    at.batch = b->m;
    at.q = b->q;
    at.kv = r.kv;
    at.positions = b->positions;
    at.ctx = b->ctx;
    at.scratch = b->ascratch;
    at.scratch_bytes = b->ascratch_bytes;
    at.counters = b->acounters;
    at.counters_len = b->acounters_len;
    at.pdl = inf->use_pdl;
    if ((rc = b2_attn(&at, st)) != 0) return rc;
    if (inf->tp_world > 1) {
        /* this rank's heads' share of WO; h = x + the ranks' shares in rank order */
        if ((rc = dense_gemm(inf, b, &L->wo, b->ctx, inf->q_rows, NULL, 0.0f, B2_EPI_STORE, b->y_part, d, NULL,
                             st)) != 0 ||
            (rc = b2_tp_push(b->y_part, b->m * d, &inf->tp_base, 2 * l, st)) != 0 ||
            (rc = b2_tp_sum(b->x, b->h, b->m * d, &inf->tp_base, 2 * l, inf->err_d, st)) != 0)
            return rc;
    } else if ((rc = dense_gemm(inf, b, &L->wo, b->ctx, inf->q_rows, NULL, 0.0f, B2_EPI_RESID, b->h, d, b->x,
                                st)) != 0)
        return rc;
    if ((rc = dense_gemm(inf, b, &L->gu, b->h, d, L->ffn_norm, c->eps, B2_EPI_STORE, b->y_gu, 2 * inf->ffl, NULL,
                         st)) != 0)
        return rc;
    memset(&r, 0, sizeof(r));
    r.epilogue = B2_EPI_SWIGLU;
    r.m = b->m;
    r.y = b->y_gu;
    r.y_stride = 2 * inf->ffl;
    r.rows = 2 * inf->ffl;
    r.out = b->hs;
    r.out_stride = inf->ffl;
    r.err = inf->err_d;
    r.pdl = inf->use_pdl;
    if ((rc = b2_rows_epilogue(&r, st)) != 0) return rc;
    if (inf->tp_world > 1) {
        if ((rc = dense_gemm(inf, b, &L->down, b->hs, inf->ffl, NULL, 0.0f, B2_EPI_STORE, b->y_part, d, NULL, st)) !=
                0 ||
            (rc = b2_tp_push(b->y_part, b->m * d, &inf->tp_base, 2 * l + 1, st)) != 0)
            return rc;
        return b2_tp_sum(b->h, b->x, b->m * d, &inf->tp_base, 2 * l + 1, inf->err_d, st);
    }
    return dense_gemm(inf, b, &L->down, b->hs, inf->ffl, NULL, 0.0f, B2_EPI_RESID, b->x, d, b->h, st);
}

/* Scratch of the GEMMs of one m-row pass (the largest k-split partials). */
static size_t dense_gscratch(att1_infer_t *inf, uint32_t m)
{
    /* every layer has the shapes of layer 0 */
    const b2_dev_mat *ws[4] = {&inf->layers[0].qkv, &inf->layers[0].wo, &inf->layers[0].gu, &inf->layers[0].down};
    b2_gemm_args g;
    size_t need = 16, s;
    uint32_t k;
    for (k = 0; k < 4; k++) {
        memset(&g, 0, sizeof(g));
        g.w = ws[k]->w;
        g.xs = inf->embed; /* any aligned non-null pointer: only the plan is asked for */
        g.out = inf->embed;
        g.out_stride = ws[k]->w.rows;
        g.m = m;
        if ((s = b2_gemm_scratch_bytes(&g)) > need) need = s;
    }
    memset(&g, 0, sizeof(g));
    g.w = inf->output.w;
    g.xs = inf->embed;
    g.out = inf->embed;
    g.out_stride = inf->output.w.rows;
    g.m = m;
    if ((s = b2_gemm_scratch_bytes(&g)) > need) need = s;
    return need;
}

static size_t dense_xs(att1_infer_t *inf, uint32_t m)
{
    size_t a = b2_gemm_xs_bytes(m, inf->cfg.d_model), b = b2_gemm_xs_bytes(m, inf->q_rows),
           f = b2_gemm_xs_bytes(m, inf->ffl);
    if (b > a) a = b;
    return f > a ? f : a;
}

/* Decode through the GEMM: buffers for the context's batch. */
static att1_status_t dense_alloc(att1_infer_t *inf)
{
    const uint32_t B = inf->batch;
    att1_status_t st;
    dfree(inf->y_qkv);
    dfree(inf->y_gu);
    dfree(inf->y_part);
    dfree(inf->xs);
    dfree(inf->gscratch);
    inf->y_qkv = inf->y_gu = inf->y_part = NULL;
    inf->xs = inf->gscratch = NULL;
    inf->xs_bytes = dense_xs(inf, B);
    inf->gscratch_bytes = dense_gscratch(inf, B);
    if ((st = dalloc(inf, (void **)&inf->y_qkv, (size_t)B * (inf->q_rows + 2 * inf->kv_rows) * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->y_gu, (size_t)B * 2 * inf->ffl * sizeof(float))) ||
        (st = dalloc(inf, &inf->xs, inf->xs_bytes)) || (st = dalloc(inf, &inf->gscratch, inf->gscratch_bytes)))
        return st;
    if (inf->tp_world > 1 &&
        (st = dalloc(inf, (void **)&inf->y_part, (size_t)B * inf->cfg.d_model * sizeof(float))) != ATT1_OK)
        return st;
    return ATT1_OK;
}

static void decode_bufs(att1_infer_t *inf, dense_bufs *b)
{
    memset(b, 0, sizeof(*b));
    b->m = inf->batch;
    b->x = inf->x;
    b->h = inf->h1;
    b->q = inf->q;
    b->ctx = inf->ctx;
    b->hs = inf->hs;
    b->y_qkv = inf->y_qkv;
    b->y_gu = inf->y_gu;
    b->y_part = inf->y_part;
    b->positions = inf->pos_d;
    b->page_table = NULL; /* each layer's own table rows (kv_layout) */
    b->xs = inf->xs;
    b->xs_bytes = inf->xs_bytes;
    b->gscratch = inf->gscratch;
    b->gscratch_bytes = inf->gscratch_bytes;
    b->ascratch = inf->scratch;
    b->ascratch_bytes = inf->scratch_bytes;
    b->acounters = inf->counters;
    b->acounters_len = inf->counters_len;
}

/* Final RMSNorm + lm_head + argmax keys for b->m rows of x. */
static int dense_head(att1_infer_t *inf, const dense_bufs *b, cudaStream_t st)
{
    b2_rows_args r;
    int rc = dense_gemm(inf, b, &inf->output, b->x, inf->cfg.d_model, inf->out_norm, inf->cfg.final_eps, B2_EPI_STORE,
                        inf->logits, inf->vl, NULL, st);
    if (rc != 0) return rc;
    memset(&r, 0, sizeof(r));
    r.epilogue = B2_EPI_LOGITS;
    r.m = b->m;
    r.y = inf->logits;
    r.y_stride = inf->vl;
    r.rows = inf->vl;
    r.argmax = inf->argmax_d;
    r.row_offset = inf->v_off;
    r.err = inf->err_d;
    r.pdl = inf->use_pdl;
    if ((rc = b2_rows_epilogue(&r, st)) != 0 || inf->tp_world == 1) return rc;
    /* this rank's vocabulary rows and argmax keys to every rank */
    return b2_tp_push_logits(inf->logits, b->m, inf->vl, inf->argmax_d, &inf->tp_base, st);
}

/* Top-k / temperature draw over the step's logits (greedy: nothing to do;
 * the step end has written the argmax tokens and advanced the positions). */
static int sample_step(att1_infer_t *inf, cudaStream_t st)
{
    if (inf->top_k <= 1) return 0;
    if (inf->tp_world > 1) {
        /* every rank draws from the same all-gathered logits: rank s's rows
         * [batch][vl] in logits slot s of this rank's exchange region */
        const float *all = (const float *)(inf->tp_region + b2_tp_region_bytes(2 * inf->cfg.n_layers,
                                                                              inf->batch * inf->cfg.d_model, 0));
        return b2_sample_topk_sharded(all, inf->batch, inf->cfg.vocab, inf->vl, (size_t)inf->batch * inf->vl, inf->vl,
                                      inf->top_k, inf->temperature, inf->sample_seed, inf->pos_d, inf->tokens_d,
                                      inf->use_pdl, st);
    }
    return b2_sample_topk(inf->logits, inf->batch, inf->cfg.vocab, inf->vl, inf->top_k, inf->temperature,
                          inf->sample_seed, inf->pos_d, inf->tokens_d, inf->use_pdl, st);
}

static int enqueue_kernels(att1_infer_t *inf)
{
    const att1_b200_config *c = &inf->cfg;
    cudaStream_t st = inf->stream;
    uint32_t l;
    int rc = b2_step_begin(inf->embed, c->vocab, c->d_model, inf->tokens_d, inf->batch, inf->x, inf->argmax_d,
                           inf->err_d, inf->use_pdl, st);
    if (inf->use_dense) {
        dense_bufs b;
        decode_bufs(inf, &b);
        for (l = 0; l < c->n_layers && rc == 0; l++) rc = dense_layer(inf, l, &b, st);
        if (rc == 0) rc = dense_head(inf, &b, st);
        if (rc != 0) return rc;
        if (inf->tp_world > 1)
            rc = b2_step_end_tp(&inf->tp_base, inf->batch, inf->tokens_d, inf->pos_d, inf->err_d, inf->use_pdl, st);
        else
            rc = b2_step_end(inf->argmax_d, inf->batch, inf->tokens_d, inf->pos_d, inf->err_d, inf->use_pdl, st);
        return rc != 0 ? rc : sample_step(inf, st);
    }
    if (inf->nccl_comm != NULL) {
        const size_t n = (size_t)inf->batch * c->d_model;
        float *gathered = (float *)(inf->tp_region + b2_tp_region_bytes(2 * c->n_layers, (uint32_t)n, 0));
        for (l = 0; l < c->n_layers && rc == 0; l++) {
            dev_layer *L = &inf->layers[l];
            rc |= b2_gemv(&L->a_qkv, st);
            rc |= b2_attn(&L->a_attn, st);
            rc |= b2_gemv(&L->a_wo, st);
            rc |= b2_nccl_allreduce_sum_f32(inf->h1, n, inf->nccl_comm, st);
            rc |= b2_gemv(&L->a_gu, st);
            rc |= b2_gemv(&L->a_down, st);
            rc |= b2_nccl_allreduce_sum_f32(inf->x, n, inf->nccl_comm, st);
        }
        if (rc == 0) rc = b2_gemv(&inf->a_out, st);
        if (rc == 0) rc = b2_nccl_allgather(inf->logits, gathered, (size_t)inf->batch * inf->vl * sizeof(float),
                                            inf->nccl_comm, st);
        if (rc == 0) rc = b2_nccl_allgather(inf->argmax_d, inf->nccl_keys, (size_t)inf->batch * sizeof(unsigned long long),
                                            inf->nccl_comm, st);
        if (rc == 0)
            rc = b2_step_end_keys(inf->nccl_keys, inf->tp_world, inf->batch, inf->tokens_d, inf->pos_d, inf->err_d,
                                  inf->use_pdl, st);
        return rc != 0 ? rc : sample_step(inf, st);
    }
    for (l = 0; l < c->n_layers && rc == 0; l++) {
        dev_layer *L = &inf->layers[l];
        rc |= b2_gemv(&L->a_qkv, st);
        rc |= b2_attn(&L->a_attn, st);
        rc |= b2_gemv(&L->a_wo, st);
        rc |= b2_gemv(&L->a_gu, st);
        rc |= b2_gemv(&L->a_down, st);
    }
    if (rc == 0) rc = b2_gemv(&inf->a_out, st);
    if (rc != 0) return rc;
    if (inf->tp_world > 1)
        rc = b2_step_end_tp(&inf->tp_base, inf->batch, inf->tokens_d, inf->pos_d, inf->err_d, inf->use_pdl, st);
    else
        rc = b2_step_end(inf->argmax_d, inf->batch, inf->tokens_d, inf->pos_d, inf->err_d, inf->use_pdl, st);
    return rc != 0 ? rc : sample_step(inf, st);
}

static int launch_step(att1_infer_t *inf)
{
    /* contexts of several GPUs may be driven from one thread */
    if (cudaSetDevice(inf->device) != cudaSuccess) return -8;
    if (inf->use_persistent && inf->plan && inf->top_k <= 1) return b2_decode_step(inf->plan, inf->stream);
    if (inf->use_graph && !inf->graph_failed) {
        if (inf->exec == NULL) {
            cudaGraph_t g = NULL;
            int rc;
            if (cudaStreamBeginCapture(inf->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
                inf->graph_failed = 1;
                cudaGetLastError();
                return enqueue_kernels(inf);
            }
            rc = enqueue_kernels(inf);
            if (cudaStreamEndCapture(inf->stream, &g) != cudaSuccess || rc != 0 ||
                cudaGraphGetNodes(g, NULL, &inf->graph_nodes) != cudaSuccess ||
                cudaGraphInstantiate(&inf->exec, g, 0) != cudaSuccess) {
                if (g) cudaGraphDestroy(g);
                inf->exec = NULL;
                inf->graph_failed = 1;
                cudaGetLastError();
                return enqueue_kernels(inf);
            }
            cudaGraphDestroy(g);
        }
        return cudaGraphLaunch(inf->exec, inf->stream) == cudaSuccess ? 0 : -8;
    }
    return enqueue_kernels(inf);
}

/* After a kernel-reported fault: clear the error word, the tile counters in
 * scratch, and put the device position back to the host position. */
static att1_status_t recover(att1_infer_t *inf, int32_t err)
{
    int32_t pos[ATT1_B200_MAX_BATCH];
    uint32_t b;
    for (b = 0; b < inf->batch; b++) pos[b] = (int32_t)inf->position;
    cudaMemsetAsync(inf->err_d, 0, sizeof(int32_t), inf->stream);
    cudaMemsetAsync(inf->counters, 0, (size_t)inf->counters_len * sizeof(int32_t), inf->stream);
    if (inf->plan) b2_decode_reset(inf->plan, inf->stream);
    cudaMemcpyAsync(inf->pos_d, pos, inf->batch * sizeof(int32_t), cudaMemcpyHostToDevice, inf->stream);
    cudaStreamSynchronize(inf->stream);
    if (err & B2_ERR_TIMEOUT) return ATT1_ERR_TIMEOUT;
    if (err & B2_ERR_TOKEN) return ATT1_ERR_INVALID_ARG;
    return ATT1_ERR_STATE;
}

/* First half of a step: token upload, the step's kernels and the read-back
 * copies, all queued on the context's stream. */
static att1_status_t step_launch(att1_infer_t *inf, const uint32_t *tokens)
{
    const att1_b200_config *c = &inf->cfg;
    uint32_t b;

    if (!inf->tp_ready) return ATT1_ERR_STATE;
    if (inf->position >= c->max_seq) return ATT1_ERR_INVALID_ARG;
    for (b = 0; b < inf->batch; b++) {
        if (tokens[b] >= c->vocab) return ATT1_ERR_INVALID_ARG;
        inf->tokens_h[b] = tokens[b];
    }
    if (inf->trace) inf->trace_t0 = att1_trace_now_us();
    if (inf->position == 0) {
        int32_t zero[ATT1_B200_MAX_BATCH] = {0};
        if (cudaMemcpyAsync(inf->pos_d, zero, inf->batch * sizeof(int32_t), cudaMemcpyHostToDevice, inf->stream) !=
            cudaSuccess)
            return ATT1_ERR_STATE;
    }
    if (inf->mmu != NULL) { /* pages for this position in every session, before the kernels append there */
        att1_status_t st;
        for (b = 0; b < inf->batch; b++)
            if ((st = b2_kv_mmu_reserve(inf->mmu, inf->mmu_slot0 + b, inf->position, 1)) != ATT1_OK) return st;
    }
    if (cudaMemcpyAsync(inf->tokens_d, inf->tokens_h, inf->batch * sizeof(uint32_t), cudaMemcpyHostToDevice,
                        inf->stream) != cudaSuccess)
        return ATT1_ERR_STATE;
    if (launch_step(inf) != 0) return ATT1_ERR_STATE;
    cudaMemcpyAsync(inf->out_h, inf->tokens_d, inf->batch * sizeof(uint32_t), cudaMemcpyDeviceToHost, inf->stream);
    cudaMemcpyAsync(inf->err_h, inf->err_d, sizeof(int32_t), cudaMemcpyDeviceToHost, inf->stream);
    inf->step_pending = 1;
    return ATT1_OK;
}

/* Second half: wait for the step and take its tokens. */
static att1_status_t step_finish(att1_infer_t *inf, uint32_t *out_tokens)
{
    const att1_b200_config *c = &inf->cfg;
    const uint64_t t0 = inf->trace_t0;
    uint32_t b;
    cudaError_t e;
    if (!inf->step_pending) return ATT1_ERR_STATE;
    inf->step_pending = 0;
    e = cudaStreamSynchronize(inf->stream);
    if (e != cudaSuccess) return b2_cuda_status(e);
    inf->logits_valid = 0;
    if (*inf->err_h != 0) return recover(inf, *inf->err_h);
    for (b = 0; b < inf->batch; b++) out_tokens[b] = inf->out_h[b];
    if (inf->trace) {
        const uint64_t us = att1_trace_now_us() - t0;
        const uint64_t reads = (uint64_t)(inf->position + 1) * c->n_heads;
        uint32_t l;
        for (l = 0; l < c->n_layers; l++) att1_trace_record_layer(inf->trace, l, us / c->n_layers, 1, reads, reads);
        att1_trace_record_logits(inf->trace, 0, (uint64_t)c->vocab * sizeof(float));
        att1_trace_record_token(inf->trace, us);
    }
    if (inf->mmu != NULL)
        for (b = 0; b < inf->batch; b++) b2_kv_mmu_advance(inf->mmu, inf->mmu_slot0 + b, 1);
    inf->position++;
    return ATT1_OK;
}

static att1_status_t step(att1_infer_t *inf, const uint32_t *tokens, uint32_t *out_tokens)
{
    att1_status_t st = step_launch(inf, tokens);
    if (st != ATT1_OK) return st;
    return step_finish(inf, out_tokens);
}

static int backend_ok(const att1_infer_t *inf)
{
    /* routing by name as in src/infer.c:143-159: the context's precision must
     * match the backend's */
    const char *n = inf->backend ? b2_backend_name(inf->backend) : NULL;
    if (n == NULL) return 1; /* contexts from att1_b200_* have no backend object */
    if (strcmp(n, "cuda-q4") == 0) return inf->cfg.dtype == 4;
    if (strcmp(n, "cuda-q8") == 0) return inf->cfg.dtype == 8;
    return 0;
}

att1_status_t att1_infer_decode_token(att1_infer_t *infer, uint32_t token_id, uint32_t *out_token)
{
    if (infer == NULL || out_token == NULL) return ATT1_ERR_INVALID_ARG;
    if (infer->batch != 1) return ATT1_ERR_STATE;
    if (token_id >= infer->cfg.vocab || infer->position >= infer->cfg.max_seq) return ATT1_ERR_INVALID_ARG;
    if (!backend_ok(infer)) return ATT1_ERR_STATE;
    return step(infer, &token_id, out_token);
}

att1_status_t att1_b200_infer_step_async(att1_infer_t *infer, const uint32_t *tokens)
{
    if (infer == NULL || tokens == NULL || infer->step_pending) return ATT1_ERR_INVALID_ARG;
    if (!backend_ok(infer)) return ATT1_ERR_STATE;
    return step_launch(infer, tokens);
}

att1_status_t att1_b200_infer_step_wait(att1_infer_t *infer, uint32_t *out_tokens)
{
    if (infer == NULL || out_tokens == NULL) return ATT1_ERR_INVALID_ARG;
    return step_finish(infer, out_tokens);
}

att1_status_t att1_b200_infer_decode_batch(att1_infer_t *infer, const uint32_t *tokens, uint32_t *out_tokens)
{
    if (infer == NULL || tokens == NULL || out_tokens == NULL) return ATT1_ERR_INVALID_ARG;
    if (!backend_ok(infer)) return ATT1_ERR_STATE;
    return step(infer, tokens, out_tokens);
}

/* ---- prompt prefill ------------------------------------------------------------------------------ */

#define PREFILL_CHUNK 512u

/* Buffers for prompt chunks of up to `cap` tokens: every row of a chunk is a
 * position of sequence 0, so the chunk's page-table rows all repeat
 * sequence 0's row. Sizes are the largest over chunk lengths 1..cap (the
 * split choices depend on the length). */
static att1_status_t prefill_alloc(att1_infer_t *inf, uint32_t cap)
{
    const att1_b200_config *c = &inf->cfg;
    const uint32_t pps = inf->pages_per_seq;
    att1_status_t st;
    b2_attn_args at;
    int32_t *pt;
    uint32_t m, i;
    size_t s;
    cudaError_t e;
    if (inf->pf_cap >= cap) return ATT1_OK;
    free_prefill(inf);
    at = inf->layers[0].a_attn;
    inf->pf_xs_bytes = inf->pf_gscratch_bytes = inf->pf_ascratch_bytes = 0;
    for (m = 1; m <= cap; m++) {
        if ((s = dense_xs(inf, m)) > inf->pf_xs_bytes) inf->pf_xs_bytes = s;
        if ((s = dense_gscratch(inf, m)) > inf->pf_gscratch_bytes) inf->pf_gscratch_bytes = s;
        at.batch = m;
        if ((s = b2_attn_scratch_bytes(&at)) > inf->pf_ascratch_bytes) inf->pf_ascratch_bytes = s;
    }
    at.batch = cap;
    inf->pf_counters_len = b2_attn_counters_len(&at);
    if ((st = dalloc(inf, (void **)&inf->pf_x, (size_t)cap * c->d_model * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->pf_h, (size_t)cap * c->d_model * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->pf_q, (size_t)cap * inf->q_rows * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->pf_ctx, (size_t)cap * inf->q_rows * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->pf_hs, (size_t)cap * inf->ffl * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->pf_yqkv, (size_t)cap * (inf->q_rows + 2 * inf->kv_rows) * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->pf_ygu, (size_t)cap * 2 * inf->ffl * sizeof(float))) ||
        (st = dalloc(inf, (void **)&inf->pf_tok, (size_t)cap * sizeof(uint32_t))) ||
        (st = dalloc(inf, (void **)&inf->pf_pos, (size_t)cap * sizeof(int32_t))) ||
        (st = dalloc(inf, (void **)&inf->pf_pt, (size_t)cap * pps * sizeof(int32_t))) ||
        (st = dalloc(inf, (void **)&inf->pf_counters, (size_t)inf->pf_counters_len * sizeof(int32_t))) ||
        (st = dalloc(inf, (void **)&inf->pf_keys, (size_t)cap * sizeof(unsigned long long))) ||
        (st = dalloc(inf, &inf->pf_xs, inf->pf_xs_bytes)) ||
        (st = dalloc(inf, &inf->pf_gscratch, inf->pf_gscratch_bytes)) ||
        (st = dalloc(inf, &inf->pf_ascratch, inf->pf_ascratch_bytes))) {
        free_prefill(inf);
        return st;
    }
    pt = malloc((size_t)cap * pps * sizeof(int32_t));
    if (pt == NULL) {
        free_prefill(inf);
        return ATT1_ERR_OOM;
    }
    /* stream-ordered after pf_pt's zero fill (dalloc) */
    e = cudaMemcpyAsync(pt, inf->page_table, pps * sizeof(int32_t), cudaMemcpyDeviceToHost, inf->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(inf->stream);
    for (i = 1; i < cap; i++) memcpy(pt + (size_t)i * pps, pt, pps * sizeof(int32_t));
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(inf->pf_pt, pt, (size_t)cap * pps * sizeof(int32_t), cudaMemcpyHostToDevice, inf->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(inf->stream);
    free(pt);
    if (e != cudaSuccess) {
        free_prefill(inf);
        return b2_cuda_status(e);
    }
    inf->pf_cap = cap;
    return ATT1_OK;
}

/* Prefill into a KV-MMU session: every row of a chunk is a position of the
 * session, so each layer's block repeats the session's row of that layer
 * (pages for the whole prompt are mapped before this). */
static att1_status_t prefill_mmu_table(att1_infer_t *inf, uint32_t rows, size_t *layer_stride)
{
    const uint32_t L = inf->cfg.n_layers;
    size_t pps, need, i;
    uint32_t l;
    int32_t *pt;
    att1_status_t st;
    cudaError_t e;
    b2_kv_mmu_row(inf->mmu, inf->mmu_slot0, 0, &pps);
    need = (size_t)L * rows * pps;
    if (need > inf->pf_mpt_elems) {
        dfree(inf->pf_mpt);
        inf->pf_mpt = NULL;
        inf->pf_mpt_elems = 0;
        if ((st = dalloc(inf, (void **)&inf->pf_mpt, need * sizeof(int32_t))) != ATT1_OK) return st;
        inf->pf_mpt_elems = need;
    }
    pt = malloc(need * sizeof(int32_t));
    if (pt == NULL) return ATT1_ERR_OOM;
    for (l = 0; l < L; l++) {
        const int32_t *row = b2_kv_mmu_row(inf->mmu, inf->mmu_slot0, l, &pps);
        for (i = 0; i < rows; i++) memcpy(pt + ((size_t)l * rows + i) * pps, row, pps * sizeof(int32_t));
    }
    /* stream-ordered after pf_mpt's zero fill and before the prefill kernels */
    e = cudaMemcpyAsync(inf->pf_mpt, pt, need * sizeof(int32_t), cudaMemcpyHostToDevice, inf->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(inf->stream);
    free(pt);
    *layer_stride = (size_t)rows * pps;
    return b2_cuda_status(e);
}

att1_status_t att1_b200_infer_prefill(att1_infer_t *inf, const uint32_t *tokens, size_t n, uint32_t *out_token)
{
    const att1_b200_config *c;
    cudaStream_t st;
    int32_t *pos_h;
    size_t done = 0, i, mpt_stride = 0;
    uint32_t cap, m = 0;
    att1_status_t s;
    int rc = 0;
    if (inf == NULL || tokens == NULL || out_token == NULL || n == 0) return ATT1_ERR_INVALID_ARG;
    c = &inf->cfg;
    if (inf->batch != 1 || inf->step_pending || !backend_ok(inf)) return ATT1_ERR_STATE;
    if (inf->tp_world > 1) return ATT1_ERR_UNSUPPORTED;
    if (n > c->max_seq || inf->position + n > c->max_seq) return ATT1_ERR_INVALID_ARG;
    for (i = 0; i < n; i++)
        if (tokens[i] >= c->vocab) return ATT1_ERR_INVALID_ARG;
    if (cudaSetDevice(inf->device) != cudaSuccess) return ATT1_ERR_STATE;
    cap = n < PREFILL_CHUNK ? (uint32_t)n : PREFILL_CHUNK;
    if ((s = prefill_alloc(inf, cap)) != ATT1_OK) return s;
    if (inf->mmu != NULL && ((s = b2_kv_mmu_reserve(inf->mmu, inf->mmu_slot0, inf->position, n)) != ATT1_OK ||
                             (s = prefill_mmu_table(inf, cap, &mpt_stride)) != ATT1_OK))
        return s;
    pos_h = malloc((size_t)cap * sizeof(int32_t));
    if (pos_h == NULL) return ATT1_ERR_OOM;
    st = inf->stream;
    while (done < n && rc == 0) {
        dense_bufs b;
        uint32_t l;
        m = (uint32_t)((n - done) < cap ? (n - done) : cap);
        for (i = 0; i < m; i++) pos_h[i] = (int32_t)(inf->position + done + i);
        /* pageable sources: each copy has left the buffer when it returns */
        if (cudaMemcpyAsync(inf->pf_tok, tokens + done, m * sizeof(uint32_t), cudaMemcpyHostToDevice, st) !=
                cudaSuccess ||
            cudaMemcpyAsync(inf->pf_pos, pos_h, m * sizeof(int32_t), cudaMemcpyHostToDevice, st) != cudaSuccess) {
            rc = -8;
            break;
        }
        memset(&b, 0, sizeof(b));
        b.m = m;
        b.x = inf->pf_x;
        b.h = inf->pf_h;
        b.q = inf->pf_q;
        b.ctx = inf->pf_ctx;
        b.hs = inf->pf_hs;
        b.y_qkv = inf->pf_yqkv;
        b.y_gu = inf->pf_ygu;
        b.positions = inf->pf_pos;
        b.page_table = inf->mmu != NULL ? inf->pf_mpt : inf->pf_pt;
        b.pt_layer_stride = mpt_stride;
        b.xs = inf->pf_xs;
        b.xs_bytes = inf->pf_xs_bytes;
        b.gscratch = inf->pf_gscratch;
        b.gscratch_bytes = inf->pf_gscratch_bytes;
        b.ascratch = inf->pf_ascratch;
        b.ascratch_bytes = inf->pf_ascratch_bytes;
        b.acounters = inf->pf_counters;
        b.acounters_len = inf->pf_counters_len;
        rc = b2_step_begin(inf->embed, c->vocab, c->d_model, inf->pf_tok, m, inf->pf_x, inf->pf_keys, inf->err_d, 0, st);
        for (l = 0; l < c->n_layers && rc == 0; l++) rc = dense_layer(inf, l, &b, st);
        done += m;
    }
    free(pos_h);
    if (rc == 0) {
        /* the last prompt token's row finishes like a decode step: final norm,
         * lm_head, greedy sampler, position = prompt end */
        const int32_t last = (int32_t)(inf->position + n - 1);
        if (cudaMemcpyAsync(inf->x, inf->pf_x + (size_t)(m - 1) * c->d_model, c->d_model * sizeof(float),
                            cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(inf->pos_d, &last, sizeof(int32_t), cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemsetAsync(inf->argmax_d, 0, sizeof(unsigned long long), st) != cudaSuccess)
            rc = -8;
    }
    if (rc == 0) {
        if (inf->use_dense) {
            dense_bufs b;
            decode_bufs(inf, &b);
            rc = dense_head(inf, &b, st);
        } else {
            rc = b2_gemv(&inf->a_out, st);
        }
    }
    if (rc == 0) rc = b2_step_end(inf->argmax_d, 1, inf->tokens_d, inf->pos_d, inf->err_d, inf->use_pdl, st);
    if (rc == 0) rc = sample_step(inf, st);
    if (rc != 0) {
        cudaStreamSynchronize(st);
        cudaGetLastError();
        return ATT1_ERR_STATE;
    }
    cudaMemcpyAsync(inf->out_h, inf->tokens_d, sizeof(uint32_t), cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(inf->err_h, inf->err_d, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) return ATT1_ERR_STATE;
    inf->logits_valid = 0;
    if (*inf->err_h != 0) return recover(inf, *inf->err_h);
    if (inf->mmu != NULL) b2_kv_mmu_advance(inf->mmu, inf->mmu_slot0, n);
    inf->position += n;
    *out_token = inf->out_h[0];
    return ATT1_OK;
}

att1_status_t att1_infer_generate(att1_infer_t *infer, const unsigned char *prompt, size_t prompt_bytes,
                                  size_t generated_token_count, uint32_t *out_tokens, size_t out_token_capacity,
                                  size_t *out_token_count)
{
    uint32_t token = 0;
    size_t i;
    att1_status_t st;
    /* same contract as src/infer.c:882-928 */
    if (infer == NULL || prompt == NULL || out_tokens == NULL || out_token_count == NULL) return ATT1_ERR_INVALID_ARG;
    if (prompt_bytes == 0 || out_token_capacity < generated_token_count) return ATT1_ERR_INVALID_ARG;
    if (infer->batch == 1 && infer->tp_world == 1) {
        /* the prompt in one pass over the weights per chunk (same results as
         * the token-by-token loop of the reference) */
        uint32_t *ids = malloc(prompt_bytes * sizeof(uint32_t));
        if (ids == NULL) return ATT1_ERR_OOM;
        for (i = 0; i < prompt_bytes; i++) ids[i] = prompt[i];
        st = att1_b200_infer_prefill(infer, ids, prompt_bytes, &token);
        free(ids);
        if (st != ATT1_OK) return st;
    } else {
        for (i = 0; i < prompt_bytes; i++) {
            uint32_t next = 0;
            st = att1_infer_decode_token(infer, (uint32_t)prompt[i], &next);
            if (st != ATT1_OK) return st;
            token = next;
        }
    }
    for (i = 0; i < generated_token_count; i++) {
        uint32_t next = 0;
        out_tokens[i] = token;
        if (i + 1 < generated_token_count) {
            st = att1_infer_decode_token(infer, token, &next);
            if (st != ATT1_OK) return st;
            token = next;
        }
    }
    *out_token_count = generated_token_count;
    return ATT1_OK;
}

static const float *logits_host(const att1_infer_t *cinfer, size_t *out_count, size_t n)
{
    att1_infer_t *infer = (att1_infer_t *)cinfer; /* lazy copy-back is internal state */
    if (infer == NULL) {
        if (out_count) *out_count = 0;
        return NULL;
    }
    if (!infer->logits_valid) {
        cudaError_t e = cudaSetDevice(infer->device);
        if (infer->tp_world > 1) {
            /* every rank's vocabulary rows, all-gathered into this rank's region */
            const size_t V = infer->cfg.vocab, vl = infer->vl;
            uint32_t s;
            for (s = 0; s < infer->tp_world && e == cudaSuccess; s++) {
                const float *src = (const float *)(infer->tp_region + b2_tp_region_bytes(2 * infer->cfg.n_layers,
                                                                                          infer->batch * infer->cfg.d_model,
                                                                                          0)) +
                                   (size_t)s * infer->batch * vl;
                e = cudaMemcpy2DAsync(infer->logits_h + (size_t)s * vl, V * sizeof(float), src, vl * sizeof(float),
                                      vl * sizeof(float), infer->batch, cudaMemcpyDeviceToHost, infer->stream);
            }
        } else if (e == cudaSuccess) {
            e = cudaMemcpyAsync(infer->logits_h, infer->logits, (size_t)infer->batch * infer->cfg.vocab * sizeof(float),
                                cudaMemcpyDeviceToHost, infer->stream);
        }
        if (e == cudaSuccess) e = cudaStreamSynchronize(infer->stream);
        if (e != cudaSuccess) {
            if (out_count) *out_count = 0;
            return NULL;
        }
        infer->logits_valid = 1;
    }
    if (out_count) *out_count = n;
    return infer->logits_h;
}

const float *att1_infer_logits(const att1_infer_t *infer, size_t *out_count)
{
    return logits_host(infer, out_count, infer ? infer->cfg.vocab : 0);
}

const float *att1_b200_infer_logits_batch(const att1_infer_t *infer, size_t *out_count)
{
    return logits_host(infer, out_count, infer ? (size_t)infer->batch * infer->cfg.vocab : 0);
}

att1_status_t att1_infer_position(const att1_infer_t *infer, size_t *out_position)
{
    if (infer == NULL || out_position == NULL) return ATT1_ERR_INVALID_ARG;
    *out_position = infer->position;
    return ATT1_OK;
}

att1_status_t att1_infer_layer_kv_length(const att1_infer_t *infer, uint32_t layer_id, size_t *out_length)
{
    if (infer == NULL || out_length == NULL || layer_id >= infer->cfg.n_layers) return ATT1_ERR_INVALID_ARG;
    *out_length = infer->position;
    return ATT1_OK;
}

att1_status_t att1_infer_set_trace(att1_infer_t *infer, att1_trace_t *trace)
{
    if (infer == NULL) return ATT1_ERR_INVALID_ARG;
    infer->trace = trace;
    return ATT1_OK;
}

att1_status_t att1_infer_set_backend(att1_infer_t *infer, att1_backend *backend)
{
    const char *n;
    uint32_t want;
    att1_status_t st;
    if (infer == NULL || backend == NULL || backend->ops == NULL) return ATT1_ERR_INVALID_ARG;
    n = b2_backend_name(backend);
    if (n == NULL || !b2_backend_is_cuda(backend)) return ATT1_ERR_UNSUPPORTED;
    if (strcmp(n, "cuda-q4") == 0) want = 4;
    else if (strcmp(n, "cuda-q8") == 0) want = 8;
    else return ATT1_ERR_UNSUPPORTED; /* the f32 "cuda" backend has no device decode path */
    if (want != infer->cfg.dtype) {
        /* switch precision: re-prepare weights from the model (src/infer.c:982-1012) */
        if (infer->model == NULL) return ATT1_ERR_UNSUPPORTED;
        /* the reference keeps its backend when the file cannot serve the new
         * precision (src/infer.c:982-1012): so does this context */
        if ((st = load_model_weights(infer, infer->model, want, 1)) != ATT1_OK) return st;
        cudaStreamSynchronize(infer->stream);
        if (infer->exec) {
            cudaGraphExecDestroy(infer->exec);
            infer->exec = NULL;
        }
        free_weights(infer);
        infer->cfg.dtype = want;
        if ((st = alloc_weights(infer, want)) || (st = load_model_weights(infer, infer->model, want, 0))) return st;
        if ((st = build_args(infer)) != ATT1_OK) return st;
    }
    if (infer->backend) att1_backend_destroy(infer->backend);
    infer->backend = backend;
    return ATT1_OK;
}

att1_status_t att1_b200_infer_set_options(att1_infer_t *infer, int use_graph, int use_pdl)
{
    if (infer == NULL) return ATT1_ERR_INVALID_ARG;
    cudaStreamSynchronize(infer->stream);
    if (infer->exec) {
        cudaGraphExecDestroy(infer->exec);
        infer->exec = NULL;
    }
    infer->graph_failed = 0;
    infer->use_graph = use_graph ? 1 : 0;
    set_pdl(infer, use_pdl ? 1 : 0);
    return ATT1_OK;
}

att1_status_t att1_b200_infer_set_sampler(att1_infer_t *infer, const att1_sampler_config *config, uint64_t seed)
{
    const int sample = config != NULL && config->top_k > 1;
    if (infer == NULL) return ATT1_ERR_INVALID_ARG;
    if (sample && (config->top_k > B2_MAX_TOP_K || config->top_k > infer->cfg.vocab ||
                   !(config->temperature > 0.0f) || !(config->temperature <= FLT_MAX)))
        return ATT1_ERR_INVALID_ARG;
    if (infer->step_pending) return ATT1_ERR_STATE;
    if (cudaSetDevice(infer->device) != cudaSuccess) return ATT1_ERR_STATE;
    cudaStreamSynchronize(infer->stream);
    if (infer->exec) { /* the captured step holds the old choice */
        cudaGraphExecDestroy(infer->exec);
        infer->exec = NULL;
    }
    infer->top_k = sample ? config->top_k : 0;
    infer->temperature = sample ? config->temperature : 0.0f;
    infer->sample_seed = seed;
    return ATT1_OK;
}

att1_status_t att1_b200_infer_set_persistent(att1_infer_t *infer, int on)
{
    if (infer == NULL) return ATT1_ERR_INVALID_ARG;
    cudaStreamSynchronize(infer->stream);
    infer->use_persistent = on ? 1 : 0;
    return (on && infer->plan == NULL) ? ATT1_ERR_UNSUPPORTED : ATT1_OK;
}

att1_status_t att1_b200_set_device(int device)
{
    return cudaSetDevice(device) == cudaSuccess ? ATT1_OK : ATT1_ERR_INVALID_ARG;
}

/* Batch item b keeps its KV in KV-MMU session session_ids[b] (pages mapped on
 * demand as positions advance; the MMU's lengths and append counters follow
 * the steps). Sessions must sit in consecutive slots in batch order (create
 * them one after another), be empty, and match the context's layers, KV
 * heads and head_dim, with max_positions >= max_seq. NULL mmu returns to the
 * context's own pools. Only at position 0, one GPU. */
att1_status_t att1_b200_infer_use_kv_mmu(att1_infer_t *infer, att1_kv_mmu *mmu, const uint64_t *session_ids)
{
    const att1_kv_mmu_config *mc;
    size_t slot0 = 0, slot, l;
    uint32_t b;
    att1_status_t st;
    if (infer == NULL || (mmu != NULL && session_ids == NULL)) return ATT1_ERR_INVALID_ARG;
    if (infer->tp_world > 1) return ATT1_ERR_UNSUPPORTED;
    if (infer->position != 0 || infer->step_pending) return ATT1_ERR_STATE;
    if (mmu != NULL) {
        mc = b2_kv_mmu_config(mmu);
        if (mc->num_layers != infer->cfg.n_layers || mc->num_heads != infer->hkv || mc->head_dim != infer->head_dim ||
            mc->max_positions < infer->cfg.max_seq)
            return ATT1_ERR_SHAPE;
        for (b = 0; b < infer->batch; b++) {
            if (!b2_kv_mmu_session_slot(mmu, session_ids[b], &slot)) return ATT1_ERR_NOT_FOUND;
            if (b == 0) slot0 = slot;
            if (slot != slot0 + b) return ATT1_ERR_UNSUPPORTED;
            for (l = 0; l < mc->num_layers; l++)
                if (b2_kv_mmu_length(mmu, slot, l) != 0) return ATT1_ERR_STATE;
        }
    }
    if (cudaSetDevice(infer->device) != cudaSuccess) return ATT1_ERR_STATE;
    cudaStreamSynchronize(infer->stream);
    infer->mmu = mmu;
    infer->mmu_sid0 = mmu != NULL ? session_ids[0] : 0;
    infer->mmu_slot0 = slot0;
    /* the kernels' arguments name the KV pools: rebuild them and the step graph */
    if (infer->exec) {
        cudaGraphExecDestroy(infer->exec);
        infer->exec = NULL;
    }
    infer->graph_failed = 0;
    if ((st = build_args(infer)) != ATT1_OK) return st;
    return b2_cuda_status(cudaStreamSynchronize(infer->stream));
}

att1_status_t att1_b200_infer_run_steps(att1_infer_t *infer, uint32_t steps)
{
    uint32_t i;
    if (infer == NULL) return ATT1_ERR_INVALID_ARG;
    if (!infer->tp_ready) return ATT1_ERR_STATE;
    if (cudaSetDevice(infer->device) != cudaSuccess) return ATT1_ERR_STATE;
    if (infer->position + steps > infer->cfg.max_seq) return ATT1_ERR_INVALID_ARG;
    if (infer->position == 0) {
        int32_t zero[ATT1_B200_MAX_BATCH] = {0};
        if (cudaMemcpyAsync(infer->pos_d, zero, infer->batch * sizeof(int32_t), cudaMemcpyHostToDevice,
                            infer->stream) != cudaSuccess)
            return ATT1_ERR_STATE;
    }
    if (infer->mmu != NULL) {
        uint32_t b;
        att1_status_t st;
        for (b = 0; b < infer->batch; b++)
            if ((st = b2_kv_mmu_reserve(infer->mmu, infer->mmu_slot0 + b, infer->position, steps)) != ATT1_OK)
                return st;
    }
    for (i = 0; i < steps; i++) {
        if (launch_step(infer) != 0) return ATT1_ERR_STATE;
    }
    if (infer->mmu != NULL) {
        uint32_t b;
        for (b = 0; b < infer->batch; b++) b2_kv_mmu_advance(infer->mmu, infer->mmu_slot0 + b, steps);
    }
    infer->position += steps;
    infer->logits_valid = 0;
    return ATT1_OK;
}

att1_status_t att1_b200_infer_sync(att1_infer_t *infer)
{
    cudaError_t e;
    if (infer == NULL) return ATT1_ERR_INVALID_ARG;
    cudaMemcpyAsync(infer->err_h, infer->err_d, sizeof(int32_t), cudaMemcpyDeviceToHost, infer->stream);
    e = cudaStreamSynchronize(infer->stream);
    if (e != cudaSuccess) return b2_cuda_status(e);
    if (*infer->err_h != 0) {
        infer->position = 0; /* device positions are unknown after a fault */
        return recover(infer, *infer->err_h);
    }
    return ATT1_OK;
}

/* ---- KV restore and seek --------------------------------------------------------------------------------- */

/* Host [count][hkv][hd] rows -> the item's pages of one layer: one strided copy
 * per (page, KV head), since a page keeps each head's tokens contiguous. */
att1_status_t att1_b200_infer_import_kv(att1_infer_t *infer, uint32_t item, uint32_t layer, size_t count,
                                        const float *keys, const float *values)
{
    size_t p0;
    uint32_t h;
    if (infer != NULL && infer->mmu != NULL) return ATT1_ERR_UNSUPPORTED; /* write through the KV-MMU */
    if (infer == NULL || keys == NULL || values == NULL || item >= infer->batch || layer >= infer->cfg.n_layers ||
        count > infer->cfg.max_seq)
        return ATT1_ERR_INVALID_ARG;
    if (infer->step_pending) return ATT1_ERR_STATE;
    {
        const size_t hd = infer->head_dim, row = (size_t)infer->hkv * hd, pt = infer->page_tokens;
        for (p0 = 0; p0 < count; p0 += pt) {
            const size_t n = count - p0 < pt ? count - p0 : pt;
            const size_t page = (size_t)item * infer->pages_per_seq + p0 / pt;
            for (h = 0; h < infer->hkv; h++) {
                const size_t off = (size_t)layer * infer->layer_pool_elems + ((page * infer->hkv + h) * pt) * hd;
                const size_t src = p0 * row + (size_t)h * hd;
                if (cudaMemcpy2DAsync(infer->k_pool + off, hd * sizeof(float), keys + src, row * sizeof(float),
                                      hd * sizeof(float), n, cudaMemcpyHostToDevice, infer->stream) != cudaSuccess ||
                    cudaMemcpy2DAsync(infer->v_pool + off, hd * sizeof(float), values + src, row * sizeof(float),
                                      hd * sizeof(float), n, cudaMemcpyHostToDevice, infer->stream) != cudaSuccess)
                    return ATT1_ERR_STATE;
            }
        }
    }
    /* the host arrays are the caller's: finish reading them before returning */
    return cudaStreamSynchronize(infer->stream) == cudaSuccess ? ATT1_OK : ATT1_ERR_STATE;
}

att1_status_t att1_b200_infer_seek(att1_infer_t *infer, size_t position)
{
    int32_t pos[ATT1_B200_MAX_BATCH];
    uint32_t b;
    if (infer == NULL || position >= infer->cfg.max_seq) return ATT1_ERR_INVALID_ARG;
    if (infer->mmu != NULL) return ATT1_ERR_UNSUPPORTED;
    if (infer->step_pending) return ATT1_ERR_STATE;
    for (b = 0; b < infer->batch; b++) pos[b] = (int32_t)position;
    if (cudaMemcpyAsync(infer->pos_d, pos, infer->batch * sizeof(int32_t), cudaMemcpyHostToDevice, infer->stream) !=
            cudaSuccess ||
        cudaStreamSynchronize(infer->stream) != cudaSuccess)
        return ATT1_ERR_STATE;
    infer->position = position;
    infer->logits_valid = 0;
    return ATT1_OK;
}

size_t att1_b200_infer_step_launches(const att1_infer_t *infer)
{
    return infer != NULL && infer->exec != NULL ? infer->graph_nodes : 0;
}

/* ---- read-back for parity tests ---------------------------------------------------------------------------- */

static att1_status_t locate(const att1_infer_t *inf, uint32_t layer, uint32_t kind, const b2_dev_mat **m,
                            uint32_t *tile_off, uint32_t *rows, uint32_t *cols, int *map, int *which)
{
    const att1_b200_config *c = &inf->cfg;
    *tile_off = 0;
    *map = B2_ROWS_PLAIN;
    *which = 0;
    if (kind == ATT1_B200_OUTPUT) {
        *m = &inf->output;
        *rows = c->vocab;
        *cols = c->d_model;
        return ATT1_OK;
    }
    if (layer >= c->n_layers) return ATT1_ERR_INVALID_ARG;
    switch (kind) {
    case ATT1_B200_WQ: *m = &inf->layers[layer].qkv; *rows = inf->q_rows; *cols = c->d_model; break;
    case ATT1_B200_WK:
        *m = &inf->layers[layer].qkv; *tile_off = inf->q_rows / 16; *rows = inf->kv_rows; *cols = c->d_model; break;
    case ATT1_B200_WV:
        *m = &inf->layers[layer].qkv; *tile_off = (inf->q_rows + inf->kv_rows) / 16; *rows = inf->kv_rows;
        *cols = c->d_model; break;
    case ATT1_B200_WO: *m = &inf->layers[layer].wo; *rows = c->d_model; *cols = inf->q_rows; break;
    case ATT1_B200_GATE:
    case ATT1_B200_UP:
        *m = &inf->layers[layer].gu; *rows = c->d_ff; *cols = c->d_model; *map = B2_ROWS_GATEUP;
        *which = kind == ATT1_B200_UP; break;
    case ATT1_B200_DOWN: *m = &inf->layers[layer].down; *rows = c->d_model; *cols = c->d_ff; break;
    default: return ATT1_ERR_INVALID_ARG;
    }
    return ATT1_OK;
}

att1_status_t att1_b200_infer_export_q4(const att1_infer_t *infer, uint32_t layer, uint32_t kind, uint8_t *packed,
                                        float *scales)
{
    const b2_dev_mat *m;
    uint32_t toff, rows, cols;
    int map, which, rc;
    void *dp = NULL, *ds = NULL;
    att1_status_t st;
    if (infer == NULL || packed == NULL || scales == NULL || infer->cfg.dtype != 4) return ATT1_ERR_INVALID_ARG;
    if ((st = locate(infer, layer, kind, &m, &toff, &rows, &cols, &map, &which)) != ATT1_OK) return st;
    if (cudaMalloc(&dp, (size_t)rows * cols / 2) != cudaSuccess ||
        cudaMalloc(&ds, (size_t)rows * (cols / 32) * sizeof(float)) != cudaSuccess) {
        st = ATT1_ERR_OOM;
        goto out;
    }
    rc = b2_q4_unpack(dp, ds, m->data, toff, rows, cols, map, which, infer->stream);
    if (rc != 0) {
        st = ATT1_ERR_STATE;
        goto out;
    }
    if (cudaStreamSynchronize(infer->stream) != cudaSuccess ||
        cudaMemcpy(packed, dp, (size_t)rows * cols / 2, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(scales, ds, (size_t)rows * (cols / 32) * sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess)
        st = ATT1_ERR_STATE;
out:
    if (dp) cudaFree(dp);
    if (ds) cudaFree(ds);
    return st;
}

att1_status_t att1_b200_infer_export_q8(const att1_infer_t *infer, uint32_t layer, uint32_t kind, int8_t *values,
                                        float *scales)
{
    const b2_dev_mat *m;
    uint32_t toff, rows, cols;
    int map, which, rc;
    void *dv = NULL, *ds = NULL;
    att1_status_t st;
    if (infer == NULL || values == NULL || scales == NULL || infer->cfg.dtype != 8) return ATT1_ERR_INVALID_ARG;
    if ((st = locate(infer, layer, kind, &m, &toff, &rows, &cols, &map, &which)) != ATT1_OK) return st;
    if (cudaMalloc(&dv, (size_t)rows * cols) != cudaSuccess || cudaMalloc(&ds, (size_t)rows * sizeof(float)) != cudaSuccess) {
        st = ATT1_ERR_OOM;
        goto out;
    }
    rc = b2_q8_unpack(dv, ds, m->data, m->row_scale, toff, rows, cols, map, which, infer->stream);
    if (rc != 0) {
        st = ATT1_ERR_STATE;
        goto out;
    }
    if (cudaStreamSynchronize(infer->stream) != cudaSuccess ||
        cudaMemcpy(values, dv, (size_t)rows * cols, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(scales, ds, (size_t)rows * sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess)
        st = ATT1_ERR_STATE;
out:
    if (dv) cudaFree(dv);
    if (ds) cudaFree(ds);
    return st;
}

att1_status_t att1_b200_infer_export_kv(const att1_infer_t *infer, uint32_t item, uint32_t layer, size_t count,
                                        float *keys, float *values)
{
    const size_t row = (size_t)infer->hkv * infer->head_dim;
    size_t p;
    if (infer != NULL && infer->mmu != NULL) return ATT1_ERR_UNSUPPORTED; /* read through att1_kv_mmu_copy_range */
    if (infer == NULL || keys == NULL || values == NULL || item >= infer->batch || layer >= infer->cfg.n_layers ||
        count > infer->cfg.max_seq)
        return ATT1_ERR_INVALID_ARG;
    if (cudaStreamSynchronize(infer->stream) != cudaSuccess) return ATT1_ERR_STATE;
    for (p = 0; p < count; p++) {
        /* identity page table: sequence item's pages are contiguous */
        /* page = [head][token][dim]: one head_dim run per head, page_tokens rows apart */
        const size_t page = (size_t)item * infer->pages_per_seq + p / infer->page_tokens;
        const size_t off = (size_t)layer * infer->layer_pool_elems +
                           (page * infer->hkv * infer->page_tokens + p % infer->page_tokens) * infer->head_dim;
        const size_t hd = infer->head_dim, pitch = (size_t)infer->page_tokens * hd * sizeof(float);
        if (cudaMemcpy2D(keys + p * row, hd * sizeof(float), infer->k_pool + off, pitch, hd * sizeof(float), infer->hkv,
                         cudaMemcpyDeviceToHost) != cudaSuccess ||
            cudaMemcpy2D(values + p * row, hd * sizeof(float), infer->v_pool + off, pitch, hd * sizeof(float),
                         infer->hkv, cudaMemcpyDeviceToHost) != cudaSuccess)
            return ATT1_ERR_STATE;
    }
    return ATT1_OK;
}
