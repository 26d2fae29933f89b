/*
 * att1_cluster.c - ATT-1 cluster API (include/att1_cluster_infer.h).
 *
 * A "tile" of the reference (src/cluster_infer.c:580-1318) is one GPU here.
 * tile_count = 1 runs the single-device path. tile_count > 1 runs the model
 * tensor parallel over GPUs 0..tile_count-1 of this process: rank r holds
 * its shard of every layer (att1_b200_infer_create_model_tp), the ranks are
 * connected by peer access, and every token is one step queued on all ranks
 * at once (their kernels exchange partial sums and logits through each
 * other's memory) and then awaited on each. Logits and tokens are the same on
 * every rank; the cluster returns rank 0's. The per-tile counters keep the
 * reference's meaning: layers run, activations received and sent (here the
 * all-reduce inputs and contributions: two per layer), logits sent.
 */
#define _POSIX_C_SOURCE 200809L
#include "att1_cluster_infer.h"
#include "att1_b200.h"
#include "att1_infer.h"
#include "b2_host.h"

#include <stdlib.h>
#include <string.h>

#define CLUSTER_MAX_TILES 8

struct att1_cluster_infer {
    att1_infer_t *rank[CLUSTER_MAX_TILES]; /* rank r on device r; rank[0] alone for one tile */
    size_t tiles;
    uint32_t n_layers;
    att1_cluster_tile_counters counters[CLUSTER_MAX_TILES];
    att1_backend *backend;                 /* tile_count > 1: the routing check (ownership) */
    int q4;
};

static void cluster_free(att1_cluster_infer_t *ci)
{
    size_t r;
    if (ci == NULL) return;
    if (ci->tiles > 1) {
        for (r = 0; r < ci->tiles; r++)
            if (ci->rank[r]) att1_b200_infer_tp_disconnect(ci->rank[r]);
    }
    for (r = 0; r < ci->tiles; r++) {
        if (ci->rank[r] == NULL) continue;
        if (ci->tiles > 1) att1_b200_set_device((int)r);
        att1_infer_destroy(ci->rank[r]);
    }
    if (ci->backend) att1_backend_destroy(ci->backend);
    free(ci);
}

static att1_status_t cluster_create(const att1_model *model, const att1_cluster_infer_config *config,
                                    att1_cluster_infer_t **out, int q4)
{
    att1_cluster_infer_t *ci;
    att1_status_t st = ATT1_OK;
    size_t r;
    int devices = 0, prev = 0;
    if (out == NULL) return ATT1_ERR_INVALID_ARG;
    *out = NULL;
    if (model == NULL || config == NULL || config->tile_count == 0) return ATT1_ERR_INVALID_ARG;
    /* src/cluster_infer.c:753-756: metadata plans are not supported for q4 */
    if (config->shard_plan_mode != ATT1_SHARD_PLAN_RUNTIME) return ATT1_ERR_UNSUPPORTED;
    if (config->tile_count > CLUSTER_MAX_TILES) return ATT1_ERR_UNSUPPORTED;
    ci = calloc(1, sizeof(*ci));
    if (ci == NULL) return ATT1_ERR_OOM;
    ci->tiles = config->tile_count;
    ci->n_layers = model->config.n_layers;
    ci->q4 = q4;
    if (ci->tiles == 1) {
        st = q4 ? att1_infer_create_q4(model, &ci->rank[0]) : att1_infer_create(model, &ci->rank[0]);
    } else {
        if (cudaGetDeviceCount(&devices) != cudaSuccess || (size_t)devices < ci->tiles) {
            cudaGetLastError();
            free(ci);
            return ATT1_ERR_UNSUPPORTED;
        }
        cudaGetDevice(&prev);
        /* src/infer.c:721-722 and :823: eps 1e-6, theta 10000 for file models */
        for (r = 0; r < ci->tiles && st == ATT1_OK; r++) {
            att1_b200_set_device((int)r);
            st = att1_b200_infer_create_model_tp(model, q4 ? 4u : 8u, 0.000001f, 0.000001f, 10000.0f, (uint32_t)r,
                                                 (uint32_t)ci->tiles, &ci->rank[r]);
        }
        if (st == ATT1_OK) st = att1_b200_infer_tp_connect_local(ci->rank, (uint32_t)ci->tiles);
        if (st == ATT1_OK)
            st = q4 ? att1_backend_cuda_q4_create(&ci->backend) : att1_backend_cuda_q8_create(&ci->backend);
        cudaSetDevice(prev);
    }
    if (st != ATT1_OK) {
        cluster_free(ci);
        return st;
    }
    for (r = 0; r < ci->tiles; r++) {
        ci->counters[r].layer_start = 0;
        ci->counters[r].layer_end = ci->n_layers;
    }
    *out = ci;
    return ATT1_OK;
}

att1_status_t att1_cluster_infer_create(const att1_model *model, const att1_cluster_infer_config *config,
                                        att1_cluster_infer_t **out)
{
    return cluster_create(model, config, out, 0);
}

att1_status_t att1_cluster_infer_create_q4(const att1_model *model, const att1_cluster_infer_config *config,
                                           att1_cluster_infer_t **out)
{
    return cluster_create(model, config, out, 1);
}

void att1_cluster_infer_destroy(att1_cluster_infer_t *ci)
{
    cluster_free(ci);
}

/* Routing by backend name as src/infer.c:143-159: the cluster's precision
 * must match the backend a caller installed. */
static int backend_matches(const att1_cluster_infer_t *ci)
{
    const char *n;
    if (ci->backend == NULL) return 1;
    n = b2_backend_name(ci->backend);
    if (n == NULL) return 0;
    return strcmp(n, ci->q4 ? "cuda-q4" : "cuda-q8") == 0;
}

att1_status_t att1_cluster_infer_decode_token(att1_cluster_infer_t *ci, uint32_t token_id, uint32_t *out_token)
{
    att1_status_t st = ATT1_OK, st2;
    size_t r, started = 0;
    uint32_t tok[CLUSTER_MAX_TILES];
    if (ci == NULL || out_token == NULL) return ATT1_ERR_INVALID_ARG;
    if (ci->tiles == 1) {
        st = att1_infer_decode_token(ci->rank[0], token_id, out_token);
    } else {
        if (!backend_matches(ci)) return ATT1_ERR_STATE;
        /* every rank takes the step, or none does */
        for (r = 0; r < ci->tiles && st == ATT1_OK; r++) {
            st = att1_b200_infer_step_async(ci->rank[r], &token_id);
            if (st == ATT1_OK) started++;
        }
        for (r = 0; r < started; r++) {
            st2 = att1_b200_infer_step_wait(ci->rank[r], &tok[r]);
            if (st == ATT1_OK) st = st2;
        }
        if (st == ATT1_OK) {
            for (r = 1; r < ci->tiles; r++)
                if (tok[r] != tok[0]) return ATT1_ERR_STATE;
            *out_token = tok[0];
        }
    }
    if (st == ATT1_OK) {
        for (r = 0; r < ci->tiles; r++) {
            att1_cluster_tile_counters *k = &ci->counters[r];
            k->layers_run += ci->n_layers;
            if (ci->tiles > 1) {
                k->activations_received += 2ull * ci->n_layers;
                k->activations_sent += 2ull * ci->n_layers;
            } else {
                k->activations_received++;
            }
        }
        ci->counters[0].logits_sent++;
    }
    return st;
}

att1_status_t att1_cluster_infer_generate(att1_cluster_infer_t *ci, const unsigned char *prompt, size_t prompt_bytes,
                                          size_t generated_token_count, uint32_t *out_tokens,
                                          size_t out_token_capacity, size_t *out_token_count)
{
    uint32_t token = 0;
    size_t i;
    att1_status_t st;
    if (ci == NULL || prompt == NULL || out_tokens == NULL || out_token_count == NULL) return ATT1_ERR_INVALID_ARG;
    if (prompt_bytes == 0 || out_token_capacity < generated_token_count) return ATT1_ERR_INVALID_ARG;
    for (i = 0; i < prompt_bytes; i++) {
        uint32_t next = 0;
        if ((st = att1_cluster_infer_decode_token(ci, prompt[i], &next)) != ATT1_OK) return st;
        token = next;
    }
    for (i = 0; i < generated_token_count; i++) {
        uint32_t next = 0;
        out_tokens[i] = token;
        if (i + 1 < generated_token_count) {
            if ((st = att1_cluster_infer_decode_token(ci, token, &next)) != ATT1_OK) return st;
            token = next;
        }
    }
    *out_token_count = generated_token_count;
    return ATT1_OK;
}

const float *att1_cluster_infer_logits(const att1_cluster_infer_t *ci, size_t *out_count)
{
    if (ci == NULL) {
        if (out_count) *out_count = 0;
        return NULL;
    }
    return att1_infer_logits(ci->rank[0], out_count);
}

att1_status_t att1_cluster_infer_position(const att1_cluster_infer_t *ci, size_t *out_position)
{
    if (ci == NULL) return ATT1_ERR_INVALID_ARG;
    return att1_infer_position(ci->rank[0], out_position);
}

att1_status_t att1_cluster_infer_get_tile_counters(const att1_cluster_infer_t *ci, uint32_t tile_id,
                                                   att1_cluster_tile_counters *out)
{
    if (ci == NULL || out == NULL || tile_id >= ci->tiles) return ATT1_ERR_INVALID_ARG;
    *out = ci->counters[tile_id];
    return ATT1_OK;
}

att1_status_t att1_cluster_infer_get_tile_shard(const att1_cluster_infer_t *ci, uint32_t tile_id,
                                                att1_layer_shard *out)
{
    if (ci == NULL || out == NULL || tile_id >= ci->tiles) return ATT1_ERR_INVALID_ARG;
    out->tile_id = tile_id;
    out->layer_start = 0;
    out->layer_end = ci->n_layers;
    return ATT1_OK;
}

att1_status_t att1_cluster_infer_set_trace(att1_cluster_infer_t *ci, att1_trace_t *trace)
{
    if (ci == NULL) return ATT1_ERR_INVALID_ARG;
    return att1_infer_set_trace(ci->rank[0], trace);
}

att1_status_t att1_cluster_infer_set_backend(att1_cluster_infer_t *ci, att1_backend *backend)
{
    if (ci == NULL) return ATT1_ERR_INVALID_ARG;
    if (ci->tiles == 1) return att1_infer_set_backend(ci->rank[0], backend);
    /* takes ownership (include/att1_infer.h): the ranks keep no per-op backend */
    if (ci->backend) att1_backend_destroy(ci->backend);
    ci->backend = backend;
    return ATT1_OK;
}
