/*
 * att1_cluster.c - ATT-1 cluster API (include/att1_cluster_infer.h).
 *
 * A "tile" of the reference (src/cluster_infer.c:580-1318) is one GPU here.
 * tile_count = 1 runs the single-device path; the per-tile counters keep the
 * reference's meaning (layers run, activations and logits handed on).
 */
#define _POSIX_C_SOURCE 200809L
#include "att1_cluster_infer.h"
#include "att1_infer.h"
#include "b2_host.h"

#include <stdlib.h>
#include <string.h>

struct att1_cluster_infer {
    att1_infer_t *single;
    size_t tiles;
    uint32_t n_layers;
    att1_cluster_tile_counters counters;
};

static att1_status_t cluster_create(const att1_model *model, const att1_cluster_infer_config *config,
                                    att1_cluster_infer_t **out, int q4)
{
    att1_cluster_infer_t *ci;
    att1_status_t st;
    if (out == NULL) return ATT1_ERR_INVALID_ARG;
    *out = NULL;
    if (model == NULL || config == NULL || config->tile_count == 0) return ATT1_ERR_INVALID_ARG;
    /* src/cluster_infer.c:753-756: metadata plans are not supported for q4 */
    if (config->shard_plan_mode != ATT1_SHARD_PLAN_RUNTIME) return ATT1_ERR_UNSUPPORTED;
    if (config->tile_count != 1) return ATT1_ERR_UNSUPPORTED;
    ci = calloc(1, sizeof(*ci));
    if (ci == NULL) return ATT1_ERR_OOM;
    st = q4 ? att1_infer_create_q4(model, &ci->single) : att1_infer_create(model, &ci->single);
    if (st != ATT1_OK) {
        free(ci);
        return st;
    }
    ci->tiles = config->tile_count;
    ci->n_layers = model->config.n_layers;
    ci->counters.layer_start = 0;
    ci->counters.layer_end = model->config.n_layers;
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
    if (ci == NULL) return;
    att1_infer_destroy(ci->single);
    free(ci);
}

att1_status_t att1_cluster_infer_decode_token(att1_cluster_infer_t *ci, uint32_t token_id, uint32_t *out_token)
{
    att1_status_t st;
    if (ci == NULL) return ATT1_ERR_INVALID_ARG;
    st = att1_infer_decode_token(ci->single, token_id, out_token);
    if (st == ATT1_OK) {
        ci->counters.activations_received++;
        ci->counters.layers_run += ci->n_layers;
        ci->counters.logits_sent++;
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
    return att1_infer_logits(ci->single, out_count);
}

att1_status_t att1_cluster_infer_position(const att1_cluster_infer_t *ci, size_t *out_position)
{
    if (ci == NULL) return ATT1_ERR_INVALID_ARG;
    return att1_infer_position(ci->single, out_position);
}

att1_status_t att1_cluster_infer_get_tile_counters(const att1_cluster_infer_t *ci, uint32_t tile_id,
                                                   att1_cluster_tile_counters *out)
{
    if (ci == NULL || out == NULL || tile_id >= ci->tiles) return ATT1_ERR_INVALID_ARG;
    *out = ci->counters;
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
    return att1_infer_set_trace(ci->single, trace);
}

att1_status_t att1_cluster_infer_set_backend(att1_cluster_infer_t *ci, att1_backend *backend)
{
    if (ci == NULL) return ATT1_ERR_INVALID_ARG;
    return att1_infer_set_backend(ci->single, backend);
}
