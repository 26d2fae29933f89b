/*
 * att1_cluster_infer.h - multi-device decode (ATT-1 cluster API).
 *
 * Same functions and argument meaning as ATT-1's include/att1_cluster_infer.h
 * (src/cluster_infer.c:580-1318). Where the reference runs contiguous layer
 * ranges on simulated tiles, each "tile" here is one GPU of the box and the
 * model is split tensor-parallel: column-parallel q/k/v and gate/up (heads
 * and FFN rows per GPU), row-parallel out/down followed by an all-reduce over
 * NVLink, vocab-split lm_head followed by an all-gather of logits. Logits are
 * the same as the single-device path within f32 reassociation error.
 * tile_count must divide n_heads (and the KV heads) and d_ff / 8.
 */
#ifndef ATT1_CLUSTER_INFER_H
#define ATT1_CLUSTER_INFER_H

#include "att1_backend.h"
#include "att1_model.h"
#include "att1_status.h"
#include "att1_trace.h"

#include <stddef.h>
#include <stdint.h>

typedef struct att1_cluster_infer att1_cluster_infer_t;

typedef enum att1_shard_plan_mode {
    ATT1_SHARD_PLAN_RUNTIME = 0,
    ATT1_SHARD_PLAN_METADATA = 1
} att1_shard_plan_mode;

typedef struct att1_layer_shard {
    uint32_t tile_id;
    uint32_t layer_start;
    uint32_t layer_end;
} att1_layer_shard;

typedef struct att1_cluster_infer_config {
    size_t tile_count;                    /* GPUs, 1..8 */
    size_t fabric_queue_capacity;         /* accepted, unused (no packet fabric) */
    size_t fabric_max_payload_bytes;      /* accepted, unused */
    att1_shard_plan_mode shard_plan_mode; /* RUNTIME only */
} att1_cluster_infer_config;

typedef struct att1_cluster_tile_counters {
    uint64_t activations_received;        /* all-reduce inputs received */
    uint64_t activations_sent;            /* all-reduce contributions sent */
    uint64_t layers_run;
    uint64_t logits_sent;
    uint32_t layer_start;
    uint32_t layer_end;
} att1_cluster_tile_counters;

att1_status_t att1_cluster_infer_create(const att1_model *model,
                                        const att1_cluster_infer_config *config,
                                        att1_cluster_infer_t **out_infer);
att1_status_t att1_cluster_infer_create_q4(const att1_model *model,
                                           const att1_cluster_infer_config *config,
                                           att1_cluster_infer_t **out_infer);
void att1_cluster_infer_destroy(att1_cluster_infer_t *infer);
att1_status_t att1_cluster_infer_decode_token(att1_cluster_infer_t *infer, uint32_t token_id,
                                              uint32_t *out_token);
att1_status_t att1_cluster_infer_generate(att1_cluster_infer_t *infer,
                                          const unsigned char *prompt, size_t prompt_bytes,
                                          size_t generated_token_count, uint32_t *out_tokens,
                                          size_t out_token_capacity, size_t *out_token_count);
const float *att1_cluster_infer_logits(const att1_cluster_infer_t *infer, size_t *out_count);
att1_status_t att1_cluster_infer_position(const att1_cluster_infer_t *infer,
                                          size_t *out_position);
att1_status_t att1_cluster_infer_get_tile_counters(const att1_cluster_infer_t *infer,
                                                   uint32_t tile_id,
                                                   att1_cluster_tile_counters *out_counters);
/* Every tile runs every layer under tensor parallelism: [0, n_layers). */
att1_status_t att1_cluster_infer_get_tile_shard(const att1_cluster_infer_t *infer,
                                                uint32_t tile_id, att1_layer_shard *out_shard);
att1_status_t att1_cluster_infer_set_trace(att1_cluster_infer_t *infer, att1_trace_t *trace);
att1_status_t att1_cluster_infer_set_backend(att1_cluster_infer_t *infer,
                                             att1_backend *backend);

#endif
