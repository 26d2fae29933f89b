/*
 * att1_trace.c - counters behind att1_trace.h (ATT-1 include/att1_trace.h).
 * Plain host bookkeeping; the decode paths call the record functions once
 * per token and per layer as the reference infer loop does
 * (src/infer.c:684-686, 803-811, 869-876).
 */
#define _POSIX_C_SOURCE 200809L
#include "att1_trace.h"

#include <stdlib.h>
#include <string.h>
#include <time.h>

struct att1_trace {
    size_t layers, tiles;
    att1_trace_counters c;
    att1_trace_layer *layer;
    att1_trace_tile *tile;
    uint64_t *token_us;
    size_t tokens, token_cap;
};

att1_status_t att1_trace_create(size_t layer_count, size_t tile_count, att1_trace_t **out)
{
    att1_trace_t *t;
    if (out == NULL) return ATT1_ERR_INVALID_ARG;
    *out = NULL;
    t = calloc(1, sizeof(*t));
    if (t == NULL) return ATT1_ERR_OOM;
    t->layers = layer_count;
    t->tiles = tile_count;
    t->layer = calloc(layer_count ? layer_count : 1, sizeof(*t->layer));
    t->tile = calloc(tile_count ? tile_count : 1, sizeof(*t->tile));
    if (t->layer == NULL || t->tile == NULL) {
        att1_trace_destroy(t);
        return ATT1_ERR_OOM;
    }
    *out = t;
    return ATT1_OK;
}

void att1_trace_destroy(att1_trace_t *t)
{
    if (t == NULL) return;
    free(t->layer);
    free(t->tile);
    free(t->token_us);
    free(t);
}

void att1_trace_reset(att1_trace_t *t)
{
    if (t == NULL) return;
    memset(&t->c, 0, sizeof(t->c));
    memset(t->layer, 0, (t->layers ? t->layers : 1) * sizeof(*t->layer));
    memset(t->tile, 0, (t->tiles ? t->tiles : 1) * sizeof(*t->tile));
    t->tokens = 0;
}

att1_status_t att1_trace_snapshot(const att1_trace_t *t, att1_trace_counters *out)
{
    if (t == NULL || out == NULL) return ATT1_ERR_INVALID_ARG;
    *out = t->c;
    return ATT1_OK;
}

att1_status_t att1_trace_layer_snapshot(const att1_trace_t *t, size_t id, att1_trace_layer *out)
{
    if (t == NULL || out == NULL || id >= t->layers) return ATT1_ERR_INVALID_ARG;
    *out = t->layer[id];
    return ATT1_OK;
}

att1_status_t att1_trace_tile_snapshot(const att1_trace_t *t, size_t id, att1_trace_tile *out)
{
    if (t == NULL || out == NULL || id >= t->tiles) return ATT1_ERR_INVALID_ARG;
    *out = t->tile[id];
    return ATT1_OK;
}

att1_status_t att1_trace_token_time_us(const att1_trace_t *t, size_t i, uint64_t *out)
{
    if (t == NULL || out == NULL || i >= t->tokens) return ATT1_ERR_INVALID_ARG;
    *out = t->token_us[i];
    return ATT1_OK;
}

size_t att1_trace_layer_count(const att1_trace_t *t) { return t ? t->layers : 0; }
size_t att1_trace_tile_count(const att1_trace_t *t) { return t ? t->tiles : 0; }
size_t att1_trace_token_count(const att1_trace_t *t) { return t ? t->tokens : 0; }

uint64_t att1_trace_now_us(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (uint64_t)ts.tv_sec * 1000000u + (uint64_t)ts.tv_nsec / 1000u;
}

void att1_trace_record_token(att1_trace_t *t, uint64_t us)
{
    if (t == NULL) return;
    t->c.tokens_decoded++;
    t->c.token_time_us_total += us;
    if (us > t->c.token_time_us_max) t->c.token_time_us_max = us;
    if (t->tokens == t->token_cap) {
        size_t cap = t->token_cap ? 2 * t->token_cap : 64;
        uint64_t *p = realloc(t->token_us, cap * sizeof(*p));
        if (p == NULL) return;
        t->token_us = p;
        t->token_cap = cap;
    }
    t->token_us[t->tokens++] = us;
}

void att1_trace_record_layer(att1_trace_t *t, size_t id, uint64_t us, uint64_t appends, uint64_t kr,
                             uint64_t vr)
{
    if (t == NULL) return;
    t->c.layer_time_us_total += us;
    t->c.kv_appends += appends;
    t->c.kv_key_reads += kr;
    t->c.kv_value_reads += vr;
    if (id < t->layers) {
        t->layer[id].executions++;
        t->layer[id].time_us_total += us;
        t->layer[id].kv_appends += appends;
        t->layer[id].kv_key_reads += kr;
        t->layer[id].kv_value_reads += vr;
    }
}

void att1_trace_record_activation_send(att1_trace_t *t, size_t id, uint64_t bytes)
{
    if (t == NULL) return;
    t->c.activation_bytes_sent += bytes;
    if (id < t->tiles) t->tile[id].activation_bytes_sent += bytes;
}

void att1_trace_record_logits(att1_trace_t *t, size_t id, uint64_t bytes)
{
    if (t == NULL) return;
    t->c.logits_bytes_produced += bytes;
    if (id < t->tiles) t->tile[id].logits_bytes_produced += bytes;
}

void att1_trace_record_fabric_send(att1_trace_t *t, uint64_t bytes)
{
    if (t == NULL) return;
    t->c.fabric_packets_sent++;
    t->c.fabric_payload_bytes_sent += bytes;
}

void att1_trace_record_fabric_receive(att1_trace_t *t, uint64_t bytes)
{
    if (t == NULL) return;
    t->c.fabric_packets_received++;
    t->c.fabric_payload_bytes_received += bytes;
}

void att1_trace_record_tile_layers(att1_trace_t *t, size_t id, uint64_t n)
{
    if (t == NULL) return;
    t->c.tile_layer_executions += n;
    if (id < t->tiles) t->tile[id].layer_executions += n;
}
