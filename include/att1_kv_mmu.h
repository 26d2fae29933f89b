/*
 * att1_kv_mmu.h - paged KV memory manager (ATT-1 KV-MMU API) on the device.
 *
 * Same functions, structs and status codes as ATT-1's include/att1_kv_mmu.h
 * (src/kv_mmu.c:318-642), so a caller of the reference's KV-MMU recompiles
 * unchanged. Here the pages are device memory: one pool of max_pages pages
 * for K and one for V, each page holding page_tokens positions of num_heads
 * heads in the layout the decode kernels read ([head][token_in_page][head_dim]
 * f32: a head's positions are contiguous), and a device page table per
 * (session, layer) that maps logical pages to physical ones.
 * att1_b200_kv_mmu_layout (att1_b200.h) hands a session's layer to the
 * attention and KV-append kernels of b2_kernels.h.
 *
 * Behaviour kept from the reference: sessions are caller-chosen ids; pages are
 * taken on demand, the lowest free physical page first, when an append opens
 * a new logical page; appends are sequential per (session, layer) from 0 (gaps
 * and repeats are rejected); destroying a session frees its pages; every
 * rejected call counts in `errors`; lookups of an existing page count a hit,
 * of a missing page a miss (appends and reads look up too); a range copy
 * counts one read per position and one range copy when it completes. Calls
 * are synchronous: host buffers in and out, the copies finished on return.
 * The handle is not thread-safe.
 */
#ifndef ATT1_KV_MMU_H
#define ATT1_KV_MMU_H

#include "att1_status.h"

#include <stddef.h>
#include <stdint.h>

typedef struct att1_kv_mmu_config {
    size_t max_sessions;
    size_t max_pages;
    size_t num_layers;
    size_t num_heads;
    size_t head_dim;
    size_t page_tokens;
    size_t max_positions;  /* per session and layer; at most max_pages * page_tokens */
} att1_kv_mmu_config;

typedef struct att1_kv_mmu_counters {
    uint64_t page_hits;
    uint64_t page_misses;
    uint64_t page_allocations;
    uint64_t append_ops;
    uint64_t read_ops;
    uint64_t range_copy_ops;
    uint64_t errors;
} att1_kv_mmu_counters;

typedef struct att1_kv_mmu_page_ref {
    uint64_t physical_page;
    uint64_t session_id;
    size_t layer_id;
    size_t logical_page;
    size_t page_tokens;
} att1_kv_mmu_page_ref;

typedef struct att1_kv_mmu att1_kv_mmu;

/* Allocates the page pools (zeroed) and page tables on the current device. */
att1_status_t att1_kv_mmu_create(const att1_kv_mmu_config *config, att1_kv_mmu **out_mmu);
void att1_kv_mmu_destroy(att1_kv_mmu *mmu);

att1_status_t att1_kv_mmu_create_session(att1_kv_mmu *mmu, uint64_t session_id);
att1_status_t att1_kv_mmu_destroy_session(att1_kv_mmu *mmu, uint64_t session_id);

/* key, value: host [num_heads][head_dim] f32 for `position` (the next one). */
att1_status_t att1_kv_mmu_append(att1_kv_mmu *mmu, uint64_t session_id, size_t layer_id, size_t position,
                                 const float *key, const float *value);
/* One head's vectors into host buffers of head_dim (either may be NULL). */
att1_status_t att1_kv_mmu_read(att1_kv_mmu *mmu, uint64_t session_id, size_t layer_id, size_t head_id,
                               size_t position, float *out_key, float *out_value);
/* position_count consecutive positions of one head, [position][head_dim]. */
att1_status_t att1_kv_mmu_copy_range(att1_kv_mmu *mmu, uint64_t session_id, size_t layer_id, size_t head_id,
                                     size_t start_position, size_t position_count, float *out_keys,
                                     float *out_values);
/* The page holding `position`; ATT1_ERR_NOT_FOUND (not an error count) if none. */
att1_status_t att1_kv_mmu_lookup_page(att1_kv_mmu *mmu, uint64_t session_id, size_t layer_id, size_t position,
                                      att1_kv_mmu_page_ref *out_page);

void att1_kv_mmu_get_counters(const att1_kv_mmu *mmu, att1_kv_mmu_counters *out_counters);
void att1_kv_mmu_reset_counters(att1_kv_mmu *mmu);

#endif
