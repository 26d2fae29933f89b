/*
 * att1_kv_mmu.c - the ATT-1 KV-MMU API (include/att1_kv_mmu.h) over device
 * page pools.
 *
 * Reference behaviour: src/kv_mmu.c:318-642 (validation order, status codes,
 * counters). The bookkeeping (sessions, page owners, per-(session, layer)
 * lengths, a host mirror of the page table) stays on the host so that lookups
 * and rejections need no device round trip; the K/V data and the page table
 * the kernels read live on the device:
 *   k_pool, v_pool   [max_pages][num_heads][page_tokens][head_dim] f32
 *   page_table       [num_layers][max_sessions][pages_per_seq] int32 (layer-major:
 *                    the rows of sessions in consecutive slots are consecutive, as
 *                    the kernels index a batch's rows)
 * Appends write one position of every head with one strided copy; range copies
 * move the contiguous run of a head inside each page with one copy per page.
 */
#define _POSIX_C_SOURCE 200809L
#include "att1_kv_mmu.h"
#include "att1_b200.h"
#include "b2_host.h"

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct kv_page_owner {
    int active;
    size_t slot, layer, logical_page;
} kv_page_owner;

struct att1_kv_mmu {
    att1_kv_mmu_config config;
    att1_kv_mmu_counters counters;
    size_t pages_per_seq;
    int device;
    uint64_t *session_id;   /* [max_sessions] */
    int *session_active;    /* [max_sessions] */
    size_t *length;         /* [max_sessions][num_layers] appended positions */
    int32_t *table;         /* host mirror [max_sessions][num_layers][pages_per_seq], -1 = none */
    kv_page_owner *owner;   /* [max_pages] */
    float *k_pool, *v_pool; /* device */
    int32_t *page_table;    /* device */
};

static void count_error(att1_kv_mmu *mmu)
{
    if (mmu != NULL) mmu->counters.errors++;
}

static int mul_ok(size_t a, size_t b, size_t *out)
{
    if (a != 0 && b > SIZE_MAX / a) return 0;
    *out = a * b;
    return 1;
}

/* src/kv_mmu.c:47-83: every dimension non-zero, no size overflow, the
 * positions of one (session, layer) fit in the page pool. */
static int config_valid(const att1_kv_mmu_config *c)
{
    size_t hd, page, cap, bytes;
    if (c == NULL) return 0;
    if (c->max_sessions == 0 || c->max_pages == 0 || c->num_layers == 0 || c->num_heads == 0 || c->head_dim == 0 ||
        c->page_tokens == 0 || c->max_positions == 0)
        return 0;
    if (!mul_ok(c->num_heads, c->head_dim, &hd) || !mul_ok(c->page_tokens, hd, &page) ||
        !mul_ok(c->max_pages, c->page_tokens, &cap) || !mul_ok(c->max_pages, page, &bytes) ||
        !mul_ok(bytes, sizeof(float), &bytes))
        return 0;
    if (c->max_positions > cap) return 0;
    /* the device page table holds 32-bit page ids */
    if (c->max_pages > (size_t)INT32_MAX) return 0;
    return page > 0;
}

static size_t page_elems(const att1_kv_mmu *mmu)
{
    return mmu->config.page_tokens * mmu->config.num_heads * mmu->config.head_dim;
}

static int find_slot(const att1_kv_mmu *mmu, uint64_t session_id, size_t *slot)
{
    size_t i;
    for (i = 0; i < mmu->config.max_sessions; i++)
        if (mmu->session_active[i] && mmu->session_id[i] == session_id) {
            *slot = i;
            return 1;
        }
    return 0;
}

static int32_t *mirror(att1_kv_mmu *mmu, size_t slot, size_t layer)
{
    return mmu->table + (slot * mmu->config.num_layers + layer) * mmu->pages_per_seq;
}

/* Offset of (slot, layer, logical page) in the device page table. */
static size_t dev_index(const att1_kv_mmu *mmu, size_t slot, size_t layer, size_t lp)
{
    return (layer * mmu->config.max_sessions + slot) * mmu->pages_per_seq + lp;
}

/* Map logical page lp of (slot, layer) to the lowest free physical page:
 * bookkeeping, device table entry, allocation counter. -1 when none is free. */
static int32_t map_page(att1_kv_mmu *mmu, size_t slot, size_t layer, size_t lp)
{
    const att1_kv_mmu_config *c = &mmu->config;
    int32_t pp;
    size_t p;
    for (p = 0; p < c->max_pages && mmu->owner[p].active; p++) {
    }
    if (p == c->max_pages) return -1;
    pp = (int32_t)p;
    /* the entry must be on the device before this returns: decode kernels on a
     * non-blocking stream do not wait for the legacy stream's copy */
    if (cudaSetDevice(mmu->device) != cudaSuccess ||
        cudaMemcpy(mmu->page_table + dev_index(mmu, slot, layer, lp), &pp, sizeof(int32_t), cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        cudaStreamSynchronize(cudaStreamLegacy) != cudaSuccess)
        return -2;
    mmu->owner[p].active = 1;
    mmu->owner[p].slot = slot;
    mmu->owner[p].layer = layer;
    mmu->owner[p].logical_page = lp;
    mirror(mmu, slot, layer)[lp] = pp;
    mmu->counters.page_allocations++;
    return pp;
}

/* src/kv_mmu.c:263-285 */
static att1_status_t check_address(att1_kv_mmu *mmu, uint64_t session_id, size_t layer_id, size_t *slot)
{
    if (mmu == NULL) return ATT1_ERR_INVALID_ARG;
    if (!find_slot(mmu, session_id, slot)) {
        count_error(mmu);
        return ATT1_ERR_NOT_FOUND;
    }
    if (layer_id >= mmu->config.num_layers) {
        count_error(mmu);
        return ATT1_ERR_INVALID_ARG;
    }
    return ATT1_OK;
}

static att1_status_t check_position(att1_kv_mmu *mmu, size_t position)
{
    if (position >= mmu->config.max_positions) {
        count_error(mmu);
        return ATT1_ERR_INVALID_ARG;
    }
    return ATT1_OK;
}

/* The physical page of `position`, counting a hit or a miss (src/kv_mmu.c:193-209). */
static int32_t lookup_counted(att1_kv_mmu *mmu, size_t slot, size_t layer, size_t position)
{
    const int32_t pp = mirror(mmu, slot, layer)[position / mmu->config.page_tokens];
    if (pp < 0)
        mmu->counters.page_misses++;
    else
        mmu->counters.page_hits++;
    return pp;
}

static void release(att1_kv_mmu *mmu)
{
    if (mmu == NULL) return;
    if (mmu->k_pool) cudaFree(mmu->k_pool);
    if (mmu->v_pool) cudaFree(mmu->v_pool);
    if (mmu->page_table) cudaFree(mmu->page_table);
    free(mmu->session_id);
    free(mmu->session_active);
    free(mmu->length);
    free(mmu->table);
    free(mmu->owner);
    free(mmu);
}

att1_status_t att1_kv_mmu_create(const att1_kv_mmu_config *config, att1_kv_mmu **out_mmu)
{
    att1_kv_mmu *mmu;
    size_t rows, pool, i;
    cudaError_t e;
    if (out_mmu == NULL) return ATT1_ERR_INVALID_ARG;
    *out_mmu = NULL;
    if (!config_valid(config)) return ATT1_ERR_INVALID_ARG;
    mmu = calloc(1, sizeof(*mmu));
    if (mmu == NULL) return ATT1_ERR_OOM;
    mmu->config = *config;
    mmu->pages_per_seq = (config->max_positions + config->page_tokens - 1) / config->page_tokens;
    if (!mul_ok(config->max_sessions, config->num_layers, &rows) || !mul_ok(rows, mmu->pages_per_seq, &rows)) {
        free(mmu);
        return ATT1_ERR_INVALID_ARG;
    }
    mmu->session_id = calloc(config->max_sessions, sizeof(uint64_t));
    mmu->session_active = calloc(config->max_sessions, sizeof(int));
    mmu->length = calloc(config->max_sessions * config->num_layers, sizeof(size_t));
    mmu->table = malloc(rows * sizeof(int32_t));
    mmu->owner = calloc(config->max_pages, sizeof(kv_page_owner));
    if (!mmu->session_id || !mmu->session_active || !mmu->length || !mmu->table || !mmu->owner) {
        release(mmu);
        return ATT1_ERR_OOM;
    }
    for (i = 0; i < rows; i++) mmu->table[i] = -1;
    pool = config->max_pages * page_elems(mmu) * sizeof(float);
    if (cudaGetDevice(&mmu->device) != cudaSuccess || cudaMalloc((void **)&mmu->k_pool, pool) != cudaSuccess ||
        cudaMalloc((void **)&mmu->v_pool, pool) != cudaSuccess ||
        cudaMalloc((void **)&mmu->page_table, rows * sizeof(int32_t)) != cudaSuccess) {
        cudaGetLastError();
        release(mmu);
        return ATT1_ERR_OOM;
    }
    /* zeroed pages; unmapped table entries name page 0, so a kernel handed a
     * position beyond a session's length reads inside the pool */
    e = cudaMemset(mmu->k_pool, 0, pool);
    if (e == cudaSuccess) e = cudaMemset(mmu->v_pool, 0, pool);
    if (e == cudaSuccess) e = cudaMemset(mmu->page_table, 0, rows * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        release(mmu);
        return b2_cuda_status(e);
    }
    *out_mmu = mmu;
    return ATT1_OK;
}

void att1_kv_mmu_destroy(att1_kv_mmu *mmu)
{
    if (mmu == NULL) return;
    cudaSetDevice(mmu->device);
    release(mmu);
}

att1_status_t att1_kv_mmu_create_session(att1_kv_mmu *mmu, uint64_t session_id)
{
    size_t i, slot;
    if (mmu == NULL) return ATT1_ERR_INVALID_ARG;
    if (find_slot(mmu, session_id, &slot)) {
        count_error(mmu);
        return ATT1_ERR_STATE;
    }
    for (i = 0; i < mmu->config.max_sessions; i++) {
        if (!mmu->session_active[i]) {
            mmu->session_active[i] = 1;
            mmu->session_id[i] = session_id;
            return ATT1_OK;
        }
    }
    count_error(mmu);
    return ATT1_ERR_OOM;
}

att1_status_t att1_kv_mmu_destroy_session(att1_kv_mmu *mmu, uint64_t session_id)
{
    size_t slot, l, p;
    if (mmu == NULL) return ATT1_ERR_INVALID_ARG;
    if (!find_slot(mmu, session_id, &slot)) {
        count_error(mmu);
        return ATT1_ERR_NOT_FOUND;
    }
    for (p = 0; p < mmu->config.max_pages; p++)
        if (mmu->owner[p].active && mmu->owner[p].slot == slot) memset(&mmu->owner[p], 0, sizeof(kv_page_owner));
    for (l = 0; l < mmu->config.num_layers; l++) {
        int32_t *row = mirror(mmu, slot, l);
        for (p = 0; p < mmu->pages_per_seq; p++) row[p] = -1;
        mmu->length[slot * mmu->config.num_layers + l] = 0;
    }
    mmu->session_active[slot] = 0;
    mmu->session_id[slot] = 0;
    return ATT1_OK;
}

att1_status_t att1_kv_mmu_append(att1_kv_mmu *mmu, uint64_t session_id, size_t layer_id, size_t position,
                                 const float *key, const float *value)
{
    const att1_kv_mmu_config *c;
    size_t slot, *len, hd;
    int32_t pp;
    att1_status_t st;
    float *kdst, *vdst;
    cudaError_t e;
    if (key == NULL || value == NULL) {
        count_error(mmu);
        return ATT1_ERR_INVALID_ARG;
    }
    if ((st = check_address(mmu, session_id, layer_id, &slot)) != ATT1_OK) return st;
    if ((st = check_position(mmu, position)) != ATT1_OK) return st;
    c = &mmu->config;
    len = &mmu->length[slot * c->num_layers + layer_id];
    if (position != *len) { /* appends are sequential from 0, no overwrite */
        count_error(mmu);
        return ATT1_ERR_STATE;
    }
    pp = lookup_counted(mmu, slot, layer_id, position);
    if (pp < 0) {
        /* a new logical page: the lowest free physical page (src/kv_mmu.c:158-191) */
        pp = map_page(mmu, slot, layer_id, position / c->page_tokens);
        if (pp < 0) {
            count_error(mmu);
            return pp == -1 ? ATT1_ERR_OOM : ATT1_ERR_STATE;
        }
    }
    /* one position of every head: head h at (h * page_tokens + t) * head_dim */
    hd = c->head_dim;
    kdst = mmu->k_pool + (size_t)pp * page_elems(mmu) + (position % c->page_tokens) * hd;
    vdst = mmu->v_pool + (size_t)pp * page_elems(mmu) + (position % c->page_tokens) * hd;
    e = cudaSetDevice(mmu->device);
    if (e == cudaSuccess)
        e = cudaMemcpy2D(kdst, c->page_tokens * hd * sizeof(float), key, hd * sizeof(float), hd * sizeof(float),
                         c->num_heads, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy2D(vdst, c->page_tokens * hd * sizeof(float), value, hd * sizeof(float), hd * sizeof(float),
                         c->num_heads, cudaMemcpyHostToDevice);
    /* a pageable host-to-device copy may still be in flight when cudaMemcpy
     * returns; kernels on other streams read the row next */
    if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamLegacy);
    if (e != cudaSuccess) {
        count_error(mmu);
        return b2_cuda_status(e);
    }
    (*len)++;
    mmu->counters.append_ops++;
    return ATT1_OK;
}

/* Device address of one head's vector at `position` in physical page pp. */
static size_t head_offset(const att1_kv_mmu *mmu, int32_t pp, size_t head, size_t position)
{
    const att1_kv_mmu_config *c = &mmu->config;
    return (size_t)pp * page_elems(mmu) + (head * c->page_tokens + position % c->page_tokens) * c->head_dim;
}

att1_status_t att1_kv_mmu_read(att1_kv_mmu *mmu, uint64_t session_id, size_t layer_id, size_t head_id,
                               size_t position, float *out_key, float *out_value)
{
    size_t slot;
    int32_t pp;
    att1_status_t st;
    cudaError_t e;
    if (out_key == NULL && out_value == NULL) {
        count_error(mmu);
        return ATT1_ERR_INVALID_ARG;
    }
    if ((st = check_address(mmu, session_id, layer_id, &slot)) != ATT1_OK) return st;
    if ((st = check_position(mmu, position)) != ATT1_OK) return st;
    if (head_id >= mmu->config.num_heads) {
        count_error(mmu);
        return ATT1_ERR_INVALID_ARG;
    }
    pp = lookup_counted(mmu, slot, layer_id, position);
    if (pp < 0 || position >= mmu->length[slot * mmu->config.num_layers + layer_id]) {
        count_error(mmu);
        return ATT1_ERR_NOT_FOUND;
    }
    e = cudaSetDevice(mmu->device);
    if (e == cudaSuccess && out_key != NULL)
        e = cudaMemcpy(out_key, mmu->k_pool + head_offset(mmu, pp, head_id, position),
                       mmu->config.head_dim * sizeof(float), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && out_value != NULL)
        e = cudaMemcpy(out_value, mmu->v_pool + head_offset(mmu, pp, head_id, position),
                       mmu->config.head_dim * sizeof(float), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        count_error(mmu);
        return b2_cuda_status(e);
    }
    mmu->counters.read_ops++;
    return ATT1_OK;
}

/* Copy positions [start, start + n) of one head, one copy per page run. */
static cudaError_t copy_runs(att1_kv_mmu *mmu, size_t slot, size_t layer, size_t head, size_t start, size_t n,
                             float *out_keys, float *out_values)
{
    const size_t T = mmu->config.page_tokens, hd = mmu->config.head_dim;
    cudaError_t e = cudaSetDevice(mmu->device);
    size_t done = 0;
    while (e == cudaSuccess && done < n) {
        const size_t pos = start + done;
        size_t run = T - pos % T;
        const int32_t pp = mirror(mmu, slot, layer)[pos / T];
        if (run > n - done) run = n - done;
        if (out_keys != NULL)
            e = cudaMemcpy(out_keys + done * hd, mmu->k_pool + head_offset(mmu, pp, head, pos),
                           run * hd * sizeof(float), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess && out_values != NULL)
            e = cudaMemcpy(out_values + done * hd, mmu->v_pool + head_offset(mmu, pp, head, pos),
                           run * hd * sizeof(float), cudaMemcpyDeviceToHost);
        done += run;
    }
    return e;
}

att1_status_t att1_kv_mmu_copy_range(att1_kv_mmu *mmu, uint64_t session_id, size_t layer_id, size_t head_id,
                                     size_t start_position, size_t position_count, float *out_keys,
                                     float *out_values)
{
    size_t slot, good, len, i;
    att1_status_t st = ATT1_OK;
    cudaError_t e;
    if (mmu == NULL) return ATT1_ERR_INVALID_ARG;
    if (out_keys == NULL && out_values == NULL) {
        count_error(mmu);
        return ATT1_ERR_INVALID_ARG;
    }
    /* src/kv_mmu.c:287-313 */
    if (position_count == 0 || start_position > SIZE_MAX - (position_count - 1) ||
        start_position + position_count > mmu->config.max_positions) {
        count_error(mmu);
        return ATT1_ERR_INVALID_ARG;
    }
    if (head_id >= mmu->config.num_heads) {
        count_error(mmu);
        return ATT1_ERR_INVALID_ARG;
    }
    /* every position is one read (address check, page lookup, presence) as
     * in the reference; the readable prefix is copied before an error returns */
    if ((st = check_address(mmu, session_id, layer_id, &slot)) != ATT1_OK) return st;
    len = mmu->length[slot * mmu->config.num_layers + layer_id];
    good = 0;
    for (i = 0; i < position_count; i++) {
        const size_t pos = start_position + i;
        const int32_t pp = lookup_counted(mmu, slot, layer_id, pos);
        if (pp < 0 || pos >= len) {
            count_error(mmu);
            st = ATT1_ERR_NOT_FOUND;
            break;
        }
        good++;
    }
    e = good > 0 ? copy_runs(mmu, slot, layer_id, head_id, start_position, good, out_keys, out_values) : cudaSuccess;
    if (e != cudaSuccess) {
        count_error(mmu);
        return b2_cuda_status(e);
    }
    mmu->counters.read_ops += good;
    if (st != ATT1_OK) return st;
    mmu->counters.range_copy_ops++;
    return ATT1_OK;
}

att1_status_t att1_kv_mmu_lookup_page(att1_kv_mmu *mmu, uint64_t session_id, size_t layer_id, size_t position,
                                      att1_kv_mmu_page_ref *out_page)
{
    size_t slot;
    int32_t pp;
    att1_status_t st;
    if (out_page == NULL) {
        count_error(mmu);
        return ATT1_ERR_INVALID_ARG;
    }
    memset(out_page, 0, sizeof(*out_page));
    if ((st = check_address(mmu, session_id, layer_id, &slot)) != ATT1_OK) return st;
    if ((st = check_position(mmu, position)) != ATT1_OK) return st;
    pp = lookup_counted(mmu, slot, layer_id, position);
    if (pp < 0) return ATT1_ERR_NOT_FOUND;
    out_page->physical_page = (uint64_t)pp;
    out_page->session_id = session_id;
    out_page->layer_id = layer_id;
    out_page->logical_page = position / mmu->config.page_tokens;
    out_page->page_tokens = mmu->config.page_tokens;
    return ATT1_OK;
}

void att1_kv_mmu_get_counters(const att1_kv_mmu *mmu, att1_kv_mmu_counters *out_counters)
{
    if (mmu == NULL || out_counters == NULL) return;
    *out_counters = mmu->counters;
}

void att1_kv_mmu_reset_counters(att1_kv_mmu *mmu)
{
    if (mmu == NULL) return;
    memset(&mmu->counters, 0, sizeof(mmu->counters));
}

att1_status_t att1_b200_kv_mmu_layout(const att1_kv_mmu *mmu, uint64_t session_id, size_t layer_id,
                                      b2_kv_layout *out)
{
    size_t slot;
    if (mmu == NULL || out == NULL || layer_id >= mmu->config.num_layers) return ATT1_ERR_INVALID_ARG;
    if (!find_slot(mmu, session_id, &slot)) return ATT1_ERR_NOT_FOUND;
    if (mmu->config.page_tokens > UINT32_MAX || mmu->pages_per_seq > UINT32_MAX ||
        mmu->config.num_heads > UINT32_MAX || mmu->config.head_dim > UINT32_MAX)
        return ATT1_ERR_UNSUPPORTED;
    out->k_pool = mmu->k_pool;
    out->v_pool = mmu->v_pool;
    out->page_table = mmu->page_table + dev_index(mmu, slot, layer_id, 0);
    out->page_tokens = (uint32_t)mmu->config.page_tokens;
    out->pages_per_seq = (uint32_t)mmu->pages_per_seq;
    out->n_kv_heads = (uint32_t)mmu->config.num_heads;
    out->head_dim = (uint32_t)mmu->config.head_dim;
    return ATT1_OK;
}

/* ---- hooks for a decode context whose batch items are KV-MMU sessions ---------------------------- */

int b2_kv_mmu_session_slot(const att1_kv_mmu *mmu, uint64_t session_id, size_t *slot)
{
    return mmu != NULL && find_slot(mmu, session_id, slot);
}

size_t b2_kv_mmu_length(const att1_kv_mmu *mmu, size_t slot, size_t layer)
{
    return mmu->length[slot * mmu->config.num_layers + layer];
}

const att1_kv_mmu_config *b2_kv_mmu_config(const att1_kv_mmu *mmu)
{
    return &mmu->config;
}

/* Pages for positions [first, first + count) of (slot, every layer), mapped
 * before the kernels append there. */
att1_status_t b2_kv_mmu_reserve(att1_kv_mmu *mmu, size_t slot, size_t first, size_t count)
{
    const size_t T = mmu->config.page_tokens;
    size_t l, lp;
    if (count == 0) return ATT1_OK;
    if (first + count > mmu->config.max_positions) return ATT1_ERR_INVALID_ARG;
    for (l = 0; l < mmu->config.num_layers; l++)
        for (lp = first / T; lp <= (first + count - 1) / T; lp++)
            if (mirror(mmu, slot, l)[lp] < 0) {
                const int32_t pp = map_page(mmu, slot, l, lp);
                if (pp < 0) {
                    count_error(mmu);
                    return pp == -1 ? ATT1_ERR_OOM : ATT1_ERR_STATE;
                }
            }
    return ATT1_OK;
}

/* Host copy of (slot, layer)'s page-table row: pages_per_seq entries, -1 = none. */
const int32_t *b2_kv_mmu_row(const att1_kv_mmu *mmu, size_t slot, size_t layer, size_t *pages_per_seq)
{
    *pages_per_seq = mmu->pages_per_seq;
    return mirror((att1_kv_mmu *)mmu, slot, layer);
}

/* The kernels appended `count` positions of (slot, every layer). */
void b2_kv_mmu_advance(att1_kv_mmu *mmu, size_t slot, size_t count)
{
    size_t l;
    for (l = 0; l < mmu->config.num_layers; l++) mmu->length[slot * mmu->config.num_layers + l] += count;
    mmu->counters.append_ops += count * mmu->config.num_layers;
}
