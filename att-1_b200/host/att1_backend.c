/*
 * att1_backend.c - the "cuda", "cuda-q8" and "cuda-q4" backends of the ATT-1
 * vtable (include/att1_backend.h), implemented with the sm_100a kernels.
 *
 * Same op contract as the reference backends (src/backend_cpu_q4.c,
 * src/backend_cuda.c:701-805): host pointers in and out, 0 on success and -1
 * on failure. Differences in how the work is done: weights are converted to
 * the device unit layout once and cached by their data pointer instead of
 * being dequantised to f32 on the host on every call
 * (src/backend_cuda.c:269-358), one stream and one set of growing device
 * buffers are reused instead of a cudaMalloc/cublasCreate per op, and alloc
 * returns pinned host memory so the copies run at full PCIe rate.
 */
#define _POSIX_C_SOURCE 200809L
#include "att1_backend.h"
#include "b2_host.h"

#include <stdlib.h>
#include <string.h>

typedef struct cached_mat {
    const void *key;
    size_t rows, cols;
    b2_dev_mat m;       /* unit layout for b2_gemv */
    void *raw;          /* or: the reference layout (packed / values, then scales) for the ordered kernels */
    size_t raw_scales;  /* byte offset of the scales in raw */
    uint32_t group;
} cached_mat;

typedef struct cuda_backend {
    cudaStream_t stream;
    int device;
    void *buf[3];
    size_t cap[3];
    void *scratch;
    size_t scratch_cap;
    int32_t *counters;
    uint32_t counters_cap;
    int32_t *err;
    unsigned long long *key;
    cached_mat *cache;
    size_t n_cache, cap_cache;
} cuda_backend;

static const att1_backend_ops cuda_f32_ops, cuda_q8_ops, cuda_q4_ops;

int b2_backend_is_cuda(const att1_backend *backend)
{
    return backend != NULL && (backend->ops == &cuda_f32_ops || backend->ops == &cuda_q8_ops ||
                               backend->ops == &cuda_q4_ops);
}

const char *b2_backend_name(const att1_backend *backend)
{
    return (backend != NULL && backend->ops != NULL) ? backend->ops->name : NULL;
}

static cuda_backend *cb(att1_backend *b) { return (cuda_backend *)b->user_data; }

static int ensure(cuda_backend *c, int slot, size_t bytes)
{
    if (c->cap[slot] >= bytes) return 0;
    if (c->buf[slot]) cudaFree(c->buf[slot]);
    c->buf[slot] = NULL;
    c->cap[slot] = 0;
    if (cudaMalloc(&c->buf[slot], bytes) != cudaSuccess) return -1;
    c->cap[slot] = bytes;
    return 0;
}

static int ensure_scratch(cuda_backend *c, size_t bytes)
{
    if (c->scratch_cap >= bytes) return 0;
    if (c->scratch) cudaFree(c->scratch);
    c->scratch = NULL;
    c->scratch_cap = 0;
    if (cudaMalloc(&c->scratch, bytes) != cudaSuccess) return -1;
    c->scratch_cap = bytes;
    return 0;
}

static int ensure_counters(cuda_backend *c, uint32_t n)
{
    if (c->counters_cap >= n) return 0;
    if (c->counters) cudaFree(c->counters);
    c->counters = NULL;
    c->counters_cap = 0;
    if (cudaMalloc((void **)&c->counters, (size_t)n * sizeof(int32_t)) != cudaSuccess) return -1;
    /* zeroed on the backend's stream, ahead of the kernels that use them (a
     * plain cudaMemset runs on the legacy stream, which a non-blocking stream
     * does not wait for) */
    if (cudaMemsetAsync(c->counters, 0, (size_t)n * sizeof(int32_t), c->stream) != cudaSuccess) return -1;
    c->counters_cap = n;
    return 0;
}

static int finish(cuda_backend *c)
{
    int32_t err = 0;
    if (cudaMemcpyAsync(&err, c->err, sizeof(err), cudaMemcpyDeviceToHost, c->stream) != cudaSuccess) return -1;
    if (cudaStreamSynchronize(c->stream) != cudaSuccess) return -1;
    if (err != 0) {
        cudaMemsetAsync(c->err, 0, sizeof(int32_t), c->stream);
        if (c->counters) cudaMemsetAsync(c->counters, 0, (size_t)c->counters_cap * sizeof(int32_t), c->stream);
        cudaStreamSynchronize(c->stream);
        return -1;
    }
    return 0;
}

/* ---- memory --------------------------------------------------------------------- */

static void *cuda_alloc(att1_backend *b, size_t bytes)
{
    void *p = NULL;
    (void)b;
    if (cudaMallocHost(&p, bytes ? bytes : 1) != cudaSuccess) return NULL;
    return p;
}

static void cuda_free(att1_backend *b, void *p)
{
    (void)b;
    if (p != NULL) cudaFreeHost(p);
}

static int cuda_sync(att1_backend *b)
{
    return cudaStreamSynchronize(cb(b)->stream) == cudaSuccess ? 0 : -1;
}

/* ---- weight cache --------------------------------------------------------------- */

static cached_mat *cache_find(cuda_backend *c, const void *key, size_t rows, size_t cols)
{
    size_t i;
    for (i = 0; i < c->n_cache; i++) {
        if (c->cache[i].key == key && c->cache[i].rows == rows && c->cache[i].cols == cols) return &c->cache[i];
    }
    return NULL;
}

static cached_mat *cache_add(cuda_backend *c)
{
    if (c->n_cache == c->cap_cache) {
        size_t cap = c->cap_cache ? 2 * c->cap_cache : 16;
        cached_mat *p = realloc(c->cache, cap * sizeof(*p));
        if (p == NULL) return NULL;
        c->cache = p;
        c->cap_cache = cap;
    }
    memset(&c->cache[c->n_cache], 0, sizeof(cached_mat));
    return &c->cache[c->n_cache++];
}

static int mat_init(b2_dev_mat *m, uint32_t fmt, uint32_t rows, uint32_t cols, cudaStream_t st)
{
    const size_t bytes = fmt == 4 ? b2_q4_bytes(rows, cols) : b2_q8_bytes(rows, cols);
    memset(m, 0, sizeof(*m));
    m->w.format = fmt;
    m->w.rows = rows;
    m->w.cols = cols;
    m->w.tiles = (rows + 15) / 16;
    m->w.kunits = fmt == 4 ? (cols + 63) / 64 : (cols + 31) / 32;
    if (cudaMalloc(&m->data, bytes) != cudaSuccess || cudaMemsetAsync(m->data, 0, bytes, st) != cudaSuccess) return -1;
    if (fmt == 8 && (cudaMalloc((void **)&m->row_scale, (size_t)m->w.tiles * 16 * 4) != cudaSuccess ||
                     cudaMemsetAsync(m->row_scale, 0, (size_t)m->w.tiles * 16 * 4, st) != cudaSuccess))
        return -1;
    m->w.data = m->data;
    m->w.row_scale = m->row_scale;
    return 0;
}

/* The unit layout holds q4 groups of 32, 64 or 128 and columns in multiples
 * of 32; anything else the reference accepts (group 16, other column counts)
 * runs the ordered kernels on a device copy of the reference layout. */
static int q4_unit_ok(const att1_q4_matrix *w)
{
    return (w->group_size == 32 || w->group_size == 64 || w->group_size == 128) && w->cols % 32 == 0 &&
           w->rows <= 0xFFFFFFFFu && w->cols <= 0xFFFFFFFFu;
}

static int q4_valid(const att1_q4_matrix *w)
{
    const uint32_t g = w->group_size;
    return w->packed != NULL && w->scales != NULL && w->rows > 0 && w->cols > 0 && g >= 16 && g <= 128 &&
           (g & (g - 1)) == 0 && w->cols % g == 0 && w->rows <= 0xFFFFFFFFu && w->cols <= 0xFFFFFFFFu;
}

static const cached_mat *raw_weight(cuda_backend *c, const void *key, const void *data, size_t data_bytes,
                                    const float *scales, size_t scale_bytes, size_t rows, size_t cols, uint32_t group)
{
    cached_mat *e = cache_find(c, key, rows, cols);
    const size_t off = (data_bytes + 255) & ~(size_t)255;
    if (e != NULL) return e;
    e = cache_add(c);
    if (e == NULL) return NULL;
    if (cudaMalloc(&e->raw, off + scale_bytes) != cudaSuccess ||
        cudaMemcpyAsync(e->raw, data, data_bytes, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
        cudaMemcpyAsync((uint8_t *)e->raw + off, scales, scale_bytes, cudaMemcpyHostToDevice, c->stream) !=
            cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess) {
        if (e->raw) cudaFree(e->raw);
        c->n_cache--;
        return NULL;
    }
    e->raw_scales = off;
    e->group = group;
    e->key = key;
    e->rows = rows;
    e->cols = cols;
    return e;
}

/* dst[lhs_rows][rows] = lhs * W^T through the ordered kernels */
static int run_ordered(cuda_backend *c, const cached_mat *e, int fmt, float *dst, const float *lhs, size_t lhs_rows)
{
    const size_t rows = e->rows, cols = e->cols;
    size_t done = 0;
    if (ensure(c, 0, lhs_rows * cols * sizeof(float)) || ensure(c, 1, lhs_rows * rows * sizeof(float))) return -1;
    if (cudaMemcpyAsync(c->buf[0], lhs, lhs_rows * cols * sizeof(float), cudaMemcpyHostToDevice, c->stream) !=
        cudaSuccess)
        return -1;
    while (done < lhs_rows) {
        const uint32_t nb = (uint32_t)((lhs_rows - done) > 65535 ? 65535 : (lhs_rows - done));
        float *out = (float *)c->buf[1] + done * rows;
        const float *x = (const float *)c->buf[0] + done * cols;
        const float *sc = (const float *)((const uint8_t *)e->raw + e->raw_scales);
        const int rc = fmt == 4 ? b2_matmul_q4_ordered(out, x, nb, (uint32_t)cols, e->raw, sc, (uint32_t)rows,
                                                      e->group, c->stream)
                                : b2_matmul_q8_ordered(out, x, nb, (uint32_t)cols, e->raw, sc, (uint32_t)rows,
                                                      c->stream);
        if (rc != 0) return -1;
        done += nb;
    }
    if (cudaMemcpyAsync(dst, c->buf[1], lhs_rows * rows * sizeof(float), cudaMemcpyDeviceToHost, c->stream) !=
        cudaSuccess)
        return -1;
    return finish(c);
}

static const b2_dev_mat *q4_weight(cuda_backend *c, const att1_q4_matrix *w)
{
    cached_mat *e = cache_find(c, w->packed, w->rows, w->cols);
    void *tmp = NULL;
    const size_t pb = w->rows * w->cols / 2, sb = w->rows * (w->cols / w->group_size) * sizeof(float);
    int rc;
    if (e != NULL) return &e->m;
    if (w->rows > 0xFFFFFFFFu || w->cols > 0xFFFFFFFFu) return NULL;
    e = cache_add(c);
    if (e == NULL) return NULL;
    if (mat_init(&e->m, 4, (uint32_t)w->rows, (uint32_t)w->cols, c->stream) != 0 ||
        cudaMalloc(&tmp, pb + sb) != cudaSuccess)
        goto fail;
    if (cudaMemcpyAsync(tmp, w->packed, pb, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
        cudaMemcpyAsync((uint8_t *)tmp + pb, w->scales, sb, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        goto fail;
    rc = b2_q4_pack(e->m.data, 0, (uint32_t)w->rows, (uint32_t)w->cols, tmp, (const float *)((uint8_t *)tmp + pb), NULL,
                    NULL, w->group_size, B2_ROWS_PLAIN, c->stream);
    if (rc != 0 || cudaStreamSynchronize(c->stream) != cudaSuccess) goto fail;
    cudaFree(tmp);
    e->key = w->packed;
    e->rows = w->rows;
    e->cols = w->cols;
    return &e->m;
fail:
    if (tmp) cudaFree(tmp);
    if (e->m.data) cudaFree(e->m.data);
    if (e->m.row_scale) cudaFree(e->m.row_scale);
    c->n_cache--;
    return NULL;
}

static const b2_dev_mat *q8_weight(cuda_backend *c, const att1_q8_matrix *w)
{
    cached_mat *e = cache_find(c, w->values, w->rows, w->cols);
    void *tmp = NULL;
    const size_t vb = w->rows * w->cols, sb = w->rows * sizeof(float);
    int rc;
    if (e != NULL) return &e->m;
    if (w->rows > 0xFFFFFFFFu || w->cols > 0xFFFFFFFFu) return NULL;
    e = cache_add(c);
    if (e == NULL) return NULL;
    if (mat_init(&e->m, 8, (uint32_t)w->rows, (uint32_t)w->cols, c->stream) != 0 ||
        cudaMalloc(&tmp, vb + sb) != cudaSuccess)
        goto fail;
    if (cudaMemcpyAsync(tmp, w->values, vb, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
        cudaMemcpyAsync((uint8_t *)tmp + vb, w->scales, sb, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        goto fail;
    rc = b2_q8_pack(e->m.data, e->m.row_scale, 0, (uint32_t)w->rows, (uint32_t)w->cols, tmp,
                    (const float *)((uint8_t *)tmp + vb), NULL, NULL, B2_ROWS_PLAIN, c->stream);
    if (rc != 0 || cudaStreamSynchronize(c->stream) != cudaSuccess) goto fail;
    cudaFree(tmp);
    e->key = w->values;
    e->rows = w->rows;
    e->cols = w->cols;
    return &e->m;
fail:
    if (tmp) cudaFree(tmp);
    if (e->m.data) cudaFree(e->m.data);
    if (e->m.row_scale) cudaFree(e->m.row_scale);
    c->n_cache--;
    return NULL;
}

/* ---- ops ----------------------------------------------------------------------------- */

/* dst[lhs_rows][rows] = lhs[lhs_rows][cols] * W^T, in batches of up to 16 rows */
static int run_gemv(cuda_backend *c, const b2_dev_mat *m, float *dst, const float *lhs, size_t lhs_rows, size_t cols)
{
    const size_t rows = m->w.rows;
    size_t done = 0;
    if (ensure(c, 0, lhs_rows * cols * sizeof(float)) || ensure(c, 1, lhs_rows * rows * sizeof(float))) return -1;
    if (cudaMemcpyAsync(c->buf[0], lhs, lhs_rows * cols * sizeof(float), cudaMemcpyHostToDevice, c->stream) !=
        cudaSuccess)
        return -1;
    uint32_t most = 16;
    while (done < lhs_rows) {
        const uint32_t nb = (uint32_t)((lhs_rows - done) > most ? most : (lhs_rows - done));
        b2_gemv_args a;
        size_t need;
        int rc;
        memset(&a, 0, sizeof(a));
        a.w = m->w;
        a.batch = nb;
        a.x = (const float *)c->buf[0] + done * cols;
        a.x_stride = (uint32_t)cols;
        a.epilogue = B2_EPI_STORE;
        a.out = (float *)c->buf[1] + done * rows;
        a.out_stride = (uint32_t)rows;
        a.err = c->err;
        need = b2_gemv_scratch_bytes(&a);
        if (ensure_scratch(c, need) || ensure_counters(c, b2_gemv_counters_len(&a))) return -1;
        a.scratch = c->scratch;
        a.scratch_bytes = c->scratch_cap;
        a.counters = c->counters;
        a.counters_len = c->counters_cap;
        rc = b2_gemv(&a, c->stream);
        if (rc == ATT1_ERR_UNSUPPORTED && nb > 1) { /* x's digit planes too large for nb items: fewer */
            most = nb / 2;
            continue;
        }
        if (rc != 0) return -1;
        done += nb;
    }
    if (cudaMemcpyAsync(dst, c->buf[1], lhs_rows * rows * sizeof(float), cudaMemcpyDeviceToHost, c->stream) !=
        cudaSuccess)
        return -1;
    return finish(c);
}

static int cuda_matmul_q4(att1_backend *b, float *dst, const float *lhs, size_t lhs_rows, size_t lhs_cols,
                          const att1_q4_matrix *w)
{
    cuda_backend *c = cb(b);
    const b2_dev_mat *m;
    if (dst == NULL || lhs == NULL || w == NULL || lhs_rows == 0 || lhs_cols == 0 || !q4_valid(w) ||
        lhs_cols != w->cols)
        return -1;
    if (!q4_unit_ok(w)) {
        const cached_mat *e = raw_weight(c, w->packed, w->packed, w->rows * w->cols / 2, w->scales,
                                         w->rows * (w->cols / w->group_size) * sizeof(float), w->rows, w->cols,
                                         w->group_size);
        return e == NULL ? -1 : run_ordered(c, e, 4, dst, lhs, lhs_rows);
    }
    m = q4_weight(c, w);
    if (m == NULL) return -1;
    return run_gemv(c, m, dst, lhs, lhs_rows, lhs_cols);
}

static int cuda_matmul_q8(att1_backend *b, float *dst, const float *lhs, size_t lhs_rows, size_t lhs_cols,
                          const att1_q8_matrix *w)
{
    cuda_backend *c = cb(b);
    const b2_dev_mat *m;
    if (dst == NULL || lhs == NULL || w == NULL || w->values == NULL || w->scales == NULL || lhs_rows == 0 ||
        lhs_cols == 0 || lhs_cols != w->cols || w->rows == 0 || w->rows > 0xFFFFFFFFu || w->cols > 0xFFFFFFFFu)
        return -1;
    if (w->cols % 32 != 0) {
        const cached_mat *e = raw_weight(c, w->values, w->values, w->rows * w->cols, w->scales,
                                         w->rows * sizeof(float), w->rows, w->cols, 0);
        return e == NULL ? -1 : run_ordered(c, e, 8, dst, lhs, lhs_rows);
    }
    m = q8_weight(c, w);
    if (m == NULL) return -1;
    return run_gemv(c, m, dst, lhs, lhs_rows, lhs_cols);
}

static int cuda_matmul_f32(att1_backend *b, float *dst, const float *lhs, const float *rhs, size_t rows, size_t cols,
                           size_t inner)
{
    cuda_backend *c = cb(b);
    if (dst == NULL || lhs == NULL || rhs == NULL || rows == 0 || cols == 0 || inner == 0) return -1;
    if (ensure(c, 0, rows * inner * 4) || ensure(c, 1, inner * cols * 4) || ensure(c, 2, rows * cols * 4)) return -1;
    if (cudaMemcpyAsync(c->buf[0], lhs, rows * inner * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
        cudaMemcpyAsync(c->buf[1], rhs, inner * cols * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        return -1;
    if (b2_matmul_f32(c->buf[2], c->buf[0], c->buf[1], (uint32_t)rows, (uint32_t)cols, (uint32_t)inner, c->stream) != 0)
        return -1;
    if (cudaMemcpyAsync(dst, c->buf[2], rows * cols * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess) return -1;
    return finish(c);
}

static int cuda_rmsnorm(att1_backend *b, float *dst, const float *src, const float *w, size_t n, float eps)
{
    cuda_backend *c = cb(b);
    if (dst == NULL || src == NULL || w == NULL || n == 0 || !(eps > 0.0f)) return -1;
    if (ensure(c, 0, n * 4) || ensure(c, 1, n * 4) || ensure(c, 2, n * 4)) return -1;
    if (cudaMemcpyAsync(c->buf[0], src, n * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
        cudaMemcpyAsync(c->buf[1], w, n * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        return -1;
    if (b2_rmsnorm(c->buf[2], c->buf[0], c->buf[1], (uint32_t)n, eps, c->stream) != 0) return -1;
    if (cudaMemcpyAsync(dst, c->buf[2], n * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess) return -1;
    return finish(c);
}

static int cuda_softmax(att1_backend *b, float *v, size_t n)
{
    cuda_backend *c = cb(b);
    if (v == NULL || n == 0) return -1;
    if (ensure(c, 0, n * 4)) return -1;
    if (cudaMemcpyAsync(c->buf[0], v, n * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess) return -1;
    if (b2_softmax(c->buf[0], (uint32_t)n, c->stream) != 0) return -1;
    if (cudaMemcpyAsync(v, c->buf[0], n * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess) return -1;
    return finish(c);
}

static int cuda_rope(att1_backend *b, float *v, size_t n, size_t pos, float theta)
{
    cuda_backend *c = cb(b);
    if (v == NULL || n == 0 || (n % 2) != 0 || !(theta > 0.0f) || pos > 0xFFFFFFFFu) return -1;
    if (ensure(c, 0, n * 4)) return -1;
    if (cudaMemcpyAsync(c->buf[0], v, n * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess) return -1;
    if (b2_rope(c->buf[0], (uint32_t)n, (uint32_t)pos, theta, c->stream) != 0) return -1;
    if (cudaMemcpyAsync(v, c->buf[0], n * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess) return -1;
    return finish(c);
}

static int cuda_swiglu(att1_backend *b, float *dst, const float *g, const float *u, size_t n)
{
    cuda_backend *c = cb(b);
    if (dst == NULL || g == NULL || u == NULL || n == 0) return -1;
    if (ensure(c, 0, n * 4) || ensure(c, 1, n * 4) || ensure(c, 2, n * 4)) return -1;
    if (cudaMemcpyAsync(c->buf[0], g, n * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
        cudaMemcpyAsync(c->buf[1], u, n * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        return -1;
    if (b2_swiglu(c->buf[2], c->buf[0], c->buf[1], (uint32_t)n, c->stream) != 0) return -1;
    if (cudaMemcpyAsync(dst, c->buf[2], n * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess) return -1;
    return finish(c);
}

static const att1_backend_ops cuda_f32_ops = {
    "cuda", cuda_alloc, cuda_free, cuda_sync, cuda_matmul_f32, NULL, NULL,
    cuda_rmsnorm, cuda_softmax, cuda_rope, cuda_swiglu};
static const att1_backend_ops cuda_q8_ops = {
    "cuda-q8", cuda_alloc, cuda_free, cuda_sync, cuda_matmul_f32, cuda_matmul_q8, NULL,
    cuda_rmsnorm, cuda_softmax, cuda_rope, cuda_swiglu};
static const att1_backend_ops cuda_q4_ops = {
    "cuda-q4", cuda_alloc, cuda_free, cuda_sync, cuda_matmul_f32, NULL, cuda_matmul_q4,
    cuda_rmsnorm, cuda_softmax, cuda_rope, cuda_swiglu};

int att1_backend_cuda_available(void)
{
    int n = 0, dev = 0, major = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return 0;
    }
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
        return 0;
    return major == 10;
}

static att1_status_t create(const att1_backend_ops *ops, att1_backend **out)
{
    att1_backend *b;
    cuda_backend *c;
    if (out == NULL) return ATT1_ERR_INVALID_ARG;
    *out = NULL;
    if (!att1_backend_cuda_available()) return ATT1_ERR_UNSUPPORTED;
    b = calloc(1, sizeof(*b));
    c = calloc(1, sizeof(*c));
    if (b == NULL || c == NULL) {
        free(b);
        free(c);
        return ATT1_ERR_OOM;
    }
    if (cudaGetDevice(&c->device) != cudaSuccess || cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc((void **)&c->err, sizeof(int32_t)) != cudaSuccess ||
        cudaMemsetAsync(c->err, 0, sizeof(int32_t), c->stream) != cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess ||
        cudaMalloc((void **)&c->key, sizeof(unsigned long long)) != cudaSuccess) {
        free(b);
        free(c);
        return ATT1_ERR_STATE;
    }
    b->ops = ops;
    b->user_data = c;
    *out = b;
    return ATT1_OK;
}

att1_status_t att1_backend_cuda_create(att1_backend **out) { return create(&cuda_f32_ops, out); }
att1_status_t att1_backend_cuda_q8_create(att1_backend **out) { return create(&cuda_q8_ops, out); }
att1_status_t att1_backend_cuda_q4_create(att1_backend **out) { return create(&cuda_q4_ops, out); }
att1_status_t att1_backend_default_create(att1_backend **out) { return create(&cuda_q4_ops, out); }

att1_status_t att1_backend_cuda_copy_host_to_device(att1_backend *b, void *dst, const void *src, size_t bytes)
{
    if (!b2_backend_is_cuda(b) || dst == NULL || src == NULL) return ATT1_ERR_INVALID_ARG;
    /* ordered with the backend's kernels, and on the device when this returns */
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, cb(b)->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(cb(b)->stream);
    return b2_cuda_status(e);
}

att1_status_t att1_backend_cuda_copy_device_to_host(att1_backend *b, void *dst, const void *src, size_t bytes)
{
    if (!b2_backend_is_cuda(b) || dst == NULL || src == NULL) return ATT1_ERR_INVALID_ARG;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, cb(b)->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(cb(b)->stream);
    return b2_cuda_status(e);
}

void att1_backend_destroy(att1_backend *b)
{
    size_t i;
    cuda_backend *c;
    if (b == NULL) return;
    if (b2_backend_is_cuda(b)) {
        c = cb(b);
        cudaStreamSynchronize(c->stream);
        for (i = 0; i < c->n_cache; i++) {
            if (c->cache[i].m.data) cudaFree(c->cache[i].m.data);
            if (c->cache[i].m.row_scale) cudaFree(c->cache[i].m.row_scale);
            if (c->cache[i].raw) cudaFree(c->cache[i].raw);
        }
        free(c->cache);
        for (i = 0; i < 3; i++)
            if (c->buf[i]) cudaFree(c->buf[i]);
        if (c->scratch) cudaFree(c->scratch);
        if (c->counters) cudaFree(c->counters);
        if (c->err) cudaFree(c->err);
        if (c->key) cudaFree(c->key);
        cudaStreamDestroy(c->stream);
        free(c);
    }
    free(b);
}
