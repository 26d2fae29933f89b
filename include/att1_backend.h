/*
 * att1_backend.h - the ATT-1 backend vtable, served by the B200 device.
 *
 * Interface of ATT-1's include/att1_backend.h:18-74 (same struct layout,
 * names, argument meaning and 0/-1 return convention of the ops). The
 * inference code of the reference routes by ops->name: "cuda-q4" reaches the
 * q4 path and "cuda-q8" the q8 path (src/infer.c:143-159).
 *
 * Pointers passed to the ops are HOST pointers, as in the reference
 * (src/attention.c dereferences backend buffers directly): alloc returns
 * pinned host memory, each op copies its operands to the device, runs one
 * sm_100a kernel and copies the result back. Weight matrices are uploaded
 * and converted to the device layout on first use and cached, keyed by their
 * packed-data pointer (views into a loaded model are stable for its life).
 * The per-op path exists for drop-in compatibility; full-speed decode runs
 * device-resident behind att1_infer_* / att1_cluster_infer_*.
 */
#ifndef ATT1_BACKEND_H
#define ATT1_BACKEND_H

#include "att1_quant.h"
#include "att1_status.h"

#include <stddef.h>
#include <stdint.h>

typedef struct att1_backend att1_backend;

typedef struct att1_backend_ops {
    const char *name;

    void *(*alloc)(att1_backend *backend, size_t bytes);
    void (*free)(att1_backend *backend, void *ptr);
    int (*sync)(att1_backend *backend);

    int (*matmul_f32)(att1_backend *backend, float *dst, const float *lhs,
                      const float *rhs, size_t rows, size_t cols, size_t inner);
    int (*matmul_q8xf32)(att1_backend *backend, float *dst, const float *lhs,
                         size_t lhs_rows, size_t lhs_cols,
                         const att1_q8_matrix *weights);
    int (*matmul_q4xf32)(att1_backend *backend, float *dst, const float *lhs,
                         size_t lhs_rows, size_t lhs_cols,
                         const att1_q4_matrix *weights);
    int (*rmsnorm_f32)(att1_backend *backend, float *dst, const float *src,
                       const float *weight, size_t count, float epsilon);
    int (*softmax_f32)(att1_backend *backend, float *values, size_t count);
    int (*rope_f32)(att1_backend *backend, float *values, size_t count,
                    size_t position, float theta);
    int (*ffn_swiglu_f32)(att1_backend *backend, float *dst, const float *gate,
                          const float *value, size_t count);
} att1_backend_ops;

struct att1_backend {
    const att1_backend_ops *ops;
    void *user_data;
};

/* 1 when a CUDA device of compute capability 10.x is present. */
int att1_backend_cuda_available(void);
/* "cuda" (f32), "cuda-q8" and "cuda-q4" backends on the current device. */
att1_status_t att1_backend_cuda_create(att1_backend **out_backend);
att1_status_t att1_backend_cuda_q8_create(att1_backend **out_backend);
att1_status_t att1_backend_cuda_q4_create(att1_backend **out_backend);
/* Raw copies between host memory and device memory of the backend's device. */
att1_status_t att1_backend_cuda_copy_host_to_device(att1_backend *backend,
                                                    void *device_dst,
                                                    const void *host_src,
                                                    size_t bytes);
att1_status_t att1_backend_cuda_copy_device_to_host(att1_backend *backend,
                                                    void *host_dst,
                                                    const void *device_src,
                                                    size_t bytes);
/* The default backend of this library is "cuda-q4". */
att1_status_t att1_backend_default_create(att1_backend **out_backend);
void att1_backend_destroy(att1_backend *backend);

#endif
