/*
 * b2_host.h - internal declarations shared by the host C files.
 */
#ifndef B2_HOST_H
#define B2_HOST_H

#include "att1_b200.h"
#include "att1_backend.h"
#include "b2_kernels.h"

#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

/* one quantised matrix on the device */
typedef struct b2_dev_mat {
    void *data;
    float *row_scale;   /* q8 only */
    b2_qweight w;
} b2_dev_mat;

/* backend internals shared with the infer context (set_backend routing) */
int b2_backend_is_cuda(const att1_backend *backend);
const char *b2_backend_name(const att1_backend *backend);

/* KV-MMU hooks for a decode context whose batch items are sessions
 * (att1_kv_mmu.c; att1_b200_infer_use_kv_mmu) */
int b2_kv_mmu_session_slot(const att1_kv_mmu *mmu, uint64_t session_id, size_t *slot);
size_t b2_kv_mmu_length(const att1_kv_mmu *mmu, size_t slot, size_t layer);
const att1_kv_mmu_config *b2_kv_mmu_config(const att1_kv_mmu *mmu);
att1_status_t b2_kv_mmu_reserve(att1_kv_mmu *mmu, size_t slot, size_t first, size_t count);
void b2_kv_mmu_advance(att1_kv_mmu *mmu, size_t slot, size_t count);
const int32_t *b2_kv_mmu_row(const att1_kv_mmu *mmu, size_t slot, size_t layer, size_t *pages_per_seq);

/* NCCL collectives of the tensor-parallel comparison arm (att1_nccl.c; NCCL is
 * loaded at run time) */
int b2_nccl_available(void);
int b2_nccl_unique_id(void *id);
int b2_nccl_comm_init(void **comm, int world, const void *id, int rank);
void b2_nccl_comm_destroy(void *comm);
int b2_nccl_allreduce_sum_f32(float *buf, size_t count, void *comm, cudaStream_t st);
int b2_nccl_allgather(const void *send, void *recv, size_t bytes_per_rank, void *comm, cudaStream_t st);

/* status of a CUDA runtime call */
static inline att1_status_t b2_cuda_status(cudaError_t e)
{
    if (e == cudaSuccess) return ATT1_OK;
    if (e == cudaErrorMemoryAllocation) return ATT1_ERR_OOM;
    return ATT1_ERR_STATE;
}

/* status of a b2_* kernel entry point (0 or a negative att1 code) */
static inline att1_status_t b2_status(int rc)
{
    return rc == 0 ? ATT1_OK : (att1_status_t)rc;
}

#endif
