/*
 * att1_nccl.c - the NCCL collectives of the tensor-parallel comparison arm.
 *
 * The tensor-parallel step exchanges partial sums inside its own kernels over
 * peer memory. For comparison the same step can run with the two per-layer
 * all-reduces and the logits all-gather as NCCL collectives on the step's
 * stream (captured into its CUDA graph). NCCL is loaded at run time
 * (libnccl.so.2: the copy a process already has, e.g. torch's, is reused), so
 * the library neither links nor needs it unless this arm is asked for.
 */
#define _GNU_SOURCE
#include "b2_host.h"

#include <dlfcn.h>
#include <nccl.h>
#include <pthread.h>
#include <string.h>

typedef struct nccl_api {
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
} nccl_api;

static nccl_api g_nccl;
static int g_nccl_ok;
static pthread_once_t g_nccl_once = PTHREAD_ONCE_INIT;

static void nccl_load(void)
{
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == NULL) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (h == NULL) return;
    *(void **)&g_nccl.get_unique_id = dlsym(h, "ncclGetUniqueId");
    *(void **)&g_nccl.comm_init_rank = dlsym(h, "ncclCommInitRank");
    *(void **)&g_nccl.comm_destroy = dlsym(h, "ncclCommDestroy");
    *(void **)&g_nccl.all_reduce = dlsym(h, "ncclAllReduce");
    *(void **)&g_nccl.all_gather = dlsym(h, "ncclAllGather");
    g_nccl_ok = g_nccl.get_unique_id && g_nccl.comm_init_rank && g_nccl.comm_destroy && g_nccl.all_reduce &&
                g_nccl.all_gather;
}

int b2_nccl_available(void)
{
    pthread_once(&g_nccl_once, nccl_load);
    return g_nccl_ok;
}

int b2_nccl_unique_id(void *id)
{
    ncclUniqueId u;
    if (id == NULL || !b2_nccl_available() || g_nccl.get_unique_id(&u) != ncclSuccess) return -1;
    memcpy(id, &u, sizeof(u));
    return 0;
}

int b2_nccl_comm_init(void **comm, int world, const void *id, int rank)
{
    ncclUniqueId u;
    ncclComm_t c = NULL;
    if (comm == NULL || id == NULL || !b2_nccl_available()) return -1;
    memcpy(&u, id, sizeof(u));
    if (g_nccl.comm_init_rank(&c, world, u, rank) != ncclSuccess) return -1;
    *comm = c;
    return 0;
}

void b2_nccl_comm_destroy(void *comm)
{
    if (comm != NULL && b2_nccl_available()) g_nccl.comm_destroy((ncclComm_t)comm);
}

int b2_nccl_allreduce_sum_f32(float *buf, size_t count, void *comm, cudaStream_t st)
{
    return g_nccl.all_reduce(buf, buf, count, ncclFloat32, ncclSum, (ncclComm_t)comm, st) == ncclSuccess ? 0 : -8;
}

int b2_nccl_allgather(const void *send, void *recv, size_t bytes_per_rank, void *comm, cudaStream_t st)
{
    return g_nccl.all_gather(send, recv, bytes_per_rank, ncclUint8, (ncclComm_t)comm, st) == ncclSuccess ? 0 : -8;
}
