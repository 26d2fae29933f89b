// b2_attn.cu - single-query attention over the paged KV cache.
//
// Replaces the per-head host loops of src/attention.c:508-541 (scores =
// q.k * 1/sqrt(hd), softmax of src/norm.c:36-71, context = sum p * v) for one
// decoded token per sequence. The KV pages use the KV-MMU page layout
// [token_in_page][head][head_dim] (src/kv_mmu.c:95-101) with n_kv_heads heads;
// the H/Hkv query heads of a KV head share every K/V read (grouped-query
// attention; the reference reaches the same numbers with expanded heads).
//
// Work split: CTA (chunk, kv head, item) covers kChunk positions; eight warps
// take four positions at a time (all K/V loads of the four issued together)
// and keep an online softmax per query head. Each CTA writes its
// (max, sum, weighted V) partial; the last CTA of a (item, kv head) to arrive
// combines the partials in chunk order (deterministic) and writes the context.
#include "b2_attn.cuh"

namespace b2 {

constexpr int kAttnWarps = 8;

struct CtaSync {
    __device__ void operator()() const { __syncthreads(); }
};

template <int DPL>  // dims per lane = ceil(head_dim / 32)
__global__ void __launch_bounds__(kAttnWarps * 32) attn_kernel(const AttnParams p)
{
    const uint32_t chunk = blockIdx.x, kvh = blockIdx.y, item = blockIdx.z;
    __shared__ __align__(16) uint8_t smem[attn_smem_bytes(DPL, kAttnWarps, kMaxGroup)];
    pdl_wait();
    pdl_launch_dependents();
    // positions beyond max_ctx would need more chunks than the grid has
    const int32_t pos = p.positions[item];
    if (pos < 0 || (uint32_t)pos >= p.max_ctx) {
        if (threadIdx.x == 0 && chunk == 0 && kvh == 0) raise_error(p.err, B2_ERR_POSITION);
        return;
    }
    const uint32_t len = (uint32_t)pos + 1;
    const uint32_t nactive = (len + kChunk - 1) / kChunk;
    if (chunk >= nactive) return;
    const uint32_t p0 = chunk * kChunk, p1 = min(p0 + kChunk, len);
    attn_chunk<DPL, kAttnWarps>(p, attn_smem<DPL, kAttnWarps>(smem, kMaxGroup), item, kvh, chunk, nactive, p0, p1, CtaSync());
}

static cudaError_t launch_attn(const AttnParams &p, dim3 grid, int pdl, cudaStream_t st)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kAttnWarps * 32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const uint32_t dpl = (p.head_dim + 31) / 32;
    switch (dpl) {
    case 1: return cudaLaunchKernelEx(&cfg, attn_kernel<1>, p);
    case 2: return cudaLaunchKernelEx(&cfg, attn_kernel<2>, p);
    case 3: return cudaLaunchKernelEx(&cfg, attn_kernel<3>, p);
    case 4: return cudaLaunchKernelEx(&cfg, attn_kernel<4>, p);
    default: return cudaErrorInvalidValue;
    }
}


static void attn_sizes(const b2_attn_args *a, uint32_t &nchunks, size_t &partial, uint32_t &counters)
{
    nchunks = (a->max_ctx + kChunk - 1) / kChunk;
    const uint32_t G = a->n_heads / a->n_kv_heads;
    partial = (size_t)a->batch * a->n_kv_heads * nchunks * G * (a->head_dim + 2) * sizeof(float);
    partial = (partial + 255) & ~(size_t)255;
    counters = a->batch * a->n_kv_heads;
}

int attn_check(const b2_attn_args *a)
{
    if (a == nullptr || a->q == nullptr || a->ctx == nullptr || a->positions == nullptr) return -1;
    if (a->batch == 0 || a->n_kv_heads == 0 || a->n_heads % a->n_kv_heads || a->head_dim == 0 ||
        a->head_dim > 32 * 4 || a->max_ctx == 0)
        return -1;
    const uint32_t G = a->n_heads / a->n_kv_heads;
    if (G > (uint32_t)kMaxGroup) return -9;
    const b2_kv_layout &kv = a->kv;
    if (!kv.k_pool || !kv.v_pool || !kv.page_table || kv.page_tokens == 0 || kv.head_dim != a->head_dim ||
        kv.n_kv_heads != a->n_kv_heads || a->max_ctx > kv.page_tokens * kv.pages_per_seq)
        return -1;
    // the chunk combine stages (max, sum) of every chunk and query head in the
    // warp-state area of the standalone kernel
    const uint32_t nchunks = (a->max_ctx + kChunk - 1) / kChunk, dpl = (a->head_dim + 31) / 32;
    if (2ull * nchunks * G > 8ull * kMaxGroup * 32 * dpl) return -9;
    return 0;
}

void attn_params(const b2_attn_args *a, uint32_t nchunks_max, AttnParams &p)
{
    p = AttnParams{};
    p.batch = a->batch;
    p.n_heads = a->n_heads;
    p.n_kv_heads = a->n_kv_heads;
    p.head_dim = a->head_dim;
    p.group = a->n_heads / a->n_kv_heads;
    p.nchunks_max = nchunks_max;
    p.max_ctx = a->max_ctx;
    p.q = a->q;
    p.kv = a->kv;
    p.positions = a->positions;
    p.ctx = a->ctx;
    p.partial = (float *)a->scratch;
    p.counters = (int *)a->counters;
    p.inv_sqrt = 1.0f / sqrtf((float)a->head_dim);  // src/attention.c:512
    p.err = a->err;
}

}  // namespace b2

using namespace b2;

extern "C" size_t b2_attn_scratch_bytes(const b2_attn_args *a)
{
    if (a == nullptr || a->n_kv_heads == 0 || a->batch == 0) return 0;
    uint32_t n, cl;
    size_t pb;
    attn_sizes(a, n, pb, cl);
    return pb;
}

extern "C" uint32_t b2_attn_counters_len(const b2_attn_args *a)
{
    if (a == nullptr || a->n_kv_heads == 0 || a->batch == 0) return 0;
    uint32_t n, cl;
    size_t pb;
    attn_sizes(a, n, pb, cl);
    return cl;
}

extern "C" int b2_attn(const b2_attn_args *a, void *stream)
{
    const int rc = attn_check(a);
    if (rc != 0) return rc;
    uint32_t nchunks, cl;
    size_t pb;
    attn_sizes(a, nchunks, pb, cl);
    if (a->scratch == nullptr || a->scratch_bytes < pb || ((uintptr_t)a->scratch & 255)) return -1;
    if (a->counters == nullptr || a->counters_len < cl) return -1;
    AttnParams p;
    attn_params(a, nchunks, p);
    const cudaError_t e = launch_attn(p, dim3(nchunks, a->n_kv_heads, a->batch), a->pdl, (cudaStream_t)stream);
    return e == cudaSuccess ? 0 : -8;
}
