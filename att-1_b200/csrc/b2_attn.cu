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
#include "b2_common.cuh"

#include <cfloat>
#include <cuda_runtime.h>

namespace b2 {

constexpr int kAttnWarps = 8;
constexpr int kPosPerIter = 4;   // positions a warp loads before reducing
constexpr uint32_t kChunk = 128;
constexpr int kMaxGroup = 8;     // query heads per KV head

struct AttnParams {
    uint32_t batch, n_heads, n_kv_heads, head_dim, group, nchunks_max, max_ctx;
    const float *q;
    b2_kv_layout kv;
    const int32_t *positions;
    float *ctx;
    float *partial;  // [batch][n_kv][nchunks_max][group][head_dim + 2]
    int *counters;   // [batch][n_kv]
    float inv_sqrt;
    int32_t *err;
};

__device__ __forceinline__ const float *kv_row(const b2_kv_layout &kv, const float *pool, uint32_t item, uint32_t pos,
                                              uint32_t head)
{
    const int32_t page = kv.page_table[(size_t)item * kv.pages_per_seq + pos / kv.page_tokens];
    const size_t slot = (size_t)page * kv.page_tokens + pos % kv.page_tokens;
    return pool + (slot * kv.n_kv_heads + head) * kv.head_dim;
}

template <int DPL>  // dims per lane = ceil(head_dim / 32)
__global__ void __launch_bounds__(kAttnWarps * 32) attn_kernel(const AttnParams p)
{
    const uint32_t chunk = blockIdx.x, kvh = blockIdx.y, item = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t hd = p.head_dim, G = p.group;
    __shared__ float q_s[kMaxGroup * 32 * DPL];
    __shared__ float wm[kAttnWarps][kMaxGroup], wl[kAttnWarps][kMaxGroup];
    __shared__ float wo[kAttnWarps][kMaxGroup][32 * DPL];
    __shared__ int last_s;

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

    // q of the G query heads of this KV head
    for (uint32_t i = threadIdx.x; i < G * hd; i += blockDim.x) {
        const uint32_t gq = i / hd, d = i % hd;
        q_s[gq * 32 * DPL + d] = __ldcg(p.q + (size_t)item * p.n_heads * hd + (size_t)(kvh * G + gq) * hd + d);
    }
    __syncthreads();

    float m[kMaxGroup], l[kMaxGroup], o[kMaxGroup][DPL];
#pragma unroll
    for (int gq = 0; gq < kMaxGroup; ++gq) {
        m[gq] = -INFINITY;
        l[gq] = 0.0f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) o[gq][i] = 0.0f;
    }

    for (uint32_t pb = p0 + warp * kPosPerIter; pb < p1; pb += kAttnWarps * kPosPerIter) {
        float kd[kPosPerIter][DPL], vd[kPosPerIter][DPL];
#pragma unroll
        for (int j = 0; j < kPosPerIter; ++j) {
            const uint32_t ps = pb + j;
            const bool in = ps < p1;
            const float *kr = in ? kv_row(p.kv, p.kv.k_pool, item, ps, kvh) : nullptr;
            const float *vr = in ? kv_row(p.kv, p.kv.v_pool, item, ps, kvh) : nullptr;
#pragma unroll
            for (int i = 0; i < DPL; ++i) {
                const uint32_t d = lane + 32 * i;
                kd[j][i] = (in && d < hd) ? __ldcg(kr + d) : 0.0f;
                vd[j][i] = (in && d < hd) ? __ldcg(vr + d) : 0.0f;
            }
        }
#pragma unroll
        for (int j = 0; j < kPosPerIter; ++j) {
            if (pb + j >= p1) break;
#pragma unroll
            for (int gq = 0; gq < kMaxGroup; ++gq) {
                if (gq < (int)G) {
                    float dot = 0.0f;
#pragma unroll
                    for (int i = 0; i < DPL; ++i) {
                        // q_s beyond head_dim is never written: do not read it
                        const float qv = (lane + 32 * i < (int)hd) ? q_s[gq * 32 * DPL + lane + 32 * i] : 0.0f;
                        dot = fmaf(qv, kd[j][i], dot);
                    }
                    dot = warp_sum(dot);
                    const float s = __fmul_rn(dot, p.inv_sqrt);  // src/attention.c:521-523
                    const float nm = fmaxf(m[gq], s);
                    const float corr = expf(m[gq] - nm);
                    const float pr = expf(s - nm);
                    l[gq] = fmaf(l[gq], corr, pr);
#pragma unroll
                    for (int i = 0; i < DPL; ++i) o[gq][i] = fmaf(o[gq][i], corr, pr * vd[j][i]);
                    m[gq] = nm;
                }
            }
        }
    }
    // combine the warps of this CTA
#pragma unroll
    for (int gq = 0; gq < kMaxGroup; ++gq) {
        if (gq < (int)G) {
            if (lane == 0) {
                wm[warp][gq] = m[gq];
                wl[warp][gq] = l[gq];
            }
#pragma unroll
            for (int i = 0; i < DPL; ++i) wo[warp][gq][lane + 32 * i] = o[gq][i];
        }
    }
    __syncthreads();
    float *part_base = p.partial + ((size_t)(item * p.n_kv_heads + kvh) * p.nchunks_max) * G * (hd + 2);
    for (uint32_t i = threadIdx.x; i < G * (hd + 2); i += blockDim.x) {
        const uint32_t gq = i / (hd + 2), d = i % (hd + 2);
        float M = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w][gq]);
        float v = 0.0f;
        if (d == 0) {
            v = M;
        } else {
            for (int w = 0; w < kAttnWarps; ++w) {
                if (wm[w][gq] == -INFINITY) continue;  // warp saw no position
                const float f = expf(wm[w][gq] - M);
                v = fmaf(d == 1 ? wl[w][gq] : wo[w][gq][d - 2], f, v);
            }
        }
        part_base[(size_t)chunk * G * (hd + 2) + i] = v;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        int *cnt = p.counters + item * p.n_kv_heads + kvh;
        last_s = (atomicAdd(cnt, 1) == (int)nactive - 1);
        if (last_s) *cnt = 0;
    }
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    // final combine over chunks, in chunk order
    for (uint32_t i = threadIdx.x; i < G * hd; i += blockDim.x) {
        const uint32_t gq = i / hd, d = i % hd;
        float M = -INFINITY;
        for (uint32_t c = 0; c < nactive; ++c) M = fmaxf(M, ld_cg(part_base + (size_t)c * G * (hd + 2) + gq * (hd + 2)));
        float L = 0.0f, O = 0.0f;
        for (uint32_t c = 0; c < nactive; ++c) {
            const float *pc = part_base + (size_t)c * G * (hd + 2) + gq * (hd + 2);
            const float f = expf(ld_cg(pc) - M);
            L = fmaf(ld_cg(pc + 1), f, L);
            O = fmaf(ld_cg(pc + 2 + d), f, O);
        }
        p.ctx[(size_t)item * p.n_heads * hd + (size_t)(kvh * G + gq) * hd + d] = __fdiv_rn(O, L);
    }
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

}  // namespace b2

using namespace b2;

static void attn_sizes(const b2_attn_args *a, uint32_t &nchunks, size_t &partial, uint32_t &counters)
{
    nchunks = (a->max_ctx + kChunk - 1) / kChunk;
    const uint32_t G = a->n_heads / a->n_kv_heads;
    partial = (size_t)a->batch * a->n_kv_heads * nchunks * G * (a->head_dim + 2) * sizeof(float);
    partial = (partial + 255) & ~(size_t)255;
    counters = a->batch * a->n_kv_heads;
}

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
    uint32_t nchunks, cl;
    size_t pb;
    attn_sizes(a, nchunks, pb, cl);
    if (a->scratch == nullptr || a->scratch_bytes < pb || ((uintptr_t)a->scratch & 255)) return -1;
    if (a->counters == nullptr || a->counters_len < cl) return -1;
    AttnParams p = {};
    p.batch = a->batch;
    p.n_heads = a->n_heads;
    p.n_kv_heads = a->n_kv_heads;
    p.head_dim = a->head_dim;
    p.group = G;
    p.nchunks_max = nchunks;
    p.max_ctx = a->max_ctx;
    p.q = a->q;
    p.kv = kv;
    p.positions = a->positions;
    p.ctx = a->ctx;
    p.partial = (float *)a->scratch;
    p.counters = (int *)a->counters;
    p.inv_sqrt = 1.0f / sqrtf((float)a->head_dim);  // src/attention.c:512
    p.err = a->err;
    const cudaError_t e = launch_attn(p, dim3(nchunks, a->n_kv_heads, a->batch), a->pdl, (cudaStream_t)stream);
    return e == cudaSuccess ? 0 : -8;
}
