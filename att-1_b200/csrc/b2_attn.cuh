// b2_attn.cuh - device side of single-query attention over the paged KV cache.
//
// Shared by the standalone attention kernel (b2_attn.cu) and the persistent
// decode kernel (b2_decode.cu). The algorithm notes are in b2_attn.cu.
#pragma once

#include "b2_common.cuh"

#include <cfloat>
#include <cuda_runtime.h>

namespace b2 {

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
    // page = [n_kv_heads][page_tokens][head_dim]: a head's tokens are contiguous
    const int32_t page = kv.page_table[(size_t)item * kv.pages_per_seq + pos / kv.page_tokens];
    return pool + (((size_t)page * kv.n_kv_heads + head) * kv.page_tokens + pos % kv.page_tokens) * kv.head_dim;
}

// Shared-memory view for one CTA of NW warps working on one (item, KV head,
// chunk): per-warp softmax state and the combine flag.
struct AttnSmem {
    float *wm;    // [NW][gs]
    float *wl;    // [NW][gs]
    float *wo;    // [NW][gs][wos]
    int *last;
    uint32_t gs;  // group stride (>= query heads per KV head)
    uint32_t wos; // dims per head held (4 * lanes per position)
};

__host__ __device__ constexpr size_t attn_smem_bytes(int lp, int nw, uint32_t gs)
{
    return (2 * (size_t)nw * gs + (size_t)nw * gs * 4 * lp) * sizeof(float) + 16;
}

template <int LP, int NW>
__device__ __forceinline__ AttnSmem attn_smem(uint8_t *base, uint32_t gs)
{
    AttnSmem s;
    s.gs = gs;
    s.wos = 4 * LP;
    s.wm = reinterpret_cast<float *>(base);
    s.wl = s.wm + NW * gs;
    s.wo = s.wl + NW * gs;
    s.last = reinterpret_cast<int *>(s.wo + NW * gs * 4 * LP);
    return s;
}

// Lanes per position for a head size: each lane holds 4 dimensions.
__host__ __device__ constexpr int attn_lanes(uint32_t hd) { return hd <= 32 ? 8 : (hd <= 64 ? 16 : 32); }

// Merge two online-softmax states (m, l, o) of the same query head.
__device__ __forceinline__ void soft_merge(float &m, float &l, float4 &o, float m2, float l2, float4 o2)
{
    const float M = fmaxf(m, m2);
    if (M == -INFINITY) return;  // both empty
    const float f1 = expf(m - M), f2 = expf(m2 - M);
    l = fmaf(l, f1, l2 * f2);
    o = make_float4(fmaf(o.x, f1, o2.x * f2), fmaf(o.y, f1, o2.y * f2), fmaf(o.z, f1, o2.z * f2),
                    fmaf(o.w, f1, o2.w * f2));
    m = M;
}

// Publish this chunk's partial (already stored at its slot of part_base) and,
// in the last chunk of an (item, KV head) to finish, combine all partials in
// chunk order into the context. `stage` holds at least 2 * nactive * group
// floats of shared memory; `last_flag` one int.
template <typename Sync>
__device__ void attn_publish(const AttnParams &p, float *stage, int *last_flag, uint32_t item, uint32_t kvh,
                             uint32_t nactive, const float *part_base, uint32_t nthreads, Sync SYNC)
{
    const uint32_t hd = p.head_dim, G = p.group;
    // publish the partial: one fence, by the thread that takes the ticket,
    // after the CTA barrier that orders every thread's stores before it
    SYNC();
    if (threadIdx.x == 0) {
        int *cnt = p.counters + item * p.n_kv_heads + kvh;
        __threadfence();
        const int last = (atomicAdd(cnt, 1) == (int)nactive - 1);
        if (last) {
            *cnt = 0;
            __threadfence();
        }
        *last_flag = last;
    }
    SYNC();
    const int last = *last_flag;
    if (!last) {
        SYNC();  // the flag may be rewritten by the next chunk of this CTA
        return;
    }
    // final combine over chunks, in chunk order: first the (max, sum) of every
    // chunk and query head, loaded in parallel into shared memory (the warp
    // state area is free now), then each output element
    float *cm = stage;                   // [nactive][G] maxima
    float *cl = stage + nactive * G;     // [nactive][G] sums
    for (uint32_t i = threadIdx.x; i < nactive * G; i += nthreads) {
        const uint32_t c = i / G, gq = i % G;
        const float *pc = part_base + (size_t)c * G * (hd + 2) + gq * (hd + 2);
        cm[i] = ld_cg(pc);
        cl[i] = ld_cg(pc + 1);
    }
    SYNC();
    for (uint32_t i = threadIdx.x; i < G * hd; i += nthreads) {
        const uint32_t gq = i / hd, d = i % hd;
        float M = -INFINITY;
        for (uint32_t c = 0; c < nactive; ++c) M = fmaxf(M, cm[c * G + gq]);
        float L = 0.0f, O = 0.0f;
#pragma unroll 8
        for (uint32_t c = 0; c < nactive; ++c) {
            const float f = expf(cm[c * G + gq] - M);
            L = fmaf(cl[c * G + gq], f, L);
            O = fmaf(ld_cg(part_base + (size_t)c * G * (hd + 2) + gq * (hd + 2) + 2 + d), f, O);
        }
        p.ctx[(size_t)item * p.n_heads * hd + (size_t)(kvh * G + gq) * hd + d] = __fdiv_rn(O, L);
    }
    SYNC();  // shared state is reused by the next chunk of this CTA
}

// One (item, KV head, chunk) of the attention: positions [p0, p1) of the
// chunk, `nactive` chunks for this (item, KV head). The NW warps of the CTA
// (threads 0 .. 32*NW-1) take part; SYNC() is their barrier. A warp covers
// 32/LP positions at a time, LP lanes per position with four dimensions
// each (one 16-byte load per lane for a K or V row), and keeps an online
// softmax per query head in every lane group; the groups and then the warps
// are merged. Writes the chunk's (max, sum, weighted V) partial; the last
// chunk to finish combines all partials in chunk order and writes the context.
template <int LP, int MG, int NW, typename Sync>
__device__ void attn_chunk(const AttnParams &p, const AttnSmem &sm, uint32_t item, uint32_t kvh, uint32_t chunk,
                           uint32_t nactive, uint32_t p0, uint32_t p1, Sync SYNC)
{
    constexpr int PPW = 32 / LP;  // positions per warp step
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane / LP, sl = lane % LP;
    const uint32_t nthreads = NW * 32;
    const uint32_t hd = p.head_dim, G = p.group;
    const uint32_t d0 = 4 * sl;
    const bool dval = d0 < hd;

    // this lane's four dimensions of q for the G query heads of the KV head
    float4 qv[MG];
#pragma unroll
    for (int gq = 0; gq < MG; ++gq) {
        qv[gq] = make_float4(0, 0, 0, 0);
        if (gq < (int)G && dval)
            qv[gq] = __ldcg(reinterpret_cast<const float4 *>(p.q + (size_t)item * p.n_heads * hd +
                                                             (size_t)(kvh * G + gq) * hd + d0));
    }
    float m[MG], l[MG];
    float4 o[MG];
#pragma unroll
    for (int gq = 0; gq < MG; ++gq) {
        m[gq] = -INFINITY;
        l[gq] = 0.0f;
        o[gq] = make_float4(0, 0, 0, 0);
    }

    constexpr int U = kPosPerIter;        // positions per lane group per iteration
    const uint32_t step = NW * PPW;       // positions between a lane group's consecutive positions
    // warp-uniform trip count (the reductions below shuffle across the warp)
    for (uint32_t wb = p0 + warp * PPW; wb < p1; wb += step * U) {
        const uint32_t pb = wb + sub;
        float4 kd[U], vd[U];
#pragma unroll
        for (int j = 0; j < U; ++j) {
            const uint32_t ps = pb + j * step;
            kd[j] = vd[j] = make_float4(0, 0, 0, 0);
            if (ps < p1 && dval) {
                kd[j] = __ldcg(reinterpret_cast<const float4 *>(kv_row(p.kv, p.kv.k_pool, item, ps, kvh) + d0));
                vd[j] = __ldcg(reinterpret_cast<const float4 *>(kv_row(p.kv, p.kv.v_pool, item, ps, kvh) + d0));
            }
        }
#pragma unroll
        for (int j = 0; j < U; ++j) {
            const bool valid = pb + j * step < p1;
#pragma unroll
            for (int gq = 0; gq < MG; ++gq) {
                if (gq < (int)G) {
                    float dot = qv[gq].x * kd[j].x + qv[gq].y * kd[j].y + qv[gq].z * kd[j].z + qv[gq].w * kd[j].w;
#pragma unroll
                    for (int off = LP / 2; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
                    if (valid) {
                        const float sc = __fmul_rn(dot, p.inv_sqrt);  // src/attention.c:521-523
                        const float nm = fmaxf(m[gq], sc);
                        const float corr = expf(m[gq] - nm);
                        const float pr = expf(sc - nm);
                        l[gq] = fmaf(l[gq], corr, pr);
                        o[gq] = make_float4(fmaf(o[gq].x, corr, pr * vd[j].x), fmaf(o[gq].y, corr, pr * vd[j].y),
                                            fmaf(o[gq].z, corr, pr * vd[j].z), fmaf(o[gq].w, corr, pr * vd[j].w));
                        m[gq] = nm;
                    }
                }
            }
        }
    }
    // merge the lane groups of the warp (positions differ, dimensions match)
#pragma unroll
    for (int off = LP; off < 32; off <<= 1) {
#pragma unroll
        for (int gq = 0; gq < MG; ++gq) {
            const float m2 = __shfl_xor_sync(0xffffffffu, m[gq], off);
            const float l2 = __shfl_xor_sync(0xffffffffu, l[gq], off);
            float4 o2;
            o2.x = __shfl_xor_sync(0xffffffffu, o[gq].x, off);
            o2.y = __shfl_xor_sync(0xffffffffu, o[gq].y, off);
            o2.z = __shfl_xor_sync(0xffffffffu, o[gq].z, off);
            o2.w = __shfl_xor_sync(0xffffffffu, o[gq].w, off);
            soft_merge(m[gq], l[gq], o[gq], m2, l2, o2);
        }
    }
    // combine the warps of this CTA
#pragma unroll
    for (int gq = 0; gq < MG; ++gq) {
        if (gq < (int)G && sub == 0) {
            if (sl == 0) {
                sm.wm[warp * sm.gs + gq] = m[gq];
                sm.wl[warp * sm.gs + gq] = l[gq];
            }
            if (dval) *reinterpret_cast<float4 *>(sm.wo + (warp * sm.gs + gq) * sm.wos + d0) = o[gq];
        }
    }
    SYNC();
    float *part_base = p.partial + ((size_t)(item * p.n_kv_heads + kvh) * p.nchunks_max) * G * (hd + 2);
    for (uint32_t i = threadIdx.x; i < G * (hd + 2); i += nthreads) {
        const uint32_t gq = i / (hd + 2), d = i % (hd + 2);
        float M = -INFINITY;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, sm.wm[w * sm.gs + gq]);
        float v = 0.0f;
        if (d == 0) {
            v = M;
        } else {
            for (int w = 0; w < NW; ++w) {
                const float wmv = sm.wm[w * sm.gs + gq];
                if (wmv == -INFINITY) continue;  // warp saw no position
                const float f = expf(wmv - M);
                v = fmaf(d == 1 ? sm.wl[w * sm.gs + gq] : sm.wo[(w * sm.gs + gq) * sm.wos + d - 2], f, v);
            }
        }
        part_base[(size_t)chunk * G * (hd + 2) + i] = v;
    }
    attn_publish(p, sm.wo, sm.last, item, kvh, nactive, part_base, nthreads, SYNC);
}

// ---- host side (b2_attn.cu) ---------------------------------------------------------
// Argument checks of b2_attn (0 or a negative status).
int attn_check(const b2_attn_args *a);
// Kernel parameters from checked arguments (scratch and counters from `a`).
void attn_params(const b2_attn_args *a, uint32_t nchunks_max, AttnParams &p);

}  // namespace b2
