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
    const int32_t page = kv.page_table[(size_t)item * kv.pages_per_seq + pos / kv.page_tokens];
    const size_t slot = (size_t)page * kv.page_tokens + pos % kv.page_tokens;
    return pool + (slot * kv.n_kv_heads + head) * kv.head_dim;
}

// Shared-memory view for one CTA of NW warps working on one (item, KV head,
// chunk): q of the group, per-warp softmax state, and the combine flag.
struct AttnSmem {
    float *q_s;   // [gs][32 * DPL]
    float *wm;    // [NW][gs]
    float *wl;    // [NW][gs]
    float *wo;    // [NW][gs][32 * DPL]
    int *last;
    uint32_t gs;  // group stride (>= query heads per KV head)
};

__host__ __device__ constexpr size_t attn_smem_bytes(int dpl, int nw, uint32_t gs)
{
    return ((size_t)gs * 32 * dpl + 2 * (size_t)nw * gs + (size_t)nw * gs * 32 * dpl) * sizeof(float) + 16;
}

template <int DPL, int NW>
__device__ __forceinline__ AttnSmem attn_smem(uint8_t *base, uint32_t gs)
{
    AttnSmem s;
    s.gs = gs;
    s.q_s = reinterpret_cast<float *>(base);
    s.wm = s.q_s + gs * 32 * DPL;
    s.wl = s.wm + NW * gs;
    s.wo = s.wl + NW * gs;
    s.last = reinterpret_cast<int *>(s.wo + NW * gs * 32 * DPL);
    return s;
}

// One (item, KV head, chunk) of the attention: positions [p0, p1) of the
// chunk, `nactive` chunks for this (item, KV head). The NW warps of the CTA
// (threads 0 .. 32*NW-1) take part; SYNC() is their barrier. Writes the
// chunk's (max, sum, weighted V) partial; the last chunk to finish combines
// all partials in chunk order and writes the context.
template <int DPL, int NW, typename Sync>
__device__ void attn_chunk(const AttnParams &p, const AttnSmem &sm, uint32_t item, uint32_t kvh, uint32_t chunk,
                           uint32_t nactive, uint32_t p0, uint32_t p1, Sync SYNC)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t nthreads = NW * 32;
    const uint32_t hd = p.head_dim, G = p.group;

    // q of the G query heads of this KV head
    for (uint32_t i = threadIdx.x; i < G * hd; i += nthreads) {
        const uint32_t gq = i / hd, d = i % hd;
        sm.q_s[gq * 32 * DPL + d] = __ldcg(p.q + (size_t)item * p.n_heads * hd + (size_t)(kvh * G + gq) * hd + d);
    }
    SYNC();

    float m[kMaxGroup], l[kMaxGroup], o[kMaxGroup][DPL];
#pragma unroll
    for (int gq = 0; gq < kMaxGroup; ++gq) {
        m[gq] = -INFINITY;
        l[gq] = 0.0f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) o[gq][i] = 0.0f;
    }

    for (uint32_t pb = p0 + warp * kPosPerIter; pb < p1; pb += NW * kPosPerIter) {
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
                        const float qv = (lane + 32 * i < (int)hd) ? sm.q_s[gq * 32 * DPL + lane + 32 * i] : 0.0f;
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
                sm.wm[warp * sm.gs + gq] = m[gq];
                sm.wl[warp * sm.gs + gq] = l[gq];
            }
#pragma unroll
            for (int i = 0; i < DPL; ++i) sm.wo[(warp * sm.gs + gq) * 32 * DPL + lane + 32 * i] = o[gq][i];
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
                v = fmaf(d == 1 ? sm.wl[w * sm.gs + gq] : sm.wo[(w * sm.gs + gq) * 32 * DPL + d - 2], f, v);
            }
        }
        part_base[(size_t)chunk * G * (hd + 2) + i] = v;
    }
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
        *sm.last = last;
    }
    SYNC();
    const int last = *sm.last;
    if (!last) {
        SYNC();  // the flag may be rewritten by the next chunk of this CTA
        return;
    }
    // final combine over chunks, in chunk order: first the (max, sum) of every
    // chunk and query head, loaded in parallel into shared memory (the warp
    // state area is free now), then each output element
    float *cm = sm.wo;                   // [nactive][G] maxima
    float *cl = sm.wo + nactive * G;     // [nactive][G] sums
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

// ---- host side (b2_attn.cu) ---------------------------------------------------------
// Argument checks of b2_attn (0 or a negative status).
int attn_check(const b2_attn_args *a);
// Kernel parameters from checked arguments (scratch and counters from `a`).
void attn_params(const b2_attn_args *a, uint32_t nchunks_max, AttnParams &p);

}  // namespace b2
