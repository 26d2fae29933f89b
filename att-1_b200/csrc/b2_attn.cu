// b2_attn.cu - single-query attention over the paged KV cache.
//
// Replaces the per-head host loops of src/attention.c:508-541 (scores =
// q.k * 1/sqrt(hd), softmax of src/norm.c:36-71, context = sum p * v) for one
// decoded token per sequence. The KV cache is paged like the reference's
// KV-MMU (src/kv_mmu.c:95-101: fixed-size pages, a page table per sequence),
// with n_kv_heads heads; inside a page the heads come first
// ([head][token_in_page][head_dim]) so that one KV head's tokens are
// contiguous runs in HBM. The H/Hkv query heads of a KV head share every K/V
// read (grouped-query attention; the reference reaches the same numbers with
// expanded heads).
//
// Work split: CTA (split, KV head, item) owns a contiguous range of one KV
// head's positions, about one CTA per SM over the step. A KV head's rows are
// contiguous inside a page, so the range streams through kBufs shared-memory
// buffers with 1-D bulk copies (the TMA engine, completion on an mbarrier);
// the scores of the query heads that share the KV head, an online softmax
// and the weighted V sum are computed from shared memory. Each CTA writes
// its (max, sum, weighted V) partial; the last CTA of an (item, KV head) to
// arrive combines the partials in split order (deterministic) and writes the
// context.
#include "b2_attn.cuh"

#include <mutex>

namespace b2 {

constexpr int kAttnWarps = 16;     // consumer warps
constexpr int kAttnThreads = kAttnWarps * 32 + 32;  // + one producer warp
constexpr uint32_t kSub = 32;       // positions per sub-tile
constexpr uint32_t kBufs = 6;       // sub-tile buffers (ring stages)
constexpr int kCtasPerSm = 1;       // resident CTAs per SM the split count aims at

struct ConsumerWarps {
    __device__ void operator()() const { asm volatile("bar.sync 1, %0;" ::"n"(kAttnWarps * 32) : "memory"); }
};

__host__ __device__ constexpr size_t attn_ring_smem(uint32_t hd)
{
    // full / empty mbarriers | kBufs sub-tile buffers of K and V | combine flag
    return 2 * kBufs * 8 + 2 * (size_t)kBufs * kSub * hd * sizeof(float) + 16;
}

// Merge two online-softmax states (m, l, o) of one query head.
__device__ __forceinline__ void soft_merge4(float &m, float &l, float4 &o, float m2, float l2, float4 o2)
{
    const float M = fmaxf(m, m2);
    if (M == -INFINITY) return;  // both empty
    const float f1 = expf(m - M), f2 = expf(m2 - M);
    l = fmaf(l, f1, l2 * f2);
    o = make_float4(fmaf(o.x, f1, o2.x * f2), fmaf(o.y, f1, o2.y * f2), fmaf(o.z, f1, o2.z * f2),
                    fmaf(o.w, f1, o2.w * f2));
    m = M;
}

// CTA (split, KV head, item) owns a contiguous range of one KV head's
// positions (about one CTA per SM over the step). Inside a page a KV head's
// rows are contiguous, so a producer warp streams the range through a ring of
// kBufs shared-memory sub-tiles with 1-D bulk copies (TMA; "full" mbarrier
// per stage, counted in bytes). Sixteen consumer warps take positions of each
// sub-tile (LP lanes per position, 4*V4 dimensions per lane: float4 chunk v of
// lane sl holds dimensions 4*(sl + v*LP)..+3, so a lane group's loads of one
// chunk are contiguous), compute the
// scores of the query heads that share the KV head with a halving exchange
// (each step hands half of the heads to the partner lane), keep an online
// softmax and the weighted V sum per lane, and release the stage on its
// "empty" mbarrier, so warps never wait for one another while streaming.
// At the end the lane groups and the warps are merged.
template <int LP, int MG, int V4>  // lanes per position, query heads per KV head (bound), float4s per lane
__global__ void __launch_bounds__(kAttnThreads, 1) attn_ring_kernel(const AttnParams p)
{
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int PPW = 32 / LP;
    const uint32_t split = blockIdx.x, S = gridDim.x, kvh = blockIdx.y, item = blockIdx.z;
    const uint32_t hd = p.head_dim, G = p.group;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);   // [kBufs]
    uint64_t *empty = full + kBufs;                          // [kBufs]
    float *Kb = reinterpret_cast<float *>(smem + 2 * kBufs * 8);  // [kBufs][kSub][hd]
    float *Vb = Kb + kBufs * kSub * hd;                             // [kBufs][kSub][hd]
    int *last = reinterpret_cast<int *>(Vb + kBufs * kSub * hd);

    // The KV rows before this step's position were written by earlier steps
    // and the position itself by the previous step's step end, so the ring
    // starts filling before the programmatic-launch wait; only the sub-tile
    // holding this step's K/V row (written by the QKV GEMV just before) and
    // q wait for it.
    const int32_t pos = __ldcg(p.positions + item);
    if (pos < 0 || (uint32_t)pos >= p.max_ctx) {
        pdl_wait();
        if (threadIdx.x == 0 && split == 0 && kvh == 0) raise_error(p.err, B2_ERR_POSITION);
        return;
    }
    const uint32_t len = (uint32_t)pos + 1;
    const uint32_t nactive = min(S, len);
    if (split >= nactive) return;
    const uint32_t p0 = (uint32_t)((uint64_t)split * len / nactive);
    const uint32_t n = (uint32_t)((uint64_t)(split + 1) * len / nactive) - p0;
    const uint32_t ntiles = (n + kSub - 1) / kSub;

    if (threadIdx.x == 0) {
        for (uint32_t b = 0; b < kBufs; ++b) {
            mbar_init(&full[b], 1);
            mbar_init(&empty[b], kAttnWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kAttnWarps) {
        // producer: sub-tile t of the range into stage t % kBufs (page pieces are contiguous)
        const uint32_t rowb = hd * sizeof(float);
        bool waited = false;
        for (uint32_t t = 0; t < ntiles; ++t) {
            const uint32_t buf = t % kBufs;
            if (t >= kBufs && !mbar_wait_bounded(&empty[buf], ((t / kBufs) - 1) & 1u, p.err)) break;
            if (!waited && split == nactive - 1 && t == ntiles - 1) {  // this sub-tile holds position len - 1
                pdl_wait();
                waited = true;
            }
            if (lane == 0) {
                const uint32_t r0 = t * kSub, nt = min(kSub, n - r0);
                mbar_arrive_expect_tx(&full[buf], 2 * nt * rowb);
                for (uint32_t r = 0; r < nt;) {
                    const uint32_t ps = p0 + r0 + r, run = min(nt - r, p.kv.page_tokens - ps % p.kv.page_tokens);
                    bulk_g2s(Kb + ((size_t)buf * kSub + r) * hd, kv_row(p.kv, p.kv.k_pool, item, ps, kvh), run * rowb,
                             &full[buf]);
                    bulk_g2s(Vb + ((size_t)buf * kSub + r) * hd, kv_row(p.kv, p.kv.v_pool, item, ps, kvh), run * rowb,
                             &full[buf]);
                    r += run;
                }
            }
            __syncwarp();
        }
        if (!waited) pdl_wait();
        pdl_launch_dependents();
        return;
    }

    // ---- consumers ----
    pdl_wait();
    pdl_launch_dependents();
    const int sub = lane / LP, sl = lane % LP;
    uint32_t dv[V4];
    bool dval[V4];
#pragma unroll
    for (int v = 0; v < V4; ++v) {
        dv[v] = 4 * (sl + v * LP);
        dval[v] = dv[v] < hd;
    }
    float4 qv[MG][V4];
#pragma unroll
    for (int gq = 0; gq < MG; ++gq)
#pragma unroll
        for (int v = 0; v < V4; ++v) {
            qv[gq][v] = make_float4(0, 0, 0, 0);
            if (gq < (int)G && dval[v])
                qv[gq][v] = __ldcg(reinterpret_cast<const float4 *>(p.q + (size_t)item * p.n_heads * hd +
                                                                    (size_t)(kvh * G + gq) * hd + dv[v]));
        }
    float m[MG], l[MG];
    float4 o[MG][V4];
#pragma unroll
    for (int gq = 0; gq < MG; ++gq) {
        m[gq] = -INFINITY;
        l[gq] = 0.0f;
#pragma unroll
        for (int v = 0; v < V4; ++v) o[gq][v] = make_float4(0, 0, 0, 0);
    }
    bool ok = true;
    for (uint32_t t = 0; t < ntiles; ++t) {
        const uint32_t buf = t % kBufs, nt = min(kSub, n - t * kSub);
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[buf], (t / kBufs) & 1u, p.err));
        const float *K = Kb + (size_t)buf * kSub * hd, *V = Vb + (size_t)buf * kSub * hd;
        // this warp's positions of the sub-tile (warp-uniform trip count); a lane
        // group takes two at a time only when the warps' groups cannot cover
        // the sub-tile in one pass (NP = 1: the second would always be empty)
        constexpr uint32_t kStride = kAttnWarps * PPW;
        constexpr int NP = kStride < kSub ? 2 : 1;
        for (uint32_t wb = warp * PPW; wb < nt; wb += NP * kStride) {
            const uint32_t ra = wb + sub, rb = ra + kStride;
            const bool va = ok && ra < nt, vb = NP == 2 && ok && rb < nt;
            float4 k4[NP][V4], v4[NP][V4];
#pragma unroll
            for (int v = 0; v < V4; ++v) {
                const float4 z = make_float4(0, 0, 0, 0);
                k4[0][v] = (va && dval[v]) ? *reinterpret_cast<const float4 *>(K + ra * hd + dv[v]) : z;
                v4[0][v] = (va && dval[v]) ? *reinterpret_cast<const float4 *>(V + ra * hd + dv[v]) : z;
                if constexpr (NP == 2) {
                    k4[NP - 1][v] = vb && dval[v] ? *reinterpret_cast<const float4 *>(K + rb * hd + dv[v]) : z;
                    v4[NP - 1][v] = vb && dval[v] ? *reinterpret_cast<const float4 *>(V + rb * hd + dv[v]) : z;
                }
            }
            float mine[NP];
#pragma unroll
            for (int j = 0; j < NP; ++j) {
                float dot[MG];
#pragma unroll
                for (int gq = 0; gq < MG; ++gq) {
                    dot[gq] = 0.0f;
#pragma unroll
                    for (int v = 0; v < V4; ++v)
                        dot[gq] += qv[gq][v].x * k4[j][v].x + qv[gq][v].y * k4[j][v].y + qv[gq][v].z * k4[j][v].z +
                                   qv[gq][v].w * k4[j][v].w;
                }
                // sum over the LP lanes of the position: while more than one head
                // is left each exchange hands half of them to the partner lane
                // (the upper lane keeps the upper half), then plain exchanges;
                // lane sl ends with head (top log2 MG bits of sl)
#pragma unroll
                for (int cnt = MG, off = LP / 2; off > 0; off >>= 1) {
                    if (cnt > 1) {
                        const bool upper = (sl & off) != 0;
#pragma unroll
                        for (int i = 0; i < cnt / 2; ++i) {
                            const float send = upper ? dot[i] : dot[i + cnt / 2];
                            const float keep = upper ? dot[i + cnt / 2] : dot[i];
                            dot[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                        }
                        cnt /= 2;
                    } else {
                        dot[0] += __shfl_xor_sync(0xffffffffu, dot[0], off);
                    }
                }
                mine[j] = __fmul_rn(dot[0], p.inv_sqrt);  // src/attention.c:521-523
            }
            // online softmax over both positions at once, per query head
#pragma unroll
            for (int gq = 0; gq < MG; ++gq) {
                if (gq < (int)G) {
                    const int src = (sub * LP) | (gq * (LP / MG));  // a lane holding head gq
                    const float sa = __shfl_sync(0xffffffffu, mine[0], src);
                    const float sb = NP == 2 ? __shfl_sync(0xffffffffu, mine[NP - 1], src) : 0.0f;
                    if (va) {
                        const float nm = fmaxf(m[gq], vb ? fmaxf(sa, sb) : sa);
                        const float corr = __expf(m[gq] - nm);
                        const float pa = __expf(sa - nm), pb = vb ? __expf(sb - nm) : 0.0f;
                        l[gq] = fmaf(l[gq], corr, pa + pb);
#pragma unroll
                        for (int v = 0; v < V4; ++v) {
                            float4 w = make_float4(pa * v4[0][v].x, pa * v4[0][v].y, pa * v4[0][v].z, pa * v4[0][v].w);
                            if constexpr (NP == 2)
                                w = make_float4(fmaf(pb, v4[NP - 1][v].x, w.x), fmaf(pb, v4[NP - 1][v].y, w.y),
                                                fmaf(pb, v4[NP - 1][v].z, w.z), fmaf(pb, v4[NP - 1][v].w, w.w));
                            o[gq][v] = make_float4(fmaf(o[gq][v].x, corr, w.x), fmaf(o[gq][v].y, corr, w.y),
                                                   fmaf(o[gq][v].z, corr, w.z), fmaf(o[gq][v].w, corr, w.w));
                        }
                        m[gq] = nm;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[buf]);
    }
    // merge the lane groups of the warp (positions differ, dimensions match)
#pragma unroll
    for (int off = LP; off < 32; off <<= 1) {
#pragma unroll
        for (int gq = 0; gq < MG; ++gq) {
            const float m2 = __shfl_xor_sync(0xffffffffu, m[gq], off);
            const float l2 = __shfl_xor_sync(0xffffffffu, l[gq], off);
            float4 o2[V4];
#pragma unroll
            for (int v = 0; v < V4; ++v) {
                o2[v].x = __shfl_xor_sync(0xffffffffu, o[gq][v].x, off);
                o2[v].y = __shfl_xor_sync(0xffffffffu, o[gq][v].y, off);
                o2[v].z = __shfl_xor_sync(0xffffffffu, o[gq][v].z, off);
                o2[v].w = __shfl_xor_sync(0xffffffffu, o[gq][v].w, off);
            }
            // the chunks share one (m, l): merge them with the same factors
            const float M = fmaxf(m[gq], m2);
            if (M != -INFINITY) {
                const float f1 = expf(m[gq] - M), f2 = expf(m2 - M);
                l[gq] = fmaf(l[gq], f1, l2 * f2);
#pragma unroll
                for (int v = 0; v < V4; ++v)
                    o[gq][v] = make_float4(fmaf(o[gq][v].x, f1, o2[v].x * f2), fmaf(o[gq][v].y, f1, o2[v].y * f2),
                                           fmaf(o[gq][v].z, f1, o2[v].z * f2), fmaf(o[gq][v].w, f1, o2[v].w * f2));
                m[gq] = M;
            }
        }
    }
    // merge the warps: state in shared memory (the ring is drained)
    ConsumerWarps SYNC;
    SYNC();
    float *wm = Kb, *wl = Kb + kAttnWarps * MG, *wo = Kb + 2 * kAttnWarps * MG;  // wo [warps][MG][hd]
#pragma unroll
    for (int gq = 0; gq < MG; ++gq) {
        if (gq < (int)G && sub == 0) {
            if (sl == 0) {
                wm[warp * MG + gq] = m[gq];
                wl[warp * MG + gq] = l[gq];
            }
#pragma unroll
            for (int v = 0; v < V4; ++v)
                if (dval[v]) *reinterpret_cast<float4 *>(wo + ((size_t)warp * MG + gq) * hd + dv[v]) = o[gq][v];
        }
    }
    SYNC();
    float *part_base = p.partial + ((size_t)(item * p.n_kv_heads + kvh) * p.nchunks_max) * G * (hd + 2);
    float *part = part_base + (size_t)split * G * (hd + 2);
    const uint32_t nthreads = kAttnWarps * 32;
    for (uint32_t i = threadIdx.x; i < G * (hd + 2); i += nthreads) {
        const uint32_t gq = i / (hd + 2), d = i % (hd + 2);
        float M = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w * MG + gq]);
        float v = 0.0f;
        if (d == 0) {
            v = M;
        } else {
            for (int w = 0; w < kAttnWarps; ++w) {
                const float wmv = wm[w * MG + gq];
                if (wmv == -INFINITY) continue;  // warp saw no position
                v = fmaf(d == 1 ? wl[w * MG + gq] : wo[((size_t)w * MG + gq) * hd + d - 2], expf(wmv - M), v);
            }
        }
        part[i] = v;
    }
    attn_publish(p, Kb + 2 * kAttnWarps * MG + (size_t)kAttnWarps * MG * hd, last, item, kvh, nactive, part_base,
                 nthreads, SYNC);
}

static cudaError_t launch_attn(const AttnParams &p, dim3 grid, int pdl, cudaStream_t st)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kAttnThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const int mg = p.group <= 4 ? 4 : 8;
    cfg.dynamicSmemBytes = attn_ring_smem(p.head_dim);
    const void *fn;
    // one float4 of dimensions per lane: 8, 16 or 32 lanes per position (16
    // lanes x 8 dimensions for head_dim 128 measured slower in the decode step:
    // 2.37 vs 2.29 ms, at the 96-register limit of 17 warps)
    switch (attn_lanes(p.head_dim) * 10 + mg) {
    case 84: fn = (const void *)attn_ring_kernel<8, 4, 1>; break;
    case 88: fn = (const void *)attn_ring_kernel<8, 8, 1>; break;
    case 164: fn = (const void *)attn_ring_kernel<16, 4, 1>; break;
    case 168: fn = (const void *)attn_ring_kernel<16, 8, 1>; break;
    case 324: fn = (const void *)attn_ring_kernel<32, 4, 1>; break;
    default: fn = (const void *)attn_ring_kernel<32, 8, 1>; break;
    }
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cfg.dynamicSmemBytes);
    if (e != cudaSuccess) return e;
    void *args[] = {const_cast<AttnParams *>(&p)};
    return cudaLaunchKernelExC(&cfg, fn, args);
}


// Splits per (item, KV head): about kCtasPerSm CTAs per SM over the grid,
// at least one position each at the longest context.
static void attn_sizes(const b2_attn_args *a, uint32_t &nchunks, size_t &partial, uint32_t &counters)
{
    const uint32_t heads = a->batch * a->n_kv_heads;
    nchunks = (uint32_t)(kCtasPerSm * sm_count()) / heads;
    if (nchunks < 1) nchunks = 1;
    if (nchunks > a->max_ctx) nchunks = a->max_ctx;
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
    // the split combine stages (max, sum) of every split in the sub-tile buffers
    uint32_t nchunks, cl;
    size_t pb;
    attn_sizes(a, nchunks, pb, cl);
    // warp states and the combine staging share the drained ring
    if (2ull * kAttnWarps * kMaxGroup + (uint64_t)kAttnWarps * kMaxGroup * a->head_dim + 2ull * nchunks * G >
        2ull * kBufs * kSub * a->head_dim)
        return -9;
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

// ---- attention without any allocation ------------------------------------------
//
// For callers that cannot allocate device memory at the point where they run
// the attention: code running inside a memory pool or arena it does not own,
// code that must not synchronise the device (cudaMalloc and cudaFree can), and
// host programs whose allocator is closed to plugins. b2_attn needs a buffer for
// the position splits' partial results and a counter array from the caller;
// b2_attn_noalloc takes both from one fixed array in device global memory, so
// the caller passes only q, the KV pages, positions, the output and a stream.
//
// The array is B2_NOALLOC_SCRATCH_BYTES long and every GPU that loads this
// library holds it until the process exits. A call whose split plan needs more
// is rejected with ATT1_ERR_UNSUPPORTED (-9) before anything is touched, as is
// any call b2_attn would reject. All calls on a device share the array: calls
// that overlap on the GPU (two streams, or two host threads) race on it and
// must be ordered by the caller. The array keeps the last call's contents; the
// counters, which must start at zero, are cleared by an asynchronous memset at
// every call (so a call cut short by a timed-out wait cannot poison the next).
//
// Host code only holds a stand-in for the array's name, not its device
// address: the first call on each device looks the address up with
// cudaGetSymbolAddress (with that device current) and caches it, so that first
// call should come before any stream capture on that device. The cached
// address belongs to the device's primary context; after a cudaDeviceReset the
// next call would use a stale address, so reset the device only after the last
// call. Nothing here allocates.

static __device__ __align__(256) unsigned char g_noalloc_scratch[B2_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
void *g_noalloc_base[kMaxDevices];
std::mutex g_noalloc_mutex;
}  // namespace

extern "C" int b2_attn_noalloc(const b2_attn_args *a, void *stream)
{
    if (a == nullptr) return -1;
    b2_attn_args c = *a;
    c.scratch = nullptr;
    c.counters = nullptr;
    // every argument error is returned before the shared array is touched, so a
    // rejected call cannot disturb a valid one still running on the device
    const int rc = attn_check(&c);
    if (rc != 0) return rc;
    uint32_t nchunks, ncnt;
    size_t need;
    attn_sizes(&c, nchunks, need, ncnt);
    const size_t cnt_bytes = ((size_t)ncnt * sizeof(int32_t) + 255) & ~(size_t)255;
    if (cnt_bytes + need > (size_t)B2_NOALLOC_SCRATCH_BYTES) return -9;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -8;
    void *base = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mutex);
        if (g_noalloc_base[dev] == nullptr) {
            void *p = nullptr;
            if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return -8;
            g_noalloc_base[dev] = p;
        }
        base = g_noalloc_base[dev];
    }
    c.counters = reinterpret_cast<int32_t *>(base);
    c.counters_len = ncnt;
    c.scratch = reinterpret_cast<uint8_t *>(base) + cnt_bytes;
    c.scratch_bytes = need;
    if (cudaMemsetAsync(c.counters, 0, (size_t)ncnt * sizeof(int32_t), (cudaStream_t)stream) != cudaSuccess) return -8;
    return b2_attn(&c, stream);
}
