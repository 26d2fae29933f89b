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

constexpr int kAttnWarps = 16;     // consumer warps (upper bound over the variants)
constexpr uint32_t kSub = 32;       // positions per sub-tile
constexpr uint32_t kBufs = 6;       // sub-tile buffers (ring stages)
constexpr int kCtasPerSm = 1;       // resident CTAs per SM the split count aims at

template <int NW>
struct ConsumerWarps {
    __device__ void operator()() const { asm volatile("bar.sync 1, %0;" ::"n"(NW * 32) : "memory"); }
};

__host__ __device__ constexpr size_t attn_ring_smem(uint32_t hd)
{
    // full / empty mbarriers | kBufs sub-tile buffers of K and V | combine flag
    return 2 * kBufs * 8 + 2 * (size_t)kBufs * kSub * hd * sizeof(float) + 16;
}

// CTA (split, KV head, item) owns a contiguous range of one KV head's
// positions (about one CTA per SM over the step). Inside a page a KV head's
// rows are contiguous, so a producer warp streams the range through a ring of
// kBufs shared-memory sub-tiles with 1-D bulk copies (TMA; "full" mbarrier
// per stage, counted in bytes). NW consumer warps take positions of each
// sub-tile, LP lanes per position and NP positions per lane group at a time.
// Scores: float4 chunk v of lane sl holds dimensions 4*(sl + v*LP)..+3 of q
// and k for every query head of the group; the partial dot products are
// summed over the LP lanes with a halving exchange (each step hands half of
// the heads to the partner lane), after which the HL = LP / MG lanes of head
// group h = sl / HL all hold the full score of query head h. Values: those HL
// lanes split the head's dimensions (chunk w of lane hl holds dimensions
// 4*(hl + w*HL)..+3), so each lane keeps the online softmax (max, sum) and the
// weighted V sum of its own query head only: no score is broadcast and every
// exponential is computed once per head. Lanes release the stage on its
// "empty" mbarrier, so warps never wait for one another while streaming. At
// the end the lane groups and the warps are merged.
template <int LP, int MG, int V4, int NW, int NP>
__global__ void __launch_bounds__(NW * 32 + 32, 1) attn_ring_kernel(const AttnParams p)
{
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int PPW = 32 / LP;          // positions per warp pass
    constexpr int HL = LP / MG;           // lanes per query head in the value sums
    constexpr int VW = V4 * MG;           // float4 chunks of V per lane
    static_assert(HL >= 1, "at most LP query heads per KV head");
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
            mbar_init(&empty[b], NW);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == NW) {
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
                    bulk_g2s_stream(Kb + ((size_t)buf * kSub + r) * hd, kv_row(p.kv, p.kv.k_pool, item, ps, kvh),
                                    run * rowb, &full[buf], l2_evict_first_policy());
                    bulk_g2s_stream(Vb + ((size_t)buf * kSub + r) * hd, kv_row(p.kv, p.kv.v_pool, item, ps, kvh),
                                    run * rowb, &full[buf], l2_evict_first_policy());
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
    const int hsel = sl / HL, hl = sl % HL;       // query head of this lane's value sums, its lane in the head
    const bool hval = hsel < (int)G;
    uint32_t dv[V4], dw[VW];
    bool dval[V4], dwv[VW];
#pragma unroll
    for (int v = 0; v < V4; ++v) {
        dv[v] = 4 * (sl + v * LP);
        dval[v] = dv[v] < hd;
    }
#pragma unroll
    for (int w = 0; w < VW; ++w) {
        dw[w] = 4 * (hl + w * HL);
        dwv[w] = dw[w] < hd;
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
    float m = -INFINITY, l = 0.0f;
    float4 o[VW];
#pragma unroll
    for (int w = 0; w < VW; ++w) o[w] = make_float4(0, 0, 0, 0);
    bool ok = true;
    constexpr uint32_t kStride = NW * PPW;     // positions of one pass of every warp's lane groups
    for (uint32_t t = 0; t < ntiles; ++t) {
        const uint32_t buf = t % kBufs, nt = min(kSub, n - t * kSub);
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[buf], (t / kBufs) & 1u, p.err));
        const float *K = Kb + (size_t)buf * kSub * hd, *V = Vb + (size_t)buf * kSub * hd;
        // this warp's positions of the sub-tile (warp-uniform trip count)
        for (uint32_t wb = warp * PPW; wb < nt; wb += NP * kStride) {
            uint32_t r[NP];
            bool va[NP];
            float4 k4[NP][V4];
#pragma unroll
            for (int j = 0; j < NP; ++j) {
                r[j] = wb + sub + j * kStride;
                va[j] = ok && r[j] < nt;
#pragma unroll
                for (int v = 0; v < V4; ++v)
                    k4[j][v] = (va[j] && dval[v]) ? *reinterpret_cast<const float4 *>(K + r[j] * hd + dv[v])
                                                  : make_float4(0, 0, 0, 0);
            }
            float sc[NP];
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
                // lane sl ends with head sl / HL
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
                sc[j] = __fmul_rn(dot[0], p.inv_sqrt);  // src/attention.c:521-523
            }
            // online softmax of this lane's head over the NP positions, then the
            // weighted values of its dimension chunks
            if (hval && va[0]) {
                float nm = m;
#pragma unroll
                for (int j = 0; j < NP; ++j)
                    if (va[j]) nm = fmaxf(nm, sc[j]);
                const float corr = __expf(m - nm);
                float pj[NP];
                float psum = 0.0f;
#pragma unroll
                for (int j = 0; j < NP; ++j) {
                    pj[j] = va[j] ? __expf(sc[j] - nm) : 0.0f;
                    psum += pj[j];
                }
                l = fmaf(l, corr, psum);
#pragma unroll
                for (int w = 0; w < VW; ++w) {
                    float4 acc = make_float4(o[w].x * corr, o[w].y * corr, o[w].z * corr, o[w].w * corr);
#pragma unroll
                    for (int j = 0; j < NP; ++j) {
                        if (va[j] && dwv[w]) {
                            const float4 vv = *reinterpret_cast<const float4 *>(V + r[j] * hd + dw[w]);
                            acc = make_float4(fmaf(pj[j], vv.x, acc.x), fmaf(pj[j], vv.y, acc.y),
                                              fmaf(pj[j], vv.z, acc.z), fmaf(pj[j], vv.w, acc.w));
                        }
                    }
                    o[w] = acc;
                }
                m = nm;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[buf]);
    }
    // merge the lane groups of the warp (positions differ, head and dimensions match)
#pragma unroll
    for (int off = LP; off < 32; off <<= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
        const float l2 = __shfl_xor_sync(0xffffffffu, l, off);
        float4 o2[VW];
#pragma unroll
        for (int w = 0; w < VW; ++w) {
            o2[w].x = __shfl_xor_sync(0xffffffffu, o[w].x, off);
            o2[w].y = __shfl_xor_sync(0xffffffffu, o[w].y, off);
            o2[w].z = __shfl_xor_sync(0xffffffffu, o[w].z, off);
            o2[w].w = __shfl_xor_sync(0xffffffffu, o[w].w, off);
        }
        const float M = fmaxf(m, m2);
        if (M != -INFINITY) {
            const float f1 = expf(m - M), f2 = expf(m2 - M);
            l = fmaf(l, f1, l2 * f2);
#pragma unroll
            for (int w = 0; w < VW; ++w)
                o[w] = make_float4(fmaf(o[w].x, f1, o2[w].x * f2), fmaf(o[w].y, f1, o2[w].y * f2),
                                   fmaf(o[w].z, f1, o2[w].z * f2), fmaf(o[w].w, f1, o2[w].w * f2));
            m = M;
        }
    }
    // merge the warps: state in shared memory (the ring is drained)
    ConsumerWarps<NW> SYNC;
    SYNC();
    float *wm = Kb, *wl = Kb + NW * MG, *wo = Kb + 2 * NW * MG;  // wo [warps][MG][hd]
    if (hval && sub == 0) {
        if (hl == 0) {
            wm[warp * MG + hsel] = m;
            wl[warp * MG + hsel] = l;
        }
#pragma unroll
        for (int w = 0; w < VW; ++w)
            if (dwv[w]) *reinterpret_cast<float4 *>(wo + ((size_t)warp * MG + hsel) * hd + dw[w]) = o[w];
    }
    SYNC();
    float *part_base = p.partial + ((size_t)(item * p.n_kv_heads + kvh) * p.nchunks_max) * G * (hd + 2);
    float *part = part_base + (size_t)split * G * (hd + 2);
    const uint32_t nthreads = NW * 32;
    // the warps' rescale factors exp(m_w - M) once per (warp, query head), in
    // the drained V ring (0 for a warp that saw no position, whose sums are 0),
    // then every element of the partial is a chain of NW fused multiply-adds
    // in warp order: the same arithmetic as one exponential per element and
    // warp, 14.2 instead of 15.6 us at context 4096
    float *wf = Vb;            // [NW][MG]
    float *wM = Vb + NW * MG;  // [MG]
    if (threadIdx.x < NW * G) {
        const uint32_t w = threadIdx.x / G, gq = threadIdx.x % G;
        float M = -INFINITY;
#pragma unroll
        for (int v = 0; v < NW; ++v) M = fmaxf(M, wm[v * MG + gq]);
        const float wmv = wm[w * MG + gq];
        wf[w * MG + gq] = wmv == -INFINITY ? 0.0f : expf(wmv - M);
        if (w == 0) wM[gq] = M;
    }
    SYNC();
    for (uint32_t i = threadIdx.x; i < G * (hd + 2); i += nthreads) {
        const uint32_t gq = i / (hd + 2), d = i % (hd + 2);
        float v = 0.0f;
        if (d == 0) {
            v = wM[gq];
        } else {
            const float *src = d == 1 ? wl + gq : wo + (size_t)gq * hd + d - 2;
            const uint32_t stride = d == 1 ? MG : MG * hd;
#pragma unroll
            for (int w = 0; w < NW; ++w) v = fmaf(src[w * stride], wf[w * MG + gq], v);
        }
        part[i] = v;
    }
    attn_publish(p, Kb + 2 * NW * MG + (size_t)NW * MG * hd, last, item, kvh, nactive, part_base, nthreads, SYNC);
}

template <int NW, int NP>
static const void *attn_fn(uint32_t hd, int mg)
{
    switch (attn_lanes(hd) * 10 + mg) {
    case 84: return (const void *)attn_ring_kernel<8, 4, 1, NW, NP>;
    case 88: return (const void *)attn_ring_kernel<8, 8, 1, NW, NP>;
    case 164: return (const void *)attn_ring_kernel<16, 4, 1, NW, NP>;
    case 168: return (const void *)attn_ring_kernel<16, 8, 1, NW, NP>;
    case 324: return (const void *)attn_ring_kernel<32, 4, 1, NW, NP>;
    default: return (const void *)attn_ring_kernel<32, 8, 1, NW, NP>;
    }
}

// Consumer warps and positions per lane group at a time. Measured at the 8B
// shape, context 4096 (one launch, CUDA events): 16 warps x 2 positions
// 15.7 us; 16 x 1 16.8 us; 8 x 4 16.5 us; 8 x 2 18.0 us. Two CTAs per SM (8
// warps, 3 sub-tile buffers, 37 splits per KV head): 27.9 us (x 4 positions),
// 30.0 us (x 2).
constexpr int kNW = 16, kNP = 2;

static cudaError_t launch_attn(const AttnParams &p, dim3 grid, int pdl, cudaStream_t st)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kNW * 32 + 32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const int mg = p.group <= 4 ? 4 : 8;
    cfg.dynamicSmemBytes = attn_ring_smem(p.head_dim);
    const void *fn = attn_fn<kNW, kNP>(p.head_dim, mg);
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
