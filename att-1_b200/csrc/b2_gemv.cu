// b2_gemv.cu - q4/q8 block-dequant matrix-vector products for decode.
//
// Replaces att1_matmul_q4xf32 (src/quant.c:340-393) and att1_matmul_q8xf32
// (src/matmul_q8.c:3-40) on the device, with the neighbouring element ops of
// the block (src/transformer_block.c:417-557) fused in:
//   prologue: optional RMSNorm (src/norm.c:5-34) of the input vector;
//   epilogue: plain store, residual add, RoPE + KV-page append
//             (src/attention.c:490-504), SwiGLU (src/ffn.c:10-30), or logits
//             with the greedy argmax key (src/sampler.c:5-34).
//
// Arithmetic. Batch-1 decode reads every weight byte once, so the kernel is
// HBM-bound; the design spends as few instructions per weight as possible:
//   * the input vector x (f32) is written, per item, as an exact 22-bit fixed
//     point number v = round(x * 2^-E) split into three signed byte digits
//     (v = d0 + 256 d1 + 65536 d2); E is chosen from max|x| so |v| <= 2^22;
//   * a q4 byte holding nibbles (a, b) yields the int8 values 16a and 16b with
//     one shift and one AND each (a nibble in the top half of a byte is its
//     two's-complement value times 16), q8 bytes are used as they are;
//   * mma.sync m16n8k32 s8 x s8 -> s32 multiplies a 16x32 weight block with
//     the digit columns exactly in integers; one group (32 columns) per MMA,
//     so the per-group q4 scale is applied once per 32 weights in f32.
// Products are exact; rounding happens only in the f32 scale/accumulate steps
// and in the 2^-22 relative quantisation of x, far inside the 1e-3 logits
// tolerance of the parity tests.
//
// Streaming. Weights sit in the panel/unit layout of b2_kernels.h: a panel
// is 16 row tiles, stored k-column by k-column (the 16 units of one column
// pair, contiguous). Each CTA owns a contiguous range of k-columns (stream-K
// over panel-major columns, balanced to one column across the grid), so at
// any moment the GPU reads ~one compact window per CTA. The range is cut into
// stages of up to kStageCols columns that never straddle a panel. One
// producer lane copies each stage into a shared-memory ring of up to
// kMaxStages stages with a single 1-D bulk copy (cp.async.bulk, completion
// counted in bytes on the stage's "full" mbarrier). Consumer warp w owns tile
// w of every panel: it multiplies unit (column, w) of each staged column,
// keeps the tile's sums in registers across stages, and releases each stage
// on its "empty" mbarrier, so the warps never meet at a CTA barrier and never
// add each other's partial sums. When the CTA's part of a panel ends, each
// warp finishes its own tile; a panel shared with neighbouring CTAs is added
// by the last CTA to finish each tile (per-tile arrival counter), in CTA
// order, so results are deterministic. The producer requests the first
// stages before griddepcontrol.wait, so under programmatic dependent launch
// the weight fetch overlaps the previous kernel.
//
// Measured alternatives, slower: tile-major units split by k between the 16
// warps (every tile then needs a cross-warp reduction in shared memory, and
// the warp doing it lags and holds back the ring: half the speed of this
// layout at 4096 columns); small bulk copies (an SM completes roughly one
// bulk copy per 0.4-0.6 us almost whatever its size, so tens of KB per copy
// are needed); per-warp contiguous ranges read with register prefetch
// (~2400 small streams over HBM, under 2.5 TB/s without arithmetic); a ring
// refilled by 16-byte cp.async from one warp.
#include "b2_common.cuh"

#include <cfloat>
#include <cstdio>
#include <mutex>
#include <cuda_runtime.h>

namespace b2 {

constexpr int kWarps = 16;                          // consumer warps (16 hide the math latency)
constexpr int kConsumers = kWarps * 32;
constexpr int kThreads = kConsumers + 32;           // + one producer warp
constexpr int kPanelTiles = 16;                     // tiles per panel: one per consumer warp
constexpr int kStageCols = 4;                       // k-columns per stage
constexpr int kStageUnits = kStageCols * kPanelTiles;  // 64 units: 40 KB of q4, one bulk copy
constexpr int kMaxStages = 8;                       // ring depth, chosen per launch
constexpr int kMaxItems = 16;
constexpr int kConsumerBarrier = 1;                 // named barrier of the consumer warps
static_assert(kPanelTiles == kWarps, "each consumer warp owns one tile of a panel");

struct GemvParams {
    const uint8_t *data;
    const float *row_scale;
    uint32_t rows, cols, tiles, kunits, panels;
    uint32_t batch;
    const float *x;
    uint32_t x_stride;
    const float *norm_w;
    float eps;
    int epilogue;
    float *out;
    uint32_t out_stride;
    const float *resid;
    uint32_t q_rows, kv_rows;
    const float *rope_freq;
    const int32_t *positions;
    b2_kv_layout kv;
    unsigned long long *argmax;
    float *partial;
    int *counters;
    uint32_t maxseg;
    int32_t *err;
    // shared-memory carve-up (bytes)
    uint32_t off_ring, off_xdig, off_tile, off_misc, stages;
};

template <int FMT>
struct Fmt;
template <>
struct Fmt<4> {
    static constexpr uint32_t kUnitBytes = B2_Q4_UNIT_BYTES;
    static constexpr uint32_t kKW = 64;  // columns per unit
};
template <>
struct Fmt<8> {
    static constexpr uint32_t kUnitBytes = B2_Q8_UNIT_BYTES;
    static constexpr uint32_t kKW = 32;
};

__device__ __forceinline__ uint32_t ordered_key(float f)
{
    uint32_t b = __float_as_uint(f == 0.0f ? 0.0f : f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// ---- prologue: per item, optional RMSNorm, exponent choice, digit planes ----
// One pass of loads (x and the norm gains together) and one reduction round
// per launch: every thread accumulates, per item, the sum of squares of x and
// the largest |x * w|; the warps' partials meet in shared memory once. The
// normed vector x * inv * w (src/norm.c:31) is bounded by inv * max|x * w|
// (times 1 + 2^-20 for the two roundings), and that bound picks the exponent,
// so no second reduction over the normed values is needed. Vectors of up to
// kPrologueVec * 4 * kConsumers elements stay in registers between the two
// steps (batch 1); otherwise the second step reads x again.
constexpr int kPrologueVec = 8;   // float4 per thread held in registers (x and gains)

template <int FMT>
__device__ __forceinline__ void store_digits(const GemvParams &p, uint8_t *xdig, uint32_t b, uint32_t k, float4 v,
                                             float sc, bool finite)
{
    constexpr uint32_t KW = Fmt<FMT>::kKW;
    const float vv[4] = {v.x, v.y, v.z, v.w};
    uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int q = finite ? __float2int_rn(__fmul_rn(vv[i], sc)) : 0;
        const int d0 = ((q + 128) & 255) - 128;
        const int q1 = (q - d0) >> 8;
        const int d1 = ((q1 + 128) & 255) - 128;
        const int d2 = (q1 - d1) >> 8;
        w0 |= ((uint32_t)d0 & 0xFFu) << (8 * i);
        w1 |= ((uint32_t)d1 & 0xFFu) << (8 * i);
        w2 |= ((uint32_t)d2 & 0xFFu) << (8 * i);
    }
    const uint32_t unit = k / KW, kk = k % KW;
    const uint32_t gi = kk >> 5, r = kk & 31;
    const uint32_t half = r >> 4, t = (r & 15) >> 2;
    uint8_t *base = xdig + ((size_t)(unit * p.batch + b) * 3) * KW + t * (KW / 4) + gi * 8 + half * 4;
    *reinterpret_cast<uint32_t *>(base) = w0;
    *reinterpret_cast<uint32_t *>(base + KW) = w1;
    *reinterpret_cast<uint32_t *>(base + 2 * KW) = w2;
}

__device__ __forceinline__ float4 normed(float4 v, float inv, float4 w)
{
    // src/norm.c:31: dst = src * scale * weight
    return make_float4(__fmul_rn(__fmul_rn(v.x, inv), w.x), __fmul_rn(__fmul_rn(v.y, inv), w.y),
                       __fmul_rn(__fmul_rn(v.z, inv), w.z), __fmul_rn(__fmul_rn(v.w, inv), w.w));
}

__device__ __forceinline__ float4 mul4(float4 a, float4 b)
{
    return make_float4(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y), __fmul_rn(a.z, b.z), __fmul_rn(a.w, b.w));
}

__device__ __forceinline__ float sumsq4(float4 v) { return v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w; }

__device__ __forceinline__ float absmax4(float4 v)
{
    const float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    // fmaxf drops NaN: make any non-finite element visible
    return (fabsf(v.x) <= FLT_MAX && fabsf(v.y) <= FLT_MAX && fabsf(v.z) <= FLT_MAX && fabsf(v.w) <= FLT_MAX)
               ? a : INFINITY;
}

__device__ __forceinline__ int pick_exponent(float m)
{
    int E = 0;
    if (m > 0.0f && m <= FLT_MAX) {
        E = ilogbf(m) - 21;  // |x| * 2^-E < 2^22
        if (E < -125) E = -125;
    }
    return E;
}

__device__ __forceinline__ void consumer_sync()
{
    asm volatile("bar.sync %0, %1;" ::"n"(kConsumerBarrier), "n"(kConsumers) : "memory");
}

// Per item: the normalisation factor (1 without a norm) and the exponent
// scale, from the item's sum of squares and max |x * w| (max |x| without a norm).
template <int FMT>
__device__ __forceinline__ void item_setup(const GemvParams &p, uint32_t b, float ss, float mw, float *inv_out,
                                           float *sc_out, bool *finite_out, float *item_scale)
{
    float inv = 1.0f, bound = mw;
    if (p.norm_w != nullptr) {
        // src/norm.c:26-28
        inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)p.cols), p.eps)));
        bound = __fmul_rn(__fmul_rn(mw, inv), 1.0f + 0x1p-20f);
    }
    const bool finite = mw <= FLT_MAX && inv <= FLT_MAX;
    const int E = pick_exponent(bound);
    *inv_out = inv;
    *sc_out = ldexpf(1.0f, -E);
    *finite_out = finite;
    if (threadIdx.x == 0) {
        item_scale[b] = ldexpf(1.0f, E - (FMT == 4 ? 4 : 0));
        if (!finite) raise_error(p.err, B2_ERR_NONFINITE);
    }
}

template <int FMT>
__device__ void prepare_x(const GemvParams &p, uint8_t *xdig, float *item_scale, float *red)
{
    const uint32_t cols = p.cols;
    const uint32_t stride = kConsumers * 4;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool norm = p.norm_w != nullptr;
    if (p.batch == 1 && cols <= stride * kPrologueVec) {
        float4 v[kPrologueVec], w[kPrologueVec];
#pragma unroll
        for (int i = 0; i < kPrologueVec; ++i) {
            const uint32_t k = threadIdx.x * 4 + i * stride;
            const bool in = k < cols;
            v[i] = in ? __ldcg(reinterpret_cast<const float4 *>(p.x + k)) : make_float4(0, 0, 0, 0);
            w[i] = (in && norm) ? __ldg(reinterpret_cast<const float4 *>(p.norm_w + k)) : make_float4(1, 1, 1, 1);
        }
        float ss = 0.0f, mw = 0.0f;
#pragma unroll
        for (int i = 0; i < kPrologueVec; ++i) {
            ss += sumsq4(v[i]);
            mw = fmaxf(mw, absmax4(norm ? mul4(v[i], w[i]) : v[i]));
        }
        ss = warp_sum(ss);
        mw = warp_max(mw);
        if (lane == 0) {
            red[warp] = ss;
            red[kWarps + warp] = mw;
        }
        consumer_sync();
        float tss = 0.0f, tmw = 0.0f;
#pragma unroll
        for (int i = 0; i < kWarps; ++i) {
            tss += red[i];
            tmw = fmaxf(tmw, red[kWarps + i]);
        }
        float inv, sc;
        bool finite;
        item_setup<FMT>(p, 0, tss, tmw, &inv, &sc, &finite, item_scale);
#pragma unroll
        for (int i = 0; i < kPrologueVec; ++i) {
            const uint32_t k = threadIdx.x * 4 + i * stride;
            if (k < cols) store_digits<FMT>(p, xdig, 0, k, norm ? normed(v[i], inv, w[i]) : v[i], sc, finite);
        }
        return;
    }
    // general path: statistics of every item in one reduction round, then the digits
    float *stats = red;  // [kMaxItems][kWarps][2]
    for (uint32_t b = 0; b < p.batch; ++b) {
        const float *xb = p.x + (size_t)b * p.x_stride;
        float ss = 0.0f, mw = 0.0f;
        for (uint32_t k = threadIdx.x * 4; k < cols; k += stride) {
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(xb + k));
            ss += sumsq4(v);
            mw = fmaxf(mw, absmax4(norm ? mul4(v, __ldg(reinterpret_cast<const float4 *>(p.norm_w + k))) : v));
        }
        ss = warp_sum(ss);
        mw = warp_max(mw);
        if (lane == 0) {
            stats[(b * kWarps + warp) * 2] = ss;
            stats[(b * kWarps + warp) * 2 + 1] = mw;
        }
    }
    consumer_sync();
    for (uint32_t b = 0; b < p.batch; ++b) {
        float tss = 0.0f, tmw = 0.0f;
#pragma unroll
        for (int i = 0; i < kWarps; ++i) {
            tss += stats[(b * kWarps + i) * 2];
            tmw = fmaxf(tmw, stats[(b * kWarps + i) * 2 + 1]);
        }
        float inv, sc;
        bool finite;
        item_setup<FMT>(p, b, tss, tmw, &inv, &sc, &finite, item_scale);
        const float *xb = p.x + (size_t)b * p.x_stride;
        for (uint32_t k = threadIdx.x * 4; k < cols; k += stride) {
            float4 v = __ldcg(reinterpret_cast<const float4 *>(xb + k));
            if (norm) v = normed(v, inv, __ldg(reinterpret_cast<const float4 *>(p.norm_w + k)));
            store_digits<FMT>(p, xdig, b, k, v, sc, finite);
        }
    }
}

// ---- epilogue on one finished 16-row tile held in shared memory [16][batch] --
__device__ void tile_epilogue(const GemvParams &p, uint32_t tile, const float *tb, unsigned long long *cta_key,
                              int lane)
{
    const uint32_t B = p.batch;
    // uniform trip count: every lane takes part in the shuffles of LOGITS
    for (uint32_t base = 0; base < 16 * B; base += 32) {
        const uint32_t idx = base + lane;
        const bool valid = idx < 16 * B;
        const uint32_t r = idx & 15, item = valid ? (idx >> 4) : 0;
        const uint32_t row = valid ? tile * 16 + r : 0xFFFFFFFFu;
        const float v = valid ? tb[r * B + item] : 0.0f;
        if (!valid && p.epilogue != B2_EPI_LOGITS) continue;
        switch (p.epilogue) {
        case B2_EPI_STORE:
            if (row < p.rows) p.out[(size_t)item * p.out_stride + row] = v;
            break;
        case B2_EPI_RESID:
            if (row < p.rows) {
                const size_t o = (size_t)item * p.out_stride + row;
                p.out[o] = __fadd_rn(__ldcg(p.resid + o), v);  // src/transformer_block.c:63-72
            }
            break;
        case B2_EPI_QKV: {
            if (row >= p.rows) break;
            const uint32_t hd = p.kv.head_dim;
            const int32_t pos = p.positions[item];
            const uint32_t cap = p.kv.pages_per_seq * p.kv.page_tokens;
            if (row < p.q_rows + p.kv_rows) {
                // RoPE on q and k (src/rope.c:20-30): interleaved pairs of a head
                const uint32_t rr = row < p.q_rows ? row : row - p.q_rows;
                const uint32_t i = rr % hd;
                const float x0 = tb[(r & ~1u) * B + item], x1 = tb[(r | 1u) * B + item];
                const float ang = __fmul_rn((float)pos, p.rope_freq[i >> 1]);
                float s, c;
                sincosf(ang, &s, &c);
                const float y = (i & 1u) ? __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c))
                                         : __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
                if (row < p.q_rows) {
                    p.out[(size_t)item * p.out_stride + row] = y;
                } else if (pos >= 0 && (uint32_t)pos < cap) {
                    const int32_t page = p.kv.page_table[(size_t)item * p.kv.pages_per_seq + pos / p.kv.page_tokens];
                    const size_t slot = (size_t)page * p.kv.page_tokens + pos % p.kv.page_tokens;
                    p.kv.k_pool[slot * p.kv.n_kv_heads * hd + rr] = y;
                } else {
                    raise_error(p.err, B2_ERR_POSITION);
                }
            } else {
                const uint32_t rr = row - p.q_rows - p.kv_rows;
                if (pos >= 0 && (uint32_t)pos < cap) {
                    const int32_t page = p.kv.page_table[(size_t)item * p.kv.pages_per_seq + pos / p.kv.page_tokens];
                    const size_t slot = (size_t)page * p.kv.page_tokens + pos % p.kv.page_tokens;
                    p.kv.v_pool[slot * p.kv.n_kv_heads * hd + rr] = v;
                } else {
                    raise_error(p.err, B2_ERR_POSITION);
                }
            }
            break;
        }
        case B2_EPI_SWIGLU:
            if (r < 8) {
                const uint32_t j = tile * 8 + r;
                if (j < p.rows / 2) {
                    const float g = v, u = tb[(r + 8) * B + item];
                    // src/ffn.c:7 silu(g) = g / (1 + expf(-g)); then * up
                    p.out[(size_t)item * p.out_stride + j] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
                }
            }
            break;
        case B2_EPI_LOGITS: {
            unsigned long long key = 0ull;
            if (row < p.rows) {
                p.out[(size_t)item * p.out_stride + row] = v;
                if (v != v) {
                    raise_error(p.err, B2_ERR_NAN_LOGITS);
                } else {
                    key = ((unsigned long long)ordered_key(v) << 32) | (0xFFFFFFFFu - row);
                }
            }
            // max over the 16 lanes of this item (lanes 16*k .. 16*k+15)
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                key = other > key ? other : key;
            }
            if ((lane & 15) == 0 && valid) atomicMax(&cta_key[item], key);
            break;
        }
        default:
            break;
        }
    }
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// The mbarrier arrives once this thread's cp.async copies issued so far land.
__device__ __forceinline__ void cp_async_arrive(uint64_t *bar)
{
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// The stage sequence of a CTA over its k-columns (a k-column is the 16 units
// of one k-unit of a panel, contiguous in memory): stage i covers columns
// [u, u + n) with n = min(kStageCols, end of the CTA range, end of the panel).
struct StageWalk {
    uint32_t u, ce, pend;
    uint32_t panel, kunits;
    __device__ StageWalk(uint32_t cb, uint32_t ce_, uint32_t kunits_) : u(cb), ce(ce_), kunits(kunits_)
    {
        panel = cb / kunits_;
        pend = (panel + 1) * kunits_;
    }
    __device__ bool more() const { return u < ce; }
    __device__ uint32_t n() const
    {
        uint32_t e = u + kStageCols;
        if (e > ce) e = ce;
        if (e > pend) e = pend;
        return e - u;
    }
    __device__ void advance(uint32_t n)
    {
        u += n;
        if (u == pend) {
            ++panel;
            pend += kunits;
        }
    }
};

template <int FMT, int NI>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const GemvParams p)
{
    constexpr uint32_t UB = Fmt<FMT>::kUnitBytes;
    constexpr uint32_t KW = Fmt<FMT>::kKW;
    constexpr uint32_t CB = kPanelTiles * UB;  // bytes of one k-column
    extern __shared__ __align__(128) uint8_t smem[];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t B = p.batch;
    const uint32_t NS = p.stages;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kMaxStages;
    uint8_t *ring = smem + p.off_ring;
    uint8_t *xdig = smem + p.off_xdig;
    float *tbufs = reinterpret_cast<float *>(smem + p.off_tile);      // [kWarps][16*B]
    float *red = reinterpret_cast<float *>(smem + p.off_misc);        // [kMaxItems][kWarps][2]
    float *item_scale = red + kMaxItems * kWarps * 2;                 // [kMaxItems]
    unsigned long long *cta_key = reinterpret_cast<unsigned long long *>(item_scale + kMaxItems);

    // k-columns; the host guarantees G <= C and C * G < 2^32
    const uint32_t C = p.panels * p.kunits, G = gridDim.x;
    const uint32_t cb = blockIdx.x * C / G, ce = (blockIdx.x + 1) * C / G;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);          // producer lane 0 + the copy's bytes
            mbar_init(&empty[s], kWarps);    // one arrival per consumer warp
        }
        fence_mbar_init();
    }
    if (threadIdx.x < kMaxItems) cta_key[threadIdx.x] = 0ull;
    __syncthreads();

    if (warp == kWarps) {
        // ---------------- producer warp: copy the CTA's stages ---------------------
        StageWalk sw(cb, ce, p.kunits);
        bool waited = false;
        for (uint32_t i = 0; sw.more(); ++i) {
            const uint32_t slot = i % NS, n = sw.n();
            if (i >= NS) {
                if (!waited) {
                    pdl_wait();
                    pdl_launch_dependents();
                    waited = true;
                }
                if (!mbar_wait_bounded(&empty[slot], ((i / NS) - 1) & 1u, p.err)) break;
            }
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[slot], n * CB);
                bulk_g2s(ring + (size_t)slot * kStageUnits * UB, p.data + (size_t)sw.u * CB, n * CB, &full[slot]);
            }
            __syncwarp();
            sw.advance(n);
        }
        if (!waited) {
            pdl_wait();
            pdl_launch_dependents();
        }
        return;
    }

    // ---------------- consumer warps: warp w owns tile w of every panel ----------------
    const int g = lane >> 2, t = lane & 3;
    pdl_wait();
    pdl_launch_dependents();
    prepare_x<FMT>(p, xdig, item_scale, red);
    consumer_sync();

    const uint32_t digit = g & 3;
    float acc[NI][2];
    int iacc[NI][4];
#pragma unroll
    for (int j = 0; j < NI; ++j) {
        acc[j][0] = acc[j][1] = 0.0f;
        iacc[j][0] = iacc[j][1] = iacc[j][2] = iacc[j][3] = 0;
    }
    bool dead = false;       // a wait timed out: keep the stage protocol, skip the math
    float *mytbuf = tbufs + (size_t)warp * 16 * B;

    StageWalk sw(cb, ce, p.kunits);
    for (uint32_t i = 0; sw.more(); ++i) {
        const uint32_t slot = i % NS, n = sw.n();
        const uint32_t ku0 = sw.u - sw.panel * p.kunits;
        if (!dead) {
            const bool got = mbar_wait_bounded(&full[slot], (i / NS) & 1u, p.err);
            dead = !__all_sync(0xffffffffu, got);
        }
        if (!dead) {
            const uint8_t *stage = ring + (size_t)slot * kStageUnits * UB;
#pragma unroll
            for (int m = 0; m < kStageCols; ++m) {
                if ((uint32_t)m < n) {
                    const uint8_t *unit = stage + ((size_t)m * kPanelTiles + warp) * UB;
                    const uint32_t ku = ku0 + m;
                    const uint4 wv = *reinterpret_cast<const uint4 *>(unit + lane * 16);
                    if (FMT == 4) {
                        const float4 sc = *reinterpret_cast<const float4 *>(unit + 512 + g * 16);
                        const uint32_t M = 0xF0F0F0F0u;
                        const uint32_t a00 = (wv.x << 4) & M, a01 = (wv.y << 4) & M, a02 = wv.x & M, a03 = wv.y & M;
                        const uint32_t a10 = (wv.z << 4) & M, a11 = (wv.w << 4) & M, a12 = wv.z & M, a13 = wv.w & M;
#pragma unroll
                        for (int j = 0; j < NI; ++j) {
                            const uint32_t item = 2 * j + (g >> 2);
                            uint4 bf = make_uint4(0, 0, 0, 0);
                            if (digit < 3 && item < B)
                                bf = *reinterpret_cast<const uint4 *>(xdig + ((size_t)(ku * B + item) * 3 + digit) * KW + t * 16);
                            int d[4], e[4];
                            imma_16832(d, a00, a01, a02, a03, bf.x, bf.y, 0, 0, 0, 0);
                            imma_16832(e, a10, a11, a12, a13, bf.z, bf.w, 0, 0, 0, 0);
                            acc[j][0] = fmaf((float)(d[0] + 256 * d[1]), sc.x, acc[j][0]);
                            acc[j][1] = fmaf((float)(d[2] + 256 * d[3]), sc.z, acc[j][1]);
                            acc[j][0] = fmaf((float)(e[0] + 256 * e[1]), sc.y, acc[j][0]);
                            acc[j][1] = fmaf((float)(e[2] + 256 * e[3]), sc.w, acc[j][1]);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < NI; ++j) {
                            const uint32_t item = 2 * j + (g >> 2);
                            uint2 bf = make_uint2(0, 0);
                            if (digit < 3 && item < B)
                                bf = *reinterpret_cast<const uint2 *>(xdig + ((size_t)(ku * B + item) * 3 + digit) * KW + t * 8);
                            imma_16832(iacc[j], wv.x, wv.y, wv.z, wv.w, bf.x, bf.y, iacc[j][0], iacc[j][1], iacc[j][2],
                                       iacc[j][3]);
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);

        const uint32_t panel = sw.panel;
        const uint32_t pfirst = panel * p.kunits, pend = sw.pend;
        sw.advance(n);
        if (sw.u != pend && sw.u != ce) continue;

        // ---- end of this CTA's part of the panel: this warp's tile is complete
        // over the CTA's columns; no other warp holds a share of it
        const uint32_t tile = panel * kPanelTiles + warp;
#pragma unroll
        for (int j = 0; j < NI; ++j) {
            float v0, v1;
            if (FMT == 4) {
                v0 = acc[j][0];
                v1 = acc[j][1];
            } else {
                v0 = __fadd_rn((float)iacc[j][0], __fmul_rn(256.0f, (float)iacc[j][1]));
                v1 = __fadd_rn((float)iacc[j][2], __fmul_rn(256.0f, (float)iacc[j][3]));
            }
            const float h0 = __shfl_down_sync(0xffffffffu, v0, 1);
            const float h1 = __shfl_down_sync(0xffffffffu, v1, 1);
            const uint32_t item = 2 * j + (t >> 1);
            if ((t & 1) == 0 && item < B) {
                const float s = item_scale[item];
                float y0 = __fmul_rn(__fadd_rn(v0, __fmul_rn(65536.0f, h0)), s);
                float y1 = __fmul_rn(__fadd_rn(v1, __fmul_rn(65536.0f, h1)), s);
                if (FMT == 8) {
                    const uint32_t r0 = tile * 16 + g, r1 = r0 + 8;
                    y0 = __fmul_rn(y0, r0 < p.rows ? p.row_scale[r0] : 0.0f);
                    y1 = __fmul_rn(y1, r1 < p.rows ? p.row_scale[r1] : 0.0f);
                }
                mytbuf[g * B + item] = y0;
                mytbuf[(g + 8) * B + item] = y1;
            }
            acc[j][0] = acc[j][1] = 0.0f;
            iacc[j][0] = iacc[j][1] = iacc[j][2] = iacc[j][3] = 0;
        }
        __syncwarp();
        if (!(pfirst >= cb && pend <= ce)) {
            // the panel is shared with neighbouring CTAs: the last CTA to finish
            // the tile adds all segments in CTA order
            const uint32_t cf = ((pfirst + 1) * G - 1) / C, cl = (pend * G - 1) / C;
            const uint32_t nseg = cl - cf + 1;
            float *pb = p.partial + (size_t)tile * p.maxseg * 16 * B;
            for (uint32_t idx = lane; idx < 16 * B; idx += 32) pb[(blockIdx.x - cf) * 16 * B + idx] = mytbuf[idx];
            __threadfence();
            __syncwarp();
            int last = 0;
            if (lane == 0) last = (atomicAdd(&p.counters[tile], 1) == (int)nseg - 1);
            last = __shfl_sync(0xffffffffu, last, 0);
            if (!last) continue;
            __threadfence();
            for (uint32_t idx = lane; idx < 16 * B; idx += 32) {
                float s = 0.0f;
                for (uint32_t sg = 0; sg < nseg; ++sg) s = __fadd_rn(s, ld_cg(pb + (size_t)sg * 16 * B + idx));
                mytbuf[idx] = s;
            }
            if (lane == 0) p.counters[tile] = 0;
            __syncwarp();
        }
        if (!dead) tile_epilogue(p, tile, mytbuf, cta_key, lane);
        __syncwarp();
    }
    if (p.epilogue == B2_EPI_LOGITS) {
        consumer_sync();
        if (threadIdx.x < B && cta_key[threadIdx.x] != 0ull) atomicMax(&p.argmax[threadIdx.x], cta_key[threadIdx.x]);
    }
}

// ---- host side ------------------------------------------------------------------

static int g_sm_count = 0;

static int sm_count()
{
    if (g_sm_count == 0) {
        int dev = 0, n = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return 148;
        g_sm_count = n;
    }
    return g_sm_count;
}

struct GemvPlan {
    int grid;
    uint32_t maxseg;
    size_t partial_bytes;
    uint32_t counter_len;
    uint32_t smem, off_ring, off_xdig, off_tile, off_misc, stages, panels;
};

static bool plan_gemv(const b2_gemv_args *a, GemvPlan &pl)
{
    const uint32_t fmt = a->w.format;
    const uint32_t UB = fmt == 4 ? B2_Q4_UNIT_BYTES : B2_Q8_UNIT_BYTES;
    const uint32_t KW = fmt == 4 ? 64u : 32u;
    const uint32_t panels = (a->w.tiles + kPanelTiles - 1) / kPanelTiles;
    const uint64_t C = (uint64_t)panels * a->w.kunits;  // k-columns
    if (C == 0) return false;
    pl.panels = panels;
    // shared memory: mbarriers | stage ring | digit planes | per-warp tile
    // buffers | misc; the ring takes what the rest leaves, up to kMaxStages
    const uint32_t xdig = a->w.kunits * a->batch * 3 * KW;
    const uint32_t tbuf = kWarps * 16 * a->batch * 4;
    const uint32_t misc = (kMaxItems * kWarps * 2 + kMaxItems) * 4 + kMaxItems * 8;
    const uint32_t fixed = 2 * kMaxStages * 8 + 128 + xdig + 128 + tbuf + 16 + misc;
    const uint32_t per_stage = kStageUnits * UB;
    const uint32_t limit = 227u * 1024u;
    if (fixed + 2 * per_stage > limit) return false;
    uint32_t ns = (limit - fixed) / per_stage;
    if (ns > kMaxStages) ns = kMaxStages;
    pl.stages = ns;
    uint32_t off = 2 * kMaxStages * 8;
    off = (off + 127) & ~127u;
    pl.off_ring = off;
    off += ns * kStageUnits * UB;
    pl.off_xdig = off;
    off += xdig;
    off = (off + 127) & ~127u;
    pl.off_tile = off;
    off += tbuf;
    off = (off + 15) & ~15u;
    pl.off_misc = off;
    off += misc;
    pl.smem = off;
    // one CTA per SM, at least one k-column per CTA
    int grid = a->grid > 0 ? a->grid : sm_count();
    if ((uint64_t)grid > C) grid = (int)C;
    if (grid < 1) grid = 1;
    if (C * (uint64_t)grid >= (1ull << 32)) return false;  // 32-bit index arithmetic in the kernel
    pl.grid = grid;
    // CTAs sharing one panel: each holds at least minc of its kunits columns
    const uint64_t minc = C / (uint64_t)grid;
    uint64_t maxseg = (a->w.kunits + minc - 1) / minc + 1;
    if (maxseg > a->w.kunits) maxseg = a->w.kunits;
    pl.maxseg = (uint32_t)maxseg;
    pl.partial_bytes = (size_t)panels * kPanelTiles * maxseg * 16 * a->batch * sizeof(float);
    pl.partial_bytes = (pl.partial_bytes + 255) & ~(size_t)255;
    pl.counter_len = panels * kPanelTiles;
    return true;
}

template <int FMT, int NI>
static cudaError_t launch_t(const GemvParams &p, const GemvPlan &pl, int pdl, cudaStream_t st)
{
    auto fn = gemv_kernel<FMT, NI>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, p);
}

}  // namespace b2

using namespace b2;

extern "C" int b2_sm_count(void) { return sm_count(); }

extern "C" size_t b2_gemv_scratch_bytes(const b2_gemv_args *a)
{
    GemvPlan pl;
    if (a == nullptr || a->batch == 0 || !plan_gemv(a, pl)) return 0;
    return pl.partial_bytes;
}

extern "C" uint32_t b2_gemv_counters_len(const b2_gemv_args *a)
{
    GemvPlan pl;
    if (a == nullptr || a->batch == 0 || !plan_gemv(a, pl)) return 0;
    return pl.counter_len;
}

extern "C" int b2_gemv(const b2_gemv_args *a, void *stream)
{
    if (a == nullptr || a->w.data == nullptr || a->x == nullptr || a->out == nullptr) return -1;
    const b2_qweight &w = a->w;
    if ((w.format != 4 && w.format != 8) || (w.format == 8 && w.row_scale == nullptr)) return -1;
    if (a->batch == 0 || a->batch > kMaxItems || w.cols == 0 || w.cols % 32 || w.rows == 0) return -1;
    if (w.tiles != (w.rows + 15) / 16 || w.kunits != (w.format == 4 ? (w.cols + 63) / 64 : (w.cols + 31) / 32)) return -1;
    if (a->x_stride < w.cols || (a->x_stride & 3) || ((uintptr_t)a->x & 15)) return -1;
    if (a->norm_w != nullptr && (((uintptr_t)a->norm_w & 15) || !(a->eps > 0.0f))) return -1;
    if (((uintptr_t)w.data & 15)) return -1;
    switch (a->epilogue) {
    case B2_EPI_STORE:
    case B2_EPI_LOGITS:
        if (a->out_stride < w.rows) return -1;
        if (a->epilogue == B2_EPI_LOGITS && a->argmax == nullptr) return -1;
        break;
    case B2_EPI_RESID:
        if (a->out_stride < w.rows || a->resid == nullptr) return -1;
        break;
    case B2_EPI_SWIGLU:
        if ((w.rows & 15) || a->out_stride < w.rows / 2) return -1;
        break;
    case B2_EPI_QKV: {
        const b2_kv_layout &kv = a->kv;
        if (!kv.k_pool || !kv.v_pool || !kv.page_table || !a->positions || !a->rope_freq) return -1;
        if (kv.head_dim == 0 || kv.head_dim % 16 || kv.page_tokens == 0 || kv.pages_per_seq == 0) return -1;
        if (a->q_rows % kv.head_dim || a->kv_rows != kv.n_kv_heads * kv.head_dim) return -1;
        if (a->q_rows + 2 * a->kv_rows != w.rows || a->out_stride < a->q_rows) return -1;
        break;
    }
    default:
        return -1;
    }
    GemvPlan pl;
    if (!plan_gemv(a, pl)) return -9;  // batch x columns too large for on-chip digit planes
    if (a->scratch == nullptr || a->scratch_bytes < pl.partial_bytes || ((uintptr_t)a->scratch & 255)) return -1;
    if (a->counters == nullptr || a->counters_len < pl.counter_len) return -1;

    GemvParams p = {};
    p.data = (const uint8_t *)w.data;
    p.row_scale = w.row_scale;
    p.rows = w.rows;
    p.cols = w.cols;
    p.tiles = w.tiles;
    p.kunits = w.kunits;
    p.panels = pl.panels;
    p.batch = a->batch;
    p.x = a->x;
    p.x_stride = a->x_stride;
    p.norm_w = a->norm_w;
    p.eps = a->eps;
    p.epilogue = a->epilogue;
    p.out = a->out;
    p.out_stride = a->out_stride;
    p.resid = a->resid;
    p.q_rows = a->q_rows;
    p.kv_rows = a->kv_rows;
    p.rope_freq = a->rope_freq;
    p.positions = a->positions;
    p.kv = a->kv;
    p.argmax = a->argmax;
    p.partial = (float *)a->scratch;
    p.counters = (int *)a->counters;
    p.maxseg = pl.maxseg;
    p.err = a->err;
    p.off_ring = pl.off_ring;
    p.stages = pl.stages;
    p.off_xdig = pl.off_xdig;
    p.off_tile = pl.off_tile;
    p.off_misc = pl.off_misc;

    const int NI = (a->batch + 1) / 2;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    if (w.format == 4) {
        if (NI <= 1) e = launch_t<4, 1>(p, pl, a->pdl, st);
        else if (NI <= 2) e = launch_t<4, 2>(p, pl, a->pdl, st);
        else if (NI <= 4) e = launch_t<4, 4>(p, pl, a->pdl, st);
        else e = launch_t<4, 8>(p, pl, a->pdl, st);
    } else {
        if (NI <= 1) e = launch_t<8, 1>(p, pl, a->pdl, st);
        else if (NI <= 2) e = launch_t<8, 2>(p, pl, a->pdl, st);
        else if (NI <= 4) e = launch_t<8, 4>(p, pl, a->pdl, st);
        else e = launch_t<8, 8>(p, pl, a->pdl, st);
    }
    return e == cudaSuccess ? 0 : -8;
}

// ---- GEMV without any allocation ------------------------------------------------
//
// For callers that cannot allocate device memory at the point where they run a
// GEMV: code that runs inside a memory pool or arena it does not own, code
// that must not synchronise the device (cudaMalloc/cudaFree can), and hosts
// whose allocator is closed to plugins. b2_gemv needs a partial-sum buffer and
// a counter array from the caller; b2_gemv_noalloc takes both from one fixed
// array in device global memory instead, so the caller passes only inputs,
// outputs and the stream.
//
// The array is B2_NOALLOC_SCRATCH_BYTES long and lives in every GPU that loads
// this library until the process exits. A call whose tiling needs more than
// that is rejected with ATT1_ERR_UNSUPPORTED (-9) before anything is launched.
// All calls on a device share the array: calls that overlap on the GPU (two
// streams, or two host threads) race on it and must be ordered by the caller.
// The array keeps the last call's contents; the counters that must start at
// zero are cleared by an asynchronous memset at every call, so a call that was
// cut short (a timed-out wait) does not poison the next one.
//
// The first call on each device looks up the array's device address with
// cudaGetSymbolAddress (once per device, with that device current) and caches
// it; that first call should come before any stream capture on that device.

static __device__ __align__(256) unsigned char g_noalloc_scratch[B2_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
void *g_noalloc_base[kMaxDevices];
std::mutex g_noalloc_mutex;
}  // namespace

extern "C" int b2_gemv_noalloc(const b2_gemv_args *a, void *stream)
{
    if (a == nullptr) return -1;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -8;
    void *base = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mutex);
        if (g_noalloc_base[dev] == nullptr) {
            // host code only holds a stand-in for g_noalloc_scratch: ask the
            // runtime for the device address of this device's copy
            void *p = nullptr;
            if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return -8;
            g_noalloc_base[dev] = p;
        }
        base = g_noalloc_base[dev];
    }
    b2_gemv_args c = *a;
    c.scratch = nullptr;
    c.counters = nullptr;
    const size_t need = b2_gemv_scratch_bytes(&c);
    const uint32_t ncnt = b2_gemv_counters_len(&c);
    if (need == 0 || ncnt == 0) return -1;
    const size_t cnt_bytes = ((size_t)ncnt * sizeof(int32_t) + 255) & ~(size_t)255;
    if (cnt_bytes + need > (size_t)B2_NOALLOC_SCRATCH_BYTES) return -9;
    c.counters = reinterpret_cast<int32_t *>(base);
    c.counters_len = ncnt;
    c.scratch = reinterpret_cast<uint8_t *>(base) + cnt_bytes;
    c.scratch_bytes = need;
    if (cudaMemsetAsync(c.counters, 0, (size_t)ncnt * sizeof(int32_t), (cudaStream_t)stream) != cudaSuccess) return -8;
    return b2_gemv(&c, stream);
}
