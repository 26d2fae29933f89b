// b2_gemv.cuh - device side of the q4/q8 block-dequant GEMV.
//
// Shared by the standalone GEMV kernel (b2_gemv.cu) and the persistent decode
// kernel (b2_decode.cu): parameters, the x prologue (RMSNorm, exponent,
// digit planes), the tile epilogues, and the producer / consumer halves of
// the bulk-copy ring. The design notes are in b2_gemv.cu.
#pragma once

#include "b2_common.cuh"

#include <cfloat>
#include <cuda_runtime.h>

namespace b2 {

constexpr int kWarps = 16;                          // consumer warps (16 hide the math latency)
constexpr int kConsumers = kWarps * 32;
constexpr int kThreads = kConsumers + 32;           // + one producer warp
constexpr int kStageUnits = 64;                     // units per stage: 40 KB of q4, one bulk copy
constexpr int kMaxStages = 8;                       // ring depth, chosen per launch
constexpr uint32_t kPreferStages = 5;               // ring depth kept before tile sums get more room
constexpr uint32_t kEarlyStages = 2;                // weight stages requested before x's digits are ready
constexpr int kMaxItems = 16;
constexpr int kConsumerBarrier = 1;                 // named barrier of the consumer warps

struct GemvParams {
    const uint8_t *data;
    const float *row_scale;
    uint32_t rows, cols, tiles, kunits;
    uint32_t round_tiles;  // tiles reduced together in shared memory (a round)
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
    uint32_t grid;  // CTAs taking part (the first `grid` CTAs of the launch)
    int32_t *err;
    b2_tp tp;       // tensor-parallel exchange (world <= 1: none)
    // shared-memory carve-up (bytes)
    uint32_t off_ring, off_xdig, off_tile, off_parts, off_misc, stages;
};

__device__ __forceinline__ bool tp_in(const GemvParams &p) { return p.tp.world > 1 && p.tp.in_point != B2_TP_NONE; }

// Input element group k..k+3 of item b: x, or under tensor parallelism the
// residual plus every rank's slot of the input point, added in rank order.
__device__ __forceinline__ float4 load_x4(const GemvParams &p, uint32_t b, uint32_t k)
{
    if (!tp_in(p)) return __ldcg(reinterpret_cast<const float4 *>(p.x + (size_t)b * p.x_stride + k));
    uint8_t *own = p.tp.peer[p.tp.rank];
    const size_t o = (size_t)b * p.cols + k;
    float4 v = __ldcg(reinterpret_cast<const float4 *>(tp_slot(own, p.tp, p.tp.in_point, 0) + o));
    for (uint32_t s = 1; s < p.tp.world; ++s) {
        const float4 w = __ldcg(reinterpret_cast<const float4 *>(tp_slot(own, p.tp, p.tp.in_point, s) + o));
        v = make_float4(__fadd_rn(v.x, w.x), __fadd_rn(v.y, w.y), __fadd_rn(v.z, w.z), __fadd_rn(v.w, w.w));
    }
    const float4 r = __ldcg(reinterpret_cast<const float4 *>(p.tp.in_resid + o));
    v = make_float4(__fadd_rn(r.x, v.x), __fadd_rn(r.y, v.y), __fadd_rn(r.z, v.z), __fadd_rn(r.w, v.w));
    if (p.tp.in_out != nullptr && blockIdx.x == 0) *reinterpret_cast<float4 *>(p.tp.in_out + o) = v;
    return v;
}

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
    // q = round(v * sc), |q| < 2^22, as balanced base-256 digits d0 + 256 d1 +
    // 65536 d2 (each in [-128, 127]): digit i is byte i of q + 0x808080 minus
    // 128. sc is a power of two, so v * sc is exact and adding 1.5 * 2^23
    // rounds it to an integer in the low mantissa bits (round to nearest even,
    // as a float-to-int conversion); byte permutes then gather the four
    // elements' digits into one word per plane.
    uint32_t u[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        u[i] = finite ? __float_as_uint(__fmaf_rn(vv[i], sc, 12582912.0f)) - (0x4B400000u - 0x808080u) : 0x808080u;
    const uint32_t lo01 = __byte_perm(u[0], u[1], 0x5140), lo23 = __byte_perm(u[2], u[3], 0x5140);
    const uint32_t hi01 = __byte_perm(u[0], u[1], 0x0062), hi23 = __byte_perm(u[2], u[3], 0x0062);
    const uint32_t w0 = __byte_perm(lo01, lo23, 0x5410) ^ 0x80808080u;
    const uint32_t w1 = __byte_perm(lo01, lo23, 0x7632) ^ 0x80808080u;
    const uint32_t w2 = __byte_perm(hi01, hi23, 0x5410) ^ 0x80808080u;
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
                                           float *sc_out, bool *finite_out, float *item_scale, bool writer)
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
    if (writer) {
        item_scale[b] = ldexpf(1.0f, E - (FMT == 4 ? 4 : 0));
        if (!finite) raise_error(p.err, B2_ERR_NONFINITE);
    }
}

template <int FMT, int NI>
__device__ void prepare_x(const GemvParams &p, uint8_t *xdig, float *item_scale, float *red)
{
    const uint32_t cols = p.cols;
    const uint32_t stride = kConsumers * 4;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool norm = p.norm_w != nullptr;
    if (tp_in(p)) {
        // every rank's contribution to the input must have landed
        int *ok = reinterpret_cast<int *>(red);
        if (threadIdx.x == 0) *ok = tp_wait(p.tp, p.tp.in_point, p.err) ? 1 : 0;
        consumer_sync();
    }
    if (p.batch == 1 && cols <= stride * kPrologueVec) {
        float4 v[kPrologueVec], w[kPrologueVec];
#pragma unroll
        for (int i = 0; i < kPrologueVec; ++i) {
            const uint32_t k = threadIdx.x * 4 + i * stride;
            const bool in = k < cols;
            v[i] = in ? load_x4(p, 0, k) : make_float4(0, 0, 0, 0);
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
        item_setup<FMT>(p, 0, tss, tmw, &inv, &sc, &finite, item_scale, threadIdx.x == 0);
#pragma unroll
        for (int i = 0; i < kPrologueVec; ++i) {
            const uint32_t k = threadIdx.x * 4 + i * stride;
            if (k < cols) store_digits<FMT>(p, xdig, 0, k, norm ? normed(v[i], inv, w[i]) : v[i], sc, finite);
        }
        return;
    }
    if constexpr (NI == 1) {
        // one or two items (the decode kernels of batch 1 and 2): the items one
        // after another. This instantiation also runs the batch-1 step, whose
        // kernel stays as small as it was (the wider path below, compiled into it,
        // made the batch-1 step 8 % slower).
        float *stats = red;  // [kMaxItems][kWarps][2]
        for (uint32_t b = 0; b < p.batch; ++b) {
            float ss = 0.0f, mw = 0.0f;
            for (uint32_t k = threadIdx.x * 4; k < cols; k += stride) {
                const float4 v = load_x4(p, b, k);
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
            item_setup<FMT>(p, b, tss, tmw, &inv, &sc, &finite, item_scale, threadIdx.x == 0);
            for (uint32_t k = threadIdx.x * 4; k < cols; k += stride) {
                float4 v = load_x4(p, b, k);
                if (norm) v = normed(v, inv, __ldg(reinterpret_cast<const float4 *>(p.norm_w + k)));
                store_digits<FMT>(p, xdig, b, k, v, sc, finite);
            }
        }
    } else {
        // general path (several items, or a row longer than the registers hold):
        // the items side by side, kConsumers / Bp threads (whole warps) each, Bp the
        // batch rounded up to a power of two. One pass of loads for every item, the
        // item's statistics from its own warps in warp order, then the digits, from
        // registers when a thread's share of the row fits them. (Taking the items
        // one after another costs a load round trip and a reduction per item.)
        uint32_t Bp = 1;
        while (Bp < p.batch) Bp <<= 1;
        const uint32_t TPI = kConsumers / Bp, wpi = TPI / 32;
        const uint32_t b = threadIdx.x / TPI, u = threadIdx.x % TPI;
        const bool live = b < p.batch;
        const uint32_t istride = TPI * 4;
        const bool held = cols <= istride * kPrologueVec;
        float *stats = red;  // [kWarps][2]
        float ss = 0.0f, mw = 0.0f;
        float4 v[kPrologueVec], w[kPrologueVec];
        if (held) {
    #pragma unroll
            for (int i = 0; i < kPrologueVec; ++i) {
                const uint32_t k = u * 4 + i * istride;
                const bool in = live && k < cols;
                v[i] = in ? load_x4(p, b, k) : make_float4(0, 0, 0, 0);
                w[i] = (in && norm) ? __ldg(reinterpret_cast<const float4 *>(p.norm_w + k)) : make_float4(1, 1, 1, 1);
            }
    #pragma unroll
            for (int i = 0; i < kPrologueVec; ++i) {
                ss += sumsq4(v[i]);
                mw = fmaxf(mw, absmax4(norm ? mul4(v[i], w[i]) : v[i]));
            }
        } else if (live) {
    #pragma unroll 4
            for (uint32_t k = u * 4; k < cols; k += istride) {
                const float4 x = load_x4(p, b, k);
                ss += sumsq4(x);
                mw = fmaxf(mw, absmax4(norm ? mul4(x, __ldg(reinterpret_cast<const float4 *>(p.norm_w + k))) : x));
            }
        }
        ss = warp_sum(ss);
        mw = warp_max(mw);
        if (lane == 0) {
            stats[warp * 2] = ss;
            stats[warp * 2 + 1] = mw;
        }
        consumer_sync();
        if (!live) return;
        float tss = 0.0f, tmw = 0.0f;
        for (uint32_t j = 0; j < wpi; ++j) {
            tss += stats[(b * wpi + j) * 2];
            tmw = fmaxf(tmw, stats[(b * wpi + j) * 2 + 1]);
        }
        float inv, sc;
        bool finite;
        item_setup<FMT>(p, b, tss, tmw, &inv, &sc, &finite, item_scale, u == 0);
        if (held) {
    #pragma unroll
            for (int i = 0; i < kPrologueVec; ++i) {
                const uint32_t k = u * 4 + i * istride;
                if (k < cols) store_digits<FMT>(p, xdig, b, k, norm ? normed(v[i], inv, w[i]) : v[i], sc, finite);
            }
        } else {
    #pragma unroll 4
            for (uint32_t k = u * 4; k < cols; k += istride) {
                float4 x = load_x4(p, b, k);
                if (norm) x = normed(x, inv, __ldg(reinterpret_cast<const float4 *>(p.norm_w + k)));
                store_digits<FMT>(p, xdig, b, k, x, sc, finite);
            }
        }
    }
}

// ---- epilogue on one finished 16-row tile held in shared memory [16][batch] --
static __device__ void tile_epilogue(const GemvParams &p, uint32_t tile, const float *tb, unsigned long long *cta_key,
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
                    p.kv.k_pool[(((size_t)page * p.kv.n_kv_heads + rr / hd) * p.kv.page_tokens +
                                 pos % p.kv.page_tokens) * hd + rr % hd] = y;
                } else {
                    raise_error(p.err, B2_ERR_POSITION);
                }
            } else {
                const uint32_t rr = row - p.q_rows - p.kv_rows;
                if (pos >= 0 && (uint32_t)pos < cap) {
                    const int32_t page = p.kv.page_table[(size_t)item * p.kv.pages_per_seq + pos / p.kv.page_tokens];
                    p.kv.v_pool[(((size_t)page * p.kv.n_kv_heads + rr / hd) * p.kv.page_tokens +
                                 pos % p.kv.page_tokens) * hd + rr % hd] = v;
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
        case B2_EPI_PUSH:
            // tensor parallel partial: into this rank's slot on every rank
            if (row < p.rows)
                for (uint32_t s = 0; s < p.tp.world; ++s)
                    tp_slot(p.tp.peer[s], p.tp, p.tp.out_point, p.tp.rank)[(size_t)item * p.rows + row] = v;
            break;
        case B2_EPI_LOGITS: {
            unsigned long long key = 0ull;
            if (row < p.rows) {
                p.out[(size_t)item * p.out_stride + row] = v;
                if (p.tp.world > 1)  // all-gather of the vocabulary shards
                    for (uint32_t s = 0; s < p.tp.world; ++s)
                        tp_slot(p.tp.peer[s], p.tp, p.tp.out_point, p.tp.rank)[(size_t)item * p.rows + row] = v;
                if (v != v) {
                    raise_error(p.err, B2_ERR_NAN_LOGITS);
                } else {
                    key = ((unsigned long long)ordered_key(v) << 32) | (0xFFFFFFFFu - (p.tp.row_offset + row));
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


// Tiles of at least kSplitStageUnits units end a stage (a stage then holds
// one tile's units); narrower tiles share stages.
constexpr uint32_t kSplitStageUnits = 16;

// The stage sequence of a CTA over its units (whole tiles [t0, t1), each
// tile's k-units contiguous): stage i covers units [u, u + n) with
// n = min(kStageUnits, end of the current round of round-tiles tiles, end of
// the tile when tiles are at least kSplitStageUnits units).
struct StageWalk {
    uint32_t u, ce, rend, kunits, rtiles, tend;
    __device__ StageWalk(uint32_t t0, uint32_t t1, uint32_t kunits_, uint32_t rtiles_)
        : u(t0 * kunits_), ce(t1 * kunits_), kunits(kunits_), rtiles(rtiles_)
    {
        rend = min(t1, t0 + rtiles_) * kunits_;
        tend = u + kunits_;
    }
    __device__ bool more() const { return u < ce; }
    __device__ uint32_t n() const
    {
        uint32_t e = u + kStageUnits;
        if (e > rend) e = rend;
        if (kunits >= kSplitStageUnits && e > tend) e = tend;
        return e - u;
    }
    // advance; true at the end of a round
    __device__ bool advance(uint32_t n)
    {
        u += n;
        if (u == tend) tend += kunits;
        if (u == rend) {
            rend = min(ce, rend + rtiles * kunits);
            return true;
        }
        return false;
    }
};

// Shared-memory view of the GEMV pipeline (same carve-up in both kernels).
struct GemvSmem {
    uint64_t *full, *empty;
    uint8_t *ring, *xdig;
    float *tbufs, *red, *item_scale;
    float *parts;  // [round tiles][kWarps][16 * batch] per-warp tile sums
    unsigned long long *cta_key;
    uint64_t *xready;  // arrives when x's digit planes are in place (null: no gate)
    uint32_t stages;
};

__device__ __forceinline__ GemvSmem gemv_smem(uint8_t *smem, const GemvParams &p)
{
    GemvSmem s;
    s.full = reinterpret_cast<uint64_t *>(smem);
    s.empty = s.full + kMaxStages;
    s.ring = smem + p.off_ring;
    s.xdig = smem + p.off_xdig;
    s.tbufs = reinterpret_cast<float *>(smem + p.off_tile);   // [kWarps][16*B]
    s.parts = reinterpret_cast<float *>(smem + p.off_parts);  // [round_tiles][kWarps][16*B]
    s.red = reinterpret_cast<float *>(smem + p.off_misc);     // [kMaxItems][kWarps][2]
    s.item_scale = s.red + kMaxItems * kWarps * 2;            // [kMaxItems]
    s.cta_key = reinterpret_cast<unsigned long long *>(s.item_scale + kMaxItems);
    s.xready = nullptr;
    s.stages = p.stages;
    return s;
}

// Barriers of the ring: "full" completes on the producer's arrival plus the
// bytes of the copy, "empty" on one arrival per consumer warp.
__device__ __forceinline__ void gemv_init_barriers(const GemvSmem &s)
{
    for (uint32_t i = 0; i < s.stages; ++i) {
        mbar_init(&s.full[i], 1);
        mbar_init(&s.empty[i], kWarps);
    }
    if (s.xready != nullptr) mbar_init(s.xready, 1);
    fence_mbar_init();
}

// The CTA's tiles [t0, t1): the first p.grid CTAs split the tiles (the
// host guarantees p.grid <= tiles and tiles * p.grid < 2^32), any further
// CTAs of a larger launch get none.
__device__ __forceinline__ void cta_range(const GemvParams &p, uint32_t &t0, uint32_t &t1)
{
    const uint32_t T = p.tiles, G = p.grid;
    if (blockIdx.x >= G) {
        t0 = t1 = 0;
        return;
    }
    t0 = blockIdx.x * T / G;
    t1 = (blockIdx.x + 1) * T / G;
}

// Producer warp: copy this CTA's stages of one GEMV into the ring. `i` counts
// stages over the life of the ring (it continues across GEMVs that share a
// ring); `waited` records that the programmatic-launch wait was taken (the
// first NS stages are requested before it). With an x-ready gate only the
// first kEarlyStages stages go out before the consumers have x's digit planes:
// the prologue's loads of x (L2 hits) otherwise queue behind a ring's worth of
// weight requests (HBM) and the prologue takes microseconds. Returns false
// after a timeout.
template <int FMT>
__device__ bool gemv_produce(const GemvParams &p, const GemvSmem &s, uint32_t &i, bool &waited)
{
    constexpr uint32_t UB = Fmt<FMT>::kUnitBytes;
    const int lane = threadIdx.x & 31;
    uint32_t t0, t1;
    cta_range(p, t0, t1);
    if (t0 == t1) return true;
    StageWalk sw(t0, t1, p.kunits, p.round_tiles);
    bool gated = s.xready != nullptr;
    for (uint32_t own = 0; sw.more(); ++i, ++own) {
        const uint32_t slot = i % s.stages, n = sw.n();
        if (i >= s.stages || (gated && own >= kEarlyStages)) {
            if (!waited) {
                pdl_wait();
                pdl_launch_dependents();
                waited = true;
            }
            if (gated) {
                if (!mbar_wait_bounded(s.xready, 0, p.err)) return false;
                gated = false;
            }
            if (i >= s.stages && !mbar_wait_bounded(&s.empty[slot], ((i / s.stages) - 1) & 1u, p.err)) return false;
        }
        if (lane == 0) {
            mbar_arrive_expect_tx(&s.full[slot], n * UB);
            bulk_g2s_stream(s.ring + (size_t)slot * kStageUnits * UB, p.data + (size_t)sw.u * UB, n * UB, &s.full[slot],
                            l2_evict_first_policy());
        }
        __syncwarp();
        sw.advance(n);
    }
    return true;
}

// Clear the CTA's argmax key and the round's per-warp tile sums (consumer
// threads). Reads nothing another kernel writes, so a launch can do it before
// its programmatic-launch wait (`prezeroed` for gemv_consume).
__device__ __forceinline__ void gemv_zero_round(const GemvParams &p, const GemvSmem &s)
{
    if (threadIdx.x < kMaxItems) s.cta_key[threadIdx.x] = 0ull;
    const uint32_t parts_n = p.round_tiles * kWarps * 16 * p.batch;
    for (uint32_t k = threadIdx.x; k < parts_n; k += kConsumers) s.parts[k] = 0.0f;
}

// Consumer warps (all kWarps of them): prologue, the CTA's stages of one GEMV
// (ring position `i`, shared with the producer's count), per-tile sums and
// epilogues. Warp w multiplies units w, w + kWarps, ... of every stage and
// keeps one tile's sums in registers; when its units move to the next tile it
// stores them in its slot of the round's per-warp tile sums. At the end of a
// round (round_tiles tiles) the warps add the slots of each tile in warp
// order (deterministic) and run the tile epilogues, one warp per tile. `dead`
// (a wait timed out) keeps the stage protocol but skips the math and stores.
template <int FMT, int NI>
__device__ void gemv_consume(const GemvParams &p, const GemvSmem &s, uint32_t &i, bool &dead, bool prezeroed = false)
{
    constexpr uint32_t UB = Fmt<FMT>::kUnitBytes;
    constexpr uint32_t KW = Fmt<FMT>::kKW;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t B = p.batch, K = p.kunits, SB = 16 * B;
    const uint32_t NS = s.stages;
    uint32_t t0, t1;
    cta_range(p, t0, t1);
    if (t0 == t1) return;  // no tiles for this CTA
    const uint32_t parts_n = p.round_tiles * kWarps * SB;
    if (!prezeroed) gemv_zero_round(p, s);
    prepare_x<FMT, NI>(p, s.xdig, s.item_scale, s.red);
    consumer_sync();
    if (s.xready != nullptr && threadIdx.x == 0) mbar_arrive(s.xready);

    const uint32_t digit = g & 3;
    float acc[NI][2];
    int iacc[NI][4];
#pragma unroll
    for (int j = 0; j < NI; ++j) {
        acc[j][0] = acc[j][1] = 0.0f;
        iacc[j][0] = iacc[j][1] = iacc[j][2] = iacc[j][3] = 0;
    }
    float *mytbuf = s.tbufs + (size_t)warp * SB;
    uint32_t round_t0 = t0;       // first tile of the current round
    uint32_t cur = 0xFFFFFFFFu;   // tile whose sums this warp holds

    // store this warp's sums of tile `cur` into its slot and clear them
    auto flush = [&]() {
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
            if ((t & 1) == 0 && item < B && cur != 0xFFFFFFFFu) {
                float *slot = s.parts + ((size_t)(cur - round_t0) * kWarps + warp) * SB;
                const float sc_item = s.item_scale[item];
                slot[g * B + item] = __fmul_rn(__fadd_rn(v0, __fmul_rn(65536.0f, h0)), sc_item);
                slot[(g + 8) * B + item] = __fmul_rn(__fadd_rn(v1, __fmul_rn(65536.0f, h1)), sc_item);
            }
            acc[j][0] = acc[j][1] = 0.0f;
            iacc[j][0] = iacc[j][1] = iacc[j][2] = iacc[j][3] = 0;
        }
    };

    StageWalk sw(t0, t1, K, p.round_tiles);
    for (; sw.more(); ++i) {
        const uint32_t slot = i % NS, n = sw.n();
        const uint32_t tile0 = sw.u / K, ku0 = sw.u - tile0 * K;
        const bool one_tile = K >= kSplitStageUnits;  // the stage holds units of tile0 only
        if (!dead) {
            const bool got = mbar_wait_bounded(&s.full[slot], (i / NS) & 1u, p.err);
            dead = !__all_sync(0xffffffffu, got);
        }
        if (one_tile && tile0 != cur && (uint32_t)warp < n) {
            flush();
            cur = tile0;
        }
        if (!dead) {
            const uint8_t *stage = s.ring + (size_t)slot * kStageUnits * UB;
            // one unit: weights and scales from the stage, digits of k-unit ku
            auto unit_math = [&](uint32_t k, uint32_t ku) {
                const uint8_t *unit = stage + (size_t)k * UB;
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
                            bf = *reinterpret_cast<const uint4 *>(s.xdig + ((size_t)(ku * B + item) * 3 + digit) * KW + t * 16);
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
                            bf = *reinterpret_cast<const uint2 *>(s.xdig + ((size_t)(ku * B + item) * 3 + digit) * KW + t * 8);
                        imma_16832(iacc[j], wv.x, wv.y, wv.z, wv.w, bf.x, bf.y, iacc[j][0], iacc[j][1], iacc[j][2],
                                   iacc[j][3]);
                    }
                }
            };
            if (one_tile) {
#pragma unroll
                for (int m = 0; m < kStageUnits / kWarps; ++m) {
                    const uint32_t k = warp + m * kWarps;
                    if (k < n) unit_math(k, ku0 + k);
                }
            } else {
                // narrow tiles share the stage (small matrices): the tile of
                // each unit, kept out of the unrolled hot loop above
#pragma unroll 1
                for (uint32_t k = warp; k < n; k += kWarps) {
                    uint32_t tile = tile0, ku = ku0 + k;
                    while (ku >= K) {
                        ku -= K;
                        ++tile;
                    }
                    if (tile != cur) {
                        flush();
                        cur = tile;
                    }
                    unit_math(k, ku);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.empty[slot]);
        if (!sw.advance(n)) continue;

        // ---- end of a round: the warps' tile sums are complete
        flush();
        cur = 0xFFFFFFFFu;
        consumer_sync();
        const uint32_t round_t1 = min(t1, round_t0 + p.round_tiles);
        for (uint32_t tile = round_t0 + warp; tile < round_t1; tile += kWarps) {
            const float *sl = s.parts + (size_t)(tile - round_t0) * kWarps * SB;
            for (uint32_t idx = lane; idx < SB; idx += 32) {
                float sum = 0.0f;
#pragma unroll
                for (int w = 0; w < kWarps; ++w) sum = __fadd_rn(sum, sl[w * SB + idx]);
                if (FMT == 8) {
                    const uint32_t row = tile * 16 + idx / B;
                    sum = __fmul_rn(sum, row < p.rows ? p.row_scale[row] : 0.0f);
                }
                mytbuf[idx] = sum;
            }
            __syncwarp();
            if (!dead) tile_epilogue(p, tile, mytbuf, s.cta_key, lane);
            __syncwarp();
        }
        consumer_sync();
        if (p.epilogue == B2_EPI_PUSH && threadIdx.x == 0) {
            // one system-scope acquire-release add per CTA round (the barrier
            // above orders every warp's peer stores before it); the round that
            // completes the GEMV on this rank has acquired all the others and
            // publishes the point with a release store (no further fence)
            const int n_round = (int)(round_t1 - round_t0);
            if (atom_add_acq_rel_sys(p.tp.done, n_round) == (int)p.tiles - n_round) {
                *p.tp.done = 0;
                tp_signal(p.tp, p.tp.out_point);
            }
        }
        for (uint32_t k = threadIdx.x; k < parts_n; k += kConsumers) s.parts[k] = 0.0f;
        round_t0 = round_t1;
        // the next round's slots are cleared before any warp stores into them
        consumer_sync();
    }
    if (p.epilogue == B2_EPI_LOGITS) {
        consumer_sync();
        if (threadIdx.x < B && s.cta_key[threadIdx.x] != 0ull) atomicMax(&p.argmax[threadIdx.x], s.cta_key[threadIdx.x]);
        if (p.tp.world > 1) {
            // the last CTA publishes this rank's logits and argmax keys
            consumer_sync();
            if (threadIdx.x == 0) {
                if (atom_add_acq_rel_sys(p.tp.done, 1) == (int)p.grid - 1) {
                    *p.tp.done = 0;
                    for (uint32_t b = 0; b < B; ++b) {
                        const uint64_t key = __ldcg(p.argmax + b);
                        for (uint32_t q = 0; q < p.tp.world; ++q) *tp_key(p.tp.peer[q], p.tp, p.tp.rank, b) = key;
                    }
                    tp_signal(p.tp, p.tp.out_point);  // release stores: the keys are ordered before
                }
            }
        }
    }
}

// ---- host side (b2_gemv.cu) -------------------------------------------------------
struct GemvPlan {
    int grid;
    size_t partial_bytes;   // scratch the caller provides (unused by the kernel; kept for the ABI)
    uint32_t counter_len;   // counters the caller provides (likewise)
    uint32_t round_tiles;
    uint32_t smem, off_ring, off_xdig, off_tile, off_parts, off_misc, stages;
};

// Argument checks of b2_gemv (0 or a negative status).
int gemv_check(const b2_gemv_args *a);
// Grid, shared-memory carve-up and scratch sizes for a standalone launch.
bool plan_gemv(const b2_gemv_args *a, GemvPlan &pl);
// Kernel parameters from checked arguments and a plan (scratch from `a`).
void gemv_params(const b2_gemv_args *a, const GemvPlan &pl, GemvParams &p);

}  // namespace b2
