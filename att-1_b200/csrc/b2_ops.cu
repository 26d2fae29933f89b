// b2_ops.cu - per-token step kernels and the element ops of the backend vtable.
//
// step_begin: embedding row copy (src/infer.c:713-715) + argmax key reset.
// step_end:   greedy token from the argmax key (src/sampler.c:5-34: lowest id
//             wins ties), position advance (src/infer.c:878).
// Element ops on device buffers, one per vtable slot of include/att1_backend.h:
// rmsnorm (src/norm.c:5-34), softmax (src/norm.c:36-71), rope (src/rope.c:5-34),
// swiglu (src/ffn.c:5-30), greedy argmax.
#include "b2_common.cuh"

#include <cfloat>
#include <cuda_runtime.h>

namespace b2 {

static cudaError_t launch_pdl(const void *fn, dim3 grid, dim3 block, int pdl, cudaStream_t st, void **args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// grid (blocks per row, batch): each thread moves float4s of the row
__global__ void step_begin_kernel(const float *embed, uint32_t vocab, uint32_t d, const uint32_t *tokens, float *x,
                                  unsigned long long *argmax, int32_t *err)
{
    pdl_wait();
    pdl_launch_dependents();
    const uint32_t item = blockIdx.y;
    const uint32_t tok = tokens[item];
    float4 *xb = reinterpret_cast<float4 *>(x + (size_t)item * d);
    const uint32_t n4 = d / 4;
    const uint32_t i0 = blockIdx.x * blockDim.x + threadIdx.x, step = gridDim.x * blockDim.x;
    if (tok >= vocab) {
        if (i0 == 0) raise_error(err, B2_ERR_TOKEN);
        for (uint32_t i = i0; i < n4; i += step) xb[i] = make_float4(0, 0, 0, 0);
    } else {
        const float4 *row = reinterpret_cast<const float4 *>(embed + (size_t)tok * d);
        for (uint32_t i = i0; i < n4; i += step) xb[i] = __ldg(row + i);
    }
    if (i0 == 0) argmax[item] = 0ull;
}

__global__ void step_end_kernel(const unsigned long long *argmax, uint32_t batch, uint32_t *tokens, int32_t *positions,
                                int32_t *err)
{
    pdl_wait();
    pdl_launch_dependents();
    const uint32_t item = threadIdx.x;
    if (item >= batch) return;
    const unsigned long long key = argmax[item];
    if (key == 0ull) {
        raise_error(err, B2_ERR_NAN_LOGITS);
    } else {
        tokens[item] = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
    }
    positions[item] += 1;
}

// Tensor parallel: the greedy token is the largest key over every rank's
// vocabulary shard (keys carry global ids); then positions and the epoch.
__global__ void step_end_tp_kernel(const b2_tp tp, uint32_t batch, uint32_t *tokens, int32_t *positions, int32_t *err)
{
    __shared__ int ok;
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x == 0) ok = tp_wait(tp, tp.points, err) ? 1 : 0;
    __syncthreads();
    const uint32_t item = threadIdx.x;
    if (item < batch) {
        unsigned long long key = 0ull;
        for (uint32_t s = 0; s < tp.world; ++s) {
            const unsigned long long k = __ldcg(tp_key(tp.peer[tp.rank], tp, s, item));
            key = k > key ? k : key;
        }
        if (!ok || key == 0ull) raise_error(err, ok ? B2_ERR_NAN_LOGITS : B2_ERR_TIMEOUT);
        else tokens[item] = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
        positions[item] += 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) *const_cast<uint32_t *>(tp.epoch) += 1;
}

// Greedy token from argmax keys gathered over `world` ranks ([world][batch]).
__global__ void step_end_keys_kernel(const unsigned long long *keys, uint32_t world, uint32_t batch, uint32_t *tokens,
                                     int32_t *positions, int32_t *err)
{
    pdl_wait();
    pdl_launch_dependents();
    const uint32_t item = threadIdx.x;
    if (item >= batch) return;
    unsigned long long key = 0ull;
    for (uint32_t s = 0; s < world; ++s) {
        const unsigned long long k = __ldcg(keys + (size_t)s * batch + item);
        key = k > key ? k : key;
    }
    if (key == 0ull) raise_error(err, B2_ERR_NAN_LOGITS);
    else tokens[item] = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
    positions[item] += 1;
}

// ---- tensor-parallel exchange for the GEMM route (the GEMVs fuse it) ----------------

// This rank's partial x[n] into its slot of `point` on every rank; the CTAs
// chain with one system-scope acquire-release add each, and the CTA that
// completes the kernel publishes the point with release stores.
__global__ void tp_push_kernel(const float *__restrict__ x, uint32_t n, const b2_tp tp, uint32_t point)
{
    pdl_wait();
    pdl_launch_dependents();
    const float4 *src = reinterpret_cast<const float4 *>(x);
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n / 4; i += gridDim.x * blockDim.x) {
        const float4 v = __ldcg(src + i);
        for (uint32_t s = 0; s < tp.world; ++s)
            reinterpret_cast<float4 *>(tp_slot(tp.peer[s], tp, point, tp.rank))[i] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0 && atom_add_acq_rel_sys(tp.done, 1) == (int)gridDim.x - 1) {
        *tp.done = 0;
        tp_signal(tp, point);
    }
}

// out = resid + the ranks' slots of `point` added in rank order, once every
// rank has published it (bounded wait).
__global__ void tp_sum_kernel(const float *resid, float *out, uint32_t n, const b2_tp tp, uint32_t point, int32_t *err)
{
    __shared__ int ok;
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x == 0) ok = tp_wait(tp, point, err) ? 1 : 0;
    __syncthreads();
    if (!ok) return;
    uint8_t *own = tp.peer[tp.rank];
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n / 4; i += gridDim.x * blockDim.x) {
        float4 v = __ldcg(reinterpret_cast<const float4 *>(tp_slot(own, tp, point, 0)) + i);
        for (uint32_t s = 1; s < tp.world; ++s) {
            const float4 w = __ldcg(reinterpret_cast<const float4 *>(tp_slot(own, tp, point, s)) + i);
            v = make_float4(__fadd_rn(v.x, w.x), __fadd_rn(v.y, w.y), __fadd_rn(v.z, w.z), __fadd_rn(v.w, w.w));
        }
        const float4 r = __ldcg(reinterpret_cast<const float4 *>(resid) + i);
        reinterpret_cast<float4 *>(out)[i] =
            make_float4(__fadd_rn(r.x, v.x), __fadd_rn(r.y, v.y), __fadd_rn(r.z, v.z), __fadd_rn(r.w, v.w));
    }
}

// This rank's logits [batch][rows] and argmax keys into every rank's logits
// slot and key row; publishes point tp.points (b2_step_end_tp waits for it).
__global__ void tp_push_logits_kernel(const float *__restrict__ logits, uint32_t batch, uint32_t rows,
                                      const unsigned long long *argmax, const b2_tp tp)
{
    pdl_wait();
    pdl_launch_dependents();
    const size_t n = (size_t)batch * rows;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = __ldcg(logits + i);
        for (uint32_t s = 0; s < tp.world; ++s) tp_slot(tp.peer[s], tp, tp.points, tp.rank)[i] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0 && atom_add_acq_rel_sys(tp.done, 1) == (int)gridDim.x - 1) {
        *tp.done = 0;
        for (uint32_t b = 0; b < batch; ++b) {
            const unsigned long long key = __ldcg(argmax + b);
            for (uint32_t q = 0; q < tp.world; ++q) *tp_key(tp.peer[q], tp, tp.rank, b) = key;
        }
        tp_signal(tp, tp.points);
    }
}

__global__ void rmsnorm_kernel(float *dst, const float *src, const float *w, uint32_t n, float eps)
{
    __shared__ float red[32];
    float ss = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(src[i], src[i], ss);
    ss = block_sum(ss, red);
    const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = __fmul_rn(__fmul_rn(src[i], inv), w[i]);
}

__global__ void softmax_kernel(float *v, uint32_t n)
{
    __shared__ float red[32];
    float m = -INFINITY;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, v[i]);
    m = block_max(m, red);
    float s = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(v[i] - m);
        v[i] = e;
        s += e;
    }
    s = block_sum(s, red);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) v[i] = __fdiv_rn(v[i], s);
}

__global__ void rope_kernel(float *v, uint32_t n, uint32_t pos, float theta)
{
    const uint32_t i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (i >= n) return;
    // src/rope.c:21-22 in f32; powf evaluated in double and rounded once, so
    // it agrees with a correctly rounded host powf
    const float e = __fdiv_rn((float)i, (float)n);
    const float freq = __fdiv_rn(1.0f, (float)pow((double)theta, (double)e));
    const float ang = __fmul_rn((float)pos, freq);
    float s, c;
    sincosf(ang, &s, &c);
    const float x0 = v[i], x1 = v[i + 1];
    v[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    v[i + 1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

__global__ void swiglu_kernel(float *dst, const float *g, const float *u, uint32_t n)
{
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float x = g[i];
        dst[i] = __fmul_rn(__fdiv_rn(x, __fadd_rn(1.0f, expf(-x))), u[i]);
    }
}

__device__ __forceinline__ uint32_t ordered_key32(float f)
{
    uint32_t b = __float_as_uint(f == 0.0f ? 0.0f : f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void argmax_kernel(const float *v, uint32_t n, unsigned long long *key)
{
    unsigned long long best = 0ull;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float f = v[i];
        if (f != f) continue;  // NaN: leaves key at 0 when every value is NaN; caller checks separately
        const unsigned long long k = ((unsigned long long)ordered_key32(f) << 32) | (0xFFFFFFFFu - i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0 && best != 0ull) atomicMax(key, best);
}

// dst[r][c] = sum_k lhs[r][k] * rhs[k][c], sequential over k per output
// (src/matmul.c order); one thread per output element, rhs reads coalesced.
__global__ void matmul_f32_kernel(float *dst, const float *lhs, const float *rhs, uint32_t rows, uint32_t cols,
                                  uint32_t inner)
{
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x, r = blockIdx.y;
    if (c >= cols) return;
    float s = 0.0f;
    for (uint32_t k = 0; k < inner; ++k) s = __fadd_rn(s, __fmul_rn(lhs[(size_t)r * inner + k], rhs[(size_t)k * cols + c]));
    dst[(size_t)r * cols + c] = s;
}

// Quantised products in the reference's own operation order, one thread per
// output: sum over groups in order, then over the group's columns, of
// x * (q * scale), each product and sum rounded on its own (no contraction),
// as src/quant.c:340-393 and src/matmul_q8.c:3-40 compiled without FMA. W is
// in the reference layout. Used by the backend vtable for the shapes the
// unit-layout GEMV does not tile (q4 group 16, columns not a multiple of 32).
__global__ void matmul_q4_ordered_kernel(float *dst, const float *lhs, uint32_t cols, const uint8_t *packed,
                                         const float *scales, uint32_t rows, uint32_t group)
{
    const uint32_t o = blockIdx.x * blockDim.x + threadIdx.x, r = blockIdx.y;
    if (o >= rows) return;
    const uint32_t ng = cols / group;
    const uint8_t *p = packed + (size_t)o * (cols / 2);
    const float *x = lhs + (size_t)r * cols;
    float sum = 0.0f;
    for (uint32_t g = 0; g < ng; ++g) {
        const float sc = scales[(size_t)o * ng + g];
        for (uint32_t j = g * group; j < (g + 1) * group; j += 2) {
            const uint32_t b = p[j >> 1];
            const float lo = (float)((int32_t)(b << 28) >> 28), hi = (float)((int32_t)(b << 24) >> 28);
            sum = __fadd_rn(sum, __fmul_rn(x[j], __fmul_rn(lo, sc)));
            sum = __fadd_rn(sum, __fmul_rn(x[j + 1], __fmul_rn(hi, sc)));
        }
    }
    dst[(size_t)r * rows + o] = sum;
}

__global__ void matmul_q8_ordered_kernel(float *dst, const float *lhs, uint32_t cols, const int8_t *values,
                                         const float *scales, uint32_t rows)
{
    const uint32_t o = blockIdx.x * blockDim.x + threadIdx.x, r = blockIdx.y;
    if (o >= rows) return;
    const int8_t *v = values + (size_t)o * cols;
    const float *x = lhs + (size_t)r * cols;
    const float sc = scales[o];
    float sum = 0.0f;
    for (uint32_t c = 0; c < cols; ++c) sum = __fadd_rn(sum, __fmul_rn(x[c], __fmul_rn((float)v[c], sc)));
    dst[(size_t)r * rows + o] = sum;
}

// ---- top-k / temperature sampling (step end, after the greedy token) --------------

constexpr int kSampleThreads = 512;

__device__ __forceinline__ uint32_t sample_key(float v) { return v != v ? 0u : ordered_key(v); }

// Exclusive prefix sum of one value per thread over the block.
__device__ uint32_t block_excl_scan(uint32_t v, uint32_t *warp_tot)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t acc = 0;
        for (int w = 0; w < kSampleThreads / 32; ++w) {
            const uint32_t t = warp_tot[w];
            warp_tot[w] = acc;
            acc += t;
        }
    }
    __syncthreads();
    const uint32_t r = warp_tot[warp] + inc - v;
    __syncthreads();
    return r;
}

// One CTA per item: the k largest logits by (value desc, id asc) through a
// 4 x 8-bit radix select of the k-th key, gathered in id order and ranked;
// weights exp((l - l_max) / T) summed in rank order; the token is the first
// rank whose running sum exceeds u * sum, u = 24 bits of
// splitmix64(splitmix64(seed) ^ (item << 32 | position)), position = the
// position after this step (the one the token will take). Logit (item, v)
// sits at logits[(v / shard_rows) * shard_stride + item * item_stride +
// v % shard_rows]: one shard for a plain [batch][stride] buffer, one per rank
// for the tensor-parallel all-gather.
__global__ void __launch_bounds__(kSampleThreads) sample_topk_kernel(const float *logits, uint32_t vocab,
                                                                     uint32_t shard_rows,
                                                                     unsigned long long shard_stride,
                                                                     uint32_t item_stride, uint32_t k,
                                                                     float temperature, unsigned long long seed,
                                                                     const int32_t *positions, uint32_t *tokens)
{
    __shared__ uint32_t hist[256];
    __shared__ uint32_t sel[3];
    __shared__ uint32_t warp_tot[kSampleThreads / 32];
    __shared__ float cv[B2_MAX_TOP_K], sv[B2_MAX_TOP_K], w[B2_MAX_TOP_K];
    __shared__ uint32_t ci[B2_MAX_TOP_K], si[B2_MAX_TOP_K];
    pdl_wait();
    pdl_launch_dependents();
    const uint32_t item = blockIdx.x, nshards = vocab / shard_rows;
    const float *L = logits + (size_t)item * item_stride;
    uint32_t prefix = 0, mask = 0, want = k;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (uint32_t b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
        __syncthreads();
        for (uint32_t s = 0; s < nshards; ++s)
            for (uint32_t i = threadIdx.x; i < shard_rows; i += blockDim.x) {
                const uint32_t key = sample_key(__ldcg(L + s * shard_stride + i));
                if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
            }
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t acc = 0, b = 255;
            while (b > 0 && acc + hist[b] < want) acc += hist[b--];
            sel[0] = prefix | (b << shift);
            sel[1] = mask | (255u << shift);
            sel[2] = want - acc;
        }
        __syncthreads();
        prefix = sel[0];
        mask = sel[1];
        want = sel[2];
        __syncthreads();
    }
    // prefix is the k-th largest key: every key above it and the `want`
    // lowest ids equal to it, in id order
    const uint32_t chunk = (vocab + blockDim.x - 1) / blockDim.x;
    const uint32_t i0 = min(threadIdx.x * chunk, vocab), i1 = min(i0 + chunk, vocab);
    const uint32_t s0 = i0 / shard_rows, r0 = i0 - s0 * shard_rows;
    uint32_t ngt = 0, neq = 0;
    for (uint32_t i = i0, s = s0, r = r0; i < i1; ++i) {
        const uint32_t key = sample_key(__ldcg(L + s * shard_stride + r));
        ngt += key > prefix;
        neq += key == prefix;
        if (++r == shard_rows) {
            r = 0;
            ++s;
        }
    }
    uint32_t ogt = block_excl_scan(ngt, warp_tot);
    uint32_t oeq = block_excl_scan(neq, warp_tot);
    const uint32_t n_gt = k - want;
    for (uint32_t i = i0, s = s0, r = r0; i < i1; ++i) {
        const float v = __ldcg(L + s * shard_stride + r);
        if (++r == shard_rows) {
            r = 0;
            ++s;
        }
        const uint32_t key = sample_key(v);
        if (key > prefix && ogt < n_gt) {
            cv[ogt] = v;
            ci[ogt] = i;
            ++ogt;
        } else if (key == prefix && oeq < want) {
            cv[n_gt + oeq] = v;
            ci[n_gt + oeq] = i;
            ++oeq;
        }
    }
    __syncthreads();
    if (threadIdx.x < k) {
        const uint32_t me = sample_key(cv[threadIdx.x]), id = ci[threadIdx.x];
        uint32_t r = 0;
        for (uint32_t j = 0; j < k; ++j) {
            const uint32_t kj = sample_key(cv[j]);
            r += (kj > me || (kj == me && ci[j] < id)) ? 1u : 0u;
        }
        sv[r] = cv[threadIdx.x];
        si[r] = id;
    }
    __syncthreads();
    // a +inf top logit takes all the probability: the +inf entries share it
    // equally (exp of inf - inf would be NaN)
    if (threadIdx.x < k)
        w[threadIdx.x] = sv[0] == INFINITY ? (sv[threadIdx.x] == INFINITY ? 1.0f : 0.0f)
                                           : expf(__fdiv_rn(__fsub_rn(sv[threadIdx.x], sv[0]), temperature));
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t j = 0;
        if (sv[0] != -INFINITY) {
            float s = 0.0f;
            for (uint32_t q = 0; q < k; ++q) s = __fadd_rn(s, w[q]);
            const unsigned long long r =
                splitmix64(splitmix64(seed) ^ (((unsigned long long)item << 32) | (uint32_t)positions[item]));
            const float u = __fmul_rn((float)(uint32_t)(r >> 40), 5.9604644775390625e-8f);  // 2^-24
            const float target = __fmul_rn(u, s);
            float acc = 0.0f;
            for (; j + 1 < k; ++j) {
                acc = __fadd_rn(acc, w[j]);
                if (acc > target) break;
            }
        }
        tokens[item] = si[j];
    }
}

}  // namespace b2

using namespace b2;

extern "C" int b2_matmul_f32(float *dst, const float *lhs, const float *rhs, uint32_t rows, uint32_t cols,
                             uint32_t inner, void *stream)
{
    if (!dst || !lhs || !rhs || rows == 0 || cols == 0 || inner == 0 || rows > 65535) return -1;
    matmul_f32_kernel<<<dim3((cols + 127) / 128, rows), 128, 0, (cudaStream_t)stream>>>(dst, lhs, rhs, rows, cols,
                                                                                        inner);
    return cudaGetLastError() == cudaSuccess ? 0 : -8;
}

extern "C" int b2_matmul_q4_ordered(float *dst, const float *lhs, uint32_t m, uint32_t cols, const uint8_t *packed,
                                    const float *scales, uint32_t rows, uint32_t group, void *stream)
{
    // group: a power of two in [16, 128] dividing cols (include/att1_quant.h)
    if (!dst || !lhs || !packed || !scales || m == 0 || m > 65535 || rows == 0 || cols == 0 || group < 16 ||
        group > 128 || (group & (group - 1)) || cols % group)
        return -1;
    matmul_q4_ordered_kernel<<<dim3((rows + 127) / 128, m), 128, 0, (cudaStream_t)stream>>>(dst, lhs, cols, packed,
                                                                                             scales, rows, group);
    return cudaGetLastError() == cudaSuccess ? 0 : -8;
}

extern "C" int b2_matmul_q8_ordered(float *dst, const float *lhs, uint32_t m, uint32_t cols, const int8_t *values,
                                    const float *scales, uint32_t rows, void *stream)
{
    if (!dst || !lhs || !values || !scales || m == 0 || m > 65535 || rows == 0 || cols == 0) return -1;
    matmul_q8_ordered_kernel<<<dim3((rows + 127) / 128, m), 128, 0, (cudaStream_t)stream>>>(dst, lhs, cols, values,
                                                                                             scales, rows);
    return cudaGetLastError() == cudaSuccess ? 0 : -8;
}

static int launched(cudaError_t e) { return e == cudaSuccess ? 0 : -8; }

extern "C" int b2_step_end_keys(const unsigned long long *keys, uint32_t world, uint32_t batch, uint32_t *tokens,
                                int32_t *positions, int32_t *err, int pdl, void *stream)
{
    if (!keys || !tokens || !positions || world == 0 || world > B2_TP_MAX || batch == 0 || batch > 1024) return -1;
    void *args[] = {(void *)&keys, (void *)&world, (void *)&batch, (void *)&tokens, (void *)&positions, (void *)&err};
    return launched(launch_pdl((const void *)step_end_keys_kernel, dim3(1), dim3(batch <= 32 ? 32 : (batch + 31) / 32 * 32),
                               pdl, (cudaStream_t)stream, args));
}

extern "C" int b2_step_begin(const float *embed, uint32_t vocab, uint32_t d_model, const uint32_t *tokens,
                             uint32_t batch, float *x, unsigned long long *argmax, int32_t *err, int pdl,
                             void *stream)
{
    if (!embed || !tokens || !x || !argmax || batch == 0 || batch > 65535 || d_model == 0 || (d_model & 3) ||
        vocab == 0 || ((uintptr_t)embed & 15) || ((uintptr_t)x & 15))
        return -1;
    void *args[] = {(void *)&embed, (void *)&vocab, (void *)&d_model, (void *)&tokens,
                    (void *)&x,     (void *)&argmax, (void *)&err};
    const uint32_t blocks = (d_model / 4 + 127) / 128;
    return launched(launch_pdl((const void *)step_begin_kernel, dim3(blocks, batch), dim3(128), pdl,
                               (cudaStream_t)stream, args));
}

extern "C" int b2_step_end(const unsigned long long *argmax, uint32_t batch, uint32_t *tokens, int32_t *positions,
                           int32_t *err, int pdl, void *stream)
{
    if (!argmax || !tokens || !positions || batch == 0 || batch > 1024) return -1;
    void *args[] = {(void *)&argmax, (void *)&batch, (void *)&tokens, (void *)&positions, (void *)&err};
    return launched(launch_pdl((const void *)step_end_kernel, dim3(1), dim3(((batch + 31) / 32) * 32), pdl,
                               (cudaStream_t)stream, args));
}

extern "C" int b2_step_end_tp(const b2_tp *tp, uint32_t batch, uint32_t *tokens, int32_t *positions, int32_t *err,
                              int pdl, void *stream)
{
    if (tp == nullptr || tokens == nullptr || positions == nullptr || batch == 0 || batch > B2_TP_MAX_ITEMS)
        return -1;
    if (tp->world < 2 || tp->world > B2_TP_MAX || tp->rank >= tp->world || tp->epoch == nullptr ||
        tp->peer[tp->rank] == nullptr)
        return -1;
    b2_tp t = *tp;
    void *args[] = {&t, &batch, &tokens, &positions, &err};
    return launch_pdl((const void *)step_end_tp_kernel, dim3(1), dim3((batch + 31) / 32 * 32), pdl,
                      (cudaStream_t)stream, args) == cudaSuccess
               ? 0
               : -8;
}

static int tp_args_ok(const b2_tp *tp)
{
    if (tp == nullptr || tp->world < 2 || tp->world > B2_TP_MAX || tp->rank >= tp->world || tp->epoch == nullptr ||
        tp->done == nullptr)
        return 0;
    for (uint32_t s = 0; s < tp->world; ++s)
        if (tp->peer[s] == nullptr || ((uintptr_t)tp->peer[s] & 15)) return 0;
    return tp->slot_floats % 4 == 0;
}

static uint32_t tp_grid(size_t n)
{
    const size_t want = (n + 255) / 256;
    const size_t cap = (size_t)sm_count() * 2;
    return (uint32_t)(want < 1 ? 1 : (want > cap ? cap : want));
}

extern "C" int b2_tp_push(const float *x, uint32_t n, const b2_tp *tp, uint32_t point, void *stream)
{
    if (x == nullptr || !tp_args_ok(tp) || n == 0 || n % 4 || n > tp->slot_floats || point >= tp->points ||
        ((uintptr_t)x & 15))
        return -1;
    const b2_tp t = *tp;
    tp_push_kernel<<<tp_grid(n / 4), 256, 0, (cudaStream_t)stream>>>(x, n, t, point);
    return launched(cudaGetLastError());
}

extern "C" int b2_tp_sum(const float *resid, float *out, uint32_t n, const b2_tp *tp, uint32_t point, int32_t *err,
                         void *stream)
{
    if (resid == nullptr || out == nullptr || !tp_args_ok(tp) || n == 0 || n % 4 || n > tp->slot_floats ||
        point >= tp->points || ((uintptr_t)resid & 15) || ((uintptr_t)out & 15))
        return -1;
    const b2_tp t = *tp;
    tp_sum_kernel<<<tp_grid(n / 4), 256, 0, (cudaStream_t)stream>>>(resid, out, n, t, point, err);
    return launched(cudaGetLastError());
}

extern "C" int b2_tp_push_logits(const float *logits, uint32_t batch, uint32_t rows,
                                 const unsigned long long *argmax, const b2_tp *tp, void *stream)
{
    if (logits == nullptr || argmax == nullptr || !tp_args_ok(tp) || batch == 0 || batch > B2_TP_MAX_ITEMS ||
        rows == 0 || (size_t)batch * rows > tp->logit_floats)
        return -1;
    const b2_tp t = *tp;
    tp_push_logits_kernel<<<tp_grid((size_t)batch * rows), 256, 0, (cudaStream_t)stream>>>(logits, batch, rows,
                                                                                           argmax, t);
    return launched(cudaGetLastError());
}

extern "C" int b2_rmsnorm(float *dst, const float *src, const float *w, uint32_t n, float eps, void *stream)
{
    if (!dst || !src || !w || n == 0 || !(eps > 0.0f)) return -1;
    rmsnorm_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(dst, src, w, n, eps);
    return launched(cudaGetLastError());
}

extern "C" int b2_softmax(float *v, uint32_t n, void *stream)
{
    if (!v || n == 0) return -1;
    softmax_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(v, n);
    return launched(cudaGetLastError());
}

extern "C" int b2_rope(float *v, uint32_t n, uint32_t pos, float theta, void *stream)
{
    if (!v || n == 0 || (n & 1) || !(theta > 0.0f)) return -1;
    const uint32_t pairs = n / 2;
    rope_kernel<<<(pairs + 127) / 128, 128, 0, (cudaStream_t)stream>>>(v, n, pos, theta);
    return launched(cudaGetLastError());
}

extern "C" int b2_swiglu(float *dst, const float *gate, const float *up, uint32_t n, void *stream)
{
    if (!dst || !gate || !up || n == 0) return -1;
    uint32_t blocks = (n + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    swiglu_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(dst, gate, up, n);
    return launched(cudaGetLastError());
}

extern "C" int b2_argmax(const float *v, uint32_t n, unsigned long long *key, void *stream)
{
    if (!v || n == 0 || !key) return -1;
    uint32_t blocks = (n + 255) / 256;
    if (blocks > 1024) blocks = 1024;
    cudaError_t e = cudaMemsetAsync(key, 0, sizeof(unsigned long long), (cudaStream_t)stream);
    if (e != cudaSuccess) return -8;
    argmax_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(v, n, key);
    return launched(cudaGetLastError());
}

extern "C" int b2_sample_topk(const float *logits, uint32_t batch, uint32_t vocab, uint32_t stride, uint32_t top_k,
                              float temperature, unsigned long long seed, const int32_t *positions, uint32_t *tokens,
                              int pdl, void *stream)
{
    return b2_sample_topk_sharded(logits, batch, vocab, vocab, 0, stride, top_k, temperature, seed, positions, tokens,
                                  pdl, stream);
}

extern "C" int b2_sample_topk_sharded(const float *logits, uint32_t batch, uint32_t vocab, uint32_t shard_rows,
                                      size_t shard_stride, uint32_t item_stride, uint32_t top_k, float temperature,
                                      unsigned long long seed, const int32_t *positions, uint32_t *tokens, int pdl,
                                      void *stream)
{
    if (logits == nullptr || positions == nullptr || tokens == nullptr || batch == 0 || vocab == 0 ||
        shard_rows == 0 || vocab % shard_rows || item_stride < shard_rows || top_k == 0 || top_k > B2_MAX_TOP_K ||
        top_k > vocab || !(temperature > 0.0f) || !(temperature <= FLT_MAX))
        return -1;
    if (vocab > shard_rows && shard_stride < (size_t)(batch - 1) * item_stride + shard_rows) return -1;
    unsigned long long ss = shard_stride;
    void *args[] = {&logits, &vocab, &shard_rows, &ss, &item_stride, &top_k, &temperature, &seed, &positions, &tokens};
    return launched(launch_pdl((const void *)sample_topk_kernel, dim3(batch), dim3(kSampleThreads), pdl,
                               (cudaStream_t)stream, args));
}
