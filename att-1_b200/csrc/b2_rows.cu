// b2_rows.cu - the GEMV epilogues applied to a dense GEMM result.
//
// When a decode batch or a prompt goes through b2_gemm (tensor cores) instead
// of the fused GEMVs, the projections land in a dense [m][rows] buffer and
// this kernel finishes them exactly as the GEMV epilogues do (same roundings):
//   B2_EPI_QKV     RoPE of q and k (src/rope.c:20-30, interleaved pairs of a
//                  head, angle = pos * freq), q to out, k and v appended to the
//                  KV pages at positions[n] (src/attention.c:490-504);
//   B2_EPI_SWIGLU  silu(gate) * up (src/ffn.c:5-30) over the interleaved
//                  gate/up rows (tile t: rows 0..7 gate 8t.., rows 8..15 up 8t..);
//   B2_EPI_LOGITS  greedy argmax key per row of y (src/sampler.c:5-34: NaN is
//                  an error, the lowest id wins ties), max-combined into argmax[n].
#include "b2_common.cuh"

namespace b2 {

__global__ void rows_qkv_kernel(const b2_rows_args a)
{
    pdl_wait();
    pdl_launch_dependents();
    const uint32_t n = blockIdx.y;
    const uint32_t hd = a.kv.head_dim;
    const int32_t pos = a.positions[n];
    const uint32_t cap = a.kv.pages_per_seq * a.kv.page_tokens;
    const float *y = a.y + (size_t)n * a.y_stride;
    const uint32_t total = a.q_rows + 2 * a.kv_rows;
    for (uint32_t row = blockIdx.x * blockDim.x + threadIdx.x; row < total; row += gridDim.x * blockDim.x) {
        if (row < a.q_rows + a.kv_rows) {
            const uint32_t rr = row < a.q_rows ? row : row - a.q_rows;
            const uint32_t i = rr % hd;
            const float x0 = y[row & ~1u], x1 = y[row | 1u];
            const float ang = __fmul_rn((float)pos, a.rope_freq[i >> 1]);
            float s, c;
            sincosf(ang, &s, &c);
            const float v = (i & 1u) ? __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c))
                                     : __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
            if (row < a.q_rows) {
                a.out[(size_t)n * a.out_stride + row] = v;
            } else if (pos >= 0 && (uint32_t)pos < cap) {
                const int32_t page = a.kv.page_table[(size_t)n * a.kv.pages_per_seq + pos / a.kv.page_tokens];
                a.kv.k_pool[(((size_t)page * a.kv.n_kv_heads + rr / hd) * a.kv.page_tokens + pos % a.kv.page_tokens) *
                                hd +
                            i] = v;
            } else {
                raise_error(a.err, B2_ERR_POSITION);
            }
        } else {
            const uint32_t rr = row - a.q_rows - a.kv_rows;
            if (pos >= 0 && (uint32_t)pos < cap) {
                const int32_t page = a.kv.page_table[(size_t)n * a.kv.pages_per_seq + pos / a.kv.page_tokens];
                a.kv.v_pool[(((size_t)page * a.kv.n_kv_heads + rr / hd) * a.kv.page_tokens + pos % a.kv.page_tokens) *
                                hd +
                            rr % hd] = y[row];
            } else {
                raise_error(a.err, B2_ERR_POSITION);
            }
        }
    }
}

__global__ void rows_swiglu_kernel(const b2_rows_args a)
{
    pdl_wait();
    pdl_launch_dependents();
    const uint32_t n = blockIdx.y;
    const float *y = a.y + (size_t)n * a.y_stride;
    for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < a.rows / 2; j += gridDim.x * blockDim.x) {
        const uint32_t t = j >> 3, r = j & 7;
        const float g = y[16 * t + r], u = y[16 * t + 8 + r];
        a.out[(size_t)n * a.out_stride + j] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
    }
}

__global__ void __launch_bounds__(256) rows_logits_kernel(const b2_rows_args a)
{
    __shared__ unsigned long long red[8];
    pdl_wait();
    pdl_launch_dependents();
    const uint32_t n = blockIdx.y;
    const float *y = a.y + (size_t)n * a.y_stride;
    unsigned long long key = 0ull;
    bool nan = false;
    for (uint32_t row = blockIdx.x * blockDim.x + threadIdx.x; row < a.rows; row += gridDim.x * blockDim.x) {
        const float v = y[row];
        if (a.out != nullptr) a.out[(size_t)n * a.out_stride + row] = v;
        if (v != v) {
            nan = true;
        } else {
            const unsigned long long k = ((unsigned long long)ordered_key(v) << 32) | (0xFFFFFFFFu - (a.row_offset + row));
            key = k > key ? k : key;
        }
    }
    if (nan) raise_error(a.err, B2_ERR_NAN_LOGITS);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = key;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (uint32_t w = 1; w < blockDim.x / 32; ++w) key = red[w] > key ? red[w] : key;
        atomicMax(a.argmax + n, key);
    }
}

static cudaError_t launch_rows(const void *fn, dim3 grid, dim3 block, int pdl, cudaStream_t st, const b2_rows_args &a)
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
    void *args[] = {(void *)&a};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace b2

using namespace b2;

extern "C" int b2_rows_epilogue(const b2_rows_args *a, void *stream)
{
    if (a == nullptr || a->y == nullptr || a->m == 0 || a->m > 65535 || a->rows == 0 || a->y_stride < a->rows)
        return -1;
    const cudaStream_t st = (cudaStream_t)stream;
    const uint32_t per_sm = (uint32_t)sm_count() * 4;
    cudaError_t e;
    switch (a->epilogue) {
    case B2_EPI_QKV: {
        const b2_kv_layout &kv = a->kv;
        if (a->out == nullptr || a->positions == nullptr || a->rope_freq == nullptr || !kv.k_pool || !kv.v_pool ||
            !kv.page_table || kv.head_dim == 0 || kv.head_dim % 2 || kv.page_tokens == 0 || kv.pages_per_seq == 0)
            return -1;
        if (a->q_rows % kv.head_dim || a->kv_rows != kv.n_kv_heads * kv.head_dim ||
            a->q_rows + 2 * a->kv_rows != a->rows || a->out_stride < a->q_rows)
            return -1;
        uint32_t bx = (a->rows + 255) / 256;
        if (bx * a->m > per_sm) bx = (per_sm + a->m - 1) / a->m;
        e = launch_rows((const void *)rows_qkv_kernel, dim3(bx ? bx : 1, a->m), dim3(256), a->pdl, st, *a);
        break;
    }
    case B2_EPI_SWIGLU: {
        if (a->out == nullptr || (a->rows & 15) || a->out_stride < a->rows / 2) return -1;
        uint32_t bx = (a->rows / 2 + 255) / 256;
        if (bx * a->m > per_sm) bx = (per_sm + a->m - 1) / a->m;
        e = launch_rows((const void *)rows_swiglu_kernel, dim3(bx ? bx : 1, a->m), dim3(256), a->pdl, st, *a);
        break;
    }
    case B2_EPI_LOGITS: {
        if (a->argmax == nullptr || (a->out != nullptr && a->out_stride < a->rows)) return -1;
        uint32_t bx = (a->rows + 4095) / 4096;
        if (bx * a->m > per_sm) bx = (per_sm + a->m - 1) / a->m;
        e = launch_rows((const void *)rows_logits_kernel, dim3(bx ? bx : 1, a->m), dim3(256), a->pdl, st, *a);
        break;
    }
    default:
        return -1;
    }
    return e == cudaSuccess ? 0 : -8;
}
