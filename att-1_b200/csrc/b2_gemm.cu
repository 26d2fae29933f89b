// b2_gemm.cu - q4/q8 dequant GEMM on the 5th-generation tensor cores (tcgen05).
//
// Replaces att1_matmul_q4xf32 (src/quant.c:340-393) and att1_matmul_q8xf32
// (src/matmul_q8.c:3-40) when many input rows share one pass over the weights:
// prompt prefill (the reference feeds the prompt through the decode step one
// token at a time, src/infer.c:905-912) and decode batches too large for the
// GEMV's on-chip digit planes. Y[m][o] = sum_k X[m][k] * W[o][k].
//
// Precision. The reference accumulates f32 products x * (q * scale). Here every
// f32 operand v is split into two bf16 numbers v = hi + lo (hi = bf16(v),
// lo = bf16(v - hi), 16 significant bits together) and the product is
//   x.w ~= x_hi w_hi + x_lo w_hi + x_hi w_lo     (q4: w = q * group scale)
//   x.w ~= (x_hi q + x_lo q) * row scale          (q8: q is exact in bf16)
// three (two) bf16 MMAs with f32 accumulation in tensor memory; the dropped
// terms are below 2^-16 relative, the same order as the GEMV's 2^-22 fixed
// point plus f32 summation, far inside the 1e-3 logits tolerance.
//
// Work split. CTA (row block, token tile, k split) computes a 128-row x BN-token
// tile of Y over a range of 64-column k steps (for BN <= 64: two 128-row blocks,
// each with its own MMA warps, dequant warps and accumulators; below for one):
//   warp 0      allocates tensor memory and streams the prepared X tiles
//               (b2_gemm_prep writes them in the MMA operand layout, k steps of
//               a token tile contiguous) into two slots of xk k steps each, one
//               1-D bulk copy of ~32 KB per slot (an SM completes bulk copies at
//               a bounded rate whatever their size);
//   warps 1, 2  one thread each issues tcgen05.mma (M=128, N=BN, K=16) for
//               alternate k steps into its own accumulator (tensor-memory
//               columns mw * acols), then tcgen05.commit releases the W stage
//               (and each X slot once both have passed it). Issuing the MMAs of
//               one k step costs a single thread about the read of their 4 KB
//               weight operands, so for small BN (decode batches) one issuer
//               set the pace; two take 126 -> 103 us for 32 tokens of the
//               gate/up matrix (four: no further gain);
//   warps 3..10 one per 16-row tile: read the tile's weight unit of each k
//               step with 16-byte loads issued two k steps ahead (each lane's
//               16 bytes are one fixed set of 32 weights), scale, split into
//               bf16 hi/lo and store them in the operand layout; after the k
//               loop they read the accumulators out of tensor memory (warp w
//               reads TMEM lanes 32*(w%4)..: one output row per thread, the two
//               warps of a lane quarter alternate 16-column chunks), add them
//               in issuer order and write Y, or the split's partial sums.
// Operands are K-major without swizzle: 8-row x 16-byte core matrices,
// element (r, k) of a tile with R rows at byte
//   (k / 8) * (R * 16) + (r / 8) * 128 + (r % 8) * 16 + (k % 8) * 2,
// so the descriptor's stride between 8-row groups is 128 bytes and the
// stride between 8-column chunks is R * 16 bytes.
// Every wait is bounded and reports B2_ERR_TIMEOUT; tensor memory is freed by
// the allocating warp after the whole CTA has passed the epilogue.
#include "b2_common.cuh"

#include <cuda_bf16.h>

namespace b2 {

constexpr uint32_t kGemmBM = 128;          // output rows per CTA (8 tiles of 16)
constexpr uint32_t kGemmBK = 64;           // columns per k step
constexpr uint32_t kGemmMaxBN = 256;       // tokens per CTA tile
constexpr int kGemmDequantWarps = 8;      // one 16-row tile each
constexpr int kGemmMmaWarps = 2;          // MMA issuers per 128-row block, alternate k steps, one accumulator each
// threads of a CTA over RBM 128-row blocks: the TMEM/X-copy warp, the MMA
// warps and the dequantising warps of every row block
template <int RBM>
__host__ __device__ constexpr int gemm_threads() { return 32 + 32 * kGemmMmaWarps * RBM + 32 * kGemmDequantWarps * RBM; }
constexpr uint32_t kGemmRb2MaxBn = 64;     // token tiles up to this size take two row blocks per CTA
constexpr uint32_t kGemmMaxStages = 6;      // W ring
constexpr uint32_t kGemmXSlots = 2;         // X ring
constexpr uint32_t kGemmXCopy = 32768;      // target bytes per X bulk copy
constexpr uint32_t kGemmMaxSplits = 16;
constexpr uint32_t kGemmSmemLimit = 227u * 1024u;

__host__ __device__ constexpr uint32_t gemm_x_stage_bytes(uint32_t bn) { return bn * kGemmBK * 2 * 2; }
__host__ __device__ constexpr uint32_t gemm_w_stage_bytes(uint32_t fmt)
{
    return kGemmBM * kGemmBK * 2 * (fmt == 4 ? 2 : 1);
}

// Token tiles of at most 128 rows keep x's hi and lo halves as ONE operand of
// 2*bn rows (hi rows, then lo rows, in every 8-column chunk): one MMA then
// multiplies w_hi with both halves, so a k step needs two MMAs for q4
// (w_hi [x_hi; x_lo], w_lo x_hi) and one for q8 instead of three and two. At
// small bn every MMA costs about the read of its 4 KB weight operand whatever
// N is, so fewer, wider MMAs are faster. Larger tiles (N would pass 256) keep
// hi and lo as separate operands.
__host__ __device__ constexpr bool gemm_stacked(uint32_t bn) { return bn <= 128; }

// Token tiling shared by b2_gemm_prep and b2_gemm: as few tiles of at most
// 256 tokens as possible, equal sizes rounded up to 16 (the MMA's N step).
__host__ __device__ inline void gemm_token_tiles(uint32_t m, uint32_t &ntiles, uint32_t &bn)
{
    ntiles = (m + kGemmMaxBN - 1) / kGemmMaxBN;
    if (ntiles == 0) ntiles = 1;
    const uint32_t per = (m + ntiles - 1) / ntiles;
    bn = (per + 15) / 16 * 16;
    if (bn < 16) bn = 16;
}

struct GemmParams {
    const uint8_t *w;
    const float *row_scale;
    uint32_t fmt, rows, cols, tiles, kunits;
    uint32_t ksteps;        // ceil(cols / 64)
    const uint8_t *xs;
    uint32_t m, bn, ntiles;
    float *out;
    uint32_t out_stride;
    const float *resid;
    uint32_t epilogue;
    float *part;            // [splits][m][rows] when splits > 1
    uint32_t splits, ksplit;  // k steps per split
    uint32_t stages;        // W ring stages (one k step each)
    uint32_t nmma;          // MMA warps in use (accumulators): kGemmMmaWarps per row block
    uint32_t rbm;           // 128-row blocks per CTA (1 or 2)
    uint32_t xk;            // k steps per X slot (one bulk copy)
    uint32_t off_x, off_w, tmem_cols;
    int32_t *err;
};

// ---- tcgen05 wrappers ------------------------------------------------------------

// Shared-memory matrix descriptor: K-major, no swizzle (layout type 0),
// version 1 (bits 46-47), base offset 0. Addresses and offsets in 16-byte units.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes)
{
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1u << 46;
    return d;
}

// Instruction descriptor, kind::f16: D f32, A and B bf16, both K-major,
// N >> 3 at bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(uint32_t m, uint32_t n)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

// Arrives on `bar` once every tcgen05 operation issued so far by this thread is complete.
__device__ __forceinline__ void umma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t cols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_free(uint32_t taddr, uint32_t cols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

// 32 lanes x 16 columns of 32 bits: thread i gets lane (base + i), columns col..col+15.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16])
{
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- operand packing ----------------------------------------------------------------

// bf16 hi/lo split of four consecutive values, packed as two bf16x2 words each.
__device__ __forceinline__ void split4(const float (&v)[4], uint2 &hi, uint2 &lo)
{
    const __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]);
    const __nv_bfloat162 h1 = __floats2bfloat162_rn(v[2], v[3]);
    const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
    const __nv_bfloat162 l0 = __floats2bfloat162_rn(v[0] - f0.x, v[1] - f0.y);
    const __nv_bfloat162 l1 = __floats2bfloat162_rn(v[2] - f1.x, v[3] - f1.y);
    hi = make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
    lo = make_uint2(*reinterpret_cast<const uint32_t *>(&l0), *reinterpret_cast<const uint32_t *>(&l1));
}

// Byte offset of element (r, k) in a K-major core-matrix tile of R rows x 64 columns.
__host__ __device__ __forceinline__ uint32_t op_off(uint32_t r, uint32_t k, uint32_t R)
{
    return (k >> 3) * (R * 16) + (r >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2;
}

// ---- X preparation: optional RMSNorm, bf16 hi/lo split, operand layout -------------------

// One CTA per padded token row n (ntiles * bn rows; rows >= m are zero).
// Output block (tile, k step): stacked tiles one 2*bn x 64 operand (row n hi,
// row bn + n lo), else [hi: bn x 64][lo: bn x 64], bf16 in op_off order.
__global__ void __launch_bounds__(256) gemm_prep_kernel(const float *__restrict__ x, uint32_t x_stride, uint32_t m,
                                                        uint32_t cols, const float *__restrict__ norm_w, float eps,
                                                        uint32_t bn, uint32_t ksteps, uint8_t *__restrict__ xs,
                                                        int32_t *err)
{
    __shared__ float red[32];
    const uint32_t n = blockIdx.x;
    const uint32_t tile = n / bn, nr = n % bn;
    const bool live = n < m;
    const float *row = x + (size_t)n * x_stride;
    float inv = 1.0f;
    if (norm_w != nullptr && live) {
        float ss = 0.0f;
        for (uint32_t k = threadIdx.x * 4; k < cols; k += blockDim.x * 4) {
            const float4 v = *reinterpret_cast<const float4 *>(row + k);
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
        ss = block_sum(ss, red);
        inv = 1.0f / sqrtf(ss / (float)cols + eps);
    }
    const uint32_t xstage = gemm_x_stage_bytes(bn);
    bool finite = true;
    // each thread writes one 8-column chunk (16 bytes of hi, 16 of lo)
    for (uint32_t c = threadIdx.x; c < ksteps * 8; c += blockDim.x) {
        const uint32_t k0 = c * 8;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.0f;
        if (live && k0 < cols) {  // cols % 32 == 0: a chunk is all in or all out
            const float4 a = *reinterpret_cast<const float4 *>(row + k0);
            const float4 b = *reinterpret_cast<const float4 *>(row + k0 + 4);
            v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
            if (norm_w != nullptr) {
                const float4 wa = *reinterpret_cast<const float4 *>(norm_w + k0);
                const float4 wb = *reinterpret_cast<const float4 *>(norm_w + k0 + 4);
                const float w8[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = v[i] * inv * w8[i];
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) finite = finite && isfinite(v[i]);
        }
        uint2 h0, l0, h1, l1;
        const float a4[4] = {v[0], v[1], v[2], v[3]}, b4[4] = {v[4], v[5], v[6], v[7]};
        split4(a4, h0, l0);
        split4(b4, h1, l1);
        uint8_t *blk = xs + (size_t)(tile * ksteps + k0 / kGemmBK) * xstage;
        const uint32_t kc = k0 % kGemmBK;
        const bool stk = gemm_stacked(bn);
        const uint32_t off_hi = stk ? op_off(nr, kc, 2 * bn) : op_off(nr, kc, bn);
        const uint32_t off_lo = stk ? op_off(bn + nr, kc, 2 * bn) : xstage / 2 + op_off(nr, kc, bn);
        *reinterpret_cast<uint4 *>(blk + off_hi) = make_uint4(h0.x, h0.y, h1.x, h1.y);
        *reinterpret_cast<uint4 *>(blk + off_lo) = make_uint4(l0.x, l0.y, l1.x, l1.y);
    }
    if (!finite) raise_error(err, B2_ERR_NONFINITE);
}

// ---- the GEMM ----------------------------------------------------------------------------

struct GemmSmem {
    uint64_t *x_full, *x_empty, *w_full, *w_empty, *acc_full;
    uint32_t *tmem_slot;
    uint8_t *x, *w;
};

__device__ __forceinline__ GemmSmem gemm_smem(uint8_t *smem, const GemmParams &p)
{
    GemmSmem s;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    s.x_full = bars;
    s.x_empty = bars + kGemmXSlots;
    s.w_full = bars + 2 * kGemmXSlots;
    s.w_empty = bars + 2 * kGemmXSlots + kGemmMaxStages;
    s.acc_full = bars + 2 * kGemmXSlots + 2 * kGemmMaxStages;
    s.tmem_slot = reinterpret_cast<uint32_t *>(s.acc_full + 1);
    s.x = smem + p.off_x;
    s.w = smem + p.off_w;
    return s;
}

// The weight bytes one dequant lane needs for one k step of its tile: q4 one
// unit (16 bytes of nibbles + the float4 of its row's scales), q8 two units.
struct RawStep {
    uint4 q0, q1;
    float4 sc;
};

template <int FMT>
__device__ __forceinline__ RawStep load_step(const GemmParams &p, uint32_t T, uint32_t ks, uint32_t lane)
{
    RawStep r;
    r.q0 = r.q1 = make_uint4(0, 0, 0, 0);
    r.sc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (T >= p.tiles) return r;
    if constexpr (FMT == 4) {
        const uint8_t *u = p.w + ((size_t)T * p.kunits + ks) * B2_Q4_UNIT_BYTES;
        r.q0 = __ldg(reinterpret_cast<const uint4 *>(u) + lane);
        r.sc = __ldg(reinterpret_cast<const float4 *>(u + 512) + (lane >> 2));
    } else {
        const uint32_t ku = 2 * ks;
        const uint8_t *u = p.w + ((size_t)T * p.kunits + ku) * B2_Q8_UNIT_BYTES;
        r.q0 = __ldg(reinterpret_cast<const uint4 *>(u) + lane);
        if (ku + 1 < p.kunits) r.q1 = __ldg(reinterpret_cast<const uint4 *>(u + B2_Q8_UNIT_BYTES) + lane);
    }
    return r;
}

// Conversions (I2F, F2F) issue at a fraction of the ALU rate, so the weights
// are decoded with bit operations and exact f32 additions instead:
//   * a 4-bit field u (0..15) at bit p <= 19 of a word, OR-ed into the bits of
//     2^23, is the float 2^23 + u 2^p; subtracting 2^23 + 8 2^p (exact) leaves
//     (u - 8) 2^p, and the word was XOR-ed with 0x8888.. so u - 8 is the
//     signed nibble q; times (s 2^-p) this is fl(q s), the reference's product
//     bit for bit (s 2^-p is exact for every normal scale);
//   * the split keeps hi = v with the low 16 bits cleared (truncation: bf16's 8
//     significant bits) and lo = bf16_rn(v - hi) (v - hi is exact in f32): the
//     pair represents v within 2^-16 relative, one conversion per two values.
__device__ __forceinline__ float field_f(uint32_t w, uint32_t mask) { return __uint_as_float((w & mask) | 0x4B000000u); }
// 2^23 + 8 * 2^p and 2^23 + 128 * 2^p (exact in f32 for the bit positions used)
__host__ __device__ constexpr float nib_off(int p) { return 8388608.0f + 8.0f * (float)(1u << p); }
__host__ __device__ constexpr float byte_off(int p) { return 8388608.0f + 128.0f * (float)(1u << p); }
static_assert(nib_off(0) == 8388616.0f && nib_off(4) == 8388736.0f && nib_off(8) == 8390656.0f &&
                  nib_off(12) == 8421376.0f && nib_off(16) == 8912896.0f,
              "nibble offsets");
static_assert(byte_off(0) == 8388736.0f && byte_off(8) == 8421376.0f, "byte offsets");

__device__ __forceinline__ void split_pair(float v0, float v1, uint32_t &hi, uint32_t &lo)
{
    const uint32_t b0 = __float_as_uint(v0) & 0xFFFF0000u, b1 = __float_as_uint(v1) & 0xFFFF0000u;
    hi = __byte_perm(b0, b1, 0x7632);  // upper halves: element 0 low, element 1 high
    const __nv_bfloat162 l = __floats2bfloat162_rn(v0 - __uint_as_float(b0), v1 - __uint_as_float(b1));
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

// Dequantise one k step of tile tl (0..7 within the row block) into the W
// stage (bf16, hi at 0 and, for q4, lo at 16 KB).
template <int FMT>
__device__ __forceinline__ void dequant_store(const RawStep &raw, uint8_t *wst, uint32_t tl, uint32_t lane)
{
    const uint32_t r = lane >> 2, t = lane & 3;
    constexpr uint32_t kLo = kGemmBM * kGemmBK * 2;  // byte offset of the lo half (q4)
    if constexpr (FMT == 4) {
        // words: {row r g0, row r+8 g0, row r g1, row r+8 g1}; scales {s(r,g0), s(r,g1), s(r+8,g0), s(r+8,g1)}
        const uint32_t wd[4] = {raw.q0.x, raw.q0.y, raw.q0.z, raw.q0.w};
        const float ws[4] = {raw.sc.x, raw.sc.z, raw.sc.y, raw.sc.w};
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
            const uint32_t row = tl * 16 + r + (j & 1) * 8;
            const uint32_t g = j >> 1;
            const uint32_t w = wd[j] ^ 0x88888888u, w12 = w >> 12;
            const float s0 = ws[j], s4 = s0 * 0x1p-4f, s8 = s0 * 0x1p-8f, s12 = s0 * 0x1p-12f, s16 = s0 * 0x1p-16f;
            // byte i: low nibble (bit 8i) = column 4t+i, high nibble (bit 8i+4) = column 16+4t+i
            float v[8];
            v[0] = (field_f(w, 0xFu) - nib_off(0)) * s0;              // bit 0
            v[1] = (field_f(w, 0xF00u) - nib_off(8)) * s8;            // bit 8
            v[2] = (field_f(w, 0xF0000u) - nib_off(16)) * s16;        // bit 16
            v[3] = (field_f(w12, 0xF000u) - nib_off(12)) * s12;       // bit 24 (12 after the shift)
            v[4] = (field_f(w, 0xF0u) - nib_off(4)) * s4;             // bit 4
            v[5] = (field_f(w, 0xF000u) - nib_off(12)) * s12;         // bit 12
            v[6] = (field_f(w12, 0xF00u) - nib_off(8)) * s8;          // bit 20 (8 after the shift)
            v[7] = (field_f(w12, 0xF0000u) - nib_off(16)) * s16;      // bit 28 (16 after the shift)
#pragma unroll
            for (uint32_t half = 0; half < 2; ++half) {
                uint32_t h0, h1, l0, l1;
                split_pair(v[4 * half + 0], v[4 * half + 1], h0, l0);
                split_pair(v[4 * half + 2], v[4 * half + 3], h1, l1);
                const uint32_t off = op_off(row, 32 * g + 16 * half + 4 * t, kGemmBM);
                *reinterpret_cast<uint2 *>(wst + off) = make_uint2(h0, h1);
                *reinterpret_cast<uint2 *>(wst + kLo + off) = make_uint2(l0, l1);
            }
        }
    } else {
        // two 32-column units; bytes {row r k 4t.., row r+8 k 4t.., row r k 16+4t.., row r+8 k 16+4t..};
        // bf16 holds the int8 values exactly: byte u = q + 128 at bit p gives
        // 2^23 + u 2^p, minus 2^23 + 128 2^p is q 2^p, whose upper half is bf16(q 2^p)
#pragma unroll
        for (uint32_t uh = 0; uh < 2; ++uh) {
            const uint4 q = uh ? raw.q1 : raw.q0;
            const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (uint32_t j = 0; j < 4; ++j) {
                const uint32_t row = tl * 16 + r + (j & 1) * 8;
                const uint32_t k = 32 * uh + 16 * (j >> 1) + 4 * t;
                const uint32_t w = wd[j] ^ 0x80808080u, w16 = w >> 16;
                const float v0 = field_f(w, 0xFFu) - byte_off(0);
                const float v1 = (field_f(w, 0xFF00u) - byte_off(8)) * 0x1p-8f;
                const float v2 = field_f(w16, 0xFFu) - byte_off(0);
                const float v3 = (field_f(w16, 0xFF00u) - byte_off(8)) * 0x1p-8f;
                const uint32_t a = __byte_perm(__float_as_uint(v0), __float_as_uint(v1), 0x7632);
                const uint32_t b = __byte_perm(__float_as_uint(v2), __float_as_uint(v3), 0x7632);
                *reinterpret_cast<uint2 *>(wst + op_off(row, k, kGemmBM)) = make_uint2(a, b);
            }
        }
    }
}

template <int FMT, int RBM>
__global__ void __launch_bounds__(gemm_threads<RBM>(), 1) att1_qgemm_kernel(const GemmParams p)
{
    extern __shared__ __align__(1024) uint8_t smem[];
    const GemmSmem s = gemm_smem(smem, p);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rb = blockIdx.x, nt = blockIdx.y, split = blockIdx.z;
    const uint32_t k0 = split * p.ksplit;
    const uint32_t k1 = min(p.ksteps, k0 + p.ksplit);
    const uint32_t nk = k1 > k0 ? k1 - k0 : 0;
    const uint32_t xstage = gemm_x_stage_bytes(p.bn);
    constexpr uint32_t wst1 = gemm_w_stage_bytes(FMT);  // one row block's part of a W stage
    constexpr uint32_t wstage = RBM * wst1;

    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < kGemmXSlots; ++i) {
            mbar_init(&s.x_full[i], 1);
            mbar_init(&s.x_empty[i], p.nmma);
        }
        for (uint32_t i = 0; i < kGemmMaxStages; ++i) {
            mbar_init(&s.w_full[i], 32 * kGemmDequantWarps * RBM);
            mbar_init(&s.w_empty[i], RBM);  // one commit per row block's MMA warp of the k step
        }
        mbar_init(s.acc_full, p.nmma);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(s.tmem_slot, p.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s.tmem_slot;
    pdl_wait();
    pdl_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            // X slot j holds k steps [j*xk, j*xk + xk): consecutive k steps of a
            // token tile are contiguous in the prepared buffer, one copy per slot
            const uint32_t nslots = (nk + p.xk - 1) / p.xk;
            for (uint32_t j = 0; j < nslots; ++j) {
                const uint32_t xs = j % kGemmXSlots, pass = j / kGemmXSlots;
                const uint32_t steps = min(p.xk, nk - j * p.xk);
                if (pass > 0) mbar_wait_bounded(&s.x_empty[xs], (pass - 1) & 1, p.err);
                mbar_arrive_expect_tx(&s.x_full[xs], steps * xstage);
                bulk_g2s(s.x + xs * p.xk * xstage, p.xs + (size_t)(nt * p.ksteps + k0 + j * p.xk) * xstage,
                         steps * xstage, &s.x_full[xs]);
            }
        }
    } else if (warp <= (uint32_t)(kGemmMmaWarps * RBM)) {
        // MMA warp mw works on row block h = mw / 2 and issues k steps of parity
        // mw % 2 into its own accumulator (columns mw * acols); every MMA warp
        // releases every X slot
        const uint32_t mw = warp - 1, nmma = p.nmma, h = mw / kGemmMmaWarps, par = mw % kGemmMmaWarps;
        if (lane == 0 && mw < nmma) {
            const bool stk = gemm_stacked(p.bn);
            const uint32_t acols = stk ? 2 * p.bn : p.bn;
            const uint32_t acc = tmem + mw * acols;
            const uint32_t idesc = umma_idesc_bf16(kGemmBM, p.bn);
            const uint32_t idesc2 = umma_idesc_bf16(kGemmBM, 2 * p.bn);  // stacked: hi and lo rows
            const uint32_t xb = smem_u32(s.x), wb = smem_u32(s.w);
            const uint32_t nslots = (nk + p.xk - 1) / p.xk;
            bool first = true;
            for (uint32_t j = 0; j < nslots; ++j) {
                const uint32_t xs = j % kGemmXSlots;
                // every MMA warp waits for every slot, even one without k steps
                // of its own: its release of the slot then cannot run ahead into
                // the slot's next fill
                mbar_wait_bounded(&s.x_full[xs], (j / kGemmXSlots) & 1, p.err);
                const uint32_t i_end = min(nk, (j + 1) * p.xk);
                uint32_t i = j * p.xk;
                i += (par + kGemmMmaWarps - i % kGemmMmaWarps) % kGemmMmaWarps;  // first k step of this warp
                for (; i < i_end; i += kGemmMmaWarps) {
                    const uint32_t st = i % p.stages, pass = i / p.stages, xi = i % p.xk;
                    mbar_wait_bounded(&s.w_full[st], pass & 1, p.err);
                    tc_fence_after();
                    const uint32_t xa = xb + (xs * p.xk + xi) * xstage, wa = wb + st * wstage + h * wst1;
                    if (stk) {
#pragma unroll
                        for (uint32_t kk = 0; kk < kGemmBK / 16; ++kk) {
                            const uint64_t a_hi = umma_desc(wa + kk * 2 * (kGemmBM * 16), kGemmBM * 16, 128);
                            // rows 0..bn-1 of this descriptor are x_hi, bn..2bn-1 x_lo
                            const uint64_t b = umma_desc(xa + kk * 2 * (2 * p.bn * 16), 2 * p.bn * 16, 128);
                            umma_bf16(acc, a_hi, b, idesc2, !(first && kk == 0));
                            if constexpr (FMT == 4) {
                                const uint64_t a_lo =
                                    umma_desc(wa + kGemmBM * kGemmBK * 2 + kk * 2 * (kGemmBM * 16), kGemmBM * 16, 128);
                                umma_bf16(acc, a_lo, b, idesc, 1);  // N = bn: the x_hi rows only
                            }
                        }
                    } else {
#pragma unroll
                        for (uint32_t kk = 0; kk < kGemmBK / 16; ++kk) {
                            // 16 columns = two 8-column chunks
                            const uint64_t a_hi = umma_desc(wa + kk * 2 * (kGemmBM * 16), kGemmBM * 16, 128);
                            const uint64_t b_hi = umma_desc(xa + kk * 2 * (p.bn * 16), p.bn * 16, 128);
                            const uint64_t b_lo = umma_desc(xa + xstage / 2 + kk * 2 * (p.bn * 16), p.bn * 16, 128);
                            umma_bf16(acc, a_hi, b_hi, idesc, !(first && kk == 0));
                            umma_bf16(acc, a_hi, b_lo, idesc, 1);
                            if constexpr (FMT == 4) {
                                const uint64_t a_lo =
                                    umma_desc(wa + kGemmBM * kGemmBK * 2 + kk * 2 * (kGemmBM * 16), kGemmBM * 16, 128);
                                umma_bf16(acc, a_lo, b_hi, idesc, 1);
                            }
                        }
                    }
                    first = false;
                    umma_commit(&s.w_empty[st]);
                }
                umma_commit(&s.x_empty[xs]);
            }
            umma_commit(s.acc_full);
            // the accumulators must be complete before tensor memory is freed
            mbar_wait_bounded(s.acc_full, 0, p.err);
        }
    } else {
        // dequant warp d owns tile d of the row block; its loads run two k
        // steps ahead of the stores
        const uint32_t d = warp - 1 - kGemmMmaWarps * RBM;  // 0 .. 8 * RBM - 1
        const uint32_t T = rb * 8 * RBM + d;
        RawStep r0 = load_step<FMT>(p, T, k0, lane);
        RawStep r1 = nk > 1 ? load_step<FMT>(p, T, k0 + 1, lane) : r0;
        for (uint32_t i = 0; i < nk; ++i) {
            const uint32_t st = i % p.stages, pass = i / p.stages;
            const RawStep cur = r0;
            r0 = r1;
            if (i + 2 < nk) r1 = load_step<FMT>(p, T, k0 + i + 2, lane);
            if (pass > 0) mbar_wait_bounded(&s.w_empty[st], (pass - 1) & 1, p.err);
            dequant_store<FMT>(cur, s.w + st * wstage + (d / 8) * wst1, d % 8, lane);
            fence_proxy_async();
            mbar_arrive(&s.w_full[st]);
        }
        // epilogue: TMEM lane = output row, column = token
        // (two warps per TMEM lane quarter take alternate 16-column chunks)
        // warp w reads TMEM lanes 32*(w%4)..; among the dequant warps of one lane
        // quarter, j = d / 4 picks the row block (j % RBM) and the half of the
        // 16-column chunks (j / RBM)
        const uint32_t q = warp & 3, j4 = d >> 2, h = j4 % RBM, part = j4 / RBM;
        const uint32_t o = (rb * RBM + h) * kGemmBM + q * 32 + lane;
        const bool ok = nk == 0 || mbar_wait_bounded(s.acc_full, 0, p.err);
        tc_fence_after();
        const float rs = (FMT == 8 && o < p.rows) ? __ldg(p.row_scale + o) : 1.0f;
        const bool stk = gemm_stacked(p.bn);
        for (uint32_t c0 = 16 * part; c0 < p.bn; c0 += 32) {
            float v[16];
            if (nk > 0) {
                // the row block's first accumulator, then its second if that
                // MMA warp had k steps
                const uint32_t acols = stk ? 2 * p.bn : p.bn;
                const uint32_t a0 = h * kGemmMmaWarps * acols;
                tmem_ld16(tmem + ((q * 32) << 16) + a0 + c0, v);
                if (stk) {  // + the x_lo columns
                    float v2[16];
                    tmem_ld16(tmem + ((q * 32) << 16) + a0 + p.bn + c0, v2);
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] += v2[j];
                }
                for (uint32_t a = 1; a < (uint32_t)kGemmMmaWarps && a < nk; ++a) {
                    float v3[16];
                    tmem_ld16(tmem + ((q * 32) << 16) + a0 + a * acols + c0, v3);
                    if (stk) {
                        float v4[16];
                        tmem_ld16(tmem + ((q * 32) << 16) + a0 + a * acols + p.bn + c0, v4);
#pragma unroll
                        for (int j = 0; j < 16; ++j) v3[j] += v4[j];
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] += v3[j];
                }
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = 0.0f;
            }
            if (!ok || o >= p.rows) continue;
#pragma unroll
            for (uint32_t j = 0; j < 16; ++j) {
                const uint32_t n = nt * p.bn + c0 + j;
                if (n >= p.m) break;
                const float y = v[j] * rs;
                if (p.splits > 1) {
                    p.part[((size_t)split * p.m + n) * p.rows + o] = y;
                } else {
                    const size_t at = (size_t)n * p.out_stride + o;
                    p.out[at] = p.epilogue == B2_EPI_RESID ? p.resid[at] + y : y;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_free(tmem, p.tmem_cols);
    }
}

// Sum of the k splits in split order (+ residual).
__global__ void gemm_reduce_kernel(const float *__restrict__ part, uint32_t splits, uint32_t m, uint32_t rows,
                                   float *out, uint32_t out_stride, const float *resid, uint32_t epilogue)
{
    const size_t total = (size_t)m * rows;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t n = (uint32_t)(i / rows), o = (uint32_t)(i % rows);
        float y = 0.0f;
        for (uint32_t s = 0; s < splits; ++s) y += part[(size_t)s * total + i];
        const size_t at = (size_t)n * out_stride + o;
        out[at] = epilogue == B2_EPI_RESID ? resid[at] + y : y;
    }
}

// ---- host side ------------------------------------------------------------------------------

struct GemmPlan {
    uint32_t ntiles, bn, row_blocks, ksteps, splits, ksplit, stages, xk, smem, off_x, off_w, tmem_cols, nmma, rbm;
};

static bool plan_gemm(const b2_gemm_args *a, GemmPlan &pl)
{
    const b2_qweight &w = a->w;
    gemm_token_tiles(a->m, pl.ntiles, pl.bn);
    // small token tiles (decode batches): two 128-row blocks per CTA, so each k
    // step of the stage protocol carries twice the weights (the MMA issue and
    // the stage round trip, not the weight bytes, pace a k step there); their
    // four accumulators fit the 512 tensor-memory columns up to kGemmRb2MaxBn
    const uint32_t acols = gemm_stacked(pl.bn) ? 2 * pl.bn : pl.bn;
    pl.rbm = (pl.bn <= kGemmRb2MaxBn && 2 * kGemmMmaWarps * acols <= 512) ? 2 : 1;
    pl.row_blocks = (w.tiles + 8 * pl.rbm - 1) / (8 * pl.rbm);
    pl.ksteps = (w.cols + kGemmBK - 1) / kGemmBK;
    const uint32_t xst = gemm_x_stage_bytes(pl.bn), wst = pl.rbm * gemm_w_stage_bytes(w.format);
    const uint32_t head = 1024;  // mbarriers + TMEM slot, then 1 KB-aligned rings
    // X: two slots of xk k steps (about kGemmXCopy bytes per bulk copy: an SM
    // completes bulk copies at a bounded rate whatever their size); W: the rest
    uint32_t xk = kGemmXCopy / xst;
    if (xk < 1) xk = 1;
    if (xk > 8) xk = 8;
    uint32_t st = 0;
    for (;; xk = xk > 1 ? xk / 2 : 0) {
        if (xk == 0) return false;
        const uint32_t xbytes = kGemmXSlots * xk * xst;
        // at least two W stages; with two row blocks, a third before larger X copies
        if (head + xbytes + (pl.rbm == 2 && xk > 1 ? 3 : 2) * wst <= kGemmSmemLimit) {
            st = (kGemmSmemLimit - head - xbytes) / wst;
            break;
        }
    }
    if (st > kGemmMaxStages) st = kGemmMaxStages;
    pl.stages = st;
    pl.xk = xk;
    pl.off_x = head;
    pl.off_w = head + kGemmXSlots * xk * xst;
    pl.smem = pl.off_w + st * wst;
    // kGemmMmaWarps accumulators per row block (2 * 256 columns at most with one)
    pl.nmma = kGemmMmaWarps * pl.rbm;
    if (pl.nmma * acols > 512) return false;
    uint32_t tc = 32;
    while (tc < pl.nmma * acols) tc <<= 1;
    pl.tmem_cols = tc;
    // k splits: fill the SMs when row blocks x token tiles do not, at least 4 k steps each
    uint32_t splits = a->splits;
    if (splits == 0) {
        const uint32_t ctas = pl.row_blocks * pl.ntiles;
        splits = (uint32_t)sm_count() / (ctas ? ctas : 1);
        const uint32_t most = pl.ksteps / 4;
        if (splits > most) splits = most;
        if (splits > kGemmMaxSplits) splits = kGemmMaxSplits;
        if (splits < 1) splits = 1;
    }
    if (splits > pl.ksteps) splits = pl.ksteps;
    pl.ksplit = (pl.ksteps + splits - 1) / splits;
    pl.splits = (pl.ksteps + pl.ksplit - 1) / pl.ksplit;
    return true;
}

static int gemm_check(const b2_gemm_args *a)
{
    if (a == nullptr || a->w.data == nullptr || a->xs == nullptr || a->out == nullptr) return -1;
    const b2_qweight &w = a->w;
    if ((w.format != 4 && w.format != 8) || (w.format == 8 && w.row_scale == nullptr)) return -1;
    if (a->m == 0 || w.rows == 0 || w.cols == 0 || w.cols % 32) return -1;
    if (w.tiles != (w.rows + 15) / 16 || w.kunits != (w.format == 4 ? (w.cols + 63) / 64 : (w.cols + 31) / 32))
        return -1;
    if (((uintptr_t)w.data & 15) || ((uintptr_t)a->xs & 15)) return -1;
    if (a->out_stride < w.rows) return -1;
    if (a->epilogue != B2_EPI_STORE && a->epilogue != B2_EPI_RESID) return -1;
    if (a->epilogue == B2_EPI_RESID && a->resid == nullptr) return -1;
    if ((uint64_t)w.tiles * w.kunits >= (1ull << 32)) return -1;
    return 0;
}

template <int FMT, int RBM>
static cudaError_t launch_gemm(const GemmParams &p, const GemmPlan &pl, int pdl, cudaStream_t st)
{
    auto fn = att1_qgemm_kernel<FMT, RBM>;
    // the whole shared-memory window (one CTA per SM either way): operand reads
    // of the tensor cores stay inside the CTA's allocation whatever the stage count
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmemLimit);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.row_blocks, pl.ntiles, pl.splits);
    cfg.blockDim = dim3(gemm_threads<RBM>());
    cfg.dynamicSmemBytes = kGemmSmemLimit;
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

extern "C" size_t b2_gemm_xs_bytes(uint32_t m, uint32_t cols)
{
    uint32_t ntiles, bn;
    gemm_token_tiles(m, ntiles, bn);
    const size_t ksteps = (cols + kGemmBK - 1) / kGemmBK;
    return (size_t)ntiles * ksteps * gemm_x_stage_bytes(bn);
}

extern "C" int b2_gemm_prep(const float *x, uint32_t x_stride, uint32_t m, uint32_t cols, const float *norm_w,
                            float eps, void *xs, int32_t *err, void *stream)
{
    if (x == nullptr || xs == nullptr || m == 0 || cols == 0 || cols % 32 || x_stride < cols || (x_stride & 3) ||
        ((uintptr_t)x & 15) || ((uintptr_t)xs & 15))
        return -1;
    if (norm_w != nullptr && (((uintptr_t)norm_w & 15) || !(eps > 0.0f))) return -1;
    uint32_t ntiles, bn;
    gemm_token_tiles(m, ntiles, bn);
    const uint32_t ksteps = (cols + kGemmBK - 1) / kGemmBK;
    gemm_prep_kernel<<<ntiles * bn, 256, 0, (cudaStream_t)stream>>>(x, x_stride, m, cols, norm_w, eps, bn, ksteps,
                                                                     (uint8_t *)xs, err);
    return cudaGetLastError() == cudaSuccess ? 0 : -8;
}

extern "C" size_t b2_gemm_scratch_bytes(const b2_gemm_args *a)
{
    GemmPlan pl;
    if (a == nullptr || gemm_check(a) != 0 || !plan_gemm(a, pl)) return 0;
    return pl.splits > 1 ? (size_t)pl.splits * a->m * a->w.rows * sizeof(float) : 16;
}

extern "C" int b2_gemm(const b2_gemm_args *a, void *stream)
{
    const int rc = gemm_check(a);
    if (rc != 0) return rc;
    GemmPlan pl;
    if (!plan_gemm(a, pl)) return -9;
    const size_t need = pl.splits > 1 ? (size_t)pl.splits * a->m * a->w.rows * sizeof(float) : 0;
    if (need > 0 && (a->scratch == nullptr || a->scratch_bytes < need || ((uintptr_t)a->scratch & 15))) return -1;
    GemmParams p = {};
    p.w = (const uint8_t *)a->w.data;
    p.row_scale = a->w.row_scale;
    p.fmt = a->w.format;
    p.rows = a->w.rows;
    p.cols = a->w.cols;
    p.tiles = a->w.tiles;
    p.kunits = a->w.kunits;
    p.ksteps = pl.ksteps;
    p.xs = (const uint8_t *)a->xs;
    p.m = a->m;
    p.bn = pl.bn;
    p.ntiles = pl.ntiles;
    p.out = a->out;
    p.out_stride = a->out_stride;
    p.resid = a->resid;
    p.epilogue = a->epilogue;
    p.part = (float *)a->scratch;
    p.splits = pl.splits;
    p.ksplit = pl.ksplit;
    p.stages = pl.stages;
    p.xk = pl.xk;
    p.off_x = pl.off_x;
    p.off_w = pl.off_w;
    p.tmem_cols = pl.tmem_cols;
    p.nmma = pl.nmma;
    p.rbm = pl.rbm;
    p.err = a->err;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = a->w.format == 4 ? (pl.rbm == 2 ? launch_gemm<4, 2>(p, pl, a->pdl, st) : launch_gemm<4, 1>(p, pl, a->pdl, st))
                                     : (pl.rbm == 2 ? launch_gemm<8, 2>(p, pl, a->pdl, st) : launch_gemm<8, 1>(p, pl, a->pdl, st));
    if (e != cudaSuccess) return -8;
    if (pl.splits > 1) {
        const size_t total = (size_t)a->m * a->w.rows;
        uint32_t blocks = (uint32_t)((total + 255) / 256);
        const uint32_t cap = (uint32_t)sm_count() * 8;
        if (blocks > cap) blocks = cap;
        gemm_reduce_kernel<<<blocks, 256, 0, st>>>((const float *)a->scratch, pl.splits, a->m, a->w.rows, a->out,
                                                    a->out_stride, a->resid, a->epilogue);
        if (cudaGetLastError() != cudaSuccess) return -8;
    }
    return 0;
}
