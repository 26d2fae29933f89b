// b2_weights.cu - q4/q8 weights in the device unit layout.
//
// Packing from the reference wire format (src/quant.c:148-174 nibble order,
// include/att1_quant.h:19-38 tensor layout), the inverse, and a device-side
// seeded generator + quantiser that reproduces the reference quantiser
// (src/quant.c:127-146, :199-226 for q4; :61-116 for q8) bit for bit, so that
// large synthetic models are built on the GPU without a host copy.
#include "b2_common.cuh"

#include <cuda_runtime.h>

namespace b2 {

__host__ __device__ __forceinline__ uint32_t ceil_div(uint32_t a, uint32_t b) { return (a + b - 1) / b; }

// Source row of device row `row` (tile-local mapping for the gate/up interleave).
// Returns which source (0/1) and the row in it.
__device__ __forceinline__ void map_row(int map, uint32_t row, uint32_t &which, uint32_t &src_row)
{
    if (map == B2_ROWS_GATEUP) {
        const uint32_t t = row >> 4, r = row & 15;
        which = r >> 3;
        src_row = t * 8 + (r & 7);
    } else {
        which = 0;
        src_row = row;
    }
}

// Device row holding source row `src_row` of source `which`.
__device__ __forceinline__ uint32_t dev_row(int map, uint32_t which, uint32_t src_row)
{
    if (map == B2_ROWS_GATEUP) return (src_row >> 3) * 16 + which * 8 + (src_row & 7);
    return src_row;
}

// Index of unit (tile, k-unit): tile-major, a tile's k-units contiguous.
__device__ __forceinline__ size_t unit_index(uint32_t tile, uint32_t ku, uint32_t kunits)
{
    return (size_t)tile * kunits + ku;
}

// Byte offset of the nibble word for (device row, 32-col group, t) inside the
// unit array, relative to the first unit of the tensor.
__device__ __forceinline__ size_t q4_word_offset(uint32_t row, uint32_t g32, uint32_t t, uint32_t kunits)
{
    const uint32_t tile = row >> 4, r = row & 15;
    const uint32_t gp = g32 >> 1, gi = g32 & 1;
    const uint32_t lane = (r & 7) * 4 + t;
    const uint32_t word = gi * 2 + (r >> 3);
    return unit_index(tile, gp, kunits) * B2_Q4_UNIT_BYTES + lane * 16 + word * 4;
}

__device__ __forceinline__ size_t q4_scale_offset(uint32_t row, uint32_t g32, uint32_t kunits)
{
    const uint32_t tile = row >> 4, r = row & 15;
    const uint32_t gp = g32 >> 1, gi = g32 & 1;
    return unit_index(tile, gp, kunits) * B2_Q4_UNIT_BYTES + 512 + (r & 7) * 16 + ((r >> 3) * 2 + gi) * 4;
}

// Write one quantised group (32 signed nibbles, q[i] in [-7,7]) of device row.
__device__ __forceinline__ void q4_store_group(uint8_t *base, uint32_t row, uint32_t g32, uint32_t kunits,
                                               const int8_t (&q)[32], float scale)
{
#pragma unroll
    for (uint32_t t = 0; t < 4; ++t) {
        uint32_t w = 0;
#pragma unroll
        for (uint32_t i = 0; i < 4; ++i) {
            const uint32_t lo = (uint32_t)(uint8_t)q[4 * t + i] & 0xFu;
            const uint32_t hi = (uint32_t)(uint8_t)q[16 + 4 * t + i] & 0xFu;
            w |= (lo | (hi << 4)) << (8 * i);
        }
        *reinterpret_cast<uint32_t *>(base + q4_word_offset(row, g32, t, kunits)) = w;
    }
    *reinterpret_cast<float *>(base + q4_scale_offset(row, g32, kunits)) = scale;
}

// ---- q4 pack from the reference layout: one thread per (device row, 32-group)
__global__ void q4_pack_kernel(uint8_t *dst, uint32_t dst_rows, uint32_t cols, const uint8_t *p0,
                               const float *s0, const uint8_t *p1, const float *s1, uint32_t group,
                               int map, uint32_t row0)
{
    const uint32_t g32n = cols / 32;
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)dst_rows * g32n) return;
    const uint32_t row = (uint32_t)(idx / g32n), g32 = (uint32_t)(idx % g32n);
    uint32_t which, srow;
    map_row(map, row, which, srow);
    const uint8_t *P = which ? p1 : p0;
    const float *S = which ? s1 : s0;
    const uint8_t *src = P + (size_t)srow * (cols / 2) + g32 * 16;
    int8_t q[32];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const uint8_t b = src[j];
        q[2 * j] = (int8_t)((int8_t)(b << 4) >> 4);
        q[2 * j + 1] = (int8_t)((int8_t)b >> 4);
    }
    const float scale = S[(size_t)srow * (cols / group) + (g32 * 32) / group];
    q4_store_group(dst, row0 + row, g32, ceil_div(cols, 64), q, scale);
}

// ---- q4 unpack to the reference layout (group 32)
__global__ void q4_unpack_kernel(uint8_t *packed, float *scales, const uint8_t *src, uint32_t rows,
                                 uint32_t cols, int map, int which, uint32_t row0)
{
    const uint32_t g32n = cols / 32;
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)rows * g32n) return;
    const uint32_t srow = (uint32_t)(idx / g32n), g32 = (uint32_t)(idx % g32n);
    const uint32_t row = row0 + dev_row(map, (uint32_t)which, srow);
    const uint32_t kunits = ceil_div(cols, 64);
    uint8_t nib[32];
#pragma unroll
    for (uint32_t t = 0; t < 4; ++t) {
        const uint32_t w = *reinterpret_cast<const uint32_t *>(src + q4_word_offset(row, g32, t, kunits));
#pragma unroll
        for (uint32_t i = 0; i < 4; ++i) {
            nib[4 * t + i] = (w >> (8 * i)) & 0xFu;
            nib[16 + 4 * t + i] = (w >> (8 * i + 4)) & 0xFu;
        }
    }
    uint8_t *dst = packed + (size_t)srow * (cols / 2) + g32 * 16;
#pragma unroll
    for (int j = 0; j < 16; ++j) dst[j] = (uint8_t)(nib[2 * j] | (nib[2 * j + 1] << 4));
    scales[(size_t)srow * g32n + g32] = *reinterpret_cast<const float *>(src + q4_scale_offset(row, g32, kunits));
}

// ---- q4 synth: reference quantiser on generated groups. One thread per
// (source, source row, 32-group).
__global__ void q4_synth_kernel(uint8_t *dst, uint32_t dst_rows, uint32_t cols, uint64_t key0,
                                uint64_t key1, float c, int map, uint32_t row0, uint32_t src_row0,
                                uint32_t src_col0, uint32_t src_cols)
{
    const uint32_t g32n = cols / 32;
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)dst_rows * g32n) return;
    const uint32_t srcs = (map == B2_ROWS_GATEUP) ? 2u : 1u;
    const uint32_t src_rows = dst_rows / srcs;
    const uint32_t which = (uint32_t)(idx / ((uint64_t)src_rows * g32n));
    const uint64_t rem = idx % ((uint64_t)src_rows * g32n);
    const uint32_t srow = (uint32_t)(rem / g32n), g32 = (uint32_t)(rem % g32n);
    const uint64_t key = which ? key1 : key0;
    float v[32];
    float max_abs = 0.0f;
    const uint64_t e0 = (uint64_t)(src_row0 + srow) * src_cols + src_col0 + (uint64_t)g32 * 32;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        v[i] = synth_normal(key, e0 + i, c);
        const float a = fabsf(v[i]);
        if (a > max_abs) max_abs = a;
    }
    // src/quant.c:143: scale = max/7 (1 when the group is all zero)
    const float scale = (max_abs > 0.0f) ? __fdiv_rn(max_abs, 7.0f) : 1.0f;
    int8_t q[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        long r = lroundf(__fdiv_rn(v[i], scale));  // src/quant.c:215
        r = r > 7 ? 7 : (r < -7 ? -7 : r);
        q[i] = (int8_t)r;
    }
    q4_store_group(dst, row0 + dev_row(map, which, srow), g32, ceil_div(cols, 64), q, scale);
}

// ---- q8 layout helpers
__device__ __forceinline__ size_t q8_byte_offset(uint32_t row, uint32_t col, uint32_t kunits)
{
    const uint32_t tile = row >> 4, r = row & 15;
    const uint32_t kb = col >> 5, k = col & 31;
    const uint32_t t = (k & 15) >> 2, i = k & 3;
    const uint32_t lane = (r & 7) * 4 + t;
    const uint32_t reg = (k >> 4) * 2 + (r >> 3);
    return unit_index(tile, kb, kunits) * B2_Q8_UNIT_BYTES + lane * 16 + reg * 4 + i;
}

// One thread per (device row, 32-col block).
__global__ void q8_pack_kernel(uint8_t *dst, float *row_scale, uint32_t dst_rows, uint32_t cols,
                               const int8_t *v0, const float *s0, const int8_t *v1, const float *s1,
                               int map, uint32_t row0)
{
    const uint32_t kbn = ceil_div(cols, 32);
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)dst_rows * kbn) return;
    const uint32_t row = (uint32_t)(idx / kbn), kb = (uint32_t)(idx % kbn);
    uint32_t which, srow;
    map_row(map, row, which, srow);
    const int8_t *V = which ? v1 : v0;
    for (uint32_t k = 0; k < 32; ++k) {
        const uint32_t col = kb * 32 + k;
        const int8_t q = (col < cols) ? V[(size_t)srow * cols + col] : (int8_t)0;
        dst[q8_byte_offset(row0 + row, col, kbn)] = (uint8_t)q;
    }
    if (kb == 0) row_scale[row] = (which ? s1 : s0)[srow];
}

__global__ void q8_unpack_kernel(int8_t *values, float *scales, const uint8_t *src, const float *row_scale,
                                 uint32_t rows, uint32_t cols, int map, int which, uint32_t row0)
{
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)rows * cols) return;
    const uint32_t srow = (uint32_t)(idx / cols), col = (uint32_t)(idx % cols);
    const uint32_t row = dev_row(map, (uint32_t)which, srow);
    values[idx] = (int8_t)src[q8_byte_offset(row0 + row, col, ceil_div(cols, 32))];
    if (col == 0) scales[srow] = row_scale[row];
}

// q8 synth: one warp per source row (max over the row, then quantise).
__global__ void q8_synth_kernel(uint8_t *dst, float *row_scale, uint32_t dst_rows, uint32_t cols,
                                uint64_t key0, uint64_t key1, float c, int map, uint32_t row0, uint32_t src_row0,
                                uint32_t src_col0, uint32_t src_cols)
{
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t warp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (warp >= dst_rows) return;
    const uint32_t srcs = (map == B2_ROWS_GATEUP) ? 2u : 1u;
    const uint32_t src_rows = dst_rows / srcs;
    const uint32_t which = (uint32_t)(warp / src_rows), srow = (uint32_t)(warp % src_rows);
    const uint64_t key = which ? key1 : key0;
    // the scale comes from the whole source row, the values from its slice
    const uint64_t e0 = (uint64_t)(src_row0 + srow) * src_cols;
    float m = 0.0f;
    for (uint32_t k = lane; k < src_cols; k += 32) m = fmaxf(m, fabsf(synth_normal(key, e0 + k, c)));
    m = warp_max(m);
    // src/quant.c:97-99
    const float scale = (m > 0.0f) ? __fdiv_rn(m, 127.0f) : 1.0f;
    const uint32_t row = dev_row(map, which, srow);
    const uint32_t kbn = ceil_div(cols, 32);
    for (uint32_t k = lane; k < cols; k += 32) {
        long r = lroundf(__fdiv_rn(synth_normal(key, e0 + src_col0 + k, c), scale));
        r = r > 127 ? 127 : (r < -127 ? -127 : r);
        dst[q8_byte_offset(row0 + row, k, kbn)] = (uint8_t)(int8_t)r;
    }
    if (lane == 0) row_scale[row] = scale;
}

// q8 from device f32: one warp per device row; w (and w2 for the up half of
// a gate/up interleave) hold [src_rows][cols], or [cols][src_rows] transposed.
__global__ void q8_quantize_f32_kernel(uint8_t *dst, float *row_scale, uint32_t dst_rows, uint32_t cols,
                                       const float *w0, const float *w1, int transposed, int map,
                                       uint32_t row0)
{
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t row = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= dst_rows) return;
    uint32_t which, srow;
    map_row(map, (uint32_t)row, which, srow);
    const uint32_t src_rows = (map == B2_ROWS_GATEUP) ? dst_rows / 2 : dst_rows;
    const float *w = which ? w1 : w0;
    auto at = [&](uint32_t k) { return transposed ? w[(size_t)k * src_rows + srow] : w[(size_t)srow * cols + k]; };
    float m = 0.0f;
    for (uint32_t k = lane; k < cols; k += 32) m = fmaxf(m, fabsf(at(k)));
    m = warp_max(m);
    const float scale = (m > 0.0f) ? __fdiv_rn(m, 127.0f) : 1.0f;
    const uint32_t kbn = ceil_div(cols, 32);
    for (uint32_t k = lane; k < cols; k += 32) {
        long r = lroundf(__fdiv_rn(at(k), scale));
        r = r > 127 ? 127 : (r < -127 ? -127 : r);
        dst[q8_byte_offset(row0 + (uint32_t)row, k, kbn)] = (uint8_t)(int8_t)r;
    }
    if (lane == 0) row_scale[row] = scale;
}

__global__ void synth_f32_kernel(float *dst, size_t n, uint64_t key, float c)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = synth_normal(key, i, c);
}

__global__ void fill_f32_kernel(float *dst, size_t n, float v)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = v;
}

static unsigned grid_for(uint64_t n, unsigned block)
{
    uint64_t g = (n + block - 1) / block;
    return (unsigned)(g > 0x7fffffffull ? 0x7fffffffull : (g == 0 ? 1 : g));
}

}  // namespace b2

using namespace b2;

extern "C" size_t b2_q4_bytes(uint32_t rows, uint32_t cols)
{
    return (size_t)ceil_div(rows, 16) * ceil_div(cols, 64) * B2_Q4_UNIT_BYTES;
}

extern "C" size_t b2_q8_bytes(uint32_t rows, uint32_t cols)
{
    return (size_t)ceil_div(rows, 16) * ceil_div(cols, 32) * B2_Q8_UNIT_BYTES;
}

static int check_launch()
{
    return cudaGetLastError() == cudaSuccess ? 0 : -8;
}

extern "C" int b2_q4_pack(void *dst, uint32_t tile_offset, uint32_t dst_rows, uint32_t cols,
                          const uint8_t *packed, const float *scales, const uint8_t *packed2,
                          const float *scales2, uint32_t group, int map, void *stream)
{
    if (!dst || !packed || !scales || dst_rows == 0 || cols == 0 || cols % 32 ||
        (group != 32 && group != 64 && group != 128) || cols % group)
        return -1;
    if (map == B2_ROWS_GATEUP && (!packed2 || !scales2 || dst_rows % 16)) return -1;
    uint8_t *base = (uint8_t *)dst;
    const uint64_t n = (uint64_t)dst_rows * (cols / 32);
    q4_pack_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(base, dst_rows, cols, packed, scales,
                                                                       packed2, scales2, group, map, tile_offset * 16);
    return check_launch();
}

extern "C" int b2_q4_unpack(uint8_t *packed, float *scales, const void *src, uint32_t tile_offset,
                            uint32_t rows, uint32_t cols, int map, int which, void *stream)
{
    if (!packed || !scales || !src || rows == 0 || cols == 0 || cols % 32 || which < 0 || which > 1) return -1;
    if (map == B2_ROWS_GATEUP && rows % 8) return -1;
    const uint8_t *base = (const uint8_t *)src;
    const uint64_t n = (uint64_t)rows * (cols / 32);
    q4_unpack_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(packed, scales, base, rows, cols, map,
                                                                         which, tile_offset * 16);
    return check_launch();
}

extern "C" int b2_q4_synth_part(void *dst, uint32_t tile_offset, uint32_t dst_rows, uint32_t cols, uint64_t seed,
                                uint64_t tensor_id, uint64_t tensor_id2, float std, int map, uint32_t src_row0,
                                uint32_t src_col0, uint32_t src_cols, void *stream)
{
    if (!dst || dst_rows == 0 || cols == 0 || cols % 32 || src_col0 % 32 || src_col0 + cols > src_cols) return -1;
    if (map == B2_ROWS_GATEUP && dst_rows % 16) return -1;
    uint8_t *base = (uint8_t *)dst;
    const float c = std * (1.0f / 131072.0f);
    const uint64_t n = (uint64_t)dst_rows * (cols / 32);
    q4_synth_kernel<<<grid_for(n, 128), 128, 0, (cudaStream_t)stream>>>(
        base, dst_rows, cols, synth_key(seed, tensor_id), synth_key(seed, tensor_id2), c, map, tile_offset * 16,
        src_row0, src_col0, src_cols);
    return check_launch();
}

extern "C" int b2_q4_synth(void *dst, uint32_t tile_offset, uint32_t dst_rows, uint32_t cols, uint64_t seed,
                           uint64_t tensor_id, uint64_t tensor_id2, float std, int map, void *stream)
{
    return b2_q4_synth_part(dst, tile_offset, dst_rows, cols, seed, tensor_id, tensor_id2, std, map, 0, 0, cols,
                            stream);
}

extern "C" int b2_q8_pack(void *dst, float *row_scale, uint32_t tile_offset, uint32_t dst_rows, uint32_t cols,
                          const int8_t *values, const float *scales, const int8_t *values2,
                          const float *scales2, int map, void *stream)
{
    if (!dst || !row_scale || !values || !scales || dst_rows == 0 || cols == 0) return -1;
    if (map == B2_ROWS_GATEUP && (!values2 || !scales2 || dst_rows % 16)) return -1;
    uint8_t *base = (uint8_t *)dst;
    const uint64_t n = (uint64_t)dst_rows * ceil_div(cols, 32);
    q8_pack_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(
        base, row_scale + (size_t)tile_offset * 16, dst_rows, cols, values, scales, values2, scales2, map,
        tile_offset * 16);
    return check_launch();
}

extern "C" int b2_q8_unpack(int8_t *values, float *scales, const void *src, const float *row_scale,
                            uint32_t tile_offset, uint32_t rows, uint32_t cols, int map, int which, void *stream)
{
    if (!values || !scales || !src || !row_scale || rows == 0 || cols == 0 || which < 0 || which > 1) return -1;
    if (map == B2_ROWS_GATEUP && rows % 8) return -1;
    const uint8_t *base = (const uint8_t *)src;
    const uint64_t n = (uint64_t)rows * cols;
    q8_unpack_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(
        values, scales, base, row_scale + (size_t)tile_offset * 16, rows, cols, map, which, tile_offset * 16);
    return check_launch();
}

extern "C" int b2_q8_synth_part(void *dst, float *row_scale, uint32_t tile_offset, uint32_t dst_rows,
                                uint32_t cols, uint64_t seed, uint64_t tensor_id, uint64_t tensor_id2, float std,
                                int map, uint32_t src_row0, uint32_t src_col0, uint32_t src_cols, void *stream)
{
    if (!dst || !row_scale || dst_rows == 0 || cols == 0 || src_col0 + cols > src_cols) return -1;
    if (map == B2_ROWS_GATEUP && dst_rows % 16) return -1;
    uint8_t *base = (uint8_t *)dst;
    const float c = std * (1.0f / 131072.0f);
    q8_synth_kernel<<<grid_for((uint64_t)dst_rows * 32, 256), 256, 0, (cudaStream_t)stream>>>(
        base, row_scale + (size_t)tile_offset * 16, dst_rows, cols, synth_key(seed, tensor_id),
        synth_key(seed, tensor_id2), c, map, tile_offset * 16, src_row0, src_col0, src_cols);
    return check_launch();
}

extern "C" int b2_q8_synth(void *dst, float *row_scale, uint32_t tile_offset, uint32_t dst_rows, uint32_t cols,
                           uint64_t seed, uint64_t tensor_id, uint64_t tensor_id2, float std, int map,
                           void *stream)
{
    return b2_q8_synth_part(dst, row_scale, tile_offset, dst_rows, cols, seed, tensor_id, tensor_id2, std, map, 0, 0,
                            cols, stream);
}

extern "C" int b2_synth_f32(float *dst, size_t count, uint64_t seed, uint64_t tensor_id, float std, void *stream)
{
    if (!dst || count == 0) return -1;
    synth_f32_kernel<<<grid_for(count, 256) > 65535u ? 65535u : grid_for(count, 256), 256, 0,
                       (cudaStream_t)stream>>>(dst, count, synth_key(seed, tensor_id), std * (1.0f / 131072.0f));
    return check_launch();
}

extern "C" int b2_fill_f32(float *dst, size_t count, float value, void *stream)
{
    if (!dst || count == 0) return -1;
    fill_f32_kernel<<<grid_for(count, 256) > 65535u ? 65535u : grid_for(count, 256), 256, 0,
                      (cudaStream_t)stream>>>(dst, count, value);
    return check_launch();
}

extern "C" int b2_q8_quantize_f32(void *dst, float *row_scale, uint32_t tile_offset, uint32_t dst_rows, uint32_t cols,
                                  const float *w, const float *w2, int transposed, int map, void *stream)
{
    if (!dst || !row_scale || !w || dst_rows == 0 || cols == 0) return -1;
    if (map == B2_ROWS_GATEUP && (!w2 || dst_rows % 16)) return -1;
    uint8_t *base = (uint8_t *)dst;
    q8_quantize_f32_kernel<<<grid_for((uint64_t)dst_rows * 32, 256), 256, 0, (cudaStream_t)stream>>>(
        base, row_scale + (size_t)tile_offset * 16, dst_rows, cols, w, w2, transposed, map, tile_offset * 16);
    return check_launch();
}
