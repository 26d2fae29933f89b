// b2_common.cuh - device helpers shared by the sm_100a kernels.
//
// PTX wrappers for the pieces the kernels build on: mbarrier + 1-D bulk
// copies (cp.async.bulk, the TMA engine without a tensor map), the int8
// tensor-core MMA used by the dequant GEMVs, programmatic dependent launch,
// and bounded waits that report a timeout through an error word instead of
// spinning forever.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "b2_kernels.h"

namespace b2 {

// SMs of the current device (host; defined in b2_gemv.cu).
int sm_count();

// ---- error word ------------------------------------------------------------
__device__ __forceinline__ void raise_error(int32_t *err, int32_t bit)
{
    if (err != nullptr) atomicOr(err, bit);
}

// Greedy-sampler key of a logit: the float's order as an unsigned integer
// (-0 and +0 equal); the high word of an argmax key whose low word is
// 0xFFFFFFFF - id, so the largest key is the largest logit with the lowest id.
__device__ __forceinline__ uint32_t ordered_key(float f)
{
    uint32_t b = __float_as_uint(f == 0.0f ? 0.0f : f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// ---- shared-memory addressing --------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait: gives up after ~`limit` polls (each poll may suspend for a
// hardware-chosen interval), raises B2_ERR_TIMEOUT and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int32_t *err)
{
    constexpr uint32_t limit = 1u << 22;
    for (uint32_t i = 0; i < limit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
    }
    raise_error(err, B2_ERR_TIMEOUT);
    return false;
}

// 1-D bulk copy global -> shared, completion signalled on `bar` (tx bytes).
// Both addresses 16-byte aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// The same copy for data read once per step (weights, KV rows), with an L2
// evict-first policy: the stream of gigabytes per step then does not push out
// of L2 what the step does reuse (activations, partial sums, counters, the
// kernels' code).
__device__ __forceinline__ uint64_t l2_evict_first_policy()
{
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_g2s_stream(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// ---- programmatic dependent launch -------------------------------------------------
__device__ __forceinline__ void pdl_wait()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void pdl_launch_dependents()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- int8 tensor-core MMA: D[16x8] = A[16x32] * B[32x8] + C ------------------------
// Fragment layout (PTX ISA, mma.m16n8k32 .s8): lane = 4*g + t;
//   A regs: {row g, k 4t..4t+3}, {row g+8, k 4t..}, {row g, k 16+4t..}, {row g+8, k 16+4t..}
//   B regs: {k 4t..4t+3, col g}, {k 16+4t.., col g}
//   C/D:    {row g, col 2t}, {row g, col 2t+1}, {row g+8, col 2t}, {row g+8, col 2t+1}
__device__ __forceinline__ void imma_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                           uint32_t a3, uint32_t b0, uint32_t b1, int c0, int c1,
                                           int c2, int c3)
{
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c2), "r"(c3));
}

// ---- reductions ----------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide reductions over all threads of the block; `red` holds >= 32 floats.
// Deterministic (fixed tree order). Every thread receives the result.
__device__ __forceinline__ float block_sum(float v, float *red)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = (lane < nwarps) ? red[lane] : 0.0f;
    r = warp_sum(r);
    return r;
}

__device__ __forceinline__ float block_max(float v, float *red)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = (lane < nwarps) ? red[lane] : 0.0f;
    r = warp_max(r);
    return r;
}

// ---- loads that bypass L1 (data written by other SMs in the same kernel) -------
__device__ __forceinline__ float ld_cg(const float *p) { return __ldcg(p); }

// ---- tensor-parallel exchange region (layout in b2_kernels.h) ---------------------
__device__ __forceinline__ uint64_t *tp_flag(uint8_t *region, uint32_t point, uint32_t src)
{
    return reinterpret_cast<uint64_t *>(region) + (size_t)point * B2_TP_MAX + src;
}

__device__ __forceinline__ uint64_t *tp_key(uint8_t *region, const b2_tp &tp, uint32_t src, uint32_t item)
{
    return reinterpret_cast<uint64_t *>(region) + (size_t)(tp.points + 1) * B2_TP_MAX + src * B2_TP_MAX_ITEMS + item;
}

__device__ __forceinline__ float *tp_slot(uint8_t *region, const b2_tp &tp, uint32_t point, uint32_t src)
{
    float *slots = reinterpret_cast<float *>(reinterpret_cast<uint64_t *>(region) + (size_t)(tp.points + 1) * B2_TP_MAX +
                                             B2_TP_MAX * B2_TP_MAX_ITEMS);
    if (point < tp.points) return slots + ((size_t)point * B2_TP_MAX + src) * tp.slot_floats;
    return slots + (size_t)tp.points * B2_TP_MAX * tp.slot_floats + (size_t)src * tp.logit_floats;
}

__device__ __forceinline__ void st_release_sys(uint64_t *p, uint64_t v)
{
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t *p)
{
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Acquire-release atomic add at system scope: this thread's earlier writes
// (and, after a CTA barrier, the CTA's) are performed before the add, and the
// adds it reads from are visible to it afterwards.
__device__ __forceinline__ int atom_add_acq_rel_sys(int *p, int v)
{
    int old;
    asm volatile("atom.acq_rel.sys.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ uint64_t tp_want(const b2_tp &tp)
{
    return (uint64_t)__ldcg(tp.epoch) + 1;
}

// Bounded wait (one thread) until every rank has set its flag of `point` in
// this rank's region for this step; false (and B2_ERR_TIMEOUT) on timeout.
__device__ __forceinline__ bool tp_wait(const b2_tp &tp, uint32_t point, int32_t *err)
{
    const uint64_t want = tp_want(tp);
    const uint32_t limit = tp.wait_polls != 0 ? tp.wait_polls : (1u << 24);
    uint8_t *own = tp.peer[tp.rank];
    for (uint32_t s = 0; s < tp.world; ++s) {
        uint32_t spins = 0;
        while (ld_acquire_sys(tp_flag(own, point, s)) < want) {
            if (++spins > limit) {
                raise_error(err, B2_ERR_TIMEOUT);
                return false;
            }
            __nanosleep(64);
        }
    }
    return true;
}

// One thread: publish this rank's contribution to `point` to every rank with
// system-scope release stores (the CTAs' stores to the slots were ordered
// before them by the acquire-release adds that chain the CTAs).
__device__ __forceinline__ void tp_signal(const b2_tp &tp, uint32_t point)
{
    const uint64_t v = tp_want(tp);
    for (uint32_t s = 0; s < tp.world; ++s) st_release_sys(tp_flag(tp.peer[s], point, tp.rank), v);
}

// ---- seeded synthetic generator (bit-identical to or_synth_normal) -------------
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x)
{
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ uint64_t synth_key(uint64_t seed, uint64_t tensor_id)
{
    return splitmix64(splitmix64(seed) ^ (tensor_id * 0xD1B54A32D192ED03ull));
}

__host__ __device__ __forceinline__ uint32_t sum16x4(uint64_t r)
{
    return (uint32_t)(r & 0xFFFFu) + (uint32_t)((r >> 16) & 0xFFFFu) +
           (uint32_t)((r >> 32) & 0xFFFFu) + (uint32_t)(r >> 48);
}

// Element e of tensor (seed, key): Irwin-Hall sum of twelve 16-bit uniforms,
// an exact integer, times one f32 constant: same bits on host and device.
__device__ __forceinline__ float synth_normal(uint64_t key, uint64_t e, float c)
{
    const uint32_t s = sum16x4(splitmix64(key + 3u * e)) + sum16x4(splitmix64(key + 3u * e + 1u)) +
                       sum16x4(splitmix64(key + 3u * e + 2u));
    return __fmul_rn((float)((int32_t)(2u * s) - 786420), c);
}

}  // namespace b2
