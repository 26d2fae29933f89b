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
// Streaming. Weights sit in the tile-major unit layout of b2_kernels.h. Each
// CTA owns whole 16-row tiles (a contiguous range of the unit stream; at most
// one tile more than the lightest CTA), so no partial sum leaves the CTA.
// One producer lane copies the range into a shared-memory ring of up to
// kMaxStages stages of kStageUnits units with single 1-D bulk copies
// (cp.async.bulk, completion counted in bytes on the stage's "full"
// mbarrier). Consumer warp w multiplies units w, w + 16, ... of every stage,
// keeps one tile's sums in registers and, when its units move on to the next
// tile, stores them in its own slot of the round's per-warp tile sums; it
// releases each stage on its "empty" mbarrier, so the warps never meet at a
// CTA barrier while streaming. At the end of a round (the CTA's tiles, or a
// share of them when shared memory is short) one CTA barrier, then the warps
// add each tile's slots in warp order (deterministic) and run the tile
// epilogues, one warp per tile. The producer requests the first stages
// before griddepcontrol.wait, so under programmatic dependent launch the
// weight fetch overlaps the previous kernel.
//
// Measured alternatives, slower: splitting the k range of tiles between CTAs
// (stream-K) balances the CTAs exactly but every shared tile costs a global
// partial, a fence and an atomic ticket, and the last CTA of each tile adds
// the partials: those round trips made the end of every launch 3-7 us long;
// a cross-warp reduction per tile at the moment the tile ends (the last warp
// adds sixteen partials while the ring waits for it: half the speed); small
// bulk copies (an SM completes roughly one bulk copy per 0.4-0.6 us almost
// whatever its size, so tens of KB per copy are needed); per-warp contiguous
// ranges read with register prefetch (~2400 small streams over HBM, under
// 2.5 TB/s without arithmetic); a ring refilled by 16-byte cp.async from one
// warp.
#include "b2_gemv.cuh"

#include <cfloat>
#include <cstdio>
#include <cuda_runtime.h>
namespace b2 {

template <int FMT, int NI>
__global__ void __launch_bounds__(kThreads, 1) att1_qgemv_kernel(const GemvParams p)
{
    extern __shared__ __align__(128) uint8_t smem[];
    GemvSmem s = gemv_smem(smem, p);
    s.xready = s.full + 2 * kMaxStages;  // after the ring's full / empty barriers
    if (threadIdx.x == 0) gemv_init_barriers(s);
    __syncthreads();
    uint32_t i = 0;
    if ((threadIdx.x >> 5) == kWarps) {
        bool waited = false;
        gemv_produce<FMT>(p, s, i, waited);
        if (!waited) {
            pdl_wait();
            pdl_launch_dependents();
        }
        return;
    }
    uint32_t t0, t1;
    cta_range(p, t0, t1);
    if (t0 != t1) gemv_zero_round(p, s);  // before the wait: nothing of the previous kernel's
    pdl_wait();
    pdl_launch_dependents();
    bool dead = false;
    gemv_consume<FMT, NI>(p, s, i, dead, true);
}

// ---- host side ------------------------------------------------------------------

static int g_sm_count = 0;

int sm_count()
{
    if (g_sm_count == 0) {
        int dev = 0, n = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return 148;
        g_sm_count = n;
    }
    return g_sm_count;
}


bool plan_gemv(const b2_gemv_args *a, GemvPlan &pl)
{
    const uint32_t fmt = a->w.format;
    const uint32_t UB = fmt == 4 ? B2_Q4_UNIT_BYTES : B2_Q8_UNIT_BYTES;
    const uint32_t KW = fmt == 4 ? 64u : 32u;
    const uint32_t T = a->w.tiles;
    if (T == 0 || a->w.kunits == 0) return false;
    // one CTA per SM, whole tiles per CTA
    int grid = a->grid > 0 ? a->grid : sm_count();
    if ((uint32_t)grid > T) grid = (int)T;
    if (grid < 1) grid = 1;
    if ((uint64_t)T * (uint64_t)grid >= (1ull << 32)) return false;  // 32-bit index arithmetic in the kernel
    if ((uint64_t)T * a->w.kunits >= (1ull << 32)) return false;
    pl.grid = grid;
    const uint32_t per_cta = (T + grid - 1) / grid;
    // shared memory: mbarriers | stage ring | digit planes | per-warp tile
    // buffers | per-warp tile sums of a round | misc. Prefer kPreferStages ring
    // stages, then as many tiles per round as fit (rounds of fewer tiles add a CTA
    // barrier each), then the ring takes what is left, up to kMaxStages.
    const uint32_t xdig = a->w.kunits * a->batch * 3 * KW;
    const uint32_t tbuf = kWarps * 16 * a->batch * 4;
    const uint32_t misc = (kMaxItems * kWarps * 2 + kMaxItems) * 4 + kMaxItems * 8;
    const uint32_t fixed = 2 * kMaxStages * 8 + 128 + xdig + 128 + tbuf + 16 + misc + 16;
    const uint32_t per_tile = kWarps * 16 * a->batch * 4;
    const uint32_t stage = kStageUnits * UB;
    const uint32_t limit = 227u * 1024u;
    if (fixed + 2 * stage + per_tile > limit) return false;
    uint32_t rt = 0;
    for (uint32_t want = kPreferStages; want >= 2 && rt == 0; --want)
        if (fixed + want * stage + per_tile <= limit) rt = (limit - fixed - want * stage) / per_tile;
    if (rt > per_cta) rt = per_cta;
    if (rt < 1) rt = 1;
    uint32_t ns = (limit - fixed - rt * per_tile) / stage;
    if (ns > kMaxStages) ns = kMaxStages;
    pl.round_tiles = rt;
    pl.stages = ns;
    uint32_t off = 2 * kMaxStages * 8 + 8;  // full / empty barriers, x-ready barrier
    off = (off + 127) & ~127u;
    pl.off_ring = off;
    off += ns * stage;
    pl.off_xdig = off;
    off += xdig;
    off = (off + 127) & ~127u;
    pl.off_tile = off;
    off += tbuf;
    pl.off_parts = off;
    off += rt * per_tile;
    off = (off + 15) & ~15u;
    pl.off_misc = off;
    off += misc;
    pl.smem = off;
    // no partial sums leave the CTA: the scratch and counters of the ABI are
    // not used (a minimal size keeps callers that allocate them working)
    pl.partial_bytes = 256;
    pl.counter_len = 1;
    return true;
}

template <int FMT, int NI>
static cudaError_t launch_t(const GemvParams &p, const GemvPlan &pl, int pdl, cudaStream_t st)
{
    auto fn = att1_qgemv_kernel<FMT, NI>;
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

static int tp_check(const b2_tp &tp)
{
    if (tp.world < 2 || tp.world > B2_TP_MAX || tp.rank >= tp.world || tp.epoch == nullptr) return -1;
    for (uint32_t s = 0; s < tp.world; ++s)
        if (tp.peer[s] == nullptr || ((uintptr_t)tp.peer[s] & 15)) return -1;
    if (tp.slot_floats % 4 || tp.logit_floats % 4) return -1;
    return 0;
}

int gemv_check(const b2_gemv_args *a)
{
    if (a == nullptr || a->w.data == nullptr) return -1;
    const bool tp = a->tp.world > 1;
    const bool tp_input = tp && a->tp.in_point != B2_TP_NONE;
    if (tp && tp_check(a->tp) != 0) return -1;
    if (tp_input && (a->tp.in_point >= a->tp.points || a->tp.in_resid == nullptr ||
                     (size_t)a->w.cols * a->batch > a->tp.slot_floats || ((uintptr_t)a->tp.in_resid & 15) ||
                     ((uintptr_t)a->tp.in_out & 15)))
        return -1;
    if (!tp_input && a->x == nullptr) return -1;
    if (a->epilogue != B2_EPI_PUSH && a->out == nullptr) return -1;
    const b2_qweight &w = a->w;
    if ((w.format != 4 && w.format != 8) || (w.format == 8 && w.row_scale == nullptr)) return -1;
    if (a->batch == 0 || a->batch > kMaxItems || w.cols == 0 || w.cols % 32 || w.rows == 0) return -1;
    if (w.tiles != (w.rows + 15) / 16 || w.kunits != (w.format == 4 ? (w.cols + 63) / 64 : (w.cols + 31) / 32)) return -1;
    if (!tp_input && (a->x_stride < w.cols || (a->x_stride & 3) || ((uintptr_t)a->x & 15))) return -1;
    if (a->norm_w != nullptr && (((uintptr_t)a->norm_w & 15) || !(a->eps > 0.0f))) return -1;
    if (((uintptr_t)w.data & 15)) return -1;
    switch (a->epilogue) {
    case B2_EPI_STORE:
    case B2_EPI_LOGITS:
        if (a->out_stride < w.rows) return -1;
        if (a->epilogue == B2_EPI_LOGITS && a->argmax == nullptr) return -1;
        if (a->epilogue == B2_EPI_LOGITS && tp &&
            (a->tp.out_point != a->tp.points || a->tp.done == nullptr ||
             (size_t)w.rows * a->batch > a->tp.logit_floats))
            return -1;
        break;
    case B2_EPI_PUSH:
        if (!tp || a->tp.done == nullptr || a->tp.out_point >= a->tp.points ||
            (size_t)w.rows * a->batch > a->tp.slot_floats)
            return -1;
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
    return 0;
}

void gemv_params(const b2_gemv_args *a, const GemvPlan &pl, GemvParams &p)
{
    const b2_qweight &w = a->w;
    p = GemvParams{};
    p.data = (const uint8_t *)w.data;
    p.row_scale = w.row_scale;
    p.rows = w.rows;
    p.cols = w.cols;
    p.tiles = w.tiles;
    p.kunits = w.kunits;
    p.round_tiles = pl.round_tiles;
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
    p.tp = a->tp;
    p.grid = (uint32_t)pl.grid;
    p.err = a->err;
    p.off_ring = pl.off_ring;
    p.stages = pl.stages;
    p.off_xdig = pl.off_xdig;
    p.off_tile = pl.off_tile;
    p.off_parts = pl.off_parts;
    p.off_misc = pl.off_misc;
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
    const int rc = gemv_check(a);
    if (rc != 0) return rc;
    GemvPlan pl;
    if (!plan_gemv(a, pl)) return -9;  // batch x columns too large for on-chip digit planes
    if (a->scratch == nullptr || a->scratch_bytes < pl.partial_bytes || ((uintptr_t)a->scratch & 255)) return -1;
    if (a->counters == nullptr || a->counters_len < pl.counter_len) return -1;
    GemvParams p;
    gemv_params(a, pl, p);
    const int NI = (a->batch + 1) / 2;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    if (a->w.format == 4) {
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

extern "C" size_t b2_tp_region_bytes(uint32_t points, uint32_t slot_floats, uint32_t logit_floats)
{
    return ((size_t)(points + 1) * B2_TP_MAX + B2_TP_MAX * B2_TP_MAX_ITEMS) * sizeof(uint64_t) +
           ((size_t)points * B2_TP_MAX * slot_floats + (size_t)B2_TP_MAX * logit_floats) * sizeof(float);
}
