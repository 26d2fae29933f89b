// b2_decode.cu - one decode step (all layers of one token) as one persistent kernel.
//
// The step of src/infer.c:656-880 is a chain of dependent operations:
// embedding row, then per layer QKV GEMV (RMSNorm prologue, RoPE + KV append),
// attention, WO GEMV (+ residual), gate/up GEMV (RMSNorm, SwiGLU), down GEMV
// (+ residual), then the lm_head GEMV with the greedy argmax and the token /
// position update. Launched as 160+ kernels, every kernel pays a launch, a
// pipeline fill at the start and a drain at the end, and the weight stream
// stops at every boundary.
//
// Here one cooperative launch of one CTA per SM runs the whole chain. The CTA
// keeps the GEMV's split (b2_gemv.cuh): one producer warp and sixteen consumer
// warps around a ring of bulk-copy stages. The producer walks the weight
// stream of every GEMV of the step in order and never waits for the
// activations, so while the consumers wait at an operation boundary (or run
// the attention) the ring keeps filling with the next matrix. The consumers
// run the operations in order, separated by a grid barrier: a monotonic
// arrival counter in global memory; the counter base of a step comes from a
// step epoch that the last operation advances, so no reset is needed between
// launches. Every wait is bounded and reports B2_ERR_TIMEOUT through the
// error word; after a timeout the consumers keep the ring protocol (so the
// producer finishes) and skip the rest of the work.
//
// Attention partial sums use one scratch region and one counter array:
// operations are separated by grid barriers and each leaves its counters at
// zero. (A GEMV keeps its partial sums inside the CTA.)
#include "b2_attn.cuh"
#include "b2_gemv.cuh"

#include <cstring>
#include <new>
#include <vector>

namespace b2 {

enum : int { OP_BEGIN = 0, OP_GEMV = 1, OP_ATTN = 2, OP_END = 3 };

constexpr uint32_t kGridSpinLimit = 1u << 24;  // polls of the grid barrier (~1 s with the back-off)
constexpr uint32_t kMinAttnChunk = 16;         // positions per attention work item, at least

struct DecodeOp {
    int kind;
    int fmt;       // OP_GEMV: 4 or 8
    GemvParams g;  // OP_GEMV
    AttnParams a;  // OP_ATTN
};

struct GridBar {
    unsigned long long count;  // arrivals, monotonic over steps
    unsigned long long epoch;  // finished steps
};

struct DecodeParams {
    const DecodeOp *ops;
    uint32_t nops, batch, d_model, vocab, lp, attn_chunks;
    const float *embed;
    const uint32_t *tokens_in;
    uint32_t *tokens_out;
    int32_t *positions;
    unsigned long long *argmax;
    float *x;
    GridBar *bar;
    int32_t *err;
    uint32_t off_ring, off_shared, off_tile, off_parts, off_misc, off_ops, stages;
};

struct ConsumerSync {
    __device__ void operator()() const { consumer_sync(); }
};

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Consumer threads of every CTA: this CTA has finished the previous
// operation; return once all CTAs have (false after a timeout). A CTA that
// already timed out (`wait` false) only arrives, so a failed step ends after
// one timeout instead of one per operation.
__device__ __forceinline__ bool grid_sync(GridBar *bar, unsigned long long target, int32_t *err, int *flag,
                                          bool wait)
{
    consumer_sync();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(&bar->count, 1ull);
        int ok = wait ? 1 : 0;
        uint32_t spins = 0;
        while (wait && ld_acquire_u64(&bar->count) < target) {
            if (++spins > kGridSpinLimit) {
                raise_error(err, B2_ERR_TIMEOUT);
                ok = 0;
                break;
            }
            __nanosleep(64);
        }
        __threadfence();
        *flag = ok;
    }
    consumer_sync();
    return *flag != 0;
}

// Embedding rows of this step's tokens (src/infer.c:713-715), split over all CTAs.
__device__ void op_begin(const DecodeParams &dp)
{
    const uint32_t n4 = dp.d_model / 4, total = dp.batch * n4;
    for (uint32_t e = blockIdx.x * kConsumers + threadIdx.x; e < total; e += gridDim.x * kConsumers) {
        const uint32_t b = e / n4, j = e % n4;
        const uint32_t tok = dp.tokens_in[b];
        float4 v = make_float4(0, 0, 0, 0);
        if (tok < dp.vocab) v = __ldg(reinterpret_cast<const float4 *>(dp.embed + (size_t)tok * dp.d_model) + j);
        reinterpret_cast<float4 *>(dp.x + (size_t)b * dp.d_model)[j] = v;
    }
    if (blockIdx.x == 0 && threadIdx.x < dp.batch) {
        if (dp.tokens_in[threadIdx.x] >= dp.vocab) raise_error(dp.err, B2_ERR_TOKEN);
        dp.argmax[threadIdx.x] = 0ull;
    }
}

// Greedy token from the argmax key (src/sampler.c:5-34, lowest id wins ties),
// position advance (src/infer.c:878), step epoch.
__device__ void op_end(const DecodeParams &dp)
{
    if (blockIdx.x != 0) return;
    if (threadIdx.x < dp.batch) {
        const uint32_t b = threadIdx.x;
        const unsigned long long key = __ldcg(dp.argmax + b);
        if (key == 0ull) raise_error(dp.err, B2_ERR_NAN_LOGITS);
        else dp.tokens_out[b] = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
        dp.positions[b] += 1;
    }
    if (threadIdx.x == 0) atomicAdd(&dp.bar->epoch, 1ull);
}

template <int LP, int MG>
__device__ void attn_items(const AttnParams &a, const DecodeParams &dp, uint8_t *sbase)
{
    const uint32_t NC = dp.attn_chunks;  // chunks per (item, KV head), at most
    const uint32_t nwork = a.batch * a.n_kv_heads * NC;
    const AttnSmem sm = attn_smem<LP, kWarps>(sbase, a.group);
    for (uint32_t w = blockIdx.x; w < nwork; w += gridDim.x) {
        const uint32_t item = w / (a.n_kv_heads * NC), kvh = (w / NC) % a.n_kv_heads, c = w % NC;
        const int32_t pos = a.positions[item];
        if (pos < 0 || (uint32_t)pos >= a.max_ctx) {
            if (threadIdx.x == 0 && kvh == 0 && c == 0) raise_error(a.err, B2_ERR_POSITION);
            continue;
        }
        const uint32_t len = (uint32_t)pos + 1;
        uint32_t nc = (len + kMinAttnChunk - 1) / kMinAttnChunk;
        if (nc > NC) nc = NC;
        if (c >= nc) continue;
        const uint32_t p0 = (uint32_t)((uint64_t)c * len / nc), p1 = (uint32_t)((uint64_t)(c + 1) * len / nc);
        attn_chunk<LP, MG, kWarps>(a, sm, item, kvh, c, nc, p0, p1, ConsumerSync());
    }
}

template <int NI>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeParams dp)
{
    extern __shared__ __align__(128) uint8_t smem[];
    GemvSmem s;
    s.full = reinterpret_cast<uint64_t *>(smem);
    s.empty = s.full + kMaxStages;
    s.ring = smem + dp.off_ring;
    s.xdig = smem + dp.off_shared;
    s.tbufs = reinterpret_cast<float *>(smem + dp.off_tile);
    s.parts = reinterpret_cast<float *>(smem + dp.off_parts);
    s.red = reinterpret_cast<float *>(smem + dp.off_misc);
    s.item_scale = s.red + kMaxItems * kWarps * 2;
    s.cta_key = reinterpret_cast<unsigned long long *>(s.item_scale + kMaxItems);
    s.stages = dp.stages;
    s.xready = nullptr;  // no x gate: the producer streams ahead across operations
    int *flag = reinterpret_cast<int *>(s.cta_key + kMaxItems);
    // the current operation's parameters, double-buffered: operation k is
    // copied into slot k & 1 while other warps may still read operation k - 1
    DecodeOp *slots = reinterpret_cast<DecodeOp *>(smem + dp.off_ops);

    if (threadIdx.x == 0) gemv_init_barriers(s);
    __syncthreads();
    uint32_t i = 0;  // ring stages, counted by the producer and by every consumer warp

    if ((threadIdx.x >> 5) == kWarps) {
        // producer: the weight stream of every GEMV of the step, in order
        bool waited = true;
        for (uint32_t k = 0; k < dp.nops; ++k) {
            if (dp.ops[k].kind != OP_GEMV) continue;
            const GemvParams g = dp.ops[k].g;
            const bool ok = dp.ops[k].fmt == 4 ? gemv_produce<4>(g, s, i, waited) : gemv_produce<8>(g, s, i, waited);
            if (!ok) break;
        }
        return;
    }

    const unsigned long long base = __ldcg(&dp.bar->epoch) * (unsigned long long)(dp.nops - 1) * gridDim.x;
    bool dead = false;
    for (uint32_t k = 0; k < dp.nops; ++k) {
        // copy the operation before the barrier so the loads overlap the wait
        DecodeOp *op = slots + (k & 1);
        {
            const uint32_t *src = reinterpret_cast<const uint32_t *>(dp.ops + k);
            uint32_t *dst = reinterpret_cast<uint32_t *>(op);
            for (uint32_t w = threadIdx.x; w < sizeof(DecodeOp) / 4; w += kConsumers) dst[w] = __ldg(src + w);
        }
        if (k > 0 && !grid_sync(dp.bar, base + (unsigned long long)k * gridDim.x, dp.err, flag, !dead)) dead = true;
        else if (k == 0) consumer_sync();
        const int kind = op->kind;
        switch (kind) {
        case OP_BEGIN:
            if (!dead) op_begin(dp);
            break;
        case OP_GEMV:
            if (op->fmt == 4) gemv_consume<4, NI>(op->g, s, i, dead);
            else gemv_consume<8, NI>(op->g, s, i, dead);
            break;
        case OP_ATTN:
            if (dead) break;
            // the plan admits at most four query heads per KV head here
            if (dp.lp == 8) attn_items<8, 4>(op->a, dp, s.xdig);
            else if (dp.lp == 16) attn_items<16, 4>(op->a, dp, s.xdig);
            else attn_items<32, 4>(op->a, dp, s.xdig);
            break;
        default:
            if (!dead) op_end(dp);
            break;
        }
    }
}

}  // namespace b2

using namespace b2;

struct b2_decode_plan {
    DecodeParams dp;
    DecodeOp *ops;
    void *scratch;
    int32_t *counters;
    GridBar *bar;
    int ni, grid;
    size_t smem;
    uint32_t counters_len;
};

static void plan_free(b2_decode_plan *p)
{
    if (p == nullptr) return;
    if (p->ops) cudaFree(p->ops);
    if (p->scratch) cudaFree(p->scratch);
    if (p->counters) cudaFree(p->counters);
    if (p->bar) cudaFree(p->bar);
    delete p;
}

template <int NI>
static cudaError_t decode_launch(const b2_decode_plan *p, cudaStream_t st)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p->grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = p->smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_kernel<NI>, p->dp);
}

template <int NI>
static cudaError_t decode_prepare(const b2_decode_plan *p)
{
    cudaError_t e = cudaFuncSetAttribute(decode_kernel<NI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p->smem);
    if (e != cudaSuccess) return e;
    int blocks = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, decode_kernel<NI>, kThreads, p->smem);
    if (e != cudaSuccess) return e;
    return blocks >= 1 ? cudaSuccess : cudaErrorCooperativeLaunchTooLarge;
}

extern "C" int b2_decode_plan_create(const b2_decode_args *a, b2_decode_plan **out)
{
    if (out == nullptr) return -1;
    *out = nullptr;
    if (a == nullptr || a->layers == nullptr || a->n_layers == 0 || a->batch == 0 || a->batch > (uint32_t)kMaxItems)
        return -1;
    if (a->embed == nullptr || a->tokens_in == nullptr || a->tokens_out == nullptr || a->positions == nullptr ||
        a->argmax == nullptr || a->x == nullptr || a->vocab == 0 || a->d_model == 0 || a->d_model % 4 ||
        ((uintptr_t)a->x & 15) || ((uintptr_t)a->embed & 15))
        return -1;
    const int grid = sm_count();
    const uint32_t B = a->batch;

    // operations in step order, each checked as its standalone entry point checks it
    std::vector<b2_gemv_args> gargs;
    std::vector<int> kinds;
    std::vector<const b2_attn_args *> aargs;
    kinds.push_back(OP_BEGIN);
    aargs.push_back(nullptr);
    gargs.push_back(b2_gemv_args{});
    for (uint32_t l = 0; l < a->n_layers; ++l) {
        const b2_decode_layer &L = a->layers[l];
        const b2_gemv_args *gs[4] = {&L.qkv, &L.wo, &L.gu, &L.down};
        for (int j = 0; j < 4; ++j) {
            kinds.push_back(OP_GEMV);
            aargs.push_back(nullptr);
            gargs.push_back(*gs[j]);
            if (j == 0) {
                kinds.push_back(OP_ATTN);
                aargs.push_back(&L.attn);
                gargs.push_back(b2_gemv_args{});
            }
        }
    }
    kinds.push_back(OP_GEMV);
    aargs.push_back(nullptr);
    gargs.push_back(a->out);
    kinds.push_back(OP_END);
    aargs.push_back(nullptr);
    gargs.push_back(b2_gemv_args{});
    const uint32_t nops = (uint32_t)kinds.size();

    // shared-memory carve-up: one ring for the whole step; the digit planes
    // and the attention state share one region
    size_t shared_need = 16, scratch = 256;
    uint32_t counters = 1, dpl = 0;
    std::vector<GemvPlan> plans(nops);
    for (uint32_t k = 0; k < nops; ++k) {
        if (kinds[k] == OP_GEMV) {
            b2_gemv_args &g = gargs[k];
            if (g.batch != B) return -1;
            g.grid = grid;
            g.pdl = 0;
            const int rc = gemv_check(&g);
            if (rc != 0) return rc;
            if (!plan_gemv(&g, plans[k])) return -9;
            const uint32_t KW = g.w.format == 4 ? 64u : 32u;
            const size_t xdig = (size_t)g.w.kunits * B * 3 * KW;
            if (xdig > shared_need) shared_need = xdig;
            if (plans[k].partial_bytes > scratch) scratch = plans[k].partial_bytes;
            if (plans[k].counter_len > counters) counters = plans[k].counter_len;
        } else if (kinds[k] == OP_ATTN) {
            const b2_attn_args *t = aargs[k];
            const int rc = attn_check(t);
            if (rc != 0) return rc;
            if (t->batch != B) return -1;
            const uint32_t d = (uint32_t)attn_lanes(t->head_dim);
            if (dpl != 0 && d != dpl) return -1;
            dpl = d;
            const uint32_t G = t->n_heads / t->n_kv_heads;
            if (G > 4) return -9;  // register budget of the persistent kernel
            const size_t need = attn_smem_bytes((int)d, kWarps, G);
            if (need > shared_need) shared_need = need;
            if (t->batch * t->n_kv_heads > counters) counters = t->batch * t->n_kv_heads;
        }
    }
    if (dpl == 0) return -1;
    // attention work items: chunks per (item, KV head) so that one wave of
    // CTAs covers the step at long context
    uint32_t heads = 0, G = 0, hd = 0;
    for (uint32_t k = 0; k < nops; ++k)
        if (kinds[k] == OP_ATTN) {
            heads = aargs[k]->batch * aargs[k]->n_kv_heads;
            G = aargs[k]->n_heads / aargs[k]->n_kv_heads;
            hd = aargs[k]->head_dim;
        }
    uint32_t attn_chunks = (uint32_t)grid / heads;
    if (attn_chunks < 1) attn_chunks = 1;
    const size_t attn_partial = ((size_t)heads * attn_chunks * G * (hd + 2) * sizeof(float) + 255) & ~(size_t)255;
    if (attn_partial > scratch) scratch = attn_partial;

    const uint32_t tbuf = kWarps * 16 * B * 4;
    // per-warp tile sums: rounds of up to 16 tiles in every GEMV of the step
    const uint32_t per_tile = kWarps * 16 * B * 4, round_cap = 16;
    const uint32_t parts = round_cap * per_tile;
    const uint32_t misc = (kMaxItems * kWarps * 2 + kMaxItems) * 4 + kMaxItems * 8 + 16;
    const uint32_t opslots = (uint32_t)((2 * sizeof(DecodeOp) + 15) & ~(size_t)15);
    const uint32_t limit = 227u * 1024u;
    uint32_t off = 2 * kMaxStages * 8;
    off = (off + 127) & ~127u;
    const uint32_t off_ring = off;
    const uint32_t stage_b = kStageUnits * B2_Q4_UNIT_BYTES;
    const uint32_t fixed = off_ring + (uint32_t)((shared_need + 127) & ~(size_t)127) + tbuf + parts + 32 + misc + opslots;
    if (fixed + 2 * stage_b > limit) return -9;
    uint32_t ns = (limit - fixed) / stage_b;
    if (ns > (uint32_t)kMaxStages) ns = kMaxStages;
    off += ns * stage_b;
    const uint32_t off_shared = off;
    off += (uint32_t)((shared_need + 127) & ~(size_t)127);
    const uint32_t off_tile = off;
    off += tbuf;
    const uint32_t off_parts = off;
    off += parts;
    off = (off + 15) & ~15u;
    const uint32_t off_misc = off;
    off += misc;
    off = (off + 15) & ~15u;
    const uint32_t off_ops = off;
    off += opslots;

    b2_decode_plan *p = new (std::nothrow) b2_decode_plan();
    if (p == nullptr) return -2;
    p->grid = grid;
    p->smem = off;
    p->ni = (int)((B + 1) / 2);
    p->counters_len = counters;
    if (cudaMalloc((void **)&p->ops, nops * sizeof(DecodeOp)) != cudaSuccess ||
        cudaMalloc(&p->scratch, scratch) != cudaSuccess ||
        cudaMalloc((void **)&p->counters, counters * sizeof(int32_t)) != cudaSuccess ||
        cudaMalloc((void **)&p->bar, sizeof(GridBar)) != cudaSuccess ||
        cudaMemset(p->counters, 0, counters * sizeof(int32_t)) != cudaSuccess ||
        cudaMemset(p->bar, 0, sizeof(GridBar)) != cudaSuccess) {
        plan_free(p);
        return -2;
    }
    std::vector<DecodeOp> ops(nops);
    for (uint32_t k = 0; k < nops; ++k) {
        DecodeOp &o = ops[k];
        std::memset(&o, 0, sizeof(o));
        o.kind = kinds[k];
        if (kinds[k] == OP_GEMV) {
            b2_gemv_args g = gargs[k];
            g.scratch = p->scratch;
            g.scratch_bytes = scratch;
            g.counters = p->counters;
            g.counters_len = counters;
            gemv_params(&g, plans[k], o.g);
            o.fmt = (int)g.w.format;
            o.g.off_ring = off_ring;
            o.g.off_xdig = off_shared;
            o.g.off_tile = off_tile;
            o.g.off_parts = off_parts;
            if (o.g.round_tiles > round_cap) o.g.round_tiles = round_cap;
            o.g.off_misc = off_misc;
            o.g.stages = ns;
        } else if (kinds[k] == OP_ATTN) {
            b2_attn_args t = *aargs[k];
            t.scratch = p->scratch;
            t.scratch_bytes = scratch;
            t.counters = p->counters;
            t.counters_len = counters;
            attn_params(&t, attn_chunks, o.a);
        }
    }
    if (cudaMemcpy(p->ops, ops.data(), nops * sizeof(DecodeOp), cudaMemcpyHostToDevice) != cudaSuccess) {
        plan_free(p);
        return -8;
    }
    DecodeParams &dp = p->dp;
    dp.ops = p->ops;
    dp.nops = nops;
    dp.batch = B;
    dp.d_model = a->d_model;
    dp.vocab = a->vocab;
    dp.lp = dpl;
    dp.attn_chunks = attn_chunks;
    dp.embed = a->embed;
    dp.tokens_in = a->tokens_in;
    dp.tokens_out = a->tokens_out;
    dp.positions = a->positions;
    dp.argmax = a->argmax;
    dp.x = a->x;
    dp.bar = p->bar;
    dp.err = a->err;
    dp.off_ring = off_ring;
    dp.off_shared = off_shared;
    dp.off_tile = off_tile;
    dp.off_parts = off_parts;
    dp.off_misc = off_misc;
    dp.off_ops = off_ops;
    dp.stages = ns;
    cudaError_t e;
    switch (p->ni) {
    case 1: e = decode_prepare<1>(p); break;
    case 2: e = decode_prepare<2>(p); break;
    case 3:
    case 4: e = decode_prepare<4>(p); break;
    default: e = decode_prepare<8>(p); break;
    }
    // the zero fills and the op table went through the legacy stream; steps run
    // on the caller's (possibly non-blocking) stream, which does not wait for it
    if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamLegacy);
    if (e != cudaSuccess) {
        plan_free(p);
        return -8;
    }
    *out = p;
    return 0;
}

extern "C" int b2_decode_step(b2_decode_plan *p, void *stream)
{
    if (p == nullptr) return -1;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    switch (p->ni) {
    case 1: e = decode_launch<1>(p, st); break;
    case 2: e = decode_launch<2>(p, st); break;
    case 3:
    case 4: e = decode_launch<4>(p, st); break;
    default: e = decode_launch<8>(p, st); break;
    }
    return e == cudaSuccess ? 0 : -8;
}

extern "C" int b2_decode_reset(b2_decode_plan *p, void *stream)
{
    if (p == nullptr) return -1;
    cudaStream_t st = (cudaStream_t)stream;
    if (cudaMemsetAsync(p->bar, 0, sizeof(GridBar), st) != cudaSuccess) return -8;
    if (cudaMemsetAsync(p->counters, 0, (size_t)p->counters_len * sizeof(int32_t), st) != cudaSuccess) return -8;
    return 0;
}

extern "C" void b2_decode_plan_destroy(b2_decode_plan *p)
{
    plan_free(p);
}
