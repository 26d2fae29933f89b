/*
 * att1_b200.h - additions to the ATT-1 API for the B200 decode path.
 *
 * Nothing here changes an existing ATT-1 signature. The additions cover what
 * the .att1 format and the batch-1 API cannot express:
 *   - model shape beyond the .att1 config: grouped-query attention
 *     (n_kv_heads), RMSNorm eps and RoPE theta (hard-coded to 1e-6 / 10000 in
 *     the reference, src/infer.c:721-722);
 *   - seeded synthetic models generated and quantised on the device (the
 *     benchmark models are tens of GB; the generator is bit-identical to the
 *     CPU one the parity tests use);
 *   - batched decode: B independent sequences in one device step;
 *   - device-side step loops and timing hooks for benchmarks, and read-back
 *     of device weights / KV pages for parity tests.
 */
#ifndef ATT1_B200_H
#define ATT1_B200_H

#include "att1_infer.h"
#include "att1_kv_mmu.h"
#include "att1_sampler.h"
#include "att1_status.h"
#include "b2_kernels.h"

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct att1_b200_config {
    uint32_t vocab, n_layers, n_heads, n_kv_heads, d_model, d_ff, max_seq;
    uint32_t group;      /* q4 group size: 32 */
    uint32_t dtype;      /* 4 = q4, 8 = q8 */
    float eps;           /* block RMSNorm eps */
    float final_eps;     /* output RMSNorm eps */
    float theta;         /* RoPE base */
} att1_b200_config;

/* Weight kinds for export (same numbering as the synthetic tensor ids). */
enum {
    ATT1_B200_WQ = 1, ATT1_B200_WK = 2, ATT1_B200_WV = 3, ATT1_B200_WO = 4,
    ATT1_B200_GATE = 6, ATT1_B200_UP = 7, ATT1_B200_DOWN = 8, ATT1_B200_OUTPUT = 9
};

/* Sequences one context decodes together. Up to 16 whose activation digit
 * planes fit the GEMVs' shared memory go through the fused GEMVs; larger
 * batches (and shapes the GEMVs cannot tile) through the tensor-core GEMM. */
#define ATT1_B200_MAX_BATCH 64

/* Synthetic model on the current device: every matrix N(0, 0.02) from
 * (seed, tensor id) quantised by the reference rule, norm gains 1.0,
 * embedding N(0, 0.02) in f32. `batch` sequences decode together. */
att1_status_t att1_b200_infer_create_synth(const att1_b200_config *cfg, uint64_t seed,
                                           uint32_t batch, att1_infer_t **out_infer);
/* Same, from a loaded .att1 model with explicit eps/theta (n_kv_heads must
 * equal n_heads: the format stores full K/V projections). */
att1_status_t att1_b200_infer_create_model(const att1_model *model, uint32_t dtype, float eps,
                                           float final_eps, float theta,
                                           att1_infer_t **out_infer);
/* Rank `rank` of `world` tensor-parallel shards of a loaded .att1 model (the
 * split of att1_b200_infer_create_synth_tp; q4 and q8 tensors are sliced
 * byte for byte, f32 tensors quantised per whole output row first). Connect
 * the ranks before the first step. */
att1_status_t att1_b200_infer_create_model_tp(const att1_model *model, uint32_t dtype, float eps,
                                              float final_eps, float theta, uint32_t rank,
                                              uint32_t world, att1_infer_t **out_infer);
uint32_t att1_b200_infer_batch(const att1_infer_t *infer);

/* One step for all sequences: tokens[batch] in, greedy next tokens out. */
/* ---- tensor parallelism over GPUs ----------------------------------------------
 * One context per GPU and rank, holding that rank's shard (query / KV heads,
 * FFN rows, vocabulary rows; WO and down by input columns); the ranks
 * exchange partial results through each other's device memory inside the
 * step's kernels. Create every rank, then connect them: across processes
 * with CUDA IPC handles (exchanged by the caller, e.g. over
 * torch.distributed), or inside one process with peer access. Every rank
 * must then run the same steps with the same tokens; logits (all vocabulary
 * rows) and tokens are the same on every rank. */
#define ATT1_B200_TP_HANDLE_BYTES 64
/* Device for the contexts created next by this thread (the library's own CUDA
 * runtime state; a context keeps its device for all later calls). */
att1_status_t att1_b200_set_device(int device);
att1_status_t att1_b200_infer_create_synth_tp(const att1_b200_config *cfg, uint64_t seed, uint32_t batch,
                                              uint32_t rank, uint32_t world, att1_infer_t **out_infer);
/* This rank's exchange-region handle (ATT1_B200_TP_HANDLE_BYTES bytes). */
att1_status_t att1_b200_infer_tp_handle(const att1_infer_t *infer, void *handle);
/* handles: world * ATT1_B200_TP_HANDLE_BYTES bytes, rank order (own entry ignored). */
att1_status_t att1_b200_infer_tp_connect(att1_infer_t *infer, const void *handles);
/* Unmaps the other ranks' regions (IPC): every rank disconnects, the caller
 * synchronises the ranks, then each destroys its context. */
att1_status_t att1_b200_infer_tp_disconnect(att1_infer_t *infer);
/* All ranks of one process (rank r on its own device), connected by peer access. */
att1_status_t att1_b200_infer_tp_connect_local(att1_infer_t *const *infers, uint32_t world);
/* The same tensor-parallel step with the exchange done by NCCL collectives on
 * the step's stream instead of the kernels' peer-memory stores, for
 * comparison: WO and down write partial sums (rank 0's carries the residual)
 * that ncclAllReduce adds, and the lm_head's logits and argmax keys are
 * gathered with ncclAllGather; logits and tokens are the same on every rank.
 * NCCL (libnccl.so.2) is loaded at run time; ATT1_ERR_UNSUPPORTED without it
 * and for batches that take the tensor-core route. One rank per process: rank
 * 0 makes the id (ATT1_B200_NCCL_ID_BYTES bytes), every rank connects with it
 * (a collective: all ranks call it together). Replaces tp_connect. */
#define ATT1_B200_NCCL_ID_BYTES 128
att1_status_t att1_b200_nccl_unique_id(void *id);
att1_status_t att1_b200_infer_tp_connect_nccl(att1_infer_t *infer, const void *id);
/* Bound of every wait for another rank inside the step's kernels, in polls of
 * the flag (about 0.1 us each; 0 = 2^24). A wait that runs out ends the step
 * with ATT1_ERR_TIMEOUT and the context stays usable. */
att1_status_t att1_b200_infer_tp_set_wait(att1_infer_t *infer, uint32_t polls);
/* After a step failed on any rank (e.g. ATT1_ERR_TIMEOUT because another rank
 * did not take it): with no rank stepping, call on every rank, synchronise the
 * ranks on the host, then step together again. Clears this rank's exchange
 * flags and step epoch; positions are the host's (the failed step did not
 * advance them). */
att1_status_t att1_b200_infer_tp_reset(att1_infer_t *infer);
/* A step in two halves, so one thread can drive several ranks: queue the
 * step on every rank, then wait for each. */
att1_status_t att1_b200_infer_step_async(att1_infer_t *infer, const uint32_t *tokens);
att1_status_t att1_b200_infer_step_wait(att1_infer_t *infer, uint32_t *out_tokens);

/* Prompt prefill (batch-1 contexts, one GPU): the same result as feeding
 * tokens[0..n) through att1_infer_decode_token one by one (KV cache, position,
 * logits of the last token, greedy next token in *out_token), computed with
 * the tensor-core GEMM over up to 512 prompt tokens at a time. On a context
 * using a KV-MMU (att1_b200_infer_use_kv_mmu) the prompt's K/V go into the
 * session's pages, mapped for the whole prompt before the first kernel. */
att1_status_t att1_b200_infer_prefill(att1_infer_t *infer, const uint32_t *tokens, size_t n, uint32_t *out_token);

att1_status_t att1_b200_infer_decode_batch(att1_infer_t *infer, const uint32_t *tokens,
                                           uint32_t *out_tokens);
/* Host copy of the last step's logits [batch][vocab]. */
const float *att1_b200_infer_logits_batch(const att1_infer_t *infer, size_t *out_count);

/* use_graph: replay one captured CUDA graph per step (default 1);
 * use_pdl: programmatic dependent launch between kernels (default 1). */
att1_status_t att1_b200_infer_set_options(att1_infer_t *infer, int use_graph, int use_pdl);
/* Run each step as one persistent launch (on) or as the per-operation kernel
 * sequence (off, the default). ATT1_ERR_UNSUPPORTED when the model's shape
 * does not fit the persistent kernel (the sequence is used). */
att1_status_t att1_b200_infer_set_persistent(att1_infer_t *infer, int on);

/* Enqueue `steps` decode steps on the device, each feeding its greedy token
 * into the next, without host synchronisation (benchmark loop). The host
 * position advances by `steps`; call att1_b200_infer_sync to wait. */
att1_status_t att1_b200_infer_run_steps(att1_infer_t *infer, uint32_t steps);
att1_status_t att1_b200_infer_sync(att1_infer_t *infer);
/* CUDA stream (cudaStream_t) all work of this context is enqueued on. */
void *att1_b200_infer_stream(const att1_infer_t *infer);

/* Read back device weights in the reference layout. */
att1_status_t att1_b200_infer_export_q4(const att1_infer_t *infer, uint32_t layer, uint32_t kind,
                                        uint8_t *packed, float *scales);
att1_status_t att1_b200_infer_export_q8(const att1_infer_t *infer, uint32_t layer, uint32_t kind,
                                        int8_t *values, float *scales);
/* Read back KV of one sequence and layer, positions [0, count), as
 * [count][n_kv_heads][head_dim] f32. */
att1_status_t att1_b200_infer_export_kv(const att1_infer_t *infer, uint32_t item, uint32_t layer,
                                        size_t count, float *keys, float *values);
/* Write KV of one sequence and layer, positions [0, count), from
 * [count][n_kv_heads][head_dim] f32 host arrays (the layout export_kv reads;
 * under tensor parallelism this rank's KV heads): restores a saved cache, or
 * sets up a deep context for a test without decoding its prefix. Returns after
 * the host arrays have been read. Not on a context using a KV-MMU (its
 * sessions are written through att1_kv_mmu.h). */
att1_status_t att1_b200_infer_import_kv(att1_infer_t *infer, uint32_t item, uint32_t layer, size_t count,
                                        const float *keys, const float *values);
/* Continue every sequence at `position` (< max_seq): the next decode step
 * attends positions [0, position] and appends there, so [0, position) must
 * hold KV (decoded or imported). Tensor-parallel ranks seek together. Not on a
 * context using a KV-MMU. */
att1_status_t att1_b200_infer_seek(att1_infer_t *infer, size_t position);
/* Operations (kernel launches and the copies captured with them) in one step
 * of the context's CUDA graph, once a step has run with graphs on; 0 before
 * that or without graphs. No reference counterpart. */
size_t att1_b200_infer_step_launches(const att1_infer_t *infer);
/* Device bytes held by the context (weights, KV pages, buffers). */
size_t att1_b200_infer_device_bytes(const att1_infer_t *infer);

/* One session's layer of a KV-MMU (att1_kv_mmu.h) as the kernels of
 * b2_kernels.h address KV: the device page pools, that session and layer's
 * device page-table row (batch item 0) and the page geometry. Valid until the
 * session is destroyed; positions the session has appended are readable by
 * b2_attn, and the QKV epilogue may append the next one. */
att1_status_t att1_b200_kv_mmu_layout(const att1_kv_mmu *mmu, uint64_t session_id, size_t layer_id,
                                      b2_kv_layout *out);
/* Batch item b of the context keeps its KV in KV-MMU session session_ids[b]:
 * pages are mapped on demand as positions advance, and the MMU's lengths and
 * append counters follow the steps, so the sessions can be read, looked up
 * and destroyed through att1_kv_mmu.h. The sessions must be empty, sit in
 * consecutive slots in batch order (created one after another) and match the
 * context (layers, KV heads, head_dim; max_positions >= max_seq). Only before
 * the first step and on one GPU; export_kv is unsupported while a KV-MMU is
 * in use (read through att1_kv_mmu_copy_range). NULL returns to the context's
 * own page pools. */
att1_status_t att1_b200_infer_use_kv_mmu(att1_infer_t *infer, att1_kv_mmu *mmu, const uint64_t *session_ids);

/* Next-token sampling of every later step (decode, device-loop steps and the
 * token after a prefill). NULL or top_k <= 1: greedy, the reference's sampler
 * and the default. top_k 2..256 with a positive finite temperature: top-k /
 * temperature sampling on the device (b2_sample_topk in b2_kernels.h); the
 * draw for item b depends only on `seed`, b and the position the token takes,
 * so a run repeats exactly. Tensor-parallel ranks draw from the all-gathered
 * logits and agree on every token when all of them set the same sampler.
 * Uses the per-kernel step, not the persistent one. */
att1_status_t att1_b200_infer_set_sampler(att1_infer_t *infer, const att1_sampler_config *config, uint64_t seed);

#ifdef __cplusplus
}
#endif
#endif
