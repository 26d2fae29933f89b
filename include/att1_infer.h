/*
 * att1_infer.h - single-device, batch-1 decode (ATT-1 model API).
 *
 * Same functions, arguments and status codes as ATT-1's include/att1_infer.h
 * (src/infer.c:519-1012). The context here lives on one B200: weights are
 * uploaded once at create time in the device unit layout, the KV cache is a
 * device page pool, and each att1_infer_decode_token is one CUDA-graph launch
 * of the fused decode kernels with only the token id going in and the next
 * token id coming back. Logits are copied to the host only when
 * att1_infer_logits is called.
 *
 * As in the reference, RMSNorm eps is 1e-6 and RoPE theta 10000 for models
 * created from a .att1 file (the format has no fields for them,
 * src/infer.c:721-722); att1_b200.h creates contexts with other values.
 */
#ifndef ATT1_INFER_H
#define ATT1_INFER_H

#include "att1_backend.h"
#include "att1_model.h"
#include "att1_status.h"
#include "att1_trace.h"

#include <stddef.h>
#include <stdint.h>

typedef struct att1_infer att1_infer_t;

/* q8 path: every 2-D weight of an f32 model is quantised per row on the
 * device by the reference's q8 rule (or taken from q8 tensors in the file). */
att1_status_t att1_infer_create(const att1_model *model, att1_infer_t **out_infer);
/* q4 path: q4 weight tensors (group size from the tensor flags). */
att1_status_t att1_infer_create_q4(const att1_model *model, att1_infer_t **out_infer);
void att1_infer_destroy(att1_infer_t *infer);

/* Decode one token id (< vocab) at the current position; *out_token = greedy
 * argmax of the logits (lowest id on ties; NaN logits -> ATT1_ERR_STATE). */
att1_status_t att1_infer_decode_token(att1_infer_t *infer, uint32_t token_id,
                                      uint32_t *out_token);
/* Feed prompt bytes as token ids, then greedy-decode generated_token_count
 * tokens (same contract as src/infer.c:882-928). */
att1_status_t att1_infer_generate(att1_infer_t *infer, const unsigned char *prompt,
                                  size_t prompt_bytes, size_t generated_token_count,
                                  uint32_t *out_tokens, size_t out_token_capacity,
                                  size_t *out_token_count);
/* Borrowed host copy of the last step's logits, valid until the next decode. */
const float *att1_infer_logits(const att1_infer_t *infer, size_t *out_count);
att1_status_t att1_infer_position(const att1_infer_t *infer, size_t *out_position);
att1_status_t att1_infer_layer_kv_length(const att1_infer_t *infer, uint32_t layer_id,
                                         size_t *out_length);
/* Borrows trace (not owned). */
att1_status_t att1_infer_set_trace(att1_infer_t *infer, att1_trace_t *trace);
/* Takes ownership of backend. "cuda-q4"/"cuda-q8" select the device q4/q8
 * path (the q8 weights are prepared on first selection); any other backend
 * is rejected with ATT1_ERR_UNSUPPORTED: there is no CPU path here. */
att1_status_t att1_infer_set_backend(att1_infer_t *infer, att1_backend *backend);

#endif
