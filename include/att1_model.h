/*
 * att1_model.h - ATT-1 model artifacts (.att1 files).
 *
 * Same API and field meaning as ATT-1's include/att1_model.h:12-84 for the
 * parts the decode path reads (config, tensor table, tensor data). The file is
 * memory-mapped read-only instead of read into a heap copy, so a large model
 * is paged in tensor by tensor while it is uploaded to the device.
 * Format (little-endian; src/model_loader.c:204-432 of the reference):
 *   header 80 B (v1) or 96 B (v2): magic "ATT1MODL", u32 version, u32 header
 *   size, u64 {config offset, config size=36, descriptor offset, tensor
 *   count, data offset, data size, shard-meta offset, shard-meta size}
 *   [v2: u64 tokenizer-meta offset, size];
 *   config: 9 x u32 (the att1_model_config fields in order);
 *   descriptors: 128 B each, name[64], u32 dtype, u32 ndims, u64 shape[4],
 *   u64 offset (from the data section), u64 nbytes, u32 shard_id, u32 flags.
 */
#ifndef ATT1_MODEL_H
#define ATT1_MODEL_H

#include "att1_status.h"

#include <stddef.h>
#include <stdint.h>

#define ATT1_MODEL_MAGIC "ATT1MODL"
#define ATT1_MODEL_MAGIC_SIZE 8u
#define ATT1_MODEL_VERSION 1u
#define ATT1_MODEL_VERSION_2 2u
#define ATT1_MODEL_NAME_SIZE 64u
#define ATT1_MODEL_MAX_DIMS 4u
#define ATT1_MODEL_HEADER_SIZE 80u
#define ATT1_MODEL_HEADER_SIZE_V2 96u
#define ATT1_MODEL_CONFIG_SIZE 36u
#define ATT1_MODEL_TENSOR_DESC_SIZE 128u

typedef enum att1_model_dtype {
    ATT1_MODEL_DTYPE_F32 = 1,
    ATT1_MODEL_DTYPE_Q8 = 2,
    ATT1_MODEL_DTYPE_Q4 = 3
} att1_model_dtype;

typedef struct att1_model_config {
    uint32_t vocab_size;
    uint32_t n_layers;
    uint32_t n_heads;
    uint32_t d_model;
    uint32_t d_ff;
    uint32_t max_seq_len;
    uint32_t rope_dim;
    uint32_t n_tiles;
    uint32_t shard_count;
} att1_model_config;

typedef struct att1_model_tensor {
    char name[ATT1_MODEL_NAME_SIZE];
    uint32_t dtype;
    uint32_t ndims;
    uint64_t shape[ATT1_MODEL_MAX_DIMS];
    uint64_t offset;
    uint64_t nbytes;
    uint32_t shard_id;
    uint32_t flags;
    const void *data;   /* into the mapping; valid while the model lives */
} att1_model_tensor;

typedef struct att1_model {
    att1_model_config config;
    uint64_t tensor_count;
    att1_model_tensor *tensors;
    unsigned char *file_data;   /* read-only mapping of the whole file */
    size_t file_size;
} att1_model;

att1_status_t att1_model_load(const char *path, att1_model *model);
void att1_model_free(att1_model *model);
const att1_model_tensor *att1_model_find_tensor(const att1_model *model,
                                                const char *name);

#endif
