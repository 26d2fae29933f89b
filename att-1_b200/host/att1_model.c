/*
 * att1_model.c - .att1 model loader (memory-mapped, read-only).
 *
 * Implements the file format described in att1_model.h with the validation
 * rules of ATT-1's loader (src/model_loader.c:53-152 tensor sizes,
 * :237-432 header/section checks): magic and version, section ranges inside
 * the file, tensor payloads inside the data section, and nbytes equal to the
 * size the dtype and shape imply (q4: rows*cols/2 + rows*(cols/group)*4 with
 * group from flags[7:0], 0 = 32, a power of two in [16, 128]).
 */
#define _DEFAULT_SOURCE
#include "att1_model.h"
#include "att1_quant.h"

#include <fcntl.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

static uint32_t rd32(const unsigned char *p)
{
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

static uint64_t rd64(const unsigned char *p)
{
    return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32);
}

static int in_range(uint64_t size, uint64_t off, uint64_t len)
{
    return off <= size && len <= size - off;
}

static int mul_ok(uint64_t a, uint64_t b, uint64_t *out)
{
    if (a != 0 && b > UINT64_MAX / a) return 0;
    *out = a * b;
    return 1;
}

/* Expected payload size of a tensor; 0 on an invalid descriptor. */
static int tensor_nbytes(const att1_model_tensor *t, uint64_t *out)
{
    uint64_t elems = 1;
    uint32_t i;

    if (t->ndims == 0 || t->ndims > ATT1_MODEL_MAX_DIMS) return 0;
    for (i = 0; i < t->ndims; i++) {
        if (t->shape[i] == 0 || !mul_ok(elems, t->shape[i], &elems)) return 0;
    }
    switch (t->dtype) {
    case ATT1_MODEL_DTYPE_F32:
        return mul_ok(elems, 4, out);
    case ATT1_MODEL_DTYPE_Q8: {
        uint64_t v, s;
        if (t->ndims != 2 || !mul_ok(t->shape[0], t->shape[1], &v) || !mul_ok(t->shape[0], 4, &s) ||
            s > UINT64_MAX - v)
            return 0;
        *out = v + s;
        return 1;
    }
    case ATT1_MODEL_DTYPE_Q4: {
        uint32_t g;
        uint64_t packed, scales;
        if (t->ndims != 2 || (t->flags & ~ATT1_Q4_FLAGS_GROUP_MASK) != 0) return 0;
        g = t->flags & ATT1_Q4_FLAGS_GROUP_MASK;
        if (g == 0) g = ATT1_Q4_GROUP_SIZE_DEFAULT;
        if (g < ATT1_Q4_GROUP_SIZE_MIN || g > ATT1_Q4_GROUP_SIZE_MAX || (g & (g - 1)) != 0) return 0;
        if (t->shape[1] % 2 != 0 || t->shape[1] % g != 0) return 0;
        if (!mul_ok(t->shape[0], t->shape[1] / 2, &packed) ||
            !mul_ok(t->shape[0], (t->shape[1] / g) * 4, &scales) || scales > UINT64_MAX - packed)
            return 0;
        *out = packed + scales;
        return 1;
    }
    default:
        return 0;
    }
}

att1_status_t att1_model_load(const char *path, att1_model *model)
{
    int fd;
    struct stat st;
    unsigned char *d;
    uint64_t size, cfg_off, cfg_size, desc_off, count, data_off, data_size, shard_off, shard_size;
    uint64_t tok_off = 0, tok_size = 0, desc_bytes, i;
    uint32_t version, header_size;
    att1_status_t rc = ATT1_ERR_BAD_FORMAT;

    if (path == NULL || model == NULL) return ATT1_ERR_INVALID_ARG;
    memset(model, 0, sizeof(*model));
    fd = open(path, O_RDONLY);
    if (fd < 0) return ATT1_ERR_IO;
    if (fstat(fd, &st) != 0 || st.st_size < (off_t)ATT1_MODEL_HEADER_SIZE) {
        close(fd);
        return st.st_size < (off_t)ATT1_MODEL_HEADER_SIZE ? ATT1_ERR_BAD_FORMAT : ATT1_ERR_IO;
    }
    size = (uint64_t)st.st_size;
    d = mmap(NULL, (size_t)size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (d == MAP_FAILED) return ATT1_ERR_IO;

    if (memcmp(d, ATT1_MODEL_MAGIC, ATT1_MODEL_MAGIC_SIZE) != 0) goto fail;
    version = rd32(d + 8);
    header_size = rd32(d + 12);
    if (version == ATT1_MODEL_VERSION) {
        if (header_size != ATT1_MODEL_HEADER_SIZE) { rc = ATT1_ERR_UNSUPPORTED; goto fail; }
    } else if (version == ATT1_MODEL_VERSION_2) {
        if (header_size != ATT1_MODEL_HEADER_SIZE_V2) { rc = ATT1_ERR_UNSUPPORTED; goto fail; }
        if (size < ATT1_MODEL_HEADER_SIZE_V2) goto fail;
        tok_off = rd64(d + 80);
        tok_size = rd64(d + 88);
    } else {
        rc = ATT1_ERR_UNSUPPORTED;
        goto fail;
    }
    cfg_off = rd64(d + 16);
    cfg_size = rd64(d + 24);
    desc_off = rd64(d + 32);
    count = rd64(d + 40);
    data_off = rd64(d + 48);
    data_size = rd64(d + 56);
    shard_off = rd64(d + 64);
    shard_size = rd64(d + 72);
    if (cfg_size != ATT1_MODEL_CONFIG_SIZE || !in_range(size, cfg_off, cfg_size) ||
        !in_range(size, data_off, data_size))
        goto fail;
    if (((shard_off == 0) != (shard_size == 0)) || (shard_size && !in_range(size, shard_off, shard_size)))
        goto fail;
    if (((tok_off == 0) != (tok_size == 0)) || (tok_size && !in_range(size, tok_off, tok_size))) goto fail;
    if (!mul_ok(count, ATT1_MODEL_TENSOR_DESC_SIZE, &desc_bytes) || !in_range(size, desc_off, desc_bytes))
        goto fail;

    model->tensors = calloc(count ? (size_t)count : 1, sizeof(att1_model_tensor));
    if (model->tensors == NULL) { rc = ATT1_ERR_OOM; goto fail; }
    {
        const unsigned char *c = d + cfg_off;
        model->config.vocab_size = rd32(c);
        model->config.n_layers = rd32(c + 4);
        model->config.n_heads = rd32(c + 8);
        model->config.d_model = rd32(c + 12);
        model->config.d_ff = rd32(c + 16);
        model->config.max_seq_len = rd32(c + 20);
        model->config.rope_dim = rd32(c + 24);
        model->config.n_tiles = rd32(c + 28);
        model->config.shard_count = rd32(c + 32);
    }
    model->tensor_count = count;
    model->file_data = d;
    model->file_size = (size_t)size;
    for (i = 0; i < count; i++) {
        const unsigned char *p = d + desc_off + i * ATT1_MODEL_TENSOR_DESC_SIZE;
        att1_model_tensor *t = &model->tensors[i];
        uint64_t want = 0;
        uint32_t k;
        memcpy(t->name, p, ATT1_MODEL_NAME_SIZE);
        t->name[ATT1_MODEL_NAME_SIZE - 1] = '\0';
        t->dtype = rd32(p + 64);
        t->ndims = rd32(p + 68);
        for (k = 0; k < ATT1_MODEL_MAX_DIMS; k++) t->shape[k] = rd64(p + 72 + 8 * k);
        t->offset = rd64(p + 104);
        t->nbytes = rd64(p + 112);
        t->shard_id = rd32(p + 120);
        t->flags = rd32(p + 124);
        if (!tensor_nbytes(t, &want) || t->nbytes != want) {
            att1_model_free(model);
            return ATT1_ERR_SHAPE;
        }
        if (!in_range(data_size, t->offset, t->nbytes)) {
            att1_model_free(model);
            return ATT1_ERR_BAD_FORMAT;
        }
        t->data = d + data_off + t->offset;
    }
    return ATT1_OK;
fail:
    free(model->tensors);
    munmap(d, (size_t)size);
    memset(model, 0, sizeof(*model));
    return rc;
}

void att1_model_free(att1_model *model)
{
    if (model == NULL) return;
    free(model->tensors);
    if (model->file_data != NULL) munmap(model->file_data, model->file_size);
    memset(model, 0, sizeof(*model));
}

const att1_model_tensor *att1_model_find_tensor(const att1_model *model, const char *name)
{
    uint64_t i;
    if (model == NULL || name == NULL) return NULL;
    for (i = 0; i < model->tensor_count; i++) {
        if (strncmp(model->tensors[i].name, name, ATT1_MODEL_NAME_SIZE) == 0) return &model->tensors[i];
    }
    return NULL;
}
