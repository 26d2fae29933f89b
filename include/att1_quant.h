/*
 * att1_quant.h - q4/q8 weight containers of the ATT-1 API.
 *
 * The structs keep the field names and meaning of ATT-1's
 * include/att1_quant.h:103-133 because the backend vtable passes them by
 * pointer. Wire format (include/att1_quant.h:19-38 in the reference):
 *   q4 [rows][cols]: packed[rows*cols/2] (low nibble = even element, signed
 *   4-bit values in [-7, 7]) followed by scales[rows*cols/group] f32, one per
 *   (row, group), row-major. Group size in the tensor flags[7:0], 0 = 32.
 *   q8 [rows][cols]: values[rows*cols] int8 then scales[rows] f32.
 * This library keeps such matrices on the GPU in a permuted unit layout
 * (see b2_kernels.h); the bytes themselves are not changed.
 */
#ifndef ATT1_QUANT_H
#define ATT1_QUANT_H

#include <stddef.h>
#include <stdint.h>

#define ATT1_Q4_GROUP_SIZE_DEFAULT 32u
#define ATT1_Q4_GROUP_SIZE_MIN     16u
#define ATT1_Q4_GROUP_SIZE_MAX     128u
#define ATT1_Q4_FLAGS_GROUP_MASK   0xFFu

typedef struct att1_q8_matrix {
    size_t rows;
    size_t cols;
    int8_t *values;   /* [rows*cols] */
    float *scales;    /* [rows] */
} att1_q8_matrix;

typedef struct att1_q4_matrix {
    size_t rows;
    size_t cols;
    uint32_t group_size;
    uint8_t *packed;  /* [rows*cols/2] */
    float *scales;    /* [rows*(cols/group_size)] */
} att1_q4_matrix;

#endif
