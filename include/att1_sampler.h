/*
 * att1_sampler.h - sampler configuration and the greedy host sampler
 * (ATT-1 include/att1_sampler.h:7-21).
 *
 * Same struct and function as the reference. att1_sampler_greedy_f32 works on
 * a host logits buffer (for example the one att1_infer_logits returns); the
 * decode step itself samples on the device (fused argmax keys and the step
 * end kernel). att1_sampler_config drives the device top-k / temperature
 * sampler of att1_b200_infer_set_sampler (att1_b200.h); the reference declares
 * the struct but samples greedily only.
 */
#ifndef ATT1_SAMPLER_H
#define ATT1_SAMPLER_H

#include <stddef.h>
#include <stdint.h>

typedef struct att1_sampler_config {
    uint32_t top_k;
    float temperature;
} att1_sampler_config;

/* Index of the largest of logits[0..count): ties go to the lowest index, any
 * NaN is rejected. Returns 0, or -1 for NULL pointers, count 0 or a NaN
 * (src/sampler.c:5-34). */
int att1_sampler_greedy_f32(const float *logits, size_t count, uint32_t *out_token);

#endif
