/*
 * att1_sampler.c - the reference's greedy sampler over a host logits buffer
 * (src/sampler.c:5-34): reject NaN, then the first maximum wins.
 */
#include "att1_sampler.h"

#include <math.h>

int att1_sampler_greedy_f32(const float *logits, size_t count, uint32_t *out_token)
{
    size_t i, best = 0;
    if (logits == NULL || out_token == NULL || count == 0) return -1;
    for (i = 0; i < count; i++)
        if (isnan(logits[i])) return -1;
    for (i = 1; i < count; i++)
        if (logits[i] > logits[best]) best = i;
    if (best > (size_t)UINT32_MAX) return -1;
    *out_token = (uint32_t)best;
    return 0;
}
