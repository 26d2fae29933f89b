/*
 * att1.h - umbrella header of the B200 implementation of ATT-1's decode path.
 * Covers the parts of ATT-1's include/att1.h that the decode hot path uses.
 */
#ifndef ATT1_H
#define ATT1_H

#include "att1_backend.h"
#include "att1_cluster_infer.h"
#include "att1_infer.h"
#include "att1_model.h"
#include "att1_quant.h"
#include "att1_sampler.h"
#include "att1_status.h"
#include "att1_trace.h"
#include "att1_b200.h"

#define ATT1_VERSION_MAJOR 0
#define ATT1_VERSION_MINOR 0
#define ATT1_VERSION_PATCH 0

#endif
