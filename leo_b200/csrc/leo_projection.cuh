// Projection of a merged parameter onto the model's constraints
// (crates/leo-core/src/parallel.rs:1169-1246): the clamp rule per tensor.
// f32::clamp and f32::max / f32::min semantics: NaN passes through clamp and
// max/min return the non-NaN operand.
#pragma once

#include <stdint.h>

#include "leo_kernels.h"

__device__ __forceinline__ float leo_clampf(float v, float lo, float hi) {
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}
__device__ __forceinline__ float leo_rmax(float a, float b) {
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a > b ? a : (b > a ? b : a);
}
__device__ __forceinline__ float leo_rmin(float a, float b) {
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a < b ? a : (b < a ? b : a);
}

// `index` is the element index inside the tensor (the recurrent rule needs the
// source neuron, index / synapses_per_neuron).
__device__ __forceinline__ float leo_project(float v, uint32_t kind, size_t index, float wmin, float wmax,
                                             const uint8_t* __restrict__ neuron_type, uint32_t synapses_per_neuron) {
    switch (kind) {
        case LEO_PROJECT_THRESHOLD: return leo_clampf(v, 0.05f, 2.0f);
        case LEO_PROJECT_RECURRENT:
            v = leo_clampf(v, wmin, wmax);
            return neuron_type[index / synapses_per_neuron] == 0 ? leo_rmax(v, 0.0f) : leo_rmin(v, 0.0f);
        case LEO_PROJECT_INPUT: return leo_clampf(v, 0.0f, wmax);
        case LEO_PROJECT_WEIGHT: return leo_clampf(v, wmin, wmax);
        default: return v;
    }
}
