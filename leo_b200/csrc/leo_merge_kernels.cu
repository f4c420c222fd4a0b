// Batch-end sparse delta merge and lane sync for sm_100a.
//
// Reference semantics: apply_mean_deltas / apply_sparse_scaled
// (crates/leo-core/src/parallel.rs:694-798, 975-1022): every parameter that
// some story changed gets base += (f32)((sum over stories in story order of
// (f64)delta) / stories), then the sparse projection and validation of
// parallel.rs:1169-1345.  The reference GPU does this with a dense lane
// reducer over every parameter (cuda_kernels.cu:6284-6439) followed by one
// scatter launch per tensor per target (cuda_kernels.cu:6721-6810); here the
// union of the lanes' changed lists drives a sparse reduction, and one fused
// scatter writes each merged value into every lane.
//
// Three passes per tensor:
//   union   each lane's changed list -> indices where some lane differs from
//           the canonical value (union marks + list); lane marks are cleared
//   apply   per union index: ordered FP64 sum over lanes, mean, projection,
//           validation, canonical update
//   sync    every lane gets the canonical value at its own changed indices
//           and at every union index (a lane whose change reverted to the
//           base value, and a lane that never touched the index, both end
//           equal to the canonical model)
#include <stdint.h>

#include "leo_device.cuh"
#include "leo_kernels.h"
#include "leo_projection.cuh"

namespace {

__device__ __forceinline__ bool set_byte_mark(uint8_t* marks, uint32_t index) {
    unsigned int* word = reinterpret_cast<unsigned int*>(reinterpret_cast<uintptr_t>(marks + index) & ~(uintptr_t)3);
    unsigned int shift = (unsigned int)((reinterpret_cast<uintptr_t>(marks + index) & 3u) * 8u);
    unsigned int bit = 1u << shift;
    return (atomicOr(word, bit) & bit) == 0u;
}

__device__ __forceinline__ uint32_t list_length(const MergeTensor& t, int lane) {
    return t.lane_lists ? t.lane_counts[lane] : t.length;
}
__device__ __forceinline__ uint32_t list_item(const MergeTensor& t, int lane, uint32_t i) {
    return t.lane_lists ? t.lane_lists[lane][i] : i;
}

__global__ void __launch_bounds__(256) merge_union_kernel(MergeTensor t, MergeScratch m, int lanes) {
    const uint32_t stride = gridDim.x * blockDim.x;
    for (int l = 0; l < lanes; ++l) {
        uint32_t count = list_length(t, l);
        const float* lv = t.lane_values[l];
        for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride) {
            uint32_t u = list_item(t, l, i);
            if (t.lane_marks) t.lane_marks[l][u] = 0;
            bool differs = false;
            size_t base = (size_t)u * t.row;
            for (uint32_t o = 0; o < t.row_len && !differs; ++o) differs = lv[base + o] != t.base[base + o];
            if (differs && set_byte_mark(m.union_mark, u)) m.union_list[atomicAdd(m.union_count, 1u)] = u;
        }
    }
}

__global__ void __launch_bounds__(256) merge_apply_kernel(MergeTensor t, MergeScratch m, int lanes, float wmin,
                                                          float wmax, const uint8_t* __restrict__ neuron_type,
                                                          uint32_t synapses_per_neuron) {
    const uint32_t stride = gridDim.x * blockDim.x;
    uint32_t count = *m.union_count;
    uint32_t total = count * t.row_len;
    uint32_t applied = 0;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        uint32_t r = i / t.row_len, o = i - r * t.row_len;
        uint32_t u = m.union_list[r];
        size_t idx = (size_t)u * t.row + o;
        float before = t.base[idx];
        double sum = 0.0;
        bool any = false;
        for (int l = 0; l < lanes; ++l) {
            float after = t.lane_values[l][idx];
            float delta = after - before;
            if (delta != 0.0f) {
                any = true;
                if (!isfinite(delta)) atomicOr(m.error_flag, LEO_ERR_CAPACITY);
                sum += (double)delta;
            }
        }
        if (!any) continue;
        float v = before + __double2float_rn(sum / (double)lanes);
        v = leo_project(v, t.kind, (size_t)u, wmin, wmax, neuron_type, synapses_per_neuron);
        if (!isfinite(v)) atomicOr(m.error_flag, 1u);
        t.base[idx] = v;
        ++applied;
    }
    if (applied) atomicAdd(m.updates, applied);
}

__global__ void __launch_bounds__(256) merge_sync_kernel(MergeTensor t, MergeScratch m, int lanes, int sync_lanes) {
    const uint32_t stride = gridDim.x * blockDim.x;
    uint32_t count = *m.union_count;
    // Every union index into every resident lane (fused multi-target scatter).
    uint32_t total = count * t.row_len;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        uint32_t r = i / t.row_len, o = i - r * t.row_len;
        size_t idx = (size_t)m.union_list[r] * t.row + o;
        float v = t.base[idx];
        for (int l = 0; l < sync_lanes; ++l) t.lane_values[l][idx] = v;
    }
    // Each lane's own changed indices (reverted changes included).
    for (int l = 0; l < lanes; ++l) {
        uint32_t n = list_length(t, l) * t.row_len;
        float* lv = t.lane_values[l];
        for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
            uint32_t r = i / t.row_len, o = i - r * t.row_len;
            size_t idx = (size_t)list_item(t, l, r) * t.row + o;
            lv[idx] = t.base[idx];
        }
    }
}

__global__ void merge_clear_kernel(MergeScratch m) {
    uint32_t count = *m.union_count;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x)
        m.union_mark[m.union_list[i]] = 0;
}

}  // namespace

namespace {
__global__ void __launch_bounds__(256) scatter_rows_kernel(float** lane_values, int lanes, const float* __restrict__ base,
                                                           const uint32_t* __restrict__ list, uint32_t count,
                                                           uint32_t row, uint32_t row_len) {
    uint32_t total = count * row_len;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        uint32_t r = i / row_len, o = i - r * row_len;
        size_t idx = (size_t)list[r] * row + o;
        float v = base[idx];
        for (int l = 0; l < lanes; ++l) lane_values[l][idx] = v;
    }
}
}  // namespace

void leo_launch_merge_tensor(const MergeTensor& t, const MergeScratch& m, int lanes, int sync_lanes, float wmin,
                             float wmax, const uint8_t* neuron_type, uint32_t synapses_per_neuron, int grid,
                             cudaStream_t stream) {
    cudaMemsetAsync(m.union_count, 0, sizeof(uint32_t), stream);
    merge_union_kernel<<<grid, 256, 0, stream>>>(t, m, lanes);
    merge_apply_kernel<<<grid, 256, 0, stream>>>(t, m, lanes, wmin, wmax, neuron_type, synapses_per_neuron);
    merge_sync_kernel<<<grid, 256, 0, stream>>>(t, m, lanes, sync_lanes);
    merge_clear_kernel<<<grid, 256, 0, stream>>>(m);
}

void leo_launch_scatter_rows(float** lane_values, int lanes, const float* base, const uint32_t* list, uint32_t count,
                             uint32_t row, uint32_t row_len, int grid, cudaStream_t stream) {
    if (count == 0 || lanes == 0) return;
    scatter_rows_kernel<<<grid, 256, 0, stream>>>(lane_values, lanes, base, list, count, row, row_len);
}
