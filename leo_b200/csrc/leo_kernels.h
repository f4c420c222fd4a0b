// Host-side launchers for the sm_100a kernels (implemented in the .cu files).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "leo_device.cuh"

// The persistent wavefront: lane_count clusters of `cluster` CTAs, each
// running its lane's schedule over steps [begin, end).
cudaError_t leo_launch_wavefront(const LaneState* lanes, int lane_count, uint32_t cluster, uint32_t begin,
                                 uint32_t end, const KernelConsts& kc, cudaStream_t stream);
size_t leo_wavefront_smem_bytes(const KernelConsts& kc);
cudaError_t leo_wavefront_configure();
// One lane over `ctas` CTAs (one per SM) in a cooperative launch.
cudaError_t leo_launch_wavefront_grid(const LaneState* lane, uint32_t ctas, uint32_t begin, uint32_t end,
                                      const KernelConsts& kc, cudaStream_t stream);
// CTAs of the whole-GPU launch that can be resident at once (0: none).
cudaError_t leo_wavefront_grid_ctas(const KernelConsts& kc, int sms, int* out);
// Clusters of `cluster` CTAs that can be resident at once.
cudaError_t leo_wavefront_max_clusters(uint32_t cluster, const KernelConsts& kc, int* out);

// Batch-end keyed context merge on the device (leo_context_merge.cu).
#define LEO_CTX_MERGE_BAD_DELTA 1u  // a lane's context delta is not finite
#define LEO_CTX_MERGE_BAD_VALUE 2u  // a merged embedding is not finite after projection

struct CtxMergeArgs {
    uint32_t slots_per_order, dim, probe_limit, stories;
    float weight_min, weight_max;
    // per entry (a lane's changed slot), lane-major
    uint32_t* lane_slots;
    uint8_t* valid;
    unsigned long long* key;
    uint32_t* order;
    uint32_t* obs_inc;
    float* delta;                 // [entries * dim]
    // per merged (order, key)
    double* msum;                 // [groups * dim]
    unsigned long long* mkey;
    uint32_t* morder;
    unsigned long long* mobs;
    // canonical slots the merge wrote
    uint32_t* canon_slots;
    uint32_t* canon_slot_count;
    uint32_t canon_slot_capacity;
    uint32_t* error;
};

struct CtxMergeWork {
    void* temp;
    size_t temp_bytes;
    uint32_t *idx_a, *idx_b, *sorted, *gstart, *k32_a, *k32_b, *count;
    unsigned long long *k64_a, *k64_b;
    uint8_t* head;
};

size_t leo_context_apply_smem(uint32_t slots_per_order);
size_t leo_context_merge_temp_bytes(uint32_t capacity);
cudaError_t leo_context_merge_configure();
cudaError_t leo_context_merge_deltas(const LaneState* lanes, const uint32_t* lane_offset, uint32_t lane_count,
                                     uint32_t max_lane_entries, LaneParams canon, const CtxMergeArgs& a,
                                     cudaStream_t stream);
cudaError_t leo_context_merge_group(uint32_t entries, const CtxMergeArgs& a, CtxMergeWork& w, uint32_t* valid_out,
                                    cudaStream_t stream);
cudaError_t leo_context_merge_sort(uint32_t valid, const CtxMergeArgs& a, CtxMergeWork& w, uint32_t* groups_out,
                                   cudaStream_t stream);
cudaError_t leo_context_merge_apply(uint32_t valid, uint32_t groups, uint32_t orders, LaneParams canon,
                                    const LaneState* lanes, int lane_count, const uint32_t* lane_slots,
                                    uint32_t lane_slot_count, const CtxMergeArgs& a, CtxMergeWork& w,
                                    cudaStream_t stream);

// Zeroes n float4 with evict-first (streaming) stores (leo_schedule.cu).
cudaError_t leo_launch_zero_streaming(float4* p, size_t n, cudaStream_t stream);

// Every lane's step schedule from the batch's story bytes (leo_schedule.cu):
// lane i's story is bytes[offsets[i], offsets[i + 1]), written to lanes[i].schedule.
cudaError_t leo_launch_build_schedules(const uint8_t* bytes, const uint64_t* offsets, const LaneState* lanes,
                                       uint32_t count, uint32_t permission, cudaStream_t stream);

// Batch-end sparse merge of one fixed f32 tensor (threshold, recurrent, input,
// output rows, bias, context output): see leo_merge_kernels.cu.
struct MergeTensor {
    float** lane_values;          // device array [lanes] of lane tensor pointers
    float* base;                  // canonical tensor
    uint32_t** lane_lists;        // device array [lanes] of changed-index lists (rows for output)
    uint32_t* lane_counts;        // device array [lanes] of list lengths
    uint8_t** lane_marks;         // device array [lanes] of changed marks (cleared by the merge)
    uint32_t row;                 // 1 for element tensors, LEO_OUTPUT_STRIDE for output rows
    uint32_t row_len;             // 1, or 257 valid entries per output row
    uint32_t length;              // elements (rows for output)
    uint32_t kind;                // projection rule, see LeoProjection
};

enum LeoProjection : uint32_t {
    LEO_PROJECT_THRESHOLD = 0,   // clamp [0.05, 2]
    LEO_PROJECT_RECURRENT = 1,   // clamp [wmin, wmax], sign by source type
    LEO_PROJECT_INPUT = 2,       // clamp [0, wmax]
    LEO_PROJECT_WEIGHT = 3,      // clamp [wmin, wmax]
    LEO_PROJECT_NONE = 4         // bias: no clamp
};

struct MergeScratch {
    uint8_t* union_mark;          // [length] cleared after use
    uint32_t* union_list;         // [length]
    uint32_t* union_count;        // [1]
    uint32_t* updates;            // [1] indices whose merged delta was applied
    uint32_t* error_flag;         // [1]
};

// `lanes` stories contribute deltas (the first entries of the pointer tables);
// all `sync_lanes` resident lanes receive the merged canonical values.
void leo_launch_merge_tensor(const MergeTensor& t, const MergeScratch& m, int lanes, int sync_lanes, float wmin,
                             float wmax, const uint8_t* neuron_type, uint32_t synapses_per_neuron, int grid,
                             cudaStream_t stream);

// Writes base[list[i] * row + o] (o < row_len) into every lane tensor.
void leo_launch_scatter_rows(float** lane_values, int lanes, const float* base, const uint32_t* list, uint32_t count,
                             uint32_t row, uint32_t row_len, int grid, cudaStream_t stream);

// Rank-local steps of the sharded (multi-GPU) merge; see leo_shard_kernels.cu.
void leo_launch_shard_marks(const MergeTensor& t, int lanes, uint8_t* marks, int grid, cudaStream_t stream);
size_t leo_compact_scratch_blocks(size_t length);
void leo_launch_compact(const uint8_t* marks, size_t length, uint32_t* list, uint32_t* total, uint32_t* block_scratch,
                        cudaStream_t stream);
void leo_launch_shard_accumulate(float** lane_values, int lanes, const float* base, const uint32_t* list,
                                 uint32_t count, double* partial, int first, uint32_t* error_flag, int grid,
                                 cudaStream_t stream);
void leo_launch_shard_finalize(const float* base, const uint32_t* list, uint32_t count, const double* partial,
                               float* values, double divisor, uint32_t kind, float wmin, float wmax,
                               const uint8_t* neuron_type, uint32_t synapses_per_neuron, uint32_t* error_flag,
                               int grid, cudaStream_t stream);
void leo_launch_shard_commit(float* base, const uint32_t* list, uint32_t count, const float* values,
                             float** lane_values, int lanes, int grid, cudaStream_t stream);
void leo_launch_shard_sync_own(const MergeTensor& t, int lanes, int grid, cudaStream_t stream);

// Sets the text leo_b200_last_error() returns on this thread.
void leo_set_last_error(const char* what);
