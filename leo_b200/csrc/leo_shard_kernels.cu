// Batch-end merge of one fixed tensor when the logical batch's stories are
// sharded over several GPUs (exact data parallelism).
//
// The merged value of element i is base[i] + (f32)((sum over the batch's
// stories, in story order, of the nonzero (f64)(lane[i] - base[i])) / stories),
// then projected (apply_mean_deltas, crates/leo-core/src/parallel.rs:715-798,
// 975-1022, 1169-1246) -- the same arithmetic as the single-GPU merge.  Each
// rank holds a contiguous range of stories, so the FP64 sum in story order is a
// scan over ranks: rank r adds its lanes' deltas, in lane order, to the partial
// sums it received from rank r - 1.  The kernels here are that rank-local work:
//   marks       element marks of this rank's lanes (some lane differs from base)
//   compact     marks (after a MAX all-reduce over ranks) -> sorted element list
//   accumulate  partial[j] (+)= this rank's nonzero lane deltas at list[j]
//   finalize    (last rank) merged value: mean, projection, finite check
//   commit      merged values into the canonical tensor and every resident lane
//   sync_own    each lane's own changed rows <- canonical; lane marks cleared
#include <stdint.h>

#include "leo_device.cuh"
#include "leo_kernels.h"
#include "leo_projection.cuh"

namespace {

constexpr uint32_t kThreads = 256;

__device__ __forceinline__ uint32_t own_length(const MergeTensor& t, int lane) {
    return t.lane_lists ? t.lane_counts[lane] : t.length;
}
__device__ __forceinline__ uint32_t own_item(const MergeTensor& t, int lane, uint32_t i) {
    return t.lane_lists ? t.lane_lists[lane][i] : i;
}

__global__ void __launch_bounds__(kThreads) shard_marks_kernel(MergeTensor t, int lanes, uint8_t* marks) {
    const uint32_t stride = gridDim.x * blockDim.x;
    for (int l = 0; l < lanes; ++l) {
        const uint32_t n = own_length(t, l) * t.row_len;
        const float* lv = t.lane_values[l];
        for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
            const uint32_t r = i / t.row_len, o = i - r * t.row_len;
            const size_t idx = (size_t)own_item(t, l, r) * t.row + o;
            if (lv[idx] - t.base[idx] != 0.0f) marks[idx] = 1;
        }
    }
}

// Sorted compaction in three launches: per-block counts of a fixed chunk,
// an exclusive scan of the block counts, then each block writes its chunk's
// marked indices in order.
__global__ void __launch_bounds__(kThreads) compact_count_kernel(const uint8_t* __restrict__ marks, size_t length,
                                                                 size_t chunk, uint32_t* block_counts) {
    const size_t begin = (size_t)blockIdx.x * chunk;
    const size_t end = begin + chunk < length ? begin + chunk : length;
    uint32_t c = 0;
    for (size_t i = begin + threadIdx.x; i < end; i += blockDim.x) c += marks[i] != 0;
    c = __reduce_add_sync(0xffffffffu, c);
    __shared__ uint32_t warp_sums[kThreads / 32];
    if ((threadIdx.x & 31u) == 0u) warp_sums[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t total = 0;
        for (uint32_t w = 0; w < kThreads / 32; ++w) total += warp_sums[w];
        block_counts[blockIdx.x] = total;
    }
}

// One block of 1024 threads, up to kScanPerThread counts per thread.
constexpr uint32_t kScanThreads = 1024, kScanPerThread = 8;

__global__ void __launch_bounds__(kScanThreads) compact_scan_kernel(uint32_t* block_counts, uint32_t blocks,
                                                                    uint32_t* total) {
    __shared__ uint32_t warp_sums[kScanThreads / 32];
    const uint32_t first = threadIdx.x * kScanPerThread;
    uint32_t local[kScanPerThread];
    uint32_t mine = 0;
#pragma unroll
    for (uint32_t k = 0; k < kScanPerThread; ++k) {
        local[k] = first + k < blocks ? block_counts[first + k] : 0u;
        mine += local[k];
    }
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    uint32_t incl = mine;
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= (uint32_t)o) incl += y;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const uint32_t w = warp_sums[lane];
        uint32_t wi = w;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= (uint32_t)o) wi += y;
        }
        warp_sums[lane] = wi - w;
        if (lane == 31) *total = wi;
    }
    __syncthreads();
    uint32_t run = warp_sums[warp] + incl - mine;
#pragma unroll
    for (uint32_t k = 0; k < kScanPerThread; ++k) {
        if (first + k < blocks) block_counts[first + k] = run;
        run += local[k];
    }
}

__global__ void __launch_bounds__(kThreads) compact_write_kernel(const uint8_t* __restrict__ marks, size_t length,
                                                                 size_t chunk, const uint32_t* block_offsets,
                                                                 uint32_t* list) {
    __shared__ uint32_t warp_sums[kThreads / 32];
    __shared__ uint32_t base;
    const size_t begin = (size_t)blockIdx.x * chunk;
    const size_t end = begin + chunk < length ? begin + chunk : length;
    if (threadIdx.x == 0) base = block_offsets[blockIdx.x];
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    for (size_t tile = begin; tile < end; tile += blockDim.x) {
        const size_t i = tile + threadIdx.x;
        const bool hit = i < end && marks[i] != 0;
        const unsigned int ballot = __ballot_sync(0xffffffffu, hit);
        if (lane == 0) warp_sums[warp] = __popc(ballot);
        __syncthreads();
        uint32_t before = 0, tile_total = 0;
        for (uint32_t w = 0; w < kThreads / 32; ++w) {
            if (w < warp) before += warp_sums[w];
            tile_total += warp_sums[w];
        }
        if (hit) list[base + before + __popc(ballot & ((1u << lane) - 1u))] = (uint32_t)i;
        __syncthreads();
        if (threadIdx.x == 0) base += tile_total;
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kThreads) shard_accumulate_kernel(float** lane_values, int lanes,
                                                                    const float* __restrict__ base,
                                                                    const uint32_t* __restrict__ list, uint32_t count,
                                                                    double* partial, int first, uint32_t* error_flag) {
    for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < count; j += gridDim.x * blockDim.x) {
        const size_t idx = list[j];
        const float before = base[idx];
        double sum = first ? 0.0 : partial[j];
        for (int l = 0; l < lanes; ++l) {
            const float delta = lane_values[l][idx] - before;
            if (delta != 0.0f) {
                if (!isfinite(delta)) atomicOr(error_flag, LEO_ERR_CAPACITY);
                sum += (double)delta;
            }
        }
        partial[j] = sum;
    }
}

__global__ void __launch_bounds__(kThreads) shard_finalize_kernel(const float* __restrict__ base,
                                                                  const uint32_t* __restrict__ list, uint32_t count,
                                                                  const double* __restrict__ partial, float* values,
                                                                  double divisor, uint32_t kind, float wmin, float wmax,
                                                                  const uint8_t* __restrict__ neuron_type,
                                                                  uint32_t synapses_per_neuron, uint32_t* error_flag) {
    for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < count; j += gridDim.x * blockDim.x) {
        const size_t idx = list[j];
        float v = base[idx] + __double2float_rn(partial[j] / divisor);
        v = leo_project(v, kind, idx, wmin, wmax, neuron_type, synapses_per_neuron);
        if (!isfinite(v)) atomicOr(error_flag, 1u);
        values[j] = v;
    }
}

__global__ void __launch_bounds__(kThreads) shard_commit_kernel(float* base, const uint32_t* __restrict__ list,
                                                                uint32_t count, const float* __restrict__ values,
                                                                float** lane_values, int lanes) {
    for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < count; j += gridDim.x * blockDim.x) {
        const size_t idx = list[j];
        const float v = values[j];
        base[idx] = v;
        for (int l = 0; l < lanes; ++l) lane_values[l][idx] = v;
    }
}

__global__ void __launch_bounds__(kThreads) shard_sync_own_kernel(MergeTensor t, int lanes) {
    const uint32_t stride = gridDim.x * blockDim.x;
    for (int l = 0; l < lanes; ++l) {
        const uint32_t n = own_length(t, l) * t.row_len;
        float* lv = t.lane_values[l];
        for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
            const uint32_t r = i / t.row_len, o = i - r * t.row_len;
            const uint32_t item = own_item(t, l, r);
            lv[(size_t)item * t.row + o] = t.base[(size_t)item * t.row + o];
            if (o == 0 && t.lane_marks) t.lane_marks[l][item] = 0;
        }
    }
}

}  // namespace

void leo_launch_shard_marks(const MergeTensor& t, int lanes, uint8_t* marks, int grid, cudaStream_t stream) {
    if (lanes > 0) shard_marks_kernel<<<grid, kThreads, 0, stream>>>(t, lanes, marks);
}

// Chunk per block grows with the length so that the block counts fit one scan block.
size_t leo_compact_chunk(size_t length) {
    size_t chunk = 16384;
    while ((length + chunk - 1) / chunk > (size_t)kScanThreads * kScanPerThread) chunk <<= 1;
    return chunk;
}

size_t leo_compact_scratch_blocks(size_t length) {
    const size_t chunk = leo_compact_chunk(length);
    return (length + chunk - 1) / chunk;
}

void leo_launch_compact(const uint8_t* marks, size_t length, uint32_t* list, uint32_t* total, uint32_t* block_scratch,
                        cudaStream_t stream) {
    const size_t chunk = leo_compact_chunk(length);
    const uint32_t blocks = (uint32_t)leo_compact_scratch_blocks(length);
    if (blocks == 0) {
        cudaMemsetAsync(total, 0, sizeof(uint32_t), stream);
        return;
    }
    compact_count_kernel<<<blocks, kThreads, 0, stream>>>(marks, length, chunk, block_scratch);
    compact_scan_kernel<<<1, kScanThreads, 0, stream>>>(block_scratch, blocks, total);
    compact_write_kernel<<<blocks, kThreads, 0, stream>>>(marks, length, chunk, block_scratch, list);
}

void leo_launch_shard_accumulate(float** lane_values, int lanes, const float* base, const uint32_t* list,
                                 uint32_t count, double* partial, int first, uint32_t* error_flag, int grid,
                                 cudaStream_t stream) {
    if (count) shard_accumulate_kernel<<<grid, kThreads, 0, stream>>>(lane_values, lanes, base, list, count, partial,
                                                                      first, error_flag);
}

void leo_launch_shard_finalize(const float* base, const uint32_t* list, uint32_t count, const double* partial,
                               float* values, double divisor, uint32_t kind, float wmin, float wmax,
                               const uint8_t* neuron_type, uint32_t synapses_per_neuron, uint32_t* error_flag,
                               int grid, cudaStream_t stream) {
    if (count)
        shard_finalize_kernel<<<grid, kThreads, 0, stream>>>(base, list, count, partial, values, divisor, kind, wmin,
                                                             wmax, neuron_type, synapses_per_neuron, error_flag);
}

void leo_launch_shard_commit(float* base, const uint32_t* list, uint32_t count, const float* values,
                             float** lane_values, int lanes, int grid, cudaStream_t stream) {
    if (count) shard_commit_kernel<<<grid, kThreads, 0, stream>>>(base, list, count, values, lane_values, lanes);
}

void leo_launch_shard_sync_own(const MergeTensor& t, int lanes, int grid, cudaStream_t stream) {
    if (lanes > 0) shard_sync_own_kernel<<<grid, kThreads, 0, stream>>>(t, lanes);
}
