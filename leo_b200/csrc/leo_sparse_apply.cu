// Batch-end sparse mean apply of one tensor, plus the sync into its replicas.
//
// Reference semantics: apply_sparse_scaled (crates/leo-core/src/parallel.rs:
// 975-1022) with divisor = number of stories -- for every index that appears
// in some story's sorted delta list, target[i] += (f32)((sum over stories in
// story order of (f64)delta) / stories) -- followed by the clamp projection
// of parallel.rs:1226-1233, and then the merged values are written into every
// replica of the tensor (the per-target scatter of cuda.rs:2869-3080 /
// cuda_kernels.cu:6721-6810, fused into one pass here).
//
// Two kernels, no atomics on the data:
//   tile_bounds  one thread per input entry: validates (index in range,
//                strictly increasing within its story, finite delta) and
//                writes, for every story, where each 4096-index tile of the
//                tensor starts in that story's list (a [stories][tiles + 1]
//                table of absolute entry positions).
//   tile_merge   one CTA per tile: stories in order, each story's entries of
//                the tile accumulated into FP64 sums in shared memory (indices
//                are unique within a story, so a story's entries never collide;
//                a barrier between stories keeps the story order), then every
//                touched index of the tile gets its mean, projection, finite
//                check and the writes to the target and all replicas.
// Every entry is read once and every merged value written once per copy, so
// the pass moves the algorithmic bytes: 8 B per input entry plus
// (4 read + 4 + 4 x replicas written) B per merged index.
#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "leo_kernels.h"
#include "leo_sparse_apply.h"

namespace {

constexpr uint32_t kTile = LEO_SPARSE_APPLY_TILE;
constexpr uint32_t kThreads = 256;

__global__ void __launch_bounds__(kThreads) tile_bounds_kernel(SparseApplyArgs a) {
    const uint64_t total = a.offsets.v[a.stories];
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint32_t* counters = a.scratch;
    uint32_t* table = a.scratch + LEO_SPARSE_APPLY_COUNTERS;
    const uint32_t row = a.tiles + 1;
    for (uint64_t j = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; j < total; j += stride) {
        // story of entry j: last s with offsets[s] <= j (empty stories skipped)
        uint32_t lo = 0, hi = a.stories;
        while (hi - lo > 1) {
            uint32_t mid = (lo + hi) >> 1;
            if (a.offsets.v[mid] <= j)
                lo = mid;
            else
                hi = mid;
        }
        const uint32_t s = lo;
        const uint64_t first = a.offsets.v[s], end = a.offsets.v[s + 1];
        const uint32_t idx = a.indices[j];
        const float d = a.deltas[j];
        bool ok = idx < a.length;
        if (!ok) atomicOr(&counters[1], LEO_SPARSE_APPLY_ERR_RANGE);
        if (!isfinite(d)) atomicOr(&counters[1], LEO_SPARSE_APPLY_ERR_DELTA);
        uint32_t t0 = 0;
        if (j > first) {
            const uint32_t prev = a.indices[j - 1];
            if (prev >= idx) {
                atomicOr(&counters[1], LEO_SPARSE_APPLY_ERR_ORDER);
                ok = false;
            }
            t0 = prev < a.length ? prev / kTile + 1 : a.tiles;
        }
        const uint32_t t1 = ok ? idx / kTile : t0 - 1;  // no writes when invalid
        for (uint32_t t = t0; ok && t <= t1; ++t) table[(size_t)s * row + t] = (uint32_t)j;
        if (j + 1 == end) {
            const uint32_t last = ok ? t1 + 1 : a.tiles;
            for (uint32_t t = last; t <= a.tiles; ++t) table[(size_t)s * row + t] = (uint32_t)end;
        }
    }
    // Empty stories: every tile starts (and ends) at the story's offset.
    for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < (uint64_t)a.stories * row; k += stride) {
        const uint32_t s = (uint32_t)(k / row);
        if (a.offsets.v[s] == a.offsets.v[s + 1]) table[k] = (uint32_t)a.offsets.v[s];
    }
}

__device__ __forceinline__ float clamp_projection(float v, float lo, float hi) {
    // f32::clamp: NaN passes through
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}

__global__ void __launch_bounds__(kThreads) tile_merge_kernel(SparseApplyArgs a) {
    __shared__ double sums[kTile];
    __shared__ uint32_t marks[kTile / 32];
    __shared__ uint32_t block_updates;
    uint32_t* counters = a.scratch;
    if (counters[1] != 0u) return;  // invalid input: nothing is modified
    const uint32_t* table = a.scratch + LEO_SPARSE_APPLY_COUNTERS;
    const uint32_t row = a.tiles + 1;
    const double divisor = (double)a.stories;
    for (uint32_t tile = blockIdx.x; tile < a.tiles; tile += gridDim.x) {
        const uint32_t base = tile * kTile;
        for (uint32_t i = threadIdx.x; i < kTile / 32; i += blockDim.x) marks[i] = 0u;
        if (threadIdx.x == 0) block_updates = 0u;
        __syncthreads();
        for (uint32_t s = 0; s < a.stories; ++s) {
            const uint32_t b = table[(size_t)s * row + tile], e = table[(size_t)s * row + tile + 1];
            for (uint32_t j = b + threadIdx.x; j < e; j += blockDim.x) {
                const uint32_t local = a.indices[j] - base;
                const double d = (double)a.deltas[j];
                const uint32_t bit = 1u << (local & 31u);
                const uint32_t old = atomicOr(&marks[local >> 5], bit);
                // The reference's sum starts at 0.0 and adds each story's delta.
                sums[local] = ((old & bit) ? sums[local] : 0.0) + d;
            }
            __syncthreads();
        }
        const uint32_t span = min(kTile, a.length - base);
        uint32_t updates = 0;
        for (uint32_t local = threadIdx.x; local < span; local += blockDim.x) {
            if (!(marks[local >> 5] & (1u << (local & 31u)))) continue;
            const uint32_t i = base + local;
            float v = a.target[i] + __double2float_rn(sums[local] / divisor);
            if (!isfinite(v)) atomicOr(&counters[1], LEO_SPARSE_APPLY_ERR_MERGED);
            v = clamp_projection(v, a.lo, a.hi);
            a.target[i] = v;
            for (uint32_t r = 0; r < a.replica_count; ++r) a.replicas.ptr[r][i] = v;
            ++updates;
        }
        updates = __reduce_add_sync(0xffffffffu, updates);
        if ((threadIdx.x & 31u) == 0u && updates) atomicAdd(&block_updates, updates);
        __syncthreads();
        if (threadIdx.x == 0 && block_updates) atomicAdd(&counters[0], block_updates);
        __syncthreads();
    }
}

struct ApplyFailure : std::runtime_error {
    using std::runtime_error::runtime_error;
};

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw ApplyFailure(std::string(what) + ": " + cudaGetErrorString(e));
}

struct DeviceScratch {
    uint32_t* ptr = nullptr;
    size_t words = 0;
    std::mutex lock;
};

DeviceScratch g_scratch[LEO_SPARSE_APPLY_MAX_DEVICES];

// Fixed scratch of leo_b200_sparse_mean_apply_static: 1 MiB of device memory
// reserved when the module loads, so that entry point never allocates.  Its
// first LEO_SPARSE_APPLY_COUNTERS words are counters that every call zeroes
// before its kernels run; the tile table after them is written in full by
// every call and needs no initial value.  One array per device, shared by
// every call on that device: calls that overlap in time (two host threads, or
// two streams without ordering between them) race on it.
static __device__ __align__(256) uint32_t leo_sparse_apply_static_scratch[LEO_SPARSE_APPLY_STATIC_WORDS];

// Device address of that array, resolved once per device (cudaGetSymbolAddress).
uint32_t* g_static_scratch[LEO_SPARSE_APPLY_MAX_DEVICES];
std::mutex g_static_lock;

uint32_t* static_scratch_address(int device) {
    std::lock_guard<std::mutex> guard(g_static_lock);
    if (g_static_scratch[device] == nullptr) {
        void* ptr = nullptr;
        check(cudaGetSymbolAddress(&ptr, leo_sparse_apply_static_scratch), "cudaGetSymbolAddress(static scratch)");
        g_static_scratch[device] = static_cast<uint32_t*>(ptr);
    }
    return g_static_scratch[device];
}

}  // namespace

size_t leo_sparse_apply_scratch_words(uint32_t length, uint32_t stories) {
    const uint64_t tiles = ((uint64_t)length + kTile - 1) / kTile;
    return (size_t)(LEO_SPARSE_APPLY_COUNTERS + (uint64_t)stories * (tiles + 1));
}

void leo_sparse_apply_prepare(SparseApplyArgs& a, float* target, uint32_t length, const uint32_t* indices,
                              const float* deltas, const uint64_t* story_offsets, uint32_t stories, float lo, float hi,
                              float* const* replicas, uint32_t replica_count) {
    if (target == nullptr && length > 0) throw ApplyFailure("target is null");
    if (stories == 0) throw ApplyFailure("cannot merge an empty worker batch");
    if (stories > LEO_SPARSE_APPLY_MAX_STORIES) throw ApplyFailure("too many stories for one sparse apply call");
    if (replica_count > LEO_SPARSE_APPLY_MAX_REPLICAS) throw ApplyFailure("too many replicas for one sparse apply call");
    if (replica_count > 0 && replicas == nullptr) throw ApplyFailure("replica table is null");
    if (story_offsets == nullptr) throw ApplyFailure("story offsets are null");
    if (story_offsets[0] != 0) throw ApplyFailure("story offsets must start at 0");
    for (uint32_t s = 0; s < stories; ++s)
        if (story_offsets[s + 1] < story_offsets[s]) throw ApplyFailure("story offsets must be non-decreasing");
    const uint64_t total = story_offsets[stories];
    if (total >= 0xffffffffull) throw ApplyFailure("too many delta entries for one sparse apply call");
    if (total > 0 && (indices == nullptr || deltas == nullptr)) throw ApplyFailure("delta arrays are null");
    if (std::isnan(lo) || std::isnan(hi) || lo > hi) throw ApplyFailure("projection bounds must satisfy lo <= hi");
    if (length == 0 && total > 0) throw ApplyFailure("delta index out of range");
    std::memset(&a, 0, sizeof(a));
    a.target = target;
    a.length = length;
    a.indices = indices;
    a.deltas = deltas;
    a.stories = stories;
    a.tiles = (uint32_t)(((uint64_t)length + kTile - 1) / kTile);
    a.lo = lo;
    a.hi = hi;
    a.replica_count = replica_count;
    for (uint32_t s = 0; s <= stories; ++s) a.offsets.v[s] = story_offsets[s];
    for (uint32_t r = 0; r < replica_count; ++r) {
        if (replicas[r] == nullptr) throw ApplyFailure("replica pointer is null");
        a.replicas.ptr[r] = replicas[r];
    }
}

// Launches both kernels on `stream` with the scratch in a.scratch (counters
// zeroed here), waits, and returns the merged index count.
uint32_t leo_sparse_apply_run(SparseApplyArgs& a, cudaStream_t stream) {
    check(cudaMemsetAsync(a.scratch, 0, LEO_SPARSE_APPLY_COUNTERS * sizeof(uint32_t), stream), "clear counters");
    if (a.length > 0) {
        int dev = 0, sms = 148;
        check(cudaGetDevice(&dev), "cudaGetDevice");
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
        const uint64_t total = a.offsets.v[a.stories];
        const uint64_t work = total > (uint64_t)a.stories * (a.tiles + 1) ? total : (uint64_t)a.stories * (a.tiles + 1);
        uint32_t grid = (uint32_t)((work + kThreads - 1) / kThreads);
        grid = grid < 1u ? 1u : (grid > (uint32_t)sms * 8u ? (uint32_t)sms * 8u : grid);
        tile_bounds_kernel<<<grid, kThreads, 0, stream>>>(a);
        check(cudaGetLastError(), "tile_bounds_kernel");
        const uint32_t merge_grid = a.tiles < (uint32_t)sms * 6u ? a.tiles : (uint32_t)sms * 6u;
        tile_merge_kernel<<<merge_grid, kThreads, 0, stream>>>(a);
        check(cudaGetLastError(), "tile_merge_kernel");
    }
    uint32_t counters[2] = {0, 0};
    check(cudaMemcpyAsync(counters, a.scratch, sizeof(counters), cudaMemcpyDeviceToHost, stream), "read counters");
    check(cudaStreamSynchronize(stream), "sparse apply");
    if (counters[1] & LEO_SPARSE_APPLY_ERR_RANGE) throw ApplyFailure("delta index out of range");
    if (counters[1] & LEO_SPARSE_APPLY_ERR_ORDER)
        throw ApplyFailure("delta indices must be strictly increasing within each story");
    if (counters[1] & LEO_SPARSE_APPLY_ERR_DELTA) throw ApplyFailure("invalid sparse worker parameter delta");
    if (counters[1] & LEO_SPARSE_APPLY_ERR_MERGED) throw ApplyFailure("merged parameter became non-finite");
    return counters[0];
}

extern "C" {

int leo_b200_sparse_mean_apply(int device, float* target, uint32_t length, const uint32_t* indices,
                               const float* deltas, const uint64_t* story_offsets, uint32_t stories, float lo,
                               float hi, float* const* replicas, uint32_t replica_count, void* stream,
                               uint32_t* updates) {
    int previous = -1;
    try {
        if (device < 0 || device >= LEO_SPARSE_APPLY_MAX_DEVICES) throw ApplyFailure("invalid device ordinal");
        SparseApplyArgs a;
        leo_sparse_apply_prepare(a, target, length, indices, deltas, story_offsets, stories, lo, hi, replicas,
                                 replica_count);
        check(cudaGetDevice(&previous), "cudaGetDevice");
        check(cudaSetDevice(device), "cudaSetDevice");
        DeviceScratch& sc = g_scratch[device];
        std::lock_guard<std::mutex> guard(sc.lock);
        const size_t words = leo_sparse_apply_scratch_words(length, stories);
        if (words > sc.words) {
            if (sc.ptr) check(cudaFree(sc.ptr), "cudaFree scratch");
            sc.ptr = nullptr;
            sc.words = 0;
            check(cudaMalloc(&sc.ptr, words * sizeof(uint32_t)), "cudaMalloc scratch");
            sc.words = words;
        }
        a.scratch = sc.ptr;
        const uint32_t n = leo_sparse_apply_run(a, (cudaStream_t)stream);
        if (updates) *updates = n;
        cudaSetDevice(previous);
        return 0;
    } catch (const std::exception& e) {
        leo_set_last_error(e.what());
        if (previous >= 0) cudaSetDevice(previous);
        return -1;
    }
}

size_t leo_b200_sparse_apply_scratch_bytes(int device) {
    if (device < 0 || device >= LEO_SPARSE_APPLY_MAX_DEVICES) return 0;
    DeviceScratch& sc = g_scratch[device];
    std::lock_guard<std::mutex> guard(sc.lock);
    return sc.words * sizeof(uint32_t);
}

// The variant of leo_b200_sparse_mean_apply that allocates nothing: its
// scratch is the fixed array above.  Every CUDA call it makes is a device
// selection, an asynchronous memset / copy on the caller's stream, the two
// kernel launches and a stream synchronisation; the first call on a device also
// resolves the array's address with cudaGetSymbolAddress.
int leo_b200_sparse_mean_apply_static(int device, float* target, uint32_t length, const uint32_t* indices,
                                      const float* deltas, const uint64_t* story_offsets, uint32_t stories,
                                      float lo, float hi, float* const* replicas, uint32_t replica_count,
                                      void* stream, uint32_t* updates) {
    int previous = -1;
    try {
        if (device < 0 || device >= LEO_SPARSE_APPLY_MAX_DEVICES) throw ApplyFailure("invalid device ordinal");
        SparseApplyArgs a;
        leo_sparse_apply_prepare(a, target, length, indices, deltas, story_offsets, stories, lo, hi, replicas,
                                 replica_count);
        const size_t words = leo_sparse_apply_scratch_words(length, stories);
        if (words > LEO_SPARSE_APPLY_STATIC_WORDS)
            throw ApplyFailure("input too large for the fixed 1 MiB scratch: stories * (ceil(length / 4096) + 1) must "
                               "not exceed 262080 (use leo_b200_sparse_mean_apply)");
        check(cudaGetDevice(&previous), "cudaGetDevice");
        check(cudaSetDevice(device), "cudaSetDevice");
        a.scratch = static_scratch_address(device);
        const uint32_t n = leo_sparse_apply_run(a, (cudaStream_t)stream);
        if (updates) *updates = n;
        cudaSetDevice(previous);
        return 0;
    } catch (const std::exception& e) {
        leo_set_last_error(e.what());
        if (previous >= 0) cudaSetDevice(previous);
        return -1;
    }
}

}  // extern "C"
