// On-device step schedules of a story batch.
//
// The host uploads the batch's story bytes once (one copy: story offsets, then
// the bytes) and this kernel writes every lane's schedule words.  Step 0 reads
// BEGIN_DOCUMENT and predicts byte 0; step s reads byte s - 1 and predicts
// byte s; the last step reads the last byte and predicts END_DOCUMENT
// (the per-story step order of Runtime::train_document,
// crates/leo-core/src/runtime.rs, and leo_build_shared_story_steps,
// crates/leo-core/src/cuda_kernels.cu:4067-4118).  Context dropout, supervised
// strength and the plasticity phase are derived by the wavefront from the
// word, the tick and the configuration, so a word is 4 bytes per step.
//
// Work is one byte read and one word written per step: a few microseconds for
// a batch, bound by launch latency.  The file also holds the lanes' streaming
// zero fill used when a lane's transient state is reset.
#include <stdint.h>

#include "../../include/leo_b200_types.h"
#include "leo_device.cuh"
#include "leo_kernels.h"

namespace {

constexpr uint32_t kThreads = 256;

__global__ void __launch_bounds__(kThreads) build_schedules_kernel(const uint8_t* __restrict__ bytes,
                                                                   const uint64_t* __restrict__ offsets,
                                                                   const LaneState* __restrict__ lanes,
                                                                   uint32_t count, uint32_t permission) {
    for (uint32_t lane = blockIdx.x; lane < count; lane += gridDim.x) {
        const uint64_t begin = offsets[lane];
        const uint64_t length = offsets[lane + 1] - begin;
        if (length == 0) continue;  // an empty story has no steps
        uint32_t* out = const_cast<uint32_t*>(lanes[lane].schedule);
        const uint8_t* story = bytes + begin;
        for (uint64_t s = threadIdx.x; s <= length; s += kThreads) {
            const uint32_t symbol = s == 0 ? LEO_B200_BEGIN_DOCUMENT : story[s - 1];
            const int target = s < length ? (int)story[s] : (int)LEO_B200_END_DOCUMENT;
            out[s] = leo_schedule_word(symbol, target, permission);
        }
    }
}

// Grid-stride zero fill with st.global.cs (streaming: evict-first in L2).
__global__ void __launch_bounds__(kThreads) zero_streaming_kernel(float4* __restrict__ p, size_t n) {
    const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (size_t)gridDim.x * kThreads) __stcs(p + i, z);
}

}  // namespace

cudaError_t leo_launch_zero_streaming(float4* p, size_t n, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    int device = 0, sms = 148;
    cudaGetDevice(&device);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    const size_t want = (n + kThreads - 1) / kThreads;
    const unsigned grid = (unsigned)(want < (size_t)sms * 8 ? want : (size_t)sms * 8);
    zero_streaming_kernel<<<grid, kThreads, 0, stream>>>(p, n);
    return cudaGetLastError();
}

cudaError_t leo_launch_build_schedules(const uint8_t* bytes, const uint64_t* offsets, const LaneState* lanes,
                                       uint32_t count, uint32_t permission, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    const uint32_t grid = count < 1024u ? count : 1024u;
    build_schedules_kernel<<<grid, kThreads, 0, stream>>>(bytes, offsets, lanes, count, permission);
    return cudaGetLastError();
}
