// TEST INFRASTRUCTURE ONLY -- launch harness for the reference's own CUDA
// kernels (crates/leo-core/src/cuda_kernels.cu, compiled unmodified beside this
// file by ./Makefile).  It times the reference's device path for the config-5
// job -- one FP32 tensor's batch-end sparse delta apply followed by the sync of
// the merged values into replica copies -- on device buffers the caller owns:
//   apply: leo_apply_shared_wavefront_deltas (cuda_kernels.cu:6441) over the
//          recurrent-weight tensor: a dense delta array plus its index list,
//          as the reference's story lanes leave them;
//   sync:  leo_scatter_f32 (cuda_kernels.cu:6721) of the merged values into
//          each replica, one launch per replica with the reference's launch
//          shape (ceil(count / 256) blocks of 256, cuda.rs:2883-2908, 7472-7484).
// Only bench.py's reference arm calls it.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

extern "C" __global__ void leo_apply_shared_wavefront_deltas(const unsigned long long* model_pointers,
                                                             const unsigned long long* delta_pointers);
extern "C" __global__ void leo_scatter_f32(float* target, const unsigned int* indices, unsigned int count,
                                           const float* values);

namespace {
thread_local std::string g_error;

struct Failure {
    std::string what;
};

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw Failure{std::string(what) + ": " + cudaGetErrorString(e)};
}

// Values of `target` at `indices`, for the sync's packet.
__global__ void gather_kernel(const float* target, const unsigned int* indices, unsigned int count, float* out) {
    for (unsigned int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x)
        out[i] = target[indices[i]];
}

struct Alloc {
    std::vector<void*> blocks;
    template <typename T>
    T* get(size_t n) {
        void* p = nullptr;
        check(cudaMalloc(&p, n * sizeof(T) > 0 ? n * sizeof(T) : 16), "cudaMalloc");
        check(cudaMemset(p, 0, n * sizeof(T) > 0 ? n * sizeof(T) : 16), "cudaMemset");
        blocks.push_back(p);
        return static_cast<T*>(p);
    }
    ~Alloc() {
        for (void* p : blocks) cudaFree(p);
    }
};
}  // namespace

extern "C" {

const char* leo_ref_last_error(void) { return g_error.c_str(); }

// One apply + sync job, `iters` times.  Device buffers: `base` (length, the
// tensor before the batch), `target` (length; receives base, then the apply),
// `neuron_type` (length / synapses_per_neuron source types), `indices` /
// `deltas` (count: the batch's union indices, ascending, and their merged
// deltas).  `replicas` is a HOST array of `replica_count` device pointers.
// The dense delta array, marks and changed lists are restored before every
// iteration (untimed, as the story lanes would write them); CUDA-event times
// of the apply launch and of the replica scatters are summed into *apply_ms
// and *sync_ms.
int leo_ref_apply_sync(int device, const float* base, float* target, uint32_t length, uint32_t synapses_per_neuron,
                       const unsigned char* neuron_type, const uint32_t* indices, const float* deltas, uint32_t count,
                       float* const* replicas, uint32_t replica_count, float weight_min, float weight_max,
                       uint32_t iters, float* apply_ms, float* sync_ms) {
    try {
        check(cudaSetDevice(device), "cudaSetDevice");
        int sms = 0;
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "sm count");
        Alloc a;
        LeoConfig cfg;
        std::memset(&cfg, 0, sizeof(cfg));
        cfg.synapses_per_neuron = synapses_per_neuron;
        cfg.weight_min = weight_min;
        cfg.weight_max = weight_max;
        cfg.context_embedding_dim = 0;  // no context projection in this job
        LeoConfig* d_cfg = a.get<LeoConfig>(1);
        check(cudaMemcpy(d_cfg, &cfg, sizeof(cfg), cudaMemcpyHostToDevice), "config upload");
        const size_t outputs = 257;
        float* dense = a.get<float>(length);
        unsigned int* dense_marks = a.get<unsigned int>(length);
        unsigned int* changed_marks = a.get<unsigned int>(length);
        unsigned int* changed_list = a.get<unsigned int>(length);
        unsigned int* changed_count = a.get<unsigned int>(1);
        unsigned int* zero_counts = a.get<unsigned int>(8);
        unsigned int* d_count = a.get<unsigned int>(1);
        unsigned int* small_marks = a.get<unsigned int>(outputs);
        unsigned int* small_list = a.get<unsigned int>(outputs);
        float* bias = a.get<float>(outputs);
        float* d_bias = a.get<float>(outputs);
        float* dummy = a.get<float>(outputs);
        float* values = a.get<float>(count);
        check(cudaMemcpy(d_count, &count, 4, cudaMemcpyHostToDevice), "count upload");
        std::vector<unsigned long long> mp(LEO_P_POINTER_COUNT, (unsigned long long)(uintptr_t)dummy);
        mp[LEO_P_CONFIG] = (uintptr_t)d_cfg;
        mp[LEO_P_RECURRENT_WEIGHT] = (uintptr_t)target;
        mp[LEO_P_NEURON_TYPE] = (uintptr_t)neuron_type;
        mp[LEO_P_OUTPUT_BIAS] = (uintptr_t)bias;
        mp[LEO_P_CHANGED_RECURRENT_MARKS] = (uintptr_t)changed_marks;
        mp[LEO_P_CHANGED_RECURRENT_LIST] = (uintptr_t)changed_list;
        mp[LEO_P_CHANGED_RECURRENT_COUNT] = (uintptr_t)changed_count;
        for (int idx : {LEO_P_CHANGED_THRESHOLD_MARKS, LEO_P_CHANGED_INPUT_MARKS, LEO_P_CHANGED_OUTPUT_MARKS,
                        LEO_P_CHANGED_CONTEXT_MARKS})
            mp[idx] = (uintptr_t)small_marks;
        for (int idx : {LEO_P_CHANGED_THRESHOLD_LIST, LEO_P_CHANGED_INPUT_LIST, LEO_P_CHANGED_OUTPUT_LIST,
                        LEO_P_CHANGED_CONTEXT_LIST})
            mp[idx] = (uintptr_t)small_list;
        for (int idx : {LEO_P_CHANGED_THRESHOLD_COUNT, LEO_P_CHANGED_INPUT_COUNT, LEO_P_CHANGED_OUTPUT_COUNT,
                        LEO_P_CHANGED_CONTEXT_COUNT})
            mp[idx] = (uintptr_t)(zero_counts + 4);
        std::vector<unsigned long long> dp(LEO_D_POINTER_COUNT, (unsigned long long)(uintptr_t)dummy);
        dp[LEO_D_RECURRENT] = (uintptr_t)dense;
        dp[LEO_D_RECURRENT_MARKS] = (uintptr_t)dense_marks;
        dp[LEO_D_RECURRENT_LIST] = (uintptr_t)indices;
        dp[LEO_D_RECURRENT_COUNT] = (uintptr_t)d_count;
        for (int idx : {LEO_D_THRESHOLD_COUNT, LEO_D_INPUT_COUNT, LEO_D_OUTPUT_COUNT, LEO_D_CONTEXT_COUNT})
            dp[idx] = (uintptr_t)zero_counts;
        dp[LEO_D_OUTPUT_BIAS] = (uintptr_t)d_bias;
        unsigned long long* d_mp = a.get<unsigned long long>(mp.size());
        unsigned long long* d_dp = a.get<unsigned long long>(dp.size());
        check(cudaMemcpy(d_mp, mp.data(), mp.size() * 8, cudaMemcpyHostToDevice), "model pointers");
        check(cudaMemcpy(d_dp, dp.data(), dp.size() * 8, cudaMemcpyHostToDevice), "delta pointers");
        cudaStream_t s;
        check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream");
        cudaEvent_t e0, e1, e2;
        check(cudaEventCreate(&e0), "event");
        check(cudaEventCreate(&e1), "event");
        check(cudaEventCreate(&e2), "event");
        const unsigned int scatter_blocks = (count + 255u) / 256u;
        float total_apply = 0.0f, total_sync = 0.0f;
        for (uint32_t it = 0; it < iters; ++it) {
            // untimed: the batch's state before the apply
            check(cudaMemcpyAsync(target, base, (size_t)length * 4, cudaMemcpyDeviceToDevice, s), "restore target");
            check(cudaMemsetAsync(changed_marks, 0, (size_t)length * 4, s), "clear marks");
            check(cudaMemsetAsync(changed_count, 0, 4, s), "clear count");
            if (count) leo_scatter_f32<<<scatter_blocks, 256, 0, s>>>(dense, indices, count, deltas);
            check(cudaGetLastError(), "delta restore");
            check(cudaEventRecord(e0, s), "record");
            leo_apply_shared_wavefront_deltas<<<(unsigned)sms * 8u, 256, 0, s>>>(d_mp, d_dp);
            check(cudaGetLastError(), "apply launch");
            check(cudaEventRecord(e1, s), "record");
            if (count) {
                gather_kernel<<<(unsigned)sms * 8u, 256, 0, s>>>(target, indices, count, values);
                check(cudaGetLastError(), "gather launch");
            }
            cudaEvent_t g;
            check(cudaEventCreate(&g), "event");
            check(cudaEventRecord(g, s), "record");
            for (uint32_t r = 0; r < replica_count && count; ++r)
                leo_scatter_f32<<<scatter_blocks, 256, 0, s>>>(replicas[r], indices, count, values);
            check(cudaGetLastError(), "scatter launch");
            check(cudaEventRecord(e2, s), "record");
            check(cudaEventSynchronize(e2), "sync");
            float t_apply = 0.0f, t_sync = 0.0f;
            check(cudaEventElapsedTime(&t_apply, e0, e1), "elapsed");
            check(cudaEventElapsedTime(&t_sync, g, e2), "elapsed");
            cudaEventDestroy(g);
            total_apply += t_apply;
            total_sync += t_sync;
        }
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        cudaEventDestroy(e2);
        cudaStreamDestroy(s);
        *apply_ms = total_apply;
        *sync_ms = total_sync;
        return 0;
    } catch (const Failure& f) {
        g_error = f.what;
        return -1;
    }
}

}  // extern "C"
