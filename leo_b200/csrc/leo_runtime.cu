// Host runtime behind the leo_b200 C ABI: device buffers, canonical model,
// story lanes, the per-byte step loop, the batch-end merge and serial replay.
//
// This replaces the reference's CUDA host runtime (crates/leo-core/src/cuda.rs,
// train_story_batch_shared_device :8407-9355) behind the same backend
// contract (RuntimeBackend::training_story_batch, backend.rs:457-463).
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <array>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/leo_b200.h"
#include "leo_device.cuh"
#include "leo_host.h"
#include "leo_kernels.h"
#include "libm_tables.inc"

namespace {

thread_local std::string g_error;

struct LeoFailure : std::runtime_error {
    using std::runtime_error::runtime_error;
};

void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw LeoFailure(std::string(what) + ": " + cudaGetErrorString(e));
}
#define CUDA_CHECK(x) check_cuda((x), #x)

struct DevMem {
    void* p = nullptr;
    DevMem() = default;
    DevMem(const DevMem&) = delete;
    DevMem& operator=(const DevMem&) = delete;
    ~DevMem() {
        if (p) cudaFree(p);
    }
};

struct MemPool {
    std::vector<std::unique_ptr<DevMem>> blocks;
    size_t bytes = 0;
    template <typename T>
    T* alloc(size_t count, int fill = 0) {
        auto m = std::make_unique<DevMem>();
        size_t b = std::max<size_t>(count * sizeof(T), 16);
        CUDA_CHECK(cudaMalloc(&m->p, b));
        CUDA_CHECK(cudaMemset(m->p, fill, b));
        // The runtime's stream is non-blocking with respect to the legacy
        // default stream the fill runs on: finish the fill before any use.
        CUDA_CHECK(cudaDeviceSynchronize());
        bytes += b;
        T* out = (T*)m->p;
        blocks.push_back(std::move(m));
        return out;
    }
};

using leo_host::ModelSizes;

struct Lane {
    MemPool mem;
    LaneState st{};
    size_t schedule_capacity = 0;
    uint32_t* schedule = nullptr;
    float* step_loss = nullptr;
    uint32_t* step_active = nullptr;
};

struct ContextRow {
    unsigned long long key;
    uint32_t obs;
    uint32_t pad;
};

}  // namespace

struct LeoB200Device {
    int device = 0;
    cudaStream_t stream = nullptr;
    LeoB200Config cfg{};
    ModelSizes z{};
    KernelConsts kc{};
    int grid = 0;
    MemPool mem;  // topology, canonical, tables, scratch
    LaneParams canon{};
    // Host mirrors of the canonical model's metadata and context tables.
    std::vector<uint8_t> neuron_type;
    std::vector<unsigned long long> ctx_keys;
    std::vector<uint32_t> ctx_obs;
    std::vector<float> ctx_emb;
    uint64_t generation = 0, revision = 0, canonical_tick = 0;
    LeoB200Statistics stats{};
    std::vector<std::unique_ptr<Lane>> lanes;
    std::unique_ptr<Lane> replay;
    LaneState* d_lanes = nullptr;  // device copy of the story lanes' LaneState
    LaneState* d_replay = nullptr;
    uint32_t lane_capacity = 0;
    // context merge staging (one lane's changed rows at a time; the sync slot list)
    ContextRow* ctx_stage_rows = nullptr;
    float* ctx_stage_emb = nullptr;
    uint32_t* ctx_sync_slots = nullptr;
    // merge scratch
    MergeScratch scratch{};
    size_t scratch_len = 0;
    float** d_lane_ptrs = nullptr;       // [max_lanes]
    uint32_t** d_lane_lists = nullptr;   // [max_lanes]
    uint32_t* d_lane_counts = nullptr;   // [max_lanes]
    uint8_t** d_lane_marks = nullptr;    // [max_lanes]
    // in-flight batch
    bool batch_open = false;
    // Trait-level entry points: a single story still runs on a lane (its delta
    // against the canonical model is exported), the exported story deltas, and
    // the canonical runtime's open document.
    bool force_lanes = false;
    struct StoryDelta {
        std::vector<uint32_t> index[LEO_B200_DELTA_TENSORS];
        std::vector<float> delta[LEO_B200_DELTA_TENSORS];
        std::vector<uint32_t> ctx_order, ctx_obs_inc;
        std::vector<unsigned long long> ctx_key;
        std::vector<float> ctx_emb;
        LeoB200Statistics stats{};
        uint64_t revision = 0;
        std::vector<uint32_t> changed[LEO_B200_CHANGE_LISTS];  // the lane's tracked indices, sorted
        uint32_t dirty = 0;                                   // bit 0 output bias, bit 1 context output
    };
    std::vector<StoryDelta> story_deltas;
    bool doc_open = false;
    uint32_t doc_steps = 0;
    uint32_t batch_lanes = 0;
    uint32_t batch_steps = 0;
    uint32_t steps_done = 0;
    int batch_permission = LEO_B200_TRAINING;
    bool single_story = false;
    std::vector<std::vector<uint8_t>> batch_stories;
    // Device keyed context merge: buffers for `ctx_capacity` lane entries
    // (grown on demand; one block of device memory), and whether the
    // configuration fits its per-order shared-memory tables.
    bool ctx_device_merge = false;
    size_t ctx_capacity = 0;
    std::unique_ptr<DevMem> ctx_mem;
    CtxMergeArgs ctx_args{};
    CtxMergeWork ctx_work{};
    uint32_t* ctx_lane_offset = nullptr;  // [max_lanes + 1]
    // The batch's story bytes staged for the on-device schedule builder.
    std::vector<uint8_t> h_stage;
    std::unique_ptr<DevMem> d_stage;
    size_t stage_capacity = 0;
    // sharded batch (multi-GPU data parallelism): this rank's lanes run
    // stories [shard_first, shard_first + batch_lanes) of batch_stories
    bool shard_mode = false;
    uint32_t shard_first = 0;
    bool shard_local_done = false;
    std::vector<LaneScalars> shard_scal;
    std::vector<uint8_t> shard_ctx_blob;       // local stories' keyed context deltas, serialised
    std::vector<uint32_t> shard_ctx_slots;     // local lanes' changed context slots
    uint32_t* shard_list[LEO_B200_FIXED_TENSORS] = {};
    uint32_t shard_count[LEO_B200_FIXED_TENSORS] = {};
    uint32_t* compact_blocks = nullptr;
    uint32_t* compact_total = nullptr;
    uint32_t* shard_error = nullptr;
    std::vector<LaneScalars> host_scalars;
    // performance counters and execution geometry
    LeoB200PerfStats perf{};
    uint32_t story_cluster_request = 0, replay_cluster_request = 0;
    // Adaptive story-pass geometry: per-lane load reported by the kernel, the
    // lane table of one chunk's launches, and streams for concurrent launches.
    int sm_count = 0;
    int fit16 = 0, fit8 = 0, fit4 = 0;  // co-resident clusters of 16 / 8 / 4 CTAs
    int grid_ctas = 0;                  // CTAs of the whole-GPU replay launch (0: unavailable)
    uint32_t replay_load = 0;           // work per step the replay lane reported last
    uint32_t story_chunk = 32;        // steps per story-pass launch while lane loads are skewed
    uint32_t* d_lane_load = nullptr;  // [max_lanes + 1], last entry: replay lane
    LaneState* d_group_table = nullptr;
    std::vector<uint32_t> lane_steps;
    // Per-target event segments (see DeviceTopology) and the settle tiers.
    uint32_t cta_min_in_degree = 0;   // listed for the CTA tier from this in-degree (0: default, see plan_segments)
    uint32_t cta_events = 256;        // a listed target with more events than this per step is sorted by a CTA
    uint32_t thread_events = 16;      // at most this many: one thread; otherwise one warp
    uint64_t seg_events_total = 0;    // sum of segment capacities (entries per lane)
    uint32_t seg_capacity_limit = 0;  // diagnostic cap on every segment (0: the exact bound)
    std::vector<uint2> seg_host;      // the plan, to detect a changed topology
    cudaStream_t aux[4] = {nullptr, nullptr, nullptr, nullptr};
    cudaEvent_t fork = nullptr, join[4] = {nullptr, nullptr, nullptr, nullptr};
    cudaEvent_t batch_start = nullptr, batch_stop = nullptr;
    cudaEvent_t wave_start = nullptr, wave_stop = nullptr;
};

namespace {

// Wall milliseconds since `t0`; the batch-end steps it times each end with a
// stream synchronize.
double ms_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

int fail(const std::exception& e) {
    g_error = e.what();
    return -1;
}

uint32_t schedule_word(uint32_t symbol, int target, int permission) {
    return leo_schedule_word(symbol, target, (uint32_t)permission);
}

KernelConsts make_consts(LeoB200Device& dev) {
    KernelConsts kc{};
    kc.cfg = dev.cfg.abi;
    kc.strength[LEO_B200_FROZEN] = 0.0f;
    kc.strength[LEO_B200_PROVISIONAL] = dev.cfg.host.provisional_strength;
    kc.strength[LEO_B200_TRAINING] = dev.cfg.host.training_strength;
    kc.strength[LEO_B200_VERIFIED] = dev.cfg.host.verified_strength;
    kc.end_document_weight = dev.cfg.host.end_document_weight;
    kc.plasticity_window = dev.cfg.host.plasticity_window;
    kc.dropout_rate = dev.cfg.host.context_dropout_rate;
    kc.seed = dev.cfg.host.seed;
    kc.track_changes = 1;
    return kc;
}

// Per-lane event segments for the current plan.
void allocate_lane_segments(LeoB200Device& dev, Lane& lane) {
    LaneState& st = lane.st;
    st.seg_count = lane.mem.alloc<uint32_t>(dev.z.n);
    st.seg_events = lane.mem.alloc<uint32_t>(std::max<uint64_t>(dev.seg_events_total, 1));
}

void allocate_lane_transient(LeoB200Device& dev, Lane& lane) {
    const ModelSizes& z = dev.z;
    MemPool& m = lane.mem;
    LaneState& st = lane.st;
    st.canon_out_weight = dev.canon.out_weight;
    uint32_t maxa = dev.cfg.abi.max_active_global, B = dev.cfg.abi.block_count, npb = dev.cfg.abi.neurons_per_block;
    st.sc = m.alloc<LaneScalars>(1);
    st.hot = m.alloc<NeuronHot>(z.n);
    st.cold = m.alloc<NeuronCold>(z.n);
    st.branches = m.alloc<float4>(z.n);
    st.touch_epoch = m.alloc<uint32_t>(z.n);
    st.touched = m.alloc<uint32_t>(z.n);
    st.block_cand = m.alloc<unsigned long long>((size_t)B * npb);
    st.block_cand_count = m.alloc<uint32_t>(B);
    st.block_cutoff = m.alloc<float>(B);
    st.block_winners = m.alloc<unsigned long long>((size_t)B * dev.cfg.abi.max_active_per_block);
    st.block_nwin = m.alloc<uint32_t>(B);
    st.ring_src = m.alloc<uint32_t>((size_t)LEO_RING * maxa);
    st.ring_act = m.alloc<float>((size_t)LEO_RING * maxa);
    st.ring_val = m.alloc<float>((size_t)LEO_RING * maxa * z.s);
    st.ev_val = m.alloc<float>(dev.kc.event_capacity);
    for (int i = 0; i < 2; ++i) {
        st.elig[i] = m.alloc<uint2>(z.synapses);
        st.in_elig[i] = m.alloc<uint2>(z.inputs);
    }
    st.traces = m.alloc<Trace>(z.synapses);
    st.in_traces = m.alloc<Trace>(z.inputs);
    st.dst_list = m.alloc<uint32_t>(z.n);
    st.dst_epoch = m.alloc<uint32_t>(z.n);
    st.signal = m.alloc<float>(z.n);
    st.errors = m.alloc<float>(LEO_OUTPUT_STRIDE);
    st.probs = m.alloc<float>(LEO_OUTPUT_STRIDE);
    st.thr_mark = m.alloc<uint8_t>((z.n + 3) & ~(size_t)3);
    st.thr_list = m.alloc<uint32_t>(z.n);
    st.rec_mark = m.alloc<uint8_t>((z.synapses + 3) & ~(size_t)3);
    st.rec_list = m.alloc<uint32_t>(z.synapses);
    st.in_mark = m.alloc<uint8_t>((z.inputs + 3) & ~(size_t)3);
    st.in_list = m.alloc<uint32_t>(z.inputs);
    st.out_mark = m.alloc<uint8_t>((z.n + 3) & ~(size_t)3);
    st.out_list = m.alloc<uint32_t>(z.n);
    st.ctx_mark = m.alloc<uint8_t>((z.ctx + 3) & ~(size_t)3);
    st.ctx_list = m.alloc<uint32_t>(z.ctx);
    allocate_lane_segments(dev, lane);
}

void allocate_lane_params(LeoB200Device& dev, Lane& lane) {
    const ModelSizes& z = dev.z;
    MemPool& m = lane.mem;
    LaneParams& p = lane.st.p;
    p.threshold = m.alloc<float>(z.n);
    p.rec_weight = m.alloc<float>(z.synapses);
    p.in_weight = m.alloc<float>(z.inputs);
    p.out_weight = m.alloc<float>(z.n * LEO_OUTPUT_STRIDE);
    p.out_bias = m.alloc<float>(LEO_OUTPUT_STRIDE);
    p.ctx_keys = m.alloc<unsigned long long>(z.ctx);
    p.ctx_obs = m.alloc<uint32_t>(z.ctx);
    p.ctx_emb = m.alloc<float>(z.ctx_emb);
    p.ctx_out = m.alloc<float>(z.ctx_out);
}

void copy_params(LeoB200Device& dev, const LaneParams& dst, const LaneParams& src) {
    const ModelSizes& z = dev.z;
    cudaStream_t s = dev.stream;
    CUDA_CHECK(cudaMemcpyAsync(dst.threshold, src.threshold, z.n * 4, cudaMemcpyDeviceToDevice, s));
    CUDA_CHECK(cudaMemcpyAsync(dst.rec_weight, src.rec_weight, z.synapses * 4, cudaMemcpyDeviceToDevice, s));
    CUDA_CHECK(cudaMemcpyAsync(dst.in_weight, src.in_weight, z.inputs * 4, cudaMemcpyDeviceToDevice, s));
    CUDA_CHECK(cudaMemcpyAsync(dst.out_weight, src.out_weight, z.n * LEO_OUTPUT_STRIDE * 4, cudaMemcpyDeviceToDevice, s));
    CUDA_CHECK(cudaMemcpyAsync(dst.out_bias, src.out_bias, LEO_OUTPUT_STRIDE * 4, cudaMemcpyDeviceToDevice, s));
    CUDA_CHECK(cudaMemcpyAsync(dst.ctx_keys, src.ctx_keys, z.ctx * 8, cudaMemcpyDeviceToDevice, s));
    CUDA_CHECK(cudaMemcpyAsync(dst.ctx_obs, src.ctx_obs, z.ctx * 4, cudaMemcpyDeviceToDevice, s));
    CUDA_CHECK(cudaMemcpyAsync(dst.ctx_emb, src.ctx_emb, z.ctx_emb * 4, cudaMemcpyDeviceToDevice, s));
    CUDA_CHECK(cudaMemcpyAsync(dst.ctx_out, src.ctx_out, z.ctx_out * 4, cudaMemcpyDeviceToDevice, s));
}

// Transient reset of one lane (runtime.rs:375-435) for a document starting
// at absolute tick `base_tick`, with per-lane statistics starting from the
// canonical values (parallel.rs:1115-1137 subtracts them back out).
void reset_lane(LeoB200Device& dev, Lane& lane, unsigned long long base_tick, uint32_t steps) {
    const ModelSizes& z = dev.z;
    cudaStream_t s = dev.stream;
    LaneState& st = lane.st;
    // The traces (32 B per synapse: 134 MB on a 65,536 x 64 model) are zeroed
    // first and with evict-first stores, so that zeroing them does not push the
    // lane's neuron state and the topology the next steps read out of L2.
    CUDA_CHECK(leo_launch_zero_streaming(reinterpret_cast<float4*>(st.traces), z.synapses * sizeof(Trace) / 16, s));
    CUDA_CHECK(leo_launch_zero_streaming(reinterpret_cast<float4*>(st.in_traces), z.inputs * sizeof(Trace) / 16, s));
    dev.perf.launches += 2;
    CUDA_CHECK(cudaMemsetAsync(st.hot, 0, z.n * sizeof(NeuronHot), s));
    CUDA_CHECK(cudaMemsetAsync(st.cold, 0, z.n * sizeof(NeuronCold), s));
    CUDA_CHECK(cudaMemsetAsync(st.branches, 0, z.n * sizeof(float4), s));
    CUDA_CHECK(cudaMemsetAsync(st.touch_epoch, 0, z.n * 4, s));
    CUDA_CHECK(cudaMemsetAsync(st.dst_epoch, 0, z.n * 4, s));
    CUDA_CHECK(cudaMemsetAsync(st.seg_count, 0, z.n * 4, s));
    CUDA_CHECK(cudaMemsetAsync(st.block_cand_count, 0, dev.cfg.abi.block_count * 4, s));
    LaneScalars sc{};
    sc.base_tick = base_tick;
    sc.steps = steps;
    sc.loss_sum = dev.stats.training_loss_sum;
    sc.active_peak = dev.stats.active_neurons_peak;
    CUDA_CHECK(cudaMemcpyAsync(st.sc, &sc, sizeof(sc), cudaMemcpyHostToDevice, s));
}

void ensure_schedule(Lane& lane, size_t steps) {
    if (lane.schedule_capacity >= steps) return;
    size_t cap = std::max<size_t>(steps, 4096);
    lane.schedule = lane.mem.alloc<uint32_t>(cap);
    lane.step_loss = lane.mem.alloc<float>(cap);
    lane.step_active = lane.mem.alloc<uint32_t>(cap);
    lane.schedule_capacity = cap;
    lane.st.schedule = lane.schedule;
    lane.st.step_loss = lane.step_loss;
    lane.st.step_active = lane.step_active;
}

void ensure_lanes(LeoB200Device& dev, uint32_t count) {
    if (count > dev.lane_capacity) throw LeoFailure("story batch exceeds the lanes reserved at open");
    while (dev.lanes.size() < count) {
        auto lane = std::make_unique<Lane>();
        allocate_lane_params(dev, *lane);
        allocate_lane_transient(dev, *lane);
        lane->st.load_out = dev.d_lane_load + dev.lanes.size();
        copy_params(dev, lane->st.p, dev.canon);
        dev.lanes.push_back(std::move(lane));
    }
}

// Uploads every resident lane's LaneState; a batch of L stories uses the first L.
void upload_lane_table(LeoB200Device& dev) {
    uint32_t count = (uint32_t)dev.lanes.size();
    std::vector<LaneState> table(count);
    for (uint32_t i = 0; i < count; ++i) table[i] = dev.lanes[i]->st;
    if (count)
        CUDA_CHECK(cudaMemcpyAsync(dev.d_lanes, table.data(), count * sizeof(LaneState), cudaMemcpyHostToDevice, dev.stream));
    CUDA_CHECK(cudaMemcpyAsync(dev.d_replay, &dev.replay->st, sizeof(LaneState), cudaMemcpyHostToDevice, dev.stream));
}

// ---------------------------------------------------------------- event segments
// Every target owns a segment of each lane's seg_events sized for the most
// events it can receive in one step: a recurrent slot delivers at most once
// per step, and in each of the four delay classes at most max_active_global
// sources fire, each with at most mult(n) slots to n -- so at most
// min(in-degree, 4 x max_active_global x mult(n)) recurrent events -- plus the
// most input slots one symbol has to n.  Targets whose recurrent in-degree is
// at least the threshold are listed in descending capacity, and CTA r of a
// lane settles listed targets r, r + C, ... whatever their count, which
// spreads the high in-degree targets (the ones with many events per step)
// evenly over the lane's CTAs; every other target is settled where the
// touched list puts it.  The default threshold is the in-degree at which
// max_active_global / N of the sources, firing, would deliver thread_events / 4
// events (power-law hubs; none on uniform topologies).
std::vector<uint2> plan_segments(LeoB200Device& dev, const uint32_t* recurrent_target, const uint32_t* input_target,
                                 bool upload) {
    const ModelSizes& z = dev.z;
    const uint32_t N = (uint32_t)z.n, S = (uint32_t)z.s, F = (uint32_t)z.f;
    const uint32_t maxa = dev.cfg.abi.max_active_global;
    uint64_t threshold = dev.cta_min_in_degree;
    if (threshold == 0)
        threshold = std::max<uint64_t>(1, ((uint64_t)dev.thread_events * N + 4ull * maxa - 1) / (4ull * maxa));
    std::vector<uint32_t> degree(N, 0), mult(N, 0), in_max(N, 0);
    std::vector<uint32_t> row(S);
    for (uint32_t src = 0; src < N; ++src) {
        for (uint32_t j = 0; j < S; ++j) row[j] = recurrent_target[(size_t)src * S + j];
        std::sort(row.begin(), row.end());
        for (uint32_t j = 0; j < S;) {
            uint32_t e = j;
            while (e < S && row[e] == row[j]) ++e;
            degree[row[j]] += e - j;
            mult[row[j]] = std::max(mult[row[j]], e - j);
            j = e;
        }
    }
    std::vector<uint32_t> in_row(F);
    for (uint32_t sym = 0; sym < LEO_B200_SYMBOL_COUNT; ++sym) {
        for (uint32_t f = 0; f < F; ++f) in_row[f] = input_target[(size_t)sym * F + f];
        std::sort(in_row.begin(), in_row.end());
        for (uint32_t f = 0; f < F;) {
            uint32_t e = f;
            while (e < F && in_row[e] == in_row[f]) ++e;
            in_max[in_row[f]] = std::max(in_max[in_row[f]], e - f);
            f = e;
        }
    }
    std::vector<uint2> seg(N);
    std::vector<std::pair<uint64_t, uint32_t>> listed;
    uint64_t total = 0;
    for (uint32_t n = 0; n < N; ++n) {
        uint64_t cap = std::min<uint64_t>(degree[n], 4ull * maxa * mult[n]) + in_max[n];
        if (dev.seg_capacity_limit) cap = std::min<uint64_t>(cap, dev.seg_capacity_limit);
        // Every segment sorts in shared memory (32,768 keys): the device limits
        // (max_active_global <= 1024, four branches) keep capacities below that.
        if (cap > 32768) throw LeoFailure("a target's events per step exceed the settle sort (32768)");
        seg[n] = make_uint2((uint32_t)total, (uint32_t)cap);
        if (degree[n] >= threshold && cap > 0) {
            seg[n].y |= LEO_SEG_LISTED;
            listed.push_back({cap, n});
        }
        total += cap;
        if (total >= 0xffffffffull) throw LeoFailure("event segment capacity exceeds 32-bit offsets");
    }
    std::sort(listed.begin(), listed.end(), [](const auto& a, const auto& b) {
        return a.first != b.first ? a.first > b.first : a.second < b.second;
    });
    if (!upload) return seg;
    DeviceTopology& t = dev.kc.topo;
    t.cta_count = (uint32_t)listed.size();
    t.cta_events = dev.cta_events;
    t.thread_events = std::min(dev.thread_events, dev.cta_events);
    dev.seg_events_total = total;
    dev.seg_host = seg;
    std::vector<uint32_t> targets(listed.size());
    for (size_t i = 0; i < listed.size(); ++i) targets[i] = listed[i].second;
    uint2* d_seg = t.seg ? const_cast<uint2*>(t.seg) : dev.mem.alloc<uint2>(N);
    CUDA_CHECK(cudaMemcpy(d_seg, seg.data(), N * sizeof(uint2), cudaMemcpyHostToDevice));
    t.seg = d_seg;
    uint32_t* d_targets = dev.mem.alloc<uint32_t>(std::max<size_t>(targets.size(), 1));
    if (!targets.empty())
        CUDA_CHECK(cudaMemcpy(d_targets, targets.data(), targets.size() * 4, cudaMemcpyHostToDevice));
    t.cta_targets = d_targets;
    return seg;
}

// ---------------------------------------------------------------- model I/O
void upload_model(LeoB200Device& dev, const LeoB200HostModel& m) {
    const ModelSizes& z = dev.z;
    std::vector<uint32_t> rec_word(z.synapses), in_word(z.inputs);
    for (size_t i = 0; i < z.synapses; ++i)
        rec_word[i] = m.recurrent_target[i] | ((uint32_t)m.recurrent_branch[i] << 24) | ((uint32_t)m.recurrent_delay[i] << 26);
    for (size_t i = 0; i < z.inputs; ++i) in_word[i] = m.input_target[i] | ((uint32_t)m.input_branch[i] << 24);
    CUDA_CHECK(cudaMemcpy((void*)dev.kc.topo.rec_word, rec_word.data(), z.synapses * 4, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy((void*)dev.kc.topo.in_word, in_word.data(), z.inputs * 4, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy((void*)dev.kc.topo.neuron_type, m.neuron_type, z.n, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy((void*)dev.kc.topo.excitability, m.excitability, z.n * 4, cudaMemcpyHostToDevice));
    dev.neuron_type.assign(m.neuron_type, m.neuron_type + z.n);
    LaneParams& p = dev.canon;
    CUDA_CHECK(cudaMemcpy(p.threshold, m.threshold, z.n * 4, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(p.rec_weight, m.recurrent_weight, z.synapses * 4, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(p.in_weight, m.input_weight, z.inputs * 4, cudaMemcpyHostToDevice));
    std::vector<float> rows(z.n * LEO_OUTPUT_STRIDE, 0.0f);
    for (size_t o = 0; o < LEO_OUTPUT_CLASSES; ++o)
        for (size_t n = 0; n < z.n; ++n) rows[n * LEO_OUTPUT_STRIDE + o] = m.output_weight[o * z.n + n];
    CUDA_CHECK(cudaMemcpy(p.out_weight, rows.data(), rows.size() * 4, cudaMemcpyHostToDevice));
    std::vector<float> bias(LEO_OUTPUT_STRIDE, 0.0f);
    std::memcpy(bias.data(), m.output_bias, LEO_OUTPUT_CLASSES * 4);
    CUDA_CHECK(cudaMemcpy(p.out_bias, bias.data(), LEO_OUTPUT_STRIDE * 4, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(p.ctx_keys, m.context_keys, z.ctx * 8, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(p.ctx_obs, m.context_observations, z.ctx * 4, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(p.ctx_emb, m.context_embeddings, z.ctx_emb * 4, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(p.ctx_out, m.context_output_weight, z.ctx_out * 4, cudaMemcpyHostToDevice));
    dev.ctx_keys.assign(m.context_keys, m.context_keys + z.ctx);
    dev.ctx_obs.assign(m.context_observations, m.context_observations + z.ctx);
    dev.ctx_emb.assign(m.context_embeddings, m.context_embeddings + z.ctx_emb);
    dev.generation = m.generation;
    dev.revision = m.parameter_revision;
    dev.stats = m.statistics;
    for (auto& lane : dev.lanes) copy_params(dev, lane->st.p, dev.canon);
    CUDA_CHECK(cudaStreamSynchronize(dev.stream));
}

void download_params(LeoB200Device& dev, const LaneParams& p, LeoB200HostModel& m) {
    const ModelSizes& z = dev.z;
    CUDA_CHECK(cudaStreamSynchronize(dev.stream));
    CUDA_CHECK(cudaMemcpy(m.threshold, p.threshold, z.n * 4, cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaMemcpy(m.recurrent_weight, p.rec_weight, z.synapses * 4, cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaMemcpy(m.input_weight, p.in_weight, z.inputs * 4, cudaMemcpyDeviceToHost));
    std::vector<float> rows(z.n * LEO_OUTPUT_STRIDE);
    CUDA_CHECK(cudaMemcpy(rows.data(), p.out_weight, rows.size() * 4, cudaMemcpyDeviceToHost));
    for (size_t o = 0; o < LEO_OUTPUT_CLASSES; ++o)
        for (size_t n = 0; n < z.n; ++n) m.output_weight[o * z.n + n] = rows[n * LEO_OUTPUT_STRIDE + o];
    CUDA_CHECK(cudaMemcpy(m.output_bias, p.out_bias, LEO_OUTPUT_CLASSES * 4, cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaMemcpy(m.context_keys, p.ctx_keys, z.ctx * 8, cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaMemcpy(m.context_observations, p.ctx_obs, z.ctx * 4, cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaMemcpy(m.context_embeddings, p.ctx_emb, z.ctx_emb * 4, cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaMemcpy(m.context_output_weight, p.ctx_out, z.ctx_out * 4, cudaMemcpyDeviceToHost));
    // Topology is immutable on the device; it is returned from the host copy.
    std::vector<uint32_t> rec_word(z.synapses), in_word(z.inputs);
    CUDA_CHECK(cudaMemcpy(rec_word.data(), dev.kc.topo.rec_word, z.synapses * 4, cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaMemcpy(in_word.data(), dev.kc.topo.in_word, z.inputs * 4, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < z.synapses; ++i) {
        m.recurrent_target[i] = rec_word[i] & LEO_TARGET_MASK;
        m.recurrent_branch[i] = (uint8_t)LEO_WORD_BRANCH(rec_word[i]);
        m.recurrent_delay[i] = (uint8_t)LEO_WORD_DELAY(rec_word[i]);
    }
    for (size_t i = 0; i < z.inputs; ++i) {
        m.input_target[i] = in_word[i] & LEO_TARGET_MASK;
        m.input_branch[i] = (uint8_t)LEO_WORD_BRANCH(in_word[i]);
    }
    std::memcpy(m.neuron_type, dev.neuron_type.data(), z.n);
    CUDA_CHECK(cudaMemcpy(m.excitability, dev.kc.topo.excitability, z.n * 4, cudaMemcpyDeviceToHost));
    m.config = dev.cfg;
}

// ---------------------------------------------------------------- stepping
// Picks the cluster size for `lanes` concurrent lanes: the requested size,
// else the largest size (<= 16) whose clusters can all be resident at once.
uint32_t pick_cluster(LeoB200Device& dev, uint32_t lanes, uint32_t request, uint32_t limit) {
    if (request) return request;
    for (uint32_t c = limit; c >= 1; c >>= 1) {
        int fit = 0;
        if (leo_wavefront_max_clusters(c, dev.kc, &fit) != cudaSuccess) {
            cudaGetLastError();  // this size is not supported here; try a smaller one
            continue;
        }
        if ((uint32_t)fit >= lanes) return c;
    }
    return 1;
}

// Runs steps [begin, end) of every lane in `d_lanes` with one persistent
// wavefront launch, timed with CUDA events on the backend's stream.
// Replay steps whose reported work per step is above this use the whole GPU
// (one CTA per SM, grid barriers) instead of one 16-CTA cluster: a grid
// barrier costs a few microseconds more, which pays off once a step moves
// more than ~50k units of work (fitted to measured replay steps).
constexpr uint32_t kWholeGpuLoad = 50000;

void run_steps(LeoB200Device& dev, const LaneState* d_lanes, int lane_count, uint32_t begin, uint32_t end,
               bool story) {
    if (end <= begin || lane_count == 0) return;
    const uint32_t first = begin;
    const bool whole_gpu = !story && lane_count == 1 && dev.grid_ctas > 0 &&
                           (dev.replay_cluster_request == LEO_B200_WHOLE_GPU ||
                            (dev.replay_cluster_request == 0 && dev.replay_load > kWholeGpuLoad));
    uint32_t cluster = 0;
    if (!whole_gpu)
        cluster = story ? pick_cluster(dev, (uint32_t)lane_count, dev.story_cluster_request, 16)
                        : pick_cluster(dev, 1, dev.replay_cluster_request == LEO_B200_WHOLE_GPU
                                                   ? 0u : dev.replay_cluster_request, 16);
    CUDA_CHECK(cudaEventRecord(dev.wave_start, dev.stream));
    if (whole_gpu)
        CUDA_CHECK(leo_launch_wavefront_grid(d_lanes, (uint32_t)dev.grid_ctas, first, end, dev.kc, dev.stream));
    else
        CUDA_CHECK(leo_launch_wavefront(d_lanes, lane_count, cluster, first, end, dev.kc, dev.stream));
    CUDA_CHECK(cudaGetLastError());
    CUDA_CHECK(cudaEventRecord(dev.wave_stop, dev.stream));
    CUDA_CHECK(cudaEventSynchronize(dev.wave_stop));
    float ms = 0.0f;
    CUDA_CHECK(cudaEventElapsedTime(&ms, dev.wave_start, dev.wave_stop));
    dev.perf.launches += 1;
    dev.perf.wavefront_launches += 1;
    dev.perf.wavefront_ms += ms;
    if (story) {
        dev.perf.story_wavefront_launches += 1;
        dev.perf.story_wavefront_ms += ms;
        dev.perf.story_cluster = cluster;
    } else {
        dev.perf.replay_cluster = whole_gpu ? (uint32_t)dev.grid_ctas : cluster;
        if (whole_gpu) dev.perf.whole_gpu_launches += 1;
        if (lane_count == 1)
            CUDA_CHECK(cudaMemcpy(&dev.replay_load, dev.d_lane_load + dev.lane_capacity, 4, cudaMemcpyDeviceToHost));
    }
}

// Cluster sizes for one chunk of the story pass.  Model of a lane's time per
// step with c CTAs (fitted to measured lanes of config 2): 50 us of latency
// plus 0.01 us per unit of reported load, divided by c^0.8.  Starting from one
// CTA per lane, the lane with the largest modelled time doubles its cluster
// (up to 16) while the sizes still pack: clusters of 4 or more CTAs occupy
// whole 4-SM units of one GPC (fit4 such units co-reside), at most fit8 / fit16
// clusters of 8 / 16, and 1- or 2-CTA clusters fill the SMs outside the units
// and any unused units.  The chunk's time is its slowest lane, so the greedy
// stops when that lane cannot grow.  Results do not depend on the sizes.
double modelled_step_us(uint32_t load, uint32_t c) { return 50.0 + 0.01 * (double)load / std::pow((double)c, 0.8); }

bool sizes_pack(const LeoB200Device& dev, const int n[5]) {
    if (n[4] > dev.fit16 || n[3] + 2 * n[4] > dev.fit8) return false;
    const int units = n[2] + 2 * n[3] + 4 * n[4];
    const int small = n[0] + 2 * n[1];
    const int outside = std::max(0, dev.sm_count - 4 * dev.fit4);
    return units + (std::max(0, small - outside) + 3) / 4 <= dev.fit4;
}

std::vector<uint32_t> assign_clusters(const LeoB200Device& dev, const std::vector<uint32_t>& lanes,
                                      const std::vector<uint32_t>& load) {
    std::vector<uint32_t> c(lanes.size(), 1u);
    std::vector<bool> settled(lanes.size(), false);  // at 16 CTAs, or no longer packable
    int n[5] = {(int)lanes.size(), 0, 0, 0, 0};
    if (!sizes_pack(dev, n)) return c;
    for (;;) {
        size_t worst = lanes.size();
        double worst_t = -1.0;
        for (size_t i = 0; i < lanes.size(); ++i) {
            if (settled[i]) continue;
            const double t = modelled_step_us(load[lanes[i]], c[i]);
            if (t > worst_t) {
                worst_t = t;
                worst = i;
            }
        }
        if (worst == lanes.size()) break;
        const int k = __builtin_ctz(c[worst]);
        n[k] -= 1;
        n[k + 1] += 1;
        if (!sizes_pack(dev, n)) {
            // The slowest growable lane cannot grow: stop here, so that a
            // smaller lane never takes the units the slower one needs next.
            n[k] += 1;
            n[k + 1] -= 1;
            break;
        }
        c[worst] *= 2u;
        if (c[worst] == 16u) settled[worst] = true;
    }
    return c;
}

// The story pass in chunks of `story_chunk` steps; each chunk launches one
// wavefront per cluster size in use (concurrently, on separate streams) over
// the lanes that still have steps, sized from the loads the previous chunk
// reported.
void run_story_adaptive(LeoB200Device& dev, int lane_count, uint32_t begin, uint32_t end) {
    std::vector<uint32_t> load(lane_count, 1u), reported(lane_count, 0u);
    CUDA_CHECK(cudaEventRecord(dev.wave_start, dev.stream));
    uint32_t largest = 0;
    uint32_t chunk = std::max(dev.story_chunk, 1u);
    for (uint32_t s = begin; s < end;) {
        const uint32_t e = std::min(end, s + chunk);
        std::vector<uint32_t> act;
        for (int l = 0; l < lane_count; ++l)
            if (dev.lane_steps[l] > s) act.push_back((uint32_t)l);
        if (act.empty()) break;
        const std::vector<uint32_t> c = assign_clusters(dev, act, load);
        std::vector<LaneState> table;
        std::vector<std::pair<uint32_t, uint32_t>> groups;  // (cluster size, lanes)
        for (uint32_t size = 16; size >= 1; size >>= 1) {
            uint32_t count = 0;
            for (size_t i = 0; i < act.size(); ++i)
                if (c[i] == size) {
                    table.push_back(dev.lanes[act[i]]->st);
                    ++count;
                }
            dev.perf.story_lane_launches[__builtin_ctz(size)] += count;
            if (count) groups.push_back({size, count});
            largest = std::max(largest, count ? size : 0u);
        }
        CUDA_CHECK(cudaMemcpyAsync(dev.d_group_table, table.data(), table.size() * sizeof(LaneState),
                                   cudaMemcpyHostToDevice, dev.stream));
        CUDA_CHECK(cudaEventRecord(dev.fork, dev.stream));
        size_t offset = 0;
        for (size_t g = 0; g < groups.size(); ++g) {
            cudaStream_t st = g == 0 ? dev.stream : dev.aux[g - 1];
            if (g > 0) CUDA_CHECK(cudaStreamWaitEvent(st, dev.fork, 0));
            CUDA_CHECK(leo_launch_wavefront(dev.d_group_table + offset, (int)groups[g].second, groups[g].first, s, e,
                                            dev.kc, st));
            CUDA_CHECK(cudaGetLastError());
            if (g > 0) CUDA_CHECK(cudaEventRecord(dev.join[g - 1], st));
            offset += groups[g].second;
            dev.perf.launches += 1;
            dev.perf.wavefront_launches += 1;
            dev.perf.story_wavefront_launches += 1;
        }
        for (size_t g = 1; g < groups.size(); ++g) CUDA_CHECK(cudaStreamWaitEvent(dev.stream, dev.join[g - 1], 0));
        CUDA_CHECK(cudaMemcpyAsync(reported.data(), dev.d_lane_load, lane_count * sizeof(uint32_t),
                                   cudaMemcpyDeviceToHost, dev.stream));
        CUDA_CHECK(cudaStreamSynchronize(dev.stream));
        for (int l = 0; l < lane_count; ++l) load[l] = std::max(reported[l], 1u);
        s = e;
        // Lanes of similar load gain nothing from re-division, and every chunk
        // boundary makes each lane wait for the chunk's slowest: use chunks four
        // times longer until some lane's load is three times the median.
        std::vector<uint32_t> live;
        for (int l = 0; l < lane_count; ++l)
            if (dev.lane_steps[l] > s) live.push_back(load[l]);
        if (!live.empty()) {
            std::sort(live.begin(), live.end());
            const bool skewed = (double)live.back() > 3.0 * (double)live[live.size() / 2];
            chunk = std::max(dev.story_chunk, 1u) * (skewed ? 1u : 4u);
        }
    }
    CUDA_CHECK(cudaEventRecord(dev.wave_stop, dev.stream));
    CUDA_CHECK(cudaEventSynchronize(dev.wave_stop));
    float ms = 0.0f;
    CUDA_CHECK(cudaEventElapsedTime(&ms, dev.wave_start, dev.wave_stop));
    dev.perf.wavefront_ms += ms;
    dev.perf.story_wavefront_ms += ms;
    dev.perf.story_cluster = largest;
}

void add_work(LeoB200Device& dev, const LaneScalars& sc, bool story) {
    for (int p = 0; p < LEO_PHASES; ++p) dev.perf.phase_cycles[p] += sc.phase_cycles[p];
    if (story) dev.perf.story_work_steps += sc.work_steps;
    dev.perf.work_deliver += sc.work_deliver;
    dev.perf.work_touched += sc.work_touched;
    dev.perf.work_eligible += sc.work_eligible;
    dev.perf.work_destinations += sc.work_destinations;
    dev.perf.work_active += sc.work_active;
    dev.perf.work_plastic += sc.work_plastic;
    dev.perf.work_steps += sc.work_steps;
    if (!story) {
        for (int p = 0; p < LEO_PHASES; ++p) dev.perf.replay_phase_cycles[p] += sc.phase_cycles[p];
        dev.perf.replay_work_steps += sc.work_steps;
        dev.perf.replay_work_touched += sc.work_touched;
        dev.perf.replay_work_active += sc.work_active;
        dev.perf.replay_work_deliver += sc.work_deliver;
        dev.perf.replay_work_eligible += sc.work_eligible;
    }
    dev.perf.work_inhibit += sc.work_inhibit;
    dev.perf.work_winners += sc.work_winners;
}

void read_scalars(LeoB200Device& dev, Lane& lane, LaneScalars& out) {
    CUDA_CHECK(cudaMemcpyAsync(&out, lane.st.sc, sizeof(LaneScalars), cudaMemcpyDeviceToHost, dev.stream));
    CUDA_CHECK(cudaStreamSynchronize(dev.stream));
}

void check_error_flag(const LaneScalars& sc) {
    if (sc.error_flag & (LEO_ERR_NONFINITE_RECURRENT)) throw LeoFailure("non-finite recurrent update rejected");
    if (sc.error_flag & LEO_ERR_NONFINITE_INPUT) throw LeoFailure("non-finite input update rejected");
    if (sc.error_flag & LEO_ERR_NONFINITE_INHIBITORY) throw LeoFailure("non-finite inhibitory update rejected");
    if (sc.error_flag & LEO_ERR_NONFINITE_BIAS) throw LeoFailure("output bias became non-finite");
    if (sc.error_flag & LEO_ERR_NONFINITE_CONTEXT) throw LeoFailure("non-finite context update rejected");
    if (sc.error_flag & LEO_ERR_CAPACITY) throw LeoFailure("a step's events exceeded a device event capacity");
    if (sc.error_flag) throw LeoFailure("device step reported an error");
}

// ---------------------------------------------------------------- context merge (host, parallel.rs:1024-1113)
__global__ void gather_context_rows_kernel(const uint32_t* __restrict__ slots, uint32_t count,
                                           const unsigned long long* __restrict__ keys, const uint32_t* __restrict__ obs,
                                           const float* __restrict__ emb, uint32_t d, ContextRow* rows, float* out_emb) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
        uint32_t slot = slots[i];
        rows[i].key = keys[slot];
        rows[i].obs = obs[slot];
        for (uint32_t k = 0; k < d; ++k) out_emb[(size_t)i * d + k] = emb[(size_t)slot * d + k];
    }
}

// Writes staged context rows (key, observations, embedding) at their slots
// into the canonical tables and every resident lane.
__global__ void scatter_context_rows_kernel(const uint32_t* __restrict__ slots, uint32_t count,
                                            const ContextRow* __restrict__ rows, const float* __restrict__ emb,
                                            uint32_t d, LaneParams canon, const LaneState* lanes, int lane_count) {
    const uint32_t total = count * (d + 1);
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const uint32_t r = i / (d + 1), k = i - r * (d + 1);
        const uint32_t slot = slots[r];
        if (k == d) {
            const ContextRow row = rows[r];
            canon.ctx_keys[slot] = row.key;
            canon.ctx_obs[slot] = row.obs;
            for (int l = 0; l < lane_count; ++l) {
                lanes[l].p.ctx_keys[slot] = row.key;
                lanes[l].p.ctx_obs[slot] = row.obs;
            }
        } else {
            const float v = emb[(size_t)r * d + k];
            canon.ctx_emb[(size_t)slot * d + k] = v;
            for (int l = 0; l < lane_count; ++l) lanes[l].p.ctx_emb[(size_t)slot * d + k] = v;
        }
    }
}

// Copies canonical context rows at `slots` into every resident lane.
__global__ void broadcast_context_rows_kernel(const uint32_t* __restrict__ slots, uint32_t count, LaneParams canon,
                                              uint32_t d, const LaneState* lanes, int lane_count) {
    const uint32_t total = count * (d + 1);
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const uint32_t r = i / (d + 1), k = i - r * (d + 1);
        const uint32_t slot = slots[r];
        for (int l = 0; l < lane_count; ++l) {
            const LaneParams& p = lanes[l].p;
            if (k == d) {
                p.ctx_keys[slot] = canon.ctx_keys[slot];
                p.ctx_obs[slot] = canon.ctx_obs[slot];
            } else {
                p.ctx_emb[(size_t)slot * d + k] = canon.ctx_emb[(size_t)slot * d + k];
            }
        }
    }
}

__global__ void clear_marks_kernel(const uint32_t* __restrict__ list, uint32_t count, uint8_t* marks) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) marks[list[i]] = 0;
}

struct CtxDelta {
    uint32_t order;
    unsigned long long key;
    std::vector<float> emb_delta;
    uint32_t obs_inc;
};

long find_slot(const LeoB200Device& dev, uint32_t order, unsigned long long key) {
    uint32_t spo = dev.cfg.abi.context_slots_per_order, base = (order - 1) * spo, start = (uint32_t)(key % spo);
    for (uint32_t off = 0; off < dev.cfg.abi.context_probe_limit; ++off) {
        uint32_t slot = base + (start + off) % spo;
        if (dev.ctx_keys[slot] == key) return slot;
    }
    return -1;
}

// model.rs:173-221 on the host mirror; returns the slot and records it.
uint32_t resolve_allocate(LeoB200Device& dev, uint32_t order, unsigned long long key, std::vector<uint32_t>& touched) {
    uint32_t spo = dev.cfg.abi.context_slots_per_order, base = (order - 1) * spo, start = (uint32_t)(key % spo);
    long empty = -1;
    uint32_t weakest = base + start, weakest_obs = 0xffffffffu;
    for (uint32_t off = 0; off < dev.cfg.abi.context_probe_limit; ++off) {
        uint32_t slot = base + (start + off) % spo;
        if (dev.ctx_keys[slot] == key) return slot;
        if (dev.ctx_keys[slot] == 0 && empty < 0) empty = slot;
        if (dev.ctx_obs[slot] < weakest_obs) {
            weakest_obs = dev.ctx_obs[slot];
            weakest = slot;
        }
    }
    uint32_t slot = empty >= 0 ? (uint32_t)empty : weakest;
    if (dev.ctx_keys[slot] != key) {
        dev.ctx_keys[slot] = key;
        dev.ctx_obs[slot] = 0;
        size_t d = dev.z.d;
        std::fill(dev.ctx_emb.begin() + slot * d, dev.ctx_emb.begin() + (slot + 1) * d, 0.0f);
        touched.push_back(slot);
    }
    return slot;
}

// context_deltas_for_slots (parallel.rs:929-973) of one lane: reads the
// lane's changed context rows, forms (order, key) deltas against the host
// mirror of the canonical context, clears the lane's context marks.  Returns
// the deltas sorted by (order, key) and appends the lane's changed slots.
std::vector<CtxDelta> collect_lane_context(LeoB200Device& dev, Lane& lane, uint32_t count,
                                           std::vector<uint32_t>& changed_slots) {
    std::vector<CtxDelta> out;
    if (count == 0) return out;
    const ModelSizes& z = dev.z;
    uint32_t d = (uint32_t)z.d, spo = dev.cfg.abi.context_slots_per_order;
    std::vector<uint32_t> slots(count);
    std::vector<ContextRow> rows(count);
    std::vector<float> emb((size_t)count * d);
    ContextRow* d_rows = dev.ctx_stage_rows;
    float* d_emb = dev.ctx_stage_emb;
    gather_context_rows_kernel<<<std::max(1u, std::min(count / 128 + 1, 1024u)), 128, 0, dev.stream>>>(
        lane.st.ctx_list, count, lane.st.p.ctx_keys, lane.st.p.ctx_obs, lane.st.p.ctx_emb, d, d_rows, d_emb);
    CUDA_CHECK(cudaGetLastError());
    dev.perf.launches += 2;  // the gather above and the mark clear below
    CUDA_CHECK(cudaMemcpyAsync(slots.data(), lane.st.ctx_list, count * 4, cudaMemcpyDeviceToHost, dev.stream));
    CUDA_CHECK(cudaMemcpyAsync(rows.data(), d_rows, count * sizeof(ContextRow), cudaMemcpyDeviceToHost, dev.stream));
    CUDA_CHECK(cudaMemcpyAsync(emb.data(), d_emb, emb.size() * 4, cudaMemcpyDeviceToHost, dev.stream));
    clear_marks_kernel<<<std::max(1u, std::min(count / 128 + 1, 1024u)), 128, 0, dev.stream>>>(lane.st.ctx_list, count,
                                                                                               lane.st.ctx_mark);
    CUDA_CHECK(cudaGetLastError());
    CUDA_CHECK(cudaStreamSynchronize(dev.stream));
    for (uint32_t i = 0; i < count; ++i) {
        changed_slots.push_back(slots[i]);
        unsigned long long key = rows[i].key;
        if (key == 0) continue;
        uint32_t order = slots[i] / spo + 1;
        long bs = find_slot(dev, order, key);
        uint32_t bobs = bs >= 0 ? dev.ctx_obs[bs] : 0;
        CtxDelta cd{order, key, std::vector<float>(d), 0};
        bool changed = false;
        for (uint32_t k = 0; k < d; ++k) {
            float before = bs >= 0 ? dev.ctx_emb[(size_t)bs * d + k] : 0.0f;
            float delta = emb[(size_t)i * d + k] - before;
            changed |= delta != 0.0f;
            cd.emb_delta[k] = delta;
        }
        cd.obs_inc = rows[i].obs > bobs ? rows[i].obs - bobs : 0;
        if (changed || cd.obs_inc > 0) out.push_back(std::move(cd));
    }
    std::sort(out.begin(), out.end(), [](const CtxDelta& a, const CtxDelta& b) {
        return a.order != b.order ? a.order < b.order : a.key < b.key;
    });
    return out;
}

// apply_context_deltas (parallel.rs:1024-1113) of every story's deltas, in
// story order, into the host mirror; projection (parallel.rs:1226-1233) and
// validation (parallel.rs:1317-1334); uploads the changed canonical rows and
// syncs every resident lane at them and at `lane_slots` (the resident lanes'
// own changed slots).  Returns the number of merged keys.
size_t merge_context_deltas(LeoB200Device& dev, const std::vector<std::vector<CtxDelta>>& per_story, size_t divisor,
                            const std::vector<uint32_t>& lane_slots) {
    const ModelSizes& z = dev.z;
    const uint32_t d = (uint32_t)z.d;
    const size_t stories = per_story.size();
    // k-way merge by (order, key) in story order (parallel.rs:1045-1089)
    struct Merged {
        uint32_t order;
        unsigned long long key;
        std::vector<double> sum;
        uint64_t obs;
    };
    std::vector<Merged> merged;
    std::vector<size_t> pos(stories, 0);
    for (;;) {
        bool any = false;
        std::pair<uint32_t, unsigned long long> next{0, 0};
        for (size_t l = 0; l < stories; ++l) {
            if (pos[l] < per_story[l].size()) {
                auto k = std::make_pair(per_story[l][pos[l]].order, per_story[l][pos[l]].key);
                if (!any || k < next) next = k;
                any = true;
            }
        }
        if (!any) break;
        Merged m{next.first, next.second, std::vector<double>(d, 0.0), 0};
        for (size_t l = 0; l < stories; ++l) {
            if (pos[l] < per_story[l].size() && per_story[l][pos[l]].order == next.first &&
                per_story[l][pos[l]].key == next.second) {
                const CtxDelta& u = per_story[l][pos[l]];
                if (u.emb_delta.size() != d) throw LeoFailure("invalid keyed context worker delta");
                for (uint32_t k = 0; k < d; ++k) {
                    if (!std::isfinite(u.emb_delta[k])) throw LeoFailure("invalid keyed context worker delta");
                    m.sum[k] += (double)u.emb_delta[k];
                }
                m.obs += u.obs_inc;
                pos[l] += 1;
            }
        }
        merged.push_back(std::move(m));
    }
    std::sort(merged.begin(), merged.end(), [](const Merged& a, const Merged& b) {
        if (a.obs != b.obs) return a.obs > b.obs;
        if (a.order != b.order) return a.order < b.order;
        return a.key < b.key;
    });
    std::vector<uint32_t> canon_slots;
    for (auto& u : merged) {
        uint32_t slot = resolve_allocate(dev, u.order, u.key, canon_slots);
        for (uint32_t k = 0; k < d; ++k) dev.ctx_emb[(size_t)slot * d + k] += (float)(u.sum[k] / (double)divisor);
        uint64_t add = std::min<uint64_t>(u.obs, 0xffffffffull);
        dev.ctx_obs[slot] = (uint32_t)std::min<uint64_t>((uint64_t)dev.ctx_obs[slot] + add, 0xffffffffull);
        canon_slots.push_back(slot);
    }
    float lo = dev.cfg.abi.weight_min, hi = dev.cfg.abi.weight_max;
    for (size_t l = 0; l < stories; ++l) {
        for (auto& u : per_story[l]) {
            long slot = find_slot(dev, u.order, u.key);
            if (slot < 0) continue;
            for (uint32_t k = 0; k < d; ++k) {
                float& v = dev.ctx_emb[(size_t)slot * d + k];
                v = std::min(std::max(v, lo), hi);
                if (!std::isfinite(v)) throw LeoFailure("merged context embedding violates canonical parameter bounds");
            }
        }
    }
    std::vector<uint32_t> sync = canon_slots;
    sync.insert(sync.end(), lane_slots.begin(), lane_slots.end());
    std::sort(sync.begin(), sync.end());
    sync.erase(std::unique(sync.begin(), sync.end()), sync.end());
    if (!sync.empty()) {
        // Stage the rows from the host mirror and scatter them in one kernel
        // (three copies for the whole list, not three per slot).
        const uint32_t n = (uint32_t)sync.size();
        std::vector<ContextRow> rows(n);
        std::vector<float> emb((size_t)n * d);
        for (uint32_t i = 0; i < n; ++i) {
            const uint32_t slot = sync[i];
            rows[i] = ContextRow{dev.ctx_keys[slot], dev.ctx_obs[slot]};
            std::copy_n(dev.ctx_emb.begin() + (size_t)slot * d, d, emb.begin() + (size_t)i * d);
        }
        CUDA_CHECK(cudaMemcpyAsync(dev.ctx_sync_slots, sync.data(), n * 4, cudaMemcpyHostToDevice, dev.stream));
        CUDA_CHECK(cudaMemcpyAsync(dev.ctx_stage_rows, rows.data(), n * sizeof(ContextRow), cudaMemcpyHostToDevice,
                                   dev.stream));
        CUDA_CHECK(cudaMemcpyAsync(dev.ctx_stage_emb, emb.data(), emb.size() * 4, cudaMemcpyHostToDevice, dev.stream));
        const uint32_t total = n * (d + 1);
        scatter_context_rows_kernel<<<std::max(1u, std::min(total / 256 + 1, 4096u)), 256, 0, dev.stream>>>(
            dev.ctx_sync_slots, n, dev.ctx_stage_rows, dev.ctx_stage_emb, d, dev.canon, dev.d_lanes,
            (int)dev.lanes.size());
        CUDA_CHECK(cudaGetLastError());
        dev.perf.launches += 1;
        CUDA_CHECK(cudaStreamSynchronize(dev.stream));
    }
    return merged.size();
}

// Device merge buffers for at least `entries` lane entries (one allocation,
// carved into the per-entry arrays; the canonical slot list is sized by the
// context table).
void ensure_ctx_merge(LeoB200Device& dev, size_t entries) {
    if (dev.ctx_capacity >= entries && dev.ctx_mem) return;
    const size_t cap = std::max<size_t>({entries, 2 * dev.ctx_capacity, (size_t)1 << 14});
    const size_t d = dev.z.d, slots = dev.z.ctx;
    const size_t temp = leo_context_merge_temp_bytes((uint32_t)cap);
    auto align = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t u32 = align(cap * 4), u64 = align(cap * 8), u8 = align(cap);
    const size_t bytes = 10 * u32 + 5 * u64 + 2 * u8 + align(cap * d * 4) + align(cap * d * 8) + align(slots * 4) +
                         align(64) + align(temp);
    dev.ctx_mem.reset();
    auto m = std::make_unique<DevMem>();
    CUDA_CHECK(cudaMalloc(&m->p, bytes));
    uint8_t* at = static_cast<uint8_t*>(m->p);
    auto take = [&](size_t n) {
        uint8_t* r = at;
        at += n;
        return r;
    };
    CtxMergeArgs& a = dev.ctx_args;
    CtxMergeWork& w = dev.ctx_work;
    a.lane_slots = (uint32_t*)take(u32);
    a.order = (uint32_t*)take(u32);
    a.obs_inc = (uint32_t*)take(u32);
    a.morder = (uint32_t*)take(u32);
    w.idx_a = (uint32_t*)take(u32);
    w.idx_b = (uint32_t*)take(u32);
    w.sorted = (uint32_t*)take(u32);
    w.gstart = (uint32_t*)take(u32);
    w.k32_a = (uint32_t*)take(u32);
    w.k32_b = (uint32_t*)take(u32);
    a.key = (unsigned long long*)take(u64);
    a.mkey = (unsigned long long*)take(u64);
    a.mobs = (unsigned long long*)take(u64);
    w.k64_a = (unsigned long long*)take(u64);
    w.k64_b = (unsigned long long*)take(u64);
    a.valid = take(u8);
    w.head = take(u8);
    a.delta = (float*)take(align(cap * d * 4));
    a.msum = (double*)take(align(cap * d * 8));
    a.canon_slots = (uint32_t*)take(align(slots * 4));
    uint32_t* small = (uint32_t*)take(align(64));
    w.count = small;
    a.canon_slot_count = small + 1;
    a.error = small + 2;
    w.temp = take(align(temp));
    w.temp_bytes = temp;
    dev.ctx_mem = std::move(m);
    dev.ctx_capacity = cap;
    a.canon_slot_capacity = (uint32_t)slots;
}

// The single-GPU batch: every story is a resident lane.  The merge runs on the
// device (leo_context_merge.cu) when the context order's slot partition fits
// its shared-memory tables; otherwise on the host.
size_t merge_context(LeoB200Device& dev, uint32_t lane_count, const std::vector<LaneScalars>& scal) {
    if (!dev.ctx_device_merge) {
        std::vector<std::vector<CtxDelta>> per_lane(lane_count);
        std::vector<uint32_t> lane_slots;
        for (uint32_t l = 0; l < lane_count; ++l)
            per_lane[l] = collect_lane_context(dev, *dev.lanes[l], scal[l].ctx_changed, lane_slots);
        return merge_context_deltas(dev, per_lane, lane_count, lane_slots);
    }
    std::vector<uint32_t> offset(lane_count + 1, 0);
    uint32_t widest = 0;
    for (uint32_t l = 0; l < lane_count; ++l) {
        offset[l + 1] = offset[l] + scal[l].ctx_changed;
        widest = std::max(widest, scal[l].ctx_changed);
    }
    const uint32_t entries = offset[lane_count];
    if (entries == 0) return 0;
    ensure_ctx_merge(dev, entries);
    CtxMergeArgs& a = dev.ctx_args;
    a.slots_per_order = dev.cfg.abi.context_slots_per_order;
    a.dim = (uint32_t)dev.z.d;
    a.probe_limit = dev.cfg.abi.context_probe_limit;
    a.stories = lane_count;
    a.weight_min = dev.cfg.abi.weight_min;
    a.weight_max = dev.cfg.abi.weight_max;
    CUDA_CHECK(cudaMemcpyAsync(dev.ctx_lane_offset, offset.data(), offset.size() * 4, cudaMemcpyHostToDevice,
                               dev.stream));
    CUDA_CHECK(cudaMemsetAsync(a.error, 0, 4, dev.stream));
    CUDA_CHECK(leo_context_merge_deltas(dev.d_lanes, dev.ctx_lane_offset, lane_count, widest, dev.canon, a,
                                        dev.stream));
    uint32_t valid = 0, groups = 0;
    CUDA_CHECK(leo_context_merge_group(entries, a, dev.ctx_work, &valid, dev.stream));
    if (valid) CUDA_CHECK(leo_context_merge_sort(valid, a, dev.ctx_work, &groups, dev.stream));
    CUDA_CHECK(leo_context_merge_apply(valid, groups, dev.cfg.abi.context_max_order, dev.canon, dev.d_lanes,
                                       (int)dev.lanes.size(), a.lane_slots, entries, a, dev.ctx_work, dev.stream));
    dev.perf.launches += 16;
    uint32_t error = 0;
    CUDA_CHECK(cudaMemcpyAsync(&error, a.error, 4, cudaMemcpyDeviceToHost, dev.stream));
    // the host mirror of the canonical context follows the device tables
    CUDA_CHECK(cudaMemcpyAsync(dev.ctx_keys.data(), dev.canon.ctx_keys, dev.ctx_keys.size() * 8,
                               cudaMemcpyDeviceToHost, dev.stream));
    CUDA_CHECK(cudaMemcpyAsync(dev.ctx_obs.data(), dev.canon.ctx_obs, dev.ctx_obs.size() * 4, cudaMemcpyDeviceToHost,
                               dev.stream));
    CUDA_CHECK(cudaMemcpyAsync(dev.ctx_emb.data(), dev.canon.ctx_emb, dev.ctx_emb.size() * 4, cudaMemcpyDeviceToHost,
                               dev.stream));
    CUDA_CHECK(cudaStreamSynchronize(dev.stream));
    if (error & LEO_CTX_MERGE_BAD_DELTA) throw LeoFailure("invalid keyed context worker delta");
    if (error & LEO_CTX_MERGE_BAD_VALUE) throw LeoFailure("merged context embedding violates canonical parameter bounds");
    return groups;
}

// ---------------------------------------------------------------- fixed tensor merge
struct TensorSpec {
    float* LaneParams::*member;
    uint32_t* LaneState::*list;
    uint8_t* LaneState::*marks;
    uint32_t LaneScalars::*count;
    uint32_t row, row_len, length, kind;
};

// The six fixed tensors in merge order (parallel.rs:715-798).
std::array<TensorSpec, LEO_B200_FIXED_TENSORS> fixed_specs(const ModelSizes& z) {
    return {{
        {&LaneParams::threshold, &LaneState::thr_list, &LaneState::thr_mark, &LaneScalars::thr_changed, 1, 1,
         (uint32_t)z.n, LEO_PROJECT_THRESHOLD},
        {&LaneParams::rec_weight, &LaneState::rec_list, &LaneState::rec_mark, &LaneScalars::rec_changed, 1, 1,
         (uint32_t)z.synapses, LEO_PROJECT_RECURRENT},
        {&LaneParams::in_weight, &LaneState::in_list, &LaneState::in_mark, &LaneScalars::in_changed, 1, 1,
         (uint32_t)z.inputs, LEO_PROJECT_INPUT},
        {&LaneParams::out_weight, &LaneState::out_list, &LaneState::out_mark, &LaneScalars::out_changed,
         LEO_OUTPUT_STRIDE, LEO_OUTPUT_CLASSES, (uint32_t)z.n, LEO_PROJECT_WEIGHT},
        {&LaneParams::out_bias, nullptr, nullptr, nullptr, 1, 1, LEO_OUTPUT_CLASSES, LEO_PROJECT_NONE},
        {&LaneParams::ctx_out, nullptr, nullptr, nullptr, 1, 1, (uint32_t)z.ctx_out, LEO_PROJECT_WEIGHT},
    }};
}

size_t merge_fixed(LeoB200Device& dev, uint32_t lane_count, const std::vector<LaneScalars>& scal) {
    const ModelSizes& z = dev.z;
    const auto specs = fixed_specs(z);
    uint32_t zero = 0;
    CUDA_CHECK(cudaMemcpyAsync(dev.scratch.updates, &zero, 4, cudaMemcpyHostToDevice, dev.stream));
    const uint32_t resident = (uint32_t)dev.lanes.size();
    for (const TensorSpec& t : specs) {
        std::vector<float*> ptrs(resident);
        std::vector<uint32_t*> lists(lane_count);
        std::vector<uint32_t> counts(lane_count);
        std::vector<uint8_t*> marks(lane_count);
        for (uint32_t l = 0; l < resident; ++l) ptrs[l] = dev.lanes[l]->st.p.*t.member;
        for (uint32_t l = 0; l < lane_count; ++l) {
            LaneState& st = dev.lanes[l]->st;
            lists[l] = t.list ? st.*t.list : nullptr;
            counts[l] = t.count ? scal[l].*t.count : t.length;
            marks[l] = t.marks ? st.*t.marks : nullptr;
        }
        CUDA_CHECK(cudaMemcpyAsync(dev.d_lane_ptrs, ptrs.data(), resident * sizeof(float*), cudaMemcpyHostToDevice, dev.stream));
        CUDA_CHECK(cudaMemcpyAsync(dev.d_lane_lists, lists.data(), lane_count * sizeof(uint32_t*), cudaMemcpyHostToDevice, dev.stream));
        CUDA_CHECK(cudaMemcpyAsync(dev.d_lane_counts, counts.data(), lane_count * 4, cudaMemcpyHostToDevice, dev.stream));
        CUDA_CHECK(cudaMemcpyAsync(dev.d_lane_marks, marks.data(), lane_count * sizeof(uint8_t*), cudaMemcpyHostToDevice, dev.stream));
        MergeTensor mt{};
        mt.lane_values = dev.d_lane_ptrs;
        mt.base = dev.canon.*t.member;
        mt.lane_lists = t.list ? dev.d_lane_lists : nullptr;
        mt.lane_counts = dev.d_lane_counts;
        mt.lane_marks = t.marks ? dev.d_lane_marks : nullptr;
        mt.row = t.row;
        mt.row_len = t.row_len;
        mt.length = t.length;
        mt.kind = t.kind;
        leo_launch_merge_tensor(mt, dev.scratch, (int)lane_count, (int)resident, dev.cfg.abi.weight_min, dev.cfg.abi.weight_max,
                                dev.kc.topo.neuron_type, (uint32_t)z.s, dev.grid, dev.stream);
        dev.perf.launches += 4;
        // Each launch sequence reuses the pointer tables: wait before rewriting them.
        CUDA_CHECK(cudaStreamSynchronize(dev.stream));
    }
    uint32_t updates = 0, err = 0;
    CUDA_CHECK(cudaMemcpy(&updates, dev.scratch.updates, 4, cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaMemcpy(&err, dev.scratch.error_flag, 4, cudaMemcpyDeviceToHost));
    if (err) throw LeoFailure("merged parameter became non-finite");
    return updates;
}

// ---------------------------------------------------------------- replay sync
// Writes canonical values at the replay lane's changed indices into every
// story lane (fused multi-target scatter) and clears the replay marks.
void sync_replay_changes(LeoB200Device& dev, const LaneScalars& rs) {
    const ModelSizes& z = dev.z;
    const uint32_t lane_count = (uint32_t)dev.lanes.size();
    upload_lane_table(dev);
    Lane& rl = *dev.replay;
    // Fixed tensors: reuse the merge kernels with the replay list as the only
    // "lane": every lane value at those indices then equals the canonical.
    struct Item {
        float* LaneParams::*member;
        uint32_t* list;
        uint8_t* marks;
        uint32_t count, row, row_len;
    };
    const Item items[] = {
        {&LaneParams::threshold, rl.st.thr_list, rl.st.thr_mark, rs.thr_changed, 1, 1},
        {&LaneParams::rec_weight, rl.st.rec_list, rl.st.rec_mark, rs.rec_changed, 1, 1},
        {&LaneParams::in_weight, rl.st.in_list, rl.st.in_mark, rs.in_changed, 1, 1},
        {&LaneParams::out_weight, rl.st.out_list, rl.st.out_mark, rs.out_changed, LEO_OUTPUT_STRIDE, LEO_OUTPUT_CLASSES},
    };
    for (const Item& it : items) {
        if (it.count == 0) continue;
        std::vector<float*> ptrs(lane_count);
        for (uint32_t l = 0; l < lane_count; ++l) ptrs[l] = dev.lanes[l]->st.p.*it.member;
        CUDA_CHECK(cudaMemcpyAsync(dev.d_lane_ptrs, ptrs.data(), lane_count * sizeof(float*), cudaMemcpyHostToDevice, dev.stream));
        leo_launch_scatter_rows(dev.d_lane_ptrs, (int)lane_count, dev.canon.*it.member, it.list, it.count, it.row,
                                it.row_len, dev.grid, dev.stream);
        clear_marks_kernel<<<std::max(1u, std::min(it.count / 256 + 1, 4096u)), 256, 0, dev.stream>>>(it.list, it.count,
                                                                                                      it.marks);
        CUDA_CHECK(cudaGetLastError());
        dev.perf.launches += 2;  // the row scatter and the mark clear
        CUDA_CHECK(cudaStreamSynchronize(dev.stream));
    }
    // Dense tensors: bias and context output weights.
    for (uint32_t l = 0; l < lane_count; ++l) {
        LaneParams& p = dev.lanes[l]->st.p;
        if (rs.bias_dirty)
            CUDA_CHECK(cudaMemcpyAsync(p.out_bias, dev.canon.out_bias, LEO_OUTPUT_STRIDE * 4, cudaMemcpyDeviceToDevice, dev.stream));
        if (rs.ctx_out_dirty)
            CUDA_CHECK(cudaMemcpyAsync(p.ctx_out, dev.canon.ctx_out, z.ctx_out * 4, cudaMemcpyDeviceToDevice, dev.stream));
    }
    // Context rows: refresh the host mirror and scatter the canonical rows.
    if (rs.ctx_changed) {
        // Allocation without a learning step cannot happen on a training
        // replay step, so the changed list covers every slot replay rewrote.
        const uint32_t n = rs.ctx_changed, d = (uint32_t)z.d;
        std::vector<uint32_t> slots(n);
        std::vector<ContextRow> rows(n);
        std::vector<float> emb((size_t)n * d);
        const uint32_t grid = std::max(1u, std::min(n / 128 + 1, 1024u));
        gather_context_rows_kernel<<<grid, 128, 0, dev.stream>>>(rl.st.ctx_list, n, dev.canon.ctx_keys,
                                                                dev.canon.ctx_obs, dev.canon.ctx_emb, d,
                                                                dev.ctx_stage_rows, dev.ctx_stage_emb);
        CUDA_CHECK(cudaGetLastError());
        CUDA_CHECK(cudaMemcpyAsync(slots.data(), rl.st.ctx_list, n * 4, cudaMemcpyDeviceToHost, dev.stream));
        CUDA_CHECK(cudaMemcpyAsync(rows.data(), dev.ctx_stage_rows, n * sizeof(ContextRow), cudaMemcpyDeviceToHost,
                                   dev.stream));
        CUDA_CHECK(cudaMemcpyAsync(emb.data(), dev.ctx_stage_emb, emb.size() * 4, cudaMemcpyDeviceToHost, dev.stream));
        const uint32_t total = n * (d + 1);
        if (lane_count > 0)
            broadcast_context_rows_kernel<<<std::max(1u, std::min(total / 256 + 1, 4096u)), 256, 0, dev.stream>>>(
                rl.st.ctx_list, n, dev.canon, d, dev.d_lanes, (int)lane_count);
        CUDA_CHECK(cudaGetLastError());
        clear_marks_kernel<<<std::max(1u, std::min(n / 256 + 1, 4096u)), 256, 0, dev.stream>>>(rl.st.ctx_list, n,
                                                                                              rl.st.ctx_mark);
        CUDA_CHECK(cudaGetLastError());
        dev.perf.launches += lane_count > 0 ? 3 : 2;
        CUDA_CHECK(cudaStreamSynchronize(dev.stream));
        for (uint32_t i = 0; i < n; ++i) {
            const uint32_t slot = slots[i];
            dev.ctx_keys[slot] = rows[i].key;
            dev.ctx_obs[slot] = rows[i].obs;
            std::copy_n(emb.begin() + (size_t)i * d, d, dev.ctx_emb.begin() + (size_t)slot * d);
        }
    }
    // Every mark is clear again: the replay lane's lists restart empty.
    LaneScalars cur;
    read_scalars(dev, rl, cur);
    cur.thr_changed = cur.rec_changed = cur.in_changed = cur.out_changed = cur.ctx_changed = 0;
    cur.bias_dirty = cur.ctx_out_dirty = 0;
    CUDA_CHECK(cudaMemcpyAsync(rl.st.sc, &cur, sizeof(cur), cudaMemcpyHostToDevice, dev.stream));
    CUDA_CHECK(cudaStreamSynchronize(dev.stream));
}

// Canonical rows that steps on the replay lane changed outside a story batch
// (begin_document / training_step_batch) written into every story lane, so
// that the next batch starts every lane from the canonical model.
void refresh_lanes_from_replay(LeoB200Device& dev) {
    LaneScalars rs;
    read_scalars(dev, *dev.replay, rs);
    if (rs.thr_changed | rs.rec_changed | rs.in_changed | rs.out_changed | rs.ctx_changed | rs.bias_dirty |
        rs.ctx_out_dirty)
        sync_replay_changes(dev, rs);
}

// ---------------------------------------------------------------- replay (training.rs:1782-1955)
struct ReplayRange {
    size_t start, end;
};

std::vector<ReplayRange> select_replay_ranges(const std::vector<float>& losses, float fraction, size_t segment) {
    std::vector<ReplayRange> selected;
    if (losses.empty() || !std::isfinite(fraction) || fraction <= 0.0f || segment == 0) return selected;
    size_t budget = (size_t)std::max(std::ceil((double)losses.size() * (double)std::min(fraction, 1.0f)), 1.0);
    std::vector<std::pair<size_t, float>> order;
    for (size_t i = 0; i < losses.size(); ++i) order.push_back({i, losses[i]});
    auto total_key = [](float f) {
        int32_t b;
        std::memcpy(&b, &f, 4);
        return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
    };
    std::sort(order.begin(), order.end(), [&](const auto& l, const auto& r) {
        int32_t a = total_key(l.second), b = total_key(r.second);
        return a != b ? a > b : l.first < r.first;
    });
    size_t picked = 0;
    for (auto& [position, loss] : order) {
        if (picked >= budget) break;
        if (!std::isfinite(loss) || loss <= 0.0f) continue;
        size_t width = std::min(std::min(segment, budget - picked), losses.size());
        size_t start = position >= width / 2 ? position - width / 2 : 0;
        size_t end = std::min(start + width, losses.size());
        start = end >= width ? end - width : 0;
        bool overlap = false;
        for (auto& e : selected)
            if (e.start < end && start < e.end) overlap = true;
        if (overlap) continue;
        picked += end - start;
        selected.push_back({start, end});
    }
    std::sort(selected.begin(), selected.end(), [](const ReplayRange& a, const ReplayRange& b) { return a.start < b.start; });
    return selected;
}

// Runs one schedule on the replay lane (canonical parameters) from a fresh
// transient state at the canonical tick, then folds its statistics into the
// canonical statistics.
void run_canonical_schedule(LeoB200Device& dev, const std::vector<uint32_t>& schedule, LaneScalars& out) {
    Lane& rl = *dev.replay;
    ensure_schedule(rl, schedule.size());
    CUDA_CHECK(cudaMemcpyAsync(rl.schedule, schedule.data(), schedule.size() * 4, cudaMemcpyHostToDevice, dev.stream));
    reset_lane(dev, rl, dev.canonical_tick, (uint32_t)schedule.size());
    CUDA_CHECK(cudaMemcpyAsync(dev.d_replay, &rl.st, sizeof(LaneState), cudaMemcpyHostToDevice, dev.stream));
    // keep the replay lane's changed marks across schedules: carry counts over
    LaneScalars carry{};
    CUDA_CHECK(cudaMemcpyAsync(&carry, rl.st.sc, sizeof(carry), cudaMemcpyDeviceToHost, dev.stream));
    CUDA_CHECK(cudaStreamSynchronize(dev.stream));
    carry.thr_changed = out.thr_changed;
    carry.rec_changed = out.rec_changed;
    carry.in_changed = out.in_changed;
    carry.out_changed = out.out_changed;
    carry.ctx_changed = out.ctx_changed;
    carry.bias_dirty = out.bias_dirty;
    carry.ctx_out_dirty = out.ctx_out_dirty;
    CUDA_CHECK(cudaMemcpyAsync(rl.st.sc, &carry, sizeof(carry), cudaMemcpyHostToDevice, dev.stream));
    run_steps(dev, dev.d_replay, 1, 0, (uint32_t)schedule.size(), false);
    LaneScalars sc;
    read_scalars(dev, rl, sc);
    check_error_flag(sc);
    add_work(dev, sc, false);
    dev.canonical_tick += schedule.size();
    dev.revision += sc.revision_increment;
    dev.stats.processed_bytes += sc.processed_bytes;
    dev.stats.training_loss_sum = sc.loss_sum;
    dev.stats.training_targets += sc.targets;
    dev.stats.active_neurons_sum += sc.active_sum;
    dev.stats.active_neurons_peak = std::max<uint64_t>(dev.stats.active_neurons_peak, sc.active_peak);
    dev.stats.synaptic_events += sc.synaptic_events;
    dev.stats.numerical_rejections += sc.numerical_rejections;
    dev.stats.persistent_ticks += sc.persistent_ticks;
    out = sc;
}

void replay_story(LeoB200Device& dev, const std::vector<uint8_t>& story, const std::vector<float>& losses,
                  int permission, LaneScalars& changes, LeoB200BatchReport* report) {
    auto ranges = select_replay_ranges(losses, dev.cfg.host.replay_fraction, dev.cfg.host.replay_segment_bytes);
    size_t len = story.size();
    for (const ReplayRange& range : ranges) {
        if (len == 0 || range.start >= range.end || range.start > len) continue;
        size_t end = std::min(range.end, len + 1);
        std::vector<uint32_t> sched;
        size_t next = range.start;
        if (next > 0) {
            sched.push_back(schedule_word(LEO_B200_BEGIN_DOCUMENT, -1, LEO_B200_FROZEN));
            for (size_t i = 0; i + 1 < next; ++i) sched.push_back(schedule_word(story[i], -1, LEO_B200_FROZEN));
            if (report) report->replay_prefix_steps += next;
        }
        if (next == 0) {
            sched.push_back(schedule_word(LEO_B200_BEGIN_DOCUMENT, story[0], permission));
            next = 1;
            if (report) report->replay_steps += 1;
        }
        for (size_t p = next; p < end; ++p) {
            int target = p < len ? story[p] : (int)LEO_B200_END_DOCUMENT;
            sched.push_back(schedule_word(story[p - 1], target, permission));
            if (report) report->replay_steps += 1;
        }
        run_canonical_schedule(dev, sched, changes);
    }
    if (report) report->replay_segments += ranges.size();
}

// Uploads stories [first, first + count) of the batch in one copy (offsets,
// then bytes) and builds their schedules on the device into the schedule
// buffers named by the device LaneState table `table` (already uploaded on
// the stream).  Every lane's schedule buffer holds at least story length + 1.
void build_schedules(LeoB200Device& dev, uint32_t first, uint32_t count, int permission, const LaneState* table) {
    std::vector<uint64_t> offsets(count + 1, 0);
    for (uint32_t i = 0; i < count; ++i) offsets[i + 1] = offsets[i] + dev.batch_stories[first + i].size();
    const size_t head = offsets.size() * sizeof(uint64_t);
    const size_t need = head + offsets[count];
    dev.h_stage.resize(need);
    std::memcpy(dev.h_stage.data(), offsets.data(), head);
    for (uint32_t i = 0; i < count; ++i) {
        const auto& story = dev.batch_stories[first + i];
        if (!story.empty()) std::memcpy(dev.h_stage.data() + head + offsets[i], story.data(), story.size());
    }
    if (dev.stage_capacity < need) {
        const size_t cap = std::max<size_t>({need, 2 * dev.stage_capacity, (size_t)1 << 16});
        dev.d_stage.reset();
        auto m = std::make_unique<DevMem>();
        CUDA_CHECK(cudaMalloc(&m->p, cap));
        dev.d_stage = std::move(m);
        dev.stage_capacity = cap;
    }
    uint8_t* d = static_cast<uint8_t*>(dev.d_stage->p);
    CUDA_CHECK(cudaMemcpyAsync(d, dev.h_stage.data(), need, cudaMemcpyHostToDevice, dev.stream));
    CUDA_CHECK(leo_launch_build_schedules(d + head, reinterpret_cast<const uint64_t*>(d), table, count,
                                          (uint32_t)permission, dev.stream));
    dev.perf.launches += 1;
}

// ---------------------------------------------------------------- trait-level exports
// Lane and canonical values of `count` rows of `row_len` floats (row stride
// `row`) at list[i].
__global__ void gather_value_pairs_kernel(const uint32_t* __restrict__ list, uint32_t count, uint32_t row,
                                          uint32_t row_len, const float* __restrict__ lane,
                                          const float* __restrict__ canon, float* out_lane, float* out_canon) {
    const uint64_t total = (uint64_t)count * row_len;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / row_len, k = i - r * row_len;
        const size_t at = (size_t)list[r] * row + k;
        out_lane[i] = lane[at];
        out_canon[i] = canon[at];
    }
}

// values (count rows of row_len floats) written to base at list[i] * row.
__global__ void write_rows_kernel(float* base, const uint32_t* __restrict__ list, uint32_t count, uint32_t row,
                                  uint32_t row_len, const float* __restrict__ values) {
    const uint64_t total = (uint64_t)count * row_len;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / row_len, k = i - r * row_len;
        base[(size_t)list[r] * row + k] = values[i];
    }
}

uint32_t grid_for(uint64_t work) { return (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>(work / 256 + 1, 4096)); }

// A temporary device buffer for one trait-level call.
struct Scratch {
    void* p = nullptr;
    explicit Scratch(size_t bytes) { CUDA_CHECK(cudaMalloc(&p, std::max<size_t>(bytes, 16))); }
    ~Scratch() { if (p) cudaFree(p); }
    template <typename T> T* as() const { return static_cast<T*>(p); }
};

// One fixed tensor of a lane: its changed-index list and the row layout.
struct LaneTensor {
    const uint32_t* list;
    uint8_t* marks;
    uint32_t count;
    uint32_t row, row_len;
    float* lane;
    const float* canon;
};

// Story deltas of lane `l` (SparseModelDelta::from_tracked_values,
// parallel.rs:461-674): every changed index with a nonzero lane - canonical
// difference, in reference indexing, sorted; keyed context deltas; the
// statistics delta relative to the canonical statistics.
void export_story_delta(LeoB200Device& dev, uint32_t l, const LaneScalars& sc, double canon_loss,
                        LeoB200Device::StoryDelta& out) {
    Lane& lane = *dev.lanes[l];
    const ModelSizes& z = dev.z;
    const uint32_t N = (uint32_t)z.n;
    const LaneTensor fixed[4] = {
        {lane.st.thr_list, lane.st.thr_mark, sc.thr_changed, 1, 1, lane.st.p.threshold, dev.canon.threshold},
        {lane.st.rec_list, lane.st.rec_mark, sc.rec_changed, 1, 1, lane.st.p.rec_weight, dev.canon.rec_weight},
        {lane.st.in_list, lane.st.in_mark, sc.in_changed, 1, 1, lane.st.p.in_weight, dev.canon.in_weight},
        {lane.st.out_list, lane.st.out_mark, sc.out_changed, LEO_OUTPUT_STRIDE, LEO_OUTPUT_CLASSES,
         lane.st.p.out_weight, dev.canon.out_weight},
    };
    for (int t = 0; t < 4; ++t) {
        const LaneTensor& lt = fixed[t];
        if (lt.count == 0) continue;
        const size_t n = (size_t)lt.count * lt.row_len;
        Scratch buf(2 * n * sizeof(float));
        gather_value_pairs_kernel<<<grid_for(n), 256, 0, dev.stream>>>(lt.list, lt.count, lt.row, lt.row_len, lt.lane,
                                                                      lt.canon, buf.as<float>(), buf.as<float>() + n);
        CUDA_CHECK(cudaGetLastError());
        std::vector<uint32_t> list(lt.count);
        std::vector<float> vals(2 * n);
        CUDA_CHECK(cudaMemcpyAsync(list.data(), lt.list, lt.count * 4, cudaMemcpyDeviceToHost, dev.stream));
        CUDA_CHECK(cudaMemcpyAsync(vals.data(), buf.p, 2 * n * sizeof(float), cudaMemcpyDeviceToHost, dev.stream));
        CUDA_CHECK(cudaStreamSynchronize(dev.stream));
        out.changed[t].assign(list.begin(), list.end());
        std::sort(out.changed[t].begin(), out.changed[t].end());
        std::vector<std::pair<uint32_t, float>> pairs;
        for (size_t r = 0; r < lt.count; ++r)
            for (uint32_t k = 0; k < lt.row_len; ++k) {
                const float d = vals[r * lt.row_len + k] - vals[n + r * lt.row_len + k];
                if (d != 0.0f) pairs.push_back({lt.row_len == 1 ? list[r] : k * N + list[r], d});
            }
        std::sort(pairs.begin(), pairs.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
        for (const auto& [i, d] : pairs) {
            out.index[t].push_back(i);
            out.delta[t].push_back(d);
        }
    }
    // Dense tensors when the lane changed them: output bias, context output weights.
    const struct {
        uint32_t dirty;
        size_t count;
        const float* lane;
        const float* canon;
        int tensor;
    } dense[2] = {{sc.bias_dirty, LEO_OUTPUT_CLASSES, lane.st.p.out_bias, dev.canon.out_bias, 4},
                  {sc.ctx_out_dirty, z.ctx_out, lane.st.p.ctx_out, dev.canon.ctx_out, 5}};
    for (const auto& dt : dense) {
        if (!dt.dirty) continue;
        std::vector<float> a(dt.count), b(dt.count);
        CUDA_CHECK(cudaMemcpyAsync(a.data(), dt.lane, dt.count * 4, cudaMemcpyDeviceToHost, dev.stream));
        CUDA_CHECK(cudaMemcpyAsync(b.data(), dt.canon, dt.count * 4, cudaMemcpyDeviceToHost, dev.stream));
        CUDA_CHECK(cudaStreamSynchronize(dev.stream));
        for (size_t i = 0; i < dt.count; ++i) {
            const float d = a[i] - b[i];
            if (d != 0.0f) {
                out.index[dt.tensor].push_back((uint32_t)i);
                out.delta[dt.tensor].push_back(d);
            }
        }
    }
    std::vector<uint32_t> slots;
    std::vector<CtxDelta> ctx = collect_lane_context(dev, lane, sc.ctx_changed, slots);
    out.changed[4].assign(slots.begin(), slots.end());
    std::sort(out.changed[4].begin(), out.changed[4].end());
    out.dirty = (sc.bias_dirty ? 1u : 0u) | (sc.ctx_out_dirty ? 2u : 0u);
    // canonicalize_order (parallel.rs:676-691): by order, then key.
    std::sort(ctx.begin(), ctx.end(), [](const CtxDelta& a, const CtxDelta& b) {
        return a.order != b.order ? a.order < b.order : a.key < b.key;
    });
    for (const CtxDelta& cd : ctx) {
        out.ctx_order.push_back(cd.order);
        out.ctx_key.push_back(cd.key);
        out.ctx_obs_inc.push_back(cd.obs_inc);
        out.ctx_emb.insert(out.ctx_emb.end(), cd.emb_delta.begin(), cd.emb_delta.end());
    }
    const auto& story = dev.batch_stories[l];
    LeoB200Statistics& st = out.stats;
    st.processed_bytes = sc.processed_bytes;
    st.processed_stories = (story.empty() || dev.batch_permission == LEO_B200_FROZEN) ? 0 : 1;
    st.training_loss_sum = sc.loss_sum - canon_loss;
    st.training_targets = sc.targets;
    st.active_neurons_sum = sc.active_sum;
    st.active_neurons_peak = sc.active_peak;
    st.synaptic_events = sc.synaptic_events;
    st.numerical_rejections = sc.numerical_rejections;
    st.persistent_ticks = sc.persistent_ticks;
    out.revision = sc.revision_increment;
}

// Lane `l` back to the canonical values at every index it changed, its marks
// cleared (the canonical model is unchanged by an exported batch).
void restore_lane(LeoB200Device& dev, uint32_t l, const LaneScalars& sc) {
    Lane& lane = *dev.lanes[l];
    const ModelSizes& z = dev.z;
    struct Item {
        float* LaneParams::*member;
        uint32_t* list;
        uint8_t* marks;
        uint32_t count, row, row_len;
    };
    const Item items[] = {
        {&LaneParams::threshold, lane.st.thr_list, lane.st.thr_mark, sc.thr_changed, 1, 1},
        {&LaneParams::rec_weight, lane.st.rec_list, lane.st.rec_mark, sc.rec_changed, 1, 1},
        {&LaneParams::in_weight, lane.st.in_list, lane.st.in_mark, sc.in_changed, 1, 1},
        {&LaneParams::out_weight, lane.st.out_list, lane.st.out_mark, sc.out_changed, LEO_OUTPUT_STRIDE, LEO_OUTPUT_CLASSES},
    };
    for (const Item& it : items) {
        if (it.count == 0) continue;
        float* ptr = lane.st.p.*it.member;
        CUDA_CHECK(cudaMemcpyAsync(dev.d_lane_ptrs, &ptr, sizeof(float*), cudaMemcpyHostToDevice, dev.stream));
        leo_launch_scatter_rows(dev.d_lane_ptrs, 1, dev.canon.*it.member, it.list, it.count, it.row, it.row_len,
                                dev.grid, dev.stream);
        clear_marks_kernel<<<grid_for(it.count), 256, 0, dev.stream>>>(it.list, it.count, it.marks);
        CUDA_CHECK(cudaGetLastError());
        CUDA_CHECK(cudaStreamSynchronize(dev.stream));
    }
    if (sc.bias_dirty)
        CUDA_CHECK(cudaMemcpyAsync(lane.st.p.out_bias, dev.canon.out_bias, LEO_OUTPUT_STRIDE * 4, cudaMemcpyDeviceToDevice,
                                   dev.stream));
    if (sc.ctx_out_dirty)
        CUDA_CHECK(cudaMemcpyAsync(lane.st.p.ctx_out, dev.canon.ctx_out, z.ctx_out * 4, cudaMemcpyDeviceToDevice,
                                   dev.stream));
    if (sc.ctx_changed) {
        broadcast_context_rows_kernel<<<grid_for((uint64_t)sc.ctx_changed * (z.d + 1)), 256, 0, dev.stream>>>(
            lane.st.ctx_list, sc.ctx_changed, dev.canon, (uint32_t)z.d, dev.d_lanes + l, 1);
        CUDA_CHECK(cudaGetLastError());
    }
    CUDA_CHECK(cudaStreamSynchronize(dev.stream));
}

// ---------------------------------------------------------------- batch
void batch_begin(LeoB200Device& dev, const uint8_t* bytes, const uint64_t* offsets, uint32_t stories, int permission) {
    if (dev.batch_open) throw LeoFailure("a story batch is already in progress");
    if (stories == 0) throw LeoFailure("training batch cannot be empty");
    if (permission < 0 || permission > 3) throw LeoFailure("invalid permission");
    refresh_lanes_from_replay(dev);
    dev.doc_open = false;
    dev.batch_stories.assign(stories, {});
    for (uint32_t i = 0; i < stories; ++i)
        dev.batch_stories[i].assign(bytes + offsets[i], bytes + offsets[i + 1]);
    dev.batch_permission = permission;
    dev.single_story = stories == 1 && !dev.force_lanes;
    dev.steps_done = 0;
    dev.batch_steps = 0;
    if (dev.single_story) {
        // training.rs:1548-1581: one story trains the canonical runtime directly.
        const auto& story = dev.batch_stories[0];
        const uint32_t steps = story.empty() ? 0 : (uint32_t)story.size() + 1;
        Lane& rl = *dev.replay;
        ensure_schedule(rl, story.size() + 1);
        reset_lane(dev, rl, dev.canonical_tick, steps);
        CUDA_CHECK(cudaMemcpyAsync(dev.d_replay, &rl.st, sizeof(LaneState), cudaMemcpyHostToDevice, dev.stream));
        build_schedules(dev, 0, 1, permission, dev.d_replay);
        dev.batch_lanes = 0;
        dev.batch_steps = steps;
    } else {
        ensure_lanes(dev, stories);
        dev.lane_steps.assign(stories, 0u);
        for (uint32_t i = 0; i < stories; ++i) {
            Lane& lane = *dev.lanes[i];
            const auto& story = dev.batch_stories[i];
            const uint32_t steps = story.empty() ? 0 : (uint32_t)story.size() + 1;
            ensure_schedule(lane, story.size() + 1);
            // Forked workers start a fresh runtime at tick 0 (backend.rs:486-488).
            reset_lane(dev, lane, 0ull, steps);
            dev.batch_steps = std::max(dev.batch_steps, steps);
            dev.lane_steps[i] = steps;
        }
        dev.batch_lanes = stories;
        upload_lane_table(dev);
        build_schedules(dev, 0, stories, permission, dev.d_lanes);
    }
    CUDA_CHECK(cudaEventRecord(dev.batch_start, dev.stream));
    dev.batch_open = true;
}

void batch_steps(LeoB200Device& dev, uint32_t count) {
    if (!dev.batch_open) throw LeoFailure("no story batch in progress");
    uint32_t end = std::min(dev.batch_steps, dev.steps_done + count);
    if (dev.single_story)
        run_steps(dev, dev.d_replay, 1, dev.steps_done, end, false);
    else if (dev.story_cluster_request)
        run_steps(dev, dev.d_lanes, (int)dev.batch_lanes, dev.steps_done, end, true);
    else
        run_story_adaptive(dev, (int)dev.batch_lanes, dev.steps_done, end);
    dev.steps_done = end;
}

// How a batch ends: the fused path (merge, serial replay, replay sync), the
// trait's training_story_batch (merge and lane sync; the caller replays), or
// its training_story_batch_deltas (per-story deltas exported, nothing merged).
enum class FinishMode { kFused, kNoReplay, kDeltas };

// Every story's replay ranges (training.rs:1782-1830) as (start, end) pairs in
// story order.
void write_replay_ranges(const LeoB200Device& dev, const std::vector<std::vector<float>>& losses, uint64_t* ranges,
                         uint32_t* range_counts) {
    size_t k = 0;
    for (size_t i = 0; i < losses.size(); ++i) {
        const auto rr = select_replay_ranges(losses[i], dev.cfg.host.replay_fraction, dev.cfg.host.replay_segment_bytes);
        if (range_counts) range_counts[i] = (uint32_t)rr.size();
        for (const ReplayRange& r : rr) {
            if (ranges) {
                ranges[2 * k] = r.start;
                ranges[2 * k + 1] = r.end;
            }
            ++k;
        }
    }
}

void batch_finish(LeoB200Device& dev, LeoB200BatchReport* report, LeoB200StorySummary* summaries, float* losses_out,
                  FinishMode mode = FinishMode::kFused, uint64_t* ranges = nullptr, uint32_t* range_counts = nullptr) {
    if (!dev.batch_open) throw LeoFailure("no story batch in progress");
    batch_steps(dev, dev.batch_steps);
    CUDA_CHECK(cudaStreamSynchronize(dev.stream));
    dev.batch_open = false;
    LeoB200BatchReport rep{};
    uint32_t stories = (uint32_t)dev.batch_stories.size();
    rep.stories = stories;
    std::vector<std::vector<float>> losses(stories);
    LaneScalars replay_changes{};
    if (dev.single_story) {
        const auto& story = dev.batch_stories[0];
        LaneScalars sc;
        read_scalars(dev, *dev.replay, sc);
        check_error_flag(sc);
        add_work(dev, sc, true);
        if (!story.empty()) {
            losses[0].resize(story.size() + 1);
            CUDA_CHECK(cudaMemcpy(losses[0].data(), dev.replay->step_loss, losses[0].size() * 4, cudaMemcpyDeviceToHost));
            dev.canonical_tick += story.size() + 1;
            dev.revision += sc.revision_increment;
            dev.stats.processed_bytes += sc.processed_bytes;
            // finish_document counts a story only after a non-frozen step
            // (runtime.rs:357-362, 492-496): every step of a story pass has
            // the batch's permission.
            dev.stats.processed_stories += dev.batch_permission != LEO_B200_FROZEN ? 1 : 0;
            dev.stats.training_loss_sum = sc.loss_sum;
            dev.stats.training_targets += sc.targets;
            dev.stats.active_neurons_sum += sc.active_sum;
            dev.stats.active_neurons_peak = std::max<uint64_t>(dev.stats.active_neurons_peak, sc.active_peak);
            dev.stats.synaptic_events += sc.synaptic_events;
            dev.stats.numerical_rejections += sc.numerical_rejections;
            dev.stats.persistent_ticks += sc.persistent_ticks;
            if (summaries) {
                summaries[0].training_loss_sum = 0.0;
                for (float v : losses[0]) summaries[0].training_loss_sum += (double)v;
                summaries[0].training_targets = sc.targets;
                summaries[0].active_neurons_sum = sc.active_sum;
                summaries[0].active_neurons_peak = sc.active_peak;
                summaries[0].synaptic_events = sc.synaptic_events;
                summaries[0].context_applied_steps = sc.context_applied_steps;
            }
        }
        replay_changes = sc;
        rep.workers = 1;
        rep.targets = losses[0].size();
        rep.input_bytes = story.size();
        double sum = 0.0;
        for (float v : losses[0]) sum += (double)v;
        rep.mean_loss = sum / (double)std::max<size_t>(losses[0].size(), 1);
        if (mode == FinishMode::kFused) replay_story(dev, story, losses[0], dev.batch_permission, replay_changes, &rep);
        sync_replay_changes(dev, replay_changes);
    } else {
        uint32_t L = dev.batch_lanes;
        std::vector<LaneScalars> scal(L);
        auto t0 = std::chrono::steady_clock::now();
        for (uint32_t l = 0; l < L; ++l) {
            read_scalars(dev, *dev.lanes[l], scal[l]);
            check_error_flag(scal[l]);
            add_work(dev, scal[l], true);
            const auto& story = dev.batch_stories[l];
            if (!story.empty()) {
                losses[l].resize(story.size() + 1);
                CUDA_CHECK(cudaMemcpy(losses[l].data(), dev.lanes[l]->step_loss, losses[l].size() * 4, cudaMemcpyDeviceToHost));
            }
            rep.input_bytes += story.size();
        }
        // apply_mean_deltas (parallel.rs:715-798): fixed tensors on the device,
        // keyed context on the host mirror, statistics and revision here.
        double canon_loss = dev.stats.training_loss_sum;
        dev.perf.collect_ms += ms_since(t0);
        if (mode == FinishMode::kDeltas) {
            // Each story's delta leaves with the caller; the lanes return to
            // the (unchanged) canonical model.
            upload_lane_table(dev);
            dev.story_deltas.assign(L, {});
            for (uint32_t l = 0; l < L; ++l) {
                export_story_delta(dev, l, scal[l], canon_loss, dev.story_deltas[l]);
                restore_lane(dev, l, scal[l]);
            }
            for (uint32_t l = 0; l < L; ++l) {
                const LaneScalars& sc = scal[l];
                if (summaries) {
                    summaries[l].training_loss_sum = 0.0;
                    for (float v : losses[l]) summaries[l].training_loss_sum += (double)v;
                    summaries[l].training_targets = sc.targets;
                    summaries[l].active_neurons_sum = sc.active_sum;
                    summaries[l].active_neurons_peak = sc.active_peak;
                    summaries[l].synaptic_events = sc.synaptic_events;
                    summaries[l].context_applied_steps = sc.context_applied_steps;
                }
            }
        } else {
        t0 = std::chrono::steady_clock::now();
        rep.fixed_parameter_updates = merge_fixed(dev, L, scal);
        dev.perf.merge_fixed_ms += ms_since(t0);
        t0 = std::chrono::steady_clock::now();
        rep.context_keys = merge_context(dev, L, scal);
        dev.perf.merge_context_ms += ms_since(t0);
        for (uint32_t l = 0; l < L; ++l) {
            const LaneScalars& sc = scal[l];
            const auto& story = dev.batch_stories[l];
            dev.stats.processed_bytes += sc.processed_bytes;
            dev.stats.processed_stories += (story.empty() || dev.batch_permission == LEO_B200_FROZEN) ? 0 : 1;
            dev.stats.training_loss_sum += sc.loss_sum - canon_loss;
            dev.stats.training_targets += sc.targets;
            dev.stats.active_neurons_sum += sc.active_sum;
            dev.stats.active_neurons_peak = std::max<uint64_t>(dev.stats.active_neurons_peak, sc.active_peak);
            dev.stats.synaptic_events += sc.synaptic_events;
            dev.stats.numerical_rejections += sc.numerical_rejections;
            dev.stats.persistent_ticks += sc.persistent_ticks;
            dev.revision += sc.revision_increment;
            if (summaries) {
                summaries[l].training_loss_sum = 0.0;
                for (float v : losses[l]) summaries[l].training_loss_sum += (double)v;
                summaries[l].training_targets = sc.targets;
                summaries[l].active_neurons_sum = sc.active_sum;
                summaries[l].active_neurons_peak = sc.active_peak;
                summaries[l].synaptic_events = sc.synaptic_events;
                summaries[l].context_applied_steps = sc.context_applied_steps;
            }
        }
        }
        rep.workers = L;
        double weighted = 0.0;
        size_t targets = 0;
        for (uint32_t l = 0; l < L; ++l) {
            double sum = 0.0;
            for (float v : losses[l]) sum += (double)v;
            double mean = sum / (double)std::max<size_t>(losses[l].size(), 1);
            weighted += mean * (double)losses[l].size();
            targets += losses[l].size();
        }
        rep.targets = targets;
        rep.mean_loss = weighted / (double)std::max<size_t>(targets, 1);
        // Serial canonical replay (training.rs:1709-1711), then one sync of the
        // replay's changed rows into every lane (training.rs:1644-1649).
        t0 = std::chrono::steady_clock::now();
        for (uint32_t l = 0; l < L && mode == FinishMode::kFused; ++l)
            replay_story(dev, dev.batch_stories[l], losses[l], dev.batch_permission, replay_changes, &rep);
        CUDA_CHECK(cudaStreamSynchronize(dev.stream));
        dev.perf.replay_ms += ms_since(t0);
        t0 = std::chrono::steady_clock::now();
        sync_replay_changes(dev, replay_changes);
        CUDA_CHECK(cudaStreamSynchronize(dev.stream));
        dev.perf.replay_sync_ms += ms_since(t0);
    }
    CUDA_CHECK(cudaEventRecord(dev.batch_stop, dev.stream));
    CUDA_CHECK(cudaEventSynchronize(dev.batch_stop));
    float batch_ms = 0.0f;
    CUDA_CHECK(cudaEventElapsedTime(&batch_ms, dev.batch_start, dev.batch_stop));
    dev.perf.batch_ms += batch_ms;
    dev.perf.batches += 1;
    if (losses_out) {
        size_t k = 0;
        for (auto& l : losses)
            for (float v : l) losses_out[k++] = v;
    }
    if (ranges || range_counts) write_replay_ranges(dev, losses, ranges, range_counts);
    if (report) *report = rep;
}


// ---------------------------------------------------------------- canonical runtime, step by step
// The replay lane holds the canonical runtime's transient state (its
// parameters are the canonical model).  A document is begun at the canonical
// tick and grows by the steps of each call; tracking of changed parameters
// persists across documents until enabled afresh.

void replay_scalars_write(LeoB200Device& dev, const LaneScalars& sc) {
    CUDA_CHECK(cudaMemcpyAsync(dev.replay->st.sc, &sc, sizeof(sc), cudaMemcpyHostToDevice, dev.stream));
    CUDA_CHECK(cudaStreamSynchronize(dev.stream));
}

void doc_begin(LeoB200Device& dev) {
    if (dev.batch_open) throw LeoFailure("a story batch is in progress");
    Lane& rl = *dev.replay;
    ensure_schedule(rl, 4096);
    LaneScalars before;
    read_scalars(dev, rl, before);
    reset_lane(dev, rl, dev.canonical_tick, 0);
    LaneScalars sc;
    read_scalars(dev, rl, sc);
    sc.thr_changed = before.thr_changed;
    sc.rec_changed = before.rec_changed;
    sc.in_changed = before.in_changed;
    sc.out_changed = before.out_changed;
    sc.ctx_changed = before.ctx_changed;
    sc.bias_dirty = before.bias_dirty;
    sc.ctx_out_dirty = before.ctx_out_dirty;
    replay_scalars_write(dev, sc);
    dev.doc_open = true;
    dev.doc_steps = 0;
}

void doc_steps(LeoB200Device& dev, const uint32_t* symbols, const int32_t* targets, uint32_t count, int permission,
               float* losses, uint32_t* actives) {
    if (!dev.doc_open) throw LeoFailure("no document begun (leo_b200_begin_document)");
    if (permission < 0 || permission > 3) throw LeoFailure("invalid permission");
    if (count == 0) return;
    if (!symbols || !targets) throw LeoFailure("steps are null");
    std::vector<uint32_t> words(count);
    for (uint32_t i = 0; i < count; ++i) {
        if (symbols[i] >= LEO_B200_SYMBOL_COUNT) throw LeoFailure("input symbol out of range");
        const int32_t t = targets[i];
        if (t < -1 || t > (int32_t)LEO_B200_END_DOCUMENT || t == (int32_t)LEO_B200_BEGIN_DOCUMENT)
            throw LeoFailure("target symbol out of range");
        words[i] = schedule_word(symbols[i], t, permission);
    }
    Lane& rl = *dev.replay;
    const uint32_t begin = dev.doc_steps, end = begin + count;
    if (rl.schedule_capacity < end) {
        // A longer document: new buffers (steps before `begin` are not read again).
        rl.schedule_capacity = 0;
        ensure_schedule(rl, std::max<size_t>(end, 2 * (size_t)end));
    }
    CUDA_CHECK(cudaMemcpyAsync(rl.schedule + begin, words.data(), count * 4, cudaMemcpyHostToDevice, dev.stream));
    LaneScalars before;
    read_scalars(dev, rl, before);
    LaneScalars sc = before;
    sc.steps = end;
    replay_scalars_write(dev, sc);
    CUDA_CHECK(cudaMemcpyAsync(dev.d_replay, &rl.st, sizeof(LaneState), cudaMemcpyHostToDevice, dev.stream));
    run_steps(dev, dev.d_replay, 1, begin, end, false);
    LaneScalars after;
    read_scalars(dev, rl, after);
    check_error_flag(after);
    // Statistics, revision and tick advance with the steps (runtime.rs:1595-1622).
    dev.canonical_tick += count;
    dev.revision += after.revision_increment - before.revision_increment;
    dev.stats.processed_bytes += after.processed_bytes - before.processed_bytes;
    dev.stats.training_loss_sum = after.loss_sum;
    dev.stats.training_targets += after.targets - before.targets;
    dev.stats.active_neurons_sum += after.active_sum - before.active_sum;
    dev.stats.active_neurons_peak = std::max<uint64_t>(dev.stats.active_neurons_peak, after.active_peak);
    dev.stats.synaptic_events += after.synaptic_events - before.synaptic_events;
    dev.stats.numerical_rejections += after.numerical_rejections - before.numerical_rejections;
    dev.stats.persistent_ticks += after.persistent_ticks - before.persistent_ticks;
    if (losses) CUDA_CHECK(cudaMemcpy(losses, rl.step_loss + begin, count * 4, cudaMemcpyDeviceToHost));
    if (actives) CUDA_CHECK(cudaMemcpy(actives, rl.step_active + begin, count * 4, cudaMemcpyDeviceToHost));
    dev.doc_steps = end;
}

// The replay lane's changed-index lists (one per tracked tensor).
struct TrackedList {
    uint32_t* list;
    uint8_t* marks;
    uint32_t count;
};

// A new window: changes the canonical runtime made before it are first written
// into every lane and the host mirror (their lists then restart empty), so no
// change is lost to the lanes when the lists are reset.
void tracking_enable(LeoB200Device& dev) {
    if (dev.batch_open) throw LeoFailure("a story batch is in progress");
    refresh_lanes_from_replay(dev);
}

void tracking_changes(LeoB200Device& dev, LeoB200ParameterChangeSizes* sizes, const LeoB200ParameterChanges* out) {
    Lane& rl = *dev.replay;
    LaneScalars sc;
    read_scalars(dev, rl, sc);
    const TrackedList lists[] = {{rl.st.thr_list, nullptr, sc.thr_changed},
                                 {rl.st.rec_list, nullptr, sc.rec_changed},
                                 {rl.st.in_list, nullptr, sc.in_changed},
                                 {rl.st.out_list, nullptr, sc.out_changed},
                                 {rl.st.ctx_list, nullptr, sc.ctx_changed}};
    uint32_t* dst[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
    if (out) {
        dst[0] = out->threshold;
        dst[1] = out->recurrent_weight;
        dst[2] = out->input_weight;
        dst[3] = out->output_neurons;
        dst[4] = out->context_slots;
    }
    if (sizes) {
        sizes->threshold = sc.thr_changed;
        sizes->recurrent_weight = sc.rec_changed;
        sizes->input_weight = sc.in_changed;
        sizes->output_neurons = sc.out_changed;
        sizes->context_slots = sc.ctx_changed;
        sizes->output_bias_dirty = sc.bias_dirty;
        sizes->context_output_dirty = sc.ctx_out_dirty;
    }
    for (int i = 0; i < 5; ++i) {
        if (!dst[i] || lists[i].count == 0) continue;
        CUDA_CHECK(cudaMemcpy(dst[i], lists[i].list, lists[i].count * 4, cudaMemcpyDeviceToHost));
        std::sort(dst[i], dst[i] + lists[i].count);
    }
}

// PackedSparseModelUpdate::apply_to_model (parallel.rs:196-300) on the
// canonical model, then the same values into every resident lane.
// `close_window`: synchronize_packed_model first writes the canonical
// runtime's tracked changes into the lanes (closing the tracking window);
// commit_packed_host_model keeps the window open (cuda.rs:2861-2866).
void packed_update(LeoB200Device& dev, const LeoB200PackedUpdate& u, bool close_window = true) {
    if (dev.batch_open) throw LeoFailure("a story batch is in progress");
    const ModelSizes& z = dev.z;
    if (close_window) refresh_lanes_from_replay(dev);
    upload_lane_table(dev);
    const uint32_t lane_count = (uint32_t)dev.lanes.size();
    struct Item {
        const uint32_t* idx;
        const float* vals;
        uint64_t count;
        float* LaneParams::*member;
        size_t length;
        uint32_t row, row_len;
        const char* label;
    };
    const Item items[] = {
        {u.threshold_indices, u.threshold_values, u.threshold_count, &LaneParams::threshold, z.n, 1, 1, "threshold"},
        {u.recurrent_indices, u.recurrent_values, u.recurrent_count, &LaneParams::rec_weight, z.synapses, 1, 1,
         "recurrent"},
        {u.input_indices, u.input_values, u.input_count, &LaneParams::in_weight, z.inputs, 1, 1, "input"},
        {u.output_neurons, u.output_values_by_neuron, u.output_count, &LaneParams::out_weight, z.n, LEO_OUTPUT_STRIDE,
         LEO_OUTPUT_CLASSES, "output"},
    };
    for (const Item& it : items) {
        if (it.count == 0) continue;
        if (!it.idx || !it.vals) throw LeoFailure(std::string(it.label) + " packed sparse arrays are null");
        for (uint64_t i = 0; i < it.count; ++i)
            if (it.idx[i] >= it.length) throw LeoFailure(std::string(it.label) + " packed sparse index is outside model");
    }
    if (u.context_count && (!u.context_slots || !u.context_keys || !u.context_observations || !u.context_embeddings))
        throw LeoFailure("packed context rows are null");
    for (uint64_t i = 0; i < u.context_count; ++i)
        if (u.context_slots[i] >= z.ctx) throw LeoFailure("packed context slot is outside the model");
    for (const Item& it : items) {
        if (it.count == 0) continue;
        const size_t n = (size_t)it.count * it.row_len;
        Scratch buf(it.count * 4 + n * 4);
        uint32_t* d_idx = buf.as<uint32_t>();
        float* d_val = reinterpret_cast<float*>(d_idx + it.count);
        CUDA_CHECK(cudaMemcpyAsync(d_idx, it.idx, it.count * 4, cudaMemcpyHostToDevice, dev.stream));
        CUDA_CHECK(cudaMemcpyAsync(d_val, it.vals, n * 4, cudaMemcpyHostToDevice, dev.stream));
        write_rows_kernel<<<grid_for(n), 256, 0, dev.stream>>>(dev.canon.*it.member, d_idx, (uint32_t)it.count, it.row,
                                                              it.row_len, d_val);
        CUDA_CHECK(cudaGetLastError());
        if (lane_count) {
            std::vector<float*> ptrs(lane_count);
            for (uint32_t l = 0; l < lane_count; ++l) ptrs[l] = dev.lanes[l]->st.p.*it.member;
            CUDA_CHECK(cudaMemcpyAsync(dev.d_lane_ptrs, ptrs.data(), lane_count * sizeof(float*), cudaMemcpyHostToDevice,
                                       dev.stream));
            leo_launch_scatter_rows(dev.d_lane_ptrs, (int)lane_count, dev.canon.*it.member, d_idx, (uint32_t)it.count,
                                    it.row, it.row_len, dev.grid, dev.stream);
        }
        CUDA_CHECK(cudaStreamSynchronize(dev.stream));
    }
    if (u.context_count) {
        const uint32_t n = (uint32_t)u.context_count, d = (uint32_t)z.d;
        std::vector<ContextRow> rows(n);
        for (uint32_t i = 0; i < n; ++i) {
            rows[i].key = u.context_keys[i];
            rows[i].obs = u.context_observations[i];
        }
        const size_t head = ((size_t)n * 4 + 15) & ~(size_t)15;
        Scratch buf(head + n * sizeof(ContextRow) + (size_t)n * d * 4);
        uint32_t* d_slots = buf.as<uint32_t>();
        ContextRow* d_rows = reinterpret_cast<ContextRow*>(buf.as<char>() + head);
        float* d_emb = reinterpret_cast<float*>(d_rows + n);
        CUDA_CHECK(cudaMemcpyAsync(d_slots, u.context_slots, n * 4, cudaMemcpyHostToDevice, dev.stream));
        CUDA_CHECK(cudaMemcpyAsync(d_rows, rows.data(), n * sizeof(ContextRow), cudaMemcpyHostToDevice, dev.stream));
        CUDA_CHECK(cudaMemcpyAsync(d_emb, u.context_embeddings, (size_t)n * d * 4, cudaMemcpyHostToDevice, dev.stream));
        scatter_context_rows_kernel<<<grid_for((uint64_t)n * (d + 1)), 256, 0, dev.stream>>>(
            d_slots, n, d_rows, d_emb, d, dev.canon, dev.d_lanes, (int)lane_count);
        CUDA_CHECK(cudaGetLastError());
        CUDA_CHECK(cudaStreamSynchronize(dev.stream));
        for (uint32_t i = 0; i < n; ++i) {
            const uint32_t slot = u.context_slots[i];
            dev.ctx_keys[slot] = u.context_keys[i];
            dev.ctx_obs[slot] = u.context_observations[i];
            std::copy_n(u.context_embeddings + (size_t)i * d, d, dev.ctx_emb.begin() + (size_t)slot * d);
        }
    }
    std::vector<float*> bias_targets{dev.canon.out_bias}, ctx_targets{dev.canon.ctx_out};
    for (auto& l : dev.lanes) {
        bias_targets.push_back(l->st.p.out_bias);
        ctx_targets.push_back(l->st.p.ctx_out);
    }
    if (u.output_bias)
        for (float* t : bias_targets)
            CUDA_CHECK(cudaMemcpyAsync(t, u.output_bias, LEO_OUTPUT_CLASSES * 4, cudaMemcpyHostToDevice, dev.stream));
    if (u.context_output_weights)
        for (float* t : ctx_targets)
            CUDA_CHECK(cudaMemcpyAsync(t, u.context_output_weights, z.ctx_out * 4, cudaMemcpyHostToDevice, dev.stream));
    CUDA_CHECK(cudaStreamSynchronize(dev.stream));
    dev.generation = u.generation;
    dev.revision = u.parameter_revision;
    dev.stats = u.statistics;
}

// Sizes of the exported story deltas, then the copy into caller buffers.
void story_delta_sizes(const LeoB200Device& dev, LeoB200StoryDeltaSizes* sizes) {
    if (!sizes) return;
    *sizes = LeoB200StoryDeltaSizes{};
    sizes->stories = (uint32_t)dev.story_deltas.size();
    sizes->embedding_dim = (uint32_t)dev.z.d;
    for (const auto& sd : dev.story_deltas) {
        for (int t = 0; t < LEO_B200_DELTA_TENSORS; ++t) sizes->entries[t] += sd.index[t].size();
        sizes->context_entries += sd.ctx_key.size();
        for (int l = 0; l < LEO_B200_CHANGE_LISTS; ++l) sizes->changes[l] += sd.changed[l].size();
    }
}

void story_deltas_copy(const LeoB200Device& dev, const LeoB200StoryDeltas& out) {
    const size_t d = dev.z.d;
    for (int t = 0; t < LEO_B200_DELTA_TENSORS; ++t) {
        uint64_t at = 0;
        for (size_t s = 0; s < dev.story_deltas.size(); ++s) {
            const auto& sd = dev.story_deltas[s];
            if (out.offsets[t]) out.offsets[t][s] = at;
            const size_t n = sd.index[t].size();
            if (n && out.indices[t]) std::copy_n(sd.index[t].data(), n, out.indices[t] + at);
            if (n && out.deltas[t]) std::copy_n(sd.delta[t].data(), n, out.deltas[t] + at);
            at += n;
        }
        if (out.offsets[t]) out.offsets[t][dev.story_deltas.size()] = at;
    }
    uint64_t at = 0;
    for (size_t s = 0; s < dev.story_deltas.size(); ++s) {
        const auto& sd = dev.story_deltas[s];
        if (out.context_offsets) out.context_offsets[s] = at;
        const size_t n = sd.ctx_key.size();
        if (n) {
            if (out.context_orders) std::copy_n(sd.ctx_order.data(), n, out.context_orders + at);
            if (out.context_keys)
                for (size_t i = 0; i < n; ++i) out.context_keys[at + i] = sd.ctx_key[i];
            if (out.context_observation_increments)
                std::copy_n(sd.ctx_obs_inc.data(), n, out.context_observation_increments + at);
            if (out.context_embedding_deltas) std::copy_n(sd.ctx_emb.data(), n * d, out.context_embedding_deltas + at * d);
        }
        if (out.statistics) out.statistics[s] = sd.stats;
        if (out.revision_increments) out.revision_increments[s] = sd.revision;
        at += n;
    }
    if (out.context_offsets) out.context_offsets[dev.story_deltas.size()] = at;
    for (int l = 0; l < LEO_B200_CHANGE_LISTS; ++l) {
        uint64_t pos = 0;
        for (size_t s = 0; s < dev.story_deltas.size(); ++s) {
            const auto& c = dev.story_deltas[s].changed[l];
            if (out.change_offsets[l]) out.change_offsets[l][s] = pos;
            if (out.change_indices[l] && !c.empty()) std::copy(c.begin(), c.end(), out.change_indices[l] + pos);
            pos += c.size();
        }
        if (out.change_offsets[l]) out.change_offsets[l][dev.story_deltas.size()] = pos;
    }
    if (out.dirty_flags)
        for (size_t s = 0; s < dev.story_deltas.size(); ++s) out.dirty_flags[s] = dev.story_deltas[s].dirty;
}

// ---------------------------------------------------------------- sharded batch (multi-GPU)
// The logical batch's stories are split into contiguous ranges, one per rank
// (work_balanced_story_ranges, training.rs:926-964); every rank holds every
// story (for the serial replay) and runs its range on its lanes.  The merge
// is exchanged by the caller between the rank-local steps below, so that
// every rank ends with the same canonical model as one GPU running the whole
// batch (MultiGpuBatchTrainer::train_story_batch, training.rs:1212-1420, with
// the default serial canonical replay).

size_t tensor_elements(const TensorSpec& t) { return (size_t)t.length * t.row; }

void shard_begin(LeoB200Device& dev, const uint8_t* bytes, const uint64_t* offsets, uint32_t stories, uint32_t first,
                 uint32_t count, int permission) {
    if (dev.batch_open) throw LeoFailure("a story batch is already in progress");
    if (stories < 2) throw LeoFailure("a sharded batch needs at least two stories (one story trains the canonical model)");
    if (first > stories || count > stories - first) throw LeoFailure("shard range exceeds the batch");
    if (permission < 0 || permission > 3) throw LeoFailure("invalid permission");
    refresh_lanes_from_replay(dev);
    dev.doc_open = false;
    dev.batch_stories.assign(stories, {});
    for (uint32_t i = 0; i < stories; ++i) dev.batch_stories[i].assign(bytes + offsets[i], bytes + offsets[i + 1]);
    dev.batch_permission = permission;
    dev.single_story = false;
    dev.shard_mode = true;
    dev.shard_first = first;
    dev.shard_local_done = false;
    dev.steps_done = 0;
    dev.batch_steps = 0;
    ensure_lanes(dev, count);
    dev.lane_steps.assign(count, 0u);
    for (uint32_t i = 0; i < count; ++i) {
        Lane& lane = *dev.lanes[i];
        const auto& story = dev.batch_stories[first + i];
        const uint32_t steps = story.empty() ? 0 : (uint32_t)story.size() + 1;
        ensure_schedule(lane, story.size() + 1);
        reset_lane(dev, lane, 0ull, steps);
        dev.batch_steps = std::max(dev.batch_steps, steps);
        dev.lane_steps[i] = steps;
    }
    dev.batch_lanes = count;
    upload_lane_table(dev);
    build_schedules(dev, first, count, permission, dev.d_lanes);
    if (!dev.compact_total) {
        const auto specs = fixed_specs(dev.z);
        size_t blocks = 1;
        for (int t = 0; t < LEO_B200_FIXED_TENSORS; ++t) {
            dev.shard_list[t] = dev.mem.alloc<uint32_t>(std::max<size_t>(tensor_elements(specs[t]), 1));
            blocks = std::max(blocks, leo_compact_scratch_blocks(tensor_elements(specs[t])));
        }
        dev.compact_blocks = dev.mem.alloc<uint32_t>(blocks);
        dev.compact_total = dev.mem.alloc<uint32_t>(1);
        dev.shard_error = dev.mem.alloc<uint32_t>(1);
    }
    CUDA_CHECK(cudaEventRecord(dev.batch_start, dev.stream));
    dev.batch_open = true;
}

void require_shard(const LeoB200Device& dev) {
    if (!dev.batch_open || !dev.shard_mode) throw LeoFailure("no sharded story batch in progress");
}

// Finishes this rank's story pass and reports its stories.
void shard_local(LeoB200Device& dev, LeoB200ShardStory* out, float* losses_out) {
    require_shard(dev);
    if (dev.shard_local_done) throw LeoFailure("the shard's stories were already reported");
    batch_steps(dev, dev.batch_steps);
    CUDA_CHECK(cudaStreamSynchronize(dev.stream));
    const uint32_t L = dev.batch_lanes;
    dev.shard_scal.assign(L, LaneScalars{});
    size_t k = 0;
    dev.shard_ctx_blob.clear();
    dev.shard_ctx_slots.clear();
    const uint32_t d = (uint32_t)dev.z.d;
    for (uint32_t l = 0; l < L; ++l) {
        LaneScalars& sc = dev.shard_scal[l];
        read_scalars(dev, *dev.lanes[l], sc);
        check_error_flag(sc);
        add_work(dev, sc, true);
        const auto& story = dev.batch_stories[dev.shard_first + l];
        LeoB200ShardStory r{};
        r.loss_sum = sc.loss_sum;
        r.processed_bytes = sc.processed_bytes;
        r.targets = sc.targets;
        r.active_sum = sc.active_sum;
        r.active_peak = sc.active_peak;
        r.synaptic_events = sc.synaptic_events;
        r.numerical_rejections = sc.numerical_rejections;
        r.persistent_ticks = sc.persistent_ticks;
        r.revision_increment = sc.revision_increment;
        r.context_applied_steps = sc.context_applied_steps;
        r.story_bytes = story.size();
        if (out) out[l] = r;
        if (!story.empty()) {
            if (losses_out)
                CUDA_CHECK(cudaMemcpy(losses_out + k, dev.lanes[l]->step_loss, (story.size() + 1) * 4,
                                      cudaMemcpyDeviceToHost));
            k += story.size() + 1;
        }
        // keyed context deltas: u32 count, then per entry u32 order, u32
        // observation increment, u64 key, f32 delta[embedding_dim]
        auto deltas = collect_lane_context(dev, *dev.lanes[l], sc.ctx_changed, dev.shard_ctx_slots);
        auto put = [&](const void* p, size_t n) {
            const uint8_t* b = static_cast<const uint8_t*>(p);
            dev.shard_ctx_blob.insert(dev.shard_ctx_blob.end(), b, b + n);
        };
        uint32_t n = (uint32_t)deltas.size();
        put(&n, 4);
        for (const CtxDelta& u : deltas) {
            put(&u.order, 4);
            put(&u.obs_inc, 4);
            put(&u.key, 8);
            put(u.emb_delta.data(), (size_t)d * 4);
        }
    }
    dev.shard_local_done = true;
}

MergeTensor shard_tensor(LeoB200Device& dev, int t) {
    require_shard(dev);
    if (t < 0 || t >= LEO_B200_FIXED_TENSORS) throw LeoFailure("fixed tensor index out of range");
    if (!dev.shard_local_done) throw LeoFailure("report the shard's stories before merging");
    const TensorSpec spec = fixed_specs(dev.z)[t];
    const uint32_t resident = (uint32_t)dev.lanes.size(), L = dev.batch_lanes;
    std::vector<float*> ptrs(std::max(resident, 1u));
    std::vector<uint32_t*> lists(std::max(L, 1u));
    std::vector<uint32_t> counts(std::max(L, 1u));
    std::vector<uint8_t*> marks(std::max(L, 1u));
    for (uint32_t l = 0; l < resident; ++l) ptrs[l] = dev.lanes[l]->st.p.*spec.member;
    for (uint32_t l = 0; l < L; ++l) {
        LaneState& st = dev.lanes[l]->st;
        lists[l] = spec.list ? st.*spec.list : nullptr;
        counts[l] = spec.count ? dev.shard_scal[l].*spec.count : spec.length;
        marks[l] = spec.marks ? st.*spec.marks : nullptr;
    }
    if (resident)
        CUDA_CHECK(cudaMemcpyAsync(dev.d_lane_ptrs, ptrs.data(), resident * sizeof(float*), cudaMemcpyHostToDevice,
                                   dev.stream));
    if (L) {
        CUDA_CHECK(cudaMemcpyAsync(dev.d_lane_lists, lists.data(), L * sizeof(uint32_t*), cudaMemcpyHostToDevice, dev.stream));
        CUDA_CHECK(cudaMemcpyAsync(dev.d_lane_counts, counts.data(), L * 4, cudaMemcpyHostToDevice, dev.stream));
        CUDA_CHECK(cudaMemcpyAsync(dev.d_lane_marks, marks.data(), L * sizeof(uint8_t*), cudaMemcpyHostToDevice, dev.stream));
    }
    MergeTensor mt{};
    mt.lane_values = dev.d_lane_ptrs;
    mt.base = dev.canon.*spec.member;
    mt.lane_lists = spec.list ? dev.d_lane_lists : nullptr;
    mt.lane_counts = dev.d_lane_counts;
    mt.lane_marks = spec.marks ? dev.d_lane_marks : nullptr;
    mt.row = spec.row;
    mt.row_len = spec.row_len;
    mt.length = spec.length;
    mt.kind = spec.kind;
    return mt;
}

void shard_finish(LeoB200Device& dev, const LeoB200ShardStory* all, const float* all_losses, const uint8_t* ctx,
                  const uint64_t* ctx_offsets, uint64_t fixed_updates, LeoB200BatchReport* report,
                  LeoB200StorySummary* summaries, float* losses_out) {
    require_shard(dev);
    if (!dev.shard_local_done) throw LeoFailure("report the shard's stories before finishing");
    const uint32_t stories = (uint32_t)dev.batch_stories.size();
    const uint32_t d = (uint32_t)dev.z.d;
    LeoB200BatchReport rep{};
    rep.stories = stories;
    rep.workers = stories;
    rep.fixed_parameter_updates = fixed_updates;
    std::vector<std::vector<float>> losses(stories);
    size_t k = 0;
    for (uint32_t i = 0; i < stories; ++i) {
        const auto& story = dev.batch_stories[i];
        if (all[i].story_bytes != story.size()) throw LeoFailure("shard story reports do not match the batch");
        if (!story.empty()) {
            losses[i].assign(all_losses + k, all_losses + k + story.size() + 1);
            k += story.size() + 1;
        }
        rep.input_bytes += story.size();
    }
    // keyed context: every story's deltas in story order
    std::vector<std::vector<CtxDelta>> per_story(stories);
    for (uint32_t i = 0; i < stories; ++i) {
        const uint8_t* p = ctx + ctx_offsets[i];
        const uint8_t* end = ctx + ctx_offsets[i + 1];
        auto take = [&](void* dst, size_t n) {
            if (p + n > end) throw LeoFailure("malformed keyed context deltas");
            std::memcpy(dst, p, n);
            p += n;
        };
        uint32_t n = 0;
        take(&n, 4);
        for (uint32_t e = 0; e < n; ++e) {
            CtxDelta u{0, 0, std::vector<float>(d), 0};
            take(&u.order, 4);
            take(&u.obs_inc, 4);
            take(&u.key, 8);
            take(u.emb_delta.data(), (size_t)d * 4);
            if (u.order == 0 || u.order > dev.cfg.abi.context_max_order || u.key == 0)
                throw LeoFailure("invalid keyed context worker delta");
            per_story[i].push_back(std::move(u));
        }
        if (p != end) throw LeoFailure("malformed keyed context deltas");
    }
    const double canon_loss = dev.stats.training_loss_sum;
    rep.context_keys = merge_context_deltas(dev, per_story, stories, dev.shard_ctx_slots);
    // statistics and revision (parallel.rs:1115-1167) in story order
    for (uint32_t i = 0; i < stories; ++i) {
        const LeoB200ShardStory& sc = all[i];
        dev.stats.processed_bytes += sc.processed_bytes;
        dev.stats.processed_stories += (sc.story_bytes == 0 || dev.batch_permission == LEO_B200_FROZEN) ? 0 : 1;
        dev.stats.training_loss_sum += sc.loss_sum - canon_loss;
        dev.stats.training_targets += sc.targets;
        dev.stats.active_neurons_sum += sc.active_sum;
        dev.stats.active_neurons_peak = std::max<uint64_t>(dev.stats.active_neurons_peak, sc.active_peak);
        dev.stats.synaptic_events += sc.synaptic_events;
        dev.stats.numerical_rejections += sc.numerical_rejections;
        dev.stats.persistent_ticks += sc.persistent_ticks;
        dev.revision += sc.revision_increment;
        if (summaries) {
            summaries[i].training_loss_sum = 0.0;
            for (float v : losses[i]) summaries[i].training_loss_sum += (double)v;
            summaries[i].training_targets = sc.targets;
            summaries[i].active_neurons_sum = sc.active_sum;
            summaries[i].active_neurons_peak = sc.active_peak;
            summaries[i].synaptic_events = sc.synaptic_events;
            summaries[i].context_applied_steps = sc.context_applied_steps;
        }
    }
    double weighted = 0.0;
    size_t targets = 0;
    for (uint32_t i = 0; i < stories; ++i) {
        double sum = 0.0;
        for (float v : losses[i]) sum += (double)v;
        double mean = sum / (double)std::max<size_t>(losses[i].size(), 1);
        weighted += mean * (double)losses[i].size();
        targets += losses[i].size();
    }
    rep.targets = targets;
    rep.mean_loss = weighted / (double)std::max<size_t>(targets, 1);
    // Serial canonical replay of every story on every rank: identical inputs
    // and arithmetic keep the replicas bit-identical without a broadcast.
    LaneScalars replay_changes{};
    for (uint32_t i = 0; i < stories; ++i)
        replay_story(dev, dev.batch_stories[i], losses[i], dev.batch_permission, replay_changes, &rep);
    sync_replay_changes(dev, replay_changes);
    CUDA_CHECK(cudaEventRecord(dev.batch_stop, dev.stream));
    CUDA_CHECK(cudaEventSynchronize(dev.batch_stop));
    float batch_ms = 0.0f;
    CUDA_CHECK(cudaEventElapsedTime(&batch_ms, dev.batch_start, dev.batch_stop));
    dev.perf.batch_ms += batch_ms;
    dev.perf.batches += 1;
    dev.batch_open = false;
    dev.shard_mode = false;
    dev.shard_local_done = false;
    if (losses_out) {
        size_t j = 0;
        for (auto& l : losses)
            for (float v : l) losses_out[j++] = v;
    }
    if (report) *report = rep;
}

}  // namespace

// ============================================================================ C ABI
// Error text for C-ABI entry points defined in other translation units.
void leo_set_last_error(const char* what) { g_error = what; }

extern "C" {

const char* leo_b200_last_error(void) { return g_error.c_str(); }
uint32_t leo_b200_abi_version(void) { return LEO_CUDA_ABI_VERSION; }

int leo_b200_config_validate(const LeoB200Config* cfg) {
    const char* e = leo_host::validate_config(*cfg);
    if (*e) {
        g_error = e;
        return -1;
    }
    return 0;
}

int leo_b200_model_initialize(const LeoB200Config* cfg, int topology, LeoB200HostModel* model) {
    try {
        const char* e = leo_host::validate_config(*cfg);
        if (*e) throw LeoFailure(e);
        if (topology < 0 || topology > 2) throw LeoFailure("unknown topology");
        model->config = *cfg;
        leo_host::initialize_model(*cfg, topology, *model);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_model_validate(const LeoB200HostModel* model) {
    const char* e = leo_host::validate_model(*model);
    if (*e) {
        g_error = e;
        return -1;
    }
    return 0;
}

int leo_b200_training_state_hash(const LeoB200HostModel* model, uint8_t out[32]) {
    leo_host::training_state_hash(*model, out);
    return 0;
}

int leo_b200_open(int device, const LeoB200HostModel* canonical, uint32_t max_lanes, LeoB200Device** out) {
    try {
        const char* e = leo_host::validate_model(*canonical);
        if (*e) throw LeoFailure(e);
        if (max_lanes == 0 || max_lanes > 1024) throw LeoFailure("max_lanes must be in 1..=1024");
        auto dev = std::make_unique<LeoB200Device>();
        dev->device = device;
        CUDA_CHECK(cudaSetDevice(device));
        cudaDeviceProp prop;
        CUDA_CHECK(cudaGetDeviceProperties(&prop, device));
        if (prop.major < 10) throw LeoFailure("leo_b200 requires an sm_100 (Blackwell) device");
        CUDA_CHECK(cudaStreamCreateWithFlags(&dev->stream, cudaStreamNonBlocking));
        CUDA_CHECK(cudaEventCreate(&dev->batch_start));
        CUDA_CHECK(cudaEventCreate(&dev->batch_stop));
        CUDA_CHECK(cudaEventCreate(&dev->wave_start));
        CUDA_CHECK(cudaEventCreate(&dev->wave_stop));
        dev->cfg = canonical->config;
        dev->z = leo_host::sizes_of(dev->cfg);
        dev->kc = make_consts(*dev);
        const ModelSizes& z = dev->z;
        DeviceTopology& t = dev->kc.topo;
        t.n = (uint32_t)z.n;
        t.s = (uint32_t)z.s;
        t.f = (uint32_t)z.f;
        t.d = (uint32_t)z.d;
        t.k = dev->cfg.abi.context_max_order;
        t.spo = dev->cfg.abi.context_slots_per_order;
        t.ctx_slots = (uint32_t)z.ctx;
        t.blocks = dev->cfg.abi.block_count;
        t.npb = dev->cfg.abi.neurons_per_block;
        t.keep = dev->cfg.abi.max_active_per_block;
        t.max_active = dev->cfg.abi.max_active_global;
        // A tick's winners are bounded by the block capacity as well as the global cap.
        uint32_t winners = std::min<uint32_t>(t.blocks * t.keep, t.max_active);
        t.max_active = std::max<uint32_t>(t.max_active, winners);
        t.rec_word = dev->mem.alloc<uint32_t>(z.synapses);
        t.in_word = dev->mem.alloc<uint32_t>(z.inputs);
        t.neuron_type = dev->mem.alloc<uint8_t>(z.n);
        t.excitability = dev->mem.alloc<float>(z.n);
        dev->kc.event_capacity = 4u * t.max_active * t.s + t.f;
        dev->kc.event_bits = 1;
        while ((1u << dev->kc.event_bits) < dev->kc.event_capacity) ++dev->kc.event_bits;
        if (dev->kc.event_bits > 29) throw LeoFailure("event order exceeds 29 bits");
        // libm exception tables (leo_math.cuh) as open-addressing hash tables
        auto build_table = [&](const uint32_t* keys, const uint32_t* values, size_t count, uint32_t* mask_out) {
            size_t cap = 1024;
            while (cap < count * 3) cap <<= 1;
            std::vector<uint2> table(cap, make_uint2(0xffffffffu, 0u));
            uint32_t mask = (uint32_t)cap - 1u;
            for (size_t i = 0; i < count; ++i) {
                if (keys[i] == 0xffffffffu) continue;
                uint32_t h = (keys[i] * 0x9E3779B1u) & mask;
                while (table[h].x != 0xffffffffu) h = (h + 1u) & mask;
                table[h] = make_uint2(keys[i], values[i]);
            }
            uint2* d = dev->mem.alloc<uint2>(cap);
            CUDA_CHECK(cudaMemcpy(d, table.data(), cap * sizeof(uint2), cudaMemcpyHostToDevice));
            *mask_out = mask;
            return (const uint2*)d;
        };
        dev->kc.exp_table = build_table(leo_exp_exception_keys, leo_exp_exception_values, LEO_EXP_EXCEPTIONS,
                                        &dev->kc.exp_mask);
        dev->kc.log_table = build_table(leo_log_exception_keys, leo_log_exception_values, LEO_LOG_EXCEPTIONS,
                                        &dev->kc.log_mask);
        // canonical parameters
        LaneParams& p = dev->canon;
        p.threshold = dev->mem.alloc<float>(z.n);
        p.rec_weight = dev->mem.alloc<float>(z.synapses);
        p.in_weight = dev->mem.alloc<float>(z.inputs);
        p.out_weight = dev->mem.alloc<float>(z.n * LEO_OUTPUT_STRIDE);
        p.out_bias = dev->mem.alloc<float>(LEO_OUTPUT_STRIDE);
        p.ctx_keys = dev->mem.alloc<unsigned long long>(z.ctx);
        p.ctx_obs = dev->mem.alloc<uint32_t>(z.ctx);
        p.ctx_emb = dev->mem.alloc<float>(z.ctx_emb);
        p.ctx_out = dev->mem.alloc<float>(z.ctx_out);
        // merge scratch sized for the largest tensor
        size_t longest = std::max({z.n, z.synapses, z.inputs, z.ctx_out, (size_t)LEO_OUTPUT_STRIDE});
        dev->scratch.union_mark = dev->mem.alloc<uint8_t>((longest + 3) & ~(size_t)3);
        dev->scratch.union_list = dev->mem.alloc<uint32_t>(longest);
        dev->scratch.union_count = dev->mem.alloc<uint32_t>(1);
        dev->scratch.updates = dev->mem.alloc<uint32_t>(1);
        dev->scratch.error_flag = dev->mem.alloc<uint32_t>(1);
        dev->lane_capacity = max_lanes;
        dev->d_lane_ptrs = dev->mem.alloc<float*>(max_lanes);
        dev->d_lane_lists = dev->mem.alloc<uint32_t*>(max_lanes);
        dev->d_lane_counts = dev->mem.alloc<uint32_t>(max_lanes);
        dev->d_lane_marks = dev->mem.alloc<uint8_t*>(max_lanes);
        dev->d_lanes = dev->mem.alloc<LaneState>(max_lanes);
        dev->ctx_stage_rows = dev->mem.alloc<ContextRow>(z.ctx);
        dev->ctx_stage_emb = dev->mem.alloc<float>(z.ctx_emb);
        dev->ctx_sync_slots = dev->mem.alloc<uint32_t>(z.ctx);
        dev->d_replay = dev->mem.alloc<LaneState>(1);
        dev->d_lane_load = dev->mem.alloc<uint32_t>(max_lanes + 1);
        dev->d_group_table = dev->mem.alloc<LaneState>(max_lanes);
        for (cudaStream_t& st : dev->aux) CUDA_CHECK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
        CUDA_CHECK(cudaEventCreateWithFlags(&dev->fork, cudaEventDisableTiming));
        for (cudaEvent_t& ev : dev->join) CUDA_CHECK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
        dev->sm_count = prop.multiProcessorCount;
        // replay lane: canonical parameters, private transient state
        plan_segments(*dev, canonical->recurrent_target, canonical->input_target, true);
        dev->replay = std::make_unique<Lane>();
        dev->replay->st.p = dev->canon;
        allocate_lane_transient(*dev, *dev->replay);
        dev->grid = prop.multiProcessorCount * 4;
        if (leo_wavefront_smem_bytes(dev->kc) > 160 * 1024) throw LeoFailure("block winners exceed shared memory");
        CUDA_CHECK(leo_wavefront_configure());
        if (leo_wavefront_max_clusters(16, dev->kc, &dev->fit16) != cudaSuccess) {
            cudaGetLastError();
            dev->fit16 = 0;
        }
        if (leo_wavefront_max_clusters(8, dev->kc, &dev->fit8) != cudaSuccess) {
            cudaGetLastError();
            dev->fit8 = 0;
        }
        if (leo_wavefront_max_clusters(4, dev->kc, &dev->fit4) != cudaSuccess) {
            cudaGetLastError();
            dev->fit4 = 0;
        }
        dev->replay->st.load_out = dev->d_lane_load + max_lanes;
        if (leo_wavefront_grid_ctas(dev->kc, dev->sm_count, &dev->grid_ctas) != cudaSuccess) {
            cudaGetLastError();
            dev->grid_ctas = 0;
        }
        dev->ctx_lane_offset = dev->mem.alloc<uint32_t>(max_lanes + 1);
        dev->ctx_device_merge = leo_context_apply_smem(dev->cfg.abi.context_slots_per_order) <= 200u * 1024u &&
                                leo_context_merge_configure() == cudaSuccess;
        upload_model(*dev, *canonical);
        *out = dev.release();
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

void leo_b200_close(LeoB200Device* dev) {
    if (!dev) return;
    cudaSetDevice(dev->device);
    cudaStreamSynchronize(dev->stream);
    cudaStream_t s = dev->stream;
    if (dev->wave_start) cudaEventDestroy(dev->wave_start);
    if (dev->wave_stop) cudaEventDestroy(dev->wave_stop);
    if (dev->batch_start) cudaEventDestroy(dev->batch_start);
    if (dev->batch_stop) cudaEventDestroy(dev->batch_stop);
    if (dev->fork) cudaEventDestroy(dev->fork);
    for (cudaEvent_t ev : dev->join)
        if (ev) cudaEventDestroy(ev);
    for (cudaStream_t st : dev->aux)
        if (st) cudaStreamDestroy(st);
    delete dev;
    cudaStreamDestroy(s);
}

int leo_b200_upload_canonical(LeoB200Device* dev, const LeoB200HostModel* model) {
    try {
        const char* e = leo_host::validate_model(*model);
        if (*e) throw LeoFailure(e);
        CUDA_CHECK(cudaSetDevice(dev->device));
        const std::vector<uint2> seg = plan_segments(*dev, model->recurrent_target, model->input_target, false);
        bool same = seg.size() == dev->seg_host.size();
        for (size_t n = 0; same && n < seg.size(); ++n)
            same = seg[n].x == dev->seg_host[n].x && (seg[n].y & LEO_SEG_CAPACITY) == (dev->seg_host[n].y & LEO_SEG_CAPACITY);
        if (!same) throw LeoFailure("the recurrent topology changed: open a new backend for it");
        upload_model(*dev, *model);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_download_model(LeoB200Device* dev, LeoB200HostModel* model) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        download_params(*dev, dev->canon, *model);
        model->generation = dev->generation;
        model->parameter_revision = dev->revision;
        model->statistics = dev->stats;
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

uint64_t leo_b200_canonical_tick(LeoB200Device* dev) { return dev->canonical_tick; }

int leo_b200_set_canonical_tick(LeoB200Device* dev, uint64_t tick) {
    dev->canonical_tick = tick;
    return 0;
}

int leo_b200_batch_begin(LeoB200Device* dev, const uint8_t* bytes, const uint64_t* offsets, uint32_t stories,
                         int permission) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        batch_begin(*dev, bytes, offsets, stories, permission);
        return 0;
    } catch (const std::exception& e) {
        dev->batch_open = false;
        return fail(e);
    }
}

int leo_b200_batch_steps(LeoB200Device* dev, uint32_t count, uint32_t* steps_done) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        batch_steps(*dev, count);
        CUDA_CHECK(cudaStreamSynchronize(dev->stream));
        if (steps_done) *steps_done = dev->steps_done;
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_batch_finish(LeoB200Device* dev, LeoB200BatchReport* report, LeoB200StorySummary* summaries,
                          float* losses) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        batch_finish(*dev, report, summaries, losses);
        return 0;
    } catch (const std::exception& e) {
        dev->batch_open = false;
        return fail(e);
    }
}

int leo_b200_train_story_batch(LeoB200Device* dev, const uint8_t* bytes, const uint64_t* offsets, uint32_t stories,
                               int permission, LeoB200BatchReport* report, LeoB200StorySummary* summaries,
                               float* losses) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        batch_begin(*dev, bytes, offsets, stories, permission);
        batch_finish(*dev, report, summaries, losses);
        return 0;
    } catch (const std::exception& e) {
        dev->batch_open = false;
        return fail(e);
    }
}

// Runs one batch on story lanes (a single story too) and ends it in `mode`.
int trait_batch(LeoB200Device* dev, const uint8_t* bytes, const uint64_t* offsets, uint32_t stories, int permission,
                LeoB200BatchReport* report, LeoB200StorySummary* summaries, float* losses, uint64_t* ranges,
                uint32_t* range_counts, FinishMode mode) {
    CUDA_CHECK(cudaSetDevice(dev->device));
    dev->force_lanes = true;
    try {
        batch_begin(*dev, bytes, offsets, stories, permission);
    } catch (...) {
        dev->force_lanes = false;
        throw;
    }
    dev->force_lanes = false;
    batch_finish(*dev, report, summaries, losses, mode, ranges, range_counts);
    return 0;
}

int leo_b200_training_story_batch(LeoB200Device* dev, const uint8_t* bytes, const uint64_t* offsets, uint32_t stories,
                                  int permission, LeoB200BatchReport* report, LeoB200StorySummary* summaries,
                                  float* losses, uint64_t* ranges, uint32_t* range_counts) {
    try {
        // backend.rs:587-589: fewer than two stories are not a device batch.
        if (stories < 2) return LEO_B200_UNSUPPORTED;
        return trait_batch(dev, bytes, offsets, stories, permission, report, summaries, losses, ranges, range_counts,
                           FinishMode::kNoReplay);
    } catch (const std::exception& e) {
        dev->batch_open = false;
        return fail(e);
    }
}

int leo_b200_training_story_batch_deltas(LeoB200Device* dev, const uint8_t* bytes, const uint64_t* offsets,
                                         uint32_t stories, int permission, LeoB200BatchReport* report,
                                         LeoB200StorySummary* summaries, float* losses, uint64_t* ranges,
                                         uint32_t* range_counts, LeoB200StoryDeltaSizes* sizes) {
    try {
        if (stories == 0) return LEO_B200_UNSUPPORTED;
        dev->story_deltas.clear();
        trait_batch(dev, bytes, offsets, stories, permission, report, summaries, losses, ranges, range_counts,
                    FinishMode::kDeltas);
        story_delta_sizes(*dev, sizes);
        return 0;
    } catch (const std::exception& e) {
        dev->batch_open = false;
        return fail(e);
    }
}

int leo_b200_story_deltas(LeoB200Device* dev, const LeoB200StoryDeltas* out) {
    try {
        if (!out) throw LeoFailure("story delta buffers are null");
        story_deltas_copy(*dev, *out);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_begin_document(LeoB200Device* dev) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        doc_begin(*dev);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_reset_transient_state(LeoB200Device* dev) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        doc_begin(*dev);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_training_step_batch(LeoB200Device* dev, const uint32_t* symbols, const int32_t* targets, uint32_t count,
                                 int permission, float* losses, uint32_t* active_neurons) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        doc_steps(*dev, symbols, targets, count, permission, losses, active_neurons);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_advance_frozen_batch(LeoB200Device* dev, const uint32_t* symbols, const int32_t* targets,
                                  uint32_t count) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        doc_steps(*dev, symbols, targets, count, LEO_B200_FROZEN, nullptr, nullptr);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_enable_parameter_tracking(LeoB200Device* dev) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        tracking_enable(*dev);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_parameter_changes(LeoB200Device* dev, LeoB200ParameterChangeSizes* sizes,
                               const LeoB200ParameterChanges* changes) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        tracking_changes(*dev, sizes, changes);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_synchronize_packed_model(LeoB200Device* dev, const LeoB200PackedUpdate* update) {
    try {
        if (!update) throw LeoFailure("packed update is null");
        CUDA_CHECK(cudaSetDevice(dev->device));
        packed_update(*dev, *update);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_commit_packed_host_model(LeoB200Device* dev, const LeoB200PackedUpdate* update) {
    try {
        if (!update) throw LeoFailure("packed update is null");
        CUDA_CHECK(cudaSetDevice(dev->device));
        packed_update(*dev, *update, false);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_shard_begin(LeoB200Device* dev, const uint8_t* bytes, const uint64_t* offsets, uint32_t stories,
                         uint32_t first, uint32_t count, int permission) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        shard_begin(*dev, bytes, offsets, stories, first, count, permission);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_shard_local(LeoB200Device* dev, LeoB200ShardStory* stories, float* losses, size_t* context_bytes) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        shard_local(*dev, stories, losses);
        if (context_bytes) *context_bytes = dev->shard_ctx_blob.size();
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_shard_context(LeoB200Device* dev, uint8_t* out, size_t capacity) {
    try {
        require_shard(*dev);
        if (capacity < dev->shard_ctx_blob.size()) throw LeoFailure("context buffer too small");
        if (!dev->shard_ctx_blob.empty()) std::memcpy(out, dev->shard_ctx_blob.data(), dev->shard_ctx_blob.size());
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_shard_tensor_elements(LeoB200Device* dev, uint32_t tensor, size_t* elements) {
    if (tensor >= LEO_B200_FIXED_TENSORS) return fail(LeoFailure("fixed tensor index out of range"));
    *elements = tensor_elements(fixed_specs(dev->z)[tensor]);
    return 0;
}

int leo_b200_shard_marks(LeoB200Device* dev, uint32_t tensor, uint8_t* marks) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        MergeTensor mt = shard_tensor(*dev, (int)tensor);
        const size_t n = tensor_elements(fixed_specs(dev->z)[tensor]);
        CUDA_CHECK(cudaMemsetAsync(marks, 0, n, dev->stream));
        leo_launch_shard_marks(mt, (int)dev->batch_lanes, marks, dev->grid, dev->stream);
        CUDA_CHECK(cudaGetLastError());
        CUDA_CHECK(cudaStreamSynchronize(dev->stream));
        dev->perf.launches += 1;
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_shard_plan(LeoB200Device* dev, uint32_t tensor, const uint8_t* marks, uint32_t* count) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        shard_tensor(*dev, (int)tensor);
        const size_t n = tensor_elements(fixed_specs(dev->z)[tensor]);
        leo_launch_compact(marks, n, dev->shard_list[tensor], dev->compact_total, dev->compact_blocks, dev->stream);
        CUDA_CHECK(cudaGetLastError());
        uint32_t total = 0;
        CUDA_CHECK(cudaMemcpyAsync(&total, dev->compact_total, 4, cudaMemcpyDeviceToHost, dev->stream));
        CUDA_CHECK(cudaStreamSynchronize(dev->stream));
        dev->shard_count[tensor] = total;
        dev->perf.launches += 3;
        *count = total;
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_shard_accumulate(LeoB200Device* dev, uint32_t tensor, double* partial, int first) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        MergeTensor mt = shard_tensor(*dev, (int)tensor);
        CUDA_CHECK(cudaMemsetAsync(dev->shard_error, 0, 4, dev->stream));
        leo_launch_shard_accumulate(mt.lane_values, (int)dev->batch_lanes, mt.base, dev->shard_list[tensor],
                                    dev->shard_count[tensor], partial, first, dev->shard_error, dev->grid, dev->stream);
        CUDA_CHECK(cudaGetLastError());
        uint32_t err = 0;
        CUDA_CHECK(cudaMemcpyAsync(&err, dev->shard_error, 4, cudaMemcpyDeviceToHost, dev->stream));
        CUDA_CHECK(cudaStreamSynchronize(dev->stream));
        dev->perf.launches += 1;
        if (err) throw LeoFailure("invalid sparse worker parameter delta");
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_shard_finalize(LeoB200Device* dev, uint32_t tensor, const double* partial, float* values) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        MergeTensor mt = shard_tensor(*dev, (int)tensor);
        CUDA_CHECK(cudaMemsetAsync(dev->shard_error, 0, 4, dev->stream));
        leo_launch_shard_finalize(mt.base, dev->shard_list[tensor], dev->shard_count[tensor], partial, values,
                                  (double)dev->batch_stories.size(), mt.kind, dev->cfg.abi.weight_min,
                                  dev->cfg.abi.weight_max, dev->kc.topo.neuron_type, (uint32_t)dev->z.s,
                                  dev->shard_error, dev->grid, dev->stream);
        CUDA_CHECK(cudaGetLastError());
        uint32_t err = 0;
        CUDA_CHECK(cudaMemcpyAsync(&err, dev->shard_error, 4, cudaMemcpyDeviceToHost, dev->stream));
        CUDA_CHECK(cudaStreamSynchronize(dev->stream));
        dev->perf.launches += 1;
        if (err) throw LeoFailure("merged parameter became non-finite");
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_shard_commit(LeoB200Device* dev, uint32_t tensor, const float* values) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        MergeTensor mt = shard_tensor(*dev, (int)tensor);
        leo_launch_shard_commit(mt.base, dev->shard_list[tensor], dev->shard_count[tensor], values, mt.lane_values,
                                (int)dev->lanes.size(), dev->grid, dev->stream);
        leo_launch_shard_sync_own(mt, (int)dev->batch_lanes, dev->grid, dev->stream);
        CUDA_CHECK(cudaGetLastError());
        CUDA_CHECK(cudaStreamSynchronize(dev->stream));
        dev->perf.launches += 2;
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_shard_finish(LeoB200Device* dev, const LeoB200ShardStory* stories, const float* losses,
                          const uint8_t* context, const uint64_t* context_offsets, uint64_t fixed_updates,
                          LeoB200BatchReport* report, LeoB200StorySummary* summaries, float* losses_out) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        shard_finish(*dev, stories, losses, context, context_offsets, fixed_updates, report, summaries, losses_out);
        return 0;
    } catch (const std::exception& e) {
        dev->batch_open = false;
        dev->shard_mode = false;
        dev->shard_local_done = false;
        return fail(e);
    }
}

int leo_b200_state_digest(LeoB200Device* dev, uint8_t out[32]) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        const ModelSizes& z = dev->z;
        std::vector<float> thr(z.n), exc(z.n), rw(z.synapses), iw(z.inputs), ow(z.outputs), bias(LEO_B200_OUTPUT_CLASSES);
        std::vector<float> emb(z.ctx_emb), cow(z.ctx_out);
        std::vector<uint8_t> nt(z.n), rb(z.synapses), rd(z.synapses), ib(z.inputs);
        std::vector<uint32_t> rt(z.synapses), it(z.inputs), obs(z.ctx);
        std::vector<uint64_t> keys(z.ctx);
        LeoB200HostModel m{};
        m.threshold = thr.data(); m.excitability = exc.data(); m.neuron_type = nt.data();
        m.recurrent_target = rt.data(); m.recurrent_branch = rb.data(); m.recurrent_delay = rd.data();
        m.recurrent_weight = rw.data(); m.input_target = it.data(); m.input_branch = ib.data();
        m.input_weight = iw.data(); m.output_weight = ow.data(); m.output_bias = bias.data();
        m.context_keys = keys.data(); m.context_embeddings = emb.data(); m.context_observations = obs.data();
        m.context_output_weight = cow.data();
        download_params(*dev, dev->canon, m);
        m.generation = dev->generation;
        m.parameter_revision = dev->revision;
        m.statistics = dev->stats;
        leo_host::training_state_hash(m, out);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// Debug/parity inspection: the learned parameters of one story lane (or the
// canonical model when lane == UINT32_MAX) in the checkpoint layout.
int leo_b200_lane_model(LeoB200Device* dev, uint32_t lane, LeoB200HostModel* model) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        if (lane != 0xffffffffu && lane >= dev->lanes.size()) throw LeoFailure("lane out of range");
        const LaneParams& p = lane == 0xffffffffu ? dev->canon : dev->lanes[lane]->st.p;
        download_params(*dev, p, *model);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// Debug/parity inspection of one lane's transient state by name; `lane ==
// UINT32_MAX` selects the canonical (replay / single-story) lane.  Arrays are
// converted to the reference runtime's layout (runtime.rs:112-186).
int leo_b200_lane_array(LeoB200Device* dev, uint32_t lane, const char* name, void* out, size_t capacity,
                        size_t* written) {
    try {
        CUDA_CHECK(cudaSetDevice(dev->device));
        CUDA_CHECK(cudaStreamSynchronize(dev->stream));
        if (lane != 0xffffffffu && lane >= dev->lanes.size()) throw LeoFailure("lane out of range");
        Lane& L = lane == 0xffffffffu ? *dev->replay : *dev->lanes[lane];
        const ModelSizes& z = dev->z;
        std::string k(name);
        LaneScalars sc;
        CUDA_CHECK(cudaMemcpy(&sc, L.st.sc, sizeof(sc), cudaMemcpyDeviceToHost));
        auto emit = [&](const void* src, size_t bytes) {
            if (bytes > capacity) throw LeoFailure("capacity too small for " + k);
            std::memcpy(out, src, bytes);
            *written = bytes;
        };
        if (k == "scalars") {
            emit(&sc, sizeof(sc));
            return 0;
        }
        std::vector<NeuronHot> hot;
        std::vector<NeuronCold> cold;
        auto load_neurons = [&]() {
            hot.resize(z.n);
            cold.resize(z.n);
            CUDA_CHECK(cudaMemcpy(hot.data(), L.st.hot, z.n * sizeof(NeuronHot), cudaMemcpyDeviceToHost));
            CUDA_CHECK(cudaMemcpy(cold.data(), L.st.cold, z.n * sizeof(NeuronCold), cudaMemcpyDeviceToHost));
        };
        std::vector<float> f;
        std::vector<uint64_t> u;
        if (k == "membrane" || k == "fatigue" || k == "adaptation_fast" || k == "adaptation_medium" ||
            k == "adaptation_slow" || k == "activation" || k == "selection_surrogate" || k == "refractory_until" ||
            k == "branch_last_tick" || k == "neuron_last_tick") {
            load_neurons();
            uint32_t tick = dev->steps_done;  // ticks are relative to the lane's reset
            for (size_t n = 0; n < z.n; ++n) {
                if (k == "membrane") f.push_back(cold[n].membrane);
                else if (k == "fatigue") f.push_back(cold[n].fatigue);
                else if (k == "adaptation_fast") f.push_back(cold[n].adaptation[0]);
                else if (k == "adaptation_medium") f.push_back(cold[n].adaptation[1]);
                else if (k == "adaptation_slow") f.push_back(cold[n].adaptation[2]);
                else if (k == "activation") f.push_back(hot[n].activation);
                else if (k == "selection_surrogate")
                    f.push_back((hot[n].tag >> 2) == tick ? hot[n].surrogate : 0.0f);
                else if (k == "refractory_until") u.push_back(sc.base_tick + hot[n].refractory_until);
                else if (k == "branch_last_tick") u.push_back(sc.base_tick + cold[n].branch_tick);
                else u.push_back(sc.base_tick + cold[n].neuron_tick);
            }
            (void)tick;
        } else if (k == "branches") {
            std::vector<float4> br(z.n);
            CUDA_CHECK(cudaMemcpy(br.data(), L.st.branches, z.n * sizeof(float4), cudaMemcpyDeviceToHost));
            for (auto& b : br) {
                f.push_back(b.x);
                f.push_back(b.y);
                f.push_back(b.z);
                f.push_back(b.w);
            }
        } else if (k.rfind("rec_", 0) == 0 || k.rfind("input_", 0) == 0) {
            bool input = k.rfind("input_", 0) == 0;
            size_t count = input ? z.inputs : z.synapses;
            std::vector<Trace> tr(count);
            CUDA_CHECK(cudaMemcpy(tr.data(), input ? L.st.in_traces : L.st.traces, count * sizeof(Trace), cudaMemcpyDeviceToHost));
            std::string field = k.substr(input ? 6 : 4);
            for (auto& t : tr) {
                if (field == "branch_sensitivity") f.push_back(t.branch_sens);
                else if (field == "membrane_sensitivity") f.push_back(t.membrane_sens);
                else if (field == "fatigue_sensitivity") f.push_back(t.fatigue_sens);
                else if (field == "adaptation_fast_sensitivity") f.push_back(t.adaptation_sens[0]);
                else if (field == "adaptation_medium_sensitivity") f.push_back(t.adaptation_sens[1]);
                else if (field == "adaptation_slow_sensitivity") f.push_back(t.adaptation_sens[2]);
                else if (field == "eligibility") f.push_back(t.eligibility);
                else if (field == "last_tick") u.push_back(sc.base_tick + (t.tick_mark >> 1));
                else throw LeoFailure("unknown lane array: " + k);
            }
        } else if (k == "eligible_recurrent_slots" || k == "eligible_input_slots") {
            bool input = k == "eligible_input_slots";
            uint32_t count = input ? sc.in_elig_count[sc.elig_cur] : sc.elig_count[sc.elig_cur];
            std::vector<uint2> e(count);
            if (count)
                CUDA_CHECK(cudaMemcpy(e.data(), input ? L.st.in_elig[sc.elig_cur] : L.st.elig[sc.elig_cur],
                                      count * sizeof(uint2), cudaMemcpyDeviceToHost));
            for (auto& x : e) u.push_back(x.x);
        } else if (k == "active") {
            uint32_t entry = (dev->steps_done + LEO_RING - 1) % LEO_RING;
            uint32_t count = dev->steps_done ? sc.ring_count[entry] : 0;
            std::vector<uint32_t> src(count);
            if (count)
                CUDA_CHECK(cudaMemcpy(src.data(), L.st.ring_src + (size_t)entry * dev->kc.topo.max_active, count * 4,
                                      cudaMemcpyDeviceToHost));
            for (auto x : src) u.push_back(x);
        } else if (k == "probabilities" || k == "errors") {
            f.resize(LEO_B200_OUTPUT_CLASSES);
            CUDA_CHECK(cudaMemcpy(f.data(), k == "errors" ? L.st.errors : L.st.probs, f.size() * 4, cudaMemcpyDeviceToHost));
        } else if (k == "step_loss") {
            f.resize(dev->steps_done);
            if (!f.empty()) CUDA_CHECK(cudaMemcpy(f.data(), L.step_loss, f.size() * 4, cudaMemcpyDeviceToHost));
        } else if (k == "population_inhibition") {
            f.push_back(sc.population_inhibition);
        } else if (k == "changed_context_slots" || k == "changed_threshold" || k == "changed_recurrent_weight" ||
                   k == "changed_input_weight" || k == "changed_output_neurons") {
            uint32_t* list = k == "changed_context_slots" ? L.st.ctx_list
                             : k == "changed_threshold"   ? L.st.thr_list
                             : k == "changed_recurrent_weight" ? L.st.rec_list
                             : k == "changed_input_weight"     ? L.st.in_list
                                                               : L.st.out_list;
            uint32_t count = k == "changed_context_slots" ? sc.ctx_changed
                             : k == "changed_threshold"   ? sc.thr_changed
                             : k == "changed_recurrent_weight" ? sc.rec_changed
                             : k == "changed_input_weight"     ? sc.in_changed
                                                               : sc.out_changed;
            std::vector<uint32_t> v(count);
            if (count) CUDA_CHECK(cudaMemcpy(v.data(), list, count * 4, cudaMemcpyDeviceToHost));
            for (auto x : v) u.push_back(x);
        } else {
            throw LeoFailure("unknown lane array: " + k);
        }
        if (!f.empty() || u.empty()) emit(f.data(), f.size() * 4);
        else emit(u.data(), u.size() * 8);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_set_cluster_sizes(LeoB200Device* dev, uint32_t story_cluster, uint32_t replay_cluster) {
    auto ok = [](uint32_t c) { return c == 0 || c == 1 || c == 2 || c == 4 || c == 8 || c == 16; };
    if (!ok(story_cluster) || !(ok(replay_cluster) || replay_cluster == LEO_B200_WHOLE_GPU)) {
        g_error = "cluster sizes must be 0 (default), 1, 2, 4, 8 or 16 (replay also LEO_B200_WHOLE_GPU)";
        return -1;
    }
    if (replay_cluster == LEO_B200_WHOLE_GPU && dev->grid_ctas == 0) {
        g_error = "the whole-GPU replay launch is not available on this device";
        return -1;
    }
    dev->story_cluster_request = story_cluster;
    dev->replay_cluster_request = replay_cluster;
    return 0;
}

int leo_b200_set_device_context_merge(LeoB200Device* dev, int enable) {
    if (enable && leo_context_apply_smem(dev->cfg.abi.context_slots_per_order) > 200u * 1024u)
        return fail(LeoFailure("context slots per order exceed the device merge's shared-memory tables"));
    dev->ctx_device_merge = enable != 0;
    return 0;
}

int leo_b200_set_story_chunk(LeoB200Device* dev, uint32_t steps) {
    if (steps == 0) return fail(LeoFailure("story chunk must be at least one step"));
    dev->story_chunk = steps;
    return 0;
}

int leo_b200_set_hub_threshold(LeoB200Device* dev, uint32_t min_in_degree, uint32_t cta_events,
                               uint32_t thread_events) {
    try {
        if (cta_events > 2048) throw LeoFailure("cta_events must be in 0..=2048 (0: default 256)");
        if (thread_events > 16) throw LeoFailure("thread_events must be in 0..=16 (0: default 16)");
        if (!dev->lanes.empty() || dev->batch_open)
            throw LeoFailure("the hub threshold must be set before the first story batch");
        CUDA_CHECK(cudaSetDevice(dev->device));
        const ModelSizes& z = dev->z;
        std::vector<uint32_t> rec(z.synapses), in(z.inputs);
        CUDA_CHECK(cudaMemcpy(rec.data(), dev->kc.topo.rec_word, z.synapses * 4, cudaMemcpyDeviceToHost));
        CUDA_CHECK(cudaMemcpy(in.data(), dev->kc.topo.in_word, z.inputs * 4, cudaMemcpyDeviceToHost));
        for (auto& w : rec) w &= LEO_TARGET_MASK;
        for (auto& w : in) w &= LEO_TARGET_MASK;
        dev->cta_min_in_degree = min_in_degree;
        dev->cta_events = cta_events ? cta_events : 256;
        dev->thread_events = thread_events ? thread_events : 16;
        plan_segments(*dev, rec.data(), in.data(), true);  // capacities are unchanged: lane buffers stay valid
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_set_segment_capacity_limit(LeoB200Device* dev, uint32_t limit) {
    try {
        if (!dev->lanes.empty() || dev->batch_open)
            throw LeoFailure("the segment capacity limit must be set before the first story batch");
        CUDA_CHECK(cudaSetDevice(dev->device));
        const ModelSizes& z = dev->z;
        std::vector<uint32_t> rec(z.synapses), in(z.inputs);
        CUDA_CHECK(cudaMemcpy(rec.data(), dev->kc.topo.rec_word, z.synapses * 4, cudaMemcpyDeviceToHost));
        CUDA_CHECK(cudaMemcpy(in.data(), dev->kc.topo.in_word, z.inputs * 4, cudaMemcpyDeviceToHost));
        for (auto& w : rec) w &= LEO_TARGET_MASK;
        for (auto& w : in) w &= LEO_TARGET_MASK;
        // Capacities only shrink below the ones the replay lane was sized
        // for at open, and story lanes are sized at their first batch.
        dev->seg_capacity_limit = limit;
        plan_segments(*dev, rec.data(), in.data(), true);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int leo_b200_hub_count(LeoB200Device* dev, uint32_t* hubs, uint64_t* events_per_lane) {
    if (hubs) *hubs = dev->kc.topo.cta_count;
    if (events_per_lane) *events_per_lane = dev->seg_events_total;
    return 0;
}

int leo_b200_perf_stats(LeoB200Device* dev, LeoB200PerfStats* out) {
    *out = dev->perf;
    out->fit_clusters[0] = dev->fit4;
    out->fit_clusters[1] = dev->fit8;
    out->fit_clusters[2] = dev->fit16;
    out->sm_count = dev->sm_count;
    return 0;
}

int leo_b200_reset_perf_stats(LeoB200Device* dev) {
    dev->perf = LeoB200PerfStats{};
    return 0;
}

size_t leo_b200_device_bytes(LeoB200Device* dev) {
    size_t total = dev->mem.bytes + dev->replay->mem.bytes;
    for (auto& l : dev->lanes) total += l->mem.bytes;
    return total;
}

}  // extern "C"
