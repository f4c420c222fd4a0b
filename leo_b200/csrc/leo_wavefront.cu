// Persistent per-byte wavefront for sm_100a.
//
// One thread-block cluster owns one lane (a logical story worker, or the
// canonical replay lane) and runs a span of its step schedule in one launch.
// The phases of every step are separated by cluster barriers
// (barrier.cluster.arrive.release / wait.acquire) instead of kernel
// boundaries or grid-wide syncs: lanes are independent until the batch end,
// so no lane ever waits for another and no story is held in lockstep with the
// longest one.  The replay lane alone may instead run over the whole GPU
// (leo_wavefront_grid_kernel, grid barriers) when its steps are heavy.
// Per-lane counters live in global memory (L2).
//
// Reference counterparts (crates/leo-core/src/runtime.rs = CPU,
// crates/leo-core/src/cuda_kernels.cu = the reference's GPU wavefront
// leo_shared_wavefront_persistent_grouped, :5805-6113, which uses 17
// grid.sync() per byte across all lanes):
//   deliver    start_tick touches, deliver_due_events, inject_symbol
//              (runtime.rs:537-639; cuda_kernels.cu:1705-1807) and, on one
//              warp, context resolve (runtime.rs:641-708, model.rs:173-221)
//   settle     decay-on-touch, ordered branch accumulation, integration
//              (runtime.rs:576-603, 710-717, 940-962)
//   blocks     block-local top-k with the exact (k+1)-th cutoff
//              (runtime.rs:964-997)
//   assemble   active list, global cap, population inhibition
//              (runtime.rs:998-1082; cuda_kernels.cu:2285-2586)
//   surrogate  selection surrogates and destination Jacobians
//              (runtime.rs:775-803)
//   eligible   eligibility traces over the exact worklist, ballot compaction
//              (runtime.rs:805-918; cuda_kernels.cu:2651-2846)
//   emit       post-activation dynamics and emission (runtime.rs:920-938,
//              1084-1106) beside the forward pass on the cluster's first CTA:
//              logits, context latent, softmax, loss, output bias and context
//              learning (runtime.rs:1108-1197, 1199-1384)
//   learn      learning signals, output rows, threshold homeostasis
//              (runtime.rs:1216-1303, 1567-1593)
//   plasticity recurrent / input weight updates (runtime.rs:1451-1523)
//   inhibit    inhibitory homeostasis (runtime.rs:1525-1565) + step epilogue
// Frozen steps (replay prefixes) run deliver, settle, blocks, assemble and
// emit only: nothing else can change state on a frozen step; a frozen step
// without a target shares its emit phase with the next step's deliver.  The
// blocks phase writes each block's winners into the first CTA's shared memory
// through the cluster's distributed shared memory, where assemble reads them.
//
// Exactness: every floating-point sum that the CPU forms sequentially is
// formed sequentially here in the same order (branch inputs in event order,
// logits over the active list, softmax over the 257 outputs, learning
// signals over the 257 outputs), no multiply-add is fused (-fmad=false), and
// exp/ln reproduce the platform libm (leo_math.cuh plus exception tables).
#include <cooperative_groups.h>
#include <cub/block/block_radix_sort.cuh>
#include <stdint.h>

#include "leo_device.cuh"
#include "leo_kernels.h"
#include "leo_math.cuh"

namespace cg = cooperative_groups;




// Most event keys one target's segment holds, all sorted in shared memory by
// one CTA (128 KB; the host rejects larger segment capacities).
constexpr uint32_t kHubSortShared = 32768;
// Largest event count a warp sorts in its slice of shared memory (16 warps x 2048 x 4 B = 128 KB).
constexpr uint32_t kHubWarpEvents = 2048;

namespace {

constexpr uint32_t kFrozen = 0;
constexpr uint32_t kThreads = LEO_WAVEFRONT_THREADS;
constexpr uint32_t kWarps = kThreads / 32;

__device__ __forceinline__ float clampf(float v, float lo, float hi) {
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}
// Rust f32::max / f32::min (a NaN operand yields the other operand).
__device__ __forceinline__ float rmax(float a, float b) {
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a > b ? a : (b > a ? b : a);
}
__device__ __forceinline__ float rmin(float a, float b) {
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a < b ? a : (b < a ? b : a);
}
// Rust's f32 Sum folds from -0.0.
__device__ __forceinline__ float sum3(float a, float b, float c) {
    float s = -0.0f;
    s = s + a;
    s = s + b;
    s = s + c;
    return s;
}

// Open-addressing lookup of the libm exception tables (built by the host from
// libm_tables.inc): empty slots hold key 0xffffffff, which no domain input has.
__device__ __forceinline__ bool exception_lookup(const uint2* table, uint32_t mask, uint32_t key, uint32_t* out) {
    uint32_t h = (key * 0x9E3779B1u) & mask;
    for (uint32_t probe = 0; probe <= mask; ++probe) {
        uint2 e = table[h];
        if (e.x == key) {
            *out = e.y;
            return true;
        }
        if (e.x == 0xffffffffu) return false;
        h = (h + 1u) & mask;
    }
    return false;
}
__device__ __forceinline__ float leo_expf(const KernelConsts& kc, float x) {
    if (x < -150.0f) return 0.0f;
    uint32_t out;
    if (exception_lookup(kc.exp_table, kc.exp_mask, __float_as_uint(x), &out)) return __uint_as_float(out);
    return __double2float_rn(leo_math::exp_double((double)x));
}
__device__ __forceinline__ float leo_logf(const KernelConsts& kc, float x) {
    uint32_t out;
    if (exception_lookup(kc.log_table, kc.log_mask, __float_as_uint(x), &out)) return __uint_as_float(out);
    return __double2float_rn(leo_math::log_double_of_float(x));
}

// Packed selection key: activation bits (positive floats order like their
// bits) above the complement of the rotated tie key (runtime.rs:99-101); a
// larger key is a better candidate.
// neuron, rotation < n < 2^24, so one conditional subtraction is the modulus.
__device__ __forceinline__ unsigned long long selection_key(float act, uint32_t neuron, uint32_t rotation,
                                                            uint32_t n) {
    uint32_t rotated = neuron + n - rotation;
    if (rotated >= n) rotated -= n;
    return ((unsigned long long)__float_as_uint(act) << 32) | (unsigned long long)(0xffffffffu - rotated);
}
__device__ __forceinline__ float key_value(unsigned long long key) { return __uint_as_float((uint32_t)(key >> 32)); }
__device__ __forceinline__ uint32_t key_neuron(unsigned long long key, uint32_t rotation, uint32_t n) {
    uint32_t neuron = 0xffffffffu - (uint32_t)(key & 0xffffffffu) + rotation;
    if (neuron >= n) neuron -= n;
    return neuron;
}

__device__ __forceinline__ Trace load_trace(const Trace* p) {
    const float4* q = reinterpret_cast<const float4*>(p);
    float4 a = q[0], b = q[1];
    Trace t;
    t.branch_sens = a.x;
    t.membrane_sens = a.y;
    t.fatigue_sens = a.z;
    t.adaptation_sens[0] = a.w;
    t.adaptation_sens[1] = b.x;
    t.adaptation_sens[2] = b.y;
    t.eligibility = b.z;
    t.tick_mark = __float_as_uint(b.w);
    return t;
}
__device__ __forceinline__ void store_trace(Trace* p, const Trace& t) {
    float4* q = reinterpret_cast<float4*>(p);
    q[0] = make_float4(t.branch_sens, t.membrane_sens, t.fatigue_sens, t.adaptation_sens[0]);
    q[1] = make_float4(t.adaptation_sens[1], t.adaptation_sens[2], t.eligibility, __uint_as_float(t.tick_mark));
}

// runtime.rs:737-773 advance_{recurrent,input}_trace
__device__ __forceinline__ void advance_trace(const LeoConfig& c, Trace& t, uint32_t now) {
    uint32_t last = t.tick_mark >> 1;
    if (now <= last) return;
    uint32_t e = now - last;
    t.branch_sens = t.branch_sens * leo_math::decay_for_elapsed(c.branch_decay, e);
    t.membrane_sens = t.membrane_sens * leo_math::decay_for_elapsed(c.membrane_decay, e);
    t.fatigue_sens = t.fatigue_sens * leo_math::decay_for_elapsed(c.fatigue_decay, e);
    t.adaptation_sens[0] = t.adaptation_sens[0] * leo_math::decay_for_elapsed(c.adaptation_fast_decay, e);
    t.adaptation_sens[1] = t.adaptation_sens[1] * leo_math::decay_for_elapsed(c.adaptation_medium_decay, e);
    t.adaptation_sens[2] = t.adaptation_sens[2] * leo_math::decay_for_elapsed(c.adaptation_slow_decay, e);
    t.tick_mark = (now << 1) | (t.tick_mark & 1u);
}

// Byte marks set with a 32-bit atomicOr on the containing word; the thread
// that flips the byte from 0 appends the index.
__device__ __forceinline__ void mark_and_append(uint8_t* marks, uint32_t* list, uint32_t* count, uint32_t index) {
    if (marks[index] != 0) return;
    unsigned int* word = reinterpret_cast<unsigned int*>(reinterpret_cast<uintptr_t>(marks + index) & ~(uintptr_t)3);
    unsigned int shift = (unsigned int)((reinterpret_cast<uintptr_t>(marks + index) & 3u) * 8u);
    unsigned int bit = 1u << shift;
    unsigned int old = atomicOr(word, bit);
    if ((old & bit) == 0u) list[atomicAdd(count, 1u)] = index;
}

// Appends `item` to a list whose length lives at *count, one atomic per group
// of converged threads (the list order is free: every consumer treats these
// lists as sets).
__device__ __forceinline__ void append_coalesced(uint32_t* list, uint32_t* count, uint32_t item) {
    cg::coalesced_group g = cg::coalesced_threads();
    uint32_t base = 0;
    if (g.thread_rank() == 0) base = atomicAdd(count, g.size());
    base = g.shfl(base, 0);
    list[base + g.thread_rank()] = item;
}


// Neurons a CTA touches in one deliver phase, gathered in shared memory and
// appended to the lane's touched list with one reservation per CTA (one
// atomic per neuron on the lane's single counter serialises at that address).
constexpr uint32_t kTouchBuffer = 2048;
struct TouchBuffer {
    uint32_t count;
    uint32_t base;
    uint32_t items[kTouchBuffer];
};

__device__ __forceinline__ void touch_buffered(const LaneState& ln, uint32_t n, uint32_t epoch, TouchBuffer& tb) {
    if (*(volatile uint32_t*)&ln.touch_epoch[n] == epoch) return;
    if (atomicExch(&ln.touch_epoch[n], epoch) == epoch) return;

    const uint32_t pos = atomicAdd(&tb.count, 1u);
    if (pos < kTouchBuffer)
        tb.items[pos] = n;
    else
        append_coalesced(ln.touched, &ln.sc->touched_count, n);
}

// Appends the CTA's buffered touches to the lane's touched list; every thread
// of the CTA calls it at the end of its deliver phase.
__device__ __forceinline__ void flush_touches(const LaneState& ln, TouchBuffer& tb) {
    __syncthreads();
    const uint32_t count = tb.count < kTouchBuffer ? tb.count : kTouchBuffer;
    if (threadIdx.x == 0 && count) tb.base = atomicAdd(&ln.sc->touched_count, count);
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < count; i += kThreads) ln.touched[tb.base + i] = tb.items[i];
}

// An event: its value is stored by event order, and its key (branch << 30 |
// event order) appended to the target's segment, one atomic per group of
// converged threads with the same target; settle restores the order by
// sorting the keys.  Every event group also touches its target.  A segment holds every event the target can receive in one step
// (the bound is computed from the topology); an overrun is reported.
constexpr uint32_t kEventOrderMask = 0x3fffffffu;
// Due slots a deliver thread loads together (see phase_deliver).
constexpr uint32_t kDeliverBatch = 4;
__device__ __forceinline__ void push_event(const LaneState& ln, const KernelConsts& kc, uint32_t n, uint32_t key,
                                           float value, uint32_t epoch, TouchBuffer& tb) {
    const uint2 seg = kc.topo.seg[n];
    cg::coalesced_group g = cg::coalesced_threads();
    cg::coalesced_group peers = cg::labeled_partition(g, n);
    uint32_t base = 0;
    if (peers.thread_rank() == 0) {
        base = atomicAdd(&ln.seg_count[n], peers.size());
        // One touch per group, issued while the count is in flight (its plain
        // read skips the atomic for a target touched before).
        touch_buffered(ln, n, epoch, tb);
    }
    base = peers.shfl(base, 0);
    const uint32_t pos = base + peers.thread_rank();
    ln.ev_val[key & kEventOrderMask] = value;
    if (pos < (seg.y & LEO_SEG_CAPACITY))
        ln.seg_events[seg.x + pos] = key;
    else
        atomicOr(&ln.sc->error_flag, LEO_ERR_CAPACITY);
}

__device__ __forceinline__ void add_destination(const LaneState& ln, uint32_t n, uint32_t epoch) {
    if (atomicExch(&ln.dst_epoch[n], epoch) != epoch) append_coalesced(ln.dst_list, &ln.sc->dst_count, n);
}

// ---------------------------------------------------------------------------
// Context resolve on one warp (runtime.rs:641-699, model.rs:173-221): lane
// `order - 1` hashes its order and issues all its probe loads at once; the
// slot choice per order is independent (orders own disjoint partitions); lane
// 0 then forms the confidence scales in order.
__device__ void context_resolve_warp(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t symbol,
                                     bool frozen, bool forward) {
    LaneScalars* sc = ln.sc;
    const LeoConfig& c = kc.cfg;
    const uint32_t lane = threadIdx.x & 31u, K = kc.topo.k;
    uint32_t len = sc->ctx_history_len;
    // history push (runtime.rs:642-646)
    uint32_t hist[LEO_MAX_CONTEXT_ORDER];
    for (uint32_t i = 0; i < len; ++i) hist[i] = sc->ctx_history[i];
    if (len == K) {
        for (uint32_t i = 0; i + 1 < K; ++i) hist[i] = hist[i + 1];
        len = K - 1;
    }
    hist[len++] = symbol;
    bool enabled = frozen;
    if (!frozen) {
        enabled = true;
        if (kc.dropout_rate > 0.0f) {  // runtime.rs:103-116 context_survives_dropout
            unsigned long long tick = sc->base_tick + s;
            unsigned long long v = kc.seed ^ (tick * 0x9e3779b97f4a7c15ull) ^
                                   ((unsigned long long)symbol * 0xbf58476d1ce4e5b9ull);
            v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
            v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
            v ^= v >> 31;
            enabled = (float)(uint32_t)(v >> 40) / (float)(1u << 24) >= kc.dropout_rate;
        }
    }
    // A frozen step without a target runs no forward pass and no learning, the
    // only readers of the resolved slots, and resolving never allocates when
    // frozen: only the history push matters for it.
    if (!forward) enabled = false;
    bool allocate = !frozen && enabled;
    uint32_t available = len < K ? len : K;
    int32_t slot = -1;
    uint32_t probes = 0;
    float scale = 0.0f;
    uint32_t order = lane + 1;
    if (enabled && order <= available) {
        unsigned long long h = 0xcbf29ce484222325ull ^ (unsigned long long)order;
        for (uint32_t i = len - order; i < len; ++i) {
            uint32_t sym = hist[i];
            for (int byte = 0; byte < 4; ++byte) {
                h ^= (unsigned long long)((sym >> (8 * byte)) & 0xffu);
                h *= 0x100000001b3ull;
            }
        }
        unsigned long long key = h > 1ull ? h : 1ull;
        uint32_t spo = kc.topo.spo, limit = c.context_probe_limit, D = kc.topo.d;
        uint32_t base = (order - 1) * spo, start = (uint32_t)(key % (unsigned long long)spo);
        constexpr uint32_t kBatch = 8;
        int32_t empty = -1;
        uint32_t weakest = base + start, weakest_obs = 0xffffffffu;
        for (uint32_t off0 = 0; off0 < limit && slot < 0; off0 += kBatch) {
            unsigned long long keys[kBatch];
            uint32_t obs[kBatch];
            uint32_t n = limit - off0 < kBatch ? limit - off0 : kBatch;
#pragma unroll
            for (uint32_t j = 0; j < kBatch; ++j) {
                if (j < n) {
                    uint32_t sl = base + (start + off0 + j) % spo;
                    keys[j] = ln.p.ctx_keys[sl];
                    obs[j] = ln.p.ctx_obs[sl];
                }
            }
            for (uint32_t j = 0; j < n; ++j) {
                uint32_t sl = base + (start + off0 + j) % spo;
                ++probes;
                if (keys[j] == key) {
                    slot = (int32_t)sl;
                    break;
                }
                if (keys[j] == 0ull && empty < 0) empty = (int32_t)sl;
                if (obs[j] < weakest_obs) {
                    weakest_obs = obs[j];
                    weakest = sl;
                }
            }
        }
        if (slot < 0 && allocate) {
            uint32_t sl = empty >= 0 ? (uint32_t)empty : weakest;
            if (ln.p.ctx_keys[sl] != key) {
                ln.p.ctx_keys[sl] = key;
                ln.p.ctx_obs[sl] = 0;
                for (uint32_t k = 0; k < D; ++k) ln.p.ctx_emb[(size_t)sl * D + k] = 0.0f;
            }
            slot = (int32_t)sl;
        }
        if (slot >= 0) {
            float o = (float)ln.p.ctx_obs[slot];
            float confidence = o / (o + (float)c.context_confidence_observations);
            scale = confidence * (float)order;
        }
    }
    __syncwarp();
    if (lane == 0) {
        for (uint32_t i = 0; i < len; ++i) sc->ctx_history[i] = hist[i];
        sc->ctx_history_len = len;
        sc->ctx_applied = enabled ? 1u : 0u;
    }
    uint32_t total_probes = probes;
    for (int o = 16; o > 0; o >>= 1) total_probes += __shfl_xor_sync(0xffffffffu, total_probes, o);
    // scale_sum in order (runtime.rs:661-677): lane 0 walks the orders.
    uint32_t count = 0;
    float scale_sum = 0.0f;
    uint32_t slots[LEO_MAX_CONTEXT_ORDER];
    float scales[LEO_MAX_CONTEXT_ORDER];
    for (uint32_t i = 0; i < K; ++i) {
        int32_t si = __shfl_sync(0xffffffffu, slot, (int)i);
        float sci = __shfl_sync(0xffffffffu, scale, (int)i);
        if (si >= 0) {
            slots[count] = (uint32_t)si;
            scales[count] = sci;
            ++count;
            scale_sum = scale_sum + sci;
        }
    }
    if (lane == 0) {
        if (scale_sum > 0.0f)
            for (uint32_t i = 0; i < count; ++i) scales[i] = scales[i] / scale_sum;
        for (uint32_t i = 0; i < count; ++i) {
            sc->ctx_slots[i] = slots[i];
            sc->ctx_scales[i] = scales[i];
        }
        sc->ctx_count = count;
        sc->ctx_probes = total_probes;
    }
}

// ---------------------------------------------------------------------------
// deliver (runtime.rs:537-639).  Event order within a lane is the CPU's:
// previous actives, then due events from emission ticks s-8, s-4, s-2, s-1
// (rank, then slot), then the symbol's input slots; the event index q (the
// position among all scanned slots, then the input slots) encodes it.  The
// scanned slots are spread over all threads; the slots whose delay matches
// deliver.
//
// `fresh_d1`: the previous step was frozen and its emit phase runs beside this
// deliver, so its ring values are not written yet; a delay-1 event's value is
// formed here from the same operands (activation x weight; no learning step
// separates emission and delivery, so the weight is the one emit reads).

__device__ __forceinline__ void deliver_trace(const LaneState& ln, const KernelConsts& kc, Trace* traces, uint2* const* lists,
                                              uint32_t* counts, uint32_t cur, uint32_t slot, uint32_t s, float a) {
    // activate_{recurrent,input}_trace (runtime.rs:719-735); one event per slot per tick
    Trace t = load_trace(&traces[slot]);
    advance_trace(kc.cfg, t, s);
    t.branch_sens = t.branch_sens + a;
    if ((t.tick_mark & 1u) == 0u) {
        t.tick_mark |= 1u;
        cg::coalesced_group g = cg::coalesced_threads();
        uint32_t base = 0;
        if (g.thread_rank() == 0) base = atomicAdd(&counts[cur], g.size());
        base = g.shfl(base, 0);
        lists[cur][base + g.thread_rank()] = make_uint2(slot, 0u);
    }
    store_trace(&traces[slot], t);
}

__device__ uint32_t phase_deliver(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t worker,
                                  uint32_t workers, bool learn, uint32_t symbol, bool fresh_d1) {
    const uint32_t S = kc.topo.s, F = kc.topo.f, maxa = kc.topo.max_active;
    LaneScalars* sc = ln.sc;
    const uint32_t prev = s >= 1 ? sc->ring_count[(s - 1) % LEO_RING] : 0u;
    const uint32_t a8 = s >= 8 ? sc->ring_count[(s - 8) % LEO_RING] : 0u;
    const uint32_t a4 = s >= 4 ? sc->ring_count[(s - 4) % LEO_RING] : 0u;
    const uint32_t a2 = s >= 2 ? sc->ring_count[(s - 2) % LEO_RING] : 0u;
    const uint32_t e8 = a8 * S, e4 = a4 * S, e2 = a2 * S, e1 = prev * S;
    const uint32_t events = e8 + e4 + e2 + e1;
    const uint32_t cur = sc->elig_cur;
    if (worker == 0) {
        sc->elig_count[cur ^ 1u] = 0;
        sc->in_elig_count[cur ^ 1u] = 0;
    }
    const uint32_t epoch = s + 1;
    const uint32_t lane = threadIdx.x & 31u, gwarp = worker >> 5, gwarps = workers >> 5;
    __shared__ TouchBuffer tb;
    if (threadIdx.x == 0) tb.count = 0u;
    __syncthreads();
    // previous actives are touched (start_tick, runtime.rs:537-561)
    for (uint32_t i = worker; i < prev; i += workers)
        touch_buffered(ln, ln.ring_src[((s - 1) % LEO_RING) * maxa + i], epoch, tb);
    // due recurrent events (ring entry of their delay class, rank, slot), kDeliverBatch
    // slots per thread at a time: each stage's loads for all of them are in
    // flight together (source, topology word, then the due ones' values), so a
    // thread pays the dependent round trips once per batch, not once per slot.
    for (uint32_t q0 = worker; q0 < events; q0 += workers * kDeliverBatch) {
        uint32_t dl[kDeliverBatch], ent[kDeliverBatch], rr[kDeliverBatch], jj[kDeliverBatch], src[kDeliverBatch];
#pragma unroll
        for (uint32_t k = 0; k < kDeliverBatch; ++k) {
            const uint32_t q = q0 + k * workers;
            uint32_t d = 1, off = 0;
            if (q < e8) {
                d = 8; off = q;
            } else if (q < e8 + e4) {
                d = 4; off = q - e8;
            } else if (q < e8 + e4 + e2) {
                d = 2; off = q - e8 - e4;
            } else if (q < events) {
                d = 1; off = q - e8 - e4 - e2;
            }
            dl[k] = q < events ? d : 0u;  // 0: no slot (no word has delay 0)
            ent[k] = (s - d) % LEO_RING;
            rr[k] = off / S;
            jj[k] = off - rr[k] * S;
            src[k] = q < events ? ln.ring_src[ent[k] * maxa + rr[k]] : 0u;
        }
        uint32_t word[kDeliverBatch];
#pragma unroll
        for (uint32_t k = 0; k < kDeliverBatch; ++k) word[k] = dl[k] ? kc.topo.rec_word[src[k] * S + jj[k]] : 0u;
        float act[kDeliverBatch], val[kDeliverBatch];
#pragma unroll
        for (uint32_t k = 0; k < kDeliverBatch; ++k) {
            act[k] = 0.0f;
            val[k] = 0.0f;
            if (dl[k] && LEO_WORD_DELAY(word[k]) == dl[k]) {
                act[k] = ln.ring_act[ent[k] * maxa + rr[k]];
                val[k] = (fresh_d1 && dl[k] == 1u) ? ln.p.rec_weight[src[k] * S + jj[k]]
                                                  : ln.ring_val[((size_t)ent[k] * maxa + rr[k]) * S + jj[k]];
            }
        }
#pragma unroll
        for (uint32_t k = 0; k < kDeliverBatch; ++k) {
            if (!dl[k] || LEO_WORD_DELAY(word[k]) != dl[k]) continue;
            const uint32_t q = q0 + k * workers;
            const uint32_t n = word[k] & LEO_TARGET_MASK, b = LEO_WORD_BRANCH(word[k]);
            // a delay-1 event of a step whose emit is still open: activation x weight, as emit forms it
            const float value = (fresh_d1 && dl[k] == 1u) ? act[k] * val[k] : val[k];
            push_event(ln, kc, n, (b << 30) | q, value, epoch, tb);
            if (learn) deliver_trace(ln, kc, ln.traces, ln.elig, sc->elig_count, cur, src[k] * S + jj[k], s, act[k]);
        }
    }
    // the symbol's input slots (inject_symbol, runtime.rs:627-639)
    for (uint32_t f = worker; f < F; f += workers) {
        const uint32_t slot = symbol * F + f;
        const uint32_t word = kc.topo.in_word[slot];
        const uint32_t n = word & LEO_TARGET_MASK, b = LEO_WORD_BRANCH(word);
        push_event(ln, kc, n, (b << 30) | (events + f), ln.p.in_weight[slot], epoch, tb);
        if (learn) deliver_trace(ln, kc, ln.in_traces, ln.in_elig, sc->in_elig_count, cur, slot, s, 1.0f);
    }
    flush_touches(ln, tb);
    return events + F;
}

// ---------------------------------------------------------------------------
// settle (runtime.rs:576-603, 710-717, 541-548, 947-962).

// Decay-on-touch of one neuron's branches and state.
__device__ __forceinline__ void settle_decay(const LeoConfig& c, uint32_t s, NeuronCold& cold, float4& br) {
    if (s > cold.branch_tick) {
        float dec = leo_math::decay_for_elapsed(c.branch_decay, s - cold.branch_tick);
        br.x = br.x * dec;
        br.y = br.y * dec;
        br.z = br.z * dec;
        br.w = br.w * dec;
        cold.branch_tick = s;
    }
    if (s > cold.neuron_tick) {
        uint32_t e = s - cold.neuron_tick;
        cold.membrane = cold.membrane * leo_math::decay_for_elapsed(c.membrane_decay, e);
        cold.fatigue = cold.fatigue * leo_math::decay_for_elapsed(c.fatigue_decay, e);
        cold.adaptation[0] = cold.adaptation[0] * leo_math::decay_for_elapsed(c.adaptation_fast_decay, e);
        cold.adaptation[1] = cold.adaptation[1] * leo_math::decay_for_elapsed(c.adaptation_medium_decay, e);
        cold.adaptation[2] = cold.adaptation[2] * leo_math::decay_for_elapsed(c.adaptation_slow_decay, e);
        cold.neuron_tick = s;
    }
}

// Per-neuron values settle needs after the branch sums, loaded up front so
// their latency overlaps the event-list walk.
struct SettlePre {
    float threshold, excitability;
    uint32_t refractory_until;
};

__device__ __forceinline__ SettlePre settle_preload(const LaneState& ln, const KernelConsts& kc, uint32_t n) {
    return SettlePre{ln.p.threshold[n], kc.topo.excitability[n], ln.hot[n].refractory_until};
}

// Integration after the branch sums; stores the neuron and returns its block
// candidate key (0: not a candidate).
__device__ __forceinline__ unsigned long long settle_integrate_key(const LaneState& ln, const KernelConsts& kc,
                                                                   uint32_t n, uint32_t s, NeuronCold cold, float4 br,
                                                                   float pop_inh, uint32_t rotation, SettlePre pre) {
    unsigned long long key = 0ull;
    ln.hot[n].activation = 0.0f;
    bool refractory = pre.refractory_until > s;
    if (!refractory) {
        float gate = clampf(br.w, 0.0f, 1.0f);
        float inhibitory = br.y;
        float net = br.x + br.z * gate + inhibitory;
        float adaptation = sum3(cold.adaptation[0], cold.adaptation[1], cold.adaptation[2]);
        float drive = pre.excitability * net - cold.fatigue - adaptation - pop_inh;
        cold.membrane = cold.membrane + drive;
        float act = clampf(cold.membrane - pre.threshold, 0.0f, 1.0f);
        if (act > 0.0f) key = selection_key(act, n, rotation, kc.topo.n);
    }
    ln.cold[n] = cold;
    ln.branches[n] = br;
    return key;
}

// Integration and block candidate after the branch sums; stores the neuron.
__device__ __forceinline__ void settle_integrate(const LaneState& ln, const KernelConsts& kc, uint32_t n, uint32_t s,
                                                 NeuronCold cold, float4 br, float pop_inh, uint32_t rotation,
                                                 SettlePre pre) {
    const unsigned long long key = settle_integrate_key(ln, kc, n, s, cold, br, pop_inh, rotation, pre);
    if (key) {
        const uint32_t npb = kc.topo.npb, blk = n / npb;
        const uint32_t pos = atomicAdd(&ln.block_cand_count[blk], 1u);
        ln.block_cand[(size_t)blk * npb + pos] = key;
    }
}

// Bounds of one branch in a hub's sorted keys (branch in the top two bits).
__device__ __forceinline__ uint32_t hub_branch_begin(const uint32_t* keys, uint32_t k, uint32_t branch) {
    uint32_t lo = 0, hi = k;
    while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if ((keys[mid] >> 30) < branch)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

// Strictly sequential sum of vals[lo, hi) onto `a`, loads issued eight at a time.
__device__ __forceinline__ float ordered_sum(const float* vals, uint32_t lo, uint32_t hi, float a) {
    uint32_t i = lo;
    for (; i + 8 <= hi; i += 8) {
        float v[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) v[x] = vals[i + x];
#pragma unroll
        for (int x = 0; x < 8; ++x) a = a + v[x];
    }
    for (; i < hi; ++i) a = a + vals[i];
    return a;
}

// keys[i] = src[i] for i < k and the sort padding for k <= i < P, for the
// group's threads (tid, stride `lanes`), eight loads in flight per thread.
__device__ __forceinline__ void load_keys(uint32_t* keys, const uint32_t* __restrict__ src, uint32_t k, uint32_t P,
                                          uint32_t tid, uint32_t lanes) {
    for (uint32_t base = tid; base < P; base += lanes * 8) {
        uint32_t v[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) {
            const uint32_t i = base + x * lanes;
            v[x] = i < k ? src[i] : 0xffffffffu;
        }
#pragma unroll
        for (int x = 0; x < 8; ++x) {
            const uint32_t i = base + x * lanes;
            if (i < P) keys[i] = v[x];
        }
    }
}

// Replaces sorted keys[0, k) by their events' values (by event order).
__device__ __forceinline__ void gather_values(uint32_t* keys, const float* __restrict__ ev_val, uint32_t k, uint32_t tid,
                                              uint32_t lanes) {
    float* vals = reinterpret_cast<float*>(keys);
    for (uint32_t base = tid; base < k; base += lanes * 8) {
        float v[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) {
            const uint32_t i = base + x * lanes;
            v[x] = i < k ? ev_val[keys[i] & kEventOrderMask] : 0.0f;
        }
#pragma unroll
        for (int x = 0; x < 8; ++x) {
            const uint32_t i = base + x * lanes;
            if (i < k) vals[i] = v[x];
        }
    }
}

struct BlockSync {
    __device__ void operator()() const { __syncthreads(); }
};
struct WarpSync {
    __device__ void operator()() const { __syncwarp(); }
};

// Bitonic sort (ascending) of P 4-byte keys by the `lanes` threads of `tid`'s
// group; `sync` orders the group between stages.
template <typename Sync>
__device__ __forceinline__ void bitonic_sort_keys(uint32_t* keys, uint32_t P, uint32_t tid, uint32_t lanes, Sync sync) {
    for (uint32_t width = 2; width <= P; width <<= 1) {
        for (uint32_t stride = width >> 1; stride > 0; stride >>= 1) {
            for (uint32_t i = tid; i < P; i += lanes) {
                const uint32_t other = i ^ stride;
                if (other > i) {
                    const bool up = (i & width) == 0;
                    const uint32_t x = keys[i], y = keys[other];
                    if (up ? (x > y) : (x < y)) {
                        keys[i] = y;
                        keys[other] = x;
                    }
                }
            }
            sync();
        }
    }
}

// ---------------------------------------------------------------------------
// Register-resident bitonic sort of a warp's 256 keys, 8 per lane in blocked
// layout (lane t holds elements 8t .. 8t+7): strides below 8 exchange
// registers, strides 8..128 exchange with the partner lane by shuffle.
constexpr uint32_t kSortPer = 8;
constexpr uint32_t kWarpSortKeys = 32 * kSortPer;
constexpr uint32_t kCtaSortKeys = kThreads * kSortPer;  // the CTA's radix sort: up to 8 keys per thread

template <int S>
__device__ __forceinline__ void sort_regs(uint32_t (&v)[kSortPer], uint32_t e0, uint32_t w) {
#pragma unroll
    for (int r = 0; r < (int)kSortPer; ++r) {
        if ((r & S) == 0) {
            const bool asc = ((e0 + (uint32_t)r) & w) == 0u;
            const uint32_t a = v[r], b = v[r | S];
            const uint32_t lo = a < b ? a : b, hi = a < b ? b : a;
            v[r] = asc ? lo : hi;
            v[r | S] = asc ? hi : lo;
        }
    }
}

__device__ __forceinline__ void sort_shfl(uint32_t (&v)[kSortPer], uint32_t e0, uint32_t w, uint32_t stride) {
    const bool keep_min = ((e0 & stride) == 0u) == ((e0 & w) == 0u);
    const int lane_mask = (int)(stride / kSortPer);
#pragma unroll
    for (int r = 0; r < (int)kSortPer; ++r) {
        const uint32_t o = __shfl_xor_sync(0xffffffffu, v[r], lane_mask);
        v[r] = keep_min ? (v[r] < o ? v[r] : o) : (v[r] < o ? o : v[r]);
    }
}

// Ascending sort of the warp's kWarpSortKeys keys (lane index t).
__device__ __forceinline__ void warp_sort_regs(uint32_t (&v)[kSortPer], uint32_t t) {
    const uint32_t e0 = t * kSortPer;
    for (uint32_t w = 2; w <= kWarpSortKeys; w <<= 1) {
        for (uint32_t stride = w >> 1; stride >= kSortPer; stride >>= 1) sort_shfl(v, e0, w, stride);
        if (w >= 8) sort_regs<4>(v, e0, w);
        if (w >= 4) sort_regs<2>(v, e0, w);
        sort_regs<1>(v, e0, w);
    }
}

// Strictly sequential sum of shared vals[lo, hi) onto `a`, the next eight
// loads issued before the current eight adds.
__device__ __forceinline__ float ordered_sum_pipelined(const float* vals, uint32_t lo, uint32_t hi, float a) {
    uint32_t i = lo;
    if (i + 8 <= hi) {
        float nxt[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) nxt[x] = vals[i + x];
        for (;;) {
            float cur[8];
#pragma unroll
            for (int x = 0; x < 8; ++x) cur[x] = nxt[x];
            i += 8;
            const bool more = i + 8 <= hi;
            if (more) {
#pragma unroll
                for (int x = 0; x < 8; ++x) nxt[x] = vals[i + x];
            }
#pragma unroll
            for (int x = 0; x < 8; ++x) a = a + cur[x];
            if (!more) break;
        }
    }
    for (; i < hi; ++i) a = a + vals[i];
    return a;
}

// Per-branch counts of the sorted keys e < k held in v (blocked layout).
__device__ __forceinline__ void branch_counts(const uint32_t (&v)[kSortPer], uint32_t e0, uint32_t k, uint32_t (&cnt)[4]) {
#pragma unroll
    for (int b = 0; b < 4; ++b) cnt[b] = 0u;
#pragma unroll
    for (int r = 0; r < (int)kSortPer; ++r) {
        const uint32_t b = e0 + (uint32_t)r < k ? v[r] >> 30 : 4u;
#pragma unroll
        for (int x = 0; x < 4; ++x) cnt[x] += b == (uint32_t)x ? 1u : 0u;
    }
}

// Bitonic sorting network over the first N of 16 keys in registers (N a
// power of two; entries past the target's count hold the 0xffffffff padding).
template <int N>
__device__ __forceinline__ void sort_network(uint32_t (&e)[16]) {
#pragma unroll
    for (int w = 2; w <= N; w <<= 1) {
#pragma unroll
        for (int st = w >> 1; st > 0; st >>= 1) {
#pragma unroll
            for (int i = 0; i < N; ++i) {
                const int j = i ^ st;
                if (j > i) {
                    const bool asc = (i & w) == 0;
                    const uint32_t a = e[i], b = e[j];
                    const uint32_t lo = a < b ? a : b, hi = a < b ? b : a;
                    e[i] = asc ? lo : hi;
                    e[j] = asc ? hi : lo;
                }
            }
        }
    }
}

// Adds `v` to the accumulator of `branch` (registers, no indexed array).
__device__ __forceinline__ void add_branch(float4& acc, uint32_t branch, float v) {
    if (branch == 0u)
        acc.x = acc.x + v;
    else if (branch == 1u)
        acc.y = acc.y + v;
    else if (branch == 2u)
        acc.z = acc.z + v;
    else
        acc.w = acc.w + v;
}

// The CTA's radix sort of one target's k keys (k <= ITEMS x kThreads) by
// (branch, event order) -- the key compacted to qbits + 2 bits, the branch
// above the event order -- loaded striped (coalesced; the sort takes any
// arrangement) and left blocked; each sorted key's event value is gathered
// and written to smem[0, k) in order, and the per-branch counts added to s_cnt.
// The sort's temporary storage follows the value area (kCtaSortKeys words).
template <int ITEMS>
__device__ __forceinline__ void cta_radix_values(const LaneState& ln, uint32_t* smem, const uint32_t* ev, uint32_t k,
                                                 uint32_t qbits, uint32_t* s_cnt) {
    using Sort = cub::BlockRadixSort<uint32_t, kThreads, ITEMS>;
    static_assert(sizeof(typename Sort::TempStorage) + kCtaSortKeys * sizeof(uint32_t) <=
                      (size_t)kWarps * kHubWarpEvents * sizeof(uint32_t), "radix sort storage fits the scratch");
    typename Sort::TempStorage& temp = *reinterpret_cast<typename Sort::TempStorage*>(smem + kCtaSortKeys);
    const uint32_t tid = threadIdx.x;
    const uint32_t qmask = (1u << qbits) - 1u, pad = (1u << (qbits + 2u)) - 1u;
    uint32_t key[ITEMS];
#pragma unroll
    for (int r = 0; r < ITEMS; ++r) {
        const uint32_t e = (uint32_t)r * kThreads + tid;
        const uint32_t raw = e < k ? ev[e] : 0u;
        key[r] = e < k ? ((raw >> 30) << qbits) | (raw & qmask) : pad;
    }
    Sort(temp).Sort(key, 0, (int)qbits + 2);
    const uint32_t e0 = tid * ITEMS;
    float val[ITEMS];
    uint32_t cnt[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int r = 0; r < ITEMS; ++r) {
        const bool live = e0 + (uint32_t)r < k;
        val[r] = live ? ln.ev_val[key[r] & qmask] : 0.0f;
        const uint32_t b = live ? key[r] >> qbits : 4u;
#pragma unroll
        for (int x = 0; x < 4; ++x) cnt[x] += b == (uint32_t)x ? 1u : 0u;
    }
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const uint32_t c = __reduce_add_sync(0xffffffffu, cnt[b]);
        if ((tid & 31u) == 0u && c) atomicAdd(&s_cnt[b], c);
    }
#pragma unroll
    for (int r = 0; r < ITEMS; ++r)
        if (e0 + (uint32_t)r < k) reinterpret_cast<float*>(smem)[e0 + r] = val[r];
}

// One target settled by the whole CTA (every thread calls it): its k keys
// sorted (registers up to 4096, shared memory above), each key's event
// value gathered, and each branch summed in ascending event order onto the
// decayed branch value by one thread per branch; then integration.  Resets
// the target's count unless `keep_count` (the blocks phase resets it then).
__device__ void settle_target_cta(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t n, uint32_t k,
                                  uint32_t offset, uint32_t* smem, float pop_inh, uint32_t rotation,
                                  bool keep_count = false) {
    __shared__ float s_acc[4];
    __shared__ uint32_t s_cnt[4];
    __shared__ uint32_t s_bound[5];
    __shared__ NeuronCold s_cold;
    __shared__ SettlePre s_pre;
    const uint32_t tid = threadIdx.x;
    const uint32_t* ev = ln.seg_events + offset;
    if (tid == 0) {
        NeuronCold cold = ln.cold[n];
        float4 br = ln.branches[n];
        s_pre = settle_preload(ln, kc, n);
        settle_decay(kc.cfg, s, cold, br);
        s_cold = cold;
        s_acc[0] = br.x;
        s_acc[1] = br.y;
        s_acc[2] = br.z;
        s_acc[3] = br.w;
    }
    if (tid < 4) s_cnt[tid] = 0u;
    if (k <= kCtaSortKeys) {
        // Radix sort with 1, 2, 4 or 8 keys per thread.
        const uint32_t qbits = kc.event_bits;
        __syncthreads();  // s_cnt cleared
        if (k <= kThreads)
            cta_radix_values<1>(ln, smem, ev, k, qbits, s_cnt);
        else if (k <= 2 * kThreads)
            cta_radix_values<2>(ln, smem, ev, k, qbits, s_cnt);
        else if (k <= 4 * kThreads)
            cta_radix_values<4>(ln, smem, ev, k, qbits, s_cnt);
        else
            cta_radix_values<8>(ln, smem, ev, k, qbits, s_cnt);
        __syncthreads();
        if (tid == 0) {
            s_bound[0] = 0u;
            for (int b = 0; b < 4; ++b) s_bound[b + 1] = s_bound[b] + s_cnt[b];
        }
        __syncthreads();
        const float* vals = reinterpret_cast<const float*>(smem);
        if (tid < 4) s_acc[tid] = ordered_sum_pipelined(vals, s_bound[tid], s_bound[tid + 1], s_acc[tid]);
    } else {
        // More keys than one register sort: bitonic sort in shared memory
        // (segment capacities are at most kHubSortShared keys).
        uint32_t P = 1;
        while (P < k) P <<= 1;
        load_keys(smem, ev, k, P, tid, kThreads);
        __syncthreads();
        bitonic_sort_keys(smem, P, tid, kThreads, BlockSync{});
        if (tid <= 4) s_bound[tid] = tid == 4 ? k : hub_branch_begin(smem, k, tid);
        __syncthreads();
        gather_values(smem, ln.ev_val, k, tid, kThreads);
        __syncthreads();
        const float* vals = reinterpret_cast<const float*>(smem);
        if (tid < 4) s_acc[tid] = ordered_sum(vals, s_bound[tid], s_bound[tid + 1], s_acc[tid]);
    }
    __syncthreads();
    if (tid == 0) {
        settle_integrate(ln, kc, n, s, s_cold, make_float4(s_acc[0], s_acc[1], s_acc[2], s_acc[3]), pop_inh, rotation,
                         s_pre);
        if (!keep_count) ln.seg_count[n] = 0u;
    }
    __syncthreads();
}

// One target settled by one warp (every lane calls it; k <= kHubWarpEvents):
// registers up to 256 keys, the warp's shared-memory slice above.  Resets
// the target's count.
__device__ void settle_target_warp(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t n, uint32_t k,
                                   uint32_t offset, uint32_t* wkeys, float pop_inh, uint32_t rotation) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t* ev = ln.seg_events + offset;
    NeuronCold cold;
    float4 br = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    SettlePre pre{};
    if (lane == 0) {
        cold = ln.cold[n];
        br = ln.branches[n];
        pre = settle_preload(ln, kc, n);
        settle_decay(kc.cfg, s, cold, br);
    }
    uint32_t lo = 0, hi = 0;  // this lane's branch range (lanes 0..3)
    const float* wvals = reinterpret_cast<const float*>(wkeys);
    if (k <= kWarpSortKeys) {
        const uint32_t e0 = lane * kSortPer;
        uint32_t v[kSortPer];
#pragma unroll
        for (int r = 0; r < (int)kSortPer; ++r) v[r] = e0 + (uint32_t)r < k ? ev[e0 + r] : 0xffffffffu;
        warp_sort_regs(v, lane);
        float val[kSortPer];
#pragma unroll
        for (int r = 0; r < (int)kSortPer; ++r) val[r] = e0 + (uint32_t)r < k ? ln.ev_val[v[r] & kEventOrderMask] : 0.0f;
        uint32_t cnt[4];
        branch_counts(v, e0, k, cnt);
        uint32_t acc_c = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const uint32_t c = __reduce_add_sync(0xffffffffu, cnt[b]);
            if ((uint32_t)b == lane) {
                lo = acc_c;
                hi = acc_c + c;
            }
            acc_c += c;
        }
        float4* vb = reinterpret_cast<float4*>(wkeys);
        vb[2 * lane] = make_float4(val[0], val[1], val[2], val[3]);
        vb[2 * lane + 1] = make_float4(val[4], val[5], val[6], val[7]);
        __syncwarp();
    } else {
        uint32_t P = 32;
        while (P < k) P <<= 1;
        load_keys(wkeys, ev, k, P, lane, 32u);
        __syncwarp();
        bitonic_sort_keys(wkeys, P, lane, 32u, WarpSync{});
        const uint32_t bound = lane <= 4 ? (lane == 4 ? k : hub_branch_begin(wkeys, k, lane)) : 0u;
        __syncwarp();
        gather_values(wkeys, ln.ev_val, k, lane, 32u);
        lo = bound;
        hi = __shfl_down_sync(0xffffffffu, bound, 1);
        __syncwarp();
    }
    br.x = __shfl_sync(0xffffffffu, br.x, 0);
    br.y = __shfl_sync(0xffffffffu, br.y, 0);
    br.z = __shfl_sync(0xffffffffu, br.z, 0);
    br.w = __shfl_sync(0xffffffffu, br.w, 0);
    float a = 0.0f;
    if (lane < 4) a = ordered_sum_pipelined(wvals, lo, hi, lane == 0 ? br.x : (lane == 1 ? br.y : (lane == 2 ? br.z : br.w)));
    const float a1 = __shfl_sync(0xffffffffu, a, 1), a2 = __shfl_sync(0xffffffffu, a, 2),
                a3 = __shfl_sync(0xffffffffu, a, 3);
    if (lane == 0) {
        settle_integrate(ln, kc, n, s, cold, make_float4(a, a1, a2, a3), pop_inh, rotation, pre);
        ln.seg_count[n] = 0u;
    }
    __syncwarp();
}

// One target settled by one thread (k <= 16): its keys, state and preloads
// all in flight at once, a sorting network in registers, the values, the
// ordered per-branch sums, integration.  Resets the target's count.
__device__ __forceinline__ void settle_target_thread(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t n,
                                                     uint32_t k, uint32_t offset, float pop_inh, uint32_t rotation) {
    uint32_t e[16];
#pragma unroll
    for (int x = 0; x < 16; ++x) e[x] = (uint32_t)x < k ? ln.seg_events[offset + x] : 0xffffffffu;
    NeuronCold cold = ln.cold[n];
    float4 br = ln.branches[n];
    const SettlePre pre = settle_preload(ln, kc, n);
    if (k > 8u)
        sort_network<16>(e);
    else if (k > 4u)
        sort_network<8>(e);
    else if (k > 1u)
        sort_network<4>(e);
    float v[16];
#pragma unroll
    for (int x = 0; x < 16; ++x) v[x] = (uint32_t)x < k ? ln.ev_val[e[x] & kEventOrderMask] : 0.0f;
    settle_decay(kc.cfg, s, cold, br);
#pragma unroll
    for (int x = 0; x < 16; ++x)
        if ((uint32_t)x < k) add_branch(br, e[x] >> 30, v[x]);
    settle_integrate(ln, kc, n, s, cold, br, pop_inh, rotation, pre);
    if (k) ln.seg_count[n] = 0u;
}

// Shares of the touched list when some CTAs sort busy targets first: every
// CTA computes the same partition from the busy targets' key counts (busy
// target i goes to CTA i mod C).  Modelled cost: one sorted key of a busy
// target costs 1 / kBusyKeyShare of one touched neuron, so CTA r's share is
// max(0, T - keys_r / kBusyKeyShare) with T chosen so the shares cover the list; the
// partition only moves work between CTAs (every entry is settled once).
// Writes [begin, end) of this CTA to range[0..1]; every thread calls it.
// Touched neurons one busy-target key is worth in the share model below
// (measured on config 3: shares from 1/2 to 1/5 of a neuron per key gave the
// same settle time; results never depend on it).
constexpr unsigned long long kBusyKeyShare = 5;
__device__ void touched_shares(const uint32_t* busy_k, uint32_t nbusy, uint32_t count, uint32_t C, uint32_t rank,
                               uint32_t* range) {
    static_assert(kThreads >= 256, "C <= 256 CTAs share one scan");
    __shared__ unsigned long long s_share[256];
    __shared__ unsigned long long s_sum[kWarps];
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    unsigned long long keys = 0;
    for (uint32_t i = tid; i < nbusy; i += C) keys += busy_k[i];  // CTA tid's busy keys (tid < C)
    // T = (count + all keys / 5) / C, so that the unclamped shares sum to count
    unsigned long long all = 0;
    for (uint32_t i = lane; i < nbusy; i += 32u) all += busy_k[i];
    for (int o = 16; o > 0; o >>= 1) all += __shfl_xor_sync(0xffffffffu, all, o);
    const unsigned long long T = ((unsigned long long)count + all / kBusyKeyShare) / C + 1u;
    unsigned long long share = 0;
    if (tid < C) share = T > keys / kBusyKeyShare ? T - keys / kBusyKeyShare : 0u;
    // inclusive scan of the shares over the CTAs
    unsigned long long incl = share;
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= (uint32_t)o) incl += y;
    }
    if (lane == 31) s_sum[warp] = incl;
    __syncthreads();
    unsigned long long before = 0;
    for (uint32_t w = 0; w < warp; ++w) before += s_sum[w];
    if (tid < 256u) s_share[tid] = before + incl;
    __syncthreads();
    if (tid == 0) {
        const unsigned long long total = s_share[C - 1];
        const unsigned long long a = rank == 0 ? 0ull : s_share[rank - 1], b = s_share[rank];
        range[0] = (uint32_t)(total ? (unsigned long long)count * a / total : 0ull);
        range[1] = (uint32_t)(total ? (unsigned long long)count * b / total : (rank + 1 == C ? count : 0ull));
    }
    __syncthreads();
}

// Unlisted targets with more events than a warp sorts: queued per CTA during
// the touched loop and settled by the CTA after it.
constexpr uint32_t kCtaQueue = 32;
// Listed targets classified per chunk of the CTA's share of the list.
constexpr uint32_t kListedChunk = kThreads;
// ---------------------------------------------------------------------------
// settle (runtime.rs:576-603, 710-717, 541-548, 947-962): every touched
// neuron adds its events per branch in ascending event order onto its decayed
// branches, then integrates (membrane, drive, block candidate).  A target's
// events of the step are the keys in its segment (seg_count[n] of them).
//   listed targets (high in-degree, descending capacity): CTA r settles listed
//     targets r, r + C, ...: those with more than cta_events events by the
//     whole CTA, more than thread_events by one of its warps, the rest (when
//     touched this step) by one of its threads;
//   every other touched neuron, in the warp that holds it in the touched list:
//     at most thread_events events by its own thread, at most kHubWarpEvents
//     by the warp, more by the CTA after the loop.
// Whoever settles a target resets its count for the next step's deliver.
__device__ void phase_settle(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t worker,
                             uint32_t workers, uint32_t rank, uint32_t C, uint32_t* smem) {
    __shared__ uint32_t s_list[3][kListedChunk];
    __shared__ uint32_t s_list_k[3][kListedChunk];
    __shared__ uint32_t s_queue[kCtaQueue], s_queue_k[kCtaQueue];
    __shared__ uint32_t s_nlist[3], s_nqueue;
    const uint32_t n_count = kc.topo.n;
    LaneScalars* sc = ln.sc;
    const uint32_t count = sc->touched_count;
    const float pop_inh = sc->population_inhibition;
    const uint32_t rotation = (uint32_t)((sc->base_tick + s) % (unsigned long long)n_count);
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t epoch = s + 1;
    uint32_t* wkeys = smem + (size_t)warp * kHubWarpEvents;
    if (tid == 0) s_nqueue = 0u;
    const unsigned long long t0 = clock64();
    const uint32_t listed = kc.topo.cta_count;
    // The first kThreads listed targets (the largest capacities, where the
    // busy ones are): every CTA reads their counts, numbers the ones with
    // more than cta_events events in list order, and sorts those whose number
    // is its rank modulo C -- one CTA sort per CTA while at most C are busy,
    // whichever targets they are this step.  Their counts stay until the
    // blocks phase, since every CTA classifies them by their counts here.
    const uint32_t top = listed < kThreads ? listed : kThreads;
    // The touched list's range of this CTA: equal shares, or (with busy
    // targets this step) shares shrunk by each CTA's busy-target keys.
    __shared__ uint32_t s_range[2];
    bool weighted = false;
    if (top > 0u) {
        __shared__ uint32_t s_warp_busy[kWarps];
        __shared__ uint32_t s_busy_k[kThreads];
        uint32_t n = 0, k = 0;
        if (tid < top) {
            n = kc.topo.cta_targets[tid];
            k = min(ln.seg_count[n], kc.topo.seg[n].y & LEO_SEG_CAPACITY);
        }
        const bool busy = tid < top && k > kc.topo.cta_events;
        const unsigned int ballot = __ballot_sync(0xffffffffu, busy);
        if (lane == 0) s_warp_busy[warp] = (uint32_t)__popc(ballot);
        if (tid == 0) s_nlist[0] = 0u;
        __syncthreads();
        uint32_t before = (uint32_t)__popc(ballot & ((1u << lane) - 1u));
        for (uint32_t w = 0; w < warp; ++w) before += s_warp_busy[w];
        if (busy && before % C == rank) {
            const uint32_t pos = atomicAdd(&s_nlist[0], 1u);
            s_list[0][pos] = n;
            s_list_k[0][pos] = k;
        }
        if (busy) s_busy_k[before] = k;
        uint32_t nbusy = 0;
        for (uint32_t w = 0; w < kWarps; ++w) nbusy += s_warp_busy[w];
        __syncthreads();
        weighted = nbusy > 0u && count > 0u;
        if (weighted) touched_shares(s_busy_k, nbusy, count, C, rank, s_range);
        const uint32_t nbig = s_nlist[0];
        for (uint32_t j = 0; j < nbig; ++j)
            settle_target_cta(ln, s, kc, s_list[0][j], s_list_k[0][j], kc.topo.seg[s_list[0][j]].x, smem, pop_inh,
                              rotation, true);
    }
    // Every listed target not sorted above, one chunk of this CTA's share at a
    // time: classified by the step's event count into CTA / warp / thread work.
    for (uint32_t round0 = 0; round0 * C < listed; round0 += kListedChunk) {
        if (tid < 3) s_nlist[tid] = 0u;
        __syncthreads();
        // Round r of the list goes to the CTAs in alternating directions, so
        // the CTA with the largest target of one round gets the smallest of
        // the next.
        const uint32_t round = round0 + tid;
        const uint32_t i = round * C + ((round & 1u) ? C - 1u - rank : rank);
        if (i < listed) {
            const uint32_t n = kc.topo.cta_targets[i];
            const uint32_t k = min(ln.seg_count[n], kc.topo.seg[n].y & LEO_SEG_CAPACITY);
            const int tier = k > kc.topo.cta_events ? 0 : (k > kc.topo.thread_events ? 1 : 2);
            if ((tier > 0 || i >= top) && (tier < 2 || k > 0u || ln.touch_epoch[n] == epoch)) {
                const uint32_t pos = atomicAdd(&s_nlist[tier], 1u);
                s_list[tier][pos] = n;
                s_list_k[tier][pos] = k;
            }
        }
        __syncthreads();
        const uint32_t nbig = s_nlist[0], nmid = s_nlist[1], nsmall = s_nlist[2];
        for (uint32_t j = 0; j < nbig; ++j)
            settle_target_cta(ln, s, kc, s_list[0][j], s_list_k[0][j], kc.topo.seg[s_list[0][j]].x, smem, pop_inh,
                              rotation);
        if (tid < nsmall)
            settle_target_thread(ln, s, kc, s_list[2][tid], s_list_k[2][tid], kc.topo.seg[s_list[2][tid]].x, pop_inh,
                                 rotation);
        for (uint32_t j = warp; j < nmid; j += kWarps)
            settle_target_warp(ln, s, kc, s_list[1][j], s_list_k[1][j], kc.topo.seg[s_list[1][j]].x, wkeys, pop_inh,
                               rotation);
        __syncthreads();
    }
    // Listed share of settle (first CTA), reported as the last phase counter.
    if (rank == 0 && tid == 0 && listed) sc->phase_cycles[LEO_PHASES - 1] += clock64() - t0;
    __syncthreads();
    // The touched list, in warp-aligned ranges: strided over the whole group,
    // or this CTA's own range when the shares are weighted.
    const uint32_t lo = weighted ? s_range[0] : 0u, hi = weighted ? s_range[1] : count;
    const uint32_t first = weighted ? lo + (tid - lane) : worker - lane, stride = weighted ? kThreads : workers;
    for (uint32_t base = first; base < hi; base += stride) {
        const uint32_t i = base + lane;
        const bool valid = i < hi;
        const uint32_t n = valid ? ln.touched[i] : 0u;
        uint2 seg = make_uint2(0u, LEO_SEG_LISTED);
        uint32_t k = 0;
        if (valid) {
            seg = kc.topo.seg[n];
            // An overrun count (events past the capacity were dropped and
            // flagged) never reads past the segment.
            k = min(ln.seg_count[n], seg.y & LEO_SEG_CAPACITY);
        }
        const bool listed = (seg.y & LEO_SEG_LISTED) != 0u;
        const bool alone = !listed && k <= kc.topo.thread_events;
        if (alone) settle_target_thread(ln, s, kc, n, k, seg.x, pop_inh, rotation);
        const bool by_warp = !listed && !alone && k <= kHubWarpEvents;
        if (!listed && !alone && !by_warp) {
            const uint32_t pos = atomicAdd(&s_nqueue, 1u);
            if (pos < kCtaQueue) {
                s_queue[pos] = n;
                s_queue_k[pos] = k;
            } else {
                atomicOr(&sc->error_flag, LEO_ERR_CAPACITY);
            }
        }
        unsigned int mask = __ballot_sync(0xffffffffu, by_warp);
        while (mask) {
            const int j = __ffs(mask) - 1;
            mask &= mask - 1u;
            const uint32_t nj = __shfl_sync(0xffffffffu, n, j), kj = __shfl_sync(0xffffffffu, k, j),
                           oj = __shfl_sync(0xffffffffu, seg.x, j);
            settle_target_warp(ln, s, kc, nj, kj, oj, wkeys, pop_inh, rotation);
        }
    }
    __syncthreads();
    const uint32_t nqueue = s_nqueue < kCtaQueue ? s_nqueue : kCtaQueue;
    for (uint32_t j = 0; j < nqueue; ++j)
        settle_target_cta(ln, s, kc, s_queue[j], s_queue_k[j], kc.topo.seg[s_queue[j]].x, smem, pop_inh, rotation);
}

// ---------------------------------------------------------------------------
// blocks: block-local top-k and the exact (k+1)-th cutoff (runtime.rs:964-997),
// one warp per block; keys are unique, so "largest key below the previous
// winner" enumerates the block in rank order.
//
// `winners` / `nwin` receive each block's winners and their count: the first
// CTA's shared memory (through the cluster's distributed shared memory) in
// the cluster wavefront, global memory in the whole-GPU launch.
__device__ void phase_blocks(const LaneState& ln, const KernelConsts& kc, uint32_t gwarp, uint32_t gwarps,
                             unsigned long long* winners, uint32_t* nwin) {
    const uint32_t B = kc.topo.blocks, npb = kc.topo.npb, keep = kc.topo.keep;
    const uint32_t lane = threadIdx.x & 31u;
    uint32_t supra = 0;
    for (uint32_t b = gwarp; b < B; b += gwarps) {
        uint32_t count = ln.block_cand_count[b];
        const unsigned long long* cand = ln.block_cand + (size_t)b * npb;
        // The first 256 candidates in registers (static indices; a key of a
        // candidate is never 0), the rest re-read from global memory per round.
        constexpr uint32_t kLocal = 8;
        unsigned long long mine[kLocal];
#pragma unroll
        for (uint32_t x = 0; x < kLocal; ++x) mine[x] = lane + 32u * x < count ? cand[lane + 32u * x] : 0ull;
        bool spill = count > 32 * kLocal;
        unsigned long long prev = ~0ull;
        uint32_t rounds = count < keep + 1 ? count : keep + 1;
        float cutoff = 0.0f;
        for (uint32_t k = 0; k < rounds; ++k) {
            unsigned long long best = 0ull;
#pragma unroll
            for (uint32_t x = 0; x < kLocal; ++x)
                if (mine[x] < prev && mine[x] > best) best = mine[x];
            if (spill)
                for (uint32_t idx = lane + 32 * kLocal; idx < count; idx += 32) {
                    unsigned long long key = cand[idx];
                    if (key < prev && key > best) best = key;
                }
            for (int o = 16; o > 0; o >>= 1) {
                unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
                best = other > best ? other : best;
            }
            if (k < keep) {
                if (lane == 0) winners[(size_t)b * keep + k] = best;
            } else {
                cutoff = key_value(best);
            }
            prev = best;
        }
        if (lane == 0) {
            nwin[b] = count < keep ? count : keep;
            ln.block_cutoff[b] = count > keep ? cutoff : 0.0f;
            ln.block_cand_count[b] = 0;
            supra += count;
        }
    }
    if (lane == 0 && supra) atomicAdd(&ln.sc->step_supra, supra);
}

// ---------------------------------------------------------------------------
// assemble (one CTA): active list in block order, the global cap
// (runtime.rs:998-1064), population inhibition (runtime.rs:1076-1082), the
// active ring entry, activations, and the actives as learning destinations.
//
// `nwin` / `winners`: the blocks phase's winner counts and winners (global in
// the wavefront's global arrays or the first CTA's shared memory); `active_out`, when
// given, receives the step's active count from thread 0.
__device__ void phase_assemble(const LaneState& ln, uint32_t s, const KernelConsts& kc, bool learning,
                               unsigned long long* sorted, const uint32_t* nwin, const unsigned long long* winners,
                               uint32_t* active_out) {
    __shared__ uint32_t s_offset[1025];
    __shared__ uint32_t s_warp_sums[kWarps];
    LaneScalars* sc = ln.sc;
    const LeoConfig& c = kc.cfg;
    const uint32_t B = kc.topo.blocks, keep = kc.topo.keep, n_count = kc.topo.n, maxa = kc.topo.max_active;
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t rotation = (uint32_t)((sc->base_tick + s) % (unsigned long long)n_count);
    // Thread 0's scalars, loaded now so their latency overlaps the scan.
    float pop_inh = 0.0f;
    uint32_t supra = 0;
    if (tid == 0) {
        pop_inh = sc->population_inhibition;
        supra = sc->step_supra;
    }
    // exclusive scan of block winner counts (B <= 1024, two blocks per thread)
    uint32_t b0 = 2 * tid, b1 = 2 * tid + 1;
    uint32_t v0 = b0 < B ? nwin[b0] : 0u, v1 = b1 < B ? nwin[b1] : 0u;
    uint32_t pair = v0 + v1, incl = pair;
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= (uint32_t)o) incl += y;
    }
    if (lane == 31) s_warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < kWarps ? s_warp_sums[lane] : 0u, wi = w;
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t y = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= (uint32_t)o) wi += y;
        }
        if (lane < kWarps) s_warp_sums[lane] = wi - w;
    }
    __syncthreads();
    uint32_t excl = s_warp_sums[warp] + incl - pair;
    if (b0 < B) s_offset[b0] = excl;
    if (b1 < B) s_offset[b1] = excl + v0;
    if (tid == kThreads - 1) s_offset[B] = excl + pair;  // thread kThreads-1 holds the grand total
    __syncthreads();
    uint32_t selected = s_offset[B];
    for (uint32_t i = tid; i < B * keep; i += kThreads) {
        uint32_t b = i / keep, k = i - b * keep;
        if (k < nwin[b]) sorted[s_offset[b] + k] = winners[i];
    }
    __syncthreads();
    uint32_t cap = c.max_active_global;
    uint32_t active = selected;
    float pop_cutoff = 0.0f;
    uint32_t clipped = 0;
    bool redundant = cap >= B * keep;
    if (!redundant && selected > 0) {
        // Global rank (runtime.rs:1014-1030): bitonic sort descending.
        uint32_t span = 1;
        while (span < selected) span <<= 1;
        for (uint32_t i = selected + tid; i < span; i += kThreads) sorted[i] = 0ull;
        __syncthreads();
        for (uint32_t width = 2; width <= span; width <<= 1) {
            for (uint32_t stride = width >> 1; stride > 0; stride >>= 1) {
                for (uint32_t i = tid; i < span; i += kThreads) {
                    uint32_t other = i ^ stride;
                    if (other > i) {
                        bool descending = (i & width) == 0;
                        unsigned long long a = sorted[i], b = sorted[other];
                        if (descending ? (a < b) : (a > b)) {
                            sorted[i] = b;
                            sorted[other] = a;
                        }
                    }
                }
                __syncthreads();
            }
        }
        if (selected > cap) {
            // The cutoff is the first clipped neuron's margin clamped to
            // [0, population_inhibition_max] -- not its activation, which is
            // clamped to [0, 1] -- so a saturated neuron can set a cutoff
            // above 1 (runtime.rs:1045-1050).
            const uint32_t cut = key_neuron(sorted[cap], rotation, n_count);
            pop_cutoff = clampf(ln.cold[cut].membrane - ln.p.threshold[cut], 0.0f, c.population_inhibition_max);
            clipped = selected - cap;
            active = cap;
        }
    }
    uint32_t entry = s % LEO_RING;
    for (uint32_t r = tid; r < active; r += kThreads) {
        unsigned long long key = sorted[r];
        uint32_t n = key_neuron(key, rotation, n_count);
        float act = key_value(key);
        ln.ring_src[entry * maxa + r] = n;
        ln.ring_act[entry * maxa + r] = act;
        ln.hot[n].activation = act;
        // Every active neuron is a learning destination (runtime.rs:1240-1245);
        // the destination list is read only by a learning step's learn phase.
        if (learning) add_destination(ln, n, s + 1);
    }
    if (tid == 0) {
        if (active_out) *active_out = active;
        ln.step_active[s] = active;
        sc->ring_count[entry] = active;
        float activity = (float)active / (float)(n_count > 0 ? n_count : 1);
        float error = activity - c.target_activity;
        sc->population_inhibition =
            clampf(pop_inh + c.population_inhibition_rate * error, 0.0f, c.population_inhibition_max);
        sc->population_cutoff = redundant ? 0.0f : pop_cutoff;
        sc->last_active = active;
        sc->last_suprathreshold = supra;
        sc->last_block_selected = selected;
        sc->last_clipped = clipped;
        sc->step_supra = 0;
    }
}

// ---------------------------------------------------------------------------
// surrogate: runtime.rs:787-803 plus the Jacobians of runtime.rs:775-783 /
// learning.rs:28-50, packed into the 32-byte record the eligibility gather reads.
__device__ void phase_surrogate(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t worker,
                                uint32_t workers) {
    const LeoConfig& c = kc.cfg;
    const uint32_t npb = kc.topo.npb;
    LaneScalars* sc = ln.sc;
    uint32_t count = sc->touched_count;
    float pop_cutoff = sc->population_cutoff;
    for (uint32_t i = worker; i < count; i += workers) {
        uint32_t n = ln.touched[i];
        NeuronHot h = ln.hot[n];
        bool refractory = h.refractory_until > s;
        bool selected = h.activation > 0.0f;
        float surrogate = 0.0f;
        if (!refractory) {
            float margin = ln.cold[n].membrane - ln.p.threshold[n];
            float cutoff = rmax(ln.block_cutoff[n / npb], pop_cutoff);
            float direct = (selected && margin > 0.0f && margin < 1.0f) ? 1.0f : 0.0f;
            surrogate = direct;
            if (c.surrogate_width > 0.0f && c.surrogate_gain > 0.0f) {
                float boundary = clampf(1.0f - fabsf(margin - cutoff) / c.surrogate_width, 0.0f, 1.0f);
                surrogate = direct + c.surrogate_gain * boundary;
            }
        }
        float4 br = ln.branches[n];
        float exc = kc.topo.excitability[n];
        float gate = clampf(br.w, 0.0f, 1.0f);
        float gate_derivative = (br.w > 0.0f && br.w < 1.0f) ? 1.0f : 0.0f;
        h.tag = ((s + 1u) << 2) | (selected ? 2u : 0u) | (refractory ? 0u : 1u);
        h.surrogate = surrogate;
        h.j_exc = exc;
        h.j_temporal = exc * gate;
        h.j_gate = exc * br.z * gate_derivative;
        ln.hot[n] = h;
    }
}

// ---------------------------------------------------------------------------
// eligible: runtime.rs:832-918 over the recurrent and input worklists.  Kept
// slots go to the next worklist with one atomic per warp (ballot compaction)
// and their destinations become learning destinations.
template <bool kInput>
__device__ __forceinline__ void eligibility_item(const LaneState& ln, const KernelConsts& kc, uint32_t s, uint2 entry,
                                                 bool valid, uint32_t next, uint32_t& plastic) {
    const LeoConfig& c = kc.cfg;
    LaneScalars* sc = ln.sc;
    bool keep = false;
    uint32_t dest = 0;
    float e = 0.0f;
    if (valid) {
        Trace* tp = kInput ? &ln.in_traces[entry.x] : &ln.traces[entry.x];
        const uint32_t word = kInput ? kc.topo.in_word[entry.x] : kc.topo.rec_word[entry.x];
        Trace t = load_trace(tp);
        advance_trace(c, t, s);
        dest = word & LEO_TARGET_MASK;
        uint32_t branch = LEO_WORD_BRANCH(word);
        NeuronHot h = ln.hot[dest];
        bool touched_now = (h.tag >> 2) == s + 1u;
        if (!(touched_now && (h.tag & 1u))) {
            e = t.eligibility * c.eligibility_decay;
        } else {
            float j = branch == 2u ? h.j_temporal : (branch == 3u ? h.j_gate : h.j_exc);
            float adaptation_sum = sum3(t.adaptation_sens[0], t.adaptation_sens[1], t.adaptation_sens[2]);
            float ms = t.membrane_sens + j * t.branch_sens - t.fatigue_sens - adaptation_sum;
            t.membrane_sens = ms;
            e = h.surrogate * ms;
        }
        t.eligibility = e;
        if (touched_now && (h.tag & 2u)) {
            t.fatigue_sens = t.fatigue_sens + c.fatigue_gain * e;
            t.adaptation_sens[0] = t.adaptation_sens[0] + c.adaptation_fast_gain * e;
            t.adaptation_sens[1] = t.adaptation_sens[1] + c.adaptation_medium_gain * e;
            t.adaptation_sens[2] = t.adaptation_sens[2] + c.adaptation_slow_gain * e;
        }
        float mag = rmax(rmax(rmax(fabsf(t.branch_sens), fabsf(t.membrane_sens)), fabsf(t.fatigue_sens)), fabsf(e));
        mag = rmax(mag, fabsf(t.adaptation_sens[0]));
        mag = rmax(mag, fabsf(t.adaptation_sens[1]));
        mag = rmax(mag, fabsf(t.adaptation_sens[2]));
        keep = mag > c.eligibility_epsilon;
        t.tick_mark = (t.tick_mark & ~1u) | (keep ? 1u : 0u);
        store_trace(tp, t);
    }
    unsigned int ballot = __ballot_sync(0xffffffffu, keep);
    uint32_t lane = threadIdx.x & 31u;
    plastic += (keep && e != 0.0f) ? 1u : 0u;
    uint32_t base = 0;
    if (ballot) {
        uint32_t* counter = kInput ? &sc->in_elig_count[next] : &sc->elig_count[next];
        int leader = __ffs(ballot) - 1;
        if ((int)lane == leader) base = atomicAdd(counter, (uint32_t)__popc(ballot));
        base = __shfl_sync(0xffffffffu, base, leader);
    }
    if (keep) {
        uint32_t pos = base + (uint32_t)__popc(ballot & ((1u << lane) - 1u));
        uint2* out = kInput ? ln.in_elig[next] : ln.elig[next];
        out[pos] = make_uint2(entry.x, __float_as_uint(e));
        // A slot with eligibility +-0 leaves its weight bit-for-bit unchanged
        // (old + (+-0) = old for every weight the model can hold, since no
        // update produces -0), so only nonzero-eligibility slots need their
        // destination's learning signal.
        if (e != 0.0f) add_destination(ln, dest, s + 1);
    }
}

__device__ void phase_eligible(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t worker,
                               uint32_t workers) {
    LaneScalars* sc = ln.sc;
    const uint32_t cur = sc->elig_cur, next = cur ^ 1u;
    uint32_t rec = sc->elig_count[cur], inp = sc->in_elig_count[cur];
    uint32_t rec_pad = (rec + 31u) & ~31u;
    uint32_t total = rec_pad + inp;
    uint32_t plastic = 0;
    // Warp-uniform iteration over warp-aligned ranges: each ballot covers one list.
    for (uint32_t base = worker & ~31u; base < total; base += workers) {
        uint32_t i = base + (threadIdx.x & 31u);
        if (base < rec_pad) {
            bool valid = i < rec;
            uint2 entry = valid ? ln.elig[cur][i] : make_uint2(0, 0);
            eligibility_item<false>(ln, kc, s, entry, valid, next, plastic);
        } else {
            uint32_t k = i - rec_pad;
            bool valid = k < inp;
            uint2 entry = valid ? ln.in_elig[cur][k] : make_uint2(0, 0);
            eligibility_item<true>(ln, kc, s, entry, valid, next, plastic);
        }
    }
    // Work counter: one add per warp per step (kept slots with nonzero eligibility).
    plastic = __reduce_add_sync(0xffffffffu, plastic);
    if ((threadIdx.x & 31u) == 0u && plastic) atomicAdd(&sc->work_plastic, (unsigned long long)plastic);
}

// ---------------------------------------------------------------------------
// forward (one CTA): logits, context latent, softmax, loss, errors, output bias
// and context learning (runtime.rs:1108-1197, 1199-1384), step statistics
// (runtime.rs:1595-1622).
__device__ void phase_forward(const LaneState& ln, uint32_t s, const KernelConsts& kc) {
    __shared__ float s_logits[LEO_OUTPUT_STRIDE];
    __shared__ float s_probs[LEO_OUTPUT_STRIDE];
    __shared__ float s_latent[LEO_MAX_EMBEDDING];
    __shared__ float s_grad[LEO_MAX_EMBEDDING];
    __shared__ float s_act[1024];
    __shared__ const float* s_row[1024];
    __shared__ float s_max, s_sum;
    LaneScalars* sc = ln.sc;
    const LeoConfig& c = kc.cfg;
    const uint32_t D = kc.topo.d, S = kc.topo.s, maxa = kc.topo.max_active;
    const uint32_t sched = ln.schedule[s];
    const uint32_t perm = LEO_SCHED_PERMISSION(sched);
    const int target = LEO_SCHED_TARGET(sched);
    const uint32_t symbol = LEO_SCHED_SYMBOL(sched);
    const bool frozen = perm == kFrozen;
    const uint32_t entry = s % LEO_RING;
    const uint32_t active = sc->ring_count[entry];
    const uint32_t tid = threadIdx.x;
    const int target_index = target < 0 ? -1 : (target < 256 ? target : 256);

    for (uint32_t r = tid; r < active; r += kThreads) {
        uint32_t n = ln.ring_src[entry * maxa + r];
        const float* rows = ln.out_mark[n] ? ln.p.out_weight : ln.canon_out_weight;
        s_row[r] = rows + (size_t)n * LEO_OUTPUT_STRIDE;
        s_act[r] = ln.ring_act[entry * maxa + r];
    }
    __syncthreads();
    // logits (runtime.rs:1109-1116): bias, then each active neuron in active order
    if (tid < LEO_OUTPUT_CLASSES) {
        float logit = ln.p.out_bias[tid];
        uint32_t r = 0;
        for (; r + 4 <= active; r += 4) {
            float w0 = s_row[r][tid];
            float w1 = s_row[r + 1][tid];
            float w2 = s_row[r + 2][tid];
            float w3 = s_row[r + 3][tid];
            logit = logit + w0 * s_act[r];
            logit = logit + w1 * s_act[r + 1];
            logit = logit + w2 * s_act[r + 2];
            logit = logit + w3 * s_act[r + 3];
        }
        for (; r < active; ++r) logit = logit + s_row[r][tid] * s_act[r];
        s_logits[tid] = logit;
    }
    // context latent (runtime.rs:1118-1136)
    uint32_t ctx_count = sc->ctx_count;
    if (tid < D) {
        float v = 0.0f;
        for (uint32_t i = 0; i < ctx_count; ++i) {
            float scale = sc->ctx_scales[i];
            if (scale <= 0.0f) continue;
            v = v + ln.p.ctx_emb[(size_t)sc->ctx_slots[i] * D + tid] * scale;
        }
        s_latent[tid] = v;
    }
    __syncthreads();
    if (ctx_count > 0 && tid < LEO_OUTPUT_CLASSES) {
        float contribution = 0.0f;
        for (uint32_t k = 0; k < D; ++k) contribution = contribution + ln.p.ctx_out[(size_t)tid * D + k] * s_latent[k];
        s_logits[tid] = s_logits[tid] + contribution;
    }
    __syncthreads();
    // normalize_probabilities (runtime.rs:1167-1188)
    if (tid < 32) {
        float m = -INFINITY;
        for (uint32_t o = tid; o < LEO_OUTPUT_CLASSES; o += 32) m = rmax(m, s_logits[o]);
        for (int off = 16; off > 0; off >>= 1) m = rmax(m, __shfl_xor_sync(0xffffffffu, m, off));
        if (tid == 0) s_max = m;
    }
    __syncthreads();
    if (tid < LEO_OUTPUT_CLASSES) s_probs[tid] = leo_expf(kc, s_logits[tid] - s_max);
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;
        for (uint32_t o = 0; o < LEO_OUTPUT_CLASSES; ++o) sum = sum + s_probs[o];
        s_sum = sum;
    }
    __syncthreads();
    if (tid < LEO_OUTPUT_CLASSES) {
        float sum = s_sum;
        float p = (!isfinite(sum) || sum <= 0.0f) ? 1.0f / (float)LEO_OUTPUT_CLASSES : s_probs[tid] / sum;
        s_probs[tid] = p;
        ln.probs[tid] = p;
    }
    __syncthreads();
    if (tid == 0) {
        // argmax_probability (runtime.rs:1190-1197): the lowest index among equal maxima
        int best = 0;
        for (uint32_t o = 1; o < LEO_OUTPUT_CLASSES; ++o)
            if (s_probs[o] > s_probs[best]) best = (int)o;
        sc->last_predicted = best == 256 ? 257u : (uint32_t)best;
        float loss = 0.0f;
        if (target_index >= 0) loss = -leo_logf(kc, rmax(s_probs[target_index], 1.0e-12f));
        sc->last_loss = loss;
        ln.step_loss[s] = loss;
    }
    __syncthreads();

    float strength = kc.strength[perm];
    bool learning = target_index >= 0 && strength > 0.0f;
    if (learning) {
        float target_weight = target_index == 256 ? kc.end_document_weight : 1.0f;
        float supervised = strength * target_weight;
        // plasticity_step (config.rs:137-145)
        uint32_t window = kc.plasticity_window > 0 ? kc.plasticity_window : 1u;
        uint32_t phase = sc->plasticity_phase;
        uint32_t step = (phase < window - 1 ? phase : window - 1) + 1;
        float plasticity = 0.0f;
        uint32_t next_phase = step;
        if (step == window || target_index == 256) {
            plasticity = (float)step;
            next_phase = 0;
        }
        if (tid < LEO_OUTPUT_CLASSES) {
            float err = tid == (uint32_t)target_index ? s_probs[tid] - 1.0f : s_probs[tid];
            s_probs[tid] = err;  // errors (runtime.rs:1205-1206)
            ln.errors[tid] = err;
            float raw = -c.output_learning_rate * supervised * err;
            float bias = ln.p.out_bias[tid] + clampf(raw, -c.max_update, c.max_update);
            ln.p.out_bias[tid] = bias;
            if (!isfinite(bias)) atomicOr(&sc->error_flag, LEO_ERR_NONFINITE_BIAS);
        }
        __syncthreads();
        if (sc->ctx_applied && ctx_count > 0) {  // update_context_projection (runtime.rs:1318-1384)
            if (tid < D) {
                float g = 0.0f;
                for (uint32_t o = 0; o < LEO_OUTPUT_CLASSES; ++o) g = g + ln.p.ctx_out[(size_t)o * D + tid] * s_probs[o];
                s_grad[tid] = g;
            }
            __syncthreads();
            float lr = c.context_learning_rate;
            for (uint32_t i = tid; i < LEO_OUTPUT_CLASSES * D; i += kThreads) {
                uint32_t o = i / D, k = i - o * D;
                float gradient = s_probs[o] * s_latent[k];
                float delta = clampf(-lr * supervised * gradient, -c.max_update, c.max_update);
                float updated = clampf(ln.p.ctx_out[i] + delta, c.weight_min, c.weight_max);
                if (!isfinite(updated)) atomicOr(&sc->error_flag, LEO_ERR_NONFINITE_CONTEXT);
                ln.p.ctx_out[i] = updated;
            }
            for (uint32_t i = tid; i < ctx_count * D; i += kThreads) {
                uint32_t ci = i / D, k = i - ci * D;
                uint32_t slot = sc->ctx_slots[ci];
                float gradient = sc->ctx_scales[ci] * s_grad[k];
                float delta = clampf(-lr * supervised * gradient, -c.max_update, c.max_update);
                size_t idx = (size_t)slot * D + k;
                float updated = clampf(ln.p.ctx_emb[idx] + delta, c.weight_min, c.weight_max);
                if (!isfinite(updated)) atomicOr(&sc->error_flag, LEO_ERR_NONFINITE_CONTEXT);
                ln.p.ctx_emb[idx] = updated;
            }
            __syncthreads();
            if (tid == 0) {
                for (uint32_t ci = 0; ci < ctx_count; ++ci) {
                    uint32_t slot = sc->ctx_slots[ci];
                    if (kc.track_changes && ln.ctx_mark[slot] == 0) {
                        ln.ctx_mark[slot] = 1;
                        ln.ctx_list[sc->ctx_changed++] = slot;
                    }
                    if (ln.p.ctx_obs[slot] != 0xffffffffu) ln.p.ctx_obs[slot] += 1;
                }
                if (kc.track_changes) sc->ctx_out_dirty = 1;
            }
        }
        if (tid == 0) {
            sc->step_flags = 1u | (plasticity > 0.0f ? 2u : 0u) | 4u;
            sc->step_strength = strength;
            sc->step_supervised = supervised;
            sc->step_consolidated = supervised * plasticity;
            sc->plasticity_phase = next_phase;
            sc->revision_increment += 1;
            if (kc.track_changes) sc->bias_dirty = 1;
        }
    } else if (tid == 0) {
        sc->step_flags = frozen ? 0u : 4u;
    }
    if (tid == 0 && !frozen) {  // update_statistics (runtime.rs:1595-1622)
        if (symbol < 256) sc->processed_bytes += 1;
        if (target_index >= 0) {
            sc->loss_sum += (double)sc->last_loss;
            sc->targets += 1;
        }
        sc->active_sum += active;
        if (active > sc->active_peak) sc->active_peak = active;
        sc->synaptic_events += (unsigned long long)active * S;
        sc->persistent_ticks += 1;
        sc->context_applied_steps += sc->ctx_applied ? 1 : 0;
    }
}

// emit: post-activation dynamics and emission (runtime.rs:920-938, 1084-1106).
__device__ void phase_emit(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t worker,
                           uint32_t workers) {
    const LeoConfig& c = kc.cfg;
    const uint32_t S = kc.topo.s, maxa = kc.topo.max_active;
    uint32_t entry = s % LEO_RING;
    uint32_t total = ln.sc->ring_count[entry] * S;
    for (uint32_t i = worker; i < total; i += workers) {
        uint32_t r = i / S, j = i - r * S;
        uint32_t n = ln.ring_src[entry * maxa + r];
        float a = ln.ring_act[entry * maxa + r];
        if (j == 0) {
            NeuronCold cold = ln.cold[n];
            cold.fatigue = cold.fatigue + c.fatigue_gain * a;
            cold.adaptation[0] = cold.adaptation[0] + c.adaptation_fast_gain * a;
            cold.adaptation[1] = cold.adaptation[1] + c.adaptation_medium_gain * a;
            cold.adaptation[2] = cold.adaptation[2] + c.adaptation_slow_gain * a;
            cold.membrane = cold.membrane - ln.p.threshold[n] * c.membrane_reset_fraction;
            ln.cold[n] = cold;
            ln.hot[n].refractory_until = s + c.refractory_ticks + 1u;
        }
        ln.ring_val[((size_t)entry * maxa + r) * S + j] = a * ln.p.rec_weight[(size_t)n * S + j];
    }
}

// ---------------------------------------------------------------------------
// learn: learning signals for every destination (runtime.rs:1246-1262), the
// output row of each active destination after its signal (runtime.rs:1267-1283),
// threshold homeostasis over the touched neurons (runtime.rs:1567-1593).
//
// Signals: each warp takes 32 destination rows.  For each 32-column chunk it
// loads a 32 x 32 tile (lane j reads column j of every row: one coalesced
// 128-byte segment per row, 32 independent loads in flight per lane), stores
// it transposed into padded shared memory, and lane r then adds row r's 32
// products in column order.  Every row's sum is formed strictly in output
// order, exactly like the CPU's sequential loop.
__device__ __forceinline__ const float* output_row(const LaneState& ln, uint32_t n) {
    return (ln.out_mark[n] ? ln.p.out_weight : ln.canon_out_weight) + (size_t)n * LEO_OUTPUT_STRIDE;
}

__device__ void phase_learn(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t worker,
                            uint32_t workers, uint32_t gwarp, uint32_t gwarps, float (*s_tile)[32][33]) {
    __shared__ float s_err[LEO_OUTPUT_STRIDE];
    const LeoConfig& c = kc.cfg;
    const uint32_t n_count = kc.topo.n;
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    LaneScalars* sc = ln.sc;
    uint32_t flags = sc->step_flags;
    bool learning = flags & 1u, plastic = flags & 2u, persistent = flags & 4u;
    uint32_t dsts = learning ? sc->dst_count : 0u;
    uint32_t touched = persistent ? sc->touched_count : 0u;
    for (uint32_t o = threadIdx.x; o < LEO_OUTPUT_CLASSES; o += kThreads) s_err[o] = ln.errors[o];
    __syncthreads();
    float supervised = sc->step_supervised;
    // Learning signals, 32 destinations per warp, then -- by the lane that owns
    // the row, after its signal was read -- the output row of an active
    // destination.  Every destination occurs once in the list, so no other
    // thread reads a row that this warp rewrites.
    for (uint32_t base = gwarp * 32u; base < dsts; base += gwarps * 32u) {
        uint32_t rows = dsts - base < 32u ? dsts - base : 32u;
        uint32_t my_n = lane < rows ? ln.dst_list[base + lane] : 0u;
        const float* my_row = output_row(ln, my_n);
        if (plastic) {
            float signal = 0.0f;
            for (uint32_t chunk = 0; chunk < 8; ++chunk) {
                float v[32];
#pragma unroll
                for (uint32_t r = 0; r < 32; ++r) {
                    const float* row = (const float*)__shfl_sync(0xffffffffu, (unsigned long long)my_row, (int)r);
                    v[r] = r < rows ? row[chunk * 32u + lane] : 0.0f;
                }
#pragma unroll
                for (uint32_t r = 0; r < 32; ++r) s_tile[warp][r][lane] = v[r];
                __syncwarp();
                if (lane < rows) {
#pragma unroll
                    for (uint32_t j = 0; j < 32; ++j) signal = signal + s_tile[warp][lane][j] * s_err[chunk * 32u + j];
                }
                __syncwarp();
            }
            if (lane < rows) {
                signal = signal + my_row[256] * s_err[256];
                ln.signal[my_n] = signal;
            }
        }
        if (lane < rows) {
            float a = ln.hot[my_n].activation;
            if (a > 0.0f) {
                float* row = ln.p.out_weight + (size_t)my_n * LEO_OUTPUT_STRIDE;
                for (uint32_t o = 0; o < LEO_OUTPUT_CLASSES; ++o) {
                    float raw = -c.output_learning_rate * supervised * s_err[o] * a;
                    float delta = clampf(raw, -c.max_update, c.max_update);
                    row[o] = clampf(my_row[o] + delta, c.weight_min, c.weight_max);
                }
                if (kc.track_changes) mark_and_append(ln.out_mark, ln.out_list, &sc->out_changed, my_n);
            }
        }
    }
    // threshold homeostasis
    uint32_t active = sc->ring_count[s % LEO_RING];
    float pop_error = (float)active / (float)(n_count > 0 ? n_count : 1) - c.target_activity;
    for (uint32_t i = worker; i < touched; i += workers) {
        uint32_t n = ln.touched[i];
        float local = ln.hot[n].activation > 0.0f ? 1.0f : 0.0f;
        float local_error = local - c.target_activity;
        float delta = c.threshold_homeostasis_rate * (local_error + pop_error);
        float old_t = ln.p.threshold[n];
        float new_t = clampf(old_t + delta, 0.05f, 2.0f);
        if (new_t != old_t && kc.track_changes) mark_and_append(ln.thr_mark, ln.thr_list, &sc->thr_changed, n);
        ln.p.threshold[n] = new_t;
    }
}

// plasticity: update_recurrent_synapses / update_input_synapses
// (runtime.rs:1451-1523) over the post-compaction worklists.
__device__ void phase_plasticity(const LaneState& ln, const KernelConsts& kc, uint32_t worker, uint32_t workers) {
    const LeoConfig& c = kc.cfg;
    const uint32_t S = kc.topo.s;
    LaneScalars* sc = ln.sc;
    if ((sc->step_flags & 3u) != 3u) return;
    float strength = sc->step_consolidated;
    const uint32_t next = sc->elig_cur ^ 1u;
    uint32_t rec = sc->elig_count[next], inp = sc->in_elig_count[next];
    uint32_t total = rec + inp;
    for (uint32_t i = worker; i < total; i += workers) {
        if (i < rec) {
            const uint2 e2 = ln.elig[next][i];
            if (__uint_as_float(e2.y) == 0.0f) continue;  // unchanged weight (see eligibility_item)
            uint32_t slot = e2.x, dest = kc.topo.rec_word[slot] & LEO_TARGET_MASK;
            float gradient = ln.signal[dest] * __uint_as_float(e2.y);
            float delta = clampf(-c.recurrent_learning_rate * strength * gradient, -c.max_update, c.max_update);
            float old_w = ln.p.rec_weight[slot];
            float nw = clampf(old_w + delta, c.weight_min, c.weight_max);
            nw = kc.topo.neuron_type[slot / S] == 0 ? rmax(nw, 0.0f) : rmin(nw, 0.0f);
            if (!isfinite(nw)) {
                atomicOr(&sc->error_flag, LEO_ERR_NONFINITE_RECURRENT);
                atomicAdd(&sc->numerical_rejections, 1ull);
            }
            if (nw != old_w && kc.track_changes) mark_and_append(ln.rec_mark, ln.rec_list, &sc->rec_changed, slot);
            ln.p.rec_weight[slot] = nw;
        } else {
            const uint2 e2 = ln.in_elig[next][i - rec];
            if (__uint_as_float(e2.y) == 0.0f) continue;
            uint32_t slot = e2.x, dest = kc.topo.in_word[slot] & LEO_TARGET_MASK;
            float gradient = ln.signal[dest] * __uint_as_float(e2.y);
            float delta = clampf(-c.recurrent_learning_rate * strength * gradient, -c.max_update, c.max_update);
            float old_w = ln.p.in_weight[slot];
            float nw = clampf(old_w + delta, 0.0f, c.weight_max);
            if (!isfinite(nw)) atomicOr(&sc->error_flag, LEO_ERR_NONFINITE_INPUT);
            if (nw != old_w && kc.track_changes) mark_and_append(ln.in_mark, ln.in_list, &sc->in_changed, slot);
            ln.p.in_weight[slot] = nw;
        }
    }
}

// inhibit: apply_inhibitory_homeostasis (runtime.rs:1525-1565), after the
// recurrent update.
__device__ void phase_inhibit(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t worker,
                              uint32_t workers) {
    const LeoConfig& c = kc.cfg;
    const uint32_t S = kc.topo.s, maxa = kc.topo.max_active;
    LaneScalars* sc = ln.sc;
    if (!(sc->step_flags & 1u)) return;
    float strength = sc->step_strength;
    uint32_t entry = s % LEO_RING;
    uint32_t total = sc->ring_count[entry] * S;
    uint32_t visited = 0;
    for (uint32_t i = worker; i < total; i += workers) {
        uint32_t r = i / S, j = i - r * S;
        uint32_t src = ln.ring_src[entry * maxa + r];
        if (kc.topo.neuron_type[src] == 0) continue;
        ++visited;
        float sa = ln.ring_act[entry * maxa + r];
        uint32_t slot = src * S + j;
        uint32_t target = kc.topo.rec_word[slot] & LEO_TARGET_MASK;
        float tact = ln.hot[target].activation > 0.0f ? 1.0f : 0.0f;
        float err = tact - c.target_activity;
        float delta = clampf(-c.inhibitory_learning_rate * strength * sa * err, -c.max_update, c.max_update);
        float old_w = ln.p.rec_weight[slot];
        float nw = clampf(old_w + delta, c.weight_min, 0.0f);
        if (!isfinite(nw)) atomicOr(&sc->error_flag, LEO_ERR_NONFINITE_INHIBITORY);
        if (nw != old_w && kc.track_changes) mark_and_append(ln.rec_mark, ln.rec_list, &sc->rec_changed, slot);
        ln.p.rec_weight[slot] = nw;
    }
    // Work counter: one add per warp per step.
    visited = __reduce_add_sync(0xffffffffu, visited);
    if ((threadIdx.x & 31u) == 0u && visited) atomicAdd(&sc->work_inhibit, (unsigned long long)visited);
}

// Work counters of one launch, held by the launch's first thread and added to
// the lane's scalars when the launch ends.
struct WorkTally {
    unsigned long long deliver, touched, active, steps, eligible, destinations, winners;
};

// Step epilogue (one thread): work counters, per-tick counter reset, and the
// worklist swap after an eligibility phase.  Every load is issued before the
// stores so the thread's chain is one round trip.
// A frozen step's touched list is released in its blocks phase (see
// release_touched), so the next step's deliver may run beside this epilogue.
__device__ void step_epilogue(const LaneState& ln, uint32_t s, bool frozen, WorkTally& tally) {
    LaneScalars* sc = ln.sc;
    const uint32_t cur = sc->elig_cur;
    const uint32_t touched = frozen ? 0u : sc->touched_count, active = sc->ring_count[s % LEO_RING];
    const uint32_t flags = sc->step_flags, dsts = sc->dst_count;
    const uint32_t e0 = sc->elig_count[0] + sc->in_elig_count[0], e1 = sc->elig_count[1] + sc->in_elig_count[1];
    tally.touched += touched;
    tally.active += active;
    tally.winners += sc->last_block_selected;
    tally.steps += 1;
    if (!frozen) tally.eligible += cur ? e1 : e0;
    if ((flags & 3u) == 3u) tally.destinations += dsts;
    if (!frozen) sc->touched_count = 0;
    sc->dst_count = 0;
    if (!frozen) sc->elig_cur = cur ^ 1u;
}

// After settle, a frozen step reads its touched list no more (no surrogate,
// eligibility or learning follows): count it and empty it (one thread).
__device__ __forceinline__ void release_touched(const LaneState& ln, WorkTally& tally) {
    tally.touched += ln.sc->touched_count;
    ln.sc->touched_count = 0;
}

__device__ void flush_tally(const LaneState& ln, const WorkTally& tally) {
    LaneScalars* sc = ln.sc;
    sc->work_deliver += tally.deliver;
    sc->work_touched += tally.touched;
    sc->work_active += tally.active;
    sc->work_steps += tally.steps;
    sc->work_eligible += tally.eligible;
    sc->work_destinations += tally.destinations;
    sc->work_winners += tally.winners;
}

__device__ __forceinline__ unsigned long long clock_now() { return clock64(); }

}  // namespace

// ---------------------------------------------------------------------------
// The persistent wavefront: the C CTAs of group blockIdx.x / C run that lane
// through steps [begin, end) of its schedule, `sync` separating the phases.
//
// `win_write` / `nwin_write`: where the blocks phase of every CTA puts the
// block winners; `win_read` / `nwin_read`: where the first CTA's assemble
// reads them (null: the lane's global arrays for both).
template <typename Sync>
__device__ __forceinline__ void wavefront_steps(const LaneState* __restrict__ lanes, uint32_t begin, uint32_t end,
                                                const KernelConsts& kc, uint32_t C, uint32_t rank, Sync sync,
                                                unsigned long long* smem_sorted, unsigned long long* win_write,
                                                uint32_t* nwin_write, const unsigned long long* win_read,
                                                const uint32_t* nwin_read) {
    const LaneState& ln = lanes[blockIdx.x / C];
    if (!win_write) {
        win_write = ln.block_winners;
        nwin_write = ln.block_nwin;
        win_read = ln.block_winners;
        nwin_read = ln.block_nwin;
    }
    LaneScalars* sc = ln.sc;
    const uint32_t steps = sc->steps;
    const uint32_t worker = rank * kThreads + threadIdx.x, workers = C * kThreads;
    // Warp-sized tasks (a block's top-k, 32 learning destinations) are dealt
    // over the CTAs first: task t runs on CTA t mod C, so a few hundred tasks
    // spread over every SM instead of filling the first CTAs' warps.
    const uint32_t gwarp = (threadIdx.x >> 5) * C + rank, gwarps = C * kWarps;
    const bool timer = rank == 0 && threadIdx.x == 0;
    // Phase clocks and work counters belong to the first thread alone; they
    // live in shared memory so they cost the other threads no registers.
    __shared__ unsigned long long acc[LEO_PHASES];
    __shared__ WorkTally tally;
    unsigned long long t0 = 0;
    auto mark = [&](int p) {
        if (timer) {
            unsigned long long t = clock_now();
            acc[p] += t - t0;
            t0 = t;
        }
    };
    if (timer) {
        for (int p = 0; p < LEO_PHASES; ++p) acc[p] = 0;
        tally = WorkTally{0, 0, 0, 0, 0, 0, 0};
        t0 = clock_now();
    }
    // `joined`: the previous step was frozen without a forward pass and its
    // emit phase is still open -- this step's deliver runs in it.  Nothing of
    // this step before settle reads what that emit writes except the delay-1
    // ring values, which deliver then forms from their operands.
    bool joined = false;
    for (uint32_t s = begin; s < end && s < steps; ++s) {
        const uint32_t sched = ln.schedule[s];
        const bool frozen = LEO_SCHED_PERMISSION(sched) == kFrozen;
        const uint32_t symbol = LEO_SCHED_SYMBOL(sched);
        // deliver; the cluster's last warp first resolves the context
        if (rank == C - 1 && (threadIdx.x >> 5) == kWarps - 1)
            context_resolve_warp(ln, s, kc, symbol, frozen, !frozen || LEO_SCHED_TARGET(sched) >= 0);
        const uint32_t delivered = phase_deliver(ln, s, kc, worker, workers, !frozen, symbol, joined);
        if (worker == 0) tally.deliver += delivered;
        sync();
        mark(0);
        phase_settle(ln, s, kc, worker, workers, rank, C, reinterpret_cast<uint32_t*>(smem_sorted));
        sync();
        mark(1);
        {
            // counts the settle phase kept for its busy listed targets
            const uint32_t top = kc.topo.cta_count < kThreads ? kc.topo.cta_count : kThreads;
            for (uint32_t i = worker; i < top; i += workers) ln.seg_count[kc.topo.cta_targets[i]] = 0u;
        }
        phase_blocks(ln, kc, gwarp, gwarps, win_write, nwin_write);
        if (frozen && worker == 0) release_touched(ln, tally);
        sync();
        mark(2);
        if (rank == 0) phase_assemble(ln, s, kc, !frozen, smem_sorted, nwin_read, win_read, nullptr);
        sync();
        mark(3);
        if (!frozen) {
            phase_surrogate(ln, s, kc, worker, workers);
            sync();
            mark(4);
            phase_eligible(ln, s, kc, worker, workers);
            sync();
            mark(5);
        }
        // emit beside the forward pass (the first CTA runs the forward)
        const bool forward = !frozen || LEO_SCHED_TARGET(sched) >= 0;
        if (rank == 0 && forward) phase_forward(ln, s, kc);
        if (C == 1) {
            if (forward) __syncthreads();
            phase_emit(ln, s, kc, threadIdx.x, kThreads);
        } else if (forward) {
            if (rank > 0) phase_emit(ln, s, kc, worker - kThreads, workers - kThreads);
        } else {
            phase_emit(ln, s, kc, worker, workers);
        }
        if (frozen && worker == 0) {
            if (!forward) sc->step_flags = 0;
            step_epilogue(ln, s, true, tally);
        }
        joined = !forward && s + 1 < end && s + 1 < steps;
        if (!joined) {
            sync();
            mark(6);
        }
        if (!frozen) {
            phase_learn(ln, s, kc, worker, workers, gwarp, gwarps, reinterpret_cast<float (*)[32][33]>(smem_sorted));
            sync();
            mark(7);
            phase_plasticity(ln, kc, worker, workers);
            sync();
            mark(8);
            phase_inhibit(ln, s, kc, worker, workers);
            if (worker == 0) step_epilogue(ln, s, false, tally);
            sync();
            mark(9);
        }
    }
    if (worker == 0) flush_tally(ln, tally);
    if (timer) {
        for (int p = 0; p < LEO_PHASES; ++p) sc->phase_cycles[p] += acc[p];
        if (ln.load_out) {
            const uint32_t cur = sc->elig_cur;
            const unsigned long long load = (unsigned long long)sc->elig_count[cur] + sc->in_elig_count[cur] +
                                            (unsigned long long)sc->last_active * kc.topo.s + sc->touched_count;
            *ln.load_out = load > 0xffffffffull ? 0xffffffffu : (uint32_t)load;
        }
    }
}

__host__ __device__ size_t wavefront_scratch_bytes(const KernelConsts& kc);

// A thread-block cluster per lane (phases separated by cluster barriers).
__global__ void __launch_bounds__(kThreads, 1)
    leo_wavefront_kernel(const LaneState* __restrict__ lanes, uint32_t begin, uint32_t end, KernelConsts kc) {
    extern __shared__ __align__(16) unsigned long long smem_sorted[];
    cg::cluster_group cluster = cg::this_cluster();
    // Block winners go straight to the first CTA's shared memory (distributed
    // shared memory), where its assemble reads them after the phase barrier.
    unsigned long long* win = smem_sorted + wavefront_scratch_bytes(kc) / sizeof(unsigned long long);
    uint32_t* nwin = reinterpret_cast<uint32_t*>(win + (size_t)kc.topo.blocks * kc.topo.keep);
    wavefront_steps(lanes, begin, end, kc, cluster.num_blocks(), cluster.block_rank(), [&] { cluster.sync(); },
                    smem_sorted, cluster.map_shared_rank(win, 0), cluster.map_shared_rank(nwin, 0), win, nwin);
}

// One lane over the whole GPU: one CTA per SM in a cooperative launch, phases
// separated by grid barriers.  For replay steps whose work (millions of
// eligible slots on large models) needs more bandwidth than one cluster's SMs.
__global__ void __launch_bounds__(kThreads, 1)
    leo_wavefront_grid_kernel(const LaneState* __restrict__ lanes, uint32_t begin, uint32_t end, KernelConsts kc) {
    extern __shared__ __align__(16) unsigned long long smem_sorted[];
    cg::grid_group grid = cg::this_grid();
    wavefront_steps(lanes, begin, end, kc, gridDim.x, blockIdx.x, [&] { grid.sync(); }, smem_sorted, nullptr, nullptr,
                    nullptr, nullptr);
}

// Dynamic shared memory: the assemble phase's sort buffer and the learn
// phase's transpose tiles share one region (the phases never overlap).
// Bytes of the phases' shared scratch (sort buffer, transpose tiles, hub
// sorts), a multiple of 16.
__host__ __device__ size_t wavefront_scratch_bytes(const KernelConsts& kc) {
    uint32_t winners = kc.topo.blocks * kc.topo.keep, span = 1;
    while (span < winners) span <<= 1;
    size_t sort = (size_t)span * sizeof(unsigned long long);
    size_t tiles = (size_t)kWarps * 32 * 33 * sizeof(float);
    size_t bytes = sort > tiles ? sort : tiles;
    // settle's sorts: the warps' slices, or one CTA's sort, whichever is larger
    const size_t warps = (size_t)kWarps * kHubWarpEvents * sizeof(uint32_t);
    const size_t cta = (size_t)kHubSortShared * sizeof(uint32_t);
    const size_t sorts = warps > cta ? warps : cta;
    bytes = bytes > sorts ? bytes : sorts;
    return (bytes + 15) & ~(size_t)15;
}

// The scratch, then the block winners (blocks x keep keys) and their counts.
size_t leo_wavefront_smem_bytes(const KernelConsts& kc) {
    const size_t winners = (size_t)kc.topo.blocks * kc.topo.keep;
    return wavefront_scratch_bytes(kc) + winners * sizeof(unsigned long long) + (size_t)kc.topo.blocks * sizeof(uint32_t);
}

// Function attributes the launches and occupancy queries rely on; called
// once per device before either.
cudaError_t leo_wavefront_configure() {
    cudaError_t e = cudaFuncSetAttribute(leo_wavefront_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(leo_wavefront_grid_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(leo_wavefront_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
}

cudaError_t leo_launch_wavefront(const LaneState* lanes, int lane_count, uint32_t cluster, uint32_t begin,
                                 uint32_t end, const KernelConsts& kc, cudaStream_t stream) {
    size_t smem = leo_wavefront_smem_bytes(kc);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)lane_count * cluster, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, leo_wavefront_kernel, lanes, begin, end, kc);
}

cudaError_t leo_launch_wavefront_grid(const LaneState* lane, uint32_t ctas, uint32_t begin, uint32_t end,
                                      const KernelConsts& kc, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = leo_wavefront_smem_bytes(kc);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, leo_wavefront_grid_kernel, lane, begin, end, kc);
}

cudaError_t leo_wavefront_grid_ctas(const KernelConsts& kc, int sms, int* out) {
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, leo_wavefront_grid_kernel, kThreads,
                                                                  leo_wavefront_smem_bytes(kc));
    *out = per_sm >= 1 ? sms : 0;
    return e;
}

cudaError_t leo_wavefront_max_clusters(uint32_t cluster, const KernelConsts& kc, int* out) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cluster, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = leo_wavefront_smem_bytes(kc);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaOccupancyMaxActiveClusters(out, leo_wavefront_kernel, &cfg);
}
