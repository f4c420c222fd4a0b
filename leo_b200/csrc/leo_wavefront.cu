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
#include <stdint.h>

#include "leo_device.cuh"
#include "leo_kernels.h"
#include "leo_math.cuh"

namespace cg = cooperative_groups;

// Hub event keys sorted in shared memory when their padded count fits (128 KB of 4-byte keys).
constexpr uint32_t kHubSortShared = 32768;
// Largest event count a hub's thread-level sort handles (kc.topo.hub_thread_events <= this).
constexpr uint32_t kHubThreadEvents = 16;
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

__device__ __forceinline__ void touch(const LaneState& ln, uint32_t n, uint32_t epoch) {
    // A plain read skips the atomic for targets already touched this step
    // (hub targets receive thousands of events per step).
    if (*(volatile uint32_t*)&ln.touch_epoch[n] == epoch) return;
    if (atomicExch(&ln.touch_epoch[n], epoch) != epoch) append_coalesced(ln.touched, &ln.sc->touched_count, n);
}

__device__ __forceinline__ void push_event(const LaneState& ln, uint32_t tb, uint32_t q, float value) {
    uint32_t old = atomicExch(&ln.ev_head[tb], q);
    ln.ev_next[q] = old;
    ln.ev_val[q] = value;
}

// A hub target's event: its value is stored by event order (as for listed
// events) and its key (branch << 30 | event order) appended to the hub's
// segment, one atomic per group of converged threads with the same hub; the
// order is restored by sorting the keys in settle.  Capacity is an upper
// bound computed from the topology.
constexpr uint32_t kEventOrderMask = 0x3fffffffu;
__device__ __forceinline__ void hub_push(const LaneState& ln, const KernelConsts& kc, int32_t h, uint32_t key,
                                         float value) {
    cg::coalesced_group g = cg::coalesced_threads();
    cg::coalesced_group peers = cg::labeled_partition(g, h);
    uint32_t base = 0;
    if (peers.thread_rank() == 0) base = atomicAdd(&ln.hub_count[h], peers.size());
    base = peers.shfl(base, 0);
    const uint32_t pos = base + peers.thread_rank();
    ln.ev_val[key & kEventOrderMask] = value;
    if (pos < kc.topo.hub_capacity[h])
        ln.hub_events[kc.topo.hub_offset[h] + pos] = key;
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
// deliver (runtime.rs:537-639).  Work item order within a lane is the CPU's
// event order: previous actives, then due events from emission ticks s-8,
// s-4, s-2, s-1 (rank, then slot), then the symbol's input slots; the event
// index q encodes that order.
//
// `fresh_d1`: the previous step was frozen and its emit phase runs beside this
// deliver, so its ring values are not written yet; a delay-1 event's value is
// formed here from the same operands (activation x weight; no learning step
// separates emission and delivery, so the weight is the one emit reads).
__device__ uint32_t phase_deliver(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t worker,
                                  uint32_t workers, bool learn, uint32_t symbol, bool fresh_d1) {
    const uint32_t S = kc.topo.s, F = kc.topo.f, maxa = kc.topo.max_active;
    LaneScalars* sc = ln.sc;
    uint32_t prev = s >= 1 ? sc->ring_count[(s - 1) % LEO_RING] : 0u;
    uint32_t a8 = s >= 8 ? sc->ring_count[(s - 8) % LEO_RING] : 0u;
    uint32_t a4 = s >= 4 ? sc->ring_count[(s - 4) % LEO_RING] : 0u;
    uint32_t a2 = s >= 2 ? sc->ring_count[(s - 2) % LEO_RING] : 0u;
    uint32_t e8 = a8 * S, e4 = a4 * S, e2 = a2 * S, e1 = prev * S;
    uint32_t events = e8 + e4 + e2 + e1;
    uint32_t total = prev + events + F;
    const uint32_t cur = sc->elig_cur;
    if (worker == 0) {
        sc->elig_count[cur ^ 1u] = 0;
        sc->in_elig_count[cur ^ 1u] = 0;
    }
    const uint32_t epoch = s + 1;
    for (uint32_t i = worker; i < total; i += workers) {
        if (i < prev) {
            touch(ln, ln.ring_src[((s - 1) % LEO_RING) * maxa + i], epoch);
            continue;
        }
        uint32_t q = i - prev;
        if (q < events) {
            uint32_t d, off;
            if (q < e8) {
                d = 8; off = q;
            } else if (q < e8 + e4) {
                d = 4; off = q - e8;
            } else if (q < e8 + e4 + e2) {
                d = 2; off = q - e8 - e4;
            } else {
                d = 1; off = q - e8 - e4 - e2;
            }
            uint32_t entry = (s - d) % LEO_RING;
            uint32_t r = off / S, j = off - r * S;
            uint32_t src = ln.ring_src[entry * maxa + r];
            uint32_t slot = src * S + j;
            uint32_t word = kc.topo.rec_word[slot];
            if (LEO_WORD_DELAY(word) != d) continue;
            uint32_t n = word & LEO_TARGET_MASK, b = LEO_WORD_BRANCH(word);
            const float value = (fresh_d1 && d == 1) ? ln.ring_act[entry * maxa + r] * ln.p.rec_weight[slot]
                                                     : ln.ring_val[((size_t)entry * maxa + r) * S + j];
            touch(ln, n, epoch);
            const int32_t h = kc.topo.hubs ? kc.topo.hub_of[n] : -1;
            if (h >= 0)
                hub_push(ln, kc, h, (b << 30) | q, value);
            else
                push_event(ln, n * 4 + b, q, value);
            if (learn) {  // activate_recurrent_trace (runtime.rs:719-726); one event per slot per tick
                float a = ln.ring_act[entry * maxa + r];
                Trace t = load_trace(&ln.traces[slot]);
                advance_trace(kc.cfg, t, s);
                t.branch_sens = t.branch_sens + a;
                if ((t.tick_mark & 1u) == 0u) {
                    t.tick_mark |= 1u;
                    cg::coalesced_group g = cg::coalesced_threads();
                    uint32_t base = 0;
                    if (g.thread_rank() == 0) base = atomicAdd(&sc->elig_count[cur], g.size());
                    base = g.shfl(base, 0);
                    ln.elig[cur][base + g.thread_rank()] = make_uint2(slot, 0u);
                }
                store_trace(&ln.traces[slot], t);
            }
        } else {
            uint32_t f = q - events;
            uint32_t slot = symbol * F + f;
            uint32_t word = kc.topo.in_word[slot];
            uint32_t n = word & LEO_TARGET_MASK, b = LEO_WORD_BRANCH(word);
            touch(ln, n, epoch);
            const int32_t h = kc.topo.hubs ? kc.topo.hub_of[n] : -1;
            if (h >= 0)
                hub_push(ln, kc, h, (b << 30) | q, ln.p.in_weight[slot]);
            else
                push_event(ln, n * 4 + b, q, ln.p.in_weight[slot]);
            if (learn) {
                Trace t = load_trace(&ln.in_traces[slot]);
                advance_trace(kc.cfg, t, s);
                t.branch_sens = t.branch_sens + 1.0f;
                if ((t.tick_mark & 1u) == 0u) {
                    t.tick_mark |= 1u;
                    cg::coalesced_group g = cg::coalesced_threads();
                    uint32_t base = 0;
                    if (g.thread_rank() == 0) base = atomicAdd(&sc->in_elig_count[cur], g.size());
                    base = g.shfl(base, 0);
                    ln.in_elig[cur][base + g.thread_rank()] = make_uint2(slot, 0u);
                }
                store_trace(&ln.in_traces[slot], t);
            }
        }
    }
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

// Hubs by event count this step: more than hub_cta_events -> one CTA per hub
// (hubs h = rank, rank + C, ...); more than hub_thread_events -> one warp per
// hub; the rest are settled by one thread in phase_settle.  A tier sorts the
// hub's keys (branch << 30 | event order), replaces each key by its event's
// value in place, and sums each branch's values in ascending event order.
__device__ void settle_hubs(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t rank, uint32_t C,
                            uint32_t* smem, float pop_inh, uint32_t rotation) {
    __shared__ float s_acc[4];
    __shared__ uint32_t s_bound[5];
    __shared__ NeuronCold s_cold;
    const uint32_t H = kc.topo.hubs, tid = threadIdx.x;
    for (uint32_t h = rank; h < H; h += C) {
        const uint32_t k = ln.hub_count[h];
        if (k <= kc.topo.hub_cta_events) continue;  // none, or few: a warp or a thread settles it
        const uint32_t n = kc.topo.hub_neuron[h];
        const uint32_t* ev = ln.hub_events + kc.topo.hub_offset[h];
        uint32_t P = 1;
        while (P < k) P <<= 1;
        uint32_t* keys = P <= kHubSortShared ? smem : ln.hub_sort;
        load_keys(keys, ev, k, P, tid, kThreads);
        if (tid == 0) {
            NeuronCold cold = ln.cold[n];
            float4 br = ln.branches[n];
            settle_decay(kc.cfg, s, cold, br);
            s_cold = cold;
            s_acc[0] = br.x;
            s_acc[1] = br.y;
            s_acc[2] = br.z;
            s_acc[3] = br.w;
        }
        __syncthreads();
        bitonic_sort_keys(keys, P, tid, kThreads, BlockSync{});
        if (tid <= 4) s_bound[tid] = tid == 4 ? k : hub_branch_begin(keys, k, tid);
        __syncthreads();
        gather_values(keys, ln.ev_val, k, tid, kThreads);
        __syncthreads();
        const float* vals = reinterpret_cast<const float*>(keys);
        if (tid < 4) s_acc[tid] = ordered_sum(vals, s_bound[tid], s_bound[tid + 1], s_acc[tid]);
        __syncthreads();
        if (tid == 0) settle_integrate(ln, kc, n, s, s_cold, make_float4(s_acc[0], s_acc[1], s_acc[2], s_acc[3]),
                                       pop_inh, rotation, settle_preload(ln, kc, n));
        __syncthreads();
    }
    // Medium hubs: one warp each, sorted in the warp's slice of shared memory.
    // Warps take hubs one at a time from a shared counter, largest capacity
    // first, and stop at the first hub whose capacity fits the thread tier.
    const uint32_t lane = tid & 31u, warp = tid >> 5;
    uint32_t* wkeys = smem + (size_t)warp * kHubWarpEvents;
    for (;;) {
        uint32_t h = 0;
        if (lane == 0) h = atomicAdd(&ln.sc->hub_next, 1u);
        h = __shfl_sync(0xffffffffu, h, 0);
        if (h >= H || kc.topo.hub_capacity[h] <= kc.topo.hub_thread_events) break;
        const uint32_t k = ln.hub_count[h];
        if (k <= kc.topo.hub_thread_events || k > kc.topo.hub_cta_events) continue;
        const uint32_t n = kc.topo.hub_neuron[h];
        const uint32_t* ev = ln.hub_events + kc.topo.hub_offset[h];
        uint32_t P = 32;
        while (P < k) P <<= 1;
        load_keys(wkeys, ev, k, P, lane, 32u);
        __syncwarp();
        bitonic_sort_keys(wkeys, P, lane, 32u, WarpSync{});
        const uint32_t bound = lane <= 4 ? (lane == 4 ? k : hub_branch_begin(wkeys, k, lane)) : 0u;
        __syncwarp();
        gather_values(wkeys, ln.ev_val, k, lane, 32u);
        const float* wvals = reinterpret_cast<const float*>(wkeys);
        NeuronCold cold;
        float4 br = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (lane == 0) {
            cold = ln.cold[n];
            br = ln.branches[n];
            settle_decay(kc.cfg, s, cold, br);
        }
        br.x = __shfl_sync(0xffffffffu, br.x, 0);
        br.y = __shfl_sync(0xffffffffu, br.y, 0);
        br.z = __shfl_sync(0xffffffffu, br.z, 0);
        br.w = __shfl_sync(0xffffffffu, br.w, 0);
        const uint32_t next_bound = __shfl_down_sync(0xffffffffu, bound, 1);
        __syncwarp();
        float a = 0.0f;
        if (lane < 4) a = ordered_sum(wvals, bound, next_bound, lane == 0 ? br.x : (lane == 1 ? br.y : (lane == 2 ? br.z : br.w)));
        const float a1 = __shfl_sync(0xffffffffu, a, 1), a2 = __shfl_sync(0xffffffffu, a, 2),
                    a3 = __shfl_sync(0xffffffffu, a, 3);
        if (lane == 0)
            settle_integrate(ln, kc, n, s, cold, make_float4(a, a1, a2, a3), pop_inh, rotation, settle_preload(ln, kc, n));
        __syncwarp();
    }
}

__device__ void phase_settle(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t worker,
                             uint32_t workers, uint32_t rank, uint32_t C, uint32_t* smem) {
    const LeoConfig& c = kc.cfg;
    const uint32_t n_count = kc.topo.n;
    constexpr int kCap = 24;
    LaneScalars* sc = ln.sc;
    uint32_t count = sc->touched_count;
    float pop_inh = sc->population_inhibition;
    uint32_t rotation = (uint32_t)((sc->base_tick + s) % (unsigned long long)n_count);
    if (kc.topo.hubs) {
        const unsigned long long t0 = clock64();
        settle_hubs(ln, s, kc, rank, C, smem, pop_inh, rotation);
        // Hub share of settle (first CTA), reported as the last phase counter.
        if (rank == 0 && threadIdx.x == 0) sc->phase_cycles[LEO_PHASES - 1] += clock64() - t0;
    }
    for (uint32_t i = worker; i < count; i += workers) {
        uint32_t n = ln.touched[i];
        NeuronCold cold;
        float4 br;
        if (kc.topo.hubs) {
            const int32_t h = kc.topo.hub_of[n];
            const uint32_t k = h >= 0 ? ln.hub_count[h] : 0u;
            if (k > kc.topo.hub_thread_events) continue;  // settled by a warp or a CTA above
            if (k > 0) {
                // A hub with few events: sort its keys (branch, event order) here.
                const uint32_t* ev = ln.hub_events + kc.topo.hub_offset[h];
                uint32_t e[kHubThreadEvents];
                for (uint32_t x = 0; x < k; ++x) e[x] = ev[x];
                for (uint32_t x = 1; x < k; ++x) {
                    const uint32_t v = e[x];
                    int y = (int)x - 1;
                    while (y >= 0 && e[y] > v) {
                        e[y + 1] = e[y];
                        --y;
                    }
                    e[y + 1] = v;
                }
                float vals[kHubThreadEvents];
                for (uint32_t x = 0; x < k; ++x) vals[x] = ln.ev_val[e[x] & kEventOrderMask];
                cold = ln.cold[n];
                br = ln.branches[n];
                settle_decay(c, s, cold, br);
                float acc[4] = {br.x, br.y, br.z, br.w};
                for (uint32_t x = 0; x < k; ++x) acc[e[x] >> 30] = acc[e[x] >> 30] + vals[x];
                settle_integrate(ln, kc, n, s, cold, make_float4(acc[0], acc[1], acc[2], acc[3]), pop_inh, rotation,
                                 settle_preload(ln, kc, n));
                continue;
            }
        }
        cold = ln.cold[n];
        br = ln.branches[n];
        const SettlePre pre = settle_preload(ln, kc, n);
        settle_decay(c, s, cold, br);
        float acc[4] = {br.x, br.y, br.z, br.w};
        // The four (target, branch) event lists, walked in lockstep so their
        // hops overlap; events are summed per branch in ascending event order.
        const uint4 heads = *reinterpret_cast<const uint4*>(&ln.ev_head[n * 4]);
        if ((heads.x & heads.y & heads.z & heads.w) != LEO_EMPTY)
            *reinterpret_cast<uint4*>(&ln.ev_head[n * 4]) = make_uint4(LEO_EMPTY, LEO_EMPTY, LEO_EMPTY, LEO_EMPTY);
        uint32_t p[4] = {heads.x, heads.y, heads.z, heads.w};
        uint32_t keys[kCap];
        float vals[kCap];
        int k = 0;
        bool overflow = false;
        while ((p[0] & p[1] & p[2] & p[3]) != LEO_EMPTY) {
            uint32_t nxt[4];
            float v[4];
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                nxt[b] = LEO_EMPTY;
                if (p[b] != LEO_EMPTY) {
                    nxt[b] = ln.ev_next[p[b]];
                    v[b] = ln.ev_val[p[b]];
                }
            }
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                if (p[b] == LEO_EMPTY) continue;
                if (k == kCap) {
                    overflow = true;
                    break;
                }
                keys[k] = ((uint32_t)b << 24) | p[b];
                vals[k] = v[b];
                ++k;
            }
            if (overflow) break;
#pragma unroll
            for (int b = 0; b < 4; ++b) p[b] = nxt[b];
        }
        if (!overflow) {
            for (int x = 1; x < k; ++x) {  // insertion sort by (branch, event order)
                uint32_t kk = keys[x];
                float vk = vals[x];
                int y = x - 1;
                while (y >= 0 && keys[y] > kk) {
                    keys[y + 1] = keys[y];
                    vals[y + 1] = vals[y];
                    --y;
                }
                keys[y + 1] = kk;
                vals[y + 1] = vk;
            }
            for (int x = 0; x < k; ++x) acc[keys[x] >> 24] = acc[keys[x] >> 24] + vals[x];
        } else {
            // A long list (hot target): per branch, add in ascending event
            // order by repeated scans of the list.
            const uint32_t head4[4] = {heads.x, heads.y, heads.z, heads.w};
            for (int b = 0; b < 4; ++b) {
                const uint32_t head = head4[b];
                float a = acc[b];
                uint32_t last = 0u;
                bool first = true;
                for (;;) {
                    uint32_t best = LEO_EMPTY;
                    float bv = 0.0f;
                    for (uint32_t it = head; it != LEO_EMPTY; it = ln.ev_next[it]) {
                        if ((first || it > last) && (best == LEO_EMPTY || it < best)) {
                            best = it;
                            bv = ln.ev_val[it];
                        }
                    }
                    if (best == LEO_EMPTY) break;
                    a = a + bv;
                    last = best;
                    first = false;
                }
                acc[b] = a;
            }
        }
        br = make_float4(acc[0], acc[1], acc[2], acc[3]);
        settle_integrate(ln, kc, n, s, cold, br, pop_inh, rotation, pre);
    }
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
        constexpr uint32_t kLocal = 8;
        unsigned long long mine[kLocal];
        uint32_t held = 0;
        for (uint32_t idx = lane; idx < count && held < kLocal; idx += 32) mine[held++] = cand[idx];
        bool spill = count > 32 * kLocal;
        unsigned long long prev = ~0ull;
        uint32_t rounds = count < keep + 1 ? count : keep + 1;
        float cutoff = 0.0f;
        for (uint32_t k = 0; k < rounds; ++k) {
            unsigned long long best = 0ull;
            for (uint32_t h = 0; h < held; ++h)
                if (mine[h] < prev && mine[h] > best) best = mine[h];
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
// the wavefront, shared memory in the quiet-step kernel); `active_out`, when
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
    for (uint32_t i = worker; i < total; i += workers) {
        uint32_t r = i / S, j = i - r * S;
        uint32_t src = ln.ring_src[entry * maxa + r];
        if (kc.topo.neuron_type[src] == 0) continue;
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
}

// Work counters of one launch, held by the launch's first thread and added to
// the lane's scalars when the launch ends.
struct WorkTally {
    unsigned long long deliver, touched, active, steps, eligible, destinations;
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
    if (begin == LEO_RESUME_STEP) begin = sc->resume_step;
    const uint32_t worker = rank * kThreads + threadIdx.x, workers = C * kThreads;
    const uint32_t gwarp = rank * kWarps + (threadIdx.x >> 5), gwarps = C * kWarps;
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
        tally = WorkTally{0, 0, 0, 0, 0, 0};
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
        for (uint32_t h = worker; h < kc.topo.hubs; h += workers) ln.hub_count[h] = 0;
        if (worker == 0) sc->hub_next = 0;
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

// ---------------------------------------------------------------------------
// Quiet frozen steps on one CTA (replay prefixes).
//
// A replay segment starts from a fresh transient state and runs a frozen
// prefix (no target, no learning) before its training steps, and most prefix
// steps touch a few hundred neurons.  This kernel runs such steps on one CTA
// with the step's transient lists in shared memory -- touched neurons in a
// hash table, the step's events grouped by target with a counting sort, block
// candidates grouped by block, block winners, the active list and the ring
// counts -- so a step's critical path is four global round trips (deliver's
// sources and values, their synapse words, the touched neurons' state, the
// emitters' state) and CTA barriers, where the wavefront pays cluster
// barriers around lists in global memory.  Each thread issues its deliver
// items' loads in batches so one round trip covers several items.  Arithmetic
// and order are the wavefront's: each branch sums its events in ascending
// event order, then the same integration, block top-k (same rounds), global
// cap (phase_assemble is shared) and emission.  Persistent state (neurons,
// rings, scalars) is the wavefront's, so the wavefront resumes where this
// kernel stops: at the first step that is not frozen without a target, or
// whose touched neurons, events or per-target events exceed the tables --
// checked after the step's deliver, before the step changes persistent state.
namespace {

constexpr uint32_t kQuietSlots = 4096;               // hash slots (power of two)
constexpr uint32_t kQuietTouched = kQuietSlots / 2;  // touched neurons per step
constexpr uint32_t kQuietEvents = 8192;              // events per step
constexpr uint32_t kQuietPerTarget = 64;             // events per touched neuron
constexpr uint32_t kQuietBlocks = 1024;              // blocks (phase_assemble's limit too)
constexpr uint32_t kQuietWinners = kQuietTouched;    // blocks x keep
constexpr uint32_t kQuietThreadCands = 32;           // a block with more candidates is selected by a warp

struct QuietShared {
    uint32_t key[kQuietSlots];              // neuron + 1; 0 = empty
    uint32_t start[kQuietSlots];            // events per slot, then the end of its placed run
    uint16_t touched[kQuietTouched];        // slots in touch order
    uint16_t tcount[kQuietTouched];         // events of touched[t]
    uint32_t tneuron[kQuietTouched];        // neuron of touched[t]
    uint32_t ev_key[kQuietEvents];          // branch << 24 | event order
    float ev_val[kQuietEvents];             // then: candidates grouped by block
    uint16_t ev_slot[kQuietEvents];
    uint16_t placed[kQuietEvents];          // events grouped by slot
    unsigned long long cand[kQuietTouched];  // candidate key of touched[t] (0: none); then: block winners
    uint16_t cand_pos[kQuietTouched];       // its position in its block's run
    uint32_t bcount[kQuietBlocks];
    uint32_t boff[kQuietBlocks];            // then: winners per block
    uint32_t wsum[kWarps];
    uint32_t ring[LEO_RING];                // ring_count mirror
    uint32_t hist[LEO_MAX_CONTEXT_ORDER];   // context history mirror (runtime.rs:642-646)
    uint32_t nev, ntouched, overflow, supra, active, hist_len;
};

__device__ __forceinline__ int quiet_insert(QuietShared& q, uint32_t n) {
    const uint32_t want = n + 1u;
    uint32_t h = (n * 0x9E3779B1u) >> 20;  // 12 bits: kQuietSlots == 4096
    for (uint32_t i = 0; i < kQuietSlots; ++i, h = (h + 1u) & (kQuietSlots - 1u)) {
        const uint32_t k = *(volatile uint32_t*)&q.key[h];
        if (k == want) return (int)h;
        if (k != 0u) continue;
        const uint32_t old = atomicCAS(&q.key[h], 0u, want);
        if (old == 0u) {
            // one counter update per group of converged threads
            cg::coalesced_group g = cg::coalesced_threads();
            uint32_t base = 0;
            if (g.thread_rank() == 0) base = atomicAdd(&q.ntouched, g.size());
            const uint32_t t = g.shfl(base, 0) + g.thread_rank();
            if (t < kQuietTouched) q.touched[t] = (uint16_t)h;
            else q.overflow = 1u;
            return (int)h;
        }
        if (old == want) return (int)h;
    }
    q.overflow = 1u;
    return -1;
}

__device__ __forceinline__ void quiet_event(QuietShared& q, uint32_t n, uint32_t b, uint32_t qi, float value) {
    const int h = quiet_insert(q, n);
    if (h < 0) return;
    cg::coalesced_group g = cg::coalesced_threads();
    uint32_t base = 0;
    if (g.thread_rank() == 0) base = atomicAdd(&q.nev, g.size());
    const uint32_t e = g.shfl(base, 0) + g.thread_rank();
    if (e >= kQuietEvents) {
        q.overflow = 1u;
        return;
    }
    q.ev_key[e] = (b << 24) | qi;
    q.ev_val[e] = value;
    q.ev_slot[e] = (uint16_t)h;
    if (atomicAdd(&q.start[h], 1u) >= kQuietPerTarget) q.overflow = 1u;
}

// Exclusive scan of one value per thread across the CTA; returns this
// thread's offset and leaves the total in *total (every thread).
__device__ __forceinline__ uint32_t quiet_scan(QuietShared& q, uint32_t v, uint32_t* total) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    uint32_t incl = v;
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= (uint32_t)o) incl += y;
    }
    if (lane == 31) q.wsum[warp] = incl;
    __syncthreads();
    uint32_t before = 0, all = 0;
    for (uint32_t w = 0; w < kWarps; ++w) {
        const uint32_t x = q.wsum[w];
        if (w < warp) before += x;
        all += x;
    }
    __syncthreads();
    *total = all;
    return before + incl - v;
}

// Deliver of step s into the shared tables (no global writes); the previous
// step's active list is `prev_list` (its assemble keys, rank order) when
// given, else the ring.  The delayed events are enumerated as (delay group in
// the order 8, 4, 2, 1; source rank r; synapse j), a warp per (group, source)
// and the warp's lanes over j, so each step's loads are coalesced and issued
// kQuietPairs sources at a time; an event's order is its item index in the
// wavefront's numbering (group offset + r * S + j).  Returns the step's deliver
// work items.
constexpr uint32_t kQuietPairs = 4;

__device__ uint32_t quiet_deliver(const LaneState& ln, uint32_t s, const KernelConsts& kc, uint32_t symbol,
                                  QuietShared& q, const unsigned long long* prev_list, uint32_t prev_rotation) {
    const uint32_t S = kc.topo.s, F = kc.topo.f, maxa = kc.topo.max_active, n_count = kc.topo.n;
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t prev = s >= 1 ? q.ring[(s - 1) % LEO_RING] : 0u;
    const uint32_t a8 = s >= 8 ? q.ring[(s - 8) % LEO_RING] : 0u;
    const uint32_t a4 = s >= 4 ? q.ring[(s - 4) % LEO_RING] : 0u;
    const uint32_t a2 = s >= 2 ? q.ring[(s - 2) % LEO_RING] : 0u;
    const uint32_t e8 = a8 * S, e4 = a4 * S, e2 = a2 * S, e1 = prev * S;
    const uint32_t events = e8 + e4 + e2 + e1;
    if (events + F >= (1u << 24)) {  // event order must fit the 24-bit key field
        if (threadIdx.x == 0) q.overflow = 1u;
        return 0u;
    }
    // the previous step's actives are touched (runtime.rs:537-548)
    for (uint32_t i = threadIdx.x; i < prev; i += kThreads)
        quiet_insert(q, prev_list ? key_neuron(prev_list[i], prev_rotation, n_count)
                                  : ln.ring_src[((s - 1) % LEO_RING) * maxa + i]);
    // the symbol's input slots (runtime.rs:620-639)
    for (uint32_t f = threadIdx.x; f < F; f += kThreads) {
        const uint32_t slot = symbol * F + f;
        const uint32_t word = kc.topo.in_word[slot];
        const float value = ln.p.in_weight[slot];
        quiet_event(q, word & LEO_TARGET_MASK, LEO_WORD_BRANCH(word), events + f, value);
    }
    // delayed events (runtime.rs:549-618)
    const uint32_t pairs = a8 + a4 + a2 + prev;
    for (uint32_t p0 = warp * kQuietPairs; p0 < pairs; p0 += kWarps * kQuietPairs) {
        // lane k < kQuietPairs resolves pair p0 + k: its group, ring entry and source
        uint32_t my_src = 0, my_info = 0xffffffffu;  // info: d << 28 | entry << 24 | r (r < 2^24)
        if (lane < kQuietPairs && p0 + lane < pairs) {
            uint32_t pr = p0 + lane, d;
            if (pr < a8) {
                d = 8;
            } else if (pr < a8 + a4) {
                d = 4; pr -= a8;
            } else if (pr < a8 + a4 + a2) {
                d = 2; pr -= a8 + a4;
            } else {
                d = 1; pr -= a8 + a4 + a2;
            }
            const uint32_t entry = (s - d) % LEO_RING;
            my_src = (d == 1 && prev_list) ? key_neuron(prev_list[pr], prev_rotation, n_count)
                                           : ln.ring_src[entry * maxa + pr];
            my_info = (d << 28) | (entry << 24) | pr;
        }
        for (uint32_t j0 = 0; j0 < S; j0 += 64) {
            uint32_t word[kQuietPairs][2];
            float val[kQuietPairs][2];
#pragma unroll
            for (uint32_t k = 0; k < kQuietPairs; ++k) {
                const uint32_t info = __shfl_sync(0xffffffffu, my_info, k);
                const uint32_t src = __shfl_sync(0xffffffffu, my_src, k);
#pragma unroll
                for (uint32_t h = 0; h < 2; ++h) {
                    const uint32_t j = j0 + h * 32 + lane;
                    word[k][h] = 0u;
                    if (info != 0xffffffffu && j < S) {
                        const uint32_t entry = (info >> 24) & 15u, r = info & 0xffffffu;
                        word[k][h] = kc.topo.rec_word[src * S + j];
                        val[k][h] = ln.ring_val[((size_t)entry * maxa + r) * S + j];
                    }
                }
            }
#pragma unroll
            for (uint32_t k = 0; k < kQuietPairs; ++k) {
                const uint32_t info = __shfl_sync(0xffffffffu, my_info, k);
#pragma unroll
                for (uint32_t h = 0; h < 2; ++h) {
                    const uint32_t j = j0 + h * 32 + lane;
                    if (info == 0xffffffffu || j >= S) continue;
                    const uint32_t d = info >> 28, r = info & 0xffffffu;
                    if (LEO_WORD_DELAY(word[k][h]) != d) continue;
                    const uint32_t off = d == 8 ? 0u : (d == 4 ? e8 : (d == 2 ? e8 + e4 : e8 + e4 + e2));
                    quiet_event(q, word[k][h] & LEO_TARGET_MASK, LEO_WORD_BRANCH(word[k][h]), off + r * S + j,
                                val[k][h]);
                }
            }
        }
    }
    return events + F;
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    leo_quiet_kernel(const LaneState* __restrict__ lanes, uint32_t begin, uint32_t end, KernelConsts kc) {
    extern __shared__ __align__(16) unsigned char quiet_smem[];
    QuietShared& q = *reinterpret_cast<QuietShared*>(quiet_smem);
    unsigned long long* sorted = reinterpret_cast<unsigned long long*>(quiet_smem + sizeof(QuietShared));
    const LaneState& ln = lanes[0];
    LaneScalars* sc = ln.sc;
    const LeoConfig& c = kc.cfg;
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t B = kc.topo.blocks, S = kc.topo.s, npb = kc.topo.npb, keep = kc.topo.keep, n_count = kc.topo.n;
    const uint32_t steps = sc->steps;
    const unsigned long long base_tick = sc->base_tick;
    for (uint32_t i = tid; i < kQuietSlots; i += kThreads) {
        q.key[i] = 0u;
        q.start[i] = 0u;
    }
    for (uint32_t i = tid; i < kQuietBlocks; i += kThreads) q.bcount[i] = 0u;
    if (tid < LEO_RING) q.ring[tid] = sc->ring_count[tid];
    if (tid < LEO_MAX_CONTEXT_ORDER) q.hist[tid] = sc->ctx_history[tid];
    __shared__ unsigned long long acc[LEO_QUIET_PHASES];
    __shared__ WorkTally tally;
    if (tid == 0) {
        q.nev = q.ntouched = q.overflow = q.supra = q.active = 0u;
        q.hist_len = sc->ctx_history_len;
        for (int p = 0; p < LEO_QUIET_PHASES; ++p) acc[p] = 0ull;
        tally = WorkTally{0, 0, 0, 0, 0, 0};
        const uint32_t cur = sc->elig_cur;
        sc->elig_count[cur ^ 1u] = 0;
        sc->in_elig_count[cur ^ 1u] = 0;
    }
    unsigned long long t0 = tid == 0 ? clock_now() : 0ull;
    auto mark = [&](int p) {
        if (tid == 0) {
            const unsigned long long t = clock_now();
            acc[p] += t - t0;
            t0 = t;
        }
    };
    __syncthreads();
    unsigned long long* winners = q.cand;  // after the candidates are grouped
    uint32_t* nwin = q.boff;               // after each block's run is read
    bool have_prev = false;                // `sorted` holds the previous step's active list
    uint32_t s = begin;
    for (; s < end && s < steps; ++s) {
        const uint32_t sched = ln.schedule[s];
        if (LEO_SCHED_PERMISSION(sched) != kFrozen || LEO_SCHED_TARGET(sched) >= 0) break;
        const uint32_t symbol = LEO_SCHED_SYMBOL(sched);
        const uint32_t rotation = (uint32_t)((base_tick + s) % (unsigned long long)n_count);
        const uint32_t prev_rotation = (uint32_t)((base_tick + s + n_count - 1) % (unsigned long long)n_count);
        // deliver into the tables; give the step to the wavefront if they overflow
        const uint32_t delivered = quiet_deliver(ln, s, kc, symbol, q, have_prev ? sorted : nullptr, prev_rotation);
        __syncthreads();
        if (q.overflow) break;
        mark(0);  // deliver
        // group the events by touched neuron: offsets of the per-slot counts
        const uint32_t T = q.ntouched, E = q.nev;
        const float pop_inh = sc->population_inhibition;  // latency overlaps the scan
        uint32_t mine[4], sum = 0;
        const uint32_t t_lo = tid * 4u;
        for (uint32_t k = 0; k < 4; ++k) {
            const uint32_t t = t_lo + k;
            mine[k] = t < T ? q.start[q.touched[t]] : 0u;
            sum += mine[k];
        }
        uint32_t grand = 0;
        uint32_t off = quiet_scan(q, sum, &grand);
        for (uint32_t k = 0; k < 4; ++k) {
            const uint32_t t = t_lo + k;
            if (t < T) {
                q.tcount[t] = (uint16_t)mine[k];
                q.start[q.touched[t]] = off;
            }
            off += mine[k];
        }
        __syncthreads();
        for (uint32_t e = tid; e < E; e += kThreads) q.placed[atomicAdd(&q.start[q.ev_slot[e]], 1u)] = (uint16_t)e;
        __syncthreads();
        mark(1);  // events grouped by target
        // settle (runtime.rs:576-603, 710-717, 947-962)
        for (uint32_t t = tid; t < T; t += kThreads) {
            const uint32_t h = q.touched[t];
            const uint32_t n = q.key[h] - 1u;
            const uint32_t cnt = q.tcount[t], hi = q.start[h], lo = hi - cnt;
            NeuronCold cold = ln.cold[n];
            float4 br = ln.branches[n];
            const SettlePre pre = settle_preload(ln, kc, n);
            for (uint32_t x = lo + 1; x < hi; ++x) {  // insertion sort by (branch, event order)
                const uint16_t e = q.placed[x];
                const uint32_t k = q.ev_key[e];
                uint32_t y = x;
                while (y > lo && q.ev_key[q.placed[y - 1]] > k) {
                    q.placed[y] = q.placed[y - 1];
                    --y;
                }
                q.placed[y] = e;
            }
            settle_decay(c, s, cold, br);
            float a[4] = {br.x, br.y, br.z, br.w};
            for (uint32_t x = lo; x < hi; ++x) {
                const uint16_t e = q.placed[x];
                const uint32_t b = q.ev_key[e] >> 24;
                a[b] = a[b] + q.ev_val[e];
            }
            const unsigned long long key = settle_integrate_key(ln, kc, n, s, cold, make_float4(a[0], a[1], a[2], a[3]),
                                                                pop_inh, rotation, pre);
            q.tneuron[t] = n;
            q.cand[t] = key;
            if (key) q.cand_pos[t] = (uint16_t)atomicAdd(&q.bcount[n / npb], 1u);
        }
        __syncthreads();
        mark(2);  // settle
        // candidates grouped by block: exclusive scan of the block counts (B <= 1024, two per thread)
        {
            const uint32_t b0 = 2u * tid, b1 = b0 + 1u;
            const uint32_t v0 = b0 < B ? q.bcount[b0] : 0u, v1 = b1 < B ? q.bcount[b1] : 0u;
            uint32_t all = 0;
            const uint32_t o = quiet_scan(q, v0 + v1, &all);
            if (b0 < B) q.boff[b0] = o;
            if (b1 < B) q.boff[b1] = o + v0;
        }
        __syncthreads();
        unsigned long long* grouped = reinterpret_cast<unsigned long long*>(q.ev_val);  // events are consumed
        for (uint32_t t = tid; t < T; t += kThreads) {
            const unsigned long long key = q.cand[t];
            if (key) grouped[q.boff[q.tneuron[t] / npb] + q.cand_pos[t]] = key;
            q.key[q.touched[t]] = 0u;  // empty the tables for the next step
            q.start[q.touched[t]] = 0u;
        }
        __syncthreads();
        // blocks: block-local top-k and the (k+1)-th cutoff (runtime.rs:964-997):
        // one thread per block with at most kQuietThreadCands candidates, one
        // warp per larger block; both take the largest key below the previous
        // winner keep + 1 times.
        uint32_t supra = 0;
        for (uint32_t b = tid; b < B; b += kThreads) {
            const uint32_t count = q.bcount[b];
            supra += count;
            if (count > kQuietThreadCands) continue;
            const unsigned long long* cand = grouped + q.boff[b];
            unsigned long long prev = ~0ull;
            const uint32_t rounds = count < keep + 1 ? count : keep + 1;
            float cutoff = 0.0f;
            for (uint32_t k = 0; k < rounds; ++k) {
                unsigned long long best = 0ull;
                for (uint32_t idx = 0; idx < count; ++idx) {
                    const unsigned long long key = cand[idx];
                    if (key < prev && key > best) best = key;
                }
                if (k < keep) winners[(size_t)b * keep + k] = best;
                else cutoff = key_value(best);
                prev = best;
            }
            ln.block_cutoff[b] = count > keep ? cutoff : 0.0f;
            nwin[b] = count < keep ? count : keep;  // boff[b] is read above: this thread's own slot
        }
        for (uint32_t b = warp; b < B; b += kWarps) {
            const uint32_t count = q.bcount[b];
            if (count <= kQuietThreadCands) continue;
            const unsigned long long* cand = grouped + q.boff[b];
            unsigned long long prev = ~0ull;
            const uint32_t rounds = count < keep + 1 ? count : keep + 1;
            float cutoff = 0.0f;
            for (uint32_t k = 0; k < rounds; ++k) {
                unsigned long long best = 0ull;
                for (uint32_t idx = lane; idx < count; idx += 32) {
                    const unsigned long long key = cand[idx];
                    if (key < prev && key > best) best = key;
                }
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
                    best = other > best ? other : best;
                }
                if (k < keep) {
                    if (lane == 0) winners[(size_t)b * keep + k] = best;
                } else {
                    cutoff = key_value(best);
                }
                prev = best;
            }
            __syncwarp();
            if (lane == 0) {
                nwin[b] = count < keep ? count : keep;
                ln.block_cutoff[b] = count > keep ? cutoff : 0.0f;
            }
        }
        // one add per warp of the per-thread counts
        for (int o = 16; o > 0; o >>= 1) supra += __shfl_xor_sync(0xffffffffu, supra, o);
        if (lane == 0 && supra) atomicAdd(&q.supra, supra);
        __syncthreads();
        for (uint32_t b = tid; b < B; b += kThreads) q.bcount[b] = 0u;
        if (tid == 0) {
            sc->step_supra = q.supra;
            q.supra = 0u;
        }
        mark(3);  // blocks
        // assemble (shared with the wavefront); the active list stays in `sorted`
        phase_assemble(ln, s, kc, false, sorted, nwin, winners, &q.active);
        __syncthreads();
        mark(4);  // assemble
        // emit (runtime.rs:920-938, 1084-1106) from the active list in shared memory
        const uint32_t active = q.active;
        for (uint32_t i = tid; i < active * S; i += kThreads) {
            const uint32_t r = i / S, j = i - r * S;
            const unsigned long long k = sorted[r];
            const uint32_t n = key_neuron(k, rotation, n_count);
            const float a = key_value(k);
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
            ln.ring_val[((size_t)(s % LEO_RING) * kc.topo.max_active + r) * S + j] = a * ln.p.rec_weight[(size_t)n * S + j];
        }
        if (tid == 0) {
            // context history push: a frozen step without a target resolves
            // nothing else (runtime.rs:641-646; context_resolve_warp)
            uint32_t len = q.hist_len;
            if (len == kc.topo.k) {
                for (uint32_t i = 0; i + 1 < len; ++i) q.hist[i] = q.hist[i + 1];
                len -= 1;
            }
            q.hist[len] = symbol;
            q.hist_len = len + 1;
            q.ring[s % LEO_RING] = active;
            sc->step_flags = 0;
            sc->dst_count = 0;
            tally.deliver += delivered;
            tally.touched += T;
            tally.active += active;
            tally.steps += 1;
            q.nev = 0u;
            q.ntouched = 0u;
        }
        have_prev = true;
        __syncthreads();
        mark(5);  // emit
    }
    if (tid == 0) {
        if (s > begin) {  // the context state a frozen step without a target leaves
            for (uint32_t i = 0; i < q.hist_len; ++i) sc->ctx_history[i] = q.hist[i];
            sc->ctx_history_len = q.hist_len;
            sc->ctx_applied = 0u;
            sc->ctx_count = 0u;
            sc->ctx_probes = 0u;
        }
        sc->resume_step = s;
        sc->work_quiet += tally.steps;
        flush_tally(ln, tally);
        for (int p = 0; p < LEO_QUIET_PHASES; ++p) sc->quiet_cycles[p] += acc[p];
    }
}

size_t leo_quiet_smem_bytes(const KernelConsts& kc) {
    if (kc.topo.blocks > kQuietBlocks || kc.topo.blocks * kc.topo.keep > kQuietWinners || kc.topo.n >= (1u << 31))
        return 0;
    uint32_t winners = kc.topo.blocks * kc.topo.keep, span = 1;
    while (span < winners) span <<= 1;
    const size_t bytes = sizeof(QuietShared) + (size_t)span * sizeof(unsigned long long);
    return bytes <= 200u * 1024u ? bytes : 0;
}

cudaError_t leo_launch_quiet(const LaneState* lane, uint32_t begin, uint32_t end, const KernelConsts& kc,
                             cudaStream_t stream) {
    const size_t smem = leo_quiet_smem_bytes(kc);
    if (smem == 0) return cudaErrorInvalidConfiguration;
    leo_quiet_kernel<<<1, kThreads, smem, stream>>>(lane, begin, end, kc);
    return cudaGetLastError();
}

__host__ __device__ size_t wavefront_scratch_bytes(const KernelConsts& kc);

// A thread-block cluster per lane (phases separated by cluster barriers).
__global__ void __launch_bounds__(kThreads, 1)
    leo_wavefront_kernel(const LaneState* __restrict__ lanes, uint32_t begin, uint32_t end, KernelConsts kc) {
    extern __shared__ unsigned long long smem_sorted[];
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
    extern __shared__ unsigned long long smem_sorted[];
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
    if (kc.topo.hubs) {
        // the warps' sort slices, or one CTA's sort, whichever is larger
        size_t warps = (size_t)kWarps * kHubWarpEvents * sizeof(uint32_t);
        size_t cta = (size_t)(kc.topo.hub_sort_capacity < kHubSortShared ? kc.topo.hub_sort_capacity : kHubSortShared) *
                     sizeof(uint32_t);
        size_t hub = warps > cta ? warps : cta;
        bytes = bytes > hub ? bytes : hub;
    }
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
    e = cudaFuncSetAttribute(leo_quiet_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
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
