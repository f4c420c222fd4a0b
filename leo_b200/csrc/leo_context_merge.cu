// Batch-end keyed context merge on the device (one GPU, every story a lane).
//
// apply_context_deltas (crates/leo-core/src/parallel.rs:1024-1113), with the
// deltas of context_deltas_for_slots (:929-973), the projection of
// :1226-1233 and the validation of :1317-1334:
//   1. every lane's changed context slots give (order, key) deltas against the
//      canonical table: embedding lane - canonical (0 where the key is not in
//      the canonical table) and observations max(lane - canonical, 0); rows
//      that changed nothing are dropped;
//   2. the deltas are grouped by (order, key) and summed in story order, FP64
//      per dimension, observations as u64;
//   3. the merged keys are applied in (observations descending, order, key)
//      order: each is resolved in the canonical table -- found, or placed in
//      the first empty probe slot, else the weakest (fewest observations,
//      first on ties), which resets that slot -- and its slot gets
//      embedding += (f32)(sum / stories), observations += the sum (saturating);
//   4. every merged key still in the table is clamped to [weight_min,
//      weight_max] and must be finite;
//   5. the canonical rows at every changed slot are copied to every lane.
// Steps 1, 2, 4 and 5 are parallel.  Step 3 is order-sensitive only within one
// context order (each order owns a disjoint slot partition), so it runs as one
// CTA per order, one thread walking that order's keys in the global apply
// order against the partition's keys and observations held in shared memory;
// a slot's final embedding is then written once, from the last key placed in
// it (a later key in the same slot evicted the earlier one, which resets it).
#include <cub/cub.cuh>
#include <stdint.h>

#include "leo_device.cuh"
#include "leo_kernels.h"

namespace {

constexpr uint32_t kThreads = 256;
constexpr uint32_t kApplyThreads = 512;
constexpr uint32_t kNoOwner = 0xffffffffu;

__device__ __forceinline__ void flag_error(uint32_t* error, uint32_t bit) { atomicOr(error, bit); }

// 1. per (lane, changed slot): the delta against the canonical table.
__global__ void __launch_bounds__(kThreads) ctx_delta_kernel(const LaneState* __restrict__ lanes,
                                                             const uint32_t* __restrict__ lane_offset,
                                                             LaneParams canon, CtxMergeArgs a) {
    const uint32_t lane = blockIdx.y;
    const LaneState& ln = lanes[lane];
    const uint32_t first = lane_offset[lane], count = lane_offset[lane + 1] - first;
    const uint32_t spo = a.slots_per_order, d = a.dim;
    for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < count; i += gridDim.x * kThreads) {
        const uint32_t e = first + i;
        const uint32_t slot = ln.ctx_list[i];
        ln.ctx_mark[slot] = 0;
        a.lane_slots[e] = slot;
        const unsigned long long key = ln.p.ctx_keys[slot];
        a.valid[e] = 0;
        if (key == 0ull) continue;
        const uint32_t order = slot / spo + 1u, base = (order - 1u) * spo;
        const uint32_t start = (uint32_t)(key % (unsigned long long)spo);
        int32_t found = -1;
        for (uint32_t off = 0; off < a.probe_limit; ++off) {
            const uint32_t s = base + (start + off) % spo;
            if (canon.ctx_keys[s] == key) {
                found = (int32_t)s;
                break;
            }
        }
        bool changed = false;
        for (uint32_t k = 0; k < d; ++k) {
            const float before = found >= 0 ? canon.ctx_emb[(size_t)found * d + k] : 0.0f;
            const float delta = ln.p.ctx_emb[(size_t)slot * d + k] - before;
            changed |= delta != 0.0f;
            a.delta[(size_t)e * d + k] = delta;
        }
        const uint32_t lobs = ln.p.ctx_obs[slot], cobs = found >= 0 ? canon.ctx_obs[found] : 0u;
        const uint32_t inc = lobs > cobs ? lobs - cobs : 0u;
        a.key[e] = key;
        a.order[e] = order;
        a.obs_inc[e] = inc;
        a.valid[e] = (changed || inc > 0u) ? 1 : 0;
    }
}

__global__ void iota_kernel(uint32_t* out, uint32_t n) {
    for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) out[i] = i;
}

__global__ void gather_u64_kernel(const unsigned long long* __restrict__ src, const uint32_t* __restrict__ idx,
                                  unsigned long long* out, uint32_t n, int complement) {
    for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads)
        out[i] = complement ? ~src[idx[i]] : src[idx[i]];
}

__global__ void gather_u32_kernel(const uint32_t* __restrict__ src, const uint32_t* __restrict__ idx, uint32_t* out,
                                  uint32_t n) {
    for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) out[i] = src[idx[i]];
}

// Group heads of the (order, key)-sorted entries.
__global__ void group_head_kernel(const uint32_t* __restrict__ sorted, const unsigned long long* __restrict__ key,
                                  const uint32_t* __restrict__ order, uint8_t* head, uint32_t n) {
    for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) {
        const uint32_t e = sorted[i];
        head[i] = (i == 0 || key[e] != key[sorted[i - 1]] || order[e] != order[sorted[i - 1]]) ? 1 : 0;
    }
}

// 2. one thread per merged key: story-order FP64 sums of its entries.
__global__ void __launch_bounds__(kThreads) group_sum_kernel(const uint32_t* __restrict__ sorted,
                                                             const uint32_t* __restrict__ gstart, uint32_t groups,
                                                             uint32_t entries, CtxMergeArgs a) {
    const uint32_t d = a.dim;
    for (uint32_t g = blockIdx.x * kThreads + threadIdx.x; g < groups; g += gridDim.x * kThreads) {
        const uint32_t lo = gstart[g], hi = g + 1 < groups ? gstart[g + 1] : entries;
        const uint32_t e0 = sorted[lo];
        unsigned long long obs = 0ull;
        for (uint32_t m = lo; m < hi; ++m) obs += a.obs_inc[sorted[m]];
        for (uint32_t k = 0; k < d; ++k) {
            double sum = 0.0;
            for (uint32_t m = lo; m < hi; ++m) {
                const float v = a.delta[(size_t)sorted[m] * d + k];
                if (!isfinite(v)) flag_error(a.error, LEO_CTX_MERGE_BAD_DELTA);
                sum += (double)v;
            }
            a.msum[(size_t)g * d + k] = sum;
        }
        a.mkey[g] = a.key[e0];
        a.morder[g] = a.order[e0];
        a.mobs[g] = obs;
    }
}

// 3 + 4. one CTA per context order.
__global__ void __launch_bounds__(kApplyThreads) apply_order_kernel(const uint32_t* __restrict__ apply_order,
                                                                    uint32_t groups, LaneParams canon,
                                                                    CtxMergeArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const uint32_t spo = a.slots_per_order, order = blockIdx.x + 1u, base = blockIdx.x * spo, d = a.dim;
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem);
    uint32_t* obs = reinterpret_cast<uint32_t*>(keys + spo);
    uint32_t* owner = obs + spo;
    uint8_t* reset = reinterpret_cast<uint8_t*>(owner + spo);
    __shared__ uint32_t chunk[kApplyThreads];
    __shared__ unsigned long long chunk_key[kApplyThreads], chunk_obs[kApplyThreads];
    __shared__ uint32_t chunk_start[kApplyThreads];
    __shared__ uint32_t chunk_n;
    __shared__ uint32_t warp_n[kApplyThreads / 32], warp_base[kApplyThreads / 32];
    for (uint32_t s = threadIdx.x; s < spo; s += kApplyThreads) {
        keys[s] = canon.ctx_keys[base + s];
        obs[s] = canon.ctx_obs[base + s];
        owner[s] = kNoOwner;
        reset[s] = 0;
    }
    __syncthreads();
    // Walk the merged keys in apply order, a chunk at a time: the chunk's keys
    // of this order are compacted (in order) and placed by one thread.
    for (uint32_t c0 = 0; c0 < groups; c0 += kApplyThreads) {
        const uint32_t i = c0 + threadIdx.x;
        const uint32_t g = i < groups ? apply_order[i] : 0u;
        const bool mine = i < groups && a.morder[g] == order;
        const unsigned ballot = __ballot_sync(0xffffffffu, mine);
        const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
        if (lane == 0) warp_n[warp] = __popc(ballot);
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t t = 0;
            for (uint32_t w = 0; w < kApplyThreads / 32; ++w) {
                warp_base[w] = t;
                t += warp_n[w];
            }
            chunk_n = t;
        }
        __syncthreads();
        if (mine) {  // the chunk's keys and observation sums, loaded in parallel
            const uint32_t at = warp_base[warp] + __popc(ballot & ((1u << lane) - 1u));
            chunk[at] = g;
            const unsigned long long key = a.mkey[g];
            chunk_key[at] = key;
            chunk_obs[at] = a.mobs[g];
            chunk_start[at] = (uint32_t)(key % (unsigned long long)spo);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (uint32_t x = 0; x < chunk_n; ++x) {
                const uint32_t gg = chunk[x];
                const unsigned long long key = chunk_key[x];
                const uint32_t start = chunk_start[x];
                int32_t slot = -1, empty = -1;
                uint32_t weakest = start, weakest_obs = 0xffffffffu;
                for (uint32_t off = 0; off < a.probe_limit; ++off) {
                    const uint32_t s = (start + off) % spo;
                    if (keys[s] == key) {
                        slot = (int32_t)s;
                        break;
                    }
                    if (keys[s] == 0ull && empty < 0) empty = (int32_t)s;
                    if (obs[s] < weakest_obs) {
                        weakest_obs = obs[s];
                        weakest = s;
                    }
                }
                if (slot < 0) {
                    slot = empty >= 0 ? empty : (int32_t)weakest;
                    if (keys[slot] != key) {
                        keys[slot] = key;
                        obs[slot] = 0u;
                        reset[slot] = 1;
                    }
                }
                const unsigned long long inc = chunk_obs[x] < 0xffffffffull ? chunk_obs[x] : 0xffffffffull;
                const unsigned long long sum = (unsigned long long)obs[slot] + inc;
                obs[slot] = (uint32_t)(sum < 0xffffffffull ? sum : 0xffffffffull);
                owner[slot] = gg;
            }
        }
        __syncthreads();
    }
    // Each slot's last key: its embedding (reset or kept) plus the mean delta,
    // projected onto [weight_min, weight_max] and checked finite.
    const double divisor = (double)a.stories;
    for (uint32_t i = threadIdx.x; i < spo * d; i += kApplyThreads) {
        const uint32_t s = i / d, k = i - s * d;
        const uint32_t g = owner[s];
        if (g == kNoOwner) continue;
        const size_t at = (size_t)(base + s) * d + k;
        float v = reset[s] ? 0.0f : canon.ctx_emb[at];
        v = v + (float)(a.msum[(size_t)g * d + k] / divisor);
        v = v < a.weight_min ? a.weight_min : v;  // max(v, lo), NaN kept
        v = a.weight_max < v ? a.weight_max : v;  // min(v, hi), NaN kept
        if (!isfinite(v)) flag_error(a.error, LEO_CTX_MERGE_BAD_VALUE);
        canon.ctx_emb[at] = v;
    }
    for (uint32_t s = threadIdx.x; s < spo; s += kApplyThreads) {
        if (owner[s] == kNoOwner) continue;
        canon.ctx_keys[base + s] = keys[s];
        canon.ctx_obs[base + s] = obs[s];
        a.canon_slots[atomicAdd(a.canon_slot_count, 1u)] = base + s;
    }
}

// 5. canonical rows at `slots` into every resident lane.
__global__ void ctx_broadcast_kernel(const uint32_t* __restrict__ slots, const uint32_t* __restrict__ count_ptr,
                                     uint32_t count_host, LaneParams canon, uint32_t d, const LaneState* lanes,
                                     int lane_count) {
    const uint32_t count = count_ptr ? *count_ptr : count_host;
    const uint32_t total = count * (d + 1);
    for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < total; i += gridDim.x * kThreads) {
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

uint32_t grid_for(size_t n) {
    const size_t b = (n + kThreads - 1) / kThreads;
    return (uint32_t)(b < 1 ? 1 : (b > 4096 ? 4096 : b));
}

}  // namespace

size_t leo_context_apply_smem(uint32_t slots_per_order) {
    return (size_t)slots_per_order * (8 + 4 + 4 + 1);
}

cudaError_t leo_context_merge_configure() {
    return cudaFuncSetAttribute(apply_order_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

cudaError_t leo_context_merge_deltas(const LaneState* lanes, const uint32_t* lane_offset, uint32_t lane_count,
                                     uint32_t max_lane_entries, LaneParams canon, const CtxMergeArgs& a,
                                     cudaStream_t stream) {
    if (max_lane_entries == 0) return cudaSuccess;
    const uint32_t bx = grid_for(max_lane_entries);
    ctx_delta_kernel<<<dim3(bx < 64 ? bx : 64, lane_count), kThreads, 0, stream>>>(lanes, lane_offset, canon, a);
    return cudaGetLastError();
}

cudaError_t leo_context_merge_group(uint32_t entries, const CtxMergeArgs& a, CtxMergeWork& w, uint32_t* valid_out,
                                    cudaStream_t stream) {
    // valid entries, in entry (story) order
    iota_kernel<<<grid_for(entries), kThreads, 0, stream>>>(w.idx_a, entries);
    size_t bytes = w.temp_bytes;
    cudaError_t e = cub::DeviceSelect::Flagged(w.temp, bytes, w.idx_a, a.valid, w.idx_b, w.count, (int)entries, stream);
    if (e != cudaSuccess) return e;
    e = cudaMemcpyAsync(valid_out, w.count, 4, cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return e;
    return cudaStreamSynchronize(stream);
}

cudaError_t leo_context_merge_sort(uint32_t valid, const CtxMergeArgs& a, CtxMergeWork& w, uint32_t* groups_out,
                                   cudaStream_t stream) {
    // stable by key, then stable by order: (order, key, story) order
    size_t bytes = w.temp_bytes;
    gather_u64_kernel<<<grid_for(valid), kThreads, 0, stream>>>(a.key, w.idx_b, w.k64_a, valid, 0);
    cudaError_t e = cub::DeviceRadixSort::SortPairs(w.temp, bytes, w.k64_a, w.k64_b, w.idx_b, w.idx_a, (int)valid, 0,
                                                    64, stream);
    if (e != cudaSuccess) return e;
    gather_u32_kernel<<<grid_for(valid), kThreads, 0, stream>>>(a.order, w.idx_a, w.k32_a, valid);
    bytes = w.temp_bytes;
    e = cub::DeviceRadixSort::SortPairs(w.temp, bytes, w.k32_a, w.k32_b, w.idx_a, w.sorted, (int)valid, 0, 5, stream);
    if (e != cudaSuccess) return e;
    group_head_kernel<<<grid_for(valid), kThreads, 0, stream>>>(w.sorted, a.key, a.order, w.head, valid);
    iota_kernel<<<grid_for(valid), kThreads, 0, stream>>>(w.idx_a, valid);
    bytes = w.temp_bytes;
    e = cub::DeviceSelect::Flagged(w.temp, bytes, w.idx_a, w.head, w.gstart, w.count, (int)valid, stream);
    if (e != cudaSuccess) return e;
    e = cudaMemcpyAsync(groups_out, w.count, 4, cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return e;
    return cudaStreamSynchronize(stream);
}

cudaError_t leo_context_merge_apply(uint32_t valid, uint32_t groups, uint32_t orders, LaneParams canon,
                                    const LaneState* lanes, int lane_count, const uint32_t* lane_slots,
                                    uint32_t lane_slot_count, const CtxMergeArgs& a, CtxMergeWork& w,
                                    cudaStream_t stream) {
    group_sum_kernel<<<grid_for(groups), kThreads, 0, stream>>>(w.sorted, w.gstart, groups, valid, a);
    // apply order: stable by key, by order, by observations descending
    iota_kernel<<<grid_for(groups), kThreads, 0, stream>>>(w.idx_a, groups);
    size_t bytes = w.temp_bytes;
    cudaError_t e = cub::DeviceRadixSort::SortPairs(w.temp, bytes, a.mkey, w.k64_b, w.idx_a, w.idx_b, (int)groups, 0,
                                                    64, stream);
    if (e != cudaSuccess) return e;
    gather_u32_kernel<<<grid_for(groups), kThreads, 0, stream>>>(a.morder, w.idx_b, w.k32_a, groups);
    bytes = w.temp_bytes;
    e = cub::DeviceRadixSort::SortPairs(w.temp, bytes, w.k32_a, w.k32_b, w.idx_b, w.idx_a, (int)groups, 0, 5, stream);
    if (e != cudaSuccess) return e;
    gather_u64_kernel<<<grid_for(groups), kThreads, 0, stream>>>(a.mobs, w.idx_a, w.k64_a, groups, 1);
    bytes = w.temp_bytes;
    e = cub::DeviceRadixSort::SortPairs(w.temp, bytes, w.k64_a, w.k64_b, w.idx_a, w.idx_b, (int)groups, 0, 64,
                                        stream);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(a.canon_slot_count, 0, 4, stream);
    if (e != cudaSuccess) return e;
    apply_order_kernel<<<orders, kApplyThreads, leo_context_apply_smem(a.slots_per_order), stream>>>(w.idx_b, groups,
                                                                                                   canon, a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (lane_count > 0) {
        const uint32_t d = a.dim;
        ctx_broadcast_kernel<<<grid_for((size_t)a.canon_slot_capacity * (d + 1)), kThreads, 0, stream>>>(
            a.canon_slots, a.canon_slot_count, 0u, canon, d, lanes, lane_count);
        if (lane_slot_count)
            ctx_broadcast_kernel<<<grid_for((size_t)lane_slot_count * (d + 1)), kThreads, 0, stream>>>(
                lane_slots, nullptr, lane_slot_count, canon, d, lanes, lane_count);
    }
    return cudaGetLastError();
}

size_t leo_context_merge_temp_bytes(uint32_t capacity) {
    size_t a = 0, b = 0, c = 0, d = 0;
    cub::DeviceSelect::Flagged(nullptr, a, (uint32_t*)nullptr, (uint8_t*)nullptr, (uint32_t*)nullptr,
                               (uint32_t*)nullptr, (int)capacity);
    cub::DeviceRadixSort::SortPairs(nullptr, b, (unsigned long long*)nullptr, (unsigned long long*)nullptr,
                                    (uint32_t*)nullptr, (uint32_t*)nullptr, (int)capacity, 0, 64);
    cub::DeviceRadixSort::SortPairs(nullptr, c, (uint32_t*)nullptr, (uint32_t*)nullptr, (uint32_t*)nullptr,
                                    (uint32_t*)nullptr, (int)capacity, 0, 5);
    d = a > b ? a : b;
    return d > c ? d : c;
}
