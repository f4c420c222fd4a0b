// Device-side layout of the per-byte training step (shared by the kernels and
// the host runtime).  Plain structs of device pointers; no torch types.
//
// Layout in HBM, per device:
//   * topology (read-only, one copy): one packed u32 word per recurrent slot
//     (target | branch << 24 | delay << 26) and per input slot
//     (target | branch << 24), neuron type, excitability;
//   * canonical learned parameters, and for every lane (logical story worker)
//     a private copy: thresholds, recurrent / input / output weights, bias and
//     the context tables.  Output weights are neuron-major rows of
//     LEO_OUTPUT_STRIDE floats (16-byte aligned) instead of the checkpoint's
//     output-major [257][N], so an active neuron's row is one coalesced read;
//   * transient lane state: 32-byte NeuronHot / NeuronCold records and a
//     float4 of branch accumulators per neuron, a 32-byte trace record per
//     recurrent and per input slot, the 9-tick delay ring of active lists and
//     emitted event values, per-(target, branch) event lists, the eligible
//     slot worklists (ping-pong), learning destinations and changed-parameter
//     marks and lists for the batch-end merge.
#pragma once

#include <stdint.h>

/* The generated ABI header (byte-identical to the reference build's output)
   has no include guard of its own. */
#ifndef LEO_CUDA_ABI_INCLUDED
#define LEO_CUDA_ABI_INCLUDED
#include "../../include/leo_cuda_abi.h"
#endif

#define LEO_OUTPUT_CLASSES 257u
#define LEO_OUTPUT_STRIDE 260u  // row stride of neuron-major output weights
#define LEO_SYMBOLS 258u
#define LEO_RING 9u             // max delay (8) + 1, runtime.rs:199-208
#define LEO_EMPTY 0xffffffffu
#define LEO_MAX_CONTEXT_ORDER 16u
#define LEO_MAX_EMBEDDING 256u
#define LEO_WAVEFRONT_THREADS 512u  // threads per CTA of the persistent wavefront
#define LEO_PHASES 11
// Capacity bits of DeviceTopology::seg[n].y (bit 31: listed for the CTA tier).
#define LEO_SEG_CAPACITY 0x7fffffffu
#define LEO_SEG_LISTED 0x80000000u

// Packed topology words.
#define LEO_TARGET_MASK 0x00ffffffu
#define LEO_WORD_BRANCH(w) (((w) >> 24) & 3u)
#define LEO_WORD_DELAY(w) (((w) >> 26) & 15u)

// Step schedule word: symbol | (target + 1) << 9 | permission << 19.
#define LEO_SCHED_SYMBOL(w) ((w) & 0x1ffu)
#define LEO_SCHED_TARGET(w) ((int)(((w) >> 9) & 0x3ffu) - 1)
#define LEO_SCHED_PERMISSION(w) (((w) >> 19) & 3u)

__host__ __device__ __forceinline__ uint32_t leo_schedule_word(uint32_t symbol, int target, uint32_t permission) {
    return symbol | ((uint32_t)(target + 1) << 9) | (permission << 19);
}

// Error flag bits (reported to the host after a batch).
#define LEO_ERR_NONFINITE_BIAS 1u
#define LEO_ERR_NONFINITE_OUTPUT 2u
#define LEO_ERR_NONFINITE_CONTEXT 4u
#define LEO_ERR_NONFINITE_RECURRENT 8u
#define LEO_ERR_NONFINITE_INPUT 16u
#define LEO_ERR_NONFINITE_INHIBITORY 32u
#define LEO_ERR_CAPACITY 64u

struct __align__(32) NeuronHot {
    uint32_t tag;               // ((tick + 1) << 2) | selected << 1 | (touched and not refractory)
    float surrogate;            // learning.rs:6-24 for this tick
    float j_exc;                // branch Jacobian of E and I branches (excitability)
    float j_temporal;           // exc * clamp(G, 0, 1)
    float j_gate;               // exc * T * gate'(G)
    float activation;           // > 0 only while active this tick
    uint32_t refractory_until;  // relative tick
    uint32_t reserved;
};

struct __align__(32) NeuronCold {
    float membrane;
    float fatigue;
    float adaptation[3];
    uint32_t branch_tick;   // relative tick of the last branch decay
    uint32_t neuron_tick;   // relative tick of the last membrane/fatigue/adaptation decay
    uint32_t reserved;
};

struct __align__(32) Trace {
    float branch_sens;
    float membrane_sens;
    float fatigue_sens;
    float adaptation_sens[3];
    float eligibility;
    uint32_t tick_mark;  // (last_tick << 1) | in-eligible-list
};

struct LaneParams {
    float* threshold;     // [N]
    float* rec_weight;    // [N*S]
    float* in_weight;     // [258*F]
    float* out_weight;    // [N][LEO_OUTPUT_STRIDE]
    float* out_bias;      // [LEO_OUTPUT_STRIDE]
    unsigned long long* ctx_keys;  // [C]
    uint32_t* ctx_obs;    // [C]
    float* ctx_emb;       // [C*D]
    float* ctx_out;       // [257*D]
};

// Per-lane scalars and counters, resident in device memory.
struct LaneScalars {
    unsigned long long base_tick;  // absolute tick at the last transient reset
    uint32_t steps;                // schedule length of this lane
    uint32_t plasticity_phase;
    float population_inhibition;
    float population_cutoff;
    uint32_t touched_count;
    uint32_t dst_count;
    uint32_t elig_cur;          // which worklist of each ping-pong pair is current
    uint32_t elig_count[2];
    uint32_t in_elig_count[2];
    uint32_t ring_count[LEO_RING];
    // context (runtime.rs:641-699)
    uint32_t ctx_history[LEO_MAX_CONTEXT_ORDER];
    uint32_t ctx_history_len;
    uint32_t ctx_count;
    uint32_t ctx_applied;
    uint32_t ctx_probes;
    int32_t ctx_slot_by_order[LEO_MAX_CONTEXT_ORDER];
    uint32_t ctx_slots[LEO_MAX_CONTEXT_ORDER];
    float ctx_scales[LEO_MAX_CONTEXT_ORDER];
    // per-step learning scalars written by the forward pass for later phases
    uint32_t step_flags;  // bit0 supervised learning, bit1 plasticity commit, bit2 non-frozen
    float step_strength;
    float step_supervised;
    float step_consolidated;
    // changed-parameter tracking (runtime.rs:1386-1448)
    uint32_t thr_changed, rec_changed, in_changed, out_changed, ctx_changed;
    uint32_t bias_dirty, ctx_out_dirty;
    // statistics (metrics.rs:3-15), accumulated from the lane's start values
    double loss_sum;
    unsigned long long processed_bytes, targets, active_sum, active_peak, synaptic_events;
    unsigned long long numerical_rejections, persistent_ticks, revision_increment, context_applied_steps;
    uint32_t error_flag;
    // work counters (units per phase, summed over steps; see LeoB200PerfStats)
    unsigned long long work_inhibit;   // inhibitory-source slots visited by inhibitory homeostasis
    unsigned long long work_winners;   // block winners (selection records) assembled
    unsigned long long work_deliver, work_touched, work_eligible, work_destinations, work_active, work_plastic,
        work_steps;
    unsigned long long phase_cycles[LEO_PHASES];  // SM clock cycles per phase (first CTA, first thread)
    uint32_t step_supra;                          // candidates of the current tick (all blocks)
    // last-step metrics
    uint32_t last_active, last_suprathreshold, last_block_selected, last_clipped, last_predicted;
    float last_loss;
};

struct DeviceTopology {
    uint32_t n, s, f, d, k, spo, ctx_slots, blocks, npb, keep, max_active;
    const uint32_t* rec_word;      // [N*S]
    const uint32_t* in_word;       // [258*F]
    const uint8_t* neuron_type;    // [N]
    const float* excitability;     // [N]
    // Per-target event segments: every target n owns entries
    // seg[n].x .. seg[n].x + (seg[n].y & LEO_SEG_CAPACITY) of a lane's
    // seg_events, where its events of a step are appended as keys
    // (branch << 30 | event order) and sorted in settle.  Bit 31 of seg[n].y
    // marks the listed targets (cta_targets) that the CTA tier settles.
    const uint2* seg;               // [N] (offset, capacity | listed << 31)
    const uint32_t* cta_targets;    // [cta_count] listed targets in descending capacity
    uint32_t cta_count;
    uint32_t cta_events;            // a listed target with more events than this is sorted by a whole CTA
    uint32_t thread_events;         // an unlisted target with at most this many is settled by one thread
};

struct LaneState {
    LaneParams p;
    // Canonical output rows.  A lane's private row equals the canonical row
    // until the lane changes it (out_mark set): the batch-end sync restores that
    // invariant and the canonical model is constant during a story pass, so
    // unchanged rows are read from the shared canonical copy (one L2-resident
    // matrix for every lane instead of one per lane).
    const float* canon_out_weight;
    LaneScalars* sc;
    const uint32_t* schedule;   // [steps]
    float* step_loss;           // [steps] loss per step (0 when untargeted)
    uint32_t* step_active;      // [steps] active neurons per step
    NeuronHot* hot;             // [N]
    NeuronCold* cold;           // [N]
    float4* branches;           // [N] (E, I, T, G)
    uint32_t* touch_epoch;      // [N] tick+1 of the last touch
    uint32_t* touched;          // [N]
    unsigned long long* block_cand;  // [blocks * npb] packed selection keys
    uint32_t* block_cand_count;      // [blocks]
    float* block_cutoff;             // [blocks]
    unsigned long long* block_winners;  // [blocks * keep] winners of each block in rank order
    uint32_t* block_nwin;               // [blocks]
    uint32_t* ring_src;         // [9 * max_active]
    float* ring_act;            // [9 * max_active]
    float* ring_val;            // [9 * max_active * S] emitted a * w snapshots
    float* ev_val;              // [event capacity] event values by event order
    uint32_t* seg_count;        // [N] events each target received this step
    uint32_t* seg_events;       // [sum of segment capacities] keys: branch << 30 | event order
    uint2* elig[2];             // recurrent worklists {slot, eligibility bits}
    uint2* in_elig[2];          // input worklists
    Trace* traces;              // [N*S]
    Trace* in_traces;           // [258*F]
    uint32_t* dst_list;         // [N]
    uint32_t* dst_epoch;        // [N]
    float* signal;              // [N]
    float* errors;              // [LEO_OUTPUT_STRIDE]
    float* probs;               // [LEO_OUTPUT_STRIDE]
    uint8_t* thr_mark;  uint32_t* thr_list;   // [N]
    uint8_t* rec_mark;  uint32_t* rec_list;   // [N*S]
    uint8_t* in_mark;   uint32_t* in_list;    // [258*F]
    uint8_t* out_mark;  uint32_t* out_list;   // [N]
    uint8_t* ctx_mark;  uint32_t* ctx_list;   // [C]
    // Where the first CTA reports the lane's work per step (eligible slots +
    // events emitted + touched neurons) at the end of each launch; the host
    // sizes the next launch's clusters from it.  Null: not reported.
    uint32_t* load_out;
};

struct KernelConsts {
    LeoConfig cfg;
    DeviceTopology topo;
    float strength[4];              // permission.rs:24-31
    float end_document_weight;
    uint32_t plasticity_window;
    float dropout_rate;
    uint32_t track_changes;
    unsigned long long seed;
    const uint2* exp_table;   // open-addressing (input bits, output bits), empty key 0xffffffff
    const uint2* log_table;
    uint32_t exp_mask;        // capacity - 1 (power of two)
    uint32_t log_mask;
    uint32_t event_capacity;
    uint32_t event_bits;      // bits of the largest event order (event_capacity - 1)
};
