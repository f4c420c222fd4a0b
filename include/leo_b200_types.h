/*
 * Plain-C data types shared by the leo_b200 C ABI.
 *
 * These types carry Leo's persistent model and configuration across the
 * boundary as plain pointers and sizes, with no torch or CUDA types.  The
 * kernel-side configuration is the generated `struct LeoConfig` from
 * cuda_abi.def (crates/leo-core/cuda_abi.def:4-44, emitted by
 * crates/leo-core/build.rs:97-121); the fields that file does not carry but
 * that the reference host reads from `Config` are in LeoB200HostConfig.
 *
 * This header is C++-only when included together with leo_cuda_abi.h,
 * because that generated header uses a C++ static_assert on a bare type name.
 */
#ifndef LEO_B200_TYPES_H
#define LEO_B200_TYPES_H

#include <stddef.h>
#include <stdint.h>

/* The generated ABI header (byte-identical to the reference build's output)
   has no include guard of its own. */
#ifndef LEO_CUDA_ABI_INCLUDED
#define LEO_CUDA_ABI_INCLUDED
#include "leo_cuda_abi.h"
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LEO_B200_BYTE_SYMBOLS 256u
#define LEO_B200_BEGIN_DOCUMENT 256u   /* crates/leo-core/src/symbols.rs:4 */
#define LEO_B200_END_DOCUMENT 257u     /* crates/leo-core/src/symbols.rs:5 */
#define LEO_B200_SYMBOL_COUNT 258u     /* crates/leo-core/src/symbols.rs:6 */
#define LEO_B200_OUTPUT_CLASSES 257u   /* crates/leo-core/src/symbols.rs:7 */
#define LEO_B200_END_OUTPUT_INDEX 256u /* crates/leo-core/src/symbols.rs:8 */

/* Return value of an optional device path that does not take the given input
   (the trait's Ok(None), crates/leo-core/src/backend.rs:457-474): the caller
   runs the step-level path instead.  Errors are -1. */
#define LEO_B200_UNSUPPORTED 1

/* Permission, crates/leo-core/src/permission.rs:5-11. */
enum LeoB200Permission {
    LEO_B200_FROZEN = 0,
    LEO_B200_PROVISIONAL = 1,
    LEO_B200_TRAINING = 2,
    LEO_B200_VERIFIED = 3
};

/* Model topology builders for synthetic models. */
enum LeoB200Topology {
    /* crates/leo-core/src/model.rs:79-158 exactly (local/long-range fan-out). */
    LEO_B200_TOPOLOGY_REFERENCE = 0,
    /* Fan-out lists with targets drawn uniformly without replacement and
       weights |N(0, 1/sqrt(S))| signed by source type. */
    LEO_B200_TOPOLOGY_UNIFORM = 1,
    /* As UNIFORM, but targets drawn from Zipf(s = 1.1) over a fixed random
       permutation of the neurons (power-law in-degree skew). */
    LEO_B200_TOPOLOGY_ZIPF = 2
};

/* Config fields the reference host reads from crates/leo-core/src/config.rs
   but cuda_abi.def does not carry. */
typedef struct LeoB200HostConfig {
    uint64_t seed;                  /* config.rs:23  model.seed */
    float excitatory_fraction;      /* config.rs:28  model.excitatory_fraction */
    float provisional_strength;     /* config.rs:88  learning.provisional_strength */
    float training_strength;        /* config.rs:89  learning.training_strength */
    float verified_strength;        /* config.rs:90  learning.verified_strength */
    uint32_t plasticity_window;     /* config.rs:94  learning.plasticity_window */
    float end_document_weight;      /* config.rs:96  learning.end_document_weight */
    float context_dropout_rate;     /* config.rs:109 context.dropout_rate */
    float replay_fraction;          /* config.rs:116 replay.fraction */
    uint32_t replay_segment_bytes;  /* config.rs:118 replay.segment_bytes */
    uint32_t reserved0;
} LeoB200HostConfig;

typedef struct LeoB200Config {
    struct LeoConfig abi;           /* 160 bytes, generated from cuda_abi.def */
    LeoB200HostConfig host;         /* 48 bytes */
} LeoB200Config;

/* TrainingStatistics, crates/leo-core/src/metrics.rs:3-15. */
typedef struct LeoB200Statistics {
    uint64_t processed_bytes;
    uint64_t processed_stories;
    double training_loss_sum;
    uint64_t training_targets;
    uint64_t active_neurons_sum;
    uint64_t active_neurons_peak;
    uint64_t synaptic_events;
    uint64_t numerical_rejections;
    uint64_t persistent_ticks;
} LeoB200Statistics;

/*
 * A persistent model (crates/leo-core/src/model.rs:65-76) as caller-owned
 * arrays.  Sizes follow from the config: N = neuron_count,
 * S = synapses_per_neuron, F = input_fanout, D = context_embedding_dim,
 * C = context_max_order * context_slots_per_order.  The output matrix uses the
 * checkpoint's output-major layout [257][N] (model.rs:48).
 */
typedef struct LeoB200HostModel {
    LeoB200Config config;
    uint64_t generation;
    uint64_t parameter_revision;
    LeoB200Statistics statistics;
    float* threshold;               /* [N] */
    float* excitability;            /* [N] */
    uint8_t* neuron_type;           /* [N] 0 excitatory, 1 inhibitory */
    uint32_t* recurrent_target;     /* [N*S] fan-out slots per source */
    uint8_t* recurrent_branch;      /* [N*S] */
    uint8_t* recurrent_delay;       /* [N*S] 1, 2, 4 or 8 */
    float* recurrent_weight;        /* [N*S] */
    uint32_t* input_target;         /* [258*F] */
    uint8_t* input_branch;          /* [258*F] */
    float* input_weight;            /* [258*F] */
    float* output_weight;           /* [257*N] output-major */
    float* output_bias;             /* [257] */
    uint64_t* context_keys;         /* [C] */
    float* context_embeddings;      /* [C*D] */
    uint32_t* context_observations; /* [C] */
    float* context_output_weight;   /* [257*D] output-major */
} LeoB200HostModel;

/* StepMetrics, crates/leo-core/src/metrics.rs:39-66 (subset with fixed-width
   fields; `loss` is NaN when the step had no target). */
typedef struct LeoB200StepMetrics {
    float loss;
    uint32_t predicted_symbol;
    uint32_t active_neurons;
    uint32_t emitted_events;
    uint32_t suprathreshold_neurons;
    uint32_t block_selected_neurons;
    uint32_t global_cap_clipped_neurons;
    float population_inhibition;
    uint32_t context_cells;
    uint32_t context_probes;
    uint32_t context_applied;
    float context_loss_gain;
    uint64_t output_madds;
    uint64_t eligible_recurrent_synapses;
    uint64_t eligible_input_synapses;
    float mean_abs_eligibility;
    uint32_t reserved0;
} LeoB200StepMetrics;

/* DeviceStorySummary, crates/leo-core/src/backend.rs:320-328. */
typedef struct LeoB200StorySummary {
    double training_loss_sum;
    uint64_t training_targets;
    uint64_t active_neurons_sum;
    uint64_t active_neurons_peak;
    uint64_t synaptic_events;
    uint64_t context_applied_steps;
} LeoB200StorySummary;

/* MergeMetrics, crates/leo-core/src/parallel.rs:305-310, plus replay counts
   from BatchTrainingReport (crates/leo-cli/src/training.rs). */
typedef struct LeoB200BatchReport {
    uint64_t workers;
    uint64_t fixed_parameter_updates;
    uint64_t context_keys;
    uint64_t stories;
    uint64_t input_bytes;
    uint64_t targets;
    double mean_loss;
    uint64_t replay_segments;
    uint64_t replay_steps;
    uint64_t replay_prefix_steps;
} LeoB200BatchReport;

/* One story of a sharded logical batch, as the rank that ran it reports it for
   the batch-end merge on every rank: the story's statistics delta
   (parallel.rs:1115-1137; `loss_sum` is the lane's running
   training_loss_sum, which started at the canonical value) and its length. */
typedef struct LeoB200ShardStory {
    double loss_sum;
    uint64_t processed_bytes;
    uint64_t targets;
    uint64_t active_sum;
    uint64_t active_peak;
    uint64_t synaptic_events;
    uint64_t numerical_rejections;
    uint64_t persistent_ticks;
    uint64_t revision_increment;
    uint64_t context_applied_steps;
    uint64_t story_bytes;
} LeoB200ShardStory;

/* Replay geometry of leo_b200_set_cluster_sizes: the replay lane over the
   whole GPU, one CTA per SM with grid-wide phase barriers. */
#define LEO_B200_WHOLE_GPU 0xFFFFFFFFu

/* Fixed tensors merged at the batch end, in merge order. */
#define LEO_B200_FIXED_TENSORS 6

/* Per-story sparse deltas (SparseModelDelta, crates/leo-core/src/parallel.rs:
   41-55): the fixed tensors in this order -- threshold, recurrent weight,
   input weight, output weight (reference index output * N + neuron), output
   bias, context output weight -- each a list of (index, delta) sorted by index
   with every delta nonzero, then the keyed context deltas sorted by (order,
   key), the statistics delta and the revision increment of every story. */
#define LEO_B200_DELTA_TENSORS 6

/* Tracked-index lists of a story's ParameterChanges (runtime.rs:38-46), in
   this order: threshold, recurrent weight, input weight, output neurons,
   context slots. */
#define LEO_B200_CHANGE_LISTS 5

typedef struct LeoB200StoryDeltaSizes {
    uint64_t entries[LEO_B200_DELTA_TENSORS]; /* (index, delta) pairs of all stories, per tensor */
    uint64_t context_entries;                 /* keyed context deltas of all stories */
    uint32_t embedding_dim;                   /* floats per context embedding delta */
    uint32_t stories;
    uint64_t changes[LEO_B200_CHANGE_LISTS];  /* changed indices of all stories, per list */
} LeoB200StoryDeltaSizes;

/* Caller-owned buffers for the deltas of `stories` stories; story s owns
   entries offsets[t][s] .. offsets[t][s + 1] of tensor t and context entries
   context_offsets[s] .. context_offsets[s + 1]. */
typedef struct LeoB200StoryDeltas {
    uint64_t* offsets[LEO_B200_DELTA_TENSORS];  /* stories + 1 each */
    uint32_t* indices[LEO_B200_DELTA_TENSORS];  /* entries[t] each */
    float* deltas[LEO_B200_DELTA_TENSORS];      /* entries[t] each */
    uint64_t* context_offsets;                  /* stories + 1 */
    uint32_t* context_orders;                   /* context_entries */
    uint64_t* context_keys;                     /* context_entries */
    uint32_t* context_observation_increments;   /* context_entries */
    float* context_embedding_deltas;            /* context_entries x embedding_dim */
    LeoB200Statistics* statistics;              /* stories: statistics delta (parallel.rs statistics_delta) */
    uint64_t* revision_increments;              /* stories */
    /* Each story's ParameterChanges (DeviceStoryBatchDeltaReport::story_changes,
       backend.rs:348): every index its lane changed, sorted, per list; and
       per story bit 0 output_bias_dirty, bit 1 context_output_dirty. */
    uint64_t* change_offsets[LEO_B200_CHANGE_LISTS]; /* stories + 1 each */
    uint32_t* change_indices[LEO_B200_CHANGE_LISTS]; /* changes[l] each */
    uint32_t* dirty_flags;                           /* stories */
} LeoB200StoryDeltas;

/* Changed-parameter indices of the canonical runtime since tracking was
   enabled (ParameterChanges, crates/leo-core/src/runtime.rs:38-46). */
typedef struct LeoB200ParameterChangeSizes {
    uint64_t threshold, recurrent_weight, input_weight, output_neurons, context_slots;
    uint32_t output_bias_dirty, context_output_dirty;
} LeoB200ParameterChangeSizes;

typedef struct LeoB200ParameterChanges {
    uint32_t* threshold;         /* sorted indices */
    uint32_t* recurrent_weight;
    uint32_t* input_weight;
    uint32_t* output_neurons;
    uint32_t* context_slots;
} LeoB200ParameterChanges;

/* PackedSparseModelUpdate (crates/leo-core/src/parallel.rs:78-97): host values
   written over the canonical model and every resident lane. */
typedef struct LeoB200PackedUpdate {
    const uint32_t* threshold_indices;
    const float* threshold_values;
    uint64_t threshold_count;
    const uint32_t* recurrent_indices;
    const float* recurrent_values;
    uint64_t recurrent_count;
    const uint32_t* input_indices;
    const float* input_values;
    uint64_t input_count;
    const uint32_t* output_neurons;
    const float* output_values_by_neuron; /* 257 per neuron, output order */
    uint64_t output_count;
    const uint32_t* context_slots;
    const uint64_t* context_keys;
    const uint32_t* context_observations;
    const float* context_embeddings; /* embedding_dim per slot */
    uint64_t context_count;
    const float* output_bias;            /* 257 values, or NULL: unchanged */
    const float* context_output_weights; /* 257 x embedding_dim, or NULL */
    uint64_t generation;
    uint64_t parameter_revision;
    LeoB200Statistics statistics;
} LeoB200PackedUpdate;

/* Phases of one step of the persistent wavefront, in execution order. */
#define LEO_B200_PHASES 11
enum LeoB200Phase {
    LEO_B200_PHASE_DELIVER = 0,
    LEO_B200_PHASE_SETTLE = 1,
    LEO_B200_PHASE_BLOCKS = 2,
    LEO_B200_PHASE_ASSEMBLE = 3,
    LEO_B200_PHASE_SURROGATE = 4,
    LEO_B200_PHASE_ELIGIBLE = 5,
    LEO_B200_PHASE_EMIT_FORWARD = 6,
    LEO_B200_PHASE_LEARN = 7,
    LEO_B200_PHASE_PLASTICITY = 8,
    LEO_B200_PHASE_INHIBIT = 9,
    LEO_B200_PHASE_SETTLE_HUBS = 10 /* part of SETTLE: hub targets, as the first CTA sees it */
};

/* Performance counters since the last reset.  work_* sum, over lanes and
   steps, the units each phase processed: due events plus input slots
   (deliver), touched neurons (settle, surrogate, homeostasis), eligible
   recurrent plus input slots before compaction (eligibility), learning
   destinations on plasticity steps (signals), active neurons, and kept
   slots with nonzero eligibility (the only weight updates that change a
   weight).  phase_cycles
   are SM clock cycles spent in each phase (barrier waits included) by the
   first thread of each lane's first CTA; wavefront_ms is CUDA-event time of
   the persistent wavefront launches (story_* for the story-pass launches). */
typedef struct LeoB200PerfStats {
    uint64_t launches;
    uint64_t wavefront_launches;
    double wavefront_ms;
    uint64_t story_wavefront_launches;
    double story_wavefront_ms;
    uint64_t phase_cycles[LEO_B200_PHASES];
    uint64_t work_deliver;
    uint64_t work_touched;
    uint64_t work_eligible;
    uint64_t work_destinations;
    uint64_t work_active;
    uint64_t work_plastic;
    uint64_t work_steps;
    uint64_t story_work_steps;
    uint64_t batches;
    double batch_ms;
    uint32_t story_cluster;
    uint32_t replay_cluster;
    uint64_t story_lane_launches[5]; /* story-pass lane launches at cluster size 1, 2, 4, 8, 16 */
    uint64_t whole_gpu_launches;     /* replay launches over the whole GPU (one CTA per SM) */
    int32_t fit_clusters[3];         /* co-resident clusters of 4, 8 and 16 CTAs */
    int32_t sm_count;
    /* Host wall time of the batch-end steps, summed over batches (each step
       ends with a stream synchronize, so wall time covers its device work). */
    double collect_ms;        /* lane scalars, losses and error flags read back */
    double merge_fixed_ms;    /* FP64 mean merge of the six fixed tensors */
    double merge_context_ms;  /* keyed context merge and lane context sync */
    double replay_ms;         /* serial canonical replay, range selection to last segment */
    double replay_sync_ms;    /* replay's changed rows into every lane */
    /* The replay lane alone (serial canonical replay): phase cycles of its
       first CTA's first thread (wall time of the launch, barrier waits
       included), and its work counters. */
    uint64_t replay_phase_cycles[LEO_B200_PHASES];
    uint64_t replay_work_steps;
    uint64_t replay_work_touched;
    uint64_t replay_work_active;
    uint64_t replay_work_deliver;
    uint64_t replay_work_eligible;
    uint64_t work_inhibit;  /* inhibitory-source slots visited by inhibitory homeostasis */
    uint64_t work_winners;  /* block winners (selection records) assembled */
} LeoB200PerfStats;

#ifdef __cplusplus
}
#endif

#endif /* LEO_B200_TYPES_H */
