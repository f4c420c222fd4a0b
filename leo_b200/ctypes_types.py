"""ctypes mirrors of ``include/leo_b200_types.h`` and ``include/leo_cuda_abi.h``.

The ``LeoConfig`` field list is read from ``cuda_abi.def`` itself, so the
Python view cannot drift from the generated C header
(``crates/leo-core/cuda_abi.def:4-44``).
"""

from __future__ import annotations

import ctypes as C

from .abi.generate import DEFAULT_SPEC, parse_spec

_SPEC = parse_spec(DEFAULT_SPEC.read_text(encoding="utf-8"))


class LeoConfig(C.Structure):
    _fields_ = [(name, C.c_uint32 if ty == "u32" else C.c_float) for ty, name in _SPEC.config]


assert C.sizeof(LeoConfig) == 4 * len(_SPEC.config) == 160


class LeoB200HostConfig(C.Structure):
    _fields_ = [
        ("seed", C.c_uint64),
        ("excitatory_fraction", C.c_float),
        ("provisional_strength", C.c_float),
        ("training_strength", C.c_float),
        ("verified_strength", C.c_float),
        ("plasticity_window", C.c_uint32),
        ("end_document_weight", C.c_float),
        ("context_dropout_rate", C.c_float),
        ("replay_fraction", C.c_float),
        ("replay_segment_bytes", C.c_uint32),
        ("reserved0", C.c_uint32),
    ]


class LeoB200Config(C.Structure):
    _fields_ = [("abi", LeoConfig), ("host", LeoB200HostConfig)]


class LeoB200Statistics(C.Structure):
    _fields_ = [
        ("processed_bytes", C.c_uint64),
        ("processed_stories", C.c_uint64),
        ("training_loss_sum", C.c_double),
        ("training_targets", C.c_uint64),
        ("active_neurons_sum", C.c_uint64),
        ("active_neurons_peak", C.c_uint64),
        ("synaptic_events", C.c_uint64),
        ("numerical_rejections", C.c_uint64),
        ("persistent_ticks", C.c_uint64),
    ]


class LeoB200HostModel(C.Structure):
    _fields_ = [
        ("config", LeoB200Config),
        ("generation", C.c_uint64),
        ("parameter_revision", C.c_uint64),
        ("statistics", LeoB200Statistics),
        ("threshold", C.POINTER(C.c_float)),
        ("excitability", C.POINTER(C.c_float)),
        ("neuron_type", C.POINTER(C.c_uint8)),
        ("recurrent_target", C.POINTER(C.c_uint32)),
        ("recurrent_branch", C.POINTER(C.c_uint8)),
        ("recurrent_delay", C.POINTER(C.c_uint8)),
        ("recurrent_weight", C.POINTER(C.c_float)),
        ("input_target", C.POINTER(C.c_uint32)),
        ("input_branch", C.POINTER(C.c_uint8)),
        ("input_weight", C.POINTER(C.c_float)),
        ("output_weight", C.POINTER(C.c_float)),
        ("output_bias", C.POINTER(C.c_float)),
        ("context_keys", C.POINTER(C.c_uint64)),
        ("context_embeddings", C.POINTER(C.c_float)),
        ("context_observations", C.POINTER(C.c_uint32)),
        ("context_output_weight", C.POINTER(C.c_float)),
    ]


class LeoB200StepMetrics(C.Structure):
    _fields_ = [
        ("loss", C.c_float),
        ("predicted_symbol", C.c_uint32),
        ("active_neurons", C.c_uint32),
        ("emitted_events", C.c_uint32),
        ("suprathreshold_neurons", C.c_uint32),
        ("block_selected_neurons", C.c_uint32),
        ("global_cap_clipped_neurons", C.c_uint32),
        ("population_inhibition", C.c_float),
        ("context_cells", C.c_uint32),
        ("context_probes", C.c_uint32),
        ("context_applied", C.c_uint32),
        ("context_loss_gain", C.c_float),
        ("output_madds", C.c_uint64),
        ("eligible_recurrent_synapses", C.c_uint64),
        ("eligible_input_synapses", C.c_uint64),
        ("mean_abs_eligibility", C.c_float),
        ("reserved0", C.c_uint32),
    ]


class LeoB200StorySummary(C.Structure):
    _fields_ = [
        ("training_loss_sum", C.c_double),
        ("training_targets", C.c_uint64),
        ("active_neurons_sum", C.c_uint64),
        ("active_neurons_peak", C.c_uint64),
        ("synaptic_events", C.c_uint64),
        ("context_applied_steps", C.c_uint64),
    ]


class LeoB200ShardStory(C.Structure):
    _fields_ = [
        ("loss_sum", C.c_double),
        ("processed_bytes", C.c_uint64),
        ("targets", C.c_uint64),
        ("active_sum", C.c_uint64),
        ("active_peak", C.c_uint64),
        ("synaptic_events", C.c_uint64),
        ("numerical_rejections", C.c_uint64),
        ("persistent_ticks", C.c_uint64),
        ("revision_increment", C.c_uint64),
        ("context_applied_steps", C.c_uint64),
        ("story_bytes", C.c_uint64),
    ]


FIXED_TENSORS = 6
WHOLE_GPU = 0xFFFFFFFF


class LeoB200BatchReport(C.Structure):
    _fields_ = [
        ("workers", C.c_uint64),
        ("fixed_parameter_updates", C.c_uint64),
        ("context_keys", C.c_uint64),
        ("stories", C.c_uint64),
        ("input_bytes", C.c_uint64),
        ("targets", C.c_uint64),
        ("mean_loss", C.c_double),
        ("replay_segments", C.c_uint64),
        ("replay_steps", C.c_uint64),
        ("replay_prefix_steps", C.c_uint64),
    ]


DELTA_TENSORS = 6  # threshold, recurrent weight, input weight, output weight, output bias, context output
CHANGE_LISTS = 5   # threshold, recurrent weight, input weight, output neurons, context slots
UNSUPPORTED = 1    # an optional device path that does not take the input (the trait's Ok(None))


class LeoB200StoryDeltaSizes(C.Structure):
    _fields_ = [
        ("entries", C.c_uint64 * DELTA_TENSORS),
        ("context_entries", C.c_uint64),
        ("embedding_dim", C.c_uint32),
        ("stories", C.c_uint32),
        ("changes", C.c_uint64 * CHANGE_LISTS),
    ]


class LeoB200StoryDeltas(C.Structure):
    _fields_ = [
        ("offsets", C.c_void_p * DELTA_TENSORS),
        ("indices", C.c_void_p * DELTA_TENSORS),
        ("deltas", C.c_void_p * DELTA_TENSORS),
        ("context_offsets", C.c_void_p),
        ("context_orders", C.c_void_p),
        ("context_keys", C.c_void_p),
        ("context_observation_increments", C.c_void_p),
        ("context_embedding_deltas", C.c_void_p),
        ("statistics", C.c_void_p),
        ("revision_increments", C.c_void_p),
        ("change_offsets", C.c_void_p * CHANGE_LISTS),
        ("change_indices", C.c_void_p * CHANGE_LISTS),
        ("dirty_flags", C.c_void_p),
    ]


class LeoB200ParameterChangeSizes(C.Structure):
    _fields_ = [
        ("threshold", C.c_uint64),
        ("recurrent_weight", C.c_uint64),
        ("input_weight", C.c_uint64),
        ("output_neurons", C.c_uint64),
        ("context_slots", C.c_uint64),
        ("output_bias_dirty", C.c_uint32),
        ("context_output_dirty", C.c_uint32),
    ]


class LeoB200ParameterChanges(C.Structure):
    _fields_ = [
        ("threshold", C.c_void_p),
        ("recurrent_weight", C.c_void_p),
        ("input_weight", C.c_void_p),
        ("output_neurons", C.c_void_p),
        ("context_slots", C.c_void_p),
    ]


class LeoB200PackedUpdate(C.Structure):
    _fields_ = [
        ("threshold_indices", C.c_void_p),
        ("threshold_values", C.c_void_p),
        ("threshold_count", C.c_uint64),
        ("recurrent_indices", C.c_void_p),
        ("recurrent_values", C.c_void_p),
        ("recurrent_count", C.c_uint64),
        ("input_indices", C.c_void_p),
        ("input_values", C.c_void_p),
        ("input_count", C.c_uint64),
        ("output_neurons", C.c_void_p),
        ("output_values_by_neuron", C.c_void_p),
        ("output_count", C.c_uint64),
        ("context_slots", C.c_void_p),
        ("context_keys", C.c_void_p),
        ("context_observations", C.c_void_p),
        ("context_embeddings", C.c_void_p),
        ("context_count", C.c_uint64),
        ("output_bias", C.c_void_p),
        ("context_output_weights", C.c_void_p),
        ("generation", C.c_uint64),
        ("parameter_revision", C.c_uint64),
        ("statistics", LeoB200Statistics),
    ]


FROZEN, PROVISIONAL, TRAINING, VERIFIED = 0, 1, 2, 3
TOPOLOGY_REFERENCE, TOPOLOGY_UNIFORM, TOPOLOGY_ZIPF = 0, 1, 2
BEGIN_DOCUMENT, END_DOCUMENT, SYMBOL_COUNT, OUTPUT_CLASSES = 256, 257, 258, 257


PHASES = ["deliver", "settle", "blocks", "assemble", "surrogate", "eligible", "emit_forward", "learn",
          "plasticity", "inhibit", "settle_hubs"]


class LeoB200PerfStats(C.Structure):
    _fields_ = [
        ("launches", C.c_uint64),
        ("wavefront_launches", C.c_uint64),
        ("wavefront_ms", C.c_double),
        ("story_wavefront_launches", C.c_uint64),
        ("story_wavefront_ms", C.c_double),
        ("phase_cycles", C.c_uint64 * 11),
        ("work_deliver", C.c_uint64),
        ("work_touched", C.c_uint64),
        ("work_eligible", C.c_uint64),
        ("work_destinations", C.c_uint64),
        ("work_active", C.c_uint64),
        ("work_plastic", C.c_uint64),
        ("work_steps", C.c_uint64),
        ("story_work_steps", C.c_uint64),
        ("batches", C.c_uint64),
        ("batch_ms", C.c_double),
        ("story_cluster", C.c_uint32),
        ("replay_cluster", C.c_uint32),
        ("story_lane_launches", C.c_uint64 * 5),
        ("whole_gpu_launches", C.c_uint64),
        ("fit_clusters", C.c_int32 * 3),
        ("sm_count", C.c_int32),
        ("collect_ms", C.c_double),
        ("merge_fixed_ms", C.c_double),
        ("merge_context_ms", C.c_double),
        ("replay_ms", C.c_double),
        ("replay_sync_ms", C.c_double),
        ("replay_phase_cycles", C.c_uint64 * 11),
        ("replay_work_steps", C.c_uint64),
        ("replay_work_touched", C.c_uint64),
        ("replay_work_active", C.c_uint64),
        ("replay_work_deliver", C.c_uint64),
        ("replay_work_eligible", C.c_uint64),
        ("work_inhibit", C.c_uint64),
        ("work_winners", C.c_uint64),
    ]
