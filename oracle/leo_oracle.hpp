// TEST INFRASTRUCTURE ONLY.  This is the parity oracle: a CPU restatement of
// the reference's CPU backend (crates/leo-core/src/{runtime,learning,model,rng,
// config,parallel}.rs and the CPU branch of crates/leo-cli/src/training.rs).
// Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may use
// it, and only as the checker or the timed CPU baseline -- never as the product.
//
// Parity pin: the reference is Rust and no Rust toolchain exists here, so the
// reference itself cannot be run.  The restatement is pinned by the reference's
// own known-answer tests (ported in oracle/known_answer_tests.cpp); the
// reference ships no value-level golden vectors for this path.
//
// FP32 semantics follow Rust: no FMA contraction (build with
// -ffp-contract=off), left-to-right evaluation, f32::exp/ln from the platform
// libm (glibc expf/logf), powi as right-to-left binary exponentiation.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace leo_oracle {

constexpr uint32_t BYTE_SYMBOLS = 256;
constexpr uint32_t BEGIN_DOCUMENT = 256;
constexpr uint32_t END_DOCUMENT = 257;
constexpr size_t SYMBOL_COUNT = 258;
constexpr size_t OUTPUT_CLASSES = 257;
constexpr size_t END_OUTPUT_INDEX = 256;

constexpr uint8_t BRANCH_EXCITATORY = 0;
constexpr uint8_t BRANCH_INHIBITORY = 1;
constexpr uint8_t BRANCH_TEMPORAL = 2;
constexpr uint8_t BRANCH_CONTEXT_GATE = 3;

// crates/leo-core/src/learning.rs:6-73
float analog_rank_surrogate(float margin, float cutoff, bool selected, float width, float gain);
float branch_jacobian(uint8_t branch, float exc, float temporal, float gate_acc);
float bounded_delta(float v, float maximum);
float inhibitory_homeostasis_delta(float src_act, float tgt_act, float desired, float lr, float strength,
                                   float maximum);

struct LeoError : std::runtime_error {
    enum Kind { Internal, Configuration, Numerical };
    Kind kind;
    LeoError(Kind k, const std::string& m) : std::runtime_error(m), kind(k) {}
};

// crates/leo-core/src/config.rs:8-156 (fields the path reads).
struct Config {
    // model
    uint64_t seed = 1337;
    size_t neuron_count = 32768, block_count = 128, neurons_per_block = 256;
    size_t branches_per_neuron = 4;
    float excitatory_fraction = 0.80f;
    size_t synapses_per_neuron = 48, input_fanout = 128;
    size_t max_active_per_block = 8, max_active_global = 1024;
    // dynamics
    float branch_decay = 0.85f, membrane_decay = 0.90f, fatigue_decay = 0.97f;
    float fatigue_gain = 0.02f;
    uint64_t refractory_ticks = 1;
    float target_activity = 0.02f, threshold_homeostasis_rate = 0.0001f;
    float population_inhibition_rate = 0.05f, population_inhibition_max = 2.0f;
    float adaptation_fast_decay = 0.95f, adaptation_medium_decay = 0.99f, adaptation_slow_decay = 0.999f;
    float adaptation_fast_gain = 0.005f, adaptation_medium_gain = 0.001f, adaptation_slow_gain = 0.0002f;
    float membrane_reset_fraction = 0.10f;
    // learning
    float output_learning_rate = 0.001f, recurrent_learning_rate = 0.0002f;
    float inhibitory_learning_rate = 0.00002f, eligibility_decay = 0.95f;
    float eligibility_epsilon = 1.0e-5f, surrogate_width = 0.25f, surrogate_gain = 0.10f;
    float max_update = 0.01f, weight_min = -1.0f, weight_max = 1.0f;
    float provisional_strength = 0.20f, training_strength = 1.0f, verified_strength = 1.0f;
    size_t plasticity_window = 1;
    float end_document_weight = 4.0f;
    // context
    size_t max_order = 8, embedding_dim = 32, slots_per_order = 8192, probe_limit = 4;
    float context_learning_rate = 0.05f;
    uint32_t confidence_observations = 4;
    float dropout_rate = 0.5f;
    // replay
    float replay_fraction = 0.30f;
    size_t segment_bytes = 64;

    void validate() const;  // config.rs:250-519 (fields above)
    void adaptation_decays(float out[3]) const {
        out[0] = adaptation_fast_decay; out[1] = adaptation_medium_decay; out[2] = adaptation_slow_decay;
    }
    void adaptation_gains(float out[3]) const {
        out[0] = adaptation_fast_gain; out[1] = adaptation_medium_gain; out[2] = adaptation_slow_gain;
    }
    // config.rs:137-145
    void plasticity_step(size_t phase, bool end_document, float* scale, size_t* next) const;
    // A stable digest of the config (stands in for config_fingerprint, parallel.rs:1347-1349).
    uint64_t fingerprint() const;
};

// crates/leo-core/src/metrics.rs:3-15
struct Statistics {
    uint64_t processed_bytes = 0, processed_stories = 0;
    double training_loss_sum = 0.0;
    uint64_t training_targets = 0, active_neurons_sum = 0, active_neurons_peak = 0;
    uint64_t synaptic_events = 0, numerical_rejections = 0, persistent_ticks = 0;
};

// crates/leo-core/src/rng.rs:1-43
struct SplitMix64 {
    uint64_t state;
    explicit SplitMix64(uint64_t seed) : state(seed) {}
    uint64_t next_u64();
    float next_f32();
    size_t range_usize(size_t upper_exclusive);
    float range_f32(float low, float high);
    template <typename T> void shuffle(std::vector<T>& v) {
        for (size_t index = v.size(); index-- > 1;) {
            size_t other = range_usize(index + 1);
            std::swap(v[index], v[other]);
        }
    }
};

// crates/leo-core/src/model.rs:65-76
struct Model {
    Config config;
    uint64_t generation = 0, parameter_revision = 0;
    std::vector<float> threshold, excitability;
    std::vector<uint8_t> neuron_type;
    size_t capacity_per_neuron = 0;
    std::vector<uint32_t> recurrent_target;
    std::vector<uint8_t> recurrent_branch, recurrent_delay;
    std::vector<float> recurrent_weight;
    size_t input_fanout = 0;
    std::vector<uint32_t> input_targets;
    std::vector<uint8_t> input_branches;
    std::vector<float> input_weights;
    std::vector<float> output_weights;  // [257][N]
    std::vector<float> output_bias;     // [257]
    std::vector<uint64_t> context_keys;
    std::vector<float> context_embeddings;
    std::vector<uint32_t> context_observations;
    std::vector<float> context_output_weights;  // [257][D]
    Statistics statistics;

    size_t neuron_count() const { return config.neuron_count; }
    size_t slot_start(size_t neuron) const { return neuron * capacity_per_neuron; }
    // model.rs:79-158; topology 0 = reference initialize_recurrent, 1 = uniform, 2 = zipf.
    static Model initialize(const Config& config, int topology = 0);
    // model.rs:173-221
    void resolve_context_slot(size_t order, uint64_t key, bool allocate, long* slot, size_t* probes);
    void validate() const;  // model.rs:223-396
};

// crates/leo-core/src/runtime.rs:38-46
struct ParameterChanges {
    std::vector<size_t> threshold, recurrent_weight, input_weight, output_neurons, context_slots;
    bool output_bias_dirty = false, context_output_dirty = false;
};

enum class Permission { Frozen = 0, Provisional = 1, Training = 2, Verified = 3 };
float permission_strength(Permission p, const Config& c);  // permission.rs:24-31

// crates/leo-core/src/metrics.rs:39-66
struct StepMetrics {
    bool has_loss = false;
    float loss = 0.0f;
    uint32_t predicted_symbol = 0;
    size_t active_neurons = 0, emitted_events = 0, suprathreshold_neurons = 0;
    size_t block_selected_neurons = 0, global_cap_clipped_neurons = 0;
    float population_inhibition = 0.0f;
    size_t context_cells = 0, context_probes = 0;
    bool context_applied = false;
    float context_loss_gain = 0.0f;
    size_t output_madds = 0, eligible_recurrent_synapses = 0, eligible_input_synapses = 0;
    float mean_abs_eligibility = 0.0f;
};

// crates/leo-core/src/runtime.rs:15-22
struct Event {
    uint32_t target_neuron;
    uint8_t target_branch;
    float value;
    uint32_t synapse_slot;
    float presynaptic_activation;
};

// crates/leo-core/src/runtime.rs:112-186.  Members are public so the ported
// known-answer tests can inspect the same internals the Rust tests do.
struct Runtime {
    Model model;
    // WorkerState runtime.rs:48-66
    std::vector<float> membrane, activation, fatigue;
    std::vector<uint64_t> refractory_until;
    std::vector<float> branches;
    std::vector<std::vector<Event>> delay_ring;
    std::vector<Event> due_events;
    uint64_t current_tick = 0;
    size_t plasticity_phase = 0;
    std::vector<size_t> touched;
    std::vector<uint8_t> touched_mark;
    std::vector<size_t> active, previous_active;
    std::vector<uint8_t> selected_mark;
    std::vector<float> selection_surrogate;
    std::vector<uint64_t> branch_last_tick, neuron_last_tick;
    std::vector<float> adaptation_state[3];
    std::vector<float> rec_branch_sens, rec_membrane_sens, rec_fatigue_sens, rec_adapt_sens[3];
    std::vector<float> eligibility;
    std::vector<uint64_t> eligibility_last_tick;
    std::vector<size_t> eligible_recurrent_slots;
    std::vector<uint8_t> eligible_recurrent_mark;
    std::vector<float> in_branch_sens, in_membrane_sens, in_fatigue_sens, in_adapt_sens[3];
    std::vector<float> input_eligibility;
    std::vector<uint64_t> input_eligibility_last_tick;
    std::vector<size_t> eligible_input_slots;
    std::vector<uint8_t> eligible_input_mark;
    std::vector<float> logits, probabilities, errors, learning_signal;
    std::vector<size_t> learning_destinations;
    std::vector<uint8_t> learning_destination_mark;
    std::vector<float> output_weights_by_neuron;  // [N][257]
    bool output_cache_dirty = false;
    std::vector<std::vector<std::pair<size_t, float>>> block_candidates;
    std::vector<float> block_selection_cutoff;
    float population_selection_cutoff = 0.0f;
    std::vector<uint32_t> context_history;
    std::vector<size_t> active_context_slots;
    std::vector<float> active_context_scales;
    std::vector<float> context_latent, context_latent_gradient;
    size_t active_context_probes = 0;
    bool context_applied_this_step = false;
    float population_inhibition = 0.0f;
    bool track_parameter_changes = false;
    std::vector<size_t> changed_threshold, changed_recurrent_weight, changed_input_weight;
    std::vector<size_t> changed_output_neurons, changed_context_slots;
    std::vector<uint8_t> changed_threshold_mark, changed_recurrent_weight_mark, changed_input_weight_mark;
    std::vector<uint8_t> changed_output_neuron_mark, changed_context_slot_mark;
    bool output_bias_dirty = false, context_output_dirty = false;
    bool persistent_document_activity = false, learning_trace_enabled = false;

    explicit Runtime(Model m);
    void enable_parameter_tracking();
    ParameterChanges parameter_changes() const;
    void model_changed() { output_cache_dirty = true; }
    void begin_document() { reset_transient_state(); }
    void finish_document();
    void reset_transient_state();
    StepMetrics step(uint32_t symbol, long target, Permission permission);

    // internals (runtime.rs:537-1623)
    void ensure_output_weight_cache();
    void start_tick();
    void mark_touched(size_t neuron);
    void bring_neuron_to_current_tick(size_t neuron);
    void deliver_due_events();
    void inject_symbol(uint32_t symbol);
    void activate_context(uint32_t symbol, bool allocate, bool enabled);
    uint64_t context_key(size_t order) const;
    long resolve_context_slot(size_t order, uint64_t key, bool allocate);
    void add_to_branch(size_t neuron, uint8_t branch, float value);
    void activate_recurrent_trace(size_t slot, float a);
    void activate_input_trace(size_t slot, float a);
    void advance_recurrent_trace(size_t slot);
    void advance_input_trace(size_t slot);
    float destination_branch_jacobian(size_t destination, uint8_t branch) const;
    bool neuron_is_refractory(size_t neuron) const { return refractory_until[neuron] > current_tick; }
    void cache_selection_surrogates();
    void update_forward_eligibilities();
    bool update_recurrent_forward_slot(size_t slot, float epsilon);
    bool update_input_forward_slot(size_t slot, float epsilon);
    void apply_post_activation_dynamics();
    struct SelectionMetrics { size_t suprathreshold = 0, block_selected = 0, clipped = 0; };
    SelectionMetrics select_active_neurons();
    void update_population_inhibition(size_t active_neurons);
    size_t emit_recurrent_events();
    bool compute_output_probabilities(long target_index, float* neural_loss);
    float loss_from_logits(size_t target) const;
    void normalize_probabilities();
    size_t argmax_probability() const;
    struct LearningMetrics { double abs_sum = 0.0; size_t count = 0; };
    LearningMetrics apply_learning(size_t target_output_index, float strength, float target_weight);
    void update_context_projection(float strength);
    void add_learning_destination(size_t destination);
    void update_recurrent_synapses(float strength, LearningMetrics& m);
    void update_input_synapses(float strength, LearningMetrics& m);
    void apply_inhibitory_homeostasis(float strength);
    void update_homeostasis(size_t active_neurons);
    void update_statistics(uint32_t symbol, bool has_loss, float loss, size_t emitted);
    static void mark_changed(size_t index, std::vector<uint8_t>& marks, std::vector<size_t>& list);
};

// ---- selection order, crates/leo-core/src/runtime.rs:964-1030 ---------------
bool selection_better(const std::pair<size_t, float>& l, const std::pair<size_t, float>& r, size_t rotation,
                      size_t n_count);
void select_block(std::vector<std::pair<size_t, float>>& block, size_t limit, size_t rotation, size_t n_count,
                  float* cutoff);

// ---- delta algebra, crates/leo-core/src/parallel.rs -------------------------
struct SparseF32Delta { size_t index; float delta; };
struct ContextKeyDelta {
    size_t order;
    uint64_t key;
    std::vector<float> embedding_delta;
    uint32_t observation_increment;
};
struct StatisticsDelta {
    uint64_t processed_bytes = 0, processed_stories = 0;
    double training_loss_sum = 0.0;
    uint64_t training_targets = 0, active_neurons_sum = 0, active_neurons_peak = 0;
    uint64_t synaptic_events = 0, numerical_rejections = 0, persistent_ticks = 0;
};
struct SparseModelDelta {
    uint64_t config_fingerprint = 0, base_revision = 0, revision_increment = 0;
    std::vector<SparseF32Delta> threshold, excitability, recurrent_weight, input_weight;
    std::vector<SparseF32Delta> output_weight, output_bias, context_output_weight;
    std::vector<ContextKeyDelta> context;
    StatisticsDelta statistics;
    static SparseModelDelta between(const Model& base, const Model& trained);
    static SparseModelDelta between_tracked(const Model& base, const Model& trained, const ParameterChanges& c);
    void canonicalize_order();
};
struct MergeMetrics { size_t workers = 0, fixed_parameter_updates = 0, context_keys = 0; };
MergeMetrics apply_mean_deltas(Model& master, const std::vector<SparseModelDelta>& deltas);
MergeMetrics apply_sum_deltas(Model& master, const std::vector<SparseModelDelta>& deltas);
// apply_sparse_scaled (parallel.rs:975-1022) of one tensor with divisor = stories,
// then the clamp projection of parallel.rs:1226-1233; returns the union size.
size_t sparse_mean_apply(std::vector<float>& target, const std::vector<std::vector<SparseF32Delta>>& stories, float lo,
                         float hi);
StatisticsDelta statistics_delta(const Statistics& before, const Statistics& after);

// ---- training policy, crates/leo-cli/src/training.rs -------------------------
struct Range { size_t start, end; };
std::vector<Range> select_replay_ranges(const std::vector<float>& losses, float fraction, size_t segment_targets);

struct DocumentPass {
    double mean_loss = 0.0;
    std::vector<float> losses;
    uint64_t steps = 0, active_neurons_sum = 0, active_neurons_peak = 0, emitted_events = 0;
    uint64_t context_applied_steps = 0;
};
DocumentPass train_document_pass(Runtime& runtime, const uint8_t* story, size_t len, Permission p);

struct ReplayReport { size_t segments = 0; uint64_t replay_steps = 0, prefix_steps = 0; };
// training.rs:1848-1955 (one range), executed on `canonical`.
void replay_target_range(Runtime& canonical, const uint8_t* story, size_t len, Range range,
                         Permission p, bool cleanup_after, uint64_t* prefix_steps, uint64_t* target_steps);
ReplayReport apply_replay_policy(Runtime& canonical, const uint8_t* story, size_t len,
                                 const std::vector<float>& losses, Permission p);

struct BatchReport {
    double mean_loss = 0.0;
    size_t targets = 0, stories = 0;
    ReplayReport replay;
    MergeMetrics merge;
    std::vector<std::vector<float>> losses_by_story;
    std::vector<std::vector<Range>> replay_ranges;
};
// The CPU branch's workers (training.rs:1667-1695): every story forked from
// `base` with parameter tracking, one document pass, its between_tracked delta
// (parallel.rs:385-454).  `passes` receives each story's pass.
std::vector<SparseModelDelta> worker_story_deltas(const Model& base, const std::vector<std::vector<uint8_t>>& stories,
                                                  Permission p, size_t max_threads, std::vector<DocumentPass>& passes,
                                                  std::vector<ParameterChanges>* changes = nullptr);
// training.rs:1539-1727, CPU branch (stories.len() > 1) and the single-story branch.
// `canonical` is the canonical CPU runtime (its tick persists across batches).
BatchReport train_story_batch(Runtime& canonical, const std::vector<std::vector<uint8_t>>& stories,
                              Permission p, size_t max_threads);

// ---- identity ----------------------------------------------------------------
void sha256(const uint8_t* data, size_t len, uint8_t out[32]);
struct Sha256 {
    uint32_t h[8];
    uint8_t buf[64];
    uint64_t total = 0;
    size_t fill = 0;
    Sha256();
    void update(const void* data, size_t len);
    void finalize(uint8_t out[32]);
    void block(const uint8_t* p);
};
void model_state_hash(const Model& m, uint8_t out[32]);     // crates/leo-cli/src/main.rs:1151-1185
void training_state_hash(const Model& m, uint8_t out[32]);  // crates/leo-cli/src/main.rs:1187-1202

}  // namespace leo_oracle
