// TEST INFRASTRUCTURE ONLY -- C entry points over the parity oracle, for the
// pytest suite (ctypes) and bench.py's cpu_baseline leg.  Never linked into or
// called by the product library.
#include <algorithm>
#include <cstring>
#include <string>

#include "../include/leo_b200_types.h"
#include "leo_oracle.hpp"

using namespace leo_oracle;

namespace {
thread_local std::string g_error;
thread_local std::vector<ParameterChanges> g_last_changes;

int fail(const std::exception& e) {
    g_error = e.what();
    return -1;
}

Config from_c(const LeoB200Config& c) {
    Config o;
    const LeoConfig& a = c.abi;
    o.seed = c.host.seed;
    o.neuron_count = a.neuron_count;
    o.block_count = a.block_count;
    o.neurons_per_block = a.neurons_per_block;
    o.branches_per_neuron = a.branches_per_neuron;
    o.excitatory_fraction = c.host.excitatory_fraction;
    o.synapses_per_neuron = a.synapses_per_neuron;
    o.input_fanout = a.input_fanout;
    o.max_active_per_block = a.max_active_per_block;
    o.max_active_global = a.max_active_global;
    o.branch_decay = a.branch_decay;
    o.membrane_decay = a.membrane_decay;
    o.fatigue_decay = a.fatigue_decay;
    o.fatigue_gain = a.fatigue_gain;
    o.refractory_ticks = a.refractory_ticks;
    o.target_activity = a.target_activity;
    o.threshold_homeostasis_rate = a.threshold_homeostasis_rate;
    o.population_inhibition_rate = a.population_inhibition_rate;
    o.population_inhibition_max = a.population_inhibition_max;
    o.adaptation_fast_decay = a.adaptation_fast_decay;
    o.adaptation_medium_decay = a.adaptation_medium_decay;
    o.adaptation_slow_decay = a.adaptation_slow_decay;
    o.adaptation_fast_gain = a.adaptation_fast_gain;
    o.adaptation_medium_gain = a.adaptation_medium_gain;
    o.adaptation_slow_gain = a.adaptation_slow_gain;
    o.membrane_reset_fraction = a.membrane_reset_fraction;
    o.output_learning_rate = a.output_learning_rate;
    o.recurrent_learning_rate = a.recurrent_learning_rate;
    o.inhibitory_learning_rate = a.inhibitory_learning_rate;
    o.eligibility_decay = a.eligibility_decay;
    o.eligibility_epsilon = a.eligibility_epsilon;
    o.surrogate_width = a.surrogate_width;
    o.surrogate_gain = a.surrogate_gain;
    o.max_update = a.max_update;
    o.weight_min = a.weight_min;
    o.weight_max = a.weight_max;
    o.provisional_strength = c.host.provisional_strength;
    o.training_strength = c.host.training_strength;
    o.verified_strength = c.host.verified_strength;
    o.plasticity_window = c.host.plasticity_window;
    o.end_document_weight = c.host.end_document_weight;
    o.max_order = a.context_max_order;
    o.embedding_dim = a.context_embedding_dim;
    o.slots_per_order = a.context_slots_per_order;
    o.probe_limit = a.context_probe_limit;
    o.context_learning_rate = a.context_learning_rate;
    o.confidence_observations = a.context_confidence_observations;
    o.dropout_rate = c.host.context_dropout_rate;
    o.replay_fraction = c.host.replay_fraction;
    o.segment_bytes = c.host.replay_segment_bytes;
    return o;
}

template <typename T>
void copy_in(std::vector<T>& dst, const T* src, size_t n) {
    dst.assign(src, src + n);
}

void stats_to_c(const Statistics& s, LeoB200Statistics& o) {
    o.processed_bytes = s.processed_bytes;
    o.processed_stories = s.processed_stories;
    o.training_loss_sum = s.training_loss_sum;
    o.training_targets = s.training_targets;
    o.active_neurons_sum = s.active_neurons_sum;
    o.active_neurons_peak = s.active_neurons_peak;
    o.synaptic_events = s.synaptic_events;
    o.numerical_rejections = s.numerical_rejections;
    o.persistent_ticks = s.persistent_ticks;
}
void stats_from_c(const LeoB200Statistics& o, Statistics& s) {
    s.processed_bytes = o.processed_bytes;
    s.processed_stories = o.processed_stories;
    s.training_loss_sum = o.training_loss_sum;
    s.training_targets = o.training_targets;
    s.active_neurons_sum = o.active_neurons_sum;
    s.active_neurons_peak = o.active_neurons_peak;
    s.synaptic_events = o.synaptic_events;
    s.numerical_rejections = o.numerical_rejections;
    s.persistent_ticks = o.persistent_ticks;
}
}  // namespace

extern "C" {

const char* leo_oracle_last_error(void) { return g_error.c_str(); }

int leo_oracle_config_validate(const LeoB200Config* c) {
    try {
        from_c(*c).validate();
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

void* leo_oracle_model_initialize(const LeoB200Config* c, int topology) {
    try {
        return new Model(Model::initialize(from_c(*c), topology));
    } catch (const std::exception& e) {
        fail(e);
        return nullptr;
    }
}

void* leo_oracle_model_from_host(const LeoB200HostModel* h) {
    try {
        Model* m = new Model();
        m->config = from_c(h->config);
        size_t n = m->config.neuron_count, s = m->config.synapses_per_neuron, f = m->config.input_fanout;
        size_t d = m->config.embedding_dim, ctx = m->config.max_order * m->config.slots_per_order;
        m->generation = h->generation;
        m->parameter_revision = h->parameter_revision;
        stats_from_c(h->statistics, m->statistics);
        copy_in(m->threshold, h->threshold, n);
        copy_in(m->excitability, h->excitability, n);
        copy_in(m->neuron_type, h->neuron_type, n);
        m->capacity_per_neuron = s;
        copy_in(m->recurrent_target, h->recurrent_target, n * s);
        copy_in(m->recurrent_branch, h->recurrent_branch, n * s);
        copy_in(m->recurrent_delay, h->recurrent_delay, n * s);
        copy_in(m->recurrent_weight, h->recurrent_weight, n * s);
        m->input_fanout = f;
        copy_in(m->input_targets, h->input_target, SYMBOL_COUNT * f);
        copy_in(m->input_branches, h->input_branch, SYMBOL_COUNT * f);
        copy_in(m->input_weights, h->input_weight, SYMBOL_COUNT * f);
        copy_in(m->output_weights, h->output_weight, OUTPUT_CLASSES * n);
        copy_in(m->output_bias, h->output_bias, OUTPUT_CLASSES);
        copy_in(m->context_keys, h->context_keys, ctx);
        copy_in(m->context_embeddings, h->context_embeddings, ctx * d);
        copy_in(m->context_observations, h->context_observations, ctx);
        copy_in(m->context_output_weights, h->context_output_weight, OUTPUT_CLASSES * d);
        return m;
    } catch (const std::exception& e) {
        fail(e);
        return nullptr;
    }
}

void leo_oracle_model_free(void* m) { delete (Model*)m; }
void* leo_oracle_model_clone(void* m) { return new Model(*(Model*)m); }

// Points `out` at the model's own arrays (valid until the model changes size
// or is freed) and copies the scalar fields.  `out->config` is left unchanged.
int leo_oracle_model_view(void* mp, LeoB200HostModel* out) {
    Model& m = *(Model*)mp;
    out->generation = m.generation;
    out->parameter_revision = m.parameter_revision;
    stats_to_c(m.statistics, out->statistics);
    out->threshold = m.threshold.data();
    out->excitability = m.excitability.data();
    out->neuron_type = m.neuron_type.data();
    out->recurrent_target = m.recurrent_target.data();
    out->recurrent_branch = m.recurrent_branch.data();
    out->recurrent_delay = m.recurrent_delay.data();
    out->recurrent_weight = m.recurrent_weight.data();
    out->input_target = m.input_targets.data();
    out->input_branch = m.input_branches.data();
    out->input_weight = m.input_weights.data();
    out->output_weight = m.output_weights.data();
    out->output_bias = m.output_bias.data();
    out->context_keys = m.context_keys.data();
    out->context_embeddings = m.context_embeddings.data();
    out->context_observations = m.context_observations.data();
    out->context_output_weight = m.context_output_weights.data();
    return 0;
}

int leo_oracle_model_set_scalars(void* mp, uint64_t generation, uint64_t revision, const LeoB200Statistics* s) {
    Model& m = *(Model*)mp;
    m.generation = generation;
    m.parameter_revision = revision;
    stats_from_c(*s, m.statistics);
    return 0;
}

int leo_oracle_model_validate(void* mp) {
    try {
        ((Model*)mp)->validate();
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

void leo_oracle_training_state_hash(void* mp, uint8_t out[32]) { training_state_hash(*(Model*)mp, out); }
void leo_oracle_model_state_hash(void* mp, uint8_t out[32]) { model_state_hash(*(Model*)mp, out); }
void leo_oracle_sha256(const uint8_t* data, size_t len, uint8_t out[32]) { sha256(data, len, out); }

int leo_oracle_resolve_context_slot(void* mp, size_t order, uint64_t key, int allocate, int64_t* slot,
                                    uint64_t* probes) {
    try {
        long s;
        size_t p;
        ((Model*)mp)->resolve_context_slot(order, key, allocate != 0, &s, &p);
        *slot = s;
        *probes = p;
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// ------------------------------------------------------------------ runtime
void* leo_oracle_runtime_new(void* mp) {
    try {
        return new Runtime(*(Model*)mp);
    } catch (const std::exception& e) {
        fail(e);
        return nullptr;
    }
}
void leo_oracle_runtime_free(void* rt) { delete (Runtime*)rt; }
void* leo_oracle_runtime_model(void* rt) { return &((Runtime*)rt)->model; }
void leo_oracle_runtime_model_changed(void* rt) { ((Runtime*)rt)->model_changed(); }
void leo_oracle_runtime_begin_document(void* rt) { ((Runtime*)rt)->begin_document(); }
void leo_oracle_runtime_finish_document(void* rt) { ((Runtime*)rt)->finish_document(); }
void leo_oracle_runtime_reset(void* rt) { ((Runtime*)rt)->reset_transient_state(); }
void leo_oracle_runtime_enable_tracking(void* rt) { ((Runtime*)rt)->enable_parameter_tracking(); }
uint64_t leo_oracle_runtime_tick(void* rt) { return ((Runtime*)rt)->current_tick; }
void leo_oracle_runtime_set_tick(void* rt, uint64_t t) { ((Runtime*)rt)->current_tick = t; }

int leo_oracle_runtime_step(void* rtp, uint32_t symbol, int64_t target, int permission, LeoB200StepMetrics* out) {
    try {
        Runtime& rt = *(Runtime*)rtp;
        StepMetrics m = rt.step(symbol, (long)target, (Permission)permission);
        if (out) {
            std::memset(out, 0, sizeof(*out));
            out->loss = m.has_loss ? m.loss : __builtin_nanf("");
            out->predicted_symbol = m.predicted_symbol;
            out->active_neurons = (uint32_t)m.active_neurons;
            out->emitted_events = (uint32_t)m.emitted_events;
            out->suprathreshold_neurons = (uint32_t)m.suprathreshold_neurons;
            out->block_selected_neurons = (uint32_t)m.block_selected_neurons;
            out->global_cap_clipped_neurons = (uint32_t)m.global_cap_clipped_neurons;
            out->population_inhibition = m.population_inhibition;
            out->context_cells = (uint32_t)m.context_cells;
            out->context_probes = (uint32_t)m.context_probes;
            out->context_applied = m.context_applied ? 1 : 0;
            out->context_loss_gain = m.context_loss_gain;
            out->output_madds = m.output_madds;
            out->eligible_recurrent_synapses = m.eligible_recurrent_synapses;
            out->eligible_input_synapses = m.eligible_input_synapses;
            out->mean_abs_eligibility = m.mean_abs_eligibility;
        }
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// Exposes one internal runtime array by name (read-only use by tests).
int leo_oracle_runtime_array(void* rtp, const char* name, void** ptr, size_t* elem_size, size_t* count) {
    Runtime& r = *(Runtime*)rtp;
    std::string k(name);
#define EXPOSE(label, vec)                        \
    if (k == label) {                             \
        *ptr = (void*)(vec).data();               \
        *elem_size = sizeof((vec)[0]);            \
        *count = (vec).size();                    \
        return 0;                                 \
    }
    EXPOSE("membrane", r.membrane)
    EXPOSE("activation", r.activation)
    EXPOSE("fatigue", r.fatigue)
    EXPOSE("refractory_until", r.refractory_until)
    EXPOSE("branches", r.branches)
    EXPOSE("touched", r.touched)
    EXPOSE("active", r.active)
    EXPOSE("selection_surrogate", r.selection_surrogate)
    EXPOSE("branch_last_tick", r.branch_last_tick)
    EXPOSE("neuron_last_tick", r.neuron_last_tick)
    EXPOSE("adaptation_fast", r.adaptation_state[0])
    EXPOSE("adaptation_medium", r.adaptation_state[1])
    EXPOSE("adaptation_slow", r.adaptation_state[2])
    EXPOSE("rec_branch_sensitivity", r.rec_branch_sens)
    EXPOSE("rec_membrane_sensitivity", r.rec_membrane_sens)
    EXPOSE("rec_fatigue_sensitivity", r.rec_fatigue_sens)
    EXPOSE("rec_adaptation_fast_sensitivity", r.rec_adapt_sens[0])
    EXPOSE("rec_adaptation_medium_sensitivity", r.rec_adapt_sens[1])
    EXPOSE("rec_adaptation_slow_sensitivity", r.rec_adapt_sens[2])
    EXPOSE("rec_eligibility", r.eligibility)
    EXPOSE("rec_last_tick", r.eligibility_last_tick)
    EXPOSE("eligible_recurrent_slots", r.eligible_recurrent_slots)
    EXPOSE("input_branch_sensitivity", r.in_branch_sens)
    EXPOSE("input_membrane_sensitivity", r.in_membrane_sens)
    EXPOSE("input_fatigue_sensitivity", r.in_fatigue_sens)
    EXPOSE("input_adaptation_fast_sensitivity", r.in_adapt_sens[0])
    EXPOSE("input_adaptation_medium_sensitivity", r.in_adapt_sens[1])
    EXPOSE("input_adaptation_slow_sensitivity", r.in_adapt_sens[2])
    EXPOSE("input_eligibility", r.input_eligibility)
    EXPOSE("input_last_tick", r.input_eligibility_last_tick)
    EXPOSE("eligible_input_slots", r.eligible_input_slots)
    EXPOSE("logits", r.logits)
    EXPOSE("probabilities", r.probabilities)
    EXPOSE("errors", r.errors)
    EXPOSE("learning_signal", r.learning_signal)
    EXPOSE("learning_destinations", r.learning_destinations)
    EXPOSE("block_selection_cutoff", r.block_selection_cutoff)
    EXPOSE("context_history", r.context_history)
    EXPOSE("active_context_slots", r.active_context_slots)
    EXPOSE("active_context_scales", r.active_context_scales)
    EXPOSE("context_latent", r.context_latent)
    EXPOSE("changed_threshold", r.changed_threshold)
    EXPOSE("changed_recurrent_weight", r.changed_recurrent_weight)
    EXPOSE("changed_input_weight", r.changed_input_weight)
    EXPOSE("changed_output_neurons", r.changed_output_neurons)
    EXPOSE("changed_context_slots", r.changed_context_slots)
#undef EXPOSE
    if (k == "population_inhibition") {
        *ptr = &r.population_inhibition;
        *elem_size = 4;
        *count = 1;
        return 0;
    }
    if (k == "population_selection_cutoff") {
        *ptr = &r.population_selection_cutoff;
        *elem_size = 4;
        *count = 1;
        return 0;
    }
    g_error = "unknown runtime array: " + k;
    return -1;
}

// Runs one logical story batch on the CPU backend (training.rs:1539-1727).
// `rtp` is the canonical runtime; stories are bytes[offsets[i]..offsets[i+1]].
// `out_losses` (optional) receives the initial-pass per-target losses of all
// stories concatenated in story order; `out_ranges` (optional, pairs of u64)
// receives each story's replay ranges and `out_range_counts` their counts.
int leo_oracle_train_story_batch(void* rtp, const uint8_t* bytes, const uint64_t* offsets, size_t stories,
                                 int permission, size_t threads, LeoB200BatchReport* out, float* out_losses,
                                 uint64_t* out_ranges, uint64_t* out_range_counts) {
    try {
        Runtime& rt = *(Runtime*)rtp;
        std::vector<std::vector<uint8_t>> batch(stories);
        uint64_t input_bytes = 0;
        for (size_t i = 0; i < stories; ++i) {
            batch[i].assign(bytes + offsets[i], bytes + offsets[i + 1]);
            input_bytes += batch[i].size();
        }
        BatchReport r = train_story_batch(rt, batch, (Permission)permission, threads);
        if (out) {
            std::memset(out, 0, sizeof(*out));
            out->workers = r.merge.workers;
            out->fixed_parameter_updates = r.merge.fixed_parameter_updates;
            out->context_keys = r.merge.context_keys;
            out->stories = r.stories;
            out->input_bytes = input_bytes;
            out->targets = r.targets;
            out->mean_loss = r.mean_loss;
            out->replay_segments = r.replay.segments;
            out->replay_steps = r.replay.replay_steps;
            out->replay_prefix_steps = r.replay.prefix_steps;
        }
        if (out_losses) {
            size_t k = 0;
            for (auto& l : r.losses_by_story)
                for (float v : l) out_losses[k++] = v;
        }
        if (out_ranges && out_range_counts) {
            size_t k = 0;
            for (size_t i = 0; i < r.replay_ranges.size(); ++i) {
                out_range_counts[i] = r.replay_ranges[i].size();
                for (auto& range : r.replay_ranges[i]) {
                    out_ranges[2 * k] = range.start;
                    out_ranges[2 * k + 1] = range.end;
                    ++k;
                }
            }
        }
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// Merge helpers for unit tests of the delta algebra (parallel.rs).
int leo_oracle_mean_of_models(void* master, void* const* trained, size_t count, int sum_instead) {
    try {
        Model& m = *(Model*)master;
        std::vector<SparseModelDelta> deltas;
        for (size_t i = 0; i < count; ++i) deltas.push_back(SparseModelDelta::between(m, *(Model*)trained[i]));
        if (sum_instead)
            apply_sum_deltas(m, deltas);
        else
            apply_mean_deltas(m, deltas);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// One tensor's batch-end sparse mean apply: stories' sorted (index, delta)
// lists in CSR form (offsets has stories + 1 entries).
int leo_oracle_sparse_mean_apply(float* target, size_t length, const uint32_t* indices, const float* deltas,
                                 const uint64_t* offsets, size_t stories, float lo, float hi, size_t* updates) {
    try {
        std::vector<float> t(target, target + length);
        std::vector<std::vector<SparseF32Delta>> lists(stories);
        for (size_t s = 0; s < stories; ++s)
            for (uint64_t j = offsets[s]; j < offsets[s + 1]; ++j) lists[s].push_back({indices[j], deltas[j]});
        *updates = sparse_mean_apply(t, lists, lo, hi);
        std::copy(t.begin(), t.end(), target);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// ---- story deltas (SparseModelDelta, parallel.rs:411-691) in the CSR layout
// of LeoB200StoryDeltas: tensors threshold, recurrent weight, input weight,
// output weight, output bias, context output weight.
void* leo_oracle_story_deltas(void* rtp, const uint8_t* bytes, const uint64_t* offsets, size_t stories, int permission,
                              size_t threads) {
    try {
        Runtime& rt = *(Runtime*)rtp;
        std::vector<std::vector<uint8_t>> batch(stories);
        for (size_t i = 0; i < stories; ++i) batch[i].assign(bytes + offsets[i], bytes + offsets[i + 1]);
        std::vector<DocumentPass> passes;
        auto* out = new std::vector<SparseModelDelta>(
            worker_story_deltas(rt.model, batch, (Permission)permission, threads, passes, &g_last_changes));
        return out;
    } catch (const std::exception& e) {
        fail(e);
        return nullptr;
    }
}

// One delta of the runtime's model against `base`: between_tracked with the
// runtime's parameter changes (tracked != 0) or the full between.
void* leo_oracle_runtime_delta(void* base, void* rtp, int tracked) {
    try {
        Runtime& rt = *(Runtime*)rtp;
        const Model& b = *(Model*)base;
        auto* out = new std::vector<SparseModelDelta>();
        out->push_back(tracked ? SparseModelDelta::between_tracked(b, rt.model, rt.parameter_changes())
                               : SparseModelDelta::between(b, rt.model));
        return out;
    } catch (const std::exception& e) {
        fail(e);
        return nullptr;
    }
}

void leo_oracle_deltas_free(void* h) { delete (std::vector<SparseModelDelta>*)h; }

// The per-story ParameterChanges of the last leo_oracle_story_deltas call on
// this thread: sizes (stories, then per story the five list lengths and the
// dirty bits) and, with `out` not NULL, list l of story s at out[l] in story
// order, each list sorted.
int leo_oracle_last_story_changes(uint64_t* counts, uint32_t* dirty, uint32_t* const* out) {
    const auto& v = g_last_changes;
    for (size_t s = 0; s < v.size(); ++s) {
        const std::vector<size_t>* lists[5] = {&v[s].threshold, &v[s].recurrent_weight, &v[s].input_weight,
                                               &v[s].output_neurons, &v[s].context_slots};
        for (int l = 0; l < 5; ++l) {
            if (counts) counts[s * 5 + l] = lists[l]->size();
        }
        if (dirty) dirty[s] = (v[s].output_bias_dirty ? 1u : 0u) | (v[s].context_output_dirty ? 2u : 0u);
    }
    if (out) {
        for (int l = 0; l < 5; ++l) {
            size_t at = 0;
            for (size_t s = 0; s < v.size(); ++s) {
                const std::vector<size_t>* lists[5] = {&v[s].threshold, &v[s].recurrent_weight, &v[s].input_weight,
                                                       &v[s].output_neurons, &v[s].context_slots};
                std::vector<size_t> sorted(*lists[l]);
                std::sort(sorted.begin(), sorted.end());
                for (size_t x : sorted) out[l][at++] = (uint32_t)x;
            }
        }
    }
    return 0;
}

namespace {
const std::vector<SparseF32Delta>& delta_tensor(const SparseModelDelta& d, int t) {
    switch (t) {
        case 0: return d.threshold;
        case 1: return d.recurrent_weight;
        case 2: return d.input_weight;
        case 3: return d.output_weight;
        case 4: return d.output_bias;
        default: return d.context_output_weight;
    }
}
}  // namespace

int leo_oracle_deltas_sizes(void* h, size_t embedding_dim, LeoB200StoryDeltaSizes* sizes) {
    const auto& v = *(std::vector<SparseModelDelta>*)h;
    std::memset(sizes, 0, sizeof(*sizes));
    sizes->stories = (uint32_t)v.size();
    sizes->embedding_dim = (uint32_t)embedding_dim;
    for (const auto& d : v) {
        if (!d.excitability.empty()) {
            g_error = "excitability deltas have no slot in the story delta layout";
            return -1;
        }
        for (int t = 0; t < LEO_B200_DELTA_TENSORS; ++t) sizes->entries[t] += delta_tensor(d, t).size();
        sizes->context_entries += d.context.size();
    }
    return 0;
}

int leo_oracle_deltas_copy(void* h, size_t embedding_dim, const LeoB200StoryDeltas* out) {
    const auto& v = *(std::vector<SparseModelDelta>*)h;
    for (int t = 0; t < LEO_B200_DELTA_TENSORS; ++t) {
        uint64_t at = 0;
        for (size_t s = 0; s < v.size(); ++s) {
            out->offsets[t][s] = at;
            for (const auto& e : delta_tensor(v[s], t)) {
                out->indices[t][at] = (uint32_t)e.index;
                out->deltas[t][at] = e.delta;
                ++at;
            }
        }
        out->offsets[t][v.size()] = at;
    }
    uint64_t at = 0;
    for (size_t s = 0; s < v.size(); ++s) {
        out->context_offsets[s] = at;
        for (const auto& c : v[s].context) {
            if (c.embedding_delta.size() != embedding_dim) {
                g_error = "context delta embedding has the wrong width";
                return -1;
            }
            out->context_orders[at] = (uint32_t)c.order;
            out->context_keys[at] = c.key;
            out->context_observation_increments[at] = c.observation_increment;
            std::copy(c.embedding_delta.begin(), c.embedding_delta.end(),
                      out->context_embedding_deltas + at * embedding_dim);
            ++at;
        }
        const StatisticsDelta& sd = v[s].statistics;
        LeoB200Statistics& st = out->statistics[s];
        std::memset(&st, 0, sizeof(st));
        st.processed_bytes = sd.processed_bytes;
        st.processed_stories = sd.processed_stories;
        st.training_loss_sum = sd.training_loss_sum;
        st.training_targets = sd.training_targets;
        st.active_neurons_sum = sd.active_neurons_sum;
        st.active_neurons_peak = sd.active_neurons_peak;
        st.synaptic_events = sd.synaptic_events;
        st.numerical_rejections = sd.numerical_rejections;
        st.persistent_ticks = sd.persistent_ticks;
        out->revision_increments[s] = v[s].revision_increment;
    }
    out->context_offsets[v.size()] = at;
    return 0;
}

// apply_mean_deltas / apply_sum_deltas (parallel.rs:694-798) of story deltas
// given in the CSR layout, produced from `model`'s current revision.
int leo_oracle_apply_story_deltas(void* mp, const LeoB200StoryDeltaSizes* sizes, const LeoB200StoryDeltas* in,
                                  int sum_instead, LeoB200BatchReport* merge) {
    try {
        Model& m = *(Model*)mp;
        const size_t n = sizes->stories, d = sizes->embedding_dim;
        std::vector<SparseModelDelta> deltas(n);
        for (size_t s = 0; s < n; ++s) {
            SparseModelDelta& sd = deltas[s];
            sd.config_fingerprint = m.config.fingerprint();
            sd.base_revision = m.parameter_revision;
            sd.revision_increment = in->revision_increments[s];
            for (int t = 0; t < LEO_B200_DELTA_TENSORS; ++t) {
                auto& dst = const_cast<std::vector<SparseF32Delta>&>(delta_tensor(sd, t));
                for (uint64_t j = in->offsets[t][s]; j < in->offsets[t][s + 1]; ++j)
                    dst.push_back({in->indices[t][j], in->deltas[t][j]});
            }
            for (uint64_t j = in->context_offsets[s]; j < in->context_offsets[s + 1]; ++j) {
                ContextKeyDelta c;
                c.order = in->context_orders[j];
                c.key = in->context_keys[j];
                c.observation_increment = in->context_observation_increments[j];
                c.embedding_delta.assign(in->context_embedding_deltas + j * d, in->context_embedding_deltas + (j + 1) * d);
                sd.context.push_back(std::move(c));
            }
            const LeoB200Statistics& st = in->statistics[s];
            sd.statistics.processed_bytes = st.processed_bytes;
            sd.statistics.processed_stories = st.processed_stories;
            sd.statistics.training_loss_sum = st.training_loss_sum;
            sd.statistics.training_targets = st.training_targets;
            sd.statistics.active_neurons_sum = st.active_neurons_sum;
            sd.statistics.active_neurons_peak = st.active_neurons_peak;
            sd.statistics.synaptic_events = st.synaptic_events;
            sd.statistics.numerical_rejections = st.numerical_rejections;
            sd.statistics.persistent_ticks = st.persistent_ticks;
        }
        MergeMetrics mm = sum_instead ? apply_sum_deltas(m, deltas) : apply_mean_deltas(m, deltas);
        if (merge) {
            std::memset(merge, 0, sizeof(*merge));
            merge->workers = mm.workers;
            merge->fixed_parameter_updates = mm.fixed_parameter_updates;
            merge->context_keys = mm.context_keys;
        }
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// Runtime::parameter_changes (runtime.rs:322-333): sizes, then (when `out` is
// not NULL) the indices in the order they were first changed.
int leo_oracle_runtime_parameter_changes(void* rtp, LeoB200ParameterChangeSizes* sizes,
                                         const LeoB200ParameterChanges* out) {
    const ParameterChanges c = ((Runtime*)rtp)->parameter_changes();
    sizes->threshold = c.threshold.size();
    sizes->recurrent_weight = c.recurrent_weight.size();
    sizes->input_weight = c.input_weight.size();
    sizes->output_neurons = c.output_neurons.size();
    sizes->context_slots = c.context_slots.size();
    sizes->output_bias_dirty = c.output_bias_dirty;
    sizes->context_output_dirty = c.context_output_dirty;
    if (out) {
        const std::vector<size_t>* src[5] = {&c.threshold, &c.recurrent_weight, &c.input_weight, &c.output_neurons,
                                             &c.context_slots};
        uint32_t* dst[5] = {out->threshold, out->recurrent_weight, out->input_weight, out->output_neurons,
                            out->context_slots};
        for (int i = 0; i < 5; ++i)
            if (dst[i])
                for (size_t j = 0; j < src[i]->size(); ++j) dst[i][j] = (uint32_t)(*src[i])[j];
    }
    return 0;
}

// One block's selection (select_block): candidates (value > 0 only, as the
// runtime pushes them) in, winners in rank order and the cutoff out (0 when
// at most `keep` are positive).
void leo_oracle_select_block(const float* values, const uint32_t* neurons, size_t count, size_t keep, size_t rotation,
                             size_t neuron_count, uint32_t* winners, float* winner_values, size_t* winner_count,
                             float* cutoff) {
    std::vector<std::pair<size_t, float>> block;
    for (size_t i = 0; i < count; ++i)
        if (values[i] > 0.0f) block.push_back({neurons[i], values[i]});
    float c = 0.0f;
    select_block(block, keep, rotation, neuron_count, &c);
    for (size_t i = 0; i < block.size(); ++i) {
        winners[i] = (uint32_t)block[i].first;
        winner_values[i] = block[i].second;
    }
    *winner_count = block.size();
    *cutoff = c;
}

// The global rank order of the cap (runtime.rs:1014-1030): indices of the
// candidates sorted by selection_better.
void leo_oracle_global_order(const float* values, const uint32_t* neurons, size_t count, size_t rotation,
                             size_t neuron_count, uint32_t* order) {
    std::vector<size_t> idx(count);
    for (size_t i = 0; i < count; ++i) idx[i] = i;
    std::sort(idx.begin(), idx.end(), [&](size_t a, size_t b) {
        return selection_better({neurons[a], values[a]}, {neurons[b], values[b]}, rotation, neuron_count);
    });
    for (size_t i = 0; i < count; ++i) order[i] = (uint32_t)idx[i];
}

int leo_oracle_select_replay_ranges(const float* losses, size_t n, float fraction, size_t segment, uint64_t* out,
                                    size_t cap, size_t* count) {
    std::vector<float> l(losses, losses + n);
    auto r = select_replay_ranges(l, fraction, segment);
    *count = r.size();
    for (size_t i = 0; i < r.size() && i < cap; ++i) {
        out[2 * i] = r[i].start;
        out[2 * i + 1] = r[i].end;
    }
    return 0;
}

// shuffled_story_order (crates/leo-cli/src/training/dataset.rs:9-13): the
// identity order shuffled by SplitMix64(seed + pass + 1), wrapping.
void leo_oracle_shuffled_story_order(uint64_t count, uint64_t seed, uint64_t pass, uint64_t* out) {
    std::vector<uint64_t> order(count);
    for (uint64_t i = 0; i < count; ++i) order[i] = i;
    SplitMix64 rng(seed + pass + 1);
    rng.shuffle(order);
    std::copy(order.begin(), order.end(), out);
}

}  // extern "C"
