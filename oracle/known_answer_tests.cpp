// TEST INFRASTRUCTURE ONLY -- the reference's own known-answer tests for this
// path, restated against the oracle.  Each test names the reference test it
// ports.  Run by tests/test_oracle_known_answers.py; exit status 0 = all pass.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <set>
#include <string>
#include <vector>

#include "leo_oracle.hpp"

using namespace leo_oracle;

static int g_failures = 0;
static std::string g_current;

#define CHECK(cond)                                                                    \
    do {                                                                               \
        if (!(cond)) {                                                                 \
            std::printf("FAIL %s: %s (line %d)\n", g_current.c_str(), #cond, __LINE__); \
            ++g_failures;                                                              \
            return;                                                                    \
        }                                                                              \
    } while (0)

static void run(const char* name, const std::function<void()>& fn) {
    g_current = name;
    int before = g_failures;
    try {
        fn();
    } catch (const std::exception& e) {
        std::printf("FAIL %s: exception %s\n", name, e.what());
        ++g_failures;
        return;
    }
    if (g_failures == before) std::printf("PASS %s\n", name);
}

// configs/test.toml
static Config test_config() {
    Config c;
    c.seed = 1337;
    c.neuron_count = 128; c.block_count = 8; c.neurons_per_block = 16; c.excitatory_fraction = 0.8f;
    c.synapses_per_neuron = 8; c.input_fanout = 8; c.max_active_per_block = 2; c.max_active_global = 8;
    c.branch_decay = 0.85f; c.membrane_decay = 0.90f; c.fatigue_decay = 0.97f; c.fatigue_gain = 0.02f;
    c.refractory_ticks = 1; c.target_activity = 0.04f; c.threshold_homeostasis_rate = 0.0001f;
    c.population_inhibition_rate = 0.05f; c.population_inhibition_max = 2.0f;
    c.adaptation_fast_decay = 0.95f; c.adaptation_medium_decay = 0.99f; c.adaptation_slow_decay = 0.999f;
    c.adaptation_fast_gain = 0.005f; c.adaptation_medium_gain = 0.001f; c.adaptation_slow_gain = 0.0002f;
    c.membrane_reset_fraction = 0.10f; c.output_learning_rate = 0.002f; c.recurrent_learning_rate = 0.0005f;
    c.inhibitory_learning_rate = 0.00005f; c.eligibility_decay = 0.95f; c.eligibility_epsilon = 0.00001f;
    c.surrogate_width = 0.25f; c.surrogate_gain = 0.10f; c.max_update = 0.01f; c.weight_min = -1.0f;
    c.weight_max = 1.0f; c.provisional_strength = 0.20f; c.training_strength = 1.0f; c.verified_strength = 1.0f;
    c.plasticity_window = 1; c.end_document_weight = 4.0f; c.embedding_dim = 8; c.max_order = 4;
    c.slots_per_order = 128; c.probe_limit = 4; c.context_learning_rate = 0.08f; c.confidence_observations = 2;
    c.dropout_rate = 0.0f; c.replay_fraction = 0.30f; c.segment_bytes = 8;
    c.validate();
    return c;
}

// runtime.rs:1632-1656 integrated_config()
static Config integrated_config() {
    Config c;  // Config::default() (config.rs:158-234)
    c.neuron_count = 8; c.block_count = 1; c.neurons_per_block = 8; c.synapses_per_neuron = 1; c.input_fanout = 1;
    c.max_active_per_block = 8; c.max_active_global = 8; c.fatigue_gain = 1.0e-6f; c.refractory_ticks = 1;
    c.target_activity = 0.5f; c.threshold_homeostasis_rate = 1.0e-8f; c.output_learning_rate = 1.0e-8f;
    c.recurrent_learning_rate = 0.1f; c.inhibitory_learning_rate = 1.0e-8f; c.eligibility_epsilon = 1.0e-7f;
    c.surrogate_width = 0.25f; c.surrogate_gain = 0.1f; c.max_update = 0.1f; c.max_order = 3;
    c.slots_per_order = 1024; c.context_learning_rate = 0.1f; c.confidence_observations = 1; c.dropout_rate = 0.0f;
    c.validate();
    return c;
}

static size_t out_index(uint32_t s) { return s < 256 ? s : END_OUTPUT_INDEX; }

// runtime.rs:1658-1692 causal_model(delay)
static Model causal_model(uint8_t delay) {
    Model m = Model::initialize(integrated_config());
    std::fill(m.threshold.begin(), m.threshold.end(), 0.1f);
    std::fill(m.excitability.begin(), m.excitability.end(), 1.0f);
    std::fill(m.recurrent_weight.begin(), m.recurrent_weight.end(), 0.0f);
    m.neuron_type[0] = 0;
    for (size_t s = m.slot_start(0); s < m.slot_start(0) + m.capacity_per_neuron; ++s) m.recurrent_branch[s] = BRANCH_EXCITATORY;
    std::fill(m.input_weights.begin(), m.input_weights.end(), 0.0f);
    std::fill(m.input_branches.begin(), m.input_branches.end(), BRANCH_EXCITATORY);
    std::fill(m.output_weights.begin(), m.output_weights.end(), 0.0f);
    std::fill(m.output_bias.begin(), m.output_bias.end(), 0.0f);
    m.recurrent_target[0] = 1;
    m.recurrent_branch[0] = BRANCH_EXCITATORY;
    m.recurrent_delay[0] = delay;
    m.recurrent_weight[0] = 0.5f;
    size_t in_slot = (size_t)'A' * m.input_fanout;
    m.input_targets[in_slot] = 0;
    m.input_weights[in_slot] = 1.0f;
    size_t quiet = (size_t)'B' * m.input_fanout;
    m.input_targets[quiet] = 7;
    m.input_weights[quiet] = 0.0f;
    m.output_weights[out_index('Z') * m.neuron_count() + 1] = 1.0f;
    return m;
}

// runtime.rs:1796-1826 recurrent_memory_model()
static Model recurrent_memory_model() {
    Config c = integrated_config();
    c.neuron_count = 64; c.block_count = 1; c.neurons_per_block = 64; c.synapses_per_neuron = 1; c.input_fanout = 1;
    c.max_active_per_block = 64; c.max_active_global = 64; c.target_activity = 0.01f; c.membrane_reset_fraction = 1.0f;
    c.fatigue_gain = 1.0e-6f; c.adaptation_fast_gain = 1.0e-8f; c.adaptation_medium_gain = 1.0e-8f;
    c.adaptation_slow_gain = 1.0e-8f; c.max_order = 8; c.embedding_dim = 8; c.slots_per_order = 64; c.probe_limit = 4;
    c.validate();
    Model m = Model::initialize(c);
    std::fill(m.threshold.begin(), m.threshold.end(), 0.9f);
    std::fill(m.excitability.begin(), m.excitability.end(), 2.0f);
    std::fill(m.recurrent_weight.begin(), m.recurrent_weight.end(), 0.0f);
    std::fill(m.input_weights.begin(), m.input_weights.end(), 0.0f);
    std::fill(m.output_weights.begin(), m.output_weights.end(), 0.0f);
    std::fill(m.output_bias.begin(), m.output_bias.end(), 0.0f);
    std::fill(m.context_embeddings.begin(), m.context_embeddings.end(), 0.0f);
    std::fill(m.context_output_weights.begin(), m.context_output_weights.end(), 0.0f);
    return m;
}

// runtime.rs:1828-1847 configure_chain
static size_t configure_chain(Model& m, size_t source, size_t links, uint8_t delay) {
    for (size_t off = 0; off < links; ++off) {
        size_t n = source + off, slot = m.slot_start(n);
        m.neuron_type[n] = 0;
        m.recurrent_target[slot] = (uint32_t)(n + 1);
        m.recurrent_branch[slot] = BRANCH_EXCITATORY;
        m.recurrent_delay[slot] = delay;
        m.recurrent_weight[slot] = 1.0f;
    }
    size_t endpoint = source + links;
    m.neuron_type[endpoint] = 0;
    size_t es = m.slot_start(endpoint);
    m.recurrent_branch[es] = BRANCH_EXCITATORY;
    m.recurrent_delay[es] = 1;
    m.recurrent_weight[es] = 0.0f;
    return endpoint;
}

int main() {
    // ---------------------------------------------------------------- learning.rs:83-108
    run("learning.rs:85 analog_surrogate_preserves_selected_unsaturated_gradient", [] {
        CHECK(std::fabs(analog_rank_surrogate(0.5f, 0.4f, true, 0.25f, 0.1f) - 1.06f) <= 1.0e-6f);
        CHECK(analog_rank_surrogate(1.0f, 0.4f, true, 0.25f, 0.1f) == 0.0f);
    });
    run("learning.rs:91 branch_jacobian_matches_integrated_branch_semantics", [] {
        CHECK(branch_jacobian(BRANCH_EXCITATORY, 1.0f, 0.5f, 0.5f) == 1.0f);
        CHECK(branch_jacobian(BRANCH_TEMPORAL, 1.0f, 0.5f, 0.5f) == 0.5f);
        CHECK(branch_jacobian(BRANCH_INHIBITORY, 1.0f, 0.5f, 0.5f) == 1.0f);
        CHECK(branch_jacobian(BRANCH_CONTEXT_GATE, 1.0f, 0.5f, 0.5f) == 0.5f);
    });
    run("learning.rs:99 inhibitory_homeostasis_pushes_in_the_correct_direction", [] {
        CHECK(inhibitory_homeostasis_delta(1.0f, 0.10f, 0.02f, 0.01f, 1.0f, 0.1f) < 0.0f);
        CHECK(inhibitory_homeostasis_delta(1.0f, 0.00f, 0.02f, 0.01f, 1.0f, 0.1f) > 0.0f);
    });
    run("learning.rs:105 update_clipping_is_symmetric", [] {
        CHECK(bounded_delta(1.0f, 0.1f) == 0.1f);
        CHECK(bounded_delta(-1.0f, 0.1f) == -0.1f);
    });

    // ---------------------------------------------------------------- runtime.rs tests
    run("runtime.rs:1694 frozen_execution_is_read_only", [] {
        Model m = causal_model(2);
        float w0 = m.recurrent_weight[0];
        Runtime rt(m);
        rt.begin_document();
        for (char s : std::string("ABBA")) rt.step((uint8_t)s, -1, Permission::Frozen);
        CHECK(rt.model.recurrent_weight[0] == w0);
        CHECK(rt.eligible_recurrent_slots.empty());
        CHECK(rt.eligible_input_slots.empty());
    });

    run("runtime.rs:1710 recurrent_credit_arrives_on_the_configured_delay", [] {
        for (uint8_t delay : {1, 2, 4, 8}) {
            Runtime rt(causal_model(delay));
            rt.begin_document();
            float w0 = rt.model.recurrent_weight[0];
            rt.step('A', 'Y', Permission::Training);
            CHECK(rt.model.recurrent_weight[0] == w0);
            for (int i = 1; i < delay; ++i) {
                rt.step('B', 'Y', Permission::Training);
                CHECK(rt.model.recurrent_weight[0] == w0);
            }
            rt.step('B', 'Y', Permission::Training);
            CHECK(rt.model.recurrent_weight[0] != w0);
        }
    });

    run("runtime.rs:1734 input_trace_survives_refractory_tick_and_receives_later_error", [] {
        Model m = causal_model(1);
        size_t in_slot = (size_t)'A' * m.input_fanout;
        m.input_weights[in_slot] = 0.5f;
        std::fill(m.output_weights.begin(), m.output_weights.end(), 0.0f);
        m.output_weights[out_index('Z') * m.neuron_count()] = 1.0f;
        Runtime rt(m);
        rt.begin_document();
        rt.step('A', -1, Permission::Training);
        float before = rt.model.input_weights[in_slot];
        rt.step('B', 'Y', Permission::Training);
        CHECK(rt.input_eligibility[in_slot] > 0.0f);
        CHECK(rt.model.input_weights[in_slot] < before);
    });

    run("runtime.rs:1756 context_embedding_gradient_uses_the_exact_forward_scale", [] {
        Config c = integrated_config();
        c.embedding_dim = 1;
        c.context_learning_rate = 0.1f;
        c.max_update = 1.0f;
        c.validate();
        Model m = Model::initialize(c);
        std::fill(m.context_embeddings.begin(), m.context_embeddings.end(), 0.0f);
        std::fill(m.context_output_weights.begin(), m.context_output_weights.end(), 0.0f);
        m.context_keys[0] = 1;
        m.context_keys[1] = 2;
        size_t out = out_index('X');
        m.context_output_weights[out] = 1.0f;
        Runtime rt(m);
        rt.active_context_slots = {0, 1};
        rt.active_context_scales = {0.25f, 0.75f};
        std::fill(rt.errors.begin(), rt.errors.end(), 0.0f);
        rt.errors[out] = 1.0f;
        rt.update_context_projection(1.0f);
        CHECK(std::fabs(rt.model.context_embeddings[0] + 0.025f) < 1.0e-6f);
        CHECK(std::fabs(rt.model.context_embeddings[1] + 0.075f) < 1.0e-6f);
    });

    run("runtime.rs:1783 activity_target_does_not_force_winners_without_evidence", [] {
        Model m = Model::initialize(integrated_config());
        std::fill(m.recurrent_weight.begin(), m.recurrent_weight.end(), 0.0f);
        std::fill(m.input_weights.begin(), m.input_weights.end(), 0.0f);
        std::fill(m.threshold.begin(), m.threshold.end(), 0.5f);
        Runtime rt(m);
        rt.begin_document();
        StepMetrics s = rt.step('A', -1, Permission::Frozen);
        CHECK(s.active_neurons == 0);
        CHECK(s.suprathreshold_neurons == 0);
    });

    run("runtime.rs:1849 recurrent_only_state_preserves_branch_information_beyond_context_order", [] {
        for (size_t distance : {16, 32, 64, 128}) {
            Model m = recurrent_memory_model();
            size_t links = distance / 8;
            size_t ea = configure_chain(m, 0, links, 8), eb = configure_chain(m, 32, links, 8);
            size_t ia = (size_t)'A' * m.input_fanout, ib = (size_t)'B' * m.input_fanout;
            m.input_targets[ia] = 0; m.input_targets[ib] = 32;
            m.input_branches[ia] = BRANCH_EXCITATORY; m.input_branches[ib] = BRANCH_EXCITATORY;
            m.input_weights[ia] = 1.0f; m.input_weights[ib] = 1.0f;
            size_t n = m.neuron_count();
            m.output_weights[out_index('X') * n + ea] = 1.0f;
            m.output_weights[out_index('Y') * n + eb] = 1.0f;
            m.validate();
            Runtime rt(m);
            auto predict = [&](uint8_t prefix) {
                rt.begin_document();
                rt.step(prefix, -1, Permission::Frozen);
                uint32_t p = 0;
                for (size_t i = 0; i < distance; ++i) p = rt.step('.', -1, Permission::Frozen).predicted_symbol;
                return p;
            };
            CHECK(predict('A') == 'X');
            CHECK(predict('B') == 'Y');
        }
    });

    run("runtime.rs:1899 recurrent_only_readout_learns_delayed_branches_beyond_frequency", [] {
        for (size_t distance : {16, 32, 64, 128}) {
            Model m = recurrent_memory_model();
            m.config.output_learning_rate = 0.05f;
            m.config.max_update = 0.05f;
            size_t links = distance / 8;
            configure_chain(m, 0, links, 8);
            configure_chain(m, 32, links, 8);
            size_t ia = (size_t)'A' * m.input_fanout, ib = (size_t)'B' * m.input_fanout;
            m.input_targets[ia] = 0; m.input_targets[ib] = 32;
            m.input_branches[ia] = BRANCH_EXCITATORY; m.input_branches[ib] = BRANCH_EXCITATORY;
            m.input_weights[ia] = 1.0f; m.input_weights[ib] = 1.0f;
            m.validate();
            Runtime rt(m);
            for (int rep = 0; rep < 64; ++rep) {
                for (auto pt : {std::pair<uint8_t, uint8_t>{'A', 'X'}, std::pair<uint8_t, uint8_t>{'B', 'Y'}}) {
                    rt.begin_document();
                    rt.step(pt.first, -1, Permission::Frozen);
                    for (size_t i = 0; i + 1 < distance; ++i) rt.step('.', -1, Permission::Frozen);
                    rt.step('.', pt.second, Permission::Training);
                    rt.finish_document();
                }
            }
            for (auto pe : {std::pair<uint8_t, uint8_t>{'A', 'X'}, std::pair<uint8_t, uint8_t>{'B', 'Y'}}) {
                rt.begin_document();
                rt.step(pe.first, -1, Permission::Frozen);
                uint32_t p = 0;
                for (size_t i = 0; i < distance; ++i) p = rt.step('.', -1, Permission::Frozen).predicted_symbol;
                CHECK(p == pe.second);
            }
        }
    });

    run("runtime.rs:1952 recurrent_only_ring_maintains_a_period_longer_than_context_order", [] {
        Model m = recurrent_memory_model();
        size_t period = 16, n = m.neuron_count();
        for (size_t neuron = 0; neuron < period; ++neuron) {
            size_t slot = m.slot_start(neuron);
            m.neuron_type[neuron] = 0;
            m.recurrent_target[slot] = (uint32_t)((neuron + 1) % period);
            m.recurrent_branch[slot] = BRANCH_EXCITATORY;
            m.recurrent_delay[slot] = 1;
            m.recurrent_weight[slot] = 1.0f;
            m.output_weights[out_index('A' + (uint32_t)neuron) * n + neuron] = 1.0f;
        }
        size_t in = (size_t)'!' * m.input_fanout;
        m.input_targets[in] = 0; m.input_branches[in] = BRANCH_EXCITATORY; m.input_weights[in] = 1.0f;
        m.validate();
        Runtime rt(m);
        rt.begin_document();
        std::vector<uint32_t> p;
        p.push_back(rt.step('!', -1, Permission::Frozen).predicted_symbol);
        for (size_t i = 1; i < period * 2; ++i) p.push_back(rt.step('.', -1, Permission::Frozen).predicted_symbol);
        for (size_t i = 0; i < period; ++i) CHECK(p[i] == p[i + period]);
        for (size_t i = 0; i + 1 < period; ++i) CHECK(p[i] != p[i + 1]);
    });

    run("runtime.rs:1995 context_fingerprints_separate_colliding_buckets", [] {
        Config c = integrated_config();
        c.max_order = 1; c.slots_per_order = 4; c.probe_limit = 4;
        c.validate();
        Runtime rt(Model::initialize(c));
        long first = rt.resolve_context_slot(1, 1, true), second = rt.resolve_context_slot(1, 5, true);
        CHECK(first != second);
        CHECK(rt.model.context_keys[(size_t)first] == 1);
        CHECK(rt.model.context_keys[(size_t)second] == 5);
    });

    run("runtime.rs:2013 temporal_context_learns_branching_prefixes_with_fixed_topology", [] {
        Config c = integrated_config();
        c.output_learning_rate = 1.0e-8f;
        c.context_learning_rate = 0.5f;
        c.max_update = 0.1f;
        c.validate();
        Model m = Model::initialize(c);
        std::fill(m.recurrent_weight.begin(), m.recurrent_weight.end(), 0.0f);
        std::fill(m.input_weights.begin(), m.input_weights.end(), 0.0f);
        std::fill(m.output_weights.begin(), m.output_weights.end(), 0.0f);
        std::fill(m.output_bias.begin(), m.output_bias.end(), 0.0f);
        std::fill(m.threshold.begin(), m.threshold.end(), 2.0f);
        size_t fixed = m.recurrent_weight.size();
        Runtime rt(m);
        const char* stories[2] = {"ABX", "CBY"};
        for (int rep = 0; rep < 128; ++rep) {
            for (auto s : stories) {
                rt.begin_document();
                rt.step(BEGIN_DOCUMENT, (uint8_t)s[0], Permission::Training);
                rt.step((uint8_t)s[0], (uint8_t)s[1], Permission::Training);
                rt.step((uint8_t)s[1], (uint8_t)s[2], Permission::Training);
                rt.step((uint8_t)s[2], END_DOCUMENT, Permission::Training);
                rt.finish_document();
            }
        }
        auto predict = [&](const char* prefix) {
            rt.begin_document();
            rt.step(BEGIN_DOCUMENT, -1, Permission::Frozen);
            uint32_t p = END_DOCUMENT;
            for (const char* q = prefix; *q; ++q) p = rt.step((uint8_t)*q, -1, Permission::Frozen).predicted_symbol;
            return p;
        };
        CHECK(predict("AB") == 'X');
        CHECK(predict("CB") == 'Y');
        CHECK(rt.model.recurrent_weight.size() == fixed);
    });

    run("runtime.rs:2078 context_dropout_is_deterministic_and_exposes_neural_steps", [] {
        // context_survives_dropout is runtime.rs:103-116; count survivors via the public step path's hash.
        auto survives = [](uint64_t seed, uint64_t tick, uint32_t symbol, float rate) {
            if (rate <= 0.0f) return true;
            uint64_t v = seed ^ (tick * 0x9e3779b97f4a7c15ull) ^ ((uint64_t)symbol * 0xbf58476d1ce4e5b9ull);
            v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
            v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
            v ^= v >> 31;
            return (float)(uint32_t)(v >> 40) / (float)(1u << 24) >= rate;
        };
        size_t first = 0, second = 0;
        for (uint64_t t = 0; t < 1024; ++t) first += survives(1337, t, 'A', 0.5f);
        for (uint64_t t = 0; t < 1024; ++t) second += survives(1337, t, 'A', 0.5f);
        CHECK(first == second);
        CHECK(first >= 400 && first <= 624);
        for (uint64_t t = 0; t < 32; ++t) CHECK(survives(1337, t, 'A', 0.0f));
        // The runtime applies the same rule: count context-applied steps in a training run.
        Config c = integrated_config();
        c.dropout_rate = 0.5f;
        Model m = Model::initialize(c);
        Runtime rt(m);
        rt.begin_document();
        size_t applied = 0, expected = 0;
        for (uint64_t t = 0; t < 64; ++t) {
            expected += survives(c.seed, rt.current_tick, 'A', 0.5f);
            applied += rt.step('A', 'A', Permission::Training).context_applied;
        }
        CHECK(applied == expected);
    });

    run("runtime.rs:2091 end_document_target_receives_extra_bounded_weight", [] {
        Config c = integrated_config();
        c.output_learning_rate = 0.01f;
        c.end_document_weight = 4.0f;
        c.max_update = 0.02f;
        c.dropout_rate = 0.0f;
        Model m = Model::initialize(c);
        std::fill(m.recurrent_weight.begin(), m.recurrent_weight.end(), 0.0f);
        std::fill(m.input_weights.begin(), m.input_weights.end(), 0.0f);
        std::fill(m.output_weights.begin(), m.output_weights.end(), 0.0f);
        std::fill(m.output_bias.begin(), m.output_bias.end(), 0.0f);
        std::fill(m.threshold.begin(), m.threshold.end(), 2.0f);
        Runtime rt(m);
        rt.begin_document();
        rt.step(BEGIN_DOCUMENT, END_DOCUMENT, Permission::Training);
        CHECK(rt.model.output_bias[END_OUTPUT_INDEX] >= 0.019f);
        CHECK(rt.model.output_bias[END_OUTPUT_INDEX] <= 0.02f + 1.1920929e-7f);
    });

    run("runtime.rs:2118 initialization_enforces_excitatory_and_inhibitory_routes", [] {
        Model m = Model::initialize(integrated_config());
        for (size_t src = 0; src < m.neuron_count(); ++src)
            for (size_t s = m.slot_start(src); s < m.slot_start(src) + m.capacity_per_neuron; ++s) {
                if (m.neuron_type[src] == 0) {
                    CHECK(m.recurrent_weight[s] >= 0.0f);
                    CHECK(m.recurrent_branch[s] != BRANCH_INHIBITORY);
                } else {
                    CHECK(m.recurrent_weight[s] <= 0.0f);
                    CHECK(m.recurrent_branch[s] == BRANCH_INHIBITORY);
                }
            }
    });

    run("runtime.rs:2134 adaptation_and_reset_are_part_of_every_runtime", [] {
        Model m = Model::initialize(integrated_config());
        std::fill(m.recurrent_weight.begin(), m.recurrent_weight.end(), 0.0f);
        std::fill(m.input_weights.begin(), m.input_weights.end(), 0.0f);
        std::fill(m.threshold.begin(), m.threshold.end(), 0.1f);
        size_t slot = (size_t)'A' * m.input_fanout;
        m.input_targets[slot] = 0; m.input_branches[slot] = BRANCH_EXCITATORY; m.input_weights[slot] = 1.0f;
        Runtime rt(m);
        rt.begin_document();
        StepMetrics s = rt.step('A', -1, Permission::Frozen);
        CHECK(s.active_neurons > 0);
        CHECK(rt.membrane[0] < 1.0f);
        CHECK(rt.adaptation_state[0][0] > 0.0f || rt.adaptation_state[1][0] > 0.0f || rt.adaptation_state[2][0] > 0.0f);
    });

    // ---------------------------------------------------------------- model.rs:517-535
    run("model.rs:518 validation_rejects_out_of_bounds_canonical_threshold", [] {
        Model m = Model::initialize(test_config());
        m.threshold[0] = 2.01f;
        bool threw = false;
        try { m.validate(); } catch (const LeoError&) { threw = true; }
        CHECK(threw);
    });
    run("model.rs:525 validation_rejects_out_of_bounds_learned_projection_weight", [] {
        Model m = Model::initialize(test_config());
        m.output_weights[0] = m.config.weight_max + 0.01f;
        bool threw = false;
        try { m.validate(); } catch (const LeoError&) { threw = true; }
        CHECK(threw);
    });
    run("model.rs:532 initialized_model_satisfies_canonical_parameter_bounds", [] {
        Model::initialize(test_config()).validate();
        for (int topo : {1, 2}) Model::initialize(test_config(), topo).validate();
    });

    // ---------------------------------------------------------------- runtime_smoke.rs
    run("runtime_smoke.rs:38 frozen_document_is_read_only", [] {
        Model m = Model::initialize(test_config());
        Model original = m;
        Runtime rt(m);
        rt.begin_document();
        rt.step(BEGIN_DOCUMENT, 'A', Permission::Frozen);
        rt.step('A', END_DOCUMENT, Permission::Frozen);
        rt.finish_document();
        CHECK(rt.model.recurrent_weight == original.recurrent_weight);
        CHECK(rt.model.input_weights == original.input_weights);
        CHECK(rt.model.output_weights == original.output_weights);
        CHECK(rt.model.output_bias == original.output_bias);
        CHECK(rt.model.context_keys == original.context_keys);
        CHECK(rt.model.context_embeddings == original.context_embeddings);
        CHECK(rt.model.context_output_weights == original.context_output_weights);
        CHECK(rt.model.context_observations == original.context_observations);
        CHECK(rt.model.statistics.processed_bytes == 0);
        CHECK(rt.model.statistics.processed_stories == 0);
    });
    run("runtime_smoke.rs:71 training_document_updates_persistent_statistics", [] {
        Runtime rt(Model::initialize(test_config()));
        rt.begin_document();
        rt.step(BEGIN_DOCUMENT, 'A', Permission::Training);
        rt.step('A', END_DOCUMENT, Permission::Training);
        rt.finish_document();
        CHECK(rt.model.statistics.processed_bytes == 1);
        CHECK(rt.model.statistics.processed_stories == 1);
        CHECK(rt.model.statistics.training_targets == 2);
        CHECK(rt.model.statistics.persistent_ticks == 2);
    });
    run("runtime_smoke.rs:90 sparse_selection_respects_the_global_cap", [] {
        Config c = test_config();
        c.neuron_count = 64; c.block_count = 1; c.neurons_per_block = 64; c.input_fanout = 64;
        c.max_active_per_block = 64; c.max_active_global = 8; c.target_activity = 0.02f;
        c.validate();
        Model m = Model::initialize(c);
        std::fill(m.recurrent_weight.begin(), m.recurrent_weight.end(), 0.0f);
        std::fill(m.input_weights.begin(), m.input_weights.end(), 0.0f);
        std::fill(m.threshold.begin(), m.threshold.end(), 0.1f);
        size_t start = (size_t)'A' * m.input_fanout;
        for (size_t i = 0; i < m.input_fanout; ++i) {
            m.input_targets[start + i] = (uint32_t)i;
            m.input_branches[start + i] = BRANCH_EXCITATORY;
            m.input_weights[start + i] = 1.0f;
        }
        Runtime rt(m);
        rt.begin_document();
        StepMetrics s = rt.step('A', -1, Permission::Frozen);
        CHECK(s.active_neurons <= 8);
        CHECK(s.active_neurons > 0);
    });
    run("runtime_smoke.rs:119 output_cache_matches_checkpoint_layout_and_rebuilds_after_mutation", [] {
        Model m = Model::initialize(test_config());
        std::fill(m.threshold.begin(), m.threshold.end(), 0.1f);
        std::fill(m.input_branches.begin(), m.input_branches.end(), BRANCH_EXCITATORY);
        std::fill(m.input_weights.begin(), m.input_weights.end(), 1.0f);
        Runtime rt(m);
        auto manual = [&]() {
            size_t n = rt.model.neuron_count();
            std::vector<float> logits = rt.model.output_bias;
            for (size_t neuron : rt.active)
                for (size_t o = 0; o < OUTPUT_CLASSES; ++o)
                    logits[o] += rt.model.output_weights[o * n + neuron] * rt.activation[neuron];
            float mx = -INFINITY;
            for (float l : logits) mx = std::fmax(mx, l);
            std::vector<float> p(OUTPUT_CLASSES);
            float sum = -0.0f;
            for (size_t o = 0; o < OUTPUT_CLASSES; ++o) p[o] = std::exp(logits[o] - mx);
            for (float v : p) sum += v;
            for (auto& v : p) v /= sum;
            return p;
        };
        rt.begin_document();
        rt.step(BEGIN_DOCUMENT, -1, Permission::Frozen);
        CHECK(!rt.active.empty());
        auto p = manual();
        for (size_t o = 0; o < OUTPUT_CLASSES; ++o) CHECK(std::fabs(p[o] - rt.probabilities[o]) <= 1.0e-6f);
        size_t n = rt.model.neuron_count();
        for (size_t neuron = 0; neuron < n; ++neuron) rt.model.output_weights[neuron] += 0.25f;
        rt.model_changed();
        rt.begin_document();
        rt.step(BEGIN_DOCUMENT, -1, Permission::Frozen);
        p = manual();
        for (size_t o = 0; o < OUTPUT_CLASSES; ++o) CHECK(std::fabs(p[o] - rt.probabilities[o]) <= 1.0e-6f);
    });

    // ---------------------------------------------------------------- parallel.rs:1365-1629
    run("parallel.rs:1366 fixed_parameters_merge_as_a_synchronous_mean_delta", [] {
        Model base = Model::initialize(test_config());
        Model a = base, b = base;
        a.output_bias[0] += 0.2f;
        b.output_bias[0] += 0.4f;
        a.statistics.processed_stories += 1;
        b.statistics.processed_stories += 1;
        std::vector<SparseModelDelta> d = {SparseModelDelta::between(base, a), SparseModelDelta::between(base, b)};
        Model master = base;
        MergeMetrics mm = apply_mean_deltas(master, d);
        CHECK(std::fabs(master.output_bias[0] - (base.output_bias[0] + 0.3f)) < 1.0e-6f);
        CHECK(master.statistics.processed_stories == 2);
        CHECK(mm.workers == 2);
    });
    auto delta_equal = [](const SparseModelDelta& x, const SparseModelDelta& y) {
        auto eq = [](const std::vector<SparseF32Delta>& a, const std::vector<SparseF32Delta>& b) {
            if (a.size() != b.size()) return false;
            for (size_t i = 0; i < a.size(); ++i)
                if (a[i].index != b[i].index || a[i].delta != b[i].delta) return false;
            return true;
        };
        if (!eq(x.threshold, y.threshold) || !eq(x.recurrent_weight, y.recurrent_weight) ||
            !eq(x.input_weight, y.input_weight) || !eq(x.output_weight, y.output_weight) ||
            !eq(x.output_bias, y.output_bias) || !eq(x.context_output_weight, y.context_output_weight) ||
            !eq(x.excitability, y.excitability))
            return false;
        if (x.context.size() != y.context.size()) return false;
        for (size_t i = 0; i < x.context.size(); ++i)
            if (x.context[i].order != y.context[i].order || x.context[i].key != y.context[i].key ||
                x.context[i].embedding_delta != y.context[i].embedding_delta ||
                x.context[i].observation_increment != y.context[i].observation_increment)
                return false;
        return x.revision_increment == y.revision_increment && x.base_revision == y.base_revision;
    };
    run("parallel.rs:1386 tracked_delta_matches_full_delta_for_one_worker_story", [&] {
        Model base = Model::initialize(test_config());
        Runtime rt(base);
        rt.enable_parameter_tracking();
        rt.begin_document();
        rt.step(BEGIN_DOCUMENT, 'A', Permission::Training);
        rt.step('A', END_DOCUMENT, Permission::Training);
        rt.finish_document();
        SparseModelDelta full = SparseModelDelta::between(base, rt.model);
        SparseModelDelta tracked = SparseModelDelta::between_tracked(base, rt.model, rt.parameter_changes());
        CHECK(delta_equal(full, tracked));
    });
    run("parallel.rs:1483 output_weights_merge_in_logical_worker_order_without_tree_maps", [] {
        Model base = Model::initialize(test_config());
        size_t index = 7 * base.neuron_count() + 3;
        Model a = base, b = base;
        a.output_weights[index] += 0.2f;
        b.output_weights[index] -= 0.1f;
        std::vector<SparseModelDelta> d = {SparseModelDelta::between(base, a), SparseModelDelta::between(base, b)};
        CHECK(d[0].output_weight.size() == 1 && d[1].output_weight.size() == 1);
        CHECK(d[0].output_weight[0].index == index);
        Model master = base;
        apply_mean_deltas(master, d);
        CHECK(std::fabs(master.output_weights[index] - (base.output_weights[index] + 0.05f)) < 1.0e-6f);
    });
    run("parallel.rs:1507 additive_delta_merge_preserves_local_trajectory_magnitude", [] {
        Model base = Model::initialize(test_config());
        Model a = base, b = base;
        a.output_bias[0] += 0.2f;
        b.output_bias[0] -= 0.05f;
        a.parameter_revision += 2;
        b.parameter_revision += 3;
        std::vector<SparseModelDelta> d = {SparseModelDelta::between(base, a), SparseModelDelta::between(base, b)};
        Model master = base;
        apply_sum_deltas(master, d);
        CHECK(std::fabs(master.output_bias[0] - (base.output_bias[0] + 0.15f)) < 1.0e-6f);
        CHECK(master.parameter_revision == base.parameter_revision + 5);
    });
    run("parallel.rs:1586 stale_worker_deltas_are_rejected", [] {
        Model base = Model::initialize(test_config());
        Model t = base;
        t.output_bias[0] += 0.1f;
        SparseModelDelta d = SparseModelDelta::between(base, t);
        Model adv = base;
        adv.parameter_revision += 1;
        bool threw = false;
        try {
            apply_mean_deltas(adv, {d});
        } catch (const LeoError& e) {
            threw = std::string(e.what()).find("current canonical revision") != std::string::npos;
        }
        CHECK(threw);
    });
    run("parallel.rs:1598 context_entries_merge_by_fingerprint_not_collision_slot", [] {
        Model base = Model::initialize(test_config());
        size_t slots = base.config.slots_per_order;
        uint64_t k1 = 1, k2 = 1 + slots;
        Model a = base, b = base;
        long s1, s2;
        size_t p;
        a.resolve_context_slot(1, k1, true, &s1, &p);
        b.resolve_context_slot(1, k2, true, &s2, &p);
        size_t d = base.config.embedding_dim;
        a.context_embeddings[(size_t)s1 * d] = 0.4f;
        b.context_embeddings[(size_t)s2 * d] = -0.2f;
        a.context_observations[(size_t)s1] = 1;
        b.context_observations[(size_t)s2] = 1;
        std::vector<SparseModelDelta> deltas = {SparseModelDelta::between(base, a), SparseModelDelta::between(base, b)};
        Model master = base;
        apply_mean_deltas(master, deltas);
        bool has1 = false, has2 = false;
        for (size_t i = 0; i < slots; ++i) {
            has1 |= master.context_keys[i] == k1;
            has2 |= master.context_keys[i] == k2;
        }
        CHECK(has1 && has2);
    });

    // ---------------------------------------------------------------- training.rs replay selection
    run("training.rs:1782 select_replay_ranges budget, centring and overlap", [] {
        std::vector<float> losses = {0.1f, 5.0f, 0.2f, 0.3f, 4.0f, 0.1f, 0.1f, 3.0f, 0.1f, 0.1f};
        auto r = select_replay_ranges(losses, 0.3f, 2);
        size_t total = 0;
        for (auto& x : r) total += x.end - x.start;
        // budget = ceil(10 * (f64)0.3f) = ceil(3.0000001) = 4: the f32 fraction widens before the product.
        CHECK(total == 4);
        CHECK(r.size() == 2);
        CHECK(r[0].start == 0 && r[0].end == 2);  // centred on 1, width 2
        CHECK(r[1].start == 3 && r[1].end == 5);  // centred on 4, width min(2, 4 - 2)
        CHECK(select_replay_ranges(losses, 0.0f, 2).empty());
    });

    // ---------------------------------------------------------------- artifact.rs:265 SHA-256 known vectors
    run("artifact.rs:265 sha256_known_vectors", [] {
        uint8_t out[32];
        sha256((const uint8_t*)"", 0, out);
        const uint8_t empty[4] = {0xe3, 0xb0, 0xc4, 0x42};
        CHECK(std::memcmp(out, empty, 4) == 0);
        sha256((const uint8_t*)"abc", 3, out);
        const uint8_t abc[4] = {0xba, 0x78, 0x16, 0xbf};
        CHECK(std::memcmp(out, abc, 4) == 0);
        CHECK(out[31] == 0xad);
    });

    // ---------------------------------------------------------------- a CPU story batch end to end
    run("training.rs:1667 cpu_story_batch_merges_and_replays", [] {
        Runtime canonical(Model::initialize(test_config()));
        std::vector<std::vector<uint8_t>> stories = {{'a', 'b', 'c', 'a'}, {'b', 'a'}, {'c', 'c', 'a', 'b', 'a'}};
        BatchReport r = train_story_batch(canonical, stories, Permission::Training, 0);
        CHECK(r.targets == 5 + 3 + 6);
        CHECK(canonical.model.statistics.processed_stories == 3);
        CHECK(canonical.model.statistics.training_targets == 14 + r.replay.replay_steps);
        CHECK(r.replay.replay_steps > 0);
        canonical.model.validate();
    });

    std::printf("%s: %d failure(s)\n", g_failures ? "FAILED" : "OK", g_failures);
    return g_failures ? 1 : 0;
}
