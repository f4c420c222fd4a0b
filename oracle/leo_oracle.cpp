// TEST INFRASTRUCTURE ONLY -- parity oracle (see leo_oracle.hpp for the
// contract).  Each function cites the reference file:line it restates.
#include "leo_oracle.hpp"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <limits>
#include <mutex>
#include <set>
#include <thread>
#include <unordered_map>

namespace leo_oracle {

namespace {

// Rust f32::clamp (asserts min <= max, keeps NaN).
inline float clampf(float v, float lo, float hi) {
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}
// Rust f32::max / f32::min (IEEE maxNum/minNum: a NaN operand yields the other).
inline float rmax(float a, float b) {
    if (std::isnan(a)) return b;
    if (std::isnan(b)) return a;
    return a > b ? a : (b > a ? b : a);
}
inline float rmin(float a, float b) {
    if (std::isnan(a)) return b;
    if (std::isnan(b)) return a;
    return a < b ? a : (b < a ? b : a);
}
// Rust f32::powi with a runtime exponent lowers to the compiler-rt/
// compiler-builtins routine: right-to-left binary exponentiation.
inline float powi(float base, int32_t exponent) {
    bool recip = exponent < 0;
    uint32_t e = recip ? (uint32_t)(-(int64_t)exponent) : (uint32_t)exponent;
    float result = 1.0f;
    float a = base;
    for (;;) {
        if (e & 1u) result *= a;
        e >>= 1;
        if (e == 0) break;
        a *= a;
    }
    return recip ? 1.0f / result : result;
}
// runtime.rs:78-85
inline float decay_for_elapsed(float base, uint64_t elapsed) {
    if (elapsed == 0) return 1.0f;
    if (elapsed == 1) return base;
    uint64_t e = std::min<uint64_t>(elapsed, (uint64_t)INT32_MAX);
    return powi(base, (int32_t)e);
}
// runtime.rs:99-101
inline size_t rotated_tie_key(size_t neuron, size_t rotation, size_t n) { return (neuron + n - rotation) % n; }

// runtime.rs:103-116
inline bool context_survives_dropout(uint64_t seed, uint64_t tick, uint32_t symbol, float rate) {
    if (rate <= 0.0f) return true;
    uint64_t v = seed ^ (tick * 0x9e3779b97f4a7c15ull) ^ ((uint64_t)symbol * 0xbf58476d1ce4e5b9ull);
    v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
    v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
    v ^= v >> 31;
    float draw = (float)(uint32_t)(v >> 40) / (float)(1u << 24);
    return draw >= rate;
}


// Rust's f32 Sum folds from -0.0 (Rust >= 1.83; the reference pins 1.85).
inline float sum3(float a, float b, float c) {
    float s = -0.0f;
    s += a;
    s += b;
    s += c;
    return s;
}

}  // namespace

// ---------------------------------------------------------------- learning.rs (declared in leo_oracle.hpp)
// learning.rs:6-24
float analog_rank_surrogate(float margin, float cutoff, bool selected, float width, float gain) {
    float direct = (selected && margin > 0.0f && margin < 1.0f) ? 1.0f : 0.0f;
    if (width <= 0.0f || gain <= 0.0f) return direct;
    float boundary = clampf(1.0f - std::fabs(margin - cutoff) / width, 0.0f, 1.0f);
    return direct + gain * boundary;
}
// learning.rs:28-50
float branch_jacobian(uint8_t branch, float exc, float temporal, float gate_acc) {
    float gate = clampf(gate_acc, 0.0f, 1.0f);
    switch (branch) {
        case BRANCH_EXCITATORY: return exc;
        case BRANCH_TEMPORAL: return exc * gate;
        case BRANCH_INHIBITORY: return exc;
        case BRANCH_CONTEXT_GATE: {
            float gd = (gate_acc > 0.0f && gate_acc < 1.0f) ? 1.0f : 0.0f;
            return exc * temporal * gd;
        }
        default: return 0.0f;
    }
}
// learning.rs:52-55
float bounded_delta(float v, float maximum) { return clampf(v, -maximum, maximum); }
// learning.rs:59-73
float inhibitory_homeostasis_delta(float src_act, float tgt_act, float desired, float lr, float strength,
                                          float maximum) {
    float err = tgt_act - desired;
    return bounded_delta(-lr * strength * src_act * err, maximum);
}

// ---------------------------------------------------------------- rng.rs:13-36
uint64_t SplitMix64::next_u64() {
    state += 0x9E3779B97F4A7C15ull;
    uint64_t v = state;
    v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ull;
    v = (v ^ (v >> 27)) * 0x94D049BB133111EBull;
    return v ^ (v >> 31);
}
float SplitMix64::next_f32() {
    uint32_t value = (uint32_t)(next_u64() >> 40);
    return (float)value / (float)((1u << 24) - 1);
}
size_t SplitMix64::range_usize(size_t upper) {
    if (upper <= 1) return 0;
    return (size_t)(next_u64() % (uint64_t)upper);
}
float SplitMix64::range_f32(float low, float high) { return low + (high - low) * next_f32(); }

// ------------------------------------------------------------ config.rs:250-519
void Config::validate() const {
    auto fail = [](const std::string& m) { throw LeoError(LeoError::Configuration, m); };
    if (neuron_count == 0 || block_count == 0 || neurons_per_block == 0) fail("model dimensions must be positive");
    if (block_count * neurons_per_block != neuron_count)
        fail("block_count * neurons_per_block must equal neuron_count without overflow");
    if (branches_per_neuron != 4) fail("Leo requires exactly four dendritic branches per neuron");
    if (!std::isfinite(excitatory_fraction) || !(excitatory_fraction >= 0.0f && excitatory_fraction < 1.0f))
        fail("excitatory_fraction must be finite and strictly between 0 and 1");
    if (synapses_per_neuron == 0 || input_fanout == 0) fail("synapses_per_neuron and input_fanout must be positive");
    if (synapses_per_neuron > neuron_count) fail("synapses_per_neuron cannot exceed neuron_count");
    if (input_fanout > neuron_count) fail("input_fanout cannot exceed neuron_count");
    if (max_active_per_block == 0 || max_active_per_block > neurons_per_block)
        fail("max_active_per_block must be in 1..=neurons_per_block");
    if (max_active_global == 0 || max_active_global > neuron_count) fail("max_active_global must be in 1..=neuron_count");
    if (refractory_ticks == 0) fail("refractory_ticks must be positive in the integrated architecture");
    const float unit[] = {branch_decay, membrane_decay, fatigue_decay, adaptation_fast_decay,
                          adaptation_medium_decay, adaptation_slow_decay, eligibility_decay};
    for (float v : unit)
        if (!std::isfinite(v) || !(v >= 0.0f && v < 1.0f)) fail("decay must be finite and strictly between 0 and 1");
    const float pos[] = {fatigue_gain, adaptation_fast_gain, adaptation_medium_gain, adaptation_slow_gain,
                         threshold_homeostasis_rate, population_inhibition_rate, output_learning_rate,
                         recurrent_learning_rate, inhibitory_learning_rate, eligibility_epsilon, surrogate_width,
                         surrogate_gain, max_update};
    for (float v : pos)
        if (!std::isfinite(v) || v <= 0.0f) fail("rate must be finite and positive");
    if (!std::isfinite(target_activity) || !(target_activity >= 0.0f && target_activity <= 1.0f) ||
        target_activity == 0.0f)
        fail("target_activity must be finite and in (0, 1]");
    if (!std::isfinite(population_inhibition_max) || population_inhibition_max <= 0.0f)
        fail("population_inhibition_max must be finite and positive");
    if (!std::isfinite(membrane_reset_fraction) || !(membrane_reset_fraction >= 0.0f && membrane_reset_fraction <= 1.0f) ||
        membrane_reset_fraction == 0.0f)
        fail("membrane_reset_fraction must be finite and in (0, 1]");
    size_t target_active = (size_t)std::ceil(target_activity * (float)neuron_count);
    if (target_active > max_active_global) fail("target_activity requires more neurons than max_active_global permits");
    if (weight_min >= 0.0f || weight_max <= 0.0f || weight_min >= weight_max)
        fail("weight_min must be negative and weight_max must be positive");
    if (plasticity_window == 0 || plasticity_window > 64) fail("learning.plasticity_window must be in 1..=64");
    if (!std::isfinite(end_document_weight) || !(end_document_weight >= 1.0f && end_document_weight <= 16.0f))
        fail("end_document_weight must be finite and in [1, 16]");
    const float strengths[] = {provisional_strength, training_strength, verified_strength};
    for (float s : strengths)
        if (!std::isfinite(s) || !(s >= 0.0f && s <= 1.0f) || s == 0.0f) fail("strength must be finite and in (0, 1]");
    if (max_order == 0 || embedding_dim == 0 || slots_per_order == 0 || probe_limit == 0 || confidence_observations == 0)
        fail("all context-memory dimensions must be positive");
    if (embedding_dim > 256) fail("context.embedding_dim cannot exceed 256");
    if (max_order > 16) fail("context.max_order cannot exceed 16");
    if (probe_limit > slots_per_order) fail("context.probe_limit cannot exceed slots_per_order");
    if (!std::isfinite(dropout_rate) || !(dropout_rate >= 0.0f && dropout_rate < 1.0f))
        fail("context.dropout_rate must be finite and in [0, 1)");
    if (!std::isfinite(context_learning_rate) || context_learning_rate <= 0.0f)
        fail("context.learning_rate must be finite and positive");
    if (!std::isfinite(replay_fraction) || replay_fraction < 0.0f || replay_fraction > 1.0f)
        fail("replay.fraction must be finite and in the interval [0, 1]");
    if (segment_bytes == 0) fail("all replay limits must be positive");
}

void Config::plasticity_step(size_t phase, bool end_document, float* scale, size_t* next) const {
    size_t window = std::max<size_t>(plasticity_window, 1);
    size_t step = std::min(phase, window - 1) + 1;
    if (step == window || end_document) {
        *scale = (float)step;
        *next = 0;
    } else {
        *scale = 0.0f;
        *next = step;
    }
}

uint64_t Config::fingerprint() const {
    // FNV-1a over the config's field bytes; self-consistent stand-in for the
    // TOML-text SHA-256 of parallel.rs:1347-1349.
    uint64_t h = 0xcbf29ce484222325ull;
    auto mix = [&](const void* p, size_t n) {
        const uint8_t* b = (const uint8_t*)p;
        for (size_t i = 0; i < n; ++i) { h ^= b[i]; h *= 0x100000001b3ull; }
    };
    const size_t sizes[] = {neuron_count, block_count, neurons_per_block, synapses_per_neuron, input_fanout,
                            max_active_per_block, max_active_global, plasticity_window, max_order, embedding_dim,
                            slots_per_order, probe_limit, segment_bytes};
    for (size_t v : sizes) { uint64_t x = v; mix(&x, 8); }
    const float fl[] = {excitatory_fraction, branch_decay, membrane_decay, fatigue_decay, fatigue_gain, target_activity,
                        threshold_homeostasis_rate, population_inhibition_rate, population_inhibition_max,
                        adaptation_fast_decay, adaptation_medium_decay, adaptation_slow_decay, adaptation_fast_gain,
                        adaptation_medium_gain, adaptation_slow_gain, membrane_reset_fraction, output_learning_rate,
                        recurrent_learning_rate, inhibitory_learning_rate, eligibility_decay, eligibility_epsilon,
                        surrogate_width, surrogate_gain, max_update, weight_min, weight_max, provisional_strength,
                        training_strength, verified_strength, end_document_weight, context_learning_rate, dropout_rate,
                        replay_fraction};
    mix(fl, sizeof(fl));
    mix(&seed, 8);
    mix(&refractory_ticks, 8);
    mix(&confidence_observations, 4);
    return h;
}

float permission_strength(Permission p, const Config& c) {
    switch (p) {
        case Permission::Frozen: return 0.0f;
        case Permission::Provisional: return c.provisional_strength;
        case Permission::Training: return c.training_strength;
        case Permission::Verified: return c.verified_strength;
    }
    return 0.0f;
}

// -------------------------------------------------------------- model.rs:79-158
namespace {
// model.rs:498-505
uint8_t sample_delay(SplitMix64& rng) {
    size_t r = rng.range_usize(100);
    if (r <= 49) return 1;
    if (r <= 74) return 2;
    if (r <= 89) return 4;
    return 8;
}

// model.rs:399-459
void initialize_recurrent_reference(const Config& config, SplitMix64& rng, const std::vector<uint8_t>& types,
                                    Model& m) {
    size_t n = config.neuron_count, block_size = config.neurons_per_block;
    size_t local_count = (config.synapses_per_neuron * 3) / 4;
    for (size_t source = 0; source < n; ++source) {
        uint8_t source_type = types[source];
        size_t source_block = source / block_size;
        std::set<std::pair<size_t, uint8_t>> used;
        for (size_t local = 0; local < config.synapses_per_neuron; ++local) {
            size_t slot = source * m.capacity_per_neuron + local;
            bool prefer_local = local < local_count;
            bool found = false;
            size_t target = 0;
            uint8_t branch = 0;
            for (int attempt = 0; attempt < 128; ++attempt) {
                size_t t;
                if (prefer_local) {
                    long block_delta = (long)rng.range_usize(3) - 1;
                    long block = std::clamp((long)source_block + block_delta, 0L, (long)config.block_count - 1);
                    t = (size_t)block * block_size + rng.range_usize(block_size);
                } else {
                    t = rng.range_usize(n);
                }
                uint8_t b;
                if (source_type == 0) {
                    size_t r = rng.range_usize(3);
                    b = r == 0 ? BRANCH_EXCITATORY : (r == 1 ? BRANCH_TEMPORAL : BRANCH_CONTEXT_GATE);
                } else {
                    b = BRANCH_INHIBITORY;
                }
                if (t == source && b != BRANCH_TEMPORAL) continue;
                if (used.insert({t, b}).second) {
                    target = t;
                    branch = b;
                    found = true;
                    break;
                }
            }
            if (!found) throw LeoError(LeoError::Internal, "could not initialize unique synapse");
            m.recurrent_target[slot] = (uint32_t)target;
            m.recurrent_branch[slot] = branch;
            m.recurrent_delay[slot] = sample_delay(rng);
            m.recurrent_weight[slot] = source_type == 0 ? rng.range_f32(0.01f, 0.08f) : rng.range_f32(-0.08f, -0.01f);
        }
    }
}

// Standard normal draw from two SplitMix64 doubles (Box-Muller, cosine branch).
double normal_draw(SplitMix64& rng) {
    double u1 = ((double)(rng.next_u64() >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    double u2 = (double)(rng.next_u64() >> 11) * (1.0 / 9007199254740992.0);
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

// Synthetic benchmark topology: fan-out slots with uniform (1) or Zipf(1.1)
// (2) targets, weights |N(0, 1/sqrt(S))| signed by source type.  Keeps the
// reference invariants: unique (target, branch) per source, no self-synapse
// except on the temporal branch, delay distribution of model.rs:498-505.
void initialize_recurrent_synthetic(const Config& config, SplitMix64& rng, const std::vector<uint8_t>& types,
                                    Model& m, int topology) {
    size_t n = config.neuron_count, s = config.synapses_per_neuron;
    std::vector<double> cdf;
    std::vector<uint32_t> rank_to_neuron;
    if (topology == 2) {
        cdf.resize(n);
        double acc = 0.0;
        for (size_t k = 0; k < n; ++k) {
            acc += std::pow((double)(k + 1), -1.1);
            cdf[k] = acc;
        }
        for (size_t k = 0; k < n; ++k) cdf[k] /= acc;
        rank_to_neuron.resize(n);
        for (size_t k = 0; k < n; ++k) rank_to_neuron[k] = (uint32_t)k;
        rng.shuffle(rank_to_neuron);
    }
    double sigma = 1.0 / std::sqrt((double)s);
    for (size_t source = 0; source < n; ++source) {
        uint8_t source_type = types[source];
        std::set<std::pair<size_t, uint8_t>> used;
        for (size_t local = 0; local < s; ++local) {
            size_t slot = source * m.capacity_per_neuron + local;
            bool found = false;
            size_t target = 0;
            uint8_t branch = 0;
            for (int attempt = 0; attempt < 256; ++attempt) {
                size_t t;
                if (topology == 2 && attempt < 128) {
                    double u = (double)(rng.next_u64() >> 11) * (1.0 / 9007199254740992.0);
                    size_t k = (size_t)(std::lower_bound(cdf.begin(), cdf.end(), u) - cdf.begin());
                    if (k >= n) k = n - 1;
                    t = rank_to_neuron[k];
                } else {
                    t = rng.range_usize(n);
                }
                uint8_t b;
                if (source_type == 0) {
                    size_t r = rng.range_usize(3);
                    b = r == 0 ? BRANCH_EXCITATORY : (r == 1 ? BRANCH_TEMPORAL : BRANCH_CONTEXT_GATE);
                } else {
                    b = BRANCH_INHIBITORY;
                }
                if (t == source && b != BRANCH_TEMPORAL) continue;
                if (used.insert({t, b}).second) {
                    target = t;
                    branch = b;
                    found = true;
                    break;
                }
            }
            if (!found) throw LeoError(LeoError::Internal, "could not initialize unique synapse");
            m.recurrent_target[slot] = (uint32_t)target;
            m.recurrent_branch[slot] = branch;
            m.recurrent_delay[slot] = sample_delay(rng);
            double w = std::fabs(normal_draw(rng) * sigma);
            float wf = (float)w;
            if (source_type == 0) {
                wf = std::min(wf, config.weight_max);
            } else {
                wf = std::max(-wf, config.weight_min);
            }
            m.recurrent_weight[slot] = wf;
        }
    }
}

// model.rs:461-496
void initialize_input(const Config& config, SplitMix64& rng, Model& m) {
    size_t fanout = config.input_fanout;
    size_t count = SYMBOL_COUNT * fanout;
    m.input_fanout = fanout;
    m.input_targets.assign(count, 0);
    m.input_branches.assign(count, BRANCH_EXCITATORY);
    m.input_weights.assign(count, 0.0f);
    for (size_t symbol = 0; symbol < SYMBOL_COUNT; ++symbol) {
        std::set<size_t> used;
        for (size_t index = 0; index < fanout; ++index) {
            size_t target;
            for (;;) {
                target = rng.range_usize(config.neuron_count);
                if (used.insert(target).second) break;
            }
            size_t offset = symbol * fanout + index;
            m.input_targets[offset] = (uint32_t)target;
            size_t r = index % 8;
            m.input_branches[offset] = r == 6 ? BRANCH_TEMPORAL : (r == 7 ? BRANCH_CONTEXT_GATE : BRANCH_EXCITATORY);
            m.input_weights[offset] = rng.range_f32(0.05f, 0.20f);
        }
    }
}
}  // namespace

Model Model::initialize(const Config& config, int topology) {
    config.validate();
    Model m;
    m.config = config;
    size_t n = config.neuron_count, cap = config.synapses_per_neuron;
    size_t synapses = n * cap;
    size_t context_slots = config.max_order * config.slots_per_order;
    SplitMix64 rng(config.seed);

    std::vector<uint8_t> types(n, 0);
    size_t inhibitory = (size_t)std::round((1.0f - config.excitatory_fraction) * (float)n);
    std::vector<size_t> ids(n);
    for (size_t i = 0; i < n; ++i) ids[i] = i;
    rng.shuffle(ids);
    for (size_t i = 0; i < inhibitory && i < n; ++i) types[ids[i]] = 1;
    m.neuron_type = types;
    m.threshold.assign(n, 0.0f);
    m.excitability.assign(n, 1.0f);
    for (auto& t : m.threshold) t = rng.range_f32(0.45f, 0.55f);

    m.capacity_per_neuron = cap;
    m.recurrent_target.assign(synapses, 0);
    m.recurrent_branch.assign(synapses, BRANCH_EXCITATORY);
    m.recurrent_delay.assign(synapses, 1);
    m.recurrent_weight.assign(synapses, 0.0f);
    if (topology == 0)
        initialize_recurrent_reference(config, rng, types, m);
    else
        initialize_recurrent_synthetic(config, rng, types, m, topology);

    initialize_input(config, rng, m);
    m.output_weights.assign(OUTPUT_CLASSES * n, 0.0f);
    for (auto& w : m.output_weights) w = rng.range_f32(-0.005f, 0.005f);
    m.context_output_weights.assign(OUTPUT_CLASSES * config.embedding_dim, 0.0f);
    for (auto& w : m.context_output_weights) w = rng.range_f32(-0.005f, 0.005f);
    m.output_bias.assign(OUTPUT_CLASSES, 0.0f);
    m.context_keys.assign(context_slots, 0);
    m.context_embeddings.assign(context_slots * config.embedding_dim, 0.0f);
    m.context_observations.assign(context_slots, 0);
    return m;
}

// model.rs:173-221
void Model::resolve_context_slot(size_t order, uint64_t key, bool allocate, long* out_slot, size_t* out_probes) {
    if (order == 0 || order > config.max_order || key == 0)
        throw LeoError(LeoError::Internal, "invalid context order or fingerprint");
    size_t spo = config.slots_per_order, limit = config.probe_limit;
    size_t base = (order - 1) * spo;
    size_t start = (size_t)(key % (uint64_t)spo);
    long empty_slot = -1;
    size_t weakest_slot = base + start;
    uint32_t weakest_obs = UINT32_MAX;
    size_t probes = 0;
    for (size_t offset = 0; offset < limit; ++offset) {
        size_t slot = base + (start + offset) % spo;
        probes += 1;
        uint64_t existing = context_keys[slot];
        if (existing == key) {
            *out_slot = (long)slot;
            *out_probes = probes;
            return;
        }
        if (existing == 0 && empty_slot < 0) empty_slot = (long)slot;
        uint32_t obs = context_observations[slot];
        if (obs < weakest_obs) {
            weakest_obs = obs;
            weakest_slot = slot;
        }
    }
    *out_probes = probes;
    if (!allocate) {
        *out_slot = -1;
        return;
    }
    size_t slot = empty_slot >= 0 ? (size_t)empty_slot : weakest_slot;
    if (context_keys[slot] != key) {
        context_keys[slot] = key;
        context_observations[slot] = 0;
        size_t d = config.embedding_dim;
        std::fill(context_embeddings.begin() + slot * d, context_embeddings.begin() + (slot + 1) * d, 0.0f);
    }
    *out_slot = (long)slot;
}

// model.rs:223-396
void Model::validate() const {
    config.validate();
    auto fail = [](const std::string& m) { throw LeoError(LeoError::Internal, m); };
    size_t n = config.neuron_count, cap = config.synapses_per_neuron;
    size_t synapses = n * cap, input_count = SYMBOL_COUNT * config.input_fanout;
    size_t ctx = config.max_order * config.slots_per_order;
    if (threshold.size() != n || excitability.size() != n || neuron_type.size() != n || capacity_per_neuron != cap ||
        recurrent_target.size() != synapses || recurrent_branch.size() != synapses ||
        recurrent_delay.size() != synapses || recurrent_weight.size() != synapses ||
        input_fanout != config.input_fanout || input_targets.size() != input_count ||
        input_branches.size() != input_count || input_weights.size() != input_count ||
        output_weights.size() != OUTPUT_CLASSES * n || output_bias.size() != OUTPUT_CLASSES ||
        context_keys.size() != ctx || context_embeddings.size() != ctx * config.embedding_dim ||
        context_observations.size() != ctx || context_output_weights.size() != OUTPUT_CLASSES * config.embedding_dim)
        fail("model tensor dimensions are incompatible");
    const std::vector<float>* fv[] = {&threshold, &excitability, &recurrent_weight, &input_weights,
                                      &output_weights, &output_bias, &context_embeddings, &context_output_weights};
    for (auto* v : fv)
        for (float x : *v)
            if (!std::isfinite(x)) fail("model contains NaN or infinite values");
    if (!std::isfinite(statistics.training_loss_sum)) fail("model contains NaN or infinite values");
    for (float t : threshold)
        if (t < 0.05f || t > 2.0f) fail("neuron thresholds violate canonical parameter bounds");
    for (float e : excitability)
        if (e < 0.1f || e > 4.0f) fail("neuron excitability violates canonical parameter bounds");
    float wmin = config.weight_min, wmax = config.weight_max;
    const std::vector<float>* pv[] = {&output_weights, &context_embeddings, &context_output_weights};
    for (auto* v : pv)
        for (float x : *v)
            if (x < wmin || x > wmax) fail("learned projection weights violate canonical parameter bounds");
    for (size_t i = 0; i < ctx; ++i)
        if (context_keys[i] == 0 && context_observations[i] != 0) fail("empty context slots cannot contain observations");
    for (uint8_t t : neuron_type)
        if (t > 1) fail("neuron types must be excitatory or inhibitory");
    for (size_t source = 0; source < n; ++source) {
        for (size_t slot = source * cap; slot < (source + 1) * cap; ++slot) {
            size_t target = recurrent_target[slot];
            uint8_t branch = recurrent_branch[slot], delay = recurrent_delay[slot];
            float w = recurrent_weight[slot];
            if (target >= n) fail("recurrent slot targets neuron outside the model");
            if (branch > BRANCH_CONTEXT_GATE || !(delay == 1 || delay == 2 || delay == 4 || delay == 8))
                fail("recurrent slot has invalid branch or delay");
            if (w < wmin || w > wmax) fail("recurrent slot has invalid weight");
            if (neuron_type[source] == 0) {
                if (w < 0.0f || branch == BRANCH_INHIBITORY) fail("excitatory source has incompatible slot");
            } else if (w > 0.0f || branch != BRANCH_INHIBITORY) {
                fail("inhibitory source has incompatible slot");
            }
        }
    }
    for (size_t slot = 0; slot < input_count; ++slot) {
        if (input_targets[slot] >= n || input_branches[slot] == BRANCH_INHIBITORY ||
            input_branches[slot] > BRANCH_CONTEXT_GATE || input_weights[slot] < 0.0f || input_weights[slot] > wmax)
            fail("input projection slot has invalid state");
    }
}

// ------------------------------------------------------------ runtime.rs:188-303
Runtime::Runtime(Model m) : model(std::move(m)) {
    model.validate();
    size_t n = model.neuron_count();
    size_t synapses = model.recurrent_weight.size(), inputs = model.input_weights.size();
    size_t max_delay = 8;
    for (uint8_t d : model.recurrent_delay) max_delay = std::max<size_t>(max_delay, d);
    delay_ring.assign(max_delay + 1, {});
    membrane.assign(n, 0.0f);
    activation.assign(n, 0.0f);
    fatigue.assign(n, 0.0f);
    refractory_until.assign(n, 0);
    branches.assign(n * model.config.branches_per_neuron, 0.0f);
    touched_mark.assign(n, 0);
    selected_mark.assign(n, 0);
    selection_surrogate.assign(n, 0.0f);
    branch_last_tick.assign(n, 0);
    neuron_last_tick.assign(n, 0);
    for (auto& a : adaptation_state) a.assign(n, 0.0f);
    rec_branch_sens.assign(synapses, 0.0f);
    rec_membrane_sens.assign(synapses, 0.0f);
    rec_fatigue_sens.assign(synapses, 0.0f);
    for (auto& a : rec_adapt_sens) a.assign(synapses, 0.0f);
    eligibility.assign(synapses, 0.0f);
    eligibility_last_tick.assign(synapses, 0);
    eligible_recurrent_mark.assign(synapses, 0);
    in_branch_sens.assign(inputs, 0.0f);
    in_membrane_sens.assign(inputs, 0.0f);
    in_fatigue_sens.assign(inputs, 0.0f);
    for (auto& a : in_adapt_sens) a.assign(inputs, 0.0f);
    input_eligibility.assign(inputs, 0.0f);
    input_eligibility_last_tick.assign(inputs, 0);
    eligible_input_mark.assign(inputs, 0);
    logits.assign(OUTPUT_CLASSES, 0.0f);
    probabilities.assign(OUTPUT_CLASSES, 0.0f);
    errors.assign(OUTPUT_CLASSES, 0.0f);
    learning_signal.assign(n, 0.0f);
    learning_destination_mark.assign(n, 0);
    output_cache_dirty = true;
    ensure_output_weight_cache();
    block_candidates.assign(model.config.block_count, {});
    block_selection_cutoff.assign(model.config.block_count, 0.0f);
    context_latent.assign(model.config.embedding_dim, 0.0f);
    context_latent_gradient.assign(model.config.embedding_dim, 0.0f);
}

// runtime.rs:86-97 (neuron-major cache of the output matrix)
void Runtime::ensure_output_weight_cache() {
    if (!output_cache_dirty) return;
    size_t n = model.neuron_count();
    output_weights_by_neuron.assign(n * OUTPUT_CLASSES, 0.0f);
    for (size_t o = 0; o < OUTPUT_CLASSES; ++o)
        for (size_t neuron = 0; neuron < n; ++neuron)
            output_weights_by_neuron[neuron * OUTPUT_CLASSES + o] = model.output_weights[o * n + neuron];
    output_cache_dirty = false;
}

// runtime.rs:317-326
void Runtime::enable_parameter_tracking() {
    if (track_parameter_changes) return;
    track_parameter_changes = true;
    changed_threshold_mark.assign(model.neuron_count(), 0);
    changed_recurrent_weight_mark.assign(model.recurrent_weight.size(), 0);
    changed_input_weight_mark.assign(model.input_weights.size(), 0);
    changed_output_neuron_mark.assign(model.neuron_count(), 0);
    changed_context_slot_mark.assign(model.context_keys.size(), 0);
}

// runtime.rs:328-338
ParameterChanges Runtime::parameter_changes() const {
    ParameterChanges c;
    c.threshold = changed_threshold;
    c.recurrent_weight = changed_recurrent_weight;
    c.input_weight = changed_input_weight;
    c.output_neurons = changed_output_neurons;
    c.context_slots = changed_context_slots;
    c.output_bias_dirty = output_bias_dirty;
    c.context_output_dirty = context_output_dirty;
    return c;
}

// runtime.rs:367-373
void Runtime::finish_document() {
    if (persistent_document_activity) model.statistics.processed_stories += 1;
    reset_transient_state();
}

// runtime.rs:375-435
void Runtime::reset_transient_state() {
    std::fill(membrane.begin(), membrane.end(), 0.0f);
    std::fill(activation.begin(), activation.end(), 0.0f);
    std::fill(fatigue.begin(), fatigue.end(), 0.0f);
    std::fill(refractory_until.begin(), refractory_until.end(), 0);
    std::fill(branches.begin(), branches.end(), 0.0f);
    for (auto& a : adaptation_state) std::fill(a.begin(), a.end(), 0.0f);
    for (auto& b : delay_ring) b.clear();
    due_events.clear();
    std::fill(rec_branch_sens.begin(), rec_branch_sens.end(), 0.0f);
    std::fill(rec_membrane_sens.begin(), rec_membrane_sens.end(), 0.0f);
    std::fill(rec_fatigue_sens.begin(), rec_fatigue_sens.end(), 0.0f);
    for (auto& a : rec_adapt_sens) std::fill(a.begin(), a.end(), 0.0f);
    std::fill(eligibility.begin(), eligibility.end(), 0.0f);
    std::fill(eligibility_last_tick.begin(), eligibility_last_tick.end(), current_tick);
    std::fill(eligible_recurrent_mark.begin(), eligible_recurrent_mark.end(), 0);
    eligible_recurrent_slots.clear();
    std::fill(in_branch_sens.begin(), in_branch_sens.end(), 0.0f);
    std::fill(in_membrane_sens.begin(), in_membrane_sens.end(), 0.0f);
    std::fill(in_fatigue_sens.begin(), in_fatigue_sens.end(), 0.0f);
    for (auto& a : in_adapt_sens) std::fill(a.begin(), a.end(), 0.0f);
    std::fill(input_eligibility.begin(), input_eligibility.end(), 0.0f);
    std::fill(input_eligibility_last_tick.begin(), input_eligibility_last_tick.end(), current_tick);
    std::fill(eligible_input_mark.begin(), eligible_input_mark.end(), 0);
    eligible_input_slots.clear();
    std::fill(branch_last_tick.begin(), branch_last_tick.end(), current_tick);
    std::fill(neuron_last_tick.begin(), neuron_last_tick.end(), current_tick);
    std::fill(touched_mark.begin(), touched_mark.end(), 0);
    std::fill(selected_mark.begin(), selected_mark.end(), 0);
    std::fill(selection_surrogate.begin(), selection_surrogate.end(), 0.0f);
    touched.clear();
    active.clear();
    previous_active.clear();
    for (auto& b : block_candidates) b.clear();
    std::fill(block_selection_cutoff.begin(), block_selection_cutoff.end(), 0.0f);
    population_selection_cutoff = 0.0f;
    context_history.clear();
    active_context_slots.clear();
    active_context_scales.clear();
    std::fill(context_latent.begin(), context_latent.end(), 0.0f);
    std::fill(context_latent_gradient.begin(), context_latent_gradient.end(), 0.0f);
    active_context_probes = 0;
    context_applied_this_step = false;
    population_inhibition = 0.0f;
    persistent_document_activity = false;
    learning_trace_enabled = false;
    plasticity_phase = 0;
}

// runtime.rs:437-535
StepMetrics Runtime::step(uint32_t symbol, long target, Permission permission) {
    if (symbol >= SYMBOL_COUNT) throw LeoError(LeoError::Internal, "invalid input symbol");
    long target_index = -1;
    if (target >= 0) {
        if ((uint32_t)target < BYTE_SYMBOLS)
            target_index = target;
        else if ((uint32_t)target == END_DOCUMENT)
            target_index = (long)END_OUTPUT_INDEX;
        else
            throw LeoError(LeoError::Internal, "invalid output target");
    }
    ensure_output_weight_cache();
    bool frozen = permission == Permission::Frozen;
    learning_trace_enabled = !frozen;

    start_tick();
    deliver_due_events();
    inject_symbol(symbol);
    bool context_enabled =
        frozen || context_survives_dropout(model.config.seed, current_tick, symbol, model.config.dropout_rate);
    activate_context(symbol, !frozen && context_enabled, context_enabled);
    SelectionMetrics selection = select_active_neurons();
    if (learning_trace_enabled) update_forward_eligibilities();
    apply_post_activation_dynamics();
    size_t emitted = emit_recurrent_events();
    float neural_loss = 0.0f;
    bool has_neural = compute_output_probabilities(target_index, &neural_loss);
    uint32_t predicted = (uint32_t)argmax_probability();
    if (predicted == END_OUTPUT_INDEX) predicted = END_DOCUMENT;
    bool has_loss = target_index >= 0;
    float loss = 0.0f;
    if (has_loss) loss = -std::log(rmax(probabilities[(size_t)target_index], 1.0e-12f));
    float gain = (has_neural && has_loss) ? neural_loss - loss : 0.0f;

    LearningMetrics lm;
    if (target_index >= 0) {
        float strength = permission_strength(permission, model.config);
        float target_weight = (size_t)target_index == END_OUTPUT_INDEX ? model.config.end_document_weight : 1.0f;
        if (strength > 0.0f) {
            lm = apply_learning((size_t)target_index, strength, target_weight);
            model.parameter_revision += 1;
        }
    }
    size_t active_neurons = active.size();
    if (!frozen) {
        persistent_document_activity = true;
        update_homeostasis(active_neurons);
        update_statistics(symbol, has_loss, loss, emitted);
    }
    current_tick += 1;  // finish_tick runtime.rs:563-565

    StepMetrics m;
    m.has_loss = has_loss;
    m.loss = loss;
    m.predicted_symbol = predicted;
    m.active_neurons = active_neurons;
    m.emitted_events = emitted;
    m.suprathreshold_neurons = selection.suprathreshold;
    m.block_selected_neurons = selection.block_selected;
    m.global_cap_clipped_neurons = selection.clipped;
    m.population_inhibition = population_inhibition;
    m.context_cells = active_context_slots.size();
    m.context_probes = active_context_probes;
    m.context_applied = context_applied_this_step;
    m.context_loss_gain = gain;
    m.output_madds = active_neurons * OUTPUT_CLASSES + active_context_slots.size() * model.config.embedding_dim +
                     (active_context_slots.empty() ? 0 : model.config.embedding_dim * OUTPUT_CLASSES);
    m.eligible_recurrent_synapses = eligible_recurrent_slots.size();
    m.eligible_input_synapses = eligible_input_slots.size();
    m.mean_abs_eligibility = lm.count == 0 ? 0.0f : (float)(lm.abs_sum / (double)lm.count);
    return m;
}

// runtime.rs:537-561
void Runtime::start_tick() {
    for (size_t neuron : touched) {
        touched_mark[neuron] = 0;
        selection_surrogate[neuron] = 0.0f;
    }
    touched.clear();
    std::swap(active, previous_active);
    active.clear();
    for (size_t neuron : previous_active) {
        activation[neuron] = 0.0f;
        selected_mark[neuron] = 0;
    }
    for (size_t i = 0; i < previous_active.size(); ++i) mark_touched(previous_active[i]);
    for (auto& b : block_candidates) b.clear();
    std::fill(block_selection_cutoff.begin(), block_selection_cutoff.end(), 0.0f);
    population_selection_cutoff = 0.0f;
}

// runtime.rs:567-574
void Runtime::mark_touched(size_t neuron) {
    if (touched_mark[neuron]) return;
    bring_neuron_to_current_tick(neuron);
    touched_mark[neuron] = 1;
    touched.push_back(neuron);
}

// runtime.rs:576-603
void Runtime::bring_neuron_to_current_tick(size_t neuron) {
    const Config& c = model.config;
    uint64_t be = current_tick > branch_last_tick[neuron] ? current_tick - branch_last_tick[neuron] : 0;
    if (be > 0) {
        float decay = decay_for_elapsed(c.branch_decay, be);
        for (size_t b = 0; b < 4; ++b) branches[neuron * 4 + b] *= decay;
        branch_last_tick[neuron] = current_tick;
    }
    uint64_t ne = current_tick > neuron_last_tick[neuron] ? current_tick - neuron_last_tick[neuron] : 0;
    if (ne > 0) {
        membrane[neuron] *= decay_for_elapsed(c.membrane_decay, ne);
        fatigue[neuron] *= decay_for_elapsed(c.fatigue_decay, ne);
        float decays[3];
        c.adaptation_decays(decays);
        for (int i = 0; i < 3; ++i) adaptation_state[i][neuron] *= decay_for_elapsed(decays[i], ne);
        neuron_last_tick[neuron] = current_tick;
    }
}

// runtime.rs:605-625
void Runtime::deliver_due_events() {
    size_t bucket = (size_t)(current_tick % delay_ring.size());
    std::swap(due_events, delay_ring[bucket]);
    for (size_t i = 0; i < due_events.size(); ++i) {
        Event e = due_events[i];
        if (learning_trace_enabled) activate_recurrent_trace(e.synapse_slot, e.presynaptic_activation);
        add_to_branch(e.target_neuron, e.target_branch, e.value);
    }
    due_events.clear();
}

// runtime.rs:627-639
void Runtime::inject_symbol(uint32_t symbol) {
    size_t fanout = model.input_fanout, start = (size_t)symbol * fanout;
    for (size_t offset = start; offset < start + fanout; ++offset) {
        size_t target = model.input_targets[offset];
        uint8_t branch = model.input_branches[offset];
        float value = model.input_weights[offset];
        if (learning_trace_enabled) activate_input_trace(offset, 1.0f);
        add_to_branch(target, branch, value);
    }
}

// runtime.rs:641-686
void Runtime::activate_context(uint32_t symbol, bool allocate, bool enabled) {
    size_t max_order = model.config.max_order;
    if (context_history.size() == max_order) context_history.erase(context_history.begin());
    context_history.push_back(symbol);
    active_context_slots.clear();
    active_context_scales.clear();
    std::fill(context_latent.begin(), context_latent.end(), 0.0f);
    std::fill(context_latent_gradient.begin(), context_latent_gradient.end(), 0.0f);
    active_context_probes = 0;
    context_applied_this_step = enabled;
    if (!enabled) return;
    size_t available = std::min(context_history.size(), max_order);
    float confidence_target = (float)model.config.confidence_observations;
    float scale_sum = 0.0f;
    for (size_t order = 1; order <= available; ++order) {
        uint64_t key = context_key(order);
        long slot = resolve_context_slot(order, key, allocate);
        if (slot < 0) continue;
        float obs = (float)model.context_observations[(size_t)slot];
        float confidence = obs / (obs + confidence_target);
        float scale = confidence * (float)order;
        active_context_slots.push_back((size_t)slot);
        active_context_scales.push_back(scale);
        scale_sum += scale;
    }
    if (scale_sum > 0.0f)
        for (auto& s : active_context_scales) s /= scale_sum;
}

// runtime.rs:688-699
uint64_t Runtime::context_key(size_t order) const {
    const uint64_t prime = 0x100000001b3ull;
    uint64_t hash = 0xcbf29ce484222325ull ^ (uint64_t)order;
    size_t start = context_history.size() - order;
    for (size_t i = start; i < context_history.size(); ++i) {
        uint32_t symbol = context_history[i];
        for (int b = 0; b < 4; ++b) {
            hash ^= (uint64_t)((symbol >> (8 * b)) & 0xffu);
            hash *= prime;
        }
    }
    return hash > 1 ? hash : 1;
}

// runtime.rs:701-708
long Runtime::resolve_context_slot(size_t order, uint64_t key, bool allocate) {
    long slot;
    size_t probes;
    model.resolve_context_slot(order, key, allocate, &slot, &probes);
    active_context_probes += probes;
    return slot;
}

// runtime.rs:710-717
void Runtime::add_to_branch(size_t neuron, uint8_t branch, float value) {
    if (neuron >= model.neuron_count() || branch > BRANCH_CONTEXT_GATE) return;
    mark_touched(neuron);
    branches[neuron * 4 + branch] += value;
}

// runtime.rs:719-735
void Runtime::activate_recurrent_trace(size_t slot, float a) {
    advance_recurrent_trace(slot);
    rec_branch_sens[slot] += a;
    if (!eligible_recurrent_mark[slot]) {
        eligible_recurrent_mark[slot] = 1;
        eligible_recurrent_slots.push_back(slot);
    }
}
void Runtime::activate_input_trace(size_t slot, float a) {
    advance_input_trace(slot);
    in_branch_sens[slot] += a;
    if (!eligible_input_mark[slot]) {
        eligible_input_mark[slot] = 1;
        eligible_input_slots.push_back(slot);
    }
}

// runtime.rs:737-773
void Runtime::advance_recurrent_trace(size_t slot) {
    uint64_t e = current_tick > eligibility_last_tick[slot] ? current_tick - eligibility_last_tick[slot] : 0;
    if (e == 0) return;
    const Config& c = model.config;
    rec_branch_sens[slot] *= decay_for_elapsed(c.branch_decay, e);
    rec_membrane_sens[slot] *= decay_for_elapsed(c.membrane_decay, e);
    rec_fatigue_sens[slot] *= decay_for_elapsed(c.fatigue_decay, e);
    float decays[3];
    c.adaptation_decays(decays);
    for (int i = 0; i < 3; ++i) rec_adapt_sens[i][slot] *= decay_for_elapsed(decays[i], e);
    eligibility_last_tick[slot] = current_tick;
}
void Runtime::advance_input_trace(size_t slot) {
    uint64_t e =
        current_tick > input_eligibility_last_tick[slot] ? current_tick - input_eligibility_last_tick[slot] : 0;
    if (e == 0) return;
    const Config& c = model.config;
    in_branch_sens[slot] *= decay_for_elapsed(c.branch_decay, e);
    in_membrane_sens[slot] *= decay_for_elapsed(c.membrane_decay, e);
    in_fatigue_sens[slot] *= decay_for_elapsed(c.fatigue_decay, e);
    float decays[3];
    c.adaptation_decays(decays);
    for (int i = 0; i < 3; ++i) in_adapt_sens[i][slot] *= decay_for_elapsed(decays[i], e);
    input_eligibility_last_tick[slot] = current_tick;
}

// runtime.rs:775-783
float Runtime::destination_branch_jacobian(size_t destination, uint8_t branch) const {
    size_t base = destination * 4;
    return branch_jacobian(branch, model.excitability[destination], branches[base + BRANCH_TEMPORAL],
                           branches[base + BRANCH_CONTEXT_GATE]);
}

// runtime.rs:787-803
void Runtime::cache_selection_surrogates() {
    size_t block_size = model.config.neurons_per_block;
    float width = model.config.surrogate_width, gain = model.config.surrogate_gain;
    for (size_t d : touched) {
        if (neuron_is_refractory(d)) {
            selection_surrogate[d] = 0.0f;
            continue;
        }
        float margin = membrane[d] - model.threshold[d];
        float cutoff = rmax(block_selection_cutoff[d / block_size], population_selection_cutoff);
        selection_surrogate[d] = analog_rank_surrogate(margin, cutoff, selected_mark[d] != 0, width, gain);
    }
}

// runtime.rs:805-830
void Runtime::update_forward_eligibilities() {
    float eps = model.config.eligibility_epsilon;
    size_t index = 0;
    while (index < eligible_recurrent_slots.size()) {
        size_t slot = eligible_recurrent_slots[index];
        if (update_recurrent_forward_slot(slot, eps)) {
            index += 1;
        } else {
            eligible_recurrent_mark[slot] = 0;
            eligible_recurrent_slots[index] = eligible_recurrent_slots.back();
            eligible_recurrent_slots.pop_back();
        }
    }
    index = 0;
    while (index < eligible_input_slots.size()) {
        size_t slot = eligible_input_slots[index];
        if (update_input_forward_slot(slot, eps)) {
            index += 1;
        } else {
            eligible_input_mark[slot] = 0;
            eligible_input_slots[index] = eligible_input_slots.back();
            eligible_input_slots.pop_back();
        }
    }
}

// runtime.rs:832-874
bool Runtime::update_recurrent_forward_slot(size_t slot, float epsilon) {
    advance_recurrent_trace(slot);
    size_t dest = model.recurrent_target[slot];
    uint8_t branch = model.recurrent_branch[slot];
    const Config& c = model.config;
    float e;
    if (!touched_mark[dest] || neuron_is_refractory(dest)) {
        e = eligibility[slot] * c.eligibility_decay;
    } else {
        float j = destination_branch_jacobian(dest, branch);
        float surrogate = selection_surrogate[dest];
        float adaptation_sum = sum3(rec_adapt_sens[0][slot], rec_adapt_sens[1][slot], rec_adapt_sens[2][slot]);
        float ms = rec_membrane_sens[slot] + j * rec_branch_sens[slot] - rec_fatigue_sens[slot] - adaptation_sum;
        rec_membrane_sens[slot] = ms;
        e = surrogate * ms;
    }
    eligibility[slot] = e;
    if (touched_mark[dest] && selected_mark[dest]) {
        rec_fatigue_sens[slot] += c.fatigue_gain * e;
        float gains[3];
        c.adaptation_gains(gains);
        for (int i = 0; i < 3; ++i) rec_adapt_sens[i][slot] += gains[i] * e;
    }
    float mag = rmax(rmax(rmax(std::fabs(rec_branch_sens[slot]), std::fabs(rec_membrane_sens[slot])),
                          std::fabs(rec_fatigue_sens[slot])),
                     std::fabs(e));
    for (int i = 0; i < 3; ++i) mag = rmax(mag, std::fabs(rec_adapt_sens[i][slot]));
    return mag > epsilon;
}

// runtime.rs:876-918
bool Runtime::update_input_forward_slot(size_t slot, float epsilon) {
    advance_input_trace(slot);
    size_t dest = model.input_targets[slot];
    uint8_t branch = model.input_branches[slot];
    const Config& c = model.config;
    float e;
    if (!touched_mark[dest] || neuron_is_refractory(dest)) {
        e = input_eligibility[slot] * c.eligibility_decay;
    } else {
        float j = destination_branch_jacobian(dest, branch);
        float surrogate = selection_surrogate[dest];
        float adaptation_sum = sum3(in_adapt_sens[0][slot], in_adapt_sens[1][slot], in_adapt_sens[2][slot]);
        float ms = in_membrane_sens[slot] + j * in_branch_sens[slot] - in_fatigue_sens[slot] - adaptation_sum;
        in_membrane_sens[slot] = ms;
        e = surrogate * ms;
    }
    input_eligibility[slot] = e;
    if (touched_mark[dest] && selected_mark[dest]) {
        in_fatigue_sens[slot] += c.fatigue_gain * e;
        float gains[3];
        c.adaptation_gains(gains);
        for (int i = 0; i < 3; ++i) in_adapt_sens[i][slot] += gains[i] * e;
    }
    float mag = rmax(rmax(rmax(std::fabs(in_branch_sens[slot]), std::fabs(in_membrane_sens[slot])),
                          std::fabs(in_fatigue_sens[slot])),
                     std::fabs(e));
    for (int i = 0; i < 3; ++i) mag = rmax(mag, std::fabs(in_adapt_sens[i][slot]));
    return mag > epsilon;
}

// runtime.rs:920-938
void Runtime::apply_post_activation_dynamics() {
    const Config& c = model.config;
    float gains[3];
    c.adaptation_gains(gains);
    for (size_t i = 0; i < active.size(); ++i) {
        size_t n = active[i];
        float a = activation[n];
        fatigue[n] += c.fatigue_gain * a;
        for (int k = 0; k < 3; ++k) adaptation_state[k][n] += gains[k] * a;
        membrane[n] -= model.threshold[n] * c.membrane_reset_fraction;
        refractory_until[n] = current_tick + c.refractory_ticks + 1;
    }
}

// runtime.rs:940-1074
// runtime.rs:984-997: total order of positive candidates (activation
// descending, then rotated neuron key ascending).
bool selection_better(const std::pair<size_t, float>& l, const std::pair<size_t, float>& r, size_t rotation,
                      size_t n_count) {
    if (l.second != r.second) return l.second > r.second;
    return rotated_tie_key(l.first, rotation, n_count) < rotated_tie_key(r.first, rotation, n_count);
}

// runtime.rs:964-997: a block's top `limit` candidates in rank order; when
// more are positive, *cutoff becomes the (limit + 1)-th best value.
void select_block(std::vector<std::pair<size_t, float>>& block, size_t limit, size_t rotation, size_t n_count,
                  float* cutoff) {
    auto better = [&](const std::pair<size_t, float>& l, const std::pair<size_t, float>& r) {
        return selection_better(l, r, rotation, n_count);
    };
    if (block.size() > limit) {
        std::nth_element(block.begin(), block.begin() + (long)limit, block.end(), better);
        *cutoff = block[limit].second;
        block.resize(limit);
    }
    std::sort(block.begin(), block.end(), better);
}

Runtime::SelectionMetrics Runtime::select_active_neurons() {
    const Config& c = model.config;
    size_t block_size = c.neurons_per_block;
    size_t n_count = std::max<size_t>(model.neuron_count(), 1);
    size_t rotation = (size_t)(current_tick % n_count);
    for (size_t i = 0; i < touched.size(); ++i) {
        size_t n = touched[i];
        if (neuron_is_refractory(n)) continue;
        size_t base = n * 4;
        float gate = clampf(branches[base + BRANCH_CONTEXT_GATE], 0.0f, 1.0f);
        float inhibitory = branches[base + BRANCH_INHIBITORY];
        float net = branches[base + BRANCH_EXCITATORY] + branches[base + BRANCH_TEMPORAL] * gate + inhibitory;
        float adaptation = sum3(adaptation_state[0][n], adaptation_state[1][n], adaptation_state[2][n]);
        float drive = model.excitability[n] * net - fatigue[n] - adaptation - population_inhibition;
        membrane[n] += drive;
        float act = clampf(membrane[n] - model.threshold[n], 0.0f, 1.0f);
        if (act > 0.0f) block_candidates[n / block_size].push_back({n, act});
    }
    SelectionMetrics sm;
    for (auto& b : block_candidates) sm.suprathreshold += b.size();

    size_t limit = c.max_active_per_block;
    for (size_t bi = 0; bi < block_candidates.size(); ++bi) {
        auto& block = block_candidates[bi];
        float cutoff = block_selection_cutoff[bi];
        select_block(block, limit, rotation, n_count, &cutoff);
        block_selection_cutoff[bi] = cutoff;
        for (auto& p : block) active.push_back(p.first);
    }
    sm.block_selected = active.size();
    size_t global_cap = c.max_active_global;
    size_t block_capacity = c.block_count * limit;
    if (global_cap >= block_capacity) {
        population_selection_cutoff = 0.0f;
        sm.clipped = 0;
    } else {
        auto act_of = [&](size_t n) { return clampf(membrane[n] - model.threshold[n], 0.0f, 1.0f); };
        std::sort(active.begin(), active.end(), [&](size_t l, size_t r) {
            float la = act_of(l), ra = act_of(r);
            if (la != ra) return la > ra;
            return rotated_tie_key(l, rotation, n_count) < rotated_tie_key(r, rotation, n_count);
        });
        if (active.size() > global_cap) {
            size_t cut = active[global_cap];
            population_selection_cutoff = clampf(membrane[cut] - model.threshold[cut], 0.0f, c.population_inhibition_max);
        } else {
            population_selection_cutoff = 0.0f;
        }
        size_t clipped = active.size() > global_cap ? active.size() - global_cap : 0;
        if (clipped > 0) active.resize(global_cap);
        sm.clipped = clipped;
    }
    update_population_inhibition(active.size());
    for (size_t n : active) {
        float margin = membrane[n] - model.threshold[n];
        activation[n] = clampf(margin, 0.0f, 1.0f);
        selected_mark[n] = 1;
    }
    cache_selection_surrogates();
    return sm;
}

// runtime.rs:1076-1082
void Runtime::update_population_inhibition(size_t active_neurons) {
    const Config& c = model.config;
    float activity = (float)active_neurons / (float)std::max<size_t>(model.neuron_count(), 1);
    float error = activity - c.target_activity;
    population_inhibition = clampf(population_inhibition + c.population_inhibition_rate * error, 0.0f,
                                   c.population_inhibition_max);
}

// runtime.rs:1084-1106
size_t Runtime::emit_recurrent_events() {
    size_t emitted = 0;
    for (size_t i = 0; i < active.size(); ++i) {
        size_t source = active[i];
        float a = activation[source];
        size_t start = model.slot_start(source);
        for (size_t slot = start; slot < start + model.capacity_per_neuron; ++slot) {
            size_t delay = std::max<uint8_t>(model.recurrent_delay[slot], 1);
            size_t bucket = (size_t)((current_tick + delay) % delay_ring.size());
            delay_ring[bucket].push_back(Event{model.recurrent_target[slot], model.recurrent_branch[slot],
                                               a * model.recurrent_weight[slot], (uint32_t)slot, a});
            emitted += 1;
        }
    }
    return emitted;
}

// runtime.rs:1108-1146
bool Runtime::compute_output_probabilities(long target_index, float* neural_loss) {
    std::copy(model.output_bias.begin(), model.output_bias.end(), logits.begin());
    for (size_t n : active) {
        float a = activation[n];
        size_t row = n * OUTPUT_CLASSES;
        for (size_t o = 0; o < OUTPUT_CLASSES; ++o) logits[o] += output_weights_by_neuron[row + o] * a;
    }
    bool has = target_index >= 0;
    if (has) *neural_loss = loss_from_logits((size_t)target_index);
    std::fill(context_latent.begin(), context_latent.end(), 0.0f);
    size_t d = model.config.embedding_dim;
    if (!active_context_slots.empty()) {
        for (size_t i = 0; i < active_context_slots.size(); ++i) {
            size_t slot = active_context_slots[i];
            float scale = active_context_scales[i];
            if (scale <= 0.0f) continue;
            size_t row = slot * d;
            for (size_t k = 0; k < d; ++k) context_latent[k] += model.context_embeddings[row + k] * scale;
        }
        for (size_t o = 0; o < OUTPUT_CLASSES; ++o) {
            size_t row = o * d;
            float contribution = 0.0f;
            for (size_t k = 0; k < d; ++k) contribution += model.context_output_weights[row + k] * context_latent[k];
            logits[o] += contribution;
        }
    }
    normalize_probabilities();
    return has;
}

// runtime.rs:1148-1165
float Runtime::loss_from_logits(size_t target) const {
    float maximum = -std::numeric_limits<float>::infinity();
    for (float l : logits) maximum = rmax(maximum, l);
    float sum = -0.0f;
    for (float l : logits) sum += std::exp(l - maximum);
    if (!std::isfinite(sum) || sum <= 0.0f) return std::log((float)OUTPUT_CLASSES);
    return maximum + std::log(sum) - logits[target];
}

// runtime.rs:1167-1188
void Runtime::normalize_probabilities() {
    float maximum = -std::numeric_limits<float>::infinity();
    for (float l : logits) maximum = rmax(maximum, l);
    float sum = 0.0f;
    for (size_t o = 0; o < OUTPUT_CLASSES; ++o) {
        float v = std::exp(logits[o] - maximum);
        probabilities[o] = v;
        sum += v;
    }
    if (!std::isfinite(sum) || sum <= 0.0f) {
        std::fill(probabilities.begin(), probabilities.end(), 1.0f / (float)OUTPUT_CLASSES);
    } else {
        for (auto& p : probabilities) p /= sum;
    }
}

// runtime.rs:1190-1197: max_by(total_cmp, then the lower index wins ties)
size_t Runtime::argmax_probability() const {
    size_t best = 0;
    for (size_t o = 1; o < OUTPUT_CLASSES; ++o)
        if (probabilities[o] > probabilities[best]) best = o;
    return best;
}

// runtime.rs:1199-1316
Runtime::LearningMetrics Runtime::apply_learning(size_t target_output_index, float strength, float target_weight) {
    const Config& c = model.config;
    std::copy(probabilities.begin(), probabilities.end(), errors.begin());
    errors[target_output_index] -= 1.0f;
    float supervised = strength * target_weight;
    float plasticity_scale;
    size_t next_phase;
    c.plasticity_step(plasticity_phase, target_output_index == END_OUTPUT_INDEX, &plasticity_scale, &next_phase);
    size_t n = model.neuron_count();

    for (size_t neuron : learning_destinations) {
        learning_signal[neuron] = 0.0f;
        learning_destination_mark[neuron] = 0;
    }
    learning_destinations.clear();
    if (plasticity_scale > 0.0f) {
        for (size_t slot : eligible_recurrent_slots) add_learning_destination(model.recurrent_target[slot]);
        for (size_t slot : eligible_input_slots) add_learning_destination(model.input_targets[slot]);
        for (size_t a : active) add_learning_destination(a);
        for (size_t neuron : learning_destinations) {
            size_t row = neuron * OUTPUT_CLASSES;
            float signal = 0.0f;
            for (size_t o = 0; o < OUTPUT_CLASSES; ++o) signal += output_weights_by_neuron[row + o] * errors[o];
            learning_signal[neuron] = signal;
        }
    }

    float lr = c.output_learning_rate, maxu = c.max_update, wmin = c.weight_min, wmax = c.weight_max;
    for (size_t i = 0; i < active.size(); ++i) {
        size_t neuron = active[i];
        float a = activation[neuron];
        size_t row = neuron * OUTPUT_CLASSES;
        if (track_parameter_changes) mark_changed(neuron, changed_output_neuron_mark, changed_output_neurons);
        for (size_t o = 0; o < OUTPUT_CLASSES; ++o) {
            float raw = -lr * supervised * errors[o] * a;
            float delta = bounded_delta(raw, maxu);
            float updated = clampf(model.output_weights[o * n + neuron] + delta, wmin, wmax);
            model.output_weights[o * n + neuron] = updated;
            output_weights_by_neuron[row + o] = updated;
        }
    }
    if (track_parameter_changes) output_bias_dirty = true;
    for (size_t o = 0; o < OUTPUT_CLASSES; ++o) {
        float raw = -lr * supervised * errors[o];
        model.output_bias[o] += bounded_delta(raw, maxu);
        if (!std::isfinite(model.output_bias[o])) throw LeoError(LeoError::Numerical, "output bias became non-finite");
    }
    if (context_applied_this_step) update_context_projection(supervised);

    LearningMetrics metrics;
    if (plasticity_scale > 0.0f) {
        float consolidated = supervised * plasticity_scale;
        update_recurrent_synapses(consolidated, metrics);
        update_input_synapses(consolidated, metrics);
    }
    apply_inhibitory_homeostasis(strength);
    plasticity_phase = next_phase;
    return metrics;
}

// runtime.rs:1318-1384
void Runtime::update_context_projection(float strength) {
    if (active_context_slots.empty()) return;
    const Config& c = model.config;
    float lr = c.context_learning_rate, maxu = c.max_update, wmin = c.weight_min, wmax = c.weight_max;
    size_t d = c.embedding_dim;
    std::fill(context_latent_gradient.begin(), context_latent_gradient.end(), 0.0f);
    for (size_t o = 0; o < OUTPUT_CLASSES; ++o) {
        size_t row = o * d;
        for (size_t k = 0; k < d; ++k) context_latent_gradient[k] += model.context_output_weights[row + k] * errors[o];
    }
    if (track_parameter_changes) context_output_dirty = true;
    for (size_t o = 0; o < OUTPUT_CLASSES; ++o) {
        size_t row = o * d;
        for (size_t k = 0; k < d; ++k) {
            float gradient = errors[o] * context_latent[k];
            float delta = bounded_delta(-lr * strength * gradient, maxu);
            float updated = clampf(model.context_output_weights[row + k] + delta, wmin, wmax);
            if (!std::isfinite(updated)) throw LeoError(LeoError::Numerical, "non-finite context output update rejected");
            model.context_output_weights[row + k] = updated;
        }
    }
    for (size_t i = 0; i < active_context_slots.size(); ++i) {
        size_t slot = active_context_slots[i];
        float scale = active_context_scales[i];
        size_t row = slot * d;
        for (size_t k = 0; k < d; ++k) {
            float gradient = scale * context_latent_gradient[k];
            float delta = bounded_delta(-lr * strength * gradient, maxu);
            float updated = clampf(model.context_embeddings[row + k] + delta, wmin, wmax);
            if (!std::isfinite(updated)) throw LeoError(LeoError::Internal, "non-finite context embedding update rejected");
            model.context_embeddings[row + k] = updated;
        }
        if (track_parameter_changes) mark_changed(slot, changed_context_slot_mark, changed_context_slots);
        if (model.context_observations[slot] != UINT32_MAX) model.context_observations[slot] += 1;
    }
}

void Runtime::mark_changed(size_t index, std::vector<uint8_t>& marks, std::vector<size_t>& list) {
    if (!marks[index]) {
        marks[index] = 1;
        list.push_back(index);
    }
}

// runtime.rs:1441-1448
void Runtime::add_learning_destination(size_t destination) {
    if (learning_destination_mark[destination]) return;
    learning_destination_mark[destination] = 1;
    learning_destinations.push_back(destination);
}

// runtime.rs:1451-1491
void Runtime::update_recurrent_synapses(float strength, LearningMetrics& metrics) {
    const Config& c = model.config;
    float lr = c.recurrent_learning_rate, maxu = c.max_update, wmin = c.weight_min, wmax = c.weight_max;
    for (size_t i = 0; i < eligible_recurrent_slots.size(); ++i) {
        size_t slot = eligible_recurrent_slots[i];
        size_t dest = model.recurrent_target[slot];
        float e = eligibility[slot];
        metrics.abs_sum += (double)std::fabs(e);
        metrics.count += 1;
        float gradient = learning_signal[dest] * e;
        float delta = bounded_delta(-lr * strength * gradient, maxu);
        float old_w = model.recurrent_weight[slot];
        size_t source = slot / model.capacity_per_neuron;
        float nw = clampf(old_w + delta, wmin, wmax);
        nw = model.neuron_type[source] == 0 ? rmax(nw, 0.0f) : rmin(nw, 0.0f);
        if (!std::isfinite(nw)) {
            model.statistics.numerical_rejections += 1;
            throw LeoError(LeoError::Numerical, "non-finite recurrent update rejected");
        }
        if (nw != old_w && track_parameter_changes)
            mark_changed(slot, changed_recurrent_weight_mark, changed_recurrent_weight);
        model.recurrent_weight[slot] = nw;
    }
}

// runtime.rs:1493-1523
void Runtime::update_input_synapses(float strength, LearningMetrics& metrics) {
    const Config& c = model.config;
    float lr = c.recurrent_learning_rate, maxu = c.max_update, wmax = c.weight_max;
    for (size_t i = 0; i < eligible_input_slots.size(); ++i) {
        size_t slot = eligible_input_slots[i];
        size_t dest = model.input_targets[slot];
        float e = input_eligibility[slot];
        metrics.abs_sum += (double)std::fabs(e);
        metrics.count += 1;
        float gradient = learning_signal[dest] * e;
        float delta = bounded_delta(-lr * strength * gradient, maxu);
        float old_w = model.input_weights[slot];
        float nw = clampf(old_w + delta, 0.0f, wmax);
        if (!std::isfinite(nw)) throw LeoError(LeoError::Numerical, "non-finite input update rejected");
        if (nw != old_w && track_parameter_changes) mark_changed(slot, changed_input_weight_mark, changed_input_weight);
        model.input_weights[slot] = nw;
    }
}

// runtime.rs:1525-1565
void Runtime::apply_inhibitory_homeostasis(float strength) {
    const Config& c = model.config;
    float desired = c.target_activity, lr = c.inhibitory_learning_rate, maxu = c.max_update, wmin = c.weight_min;
    for (size_t i = 0; i < active.size(); ++i) {
        size_t source = active[i];
        if (model.neuron_type[source] == 0) continue;
        float sa = activation[source];
        size_t start = model.slot_start(source);
        for (size_t slot = start; slot < start + model.capacity_per_neuron; ++slot) {
            size_t target = model.recurrent_target[slot];
            float delta = inhibitory_homeostasis_delta(sa, activation[target] > 0.0f ? 1.0f : 0.0f, desired, lr,
                                                       strength, maxu);
            float old_w = model.recurrent_weight[slot];
            float nw = clampf(old_w + delta, wmin, 0.0f);
            if (!std::isfinite(nw)) throw LeoError(LeoError::Numerical, "non-finite inhibitory update rejected");
            if (nw != old_w && track_parameter_changes)
                mark_changed(slot, changed_recurrent_weight_mark, changed_recurrent_weight);
            model.recurrent_weight[slot] = nw;
        }
    }
}

// runtime.rs:1567-1593
void Runtime::update_homeostasis(size_t active_neurons) {
    const Config& c = model.config;
    float target = c.target_activity, rate = c.threshold_homeostasis_rate;
    float pop_activity = (float)active_neurons / (float)std::max<size_t>(model.neuron_count(), 1);
    float pop_error = pop_activity - target;
    for (size_t i = 0; i < touched.size(); ++i) {
        size_t n = touched[i];
        float local = activation[n] > 0.0f ? 1.0f : 0.0f;
        float local_error = local - target;
        float dt = rate * (local_error + pop_error);
        float old_t = model.threshold[n];
        float nt = clampf(old_t + dt, 0.05f, 2.0f);
        if (nt != old_t && track_parameter_changes) mark_changed(n, changed_threshold_mark, changed_threshold);
        model.threshold[n] = nt;
    }
}

// runtime.rs:1595-1622
void Runtime::update_statistics(uint32_t symbol, bool has_loss, float loss, size_t emitted) {
    Statistics& s = model.statistics;
    if (symbol < 256) s.processed_bytes += 1;
    if (has_loss) {
        s.training_loss_sum += (double)loss;
        s.training_targets += 1;
    }
    s.active_neurons_sum += active.size();
    s.active_neurons_peak = std::max<uint64_t>(s.active_neurons_peak, active.size());
    s.synaptic_events += emitted;
    s.persistent_ticks += 1;
}

// ------------------------------------------------------------ parallel.rs
namespace {
void ensure_aligned(const Model& base, const Model& trained) {
    if (base.config.fingerprint() != trained.config.fingerprint() || base.recurrent_target != trained.recurrent_target ||
        base.recurrent_branch != trained.recurrent_branch || base.recurrent_delay != trained.recurrent_delay ||
        base.input_targets != trained.input_targets || base.input_branches != trained.input_branches ||
        base.neuron_type != trained.neuron_type)
        throw LeoError(LeoError::Internal, "worker model topology is not aligned with the canonical checkpoint");
}
// parallel.rs:884-894
std::vector<SparseF32Delta> diff_f32(const std::vector<float>& before, const std::vector<float>& after) {
    std::vector<SparseF32Delta> r;
    for (size_t i = 0; i < before.size() && i < after.size(); ++i) {
        float d = after[i] - before[i];
        if (d != 0.0f) r.push_back({i, d});
    }
    return r;
}
// parallel.rs:896-914
std::vector<SparseF32Delta> diff_selected(const std::vector<float>& before, const std::vector<float>& after,
                                          const std::vector<size_t>& indices) {
    std::vector<SparseF32Delta> r;
    for (size_t i : indices) {
        if (i >= before.size() || i >= after.size())
            throw LeoError(LeoError::Internal, "tracked parameter index is outside the model");
        float d = after[i] - before[i];
        if (d != 0.0f) r.push_back({i, d});
    }
    return r;
}
// parallel.rs:916-927
long find_context_slot(const Model& m, size_t order, uint64_t key) {
    size_t spo = m.config.slots_per_order, base = (order - 1) * spo, start = (size_t)(key % (uint64_t)spo);
    for (size_t off = 0; off < m.config.probe_limit; ++off) {
        size_t slot = base + (start + off) % spo;
        if (m.context_keys[slot] == key) return (long)slot;
    }
    return -1;
}
// parallel.rs:929-973
std::vector<ContextKeyDelta> context_deltas_for_slots(const Model& base, const Model& trained,
                                                      const std::vector<size_t>& slots) {
    size_t d = base.config.embedding_dim, spo = base.config.slots_per_order;
    std::vector<ContextKeyDelta> r;
    for (size_t slot : slots) {
        if (slot >= trained.context_keys.size()) throw LeoError(LeoError::Internal, "tracked context slot is outside the model");
        uint64_t key = trained.context_keys[slot];
        if (key == 0) continue;
        size_t order = slot / spo + 1;
        long bs = find_context_slot(base, order, key);
        uint32_t bobs = bs >= 0 ? base.context_observations[(size_t)bs] : 0;
        ContextKeyDelta cd{order, key, std::vector<float>(d), 0};
        bool changed = false;
        for (size_t k = 0; k < d; ++k) {
            float before = bs >= 0 ? base.context_embeddings[(size_t)bs * d + k] : 0.0f;
            float delta = trained.context_embeddings[slot * d + k] - before;
            changed |= delta != 0.0f;
            cd.embedding_delta[k] = delta;
        }
        uint32_t tobs = trained.context_observations[slot];
        cd.observation_increment = tobs > bobs ? tobs - bobs : 0;
        if (changed || cd.observation_increment > 0) r.push_back(std::move(cd));
    }
    return r;
}
}  // namespace

// parallel.rs:1115-1137
StatisticsDelta statistics_delta(const Statistics& b, const Statistics& a) {
    auto sat = [](uint64_t x, uint64_t y) { return x > y ? x - y : 0; };
    StatisticsDelta d;
    d.processed_bytes = sat(a.processed_bytes, b.processed_bytes);
    d.processed_stories = sat(a.processed_stories, b.processed_stories);
    d.training_loss_sum = a.training_loss_sum - b.training_loss_sum;
    d.training_targets = sat(a.training_targets, b.training_targets);
    d.active_neurons_sum = sat(a.active_neurons_sum, b.active_neurons_sum);
    d.active_neurons_peak = a.active_neurons_peak;
    d.synaptic_events = sat(a.synaptic_events, b.synaptic_events);
    d.numerical_rejections = sat(a.numerical_rejections, b.numerical_rejections);
    d.persistent_ticks = sat(a.persistent_ticks, b.persistent_ticks);
    return d;
}

// parallel.rs:313-383
SparseModelDelta SparseModelDelta::between(const Model& base, const Model& trained) {
    ensure_aligned(base, trained);
    size_t spo = base.config.slots_per_order, d = base.config.embedding_dim;
    SparseModelDelta r;
    std::unordered_map<uint64_t, size_t> base_context[17];
    for (size_t slot = 0; slot < base.context_keys.size(); ++slot)
        if (base.context_keys[slot] != 0) base_context[slot / spo + 1][base.context_keys[slot]] = slot;
    for (size_t slot = 0; slot < trained.context_keys.size(); ++slot) {
        uint64_t key = trained.context_keys[slot];
        if (key == 0) continue;
        size_t order = slot / spo + 1;
        auto it = base_context[order].find(key);
        bool has = it != base_context[order].end();
        uint32_t bobs = has ? base.context_observations[it->second] : 0;
        ContextKeyDelta cd{order, key, std::vector<float>(d), 0};
        bool changed = false;
        for (size_t k = 0; k < d; ++k) {
            float before = has ? base.context_embeddings[it->second * d + k] : 0.0f;
            float delta = trained.context_embeddings[slot * d + k] - before;
            changed |= delta != 0.0f;
            cd.embedding_delta[k] = delta;
        }
        uint32_t tobs = trained.context_observations[slot];
        cd.observation_increment = tobs > bobs ? tobs - bobs : 0;
        if (changed || cd.observation_increment > 0) r.context.push_back(std::move(cd));
    }
    r.config_fingerprint = base.config.fingerprint();
    r.base_revision = base.parameter_revision;
    r.revision_increment = trained.parameter_revision > base.parameter_revision ? trained.parameter_revision - base.parameter_revision : 0;
    r.threshold = diff_f32(base.threshold, trained.threshold);
    r.excitability = diff_f32(base.excitability, trained.excitability);
    r.recurrent_weight = diff_f32(base.recurrent_weight, trained.recurrent_weight);
    r.input_weight = diff_f32(base.input_weights, trained.input_weights);
    r.output_weight = diff_f32(base.output_weights, trained.output_weights);
    r.output_bias = diff_f32(base.output_bias, trained.output_bias);
    r.context_output_weight = diff_f32(base.context_output_weights, trained.context_output_weights);
    r.statistics = statistics_delta(base.statistics, trained.statistics);
    r.canonicalize_order();
    return r;
}

// parallel.rs:385-454
SparseModelDelta SparseModelDelta::between_tracked(const Model& base, const Model& trained, const ParameterChanges& c) {
    ensure_aligned(base, trained);
    size_t n = base.neuron_count();
    SparseModelDelta r;
    for (size_t neuron : c.output_neurons) {
        if (neuron >= n) throw LeoError(LeoError::Internal, "tracked output neuron is outside the model");
        for (size_t o = 0; o < OUTPUT_CLASSES; ++o) {
            size_t index = o * n + neuron;
            float d = trained.output_weights[index] - base.output_weights[index];
            if (d != 0.0f) r.output_weight.push_back({index, d});
        }
    }
    r.config_fingerprint = base.config.fingerprint();
    r.base_revision = base.parameter_revision;
    r.revision_increment = trained.parameter_revision > base.parameter_revision ? trained.parameter_revision - base.parameter_revision : 0;
    r.threshold = diff_selected(base.threshold, trained.threshold, c.threshold);
    r.recurrent_weight = diff_selected(base.recurrent_weight, trained.recurrent_weight, c.recurrent_weight);
    r.input_weight = diff_selected(base.input_weights, trained.input_weights, c.input_weight);
    if (c.output_bias_dirty) r.output_bias = diff_f32(base.output_bias, trained.output_bias);
    if (c.context_output_dirty) r.context_output_weight = diff_f32(base.context_output_weights, trained.context_output_weights);
    r.context = context_deltas_for_slots(base, trained, c.context_slots);
    r.statistics = statistics_delta(base.statistics, trained.statistics);
    r.canonicalize_order();
    return r;
}

// parallel.rs:676-691
void SparseModelDelta::canonicalize_order() {
    auto by_index = [](const SparseF32Delta& a, const SparseF32Delta& b) { return a.index < b.index; };
    std::sort(threshold.begin(), threshold.end(), by_index);
    std::sort(excitability.begin(), excitability.end(), by_index);
    std::sort(recurrent_weight.begin(), recurrent_weight.end(), by_index);
    std::sort(input_weight.begin(), input_weight.end(), by_index);
    std::sort(output_weight.begin(), output_weight.end(), by_index);
    std::sort(output_bias.begin(), output_bias.end(), by_index);
    std::sort(context_output_weight.begin(), context_output_weight.end(), by_index);
    std::sort(context.begin(), context.end(), [](const ContextKeyDelta& a, const ContextKeyDelta& b) {
        return a.order != b.order ? a.order < b.order : a.key < b.key;
    });
}

namespace {
// parallel.rs:975-1022
size_t apply_sparse_scaled(std::vector<float>& target, const std::vector<const std::vector<SparseF32Delta>*>& groups,
                           size_t divisor) {
    std::vector<size_t> pos(groups.size(), 0);
    size_t updates = 0;
    for (;;) {
        size_t next = SIZE_MAX;
        for (size_t g = 0; g < groups.size(); ++g)
            if (pos[g] < groups[g]->size()) next = std::min(next, (*groups[g])[pos[g]].index);
        if (next == SIZE_MAX) break;
        if (next >= target.size()) throw LeoError(LeoError::Internal, "invalid sparse worker parameter delta");
        double sum = 0.0;
        for (size_t g = 0; g < groups.size(); ++g) {
            if (pos[g] < groups[g]->size() && (*groups[g])[pos[g]].index == next) {
                float d = (*groups[g])[pos[g]].delta;
                if (!std::isfinite(d)) throw LeoError(LeoError::Internal, "invalid sparse worker parameter delta");
                sum += (double)d;
                pos[g] += 1;
            }
        }
        target[next] += (float)(sum / (double)divisor);
        if (!std::isfinite(target[next])) throw LeoError(LeoError::Internal, "merged parameter became non-finite");
        updates += 1;
    }
    return updates;
}

// parallel.rs:1024-1113
size_t apply_context_deltas(Model& master, const std::vector<SparseModelDelta>& deltas, size_t divisor) {
    struct Merged {
        size_t order;
        uint64_t key;
        std::vector<double> sum;
        uint64_t observations;
    };
    size_t d = master.config.embedding_dim;
    std::vector<size_t> pos(deltas.size(), 0);
    std::vector<Merged> merged;
    for (;;) {
        bool any = false;
        std::pair<size_t, uint64_t> next{SIZE_MAX, UINT64_MAX};
        for (size_t g = 0; g < deltas.size(); ++g) {
            if (pos[g] < deltas[g].context.size()) {
                auto& u = deltas[g].context[pos[g]];
                std::pair<size_t, uint64_t> k{u.order, u.key};
                if (!any || k < next) next = k;
                any = true;
            }
        }
        if (!any) break;
        Merged m{next.first, next.second, std::vector<double>(d, 0.0), 0};
        for (size_t g = 0; g < deltas.size(); ++g) {
            if (pos[g] < deltas[g].context.size()) {
                auto& u = deltas[g].context[pos[g]];
                if (u.order == next.first && u.key == next.second) {
                    if (u.embedding_delta.size() != d || u.order == 0 || u.order > master.config.max_order || u.key == 0)
                        throw LeoError(LeoError::Internal, "invalid keyed context worker delta");
                    for (size_t k = 0; k < d; ++k) {
                        if (!std::isfinite(u.embedding_delta[k]))
                            throw LeoError(LeoError::Internal, "invalid keyed context worker delta");
                        m.sum[k] += (double)u.embedding_delta[k];
                    }
                    m.observations += u.observation_increment;
                    pos[g] += 1;
                }
            }
        }
        merged.push_back(std::move(m));
    }
    std::sort(merged.begin(), merged.end(), [](const Merged& l, const Merged& r) {
        if (l.observations != r.observations) return l.observations > r.observations;
        if (l.order != r.order) return l.order < r.order;
        return l.key < r.key;
    });
    for (auto& u : merged) {
        long slot;
        size_t probes;
        master.resolve_context_slot(u.order, u.key, true, &slot, &probes);
        for (size_t k = 0; k < d; ++k)
            master.context_embeddings[(size_t)slot * d + k] += (float)(u.sum[k] / (double)divisor);
        uint64_t add = std::min<uint64_t>(u.observations, UINT32_MAX);
        uint64_t obs = (uint64_t)master.context_observations[(size_t)slot] + add;
        master.context_observations[(size_t)slot] = (uint32_t)std::min<uint64_t>(obs, UINT32_MAX);
    }
    return merged.size();
}

// parallel.rs:1139-1167
void apply_statistics_deltas(Statistics& s, const std::vector<SparseModelDelta>& deltas) {
    for (auto& d : deltas) {
        s.processed_bytes += d.statistics.processed_bytes;
        s.processed_stories += d.statistics.processed_stories;
        s.training_loss_sum += d.statistics.training_loss_sum;
        s.training_targets += d.statistics.training_targets;
        s.active_neurons_sum += d.statistics.active_neurons_sum;
        s.active_neurons_peak = std::max(s.active_neurons_peak, d.statistics.active_neurons_peak);
        s.synaptic_events += d.statistics.synaptic_events;
        s.numerical_rejections += d.statistics.numerical_rejections;
        s.persistent_ticks += d.statistics.persistent_ticks;
    }
}

// parallel.rs:1169-1246
void project_parameter_constraints_sparse(Model& m, const std::vector<SparseModelDelta>& deltas) {
    float lo = m.config.weight_min, hi = m.config.weight_max;
    size_t cap = m.capacity_per_neuron, d = m.config.embedding_dim;
    for (auto& delta : deltas) {
        for (auto& u : delta.threshold) m.threshold[u.index] = clampf(m.threshold[u.index], 0.05f, 2.0f);
        for (auto& u : delta.excitability) m.excitability[u.index] = clampf(m.excitability[u.index], 0.1f, 4.0f);
        for (auto& u : delta.recurrent_weight) {
            float w = clampf(m.recurrent_weight[u.index], lo, hi);
            w = m.neuron_type[u.index / cap] == 0 ? rmax(w, 0.0f) : rmin(w, 0.0f);
            m.recurrent_weight[u.index] = w;
        }
        for (auto& u : delta.input_weight) m.input_weights[u.index] = clampf(m.input_weights[u.index], 0.0f, hi);
        for (auto& u : delta.output_weight) m.output_weights[u.index] = clampf(m.output_weights[u.index], lo, hi);
        for (auto& u : delta.context) {
            long slot;
            size_t probes;
            m.resolve_context_slot(u.order, u.key, false, &slot, &probes);
            if (slot >= 0)
                for (size_t k = 0; k < d; ++k)
                    m.context_embeddings[(size_t)slot * d + k] = clampf(m.context_embeddings[(size_t)slot * d + k], lo, hi);
        }
        for (auto& u : delta.context_output_weight)
            m.context_output_weights[u.index] = clampf(m.context_output_weights[u.index], lo, hi);
    }
}

// parallel.rs:1248-1345
void validate_sparse_merge(Model& m, const std::vector<SparseModelDelta>& deltas) {
    if (!std::isfinite(m.statistics.training_loss_sum))
        throw LeoError(LeoError::Internal, "merged model statistics contain a non-finite loss");
    float lo = m.config.weight_min, hi = m.config.weight_max;
    size_t cap = m.capacity_per_neuron, d = m.config.embedding_dim;
    for (auto& delta : deltas) {
        for (auto& u : delta.threshold) {
            float v = m.threshold[u.index];
            if (!std::isfinite(v) || v < 0.05f || v > 2.0f) throw LeoError(LeoError::Internal, "merged threshold violates canonical parameter bounds");
        }
        for (auto& u : delta.recurrent_weight) {
            float w = m.recurrent_weight[u.index];
            bool sign_ok = m.neuron_type[u.index / cap] == 0 ? w >= 0.0f : w <= 0.0f;
            if (!std::isfinite(w) || w < lo || w > hi || !sign_ok)
                throw LeoError(LeoError::Internal, "merged recurrent parameter violates model constraints");
        }
        for (auto& u : delta.input_weight) {
            float w = m.input_weights[u.index];
            if (!std::isfinite(w) || w < 0.0f || w > hi) throw LeoError(LeoError::Internal, "merged input parameter violates model constraints");
        }
        for (auto& u : delta.output_weight) {
            float w = m.output_weights[u.index];
            if (!std::isfinite(w) || w < lo || w > hi) throw LeoError(LeoError::Internal, "merged output weight violates canonical parameter bounds");
        }
        for (auto& u : delta.output_bias)
            if (!std::isfinite(m.output_bias[u.index])) throw LeoError(LeoError::Internal, "merged output bias is non-finite");
        for (auto& u : delta.context) {
            long slot;
            size_t probes;
            m.resolve_context_slot(u.order, u.key, false, &slot, &probes);
            if (slot >= 0) {
                for (size_t k = 0; k < d; ++k) {
                    float v = m.context_embeddings[(size_t)slot * d + k];
                    if (!std::isfinite(v) || v < lo || v > hi)
                        throw LeoError(LeoError::Internal, "merged context embedding violates canonical parameter bounds");
                }
            }
        }
        for (auto& u : delta.context_output_weight) {
            float w = m.context_output_weights[u.index];
            if (!std::isfinite(w) || w < lo || w > hi) throw LeoError(LeoError::Internal, "merged context output weight violates canonical parameter bounds");
        }
    }
}

// parallel.rs:715-798
MergeMetrics apply_deltas_with_divisor(Model& master, const std::vector<SparseModelDelta>& deltas, size_t divisor) {
    if (deltas.empty()) throw LeoError(LeoError::Internal, "cannot merge an empty worker batch");
    if (divisor == 0) throw LeoError(LeoError::Internal, "worker merge divisor cannot be zero");
    uint64_t fp = master.config.fingerprint();
    for (auto& d : deltas)
        if (d.config_fingerprint != fp)
            throw LeoError(LeoError::Internal, "worker delta configuration does not match the canonical model");
    for (auto& d : deltas)
        if (d.base_revision != master.parameter_revision)
            throw LeoError(LeoError::Internal, "worker delta was not produced from the current canonical revision");
    auto groups = [&](auto member) {
        std::vector<const std::vector<SparseF32Delta>*> g;
        for (auto& d : deltas) g.push_back(&(d.*member));
        return g;
    };
    MergeMetrics mm;
    mm.workers = deltas.size();
    mm.fixed_parameter_updates += apply_sparse_scaled(master.threshold, groups(&SparseModelDelta::threshold), divisor);
    mm.fixed_parameter_updates += apply_sparse_scaled(master.excitability, groups(&SparseModelDelta::excitability), divisor);
    mm.fixed_parameter_updates += apply_sparse_scaled(master.recurrent_weight, groups(&SparseModelDelta::recurrent_weight), divisor);
    mm.fixed_parameter_updates += apply_sparse_scaled(master.input_weights, groups(&SparseModelDelta::input_weight), divisor);
    mm.fixed_parameter_updates += apply_sparse_scaled(master.output_weights, groups(&SparseModelDelta::output_weight), divisor);
    mm.fixed_parameter_updates += apply_sparse_scaled(master.output_bias, groups(&SparseModelDelta::output_bias), divisor);
    mm.fixed_parameter_updates +=
        apply_sparse_scaled(master.context_output_weights, groups(&SparseModelDelta::context_output_weight), divisor);
    mm.context_keys = apply_context_deltas(master, deltas, divisor);
    apply_statistics_deltas(master.statistics, deltas);
    uint64_t inc = 0;
    for (auto& d : deltas) inc += d.revision_increment;
    master.parameter_revision += inc;
    project_parameter_constraints_sparse(master, deltas);
    validate_sparse_merge(master, deltas);
    return mm;
}
}  // namespace

size_t sparse_mean_apply(std::vector<float>& target, const std::vector<std::vector<SparseF32Delta>>& stories, float lo,
                         float hi) {
    if (stories.empty()) throw LeoError(LeoError::Internal, "cannot merge an empty worker batch");
    std::vector<const std::vector<SparseF32Delta>*> groups;
    for (auto& s : stories) groups.push_back(&s);
    size_t updates = apply_sparse_scaled(target, groups, stories.size());
    // projection of parallel.rs:1226-1233 (output-weight clamp) over every delta index
    for (auto& s : stories)
        for (auto& u : s) target[u.index] = clampf(target[u.index], lo, hi);
    return updates;
}

MergeMetrics apply_mean_deltas(Model& master, const std::vector<SparseModelDelta>& deltas) {
    return apply_deltas_with_divisor(master, deltas, deltas.size());
}
MergeMetrics apply_sum_deltas(Model& master, const std::vector<SparseModelDelta>& deltas) {
    return apply_deltas_with_divisor(master, deltas, 1);
}

// ------------------------------------------------------------ training.rs
// training.rs:1782-1830
std::vector<Range> select_replay_ranges(const std::vector<float>& losses, float fraction, size_t segment_targets) {
    std::vector<Range> selected;
    if (losses.empty() || !std::isfinite(fraction) || fraction <= 0.0f || segment_targets == 0) return selected;
    size_t budget = (size_t)std::max(std::ceil((double)losses.size() * (double)std::min(fraction, 1.0f)), 1.0);
    std::vector<std::pair<size_t, float>> positions;
    for (size_t i = 0; i < losses.size(); ++i) positions.push_back({i, losses[i]});
    // total_cmp descending, then position ascending (losses are finite here or sorted by total order)
    auto total_key = [](float f) {
        int32_t b;
        std::memcpy(&b, &f, 4);
        return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
    };
    std::sort(positions.begin(), positions.end(), [&](const auto& l, const auto& r) {
        int32_t lk = total_key(l.second), rk = total_key(r.second);
        if (lk != rk) return lk > rk;
        return l.first < r.first;
    });
    size_t selected_targets = 0;
    for (auto& [position, loss] : positions) {
        if (selected_targets >= budget) break;
        if (!std::isfinite(loss) || loss <= 0.0f) continue;
        size_t remaining = budget - selected_targets;
        size_t width = std::min(std::min(segment_targets, remaining), losses.size());
        size_t start = position >= width / 2 ? position - width / 2 : 0;
        size_t end = std::min(start + width, losses.size());
        start = end >= width ? end - width : 0;
        bool overlap = false;
        for (auto& e : selected)
            if (e.start < end && start < e.end) overlap = true;
        if (overlap) continue;
        selected_targets += end - start;
        selected.push_back({start, end});
    }
    std::sort(selected.begin(), selected.end(), [](const Range& a, const Range& b) { return a.start < b.start; });
    return selected;
}

// training.rs:1729-1768
DocumentPass train_document_pass(Runtime& rt, const uint8_t* story, size_t len, Permission p) {
    DocumentPass pass;
    if (len == 0) return pass;
    rt.begin_document();
    double loss_sum = 0.0;
    for (size_t s = 0; s <= len; ++s) {
        uint32_t symbol = s == 0 ? BEGIN_DOCUMENT : story[s - 1];
        long target = s < len ? (long)story[s] : (long)END_DOCUMENT;
        StepMetrics m = rt.step(symbol, target, p);
        float loss = m.has_loss ? m.loss : 0.0f;
        pass.losses.push_back(loss);
        loss_sum += (double)loss;
        pass.steps += 1;
        pass.active_neurons_sum += m.active_neurons;
        pass.active_neurons_peak = std::max<uint64_t>(pass.active_neurons_peak, m.active_neurons);
        pass.emitted_events += m.emitted_events;
        pass.context_applied_steps += m.context_applied ? 1 : 0;
    }
    rt.finish_document();
    pass.mean_loss = loss_sum / (double)std::max<size_t>(pass.losses.size(), 1);
    return pass;
}

// training.rs:1848-1955 (classic, non-streaming replay of one target range)
void replay_target_range(Runtime& rt, const uint8_t* story, size_t len, Range range, Permission p, bool cleanup_after,
                         uint64_t* prefix_steps, uint64_t* target_steps) {
    *prefix_steps = 0;
    *target_steps = 0;
    if (len == 0 || range.start >= range.end || range.start > len) return;
    size_t end = std::min(range.end, len + 1);
    rt.begin_document();
    size_t next_target = range.start;
    if (next_target > 0) {
        rt.step(BEGIN_DOCUMENT, -1, Permission::Frozen);
        for (size_t i = 0; i + 1 < next_target; ++i) rt.step(story[i], -1, Permission::Frozen);
        *prefix_steps = next_target;
    }
    if (next_target == 0) {
        rt.step(BEGIN_DOCUMENT, story[0], p);
        *target_steps += 1;
        next_target = 1;
    }
    for (size_t pos = next_target; pos < end; ++pos) {
        uint32_t input = story[pos - 1];
        long target = pos < len ? (long)story[pos] : (long)END_DOCUMENT;
        rt.step(input, target, p);
        *target_steps += 1;
    }
    if (cleanup_after) rt.reset_transient_state();
}

// training.rs:257-393 (replay_streaming disabled, the classic path)
ReplayReport apply_replay_policy(Runtime& rt, const uint8_t* story, size_t len, const std::vector<float>& losses,
                                 Permission p) {
    ReplayReport r;
    auto ranges = select_replay_ranges(losses, rt.model.config.replay_fraction, rt.model.config.segment_bytes);
    for (size_t i = 0; i < ranges.size(); ++i) {
        uint64_t ps, ts;
        replay_target_range(rt, story, len, ranges[i], p, i + 1 == ranges.size(), &ps, &ts);
        r.replay_steps += ts;
        r.prefix_steps += ps;
    }
    r.segments = ranges.size();
    return r;
}

// training.rs:1539-1727 (CPU backend)
std::vector<SparseModelDelta> worker_story_deltas(const Model& base, const std::vector<std::vector<uint8_t>>& stories,
                                                  Permission p, size_t max_threads, std::vector<DocumentPass>& passes,
                                                  std::vector<ParameterChanges>* changes) {
    size_t count = stories.size();
    std::vector<SparseModelDelta> deltas(count);
    if (changes) changes->assign(count, ParameterChanges{});
    passes.assign(count, DocumentPass{});
    std::vector<std::string> errors(count);
    std::atomic<size_t> next{0};
    size_t threads = max_threads == 0 ? count : std::min(max_threads, count);
    auto worker = [&]() {
        for (;;) {
            size_t i = next.fetch_add(1);
            if (i >= count) return;
            try {
                Runtime w(base);  // fork: a fresh runtime (tick 0) on a copy of the canonical model
                w.enable_parameter_tracking();
                passes[i] = train_document_pass(w, stories[i].data(), stories[i].size(), p);
                deltas[i] = SparseModelDelta::between_tracked(base, w.model, w.parameter_changes());
                if (changes) (*changes)[i] = w.parameter_changes();
            } catch (const std::exception& e) {
                errors[i] = e.what();
            }
        }
    };
    std::vector<std::thread> pool;
    for (size_t t = 0; t < threads; ++t) pool.emplace_back(worker);
    for (auto& t : pool) t.join();
    for (auto& e : errors)
        if (!e.empty()) throw LeoError(LeoError::Internal, e);
    return deltas;
}

BatchReport train_story_batch(Runtime& canonical, const std::vector<std::vector<uint8_t>>& stories, Permission p,
                              size_t max_threads) {
    if (stories.empty()) throw LeoError(LeoError::Internal, "training batch cannot be empty");
    BatchReport report;
    report.stories = stories.size();
    if (stories.size() == 1) {
        DocumentPass pass = train_document_pass(canonical, stories[0].data(), stories[0].size(), p);
        report.replay = apply_replay_policy(canonical, stories[0].data(), stories[0].size(), pass.losses, p);
        report.mean_loss = pass.mean_loss;
        report.targets = pass.losses.size();
        report.merge.workers = 1;
        report.losses_by_story.push_back(pass.losses);
        report.replay_ranges.push_back(select_replay_ranges(pass.losses, canonical.model.config.replay_fraction,
                                                            canonical.model.config.segment_bytes));
        return report;
    }
    size_t count = stories.size();
    std::vector<DocumentPass> passes;
    std::vector<SparseModelDelta> deltas = worker_story_deltas(canonical.model, stories, p, max_threads, passes);
    report.merge = apply_mean_deltas(canonical.model, deltas);
    canonical.model_changed();
    canonical.reset_transient_state();
    double weighted = 0.0;
    size_t targets = 0;
    for (auto& pass : passes) {
        weighted += pass.mean_loss * (double)pass.losses.size();
        targets += pass.losses.size();
        report.losses_by_story.push_back(pass.losses);
    }
    for (size_t i = 0; i < count; ++i) {
        report.replay_ranges.push_back(select_replay_ranges(passes[i].losses, canonical.model.config.replay_fraction,
                                                            canonical.model.config.segment_bytes));
        ReplayReport rr = apply_replay_policy(canonical, stories[i].data(), stories[i].size(), passes[i].losses, p);
        report.replay.segments += rr.segments;
        report.replay.replay_steps += rr.replay_steps;
        report.replay.prefix_steps += rr.prefix_steps;
    }
    report.mean_loss = weighted / (double)std::max<size_t>(targets, 1);
    report.targets = targets;
    return report;
}

// ------------------------------------------------------------ SHA-256 (FIPS 180-4)
namespace {
const uint32_t K256[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5, 0xd807aa98,
    0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174, 0xe49b69c1, 0xefbe4786,
    0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da, 0x983e5152, 0xa831c66d, 0xb00327c8,
    0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967, 0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13,
    0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85, 0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819,
    0xd6990624, 0xf40e3585, 0x106aa070, 0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a,
    0x5b9cca4f, 0x682e6ff3, 0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7,
    0xc67178f2};
inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
}  // namespace

Sha256::Sha256() {
    const uint32_t init[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                              0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    std::memcpy(h, init, sizeof(h));
}
void Sha256::block(const uint8_t* p) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i) w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
        uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
        uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
        w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
        uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
        uint32_t ch = (e & f) ^ (~e & g);
        uint32_t t1 = hh + S1 + ch + K256[i] + w[i];
        uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
        uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
        uint32_t t2 = S0 + maj;
        hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}
void Sha256::update(const void* data, size_t len) {
    const uint8_t* p = (const uint8_t*)data;
    total += len;
    while (len > 0) {
        size_t take = std::min(len, 64 - fill);
        std::memcpy(buf + fill, p, take);
        fill += take;
        p += take;
        len -= take;
        if (fill == 64) {
            block(buf);
            fill = 0;
        }
    }
}
void Sha256::finalize(uint8_t out[32]) {
    uint64_t bits = total * 8;
    uint8_t pad = 0x80;
    update(&pad, 1);
    uint8_t zero = 0;
    while (fill != 56) update(&zero, 1);
    uint8_t lenb[8];
    for (int i = 0; i < 8; ++i) lenb[i] = (uint8_t)(bits >> (56 - 8 * i));
    update(lenb, 8);
    for (int i = 0; i < 8; ++i) {
        out[4 * i] = (uint8_t)(h[i] >> 24);
        out[4 * i + 1] = (uint8_t)(h[i] >> 16);
        out[4 * i + 2] = (uint8_t)(h[i] >> 8);
        out[4 * i + 3] = (uint8_t)h[i];
    }
}
void sha256(const uint8_t* data, size_t len, uint8_t out[32]) {
    Sha256 s;
    s.update(data, len);
    s.finalize(out);
}

// crates/leo-cli/src/main.rs:1151-1185 (little-endian value bytes in this order)
void model_state_hash(const Model& m, uint8_t out[32]) {
    Sha256 s;
    const std::vector<float>* fv[] = {&m.recurrent_weight, &m.input_weights, &m.output_weights, &m.output_bias,
                                      &m.context_embeddings, &m.context_output_weights, &m.threshold, &m.excitability};
    for (auto* v : fv) s.update(v->data(), v->size() * 4);
    s.update(m.recurrent_target.data(), m.recurrent_target.size() * 4);
    s.update(m.recurrent_branch.data(), m.recurrent_branch.size());
    s.update(m.recurrent_delay.data(), m.recurrent_delay.size());
    s.update(m.input_targets.data(), m.input_targets.size() * 4);
    s.update(m.input_branches.data(), m.input_branches.size());
    s.update(m.neuron_type.data(), m.neuron_type.size());
    s.update(m.context_keys.data(), m.context_keys.size() * 8);
    s.update(m.context_observations.data(), m.context_observations.size() * 4);
    s.finalize(out);
}

// crates/leo-cli/src/main.rs:1187-1202
void training_state_hash(const Model& m, uint8_t out[32]) {
    uint8_t inner[32];
    model_state_hash(m, inner);
    Sha256 s;
    s.update(inner, 32);
    s.update(&m.generation, 8);
    s.update(&m.parameter_revision, 8);
    const Statistics& st = m.statistics;
    s.update(&st.processed_bytes, 8);
    s.update(&st.processed_stories, 8);
    s.update(&st.training_loss_sum, 8);
    s.update(&st.training_targets, 8);
    s.update(&st.active_neurons_sum, 8);
    s.update(&st.active_neurons_peak, 8);
    s.update(&st.synaptic_events, 8);
    s.update(&st.numerical_rejections, 8);
    s.update(&st.persistent_ticks, 8);
    s.finalize(out);
}

}  // namespace leo_oracle
