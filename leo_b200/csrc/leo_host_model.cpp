// Host-side model construction, validation and state digest for the C ABI.
//
// Model::initialize (crates/leo-core/src/model.rs:79-158, rng.rs:1-43) builds
// the reference topology; the synthetic benchmark topologies replace only the
// recurrent fan-out block (uniform or Zipf(1.1) targets, |N(0, 1/sqrt(S))|
// weights signed by source type).  The state digest is the reference's
// training_state_hash (crates/leo-cli/src/main.rs:1151-1202) over SHA-256
// (FIPS 180-4).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

#include "leo_host.h"

namespace leo_host {

namespace {

struct SplitMix64 {  // rng.rs:13-36
    uint64_t state;
    explicit SplitMix64(uint64_t s) : state(s) {}
    uint64_t next_u64() {
        state += 0x9E3779B97F4A7C15ull;
        uint64_t v = state;
        v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ull;
        v = (v ^ (v >> 27)) * 0x94D049BB133111EBull;
        return v ^ (v >> 31);
    }
    float next_f32() { return (float)(uint32_t)(next_u64() >> 40) / (float)((1u << 24) - 1); }
    size_t range(size_t upper) { return upper <= 1 ? 0 : (size_t)(next_u64() % (uint64_t)upper); }
    float range_f32(float lo, float hi) { return lo + (hi - lo) * next_f32(); }
    double unit_double() { return (double)(next_u64() >> 11) * (1.0 / 9007199254740992.0); }
};

uint8_t sample_delay(SplitMix64& rng) {  // model.rs:498-505
    size_t r = rng.range(100);
    return r <= 49 ? 1 : (r <= 74 ? 2 : (r <= 89 ? 4 : 8));
}

uint8_t excitatory_branch(SplitMix64& rng) {
    size_t r = rng.range(3);
    return r == 0 ? 0 : (r == 1 ? 2 : 3);
}

}  // namespace

void initialize_model(const LeoB200Config& cfg, int topology, LeoB200HostModel& m) {
    const LeoConfig& a = cfg.abi;
    size_t n = a.neuron_count, cap = a.synapses_per_neuron, f = a.input_fanout, d = a.context_embedding_dim;
    size_t ctx = (size_t)a.context_max_order * a.context_slots_per_order;
    SplitMix64 rng(cfg.host.seed);
    // neuron types (model.rs:102-109)
    std::vector<size_t> ids(n);
    for (size_t i = 0; i < n; ++i) ids[i] = i;
    for (size_t i = n; i-- > 1;) std::swap(ids[i], ids[rng.range(i + 1)]);
    size_t inhibitory = (size_t)std::round((1.0f - cfg.host.excitatory_fraction) * (float)n);
    std::fill(m.neuron_type, m.neuron_type + n, 0);
    for (size_t i = 0; i < inhibitory && i < n; ++i) m.neuron_type[ids[i]] = 1;
    for (size_t i = 0; i < n; ++i) m.excitability[i] = 1.0f;
    for (size_t i = 0; i < n; ++i) m.threshold[i] = rng.range_f32(0.45f, 0.55f);

    if (topology == LEO_B200_TOPOLOGY_REFERENCE) {
        // model.rs:399-459
        size_t block_size = a.neurons_per_block, local_count = (cap * 3) / 4;
        for (size_t src = 0; src < n; ++src) {
            std::set<std::pair<size_t, uint8_t>> used;
            size_t src_block = src / block_size;
            for (size_t local = 0; local < cap; ++local) {
                size_t slot = src * cap + local;
                bool found = false;
                size_t target = 0;
                uint8_t branch = 0;
                for (int attempt = 0; attempt < 128 && !found; ++attempt) {
                    size_t t;
                    if (local < local_count) {
                        long delta = (long)rng.range(3) - 1;
                        long blk = std::clamp((long)src_block + delta, 0L, (long)a.block_count - 1);
                        t = (size_t)blk * block_size + rng.range(block_size);
                    } else {
                        t = rng.range(n);
                    }
                    uint8_t b = m.neuron_type[src] == 0 ? excitatory_branch(rng) : 1;
                    if (t == src && b != 2) continue;
                    if (used.insert({t, b}).second) {
                        target = t;
                        branch = b;
                        found = true;
                    }
                }
                if (!found) throw std::runtime_error("could not initialize unique synapse");
                m.recurrent_target[slot] = (uint32_t)target;
                m.recurrent_branch[slot] = branch;
                m.recurrent_delay[slot] = sample_delay(rng);
                m.recurrent_weight[slot] =
                    m.neuron_type[src] == 0 ? rng.range_f32(0.01f, 0.08f) : rng.range_f32(-0.08f, -0.01f);
            }
        }
    } else {
        std::vector<double> cdf;
        std::vector<uint32_t> rank_to_neuron;
        if (topology == LEO_B200_TOPOLOGY_ZIPF) {
            cdf.resize(n);
            double acc = 0.0;
            for (size_t k = 0; k < n; ++k) {
                acc += std::pow((double)(k + 1), -1.1);
                cdf[k] = acc;
            }
            for (size_t k = 0; k < n; ++k) cdf[k] /= acc;
            rank_to_neuron.resize(n);
            for (size_t k = 0; k < n; ++k) rank_to_neuron[k] = (uint32_t)k;
            for (size_t i = n; i-- > 1;) std::swap(rank_to_neuron[i], rank_to_neuron[rng.range(i + 1)]);
        }
        double sigma = 1.0 / std::sqrt((double)cap);
        for (size_t src = 0; src < n; ++src) {
            std::set<std::pair<size_t, uint8_t>> used;
            for (size_t local = 0; local < cap; ++local) {
                size_t slot = src * cap + local;
                bool found = false;
                size_t target = 0;
                uint8_t branch = 0;
                for (int attempt = 0; attempt < 256 && !found; ++attempt) {
                    size_t t;
                    if (topology == LEO_B200_TOPOLOGY_ZIPF && attempt < 128) {
                        double u = rng.unit_double();
                        size_t k = (size_t)(std::lower_bound(cdf.begin(), cdf.end(), u) - cdf.begin());
                        t = rank_to_neuron[std::min(k, n - 1)];
                    } else {
                        t = rng.range(n);
                    }
                    uint8_t b = m.neuron_type[src] == 0 ? excitatory_branch(rng) : 1;
                    if (t == src && b != 2) continue;
                    if (used.insert({t, b}).second) {
                        target = t;
                        branch = b;
                        found = true;
                    }
                }
                if (!found) throw std::runtime_error("could not initialize unique synapse");
                m.recurrent_target[slot] = (uint32_t)target;
                m.recurrent_branch[slot] = branch;
                m.recurrent_delay[slot] = sample_delay(rng);
                double u1 = ((double)(rng.next_u64() >> 11) + 1.0) * (1.0 / 9007199254740992.0);
                double u2 = rng.unit_double();
                double z = std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
                float w = (float)std::fabs(z * sigma);
                m.recurrent_weight[slot] =
                    m.neuron_type[src] == 0 ? std::min(w, a.weight_max) : std::max(-w, a.weight_min);
            }
        }
    }
    // model.rs:461-496
    for (size_t symbol = 0; symbol < LEO_B200_SYMBOL_COUNT; ++symbol) {
        std::set<size_t> used;
        for (size_t index = 0; index < f; ++index) {
            size_t t;
            do {
                t = rng.range(n);
            } while (!used.insert(t).second);
            size_t off = symbol * f + index;
            m.input_target[off] = (uint32_t)t;
            size_t r = index % 8;
            m.input_branch[off] = r == 6 ? 2 : (r == 7 ? 3 : 0);
            m.input_weight[off] = rng.range_f32(0.05f, 0.20f);
        }
    }
    for (size_t i = 0; i < LEO_B200_OUTPUT_CLASSES * n; ++i) m.output_weight[i] = rng.range_f32(-0.005f, 0.005f);
    for (size_t i = 0; i < LEO_B200_OUTPUT_CLASSES * d; ++i) m.context_output_weight[i] = rng.range_f32(-0.005f, 0.005f);
    for (size_t i = 0; i < LEO_B200_OUTPUT_CLASSES; ++i) m.output_bias[i] = 0.0f;
    std::memset(m.context_keys, 0, ctx * sizeof(uint64_t));
    std::memset(m.context_observations, 0, ctx * sizeof(uint32_t));
    std::memset(m.context_embeddings, 0, ctx * d * sizeof(float));
    m.generation = 0;
    m.parameter_revision = 0;
    std::memset(&m.statistics, 0, sizeof(m.statistics));
}

// ---------------------------------------------------------------- SHA-256
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
inline uint32_t rotr(uint32_t x, int k) { return (x >> k) | (x << (32 - k)); }
}  // namespace

Sha256::Sha256() {
    const uint32_t init[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                              0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    std::memcpy(h, init, sizeof(h));
}
void Sha256::compress(const uint8_t* p) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
        w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
        uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
        uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
        w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
        uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + K256[i] + w[i];
        uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
        hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}
void Sha256::update(const void* data, size_t len) {
    const uint8_t* p = (const uint8_t*)data;
    total += len;
    if (fill) {
        size_t take = std::min(len, 64 - fill);
        std::memcpy(buf + fill, p, take);
        fill += take; p += take; len -= take;
        if (fill == 64) { compress(buf); fill = 0; }
    }
    while (len >= 64) { compress(p); p += 64; len -= 64; }
    if (len) { std::memcpy(buf, p, len); fill = len; }
}
void Sha256::finalize(uint8_t out[32]) {
    uint64_t bits = total * 8;
    uint8_t pad[72] = {0x80};
    size_t padlen = (fill < 56 ? 56 - fill : 120 - fill);
    uint8_t lenb[8];
    for (int i = 0; i < 8; ++i) lenb[i] = (uint8_t)(bits >> (56 - 8 * i));
    update(pad, padlen);
    update(lenb, 8);
    for (int i = 0; i < 8; ++i) {
        out[4 * i] = (uint8_t)(h[i] >> 24); out[4 * i + 1] = (uint8_t)(h[i] >> 16);
        out[4 * i + 2] = (uint8_t)(h[i] >> 8); out[4 * i + 3] = (uint8_t)h[i];
    }
}

// crates/leo-cli/src/main.rs:1151-1202
void training_state_hash(const LeoB200HostModel& m, uint8_t out[32]) {
    const LeoConfig& a = m.config.abi;
    size_t n = a.neuron_count, syn = n * a.synapses_per_neuron, in = LEO_B200_SYMBOL_COUNT * (size_t)a.input_fanout;
    size_t d = a.context_embedding_dim, ctx = (size_t)a.context_max_order * a.context_slots_per_order;
    Sha256 s;
    s.update(m.recurrent_weight, syn * 4);
    s.update(m.input_weight, in * 4);
    s.update(m.output_weight, LEO_B200_OUTPUT_CLASSES * n * 4);
    s.update(m.output_bias, LEO_B200_OUTPUT_CLASSES * 4);
    s.update(m.context_embeddings, ctx * d * 4);
    s.update(m.context_output_weight, LEO_B200_OUTPUT_CLASSES * d * 4);
    s.update(m.threshold, n * 4);
    s.update(m.excitability, n * 4);
    s.update(m.recurrent_target, syn * 4);
    s.update(m.recurrent_branch, syn);
    s.update(m.recurrent_delay, syn);
    s.update(m.input_target, in * 4);
    s.update(m.input_branch, in);
    s.update(m.neuron_type, n);
    s.update(m.context_keys, ctx * 8);
    s.update(m.context_observations, ctx * 4);
    uint8_t inner[32];
    s.finalize(inner);
    Sha256 t;
    t.update(inner, 32);
    t.update(&m.generation, 8);
    t.update(&m.parameter_revision, 8);
    const LeoB200Statistics& st = m.statistics;
    t.update(&st.processed_bytes, 8);
    t.update(&st.processed_stories, 8);
    t.update(&st.training_loss_sum, 8);
    t.update(&st.training_targets, 8);
    t.update(&st.active_neurons_sum, 8);
    t.update(&st.active_neurons_peak, 8);
    t.update(&st.synaptic_events, 8);
    t.update(&st.numerical_rejections, 8);
    t.update(&st.persistent_ticks, 8);
    t.finalize(out);
}

}  // namespace leo_host

namespace leo_host {

// crates/leo-core/src/config.rs:250-519 (the fields this path uses), plus the
// device limits of this backend (block winners and actives per tick <= 1024).
const char* validate_config(const LeoB200Config& c) {
    const LeoConfig& a = c.abi;
    auto unit = [](float v) { return std::isfinite(v) && v >= 0.0f && v < 1.0f; };
    auto pos = [](float v) { return std::isfinite(v) && v > 0.0f; };
    if (a.neuron_count == 0 || a.block_count == 0 || a.neurons_per_block == 0) return "model dimensions must be positive";
    if ((uint64_t)a.block_count * a.neurons_per_block != a.neuron_count)
        return "block_count * neurons_per_block must equal neuron_count without overflow";
    if (a.branches_per_neuron != 4) return "Leo requires exactly four dendritic branches per neuron";
    if (!unit(c.host.excitatory_fraction)) return "excitatory_fraction must be finite and strictly between 0 and 1";
    if (a.synapses_per_neuron == 0 || a.input_fanout == 0) return "synapses_per_neuron and input_fanout must be positive";
    if (a.synapses_per_neuron > a.neuron_count) return "synapses_per_neuron cannot exceed neuron_count";
    if (a.input_fanout > a.neuron_count) return "input_fanout cannot exceed neuron_count";
    if (a.max_active_per_block == 0 || a.max_active_per_block > a.neurons_per_block)
        return "max_active_per_block must be in 1..=neurons_per_block";
    if (a.max_active_global == 0 || a.max_active_global > a.neuron_count) return "max_active_global must be in 1..=neuron_count";
    if (a.refractory_ticks == 0) return "refractory_ticks must be positive in the integrated architecture";
    const float decays[] = {a.branch_decay, a.membrane_decay, a.fatigue_decay, a.adaptation_fast_decay,
                            a.adaptation_medium_decay, a.adaptation_slow_decay, a.eligibility_decay};
    for (float v : decays)
        if (!unit(v)) return "decays must be finite and strictly between 0 and 1";
    const float rates[] = {a.fatigue_gain, a.adaptation_fast_gain, a.adaptation_medium_gain, a.adaptation_slow_gain,
                           a.threshold_homeostasis_rate, a.population_inhibition_rate, a.output_learning_rate,
                           a.recurrent_learning_rate, a.inhibitory_learning_rate, a.eligibility_epsilon,
                           a.surrogate_width, a.surrogate_gain, a.max_update};
    for (float v : rates)
        if (!pos(v)) return "rates must be finite and positive";
    if (!std::isfinite(a.target_activity) || !(a.target_activity > 0.0f && a.target_activity <= 1.0f))
        return "target_activity must be finite and in (0, 1]";
    if (!pos(a.population_inhibition_max)) return "population_inhibition_max must be finite and positive";
    if (!std::isfinite(a.membrane_reset_fraction) || !(a.membrane_reset_fraction > 0.0f && a.membrane_reset_fraction <= 1.0f))
        return "membrane_reset_fraction must be finite and in (0, 1]";
    if ((size_t)std::ceil(a.target_activity * (float)a.neuron_count) > a.max_active_global)
        return "target_activity requires more neurons than max_active_global permits";
    if (a.weight_min >= 0.0f || a.weight_max <= 0.0f || a.weight_min >= a.weight_max)
        return "weight_min must be negative and weight_max must be positive";
    if (c.host.plasticity_window == 0 || c.host.plasticity_window > 64) return "learning.plasticity_window must be in 1..=64";
    if (!std::isfinite(c.host.end_document_weight) || !(c.host.end_document_weight >= 1.0f && c.host.end_document_weight <= 16.0f))
        return "end_document_weight must be finite and in [1, 16]";
    const float strengths[] = {c.host.provisional_strength, c.host.training_strength, c.host.verified_strength};
    for (float v : strengths)
        if (!std::isfinite(v) || !(v > 0.0f && v <= 1.0f)) return "permission strengths must be finite and in (0, 1]";
    if (a.context_max_order == 0 || a.context_embedding_dim == 0 || a.context_slots_per_order == 0 ||
        a.context_probe_limit == 0 || a.context_confidence_observations == 0)
        return "all context-memory dimensions must be positive";
    if (a.context_embedding_dim > 256) return "context.embedding_dim cannot exceed 256";
    if (a.context_max_order > 16) return "context.max_order cannot exceed 16";
    if (a.context_probe_limit > a.context_slots_per_order) return "context.probe_limit cannot exceed slots_per_order";
    if (!std::isfinite(c.host.context_dropout_rate) || !(c.host.context_dropout_rate >= 0.0f && c.host.context_dropout_rate < 1.0f))
        return "context.dropout_rate must be finite and in [0, 1)";
    if (!pos(a.context_learning_rate)) return "context.learning_rate must be finite and positive";
    if (!std::isfinite(c.host.replay_fraction) || c.host.replay_fraction < 0.0f || c.host.replay_fraction > 1.0f)
        return "replay.fraction must be finite and in the interval [0, 1]";
    if (c.host.replay_segment_bytes == 0) return "all replay limits must be positive";
    // Device limits of this backend.
    if ((uint64_t)a.block_count * a.max_active_per_block > 2048) return "block_count * max_active_per_block exceeds 2048";
    if (a.block_count > 1024) return "block_count exceeds 1024";
    if (a.max_active_global > 1024) return "max_active_global exceeds 1024";
    if (a.neuron_count >= (1u << 24)) return "neuron_count must be below 2^24";
    return "";
}

// crates/leo-core/src/model.rs:223-396
const char* validate_model(const LeoB200HostModel& m) {
    const char* e = validate_config(m.config);
    if (*e) return e;
    ModelSizes z = sizes_of(m.config);
    float wmin = m.config.abi.weight_min, wmax = m.config.abi.weight_max;
    auto finite = [](const float* p, size_t n) {
        for (size_t i = 0; i < n; ++i)
            if (!std::isfinite(p[i])) return false;
        return true;
    };
    if (!finite(m.threshold, z.n) || !finite(m.excitability, z.n) || !finite(m.recurrent_weight, z.synapses) ||
        !finite(m.input_weight, z.inputs) || !finite(m.output_weight, z.outputs) ||
        !finite(m.output_bias, LEO_B200_OUTPUT_CLASSES) || !finite(m.context_embeddings, z.ctx_emb) ||
        !finite(m.context_output_weight, z.ctx_out) || !std::isfinite(m.statistics.training_loss_sum))
        return "model contains NaN or infinite values";
    for (size_t i = 0; i < z.n; ++i)
        if (m.threshold[i] < 0.05f || m.threshold[i] > 2.0f) return "neuron thresholds violate canonical parameter bounds";
    for (size_t i = 0; i < z.n; ++i)
        if (m.excitability[i] < 0.1f || m.excitability[i] > 4.0f) return "neuron excitability violates canonical parameter bounds";
    auto bounded = [&](const float* p, size_t n) {
        for (size_t i = 0; i < n; ++i)
            if (p[i] < wmin || p[i] > wmax) return false;
        return true;
    };
    if (!bounded(m.output_weight, z.outputs) || !bounded(m.context_embeddings, z.ctx_emb) ||
        !bounded(m.context_output_weight, z.ctx_out))
        return "learned projection weights violate canonical parameter bounds";
    for (size_t i = 0; i < z.ctx; ++i)
        if (m.context_keys[i] == 0 && m.context_observations[i] != 0) return "empty context slots cannot contain observations";
    for (size_t i = 0; i < z.n; ++i)
        if (m.neuron_type[i] > 1) return "neuron types must be excitatory or inhibitory";
    for (size_t src = 0; src < z.n; ++src) {
        for (size_t slot = src * z.s; slot < (src + 1) * z.s; ++slot) {
            uint32_t t = m.recurrent_target[slot];
            uint8_t b = m.recurrent_branch[slot], d = m.recurrent_delay[slot];
            float w = m.recurrent_weight[slot];
            if (t >= z.n) return "recurrent slot targets a neuron outside the model";
            if (b > 3 || !(d == 1 || d == 2 || d == 4 || d == 8)) return "recurrent slot has invalid branch or delay";
            if (w < wmin || w > wmax) return "recurrent slot has invalid weight";
            if (m.neuron_type[src] == 0 ? (w < 0.0f || b == 1) : (w > 0.0f || b != 1))
                return "recurrent slot is incompatible with its source type";
        }
    }
    for (size_t i = 0; i < z.inputs; ++i)
        if (m.input_target[i] >= z.n || m.input_branch[i] == 1 || m.input_branch[i] > 3 || m.input_weight[i] < 0.0f ||
            m.input_weight[i] > wmax)
            return "input projection slot has invalid state";
    return "";
}

}  // namespace leo_host
