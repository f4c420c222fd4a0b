// Internal host-side declarations shared by the C-ABI implementation files.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "../../include/leo_b200_types.h"

namespace leo_host {

void initialize_model(const LeoB200Config& cfg, int topology, LeoB200HostModel& m);
void training_state_hash(const LeoB200HostModel& m, uint8_t out[32]);

struct Sha256 {
    uint32_t h[8];
    uint8_t buf[64];
    uint64_t total = 0;
    size_t fill = 0;
    Sha256();
    void update(const void* data, size_t len);
    void finalize(uint8_t out[32]);
    void compress(const uint8_t* p);
};

struct ModelSizes {
    size_t n, s, f, d, ctx, synapses, inputs, outputs, ctx_emb, ctx_out;
};
inline ModelSizes sizes_of(const LeoB200Config& c) {
    ModelSizes z;
    z.n = c.abi.neuron_count;
    z.s = c.abi.synapses_per_neuron;
    z.f = c.abi.input_fanout;
    z.d = c.abi.context_embedding_dim;
    z.ctx = (size_t)c.abi.context_max_order * c.abi.context_slots_per_order;
    z.synapses = z.n * z.s;
    z.inputs = LEO_B200_SYMBOL_COUNT * z.f;
    z.outputs = LEO_B200_OUTPUT_CLASSES * z.n;
    z.ctx_emb = z.ctx * z.d;
    z.ctx_out = LEO_B200_OUTPUT_CLASSES * z.d;
    return z;
}

// Validation of the configuration as in crates/leo-core/src/config.rs:250-519;
// returns an empty string on success.
const char* validate_config(const LeoB200Config& c);
// crates/leo-core/src/model.rs:223-396; returns an empty string on success.
const char* validate_model(const LeoB200HostModel& m);

}  // namespace leo_host
