// CPU check of the kernels' exp/ln reproduction (leo_b200/csrc/leo_math.cuh
// with the generated exception tables): for random float inputs in the
// domains the per-byte step uses, "table value if listed, else one rounding of
// the double evaluation" must equal the platform libm bit for bit, as the
// reference's f32::exp / f32::ln (glibc expf / logf) produce.
// Usage: libm_check <samples> <seed>; prints "mismatches=<n> checked=<m>".
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>

#include "leo_math.cuh"
#include "libm_tables.inc"

static float f_from(uint32_t b) {
    float f;
    std::memcpy(&f, &b, 4);
    return f;
}
static uint32_t b_from(float f) {
    uint32_t b;
    std::memcpy(&b, &f, 4);
    return b;
}

static float kernel_exp(float x) {
    uint32_t out;
    if (leo_math::table_lookup(leo_exp_exception_keys, leo_exp_exception_values, LEO_EXP_EXCEPTIONS, b_from(x), &out))
        return f_from(out);
    return leo_math::double_to_float_rn(leo_math::exp_double((double)x));
}

static float kernel_log(float x) {
    uint32_t out;
    if (leo_math::table_lookup(leo_log_exception_keys, leo_log_exception_values, LEO_LOG_EXCEPTIONS, b_from(x), &out))
        return f_from(out);
    return leo_math::double_to_float_rn(leo_math::log_double_of_float(x));
}

int main(int argc, char** argv) {
    long samples = argc > 1 ? std::atol(argv[1]) : 1000000;
    unsigned seed = argc > 2 ? (unsigned)std::atol(argv[2]) : 1;
    std::mt19937_64 rng(seed);
    uint32_t exp_hi = b_from(-150.0f), log_lo = b_from(1.0e-12f), log_hi = b_from(1.0f);
    long bad = 0, checked = 0;
    for (long i = 0; i < samples; ++i) {
        uint32_t eb = 0x80000000u + (uint32_t)(rng() % (uint64_t)(exp_hi - 0x80000000u + 1));
        float x = f_from(eb);
        if (b_from(kernel_exp(x)) != b_from(std::exp(x))) ++bad;
        uint32_t lb = log_lo + (uint32_t)(rng() % (uint64_t)(log_hi - log_lo + 1));
        float y = f_from(lb);
        if (b_from(kernel_log(y)) != b_from(std::log(y))) ++bad;
        checked += 2;
    }
    // Every listed exception must reproduce libm, and stay within one ulp of
    // the double evaluation (libm is off by at most one rounding there).
    for (int i = 0; i < LEO_EXP_EXCEPTIONS; ++i) {
        float x = f_from(leo_exp_exception_keys[i]);
        if (b_from(kernel_exp(x)) != b_from(std::exp(x))) ++bad;
        float ours = leo_math::double_to_float_rn(leo_math::exp_double((double)x));
        if (std::abs((int64_t)b_from(ours) - (int64_t)b_from(std::exp(x))) > 1) ++bad;
        ++checked;
    }
    for (int i = 0; i < LEO_LOG_EXCEPTIONS; ++i) {
        float x = f_from(leo_log_exception_keys[i]);
        if (b_from(kernel_log(x)) != b_from(std::log(x))) ++bad;
        float ours = leo_math::double_to_float_rn(leo_math::log_double_of_float(x));
        if (std::abs((int64_t)b_from(ours) - (int64_t)b_from(std::log(x))) > 1) ++bad;
        ++checked;
    }
    // Edge inputs of the softmax and loss.
    const float edges[] = {-0.0f, 0.0f, -1.0e-30f, -87.0f, -103.9f, -149.9f, -150.0f};
    for (float x : edges) {
        if (b_from(kernel_exp(x)) != b_from(std::exp(x))) ++bad;
        ++checked;
    }
    const float log_edges[] = {1.0e-12f, 1.0f, 0.5f, 0.999999f, 1.0e-6f};
    for (float x : log_edges) {
        if (b_from(kernel_log(x)) != b_from(std::log(x))) ++bad;
        ++checked;
    }
    std::printf("mismatches=%ld checked=%ld exp_exceptions=%d log_exceptions=%d\n", bad, checked,
                (int)LEO_EXP_EXCEPTIONS, (int)LEO_LOG_EXCEPTIONS);
    return bad == 0 ? 0 : 1;
}
