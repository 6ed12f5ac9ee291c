// Offline host preparation (f64 quantisers, code tables, synthetic inputs); see host_prep.cpp.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <vector>

namespace hp {

struct HScale {
    int64_t mant;
    int32_t shift;
};

struct HTable {
    std::vector<int64_t> codes;
    HScale inv_step;
    int64_t lo_index;
    HScale code_scale;
};

HScale scale_from_f64(double x);
void quantize_weights(const float* w, size_t n, int32_t* codes, HScale* scale);
bool quantize_bias(const float* b, size_t n, int64_t* codes, HScale* scale);
void code_sigmoid_bias(const float* b, size_t n, int64_t* codes);
void from_reals(const float* v, size_t n, int32_t* data, HScale* scale);
void build_table(int kind, HTable* t);
void synth_normal(uint64_t seed, float sigma, uint64_t offset, size_t n, float* out);
void lcg_uniform(uint64_t seed, int64_t lo, int64_t hi, size_t n, int32_t* out);

}  // namespace hp
