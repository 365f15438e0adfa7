// The reference's seeded untrained model (gat_b200_random_model).
//
// Compiled with -O3 -mfma (see build.py): std::normal_distribution<float> is
// inline library code whose rounding depends on FMA contraction, and these are
// the flags the reference's sources are built with here (oracle/Makefile), so
// the values are bit-identical to the reference's random_model
// (baseline/src/common.cpp:50-62).
#include "gat_b200_internal.h"

#include <cmath>
#include <random>

using namespace gatb;

extern "C" {

int gat_b200_random_model(int din, int classes, int seed, float* const* w, float* const* al,
                          float* const* ar) {
    if (din <= 0 || classes <= 0 || classes > 64) return fail("invalid parameter shape (heads <=8, head_dim <=64)");
    for (int l = 0; l < 3; ++l) {
        // Layer shapes of the reference model (baseline/src/common.cpp:53).
        int in = l ? 256 : din, heads = l < 2 ? 8 : 1, dim = l < 2 ? 32 : classes;
        // Same engine, distribution and draw order as the reference's generator,
        // so the values are bit-identical under the same C++ standard library.
        std::mt19937 rng(seed + 11 * l);
        std::normal_distribution<float> norm;
        uint64_t width = uint64_t(heads) * dim;
        for (uint64_t i = 0; i < uint64_t(in) * width; ++i) w[l][i] = norm(rng) / std::sqrt(float(in));
        for (uint64_t i = 0; i < width; ++i) al[l][i] = norm(rng) / std::sqrt(float(dim));
        for (uint64_t i = 0; i < width; ++i) ar[l][i] = norm(rng) / std::sqrt(float(dim));
    }
    return 0;
}

}  // extern "C"
