// Seeded parameters of the reference's tests and model (test infrastructure).
// C++ because the reference draws them with std::mt19937 and <random>
// distributions; compiled with the same standard library and the flags the
// reference's sources get in oracle/Makefile (-O3 -mfma: the distributions are
// inline code whose rounding depends on FMA contraction), the values are
// bit-identical to the reference's.
#include <cmath>
#include <cstdint>
#include <random>

extern "C" {

// baseline/tests/boundaries.cpp:8-9 (params): W, aL, aR ~ U(-0.3, 0.3) from
// mt19937(D+K+d), drawn in the order W, aL, aR.
void oracle_boundary_params(int D, int K, int d, float* w, float* al, float* ar) {
    std::mt19937 rng(D + K + d);
    std::uniform_real_distribution<float> rnd(-.3, .3);
    for (long i = 0; i < long(D) * K * d; ++i) w[i] = rnd(rng);
    for (long i = 0; i < long(K) * d; ++i) al[i] = rnd(rng);
    for (long i = 0; i < long(K) * d; ++i) ar[i] = rnd(rng);
}

// baseline/src/common.cpp:50-62 (random_model) for one layer l of the model
// din -> 8x32 -> 8x32 -> 1xclasses.
void oracle_random_layer(int l, int din, int classes, int seed, float* w, float* al, float* ar) {
    int in = l ? 256 : din, heads = l < 2 ? 8 : 1, dim = l < 2 ? 32 : classes;
    std::mt19937 rng(seed + 11 * l);
    std::normal_distribution<float> norm;
    long width = long(heads) * dim;
    for (long i = 0; i < long(in) * width; ++i) w[i] = norm(rng) / std::sqrt(float(in));
    for (long i = 0; i < width; ++i) al[i] = norm(rng) / std::sqrt(float(dim));
    for (long i = 0; i < width; ++i) ar[i] = norm(rng) / std::sqrt(float(dim));
}
}
