// gat_b200_make_inputs: writes the GATBIN1 graph and GATWGT1 weights of a
// seeded synthetic configuration, the files the reference's driver reads
// (baseline/src/common.cpp:31-44, 63-79).
//
//   gat_b200_make_inputs CONFIG GRAPH_OUT WEIGHTS_OUT
//
// CONFIG is c1, c2, c4 or c4s with the shapes, generators and seeds of
// gat-tfs_b200/configs.py, and Glorot-uniform weights drawn as
// gatb200.glorot_model draws them. The program is linked from the library's
// host sources (synth.cpp, host.cpp) without the CUDA library, so the CPU
// reference arm of bench.py can get its inputs without loading
// libgat_b200.so into any process. tests/test_cli.py checks that its files
// equal the ones the Python binding writes.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "gat_b200.h"

namespace {

struct Spec {
    const char* name;
    bool powerlaw;
    uint64_t n, e, max_degree;
    uint32_t sources;
    int din, classes;
    uint64_t seed;
};

// The power-law and uniform configurations of configs.py (SPECS).
const Spec kSpecs[] = {
    {"c1", false, 1024, 0, 0, 15, 128, 40, 1},
    {"c2", true, 169343, 2484941, 13162, 0, 128, 40, 2},
    {"c4", true, 2449029, 126167053, 17482, 0, 100, 47, 4},
    {"c4s", true, 612257, 31541763, 8000, 0, 100, 47, 4},
};

int check(int rc) {
    if (rc) {
        std::fprintf(stderr, "FAIL %s\n", gat_b200_last_error());
        std::exit(1);
    }
    return rc;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc != 4) {
        std::fprintf(stderr, "usage: %s CONFIG GRAPH_OUT WEIGHTS_OUT  (CONFIG: c1 c2 c4 c4s)\n", argv[0]);
        return 2;
    }
    const Spec* s = nullptr;
    for (const auto& k : kSpecs)
        if (std::strcmp(k.name, argv[1]) == 0) s = &k;
    if (!s) {
        std::fprintf(stderr, "FAIL unknown configuration %s\n", argv[1]);
        return 1;
    }
    const double gamma = 2.1;
    std::vector<uint64_t> row(s->n + 1);
    std::vector<uint32_t> col;
    if (s->powerlaw) {
        col.resize(s->e);
        check(gat_b200_synth_powerlaw_graph(s->n, s->e, s->max_degree, gamma, s->seed, row.data(), col.data()));
    } else {
        col.resize(s->n * (s->sources + 1));
        check(gat_b200_synth_uniform_graph(s->n, s->sources, s->seed, row.data(), col.data()));
    }
    const uint64_t e = row[s->n];
    std::vector<float> x(s->n * uint64_t(s->din));
    check(gat_b200_synth_normal(x.size(), 1.0, s->seed, 1, x.data()));
    check(gat_b200_write_graph(argv[2], s->n, e, s->din, s->classes, row.data(), col.data(), x.data()));
    x.clear();
    x.shrink_to_fit();
    // Glorot-uniform model din -> 8x32 -> 8x32 -> 1xclasses: W ~ U(+-sqrt(6/(in+width))),
    // a ~ U(+-sqrt(6/(heads+dim))), streams 100+3l, 101+3l, 102+3l of the seed.
    const int in[3] = {s->din, 256, 256}, heads[3] = {8, 8, 1}, dim[3] = {32, 32, s->classes};
    std::vector<float> w[3], al[3], ar[3];
    for (int l = 0; l < 3; ++l) {
        const int width = heads[l] * dim[l];
        const double lw = std::sqrt(6.0 / (in[l] + width)), la = std::sqrt(6.0 / (heads[l] + dim[l]));
        w[l].resize(uint64_t(in[l]) * width);
        al[l].resize(width);
        ar[l].resize(width);
        check(gat_b200_synth_uniform(w[l].size(), -lw, lw, s->seed, 100 + 3 * l, w[l].data()));
        check(gat_b200_synth_uniform(width, -la, la, s->seed, 101 + 3 * l, al[l].data()));
        check(gat_b200_synth_uniform(width, -la, la, s->seed, 102 + 3 * l, ar[l].data()));
    }
    const float* wp[3] = {w[0].data(), w[1].data(), w[2].data()};
    const float* ap[3] = {al[0].data(), al[1].data(), al[2].data()};
    const float* rp[3] = {ar[0].data(), ar[1].data(), ar[2].data()};
    check(gat_b200_write_weights(argv[3], s->din, s->classes, wp, ap, rp));
    std::printf("INPUTS config=%s n=%llu e=%llu din=%d classes=%d graph=%s weights=%s\n", s->name,
                (unsigned long long)s->n, (unsigned long long)e, s->din, s->classes, argv[2], argv[3]);
    return 0;
}
