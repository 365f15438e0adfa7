// Helpers shared by the TFS experiment drivers (gat_b200_tfs_online,
// gat_b200_tfs_adaptive): the error metric, CHECK line and output fingerprint
// of the reference's tfs_online drivers (baseline/tfs_online/main.cpp:11-30,
// adaptive_main.cpp:22-36), and the boundary graph of its tests
// (baseline/tests/boundaries.cpp:10-13).
#pragma once
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <iomanip>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

#include "gat_b200.hpp"

namespace gat_b200_cli {

namespace gat = gat_b200;

// Max / mean absolute and relative L2 error of b against a, infinite when
// either holds a non-finite value.
inline gat::Error difference(const std::vector<float>& a, const std::vector<float>& b) {
    if (a.empty() || a.size() != b.size()) throw std::runtime_error("comparison shape");
    double mx = 0, ab = 0, sq = 0, norm = 0;
    bool bad = false;
    for (size_t i = 0; i < a.size(); ++i) {
        bad |= !std::isfinite(a[i]) || !std::isfinite(b[i]);
        const double d = double(b[i]) - a[i];
        mx = std::max(mx, std::abs(d));
        ab += std::abs(d);
        sq += d * d;
        norm += double(a[i]) * a[i];
    }
    gat::Error e;
    e.finite = !bad;
    e.max_abs = mx;
    e.mean_abs = ab / a.size();
    e.relative_l2 = norm ? std::sqrt(sq / norm) : (sq ? INFINITY : 0);
    if (bad) e.max_abs = e.mean_abs = e.relative_l2 = INFINITY;
    return e;
}

// One CHECK line with the 0.003 absolute gate; a non-finite comparison throws
// `nonfinite` (each driver keeps its reference's message).
inline void report(const std::string& path, int layer, const std::string& ref, const gat::Error& e,
                   const char* nonfinite) {
    std::cout << std::setprecision(12) << "CHECK path=" << path << " layer=" << layer << " reference=" << ref
              << " max_abs_error=" << e.max_abs << " mean_abs_error=" << e.mean_abs
              << " relative_L2_error=" << e.relative_l2 << " finite=" << e.finite
              << " original_abs_003_gate=" << (e.finite && e.max_abs <= .003 ? "PASS" : "FAIL")
              << " task_accuracy=UNVERIFIED\n";
    if (!e.finite) throw std::runtime_error(nonfinite);
}

// Order-dependent 64-bit hash of the bits of x (the profile-identity check).
inline uint64_t fingerprint(const std::vector<float>& x) {
    uint64_t out = 0;
    for (size_t i = 0; i < x.size(); ++i) {
        uint32_t bits;
        std::memcpy(&bits, x.data() + i, 4);
        uint64_t z = uint64_t(bits) ^ ((i + 1) * 0x9e3779b97f4a7c15ULL);
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
        out ^= z ^ (z >> 27);
    }
    return out;
}

// 35 nodes with degrees cycling {0,1,2,15,16,17,31,32,33,63,64,65,129} and
// smooth features: every block and chunk boundary of the aggregation kernels.
inline gat::Graph boundary_graph(int D) {
    const int deg[13] = {0, 1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 129};
    gat::Graph g;
    g.n = 35;
    g.din = D;
    g.classes = 4;
    g.row.push_back(0);
    for (int i = 0; i < 35; ++i) {
        for (int e = 0; e < deg[i % 13]; ++e) g.col.push_back(uint32_t((i * 3 + e * 7) % 35));
        g.row.push_back(g.col.size());
    }
    g.e = g.col.size();
    g.x.resize(size_t(35) * D);
    for (size_t i = 0; i < g.x.size(); ++i) g.x[i] = 0.5f * std::sin(0.17f * float(i));
    return g;
}

}  // namespace gat_b200_cli
