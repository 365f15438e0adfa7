// Seeded synthetic inputs for the benchmark configurations (host code).
//
// The reference measures on ogbn-arxiv / ogbn-products files that are not
// available here; these generators produce graphs of the same shape instead.
// Every random draw comes from a counter-based stream rng(seed, stream, i), so
// the output is bit-identical for any OpenMP thread count and on any machine.
//
// Graph semantics follow the reference's graph preparation
// (implementation/tools/prepare_arxiv.py:28-52): destination-row CSR, one
// self-loop per node, no duplicate (row, source) pairs, sources ascending.
#include "gat_b200_internal.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <vector>

namespace gatb {
namespace {

inline uint64_t splitmix64(uint64_t x) {
    x += 0x9e3779b97f4a7c15ULL;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
    return x ^ (x >> 31);
}
// Counter-based stream: independent of evaluation order.
inline uint64_t rng(uint64_t seed, uint64_t stream, uint64_t i) {
    return splitmix64(splitmix64(seed ^ splitmix64(stream + 0x632be59bd9b4e019ULL)) + i);
}
inline double unit(uint64_t r) { return double(r >> 11) * (1.0 / 9007199254740992.0); }  // [0,1)

// Standard normal by Box-Muller on draws 2i, 2i+1.
inline double normal(uint64_t seed, uint64_t stream, uint64_t i) {
    double u1 = unit(rng(seed, stream, 2 * i)), u2 = unit(rng(seed, stream, 2 * i + 1));
    u1 = u1 < 1e-300 ? 1e-300 : u1;
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

// Random permutation of [0,n) (Fisher-Yates with a single stream).
std::vector<uint32_t> permutation(uint64_t n, uint64_t seed, uint64_t stream) {
    std::vector<uint32_t> p(n);
    std::iota(p.begin(), p.end(), 0u);
    for (uint64_t i = n; i > 1; --i) {
        uint64_t j = rng(seed, stream, i) % i;
        std::swap(p[i - 1], p[j]);
    }
    return p;
}

// Walker/Vose alias table over weights w[0..n).
struct Alias {
    std::vector<double> prob;
    std::vector<uint32_t> alias;
    explicit Alias(const std::vector<double>& w) : prob(w.size()), alias(w.size()) {
        const size_t n = w.size();
        double total = 0;
        for (double v : w) total += v;
        std::vector<double> scaled(n);
        std::vector<uint32_t> small, large;
        for (size_t i = 0; i < n; ++i) {
            scaled[i] = w[i] * double(n) / total;
            (scaled[i] < 1.0 ? small : large).push_back(uint32_t(i));
        }
        while (!small.empty() && !large.empty()) {
            uint32_t s = small.back(), l = large.back();
            small.pop_back();
            prob[s] = scaled[s];
            alias[s] = l;
            scaled[l] = (scaled[l] + scaled[s]) - 1.0;
            if (scaled[l] < 1.0) {
                large.pop_back();
                small.push_back(l);
            }
        }
        for (uint32_t i : large) { prob[i] = 1.0; alias[i] = i; }
        for (uint32_t i : small) { prob[i] = 1.0; alias[i] = i; }
    }
    uint32_t draw(uint64_t r1, uint64_t r2) const {
        uint64_t i = r1 % prob.size();
        return unit(r2) < prob[i] ? uint32_t(i) : alias[i];
    }
};

// Fills row i's sources (excluding the self loop) with `deg` distinct values
// != i drawn by `draw(k)`, adds the self loop and sorts ascending.
template <class Draw>
void fill_row(uint64_t i, uint64_t deg, uint32_t* out, Draw draw) {
    uint64_t have = 0, k = 0;
    out[0] = uint32_t(i);
    // Draw in rounds, dedup by sort+unique until `deg` distinct sources exist.
    while (have < deg) {
        uint64_t need = deg - have;
        for (uint64_t t = 0; t < need; ++t) {
            uint32_t s;
            do { s = draw(k++); } while (s == uint32_t(i));
            out[1 + have + t] = s;
        }
        std::sort(out + 1, out + 1 + deg);
        have = uint64_t(std::unique(out + 1, out + 1 + deg) - (out + 1));
    }
    std::sort(out, out + 1 + deg);
}

}  // namespace

int synth_uniform_graph(uint64_t n, uint32_t sources, uint64_t seed, uint64_t* row, uint32_t* col) {
    if (n < 2 || sources >= n) return fail("uniform graph: need sources < n");
    for (uint64_t i = 0; i <= n; ++i) row[i] = i * (uint64_t(sources) + 1);
#pragma omp parallel for schedule(dynamic, 256)
    for (long long i = 0; i < (long long)n; ++i)
        fill_row(uint64_t(i), sources, col + row[i],
                 [&](uint64_t k) { return uint32_t(rng(seed, 1000 + uint64_t(i), k) % n); });
    return 0;
}

// Power-law degree sequence: row degrees (without the self loop) follow
// t(r) = A (r + r0)^-beta over ranks r, beta = 1/(gamma-1), with t(0) = max_degree-1
// and r0 solved so that the floored sequence sums to e_target - n; the last
// few units of slack are spread one per row. Node ids receive ranks through a
// seeded permutation, and the same ranks set source popularity weights, so
// high in-degree nodes are also frequent sources (as in an undirected graph).
struct PowerLaw {
    std::vector<uint64_t> node_deg;  // degree without the self loop
    std::vector<double> weight;      // source popularity
};

static int powerlaw_setup(uint64_t n, uint64_t e_target, uint64_t max_degree, double gamma, uint64_t seed,
                          PowerLaw& pl) {
    if (n < 4 || gamma <= 1.0) return fail("power-law graph: bad n/gamma");
    if (e_target < 2 * n || max_degree < 2 || max_degree > n / 2 || e_target > n * (max_degree))
        return fail("power-law graph: infeasible edge target");
    const double beta = 1.0 / (gamma - 1.0);
    const double top = double(max_degree - 1);
    const uint64_t want = e_target - n;  // non-self edges
    auto total_for = [&](double r0) {
        double A = top * std::pow(r0, beta);
        uint64_t s = 0;
        for (uint64_t r = 0; r < n; ++r) {
            double t = A * std::pow(double(r) + r0, -beta);
            uint64_t d = t < 1.0 ? 1 : uint64_t(t);
            s += std::min<uint64_t>(d, max_degree - 1);
        }
        return s;
    };
    // total_for is increasing in r0: bisection in log space.
    double lo = 1e-6, hi = double(n) * 10;
    if (total_for(hi) < want || total_for(lo) > want) return fail("power-law graph: target not reachable");
    for (int it = 0; it < 200; ++it) {
        double mid = std::sqrt(lo * hi);
        (total_for(mid) < want ? lo : hi) = mid;
    }
    const double r0 = lo, A = top * std::pow(r0, beta);
    std::vector<uint64_t> deg(n);
    uint64_t s = 0;
    for (uint64_t r = 0; r < n; ++r) {
        double t = A * std::pow(double(r) + r0, -beta);
        uint64_t d = t < 1.0 ? 1 : uint64_t(t);
        deg[r] = std::min<uint64_t>(d, max_degree - 1);
        s += deg[r];
    }
    // The top rank carries exactly the requested maximum (flooring may have
    // lost it); then spread the remaining slack one unit per row from the tail
    // of the rank order, never exceeding the cap.
    s += (max_degree - 1) - deg[0];
    deg[0] = max_degree - 1;
    if (s > want) return fail("power-law graph: degree sequence overshoots the target");
    for (uint64_t r = n; s < want && r-- > 1;)
        if (deg[r] < max_degree - 1) { ++deg[r]; ++s; }
    if (s != want) return fail("power-law graph: degree sequence did not close");
    std::vector<uint32_t> node_of_rank = permutation(n, seed, 1);
    pl.node_deg.assign(n, 0);
    pl.weight.assign(n, 0.0);
    for (uint64_t r = 0; r < n; ++r) {
        pl.node_deg[node_of_rank[r]] = deg[r];
        pl.weight[node_of_rank[r]] = std::pow(double(r) + r0, -beta);
    }
    return 0;
}

int synth_powerlaw_rows(uint64_t n, uint64_t e_target, uint64_t max_degree, double gamma, uint64_t seed,
                        uint64_t r_lo, uint64_t r_hi, uint64_t* row, uint32_t* col) {
    PowerLaw pl;
    int rc = powerlaw_setup(n, e_target, max_degree, gamma, seed, pl);
    if (rc) return rc;
    if (r_lo > r_hi || r_hi > n) return fail("power-law graph: bad row range");
    row[0] = 0;
    for (uint64_t i = 0; i < n; ++i) row[i + 1] = row[i] + pl.node_deg[i] + 1;
    if (!col) return 0;  // row pointers only
    Alias table(pl.weight);
    uint32_t* base = col - row[r_lo];  // col holds edges [row[r_lo], row[r_hi])
#pragma omp parallel for schedule(dynamic, 64)
    for (long long i = (long long)r_lo; i < (long long)r_hi; ++i)
        fill_row(uint64_t(i), pl.node_deg[i], base + row[i], [&](uint64_t k) {
            return table.draw(rng(seed, 3ull << 40 | uint64_t(i), 2 * k), rng(seed, 3ull << 40 | uint64_t(i), 2 * k + 1));
        });
    return 0;
}

int synth_powerlaw_graph(uint64_t n, uint64_t e_target, uint64_t max_degree, double gamma,
                         uint64_t seed, uint64_t* row, uint32_t* col) {
    return synth_powerlaw_rows(n, e_target, max_degree, gamma, seed, 0, n, row, col);
}

int synth_normal(uint64_t count, double scale, uint64_t seed, uint64_t stream, float* out, uint64_t offset) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)count; ++i) out[i] = float(scale * normal(seed, stream, offset + uint64_t(i)));
    return 0;
}

int synth_uniform(uint64_t count, double lo, double hi, uint64_t seed, uint64_t stream, float* out) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)count; ++i)
        out[i] = float(lo + (hi - lo) * unit(rng(seed, stream, uint64_t(i))));
    return 0;
}

}  // namespace gatb
