// Tests of the C++ mirror of the reference API (include/gat_b200.hpp), written
// the way the reference's own boundary test is (baseline/tests/boundaries.cpp):
// the same synthetic graph and parameter shapes, an in-file FP64 layer as the
// oracle, and the same gates.
//   mirror_test          host-side checks (no GPU): validation messages, RNE
//                        ties, error metrics, file round trips
//   mirror_test --gpu    the layer functions on the current CUDA device
// Prints "MIRROR PASS ..." lines; exits 1 with "MIRROR FAIL <what>" otherwise.
#include <cmath>
#include <cstdio>
#include <functional>
#include <iostream>
#include <string>
#include <vector>

#include "gat_b200.hpp"

namespace gat = gat_b200;

namespace {

void expect(bool ok, const std::string& what) {
    if (!ok) throw std::runtime_error(what);
}

void rejects(const std::string& name, const std::string& message, const std::function<void()>& f) {
    try {
        f();
    } catch (const std::exception& e) {
        expect(std::string(e.what()).find(message) != std::string::npos,
               name + ": wrong message '" + e.what() + "', wanted '" + message + "'");
        std::cout << "MIRROR PASS rejects " << name << "\n";
        return;
    }
    throw std::runtime_error(name + " was not rejected");
}

// boundaries.cpp:10-13: 35 nodes, degrees cycling {0,1,2,15,16,17,31,32,33,63,64,65,129}.
gat::Graph boundary_graph(int D) {
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

gat::Param params(int D, int K, int d, int seed) {
    gat::Param p;
    p.in = D;
    p.heads = K;
    p.dim = d;
    p.w.resize(size_t(D) * K * d);
    p.al.resize(size_t(K) * d);
    p.ar.resize(size_t(K) * d);
    for (size_t i = 0; i < p.w.size(); ++i) p.w[i] = std::cos(0.37f * float(i + seed)) / std::sqrt(float(D));
    for (size_t i = 0; i < p.al.size(); ++i) {
        p.al[i] = std::sin(0.29f * float(i + seed)) / std::sqrt(float(d));
        p.ar[i] = std::cos(0.41f * float(i + 3 * seed)) / std::sqrt(float(d));
    }
    return p;
}

// FP64 layer: Z = X W, L/R per head, leaky, stable softmax over the row, sum, ELU.
std::vector<float> fp64_layer(const gat::Graph& g, const gat::Param& p, const std::vector<float>& x, bool hidden,
                              bool quantize, std::vector<double>* row_max = nullptr) {
    const int K = p.heads, d = p.dim, W = p.width();
    std::vector<float> xs = quantize ? gat::quantized(x) : x;
    std::vector<float> ws = quantize ? gat::quantized(p.w) : p.w;
    std::vector<double> z(size_t(g.n) * W, 0.0);
    for (uint64_t i = 0; i < g.n; ++i)
        for (int k = 0; k < p.in; ++k)
            for (int c = 0; c < W; ++c) z[i * W + c] += double(xs[i * p.in + k]) * double(ws[size_t(k) * W + c]);
    std::vector<double> L(size_t(g.n) * K, 0.0), R(size_t(g.n) * K, 0.0);
    for (uint64_t i = 0; i < g.n; ++i)
        for (int h = 0; h < K; ++h)
            for (int t = 0; t < d; ++t) {
                L[i * K + h] += z[i * W + h * d + t] * p.al[h * d + t];
                R[i * K + h] += z[i * W + h * d + t] * p.ar[h * d + t];
            }
    std::vector<float> out(size_t(g.n) * W, 0.f);
    if (row_max) row_max->assign(size_t(g.n) * K, 0.0);
    for (uint64_t i = 0; i < g.n; ++i)
        for (int h = 0; h < K; ++h) {
            if (g.row[i] == g.row[i + 1]) continue;  // empty row: 0
            double m = -INFINITY;
            for (uint64_t e = g.row[i]; e < g.row[i + 1]; ++e) {
                double s = L[i * K + h] + R[size_t(g.col[e]) * K + h];
                m = std::max(m, s >= 0 ? s : 0.2 * s);
            }
            if (row_max) (*row_max)[i * K + h] = m;
            double den = 0;
            std::vector<double> acc(d, 0.0);
            for (uint64_t e = g.row[i]; e < g.row[i + 1]; ++e) {
                double s = L[i * K + h] + R[size_t(g.col[e]) * K + h];
                double pe = std::exp((s >= 0 ? s : 0.2 * s) - m);
                den += pe;
                for (int t = 0; t < d; ++t) acc[t] += pe * z[size_t(g.col[e]) * W + h * d + t];
            }
            for (int t = 0; t < d; ++t) {
                double v = acc[t] / den;
                out[i * W + h * d + t] = float(hidden && v < 0 ? std::expm1(v) : v);
            }
        }
    return out;
}

void host_checks(const std::string& dir) {
    gat::Graph g = boundary_graph(17);
    g.validate();
    rejects("nonfinite_input", "nonfinite graph input", [&] { auto b = g; b.x[0] = NAN; b.validate(); });
    rejects("nonmonotone_CSR", "nonmonotone CSR", [&] { auto b = g; b.row[3] = b.e + 1; b.validate(); });
    rejects("out_of_range_source", "source index out of bounds", [&] { auto b = g; b.col[0] = uint32_t(g.n); b.validate(); });
    rejects("bad_sizes", "invalid graph sizes", [&] { auto b = g; b.x.pop_back(); b.validate(); });
    gat::Param p = params(17, 8, 32, 1);
    p.validate();
    rejects("wrong_parameter_size", "invalid parameter shape", [&] { auto b = p; b.w.pop_back(); b.validate(); });
    rejects("bad_heads", "invalid parameter shape", [&] { auto b = p; b.heads = 9; b.validate(); });
    rejects("error_size_mismatch", "size mismatch", [&] { gat::errors({1}, {1, 2}); });
    rejects("allocation_overflow", "size overflow", [&] { gat::checked(UINT64_MAX, 2); });
    // a workspace not allocated for the call's graph and path is refused before any device work
    rejects("workspace_mismatch", "workspace z has the wrong size", [&] { gat::Workspace w; gat::standard_aggregate(g, p, w); });
    rejects("workspace_mismatch", "workspace out has the wrong size", [&] { gat::Workspace w; gat::Times t; gat::finish(g, p, w, true, t); });
    expect(!gat::errors({1}, {NAN}).finite && !gat::errors({1}, {INFINITY}).finite, "nonfinite comparison passed");
    // RNE ties and tails (boundaries.cpp:25-26)
    expect(gat::rne(1.0f + 1.0f / 256) == 0x3f80, "tie to even (down)");
    expect(gat::rne(1.0f + 3.0f / 256) == 0x3f82, "tie to even (up)");
    expect(gat::rne(1.0f + 1.0f / 256 + 1.0f / 65536) == 0x3f81, "above the tie");
    expect(gat::expand(gat::rne(2.5f)) == 2.5f, "exact value");
    std::cout << "MIRROR PASS rne\n";
    // file round trips
    gat::save_graph(g, dir + "/g.gatbin");
    gat::Graph g2 = gat::load_graph(dir + "/g.gatbin");
    expect(g2.n == g.n && g2.e == g.e && g2.row == g.row && g2.col == g.col && g2.x == g.x, "GATBIN round trip");
    gat::Model m = gat::random_model(17, 4, 11);
    gat::save_model(m, dir + "/m.gatwgt");
    gat::Model m2 = gat::load_model(dir + "/m.gatwgt", 17, 4);
    for (int l = 0; l < 3; ++l) expect(m2[l].w == m[l].w && m2[l].al == m[l].al && m2[l].ar == m[l].ar, "GATWGT round trip");
    rejects("missing_graph", "cannot open graph", [&] { gat::load_graph(dir + "/missing.gatbin"); });
    std::cout << "MIRROR PASS host\n";
}

void gpu_checks() {
    int cases = 0;
    for (int D : {17, 33})
        for (int K : {1, 8})
            for (int d : {7, 32, 47}) {
                gat::Graph g = boundary_graph(D);
                gat::Param p = params(D, K, d, D + K + d);
                gat::Prepared q = gat::prepare(p);
                gat::Workspace w;
                w.allocate(g, p, "standard_fp32");
                gat::Times t;
                // FP32 B0 stages: projection (+L/R), prescan, aggregate, finish
                gat::projection(g, p, q, g.x, w, false);
                gat::lr_from_z(g, p, w);
                gat::max_prescan(g, p, w);
                std::vector<double> m64;
                auto want = fp64_layer(g, p, g.x, true, false, &m64);
                for (size_t i = 0; i < m64.size(); ++i)
                    expect(std::fabs(w.max[i] - m64[i]) <= 1e-4 * std::max(1.0, std::fabs(m64[i])), "row max");
                gat::standard_aggregate(g, p, w, nullptr, nullptr, &t);
                gat::finish(g, p, w, true, t);
                auto e = gat::errors(want, w.out);
                expect(e.finite && e.max_abs < 1e-4 && e.relative_l2 < 1e-4, "FP32 stages vs FP64");
                for (uint64_t i = 0; i < g.n; ++i)
                    if (g.row[i] == g.row[i + 1])
                        for (int c = 0; c < p.width(); ++c) expect(w.out[i * p.width() + c] == 0.f, "empty row");
                // R0 entry point (FP32 path)
                gat::ref_layer(g, p, g.x, w, true, t);
                e = gat::errors(want, w.out);
                expect(e.finite && e.max_abs < 1e-4 && e.relative_l2 < 1e-4, "ref_layer vs FP64");
                // BF16 B0 layer against the FP64 layer on BF16-rounded X and W
                gat::Workspace wb;
                wb.allocate(g, p, "standard_bf16");
                gat::standard_layer(g, p, q, g.x, wb, true, t);
                auto want16 = fp64_layer(g, p, g.x, true, true);
                const auto eb = gat::errors(want16, wb.out);
                expect(eb.finite && eb.relative_l2 < 1e-2, "BF16 standard_layer vs FP64");
                // B1 TFS layer: every p*x product is rounded to BF16 before the
                // projection (baseline_tfs.cpp:16-110), hence its own, looser gate
                gat::Workspace wt;
                wt.allocate(g, p, "tfs_bf16");
                gat::Schedule s = gat::degree_schedule(g);
                gat::tfs_layer(g, p, q, s, g.x, wt, true, 16, t, "bf16");
                const auto et = gat::errors(want16, wt.out);
                expect(et.finite && et.relative_l2 < 3e-2, "tfs_layer vs FP64");
                // fixed-p operators (boundaries.cpp:36-42): the same p and den into the
                // standard and the TFS aggregation; TFS against the scalar BF16
                // emulation of its edge projection, at the reference's 2e-4 gate
                std::vector<float> fp(size_t(g.e) * K), fd(size_t(g.n) * K, 0.f);
                for (uint64_t i = 0; i < g.n; ++i)
                    for (uint64_t ed = g.row[i]; ed < g.row[i + 1]; ++ed)
                        for (int h = 0; h < K; ++h) {
                            fp[ed * K + h] = 0.5f + 0.45f * std::sin(float(ed * K + h));
                            fd[i * K + h] += fp[ed * K + h];
                        }
                gat::Workspace wf;
                wf.allocate(g, p, "standard_bf16");
                gat::projection(g, p, q, g.x, wf, true);
                gat::standard_aggregate(g, p, wf, fp.data(), fd.data());
                gat::finish(g, p, wf, false, t);
                std::vector<float> emu_std(wf.out.size(), 0.f);
                const int W = p.width();
                for (uint64_t i = 0; i < g.n; ++i)
                    for (int h = 0; h < K; ++h)
                        for (int c = 0; c < d; ++c) {
                            double acc = 0;
                            for (uint64_t ed = g.row[i]; ed < g.row[i + 1]; ++ed)
                                acc += double(fp[ed * K + h]) * wf.z[size_t(g.col[ed]) * W + h * d + c];
                            emu_std[i * W + h * d + c] = fd[i * K + h] > 0 ? float(acc / fd[i * K + h]) : 0.f;
                        }
                const auto es = gat::errors(emu_std, wf.out);
                expect(es.finite && es.max_abs < 1e-5 && es.relative_l2 < 1e-5, "fixed-p standard aggregate");
                gat::Workspace wt2;
                wt2.allocate(g, p, "tfs_bf16");
                gat::lr_reordered(g, p, q, g.x, wt2, "bf16");  // fills the BF16 copy of X
                gat::tfs_aggregate(g, p, q, s, wt2, 64, t, fp.data(), fd.data());
                gat::finish(g, p, wt2, false, t);
                std::vector<float> emu(wt2.out.size(), 0.f);
                for (uint64_t i = 0; i < g.n; ++i)
                    for (int h = 0; h < K; ++h) {
                        for (uint64_t ed = g.row[i]; ed < g.row[i + 1]; ++ed)
                            for (int k = 0; k < p.in; ++k) {
                                const float v = gat::expand(gat::rne(
                                    fp[ed * K + h] * gat::expand(gat::rne(g.x[size_t(g.col[ed]) * p.in + k]))));
                                for (int c = 0; c < d; ++c)
                                    emu[i * W + h * d + c] += v * gat::expand(gat::rne(p.w[size_t(k) * W + h * d + c]));
                            }
                        for (int c = 0; c < d; ++c)
                            emu[i * W + h * d + c] = fd[i * K + h] > 0 ? emu[i * W + h * d + c] / fd[i * K + h] : 0.f;
                    }
                const auto ef = gat::errors(emu, wt2.out);
                expect(ef.finite && ef.max_abs < 2e-4 && ef.relative_l2 < 2e-4,
                       "fixed-p TFS edge projection versus emulator");
                ++cases;
                std::cout << "MIRROR PASS D=" << D << " K=" << K << " d=" << d << " fp32_rel=" << e.relative_l2
                          << " bf16_rel=" << eb.relative_l2 << " tfs_rel=" << et.relative_l2
                          << " fixed_p_tfs_rel=" << ef.relative_l2 << "\n";
            }
    // degree schedule: a permutation, degrees ascending, ties by id
    gat::Graph g = boundary_graph(17);
    gat::Schedule s = gat::degree_schedule(g);
    std::vector<int> seen(g.n, 0);
    for (size_t k = 0; k < s.perm.size(); ++k) {
        expect(s.perm[k] < g.n && !seen[s.perm[k]]++, "schedule is a permutation");
        if (k) {
            uint64_t a = g.row[s.perm[k - 1] + 1] - g.row[s.perm[k - 1]], b = g.row[s.perm[k] + 1] - g.row[s.perm[k]];
            expect(a < b || (a == b && s.perm[k - 1] < s.perm[k]), "schedule order");
        }
    }
    std::cout << "MIRROR PASS gpu cases=" << cases << "\n";
}

}  // namespace

int main(int argc, char** argv) {
    try {
        const bool gpu = argc > 1 && std::string(argv[1]) == "--gpu";
        const std::string dir = argc > 2 ? argv[2] : ".";
        if (gpu)
            gpu_checks();
        else
            host_checks(dir);
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "MIRROR FAIL " << e.what() << "\n";
        return 1;
    }
}
