// Tests of the C++ mirror of the reference API (include/gat_b200.hpp), written
// the way the reference's own boundary test is (baseline/tests/boundaries.cpp):
// the same synthetic graph and parameter shapes, an in-file FP64 layer as the
// oracle, and the same gates.
//   mirror_test          host-side checks (no GPU): validation messages, RNE
//                        ties, error metrics, file round trips
//   mirror_test --gpu    the layer functions on the current CUDA device
//   mirror_test --gpu-online  the online TFS variants (icpp_online, icpp_block,
//                        icpp_heads_hybrid) on the current CUDA device
//   mirror_test --stats DIR   the online variants' statistics (host counting)
//                        for the inputs in DIR
// Prints "MIRROR PASS ..." lines; exits 1 with "MIRROR FAIL <what>" otherwise.
#include <cmath>
#include <cstdio>
#include <fstream>
#include <functional>
#include <iostream>
#include <string>
#include <vector>

#include "gat_b200_online.hpp"

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
    {  // the per-layer JSON line (common.cpp:155-170), parsed by the Python test
        gat::Times tt;
        tt.projection = 0.001;
        tt.aggregate = 0.002;
        tt.total = 0.003;
        tt.executed_fma = g.e * uint64_t(p.heads) * uint64_t(p.in) * uint64_t(p.dim) + 8;
        gat::Workspace ws;
        gat::print_times("standard_bf16", "benchmark", 2, 0, g, p, ws, tt, 0.5, 64);
    }
    // online TFS variants (icpp_online.cpp:265-290, icpp_block.cpp:244-270,
    // icpp_heads_hybrid.cpp:35-41,296-316): argument checks before device work
    {
        gat::Prepared q0;
        gat::Schedule s0;
        gat::icpp_online::Workspace wo;
        gat::icpp_online::Stats so;
        rejects("online_block", "ICPP Online block must be in [1,64]",
                [&] { gat::icpp_online::aggregate(g, p, q0, s0, wo, 0, 16, so); });
        rejects("online_panel", "ICPP Online panel must be a multiple of 16",
                [&] { gat::icpp_online::aggregate(g, p, q0, s0, wo, 16, 24, so); });
        rejects("online_period", "ICPP Online profile period must be nonnegative",
                [&] { gat::icpp_online::aggregate(g, p, q0, s0, wo, 16, 16, so, -1); });
        rejects("online_unallocated", "ICPP Online workspace or parameter shape mismatch",
                [&] { gat::icpp_online::aggregate(g, p, q0, s0, wo, 16, 16, so); });
        gat::icpp_block::Workspace wk;
        gat::icpp_block::Stats sk;
        rejects("block_size", "ICPP block size must be in [1,64]",
                [&] { gat::icpp_block::aggregate(g, p, q0, s0, wk, 65, 16, sk); });
        gat::icpp_heads_hybrid::Workspace wh;
        gat::icpp_heads_hybrid::Stats sh;
        rejects("hybrid_threshold", "ICPP heads hybrid threshold must be in [1,33]",
                [&] { gat::icpp_heads_hybrid::aggregate(g, p, q0, s0, wh, 16, 16, sh, 0, false, 34); });
        rejects("hybrid_block", "optimized ICPP heads block must be 16 or 32",
                [&] { gat::icpp_heads_hybrid::aggregate(g, p, q0, s0, wh, 8, 16, sh); });
        const gat::Param p2 = params(17, 2, 16, 1);  // not the optimized shape: icpp_block's checks
        rejects("hybrid_fallback", "ICPP block size must be in [1,64]",
                [&] { gat::icpp_heads_hybrid::aggregate(g, p2, q0, s0, wh, 0, 16, sh); });
        // the reference's batches of 16 rows of the schedule: with the identity
        // order the batches hold degrees up to 129, 129 and 33
        gat::Schedule id;
        for (uint32_t i = 0; i < g.n; ++i) id.perm.push_back(i);
        const auto b16 = gat::detail::batch_steps(g, id, 16);
        expect(b16.batches == 3 && b16.active == 3 && b16.steps == 291 && b16.blocks == 21, "batch steps");
        // the work counts of the reference's CPU schedule from the CSR and the
        // degree order (icpp_block.cpp:100-212; the identities of
        // adaptive_main.cpp:44-60), against values computed separately from
        // those formulas for this graph; tot[] holds given Online units
        const uint64_t tot[5] = {0, 0, 5, 3, 0};
        gat::Prepared qh;
        qh.padded_in = 32;
        qh.output_blocks = 2;
        gat::icpp_heads_hybrid::Stats sh2;
        gat::icpp_heads_hybrid::detail::stats_of(g, params(17, 8, 32, 1), qh, id, 32, 16, tot, sh2);
        expect(sh2.ph_calls == 140 && sh2.ph_physical_fma == 589056 && sh2.packed_H_bytes == 71680 &&
                   sh2.ub_scatter_bytes == 52224 && sh2.ph_useful_fma == 147288 && sh2.raw_H_bytes == 36822 &&
                   sh2.projection_calls == 96 && sh2.baseline.amx_calls == 192 &&
                   sh2.baseline.executed_fma == 1572864 && sh2.head_switch_store_bytes == 96 * 2048 &&
                   sh2.head_switch_reload_bytes == 72 * 2048 && sh2.baseline.rescaled_feature_elements == 5 * 32,
               "hybrid work counts");
        qh.output_blocks = 1;
        gat::icpp_block::Stats sb2;
        gat::detail::block_stats(g, params(17, 2, 16, 1), qh, id, 16, tot, sb2);
        expect(sb2.block_projection_calls == 42 && sb2.baseline.amx_calls == 42 &&
                   sb2.baseline.executed_fma == 344064 && sb2.conversion_elements == 21504 &&
                   sb2.actual_input_feature_FMA == 36822 && sb2.padded_input_feature_FMA == 69312 &&
                   sb2.logical_H_bytes == 73644 && sb2.baseline.spill_bytes == 3 * 1024,
               "block work counts");
    }
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

template <class T>
uint64_t total(const std::vector<T>& v) {
    uint64_t s = 0;
    for (const T& x : v) s += uint64_t(x);
    return s;
}

// The online TFS variants through their reference entry points: each layer
// against the FP64 layer on BF16-rounded X and W at the TFS gate, the exact
// counters against what the CSR and the schedule determine, aggregate() plus
// finish against layer(), and heads_hybrid's dispatch.
void online_checks() {
    int cases = 0;
    for (int D : {17, 33})
        for (int K : {2, 8})
            for (int d : {16, 32}) {
                gat::Graph g = boundary_graph(D);
                gat::Param p = params(D, K, d, D + K + d);
                gat::Prepared q = gat::prepare(p);
                gat::Schedule s = gat::degree_schedule(g);
                const auto want16 = fp64_layer(g, p, g.x, true, true);
                const uint64_t tiles = uint64_t(K) * ((g.n + 15) / 16);
                for (int block : {16, 32}) {
                    // per (row, head): ceil(degree / block) blocks; every update
                    // after a row's first block is a rescale
                    uint64_t blocks = 0, nonempty = 0;
                    for (uint64_t i = 0; i < g.n; ++i) {
                        const uint64_t deg = g.row[i + 1] - g.row[i];
                        blocks += K * ((deg + block - 1) / block);
                        nonempty += deg ? K : 0;
                    }
                    const auto steps = gat::detail::batch_steps(g, s, block);
                    gat::icpp_online::Timing t;
                    gat::icpp_online::Workspace wo;
                    wo.allocate(g, p, true);
                    gat::icpp_online::Stats so;
                    gat::icpp_online::layer(g, p, q, s, g.x, wo, true, block, 64, t, so, 0, true, "fp32");
                    const auto eo = gat::errors(want16, wo.base.out);
                    expect(eo.finite && eo.relative_l2 < 3e-2, "icpp_online layer vs FP64");
                    expect(so.blocks == blocks && total(wo.row_blocks) == blocks, "online blocks");
                    expect(so.max_updates >= nonempty && so.rescales == so.max_updates - nonempty, "online rescales");
                    expect(total(wo.row_max_updates) == so.max_updates && total(wo.row_rescales) == so.rescales,
                           "online row arrays");
                    expect(so.neighbor_steps == K * steps.steps && so.total_tiles == tiles && so.sampled_tiles == 0,
                           "online steps and tiles");
                    // aggregate() on the copies the layer left, then finish
                    const std::vector<float> layer_out = wo.base.out;
                    gat::icpp_online::Stats sa;
                    gat::icpp_online::aggregate(g, p, q, s, wo, block, 64, sa, 4, false);
                    expect(sa.blocks == 0 && sa.total_tiles == tiles && sa.sampled_tiles == (tiles + 3) / 4,
                           "online sampled tiles");
                    gat::Times tf;
                    gat::finish(g, p, wo.base, true, tf);
                    const auto ea = gat::errors(layer_out, wo.base.out);
                    expect(ea.finite && ea.max_abs <= 1e-5, "icpp_online aggregate + finish vs layer");
                    // icpp_block: the same Online units, one projection per batch block
                    gat::icpp_block::Workspace wk;
                    wk.allocate(g, p, true);
                    gat::icpp_block::Stats sk;
                    gat::icpp_block::layer(g, p, q, s, g.x, wk, true, block, 64, t, sk, 0, true, "fp32");
                    const auto ek = gat::errors(want16, wk.original.base.out);
                    expect(ek.finite && ek.relative_l2 < 3e-2, "icpp_block layer vs FP64");
                    expect(sk.baseline.blocks == so.blocks && sk.baseline.max_updates == so.max_updates &&
                               sk.baseline.rescales == so.rescales && sk.baseline.rescale_events == so.rescale_events,
                           "block units");
                    expect(sk.block_projection_calls == K * steps.blocks &&
                               sk.baseline.neighbor_steps == sk.block_projection_calls &&
                               sk.source_neighbor_steps == so.neighbor_steps &&
                               sk.actual_input_feature_FMA == uint64_t(K) * g.e * uint64_t(D),
                           "block calls");
                    // icpp_heads_hybrid: optimized for heads 8, dim 32, else icpp_block
                    gat::icpp_heads_hybrid::Workspace wh;
                    wh.allocate(g, p, true);
                    gat::icpp_heads_hybrid::Stats sh;
                    gat::icpp_heads_hybrid::layer(g, p, q, s, g.x, wh, true, block, 64, t, sh, 0, true, "fp32", 16);
                    const auto eh = gat::errors(want16, wh.fallback.original.base.out);
                    expect(eh.finite && eh.relative_l2 < 3e-2, "icpp_heads_hybrid layer vs FP64");
                    const bool optimized = K == 8 && d == 32;
                    expect(sh.optimized == optimized, "hybrid dispatch");
                    expect(sh.projection_calls == K * steps.blocks && sh.baseline.blocks == so.blocks &&
                               sh.baseline.rescales == so.rescales,
                           "hybrid counts");
                    if (optimized)  // the reference's work identities (adaptive_main.cpp:50-53)
                        expect(sh.ph_useful_fma == uint64_t(K) * g.e * uint64_t(D) &&
                                   sh.raw_H_bytes == g.e * uint64_t(D) * 2 && sh.baseline.spill_bytes == 0 &&
                                   sh.head_switch_reload_bytes == (steps.blocks - steps.active) * uint64_t(K) * 2048,
                               "hybrid work identities");
                    if (!optimized) {
                        const auto ef = gat::errors(wk.original.base.out, wh.fallback.original.base.out);
                        expect(ef.finite && ef.max_abs <= 1e-5, "hybrid falls back to icpp_block");
                    }
                    ++cases;
                    std::cout << "MIRROR PASS online D=" << D << " K=" << K << " d=" << d << " block=" << block
                              << " online_rel=" << eo.relative_l2 << " block_rel=" << ek.relative_l2
                              << " hybrid_rel=" << eh.relative_l2 << " rescales=" << so.rescales << "\n";
                }
            }
    std::cout << "MIRROR PASS online cases=" << cases << "\n";
    // standard_layer with an lr_reordered policy (matched attention,
    // baseline_standard.cpp:103-105): L and R are lr_reordered's, and the layer
    // meets the BF16 gate
    for (int K : {1, 8})
        for (const std::string policy : {"bf16", "fp32", "avx"}) {
            gat::Graph g = boundary_graph(33);
            gat::Param p = params(33, K, 32, 7 + K);
            gat::Prepared q = gat::prepare(p);
            gat::Workspace wm, wl;
            wm.allocate(g, p, "matched_attention");
            wl.allocate(g, p, "tfs_bf16");
            gat::Times t;
            gat::standard_layer(g, p, q, g.x, wm, true, t, false, policy);
            gat::lr_reordered(g, p, q, g.x, wl, policy);
            const auto el = gat::errors(wl.left, wm.left), er = gat::errors(wl.right, wm.right);
            expect(el.finite && er.finite && el.max_abs <= 1e-6 && er.max_abs <= 1e-6, "matched attention L/R");
            const auto em = gat::errors(fp64_layer(g, p, g.x, true, true), wm.out);
            expect(em.finite && em.relative_l2 < 1e-2, "matched attention layer vs FP64");
            std::cout << "MIRROR PASS matched K=" << K << " policy=" << policy << " rel=" << em.relative_l2 << "\n";
        }
    // R0's trace (ref_fp32.cpp:7-14) from a ref_fp32 workspace: score and the
    // row maximum bit for bit from the layer's own L/R, p within the ulps of
    // two exp implementations, den and alpha to FP32 rounding
    gat::Graph g = boundary_graph(33);
    gat::Param p = params(33, 8, 32, 5);
    gat::Workspace w;
    w.allocate(g, p, "ref_fp32");
    gat::Times t;
    gat::ref_layer(g, p, g.x, w, true, t);
    const int K = p.heads;
    expect(w.score.size() == g.e * K && w.p.size() == g.e * K && w.alpha.size() == g.e * K, "trace sizes");
    for (uint64_t i = 0; i < g.n; ++i)
        for (int h = 0; h < K; ++h) {
            float m = -INFINITY;
            double den = 0;
            for (uint64_t e = g.row[i]; e < g.row[i + 1]; ++e) {
                float sc = w.left[i * K + h] + w.right[size_t(g.col[e]) * K + h];
                sc = sc >= 0 ? sc : 0.2f * sc;
                expect(w.score[e * K + h] == sc, "R0 score");
                m = std::max(m, sc);
            }
            expect(w.max[i * K + h] == (g.row[i] == g.row[i + 1] ? 0.f : m), "R0 row maximum");
            for (uint64_t e = g.row[i]; e < g.row[i + 1]; ++e) {
                const float diff = w.score[e * K + h] - m;  // R0 subtracts in FP32
                const double want = std::exp(double(diff));
                expect(std::fabs(w.p[e * K + h] - want) <= 1e-6 * want + 1e-37, "R0 p");
                den += w.p[e * K + h];
            }
            expect(std::fabs(w.den[i * K + h] - den) <= 1e-5 * std::max(den, 1e-30), "R0 den");
            for (uint64_t e = g.row[i]; e < g.row[i + 1]; ++e) {
                const float want = w.p[e * K + h] / w.den[i * K + h];
                expect(std::fabs(w.alpha[e * K + h] - want) <= 2.5e-7f * want, "R0 alpha");
            }
        }
    std::cout << "MIRROR PASS r0_trace edges=" << g.e << "\n";
}

// --stats DIR: the online variants' statistics from the mirror's counting
// (icpp_online, icpp_block and icpp_heads_hybrid, heads 8, dim 32), for the graph, degree
// order and Online units written into DIR, one "STATS <case> <values>" line per
// case in the order of the reference's Stats fields.
template <class T>
std::vector<T> read_raw(const std::string& path) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) throw std::runtime_error("cannot open " + path);
    std::vector<T> v(size_t(f.tellg()) / sizeof(T));
    f.seekg(0);
    f.read(reinterpret_cast<char*>(v.data()), std::streamsize(v.size() * sizeof(T)));
    return v;
}
void print_stats(const std::string& name, const gat::icpp_online::Stats& s, const std::vector<uint64_t>& extra) {
    std::cout << "STATS " << name;
    for (uint64_t x : {s.blocks, s.max_updates, s.rescales, s.rescale_events, s.neighbor_steps, s.amx_calls,
                       s.executed_fma, s.rescaled_feature_elements, s.rescaled_padded_feature_elements, s.spill_bytes,
                       s.reload_bytes, s.total_tiles})
        std::cout << " " << x;
    for (uint64_t x : extra) std::cout << " " << x;
    std::cout << "\n";
}
void stats_checks(const std::string& dir) {
    const gat::Graph g = gat::load_graph(dir + "/graph.gatbin");
    gat::Schedule s;
    s.perm = read_raw<uint32_t>(dir + "/perm.u32");
    gat::Param p;
    p.in = int(g.din);
    p.heads = 8;
    p.dim = 32;
    gat::Prepared q;
    q.padded_in = (p.in + 31) / 32 * 32;
    q.output_blocks = 2;
    for (int block : {4, 16, 64}) {  // icpp_online
        const std::vector<uint64_t> tot = read_raw<uint64_t>(dir + "/units_b" + std::to_string(block) + ".u64");
        expect(tot.size() == 5, "units file");
        gat::icpp_online::Stats os;
        gat::detail::online_stats(p, q, tot.data(), os);
        std::cout << "STATS online" << block;
        for (uint64_t x : {os.blocks, os.max_updates, os.rescales, os.rescale_events, os.neighbor_steps, os.amx_calls,
                           os.executed_fma, os.rescaled_feature_elements, os.rescaled_padded_feature_elements,
                           os.spill_bytes, os.reload_bytes})
            std::cout << " " << x;
        std::cout << "\n";
    }
    for (int block : {16, 32}) {
        const std::vector<uint64_t> tot = read_raw<uint64_t>(dir + "/units_b" + std::to_string(block) + ".u64");
        expect(tot.size() == 5, "units file");
        gat::icpp_block::Stats bs;
        gat::detail::block_stats(g, p, q, s, block, tot.data(), bs);
        gat::detail::tiles(g, p.heads, 0, true, bs.baseline);
        print_stats("block" + std::to_string(block), bs.baseline,
                    {bs.actual_input_feature_FMA, bs.padded_input_feature_FMA, bs.useful_projection_FMA,
                     bs.logical_H_bytes, bs.block_projection_calls, bs.conversion_elements, bs.source_neighbor_steps});
        for (int threshold : {1, 16, 33}) {
            gat::icpp_heads_hybrid::Stats hs;
            hs.optimized = true;
            gat::icpp_heads_hybrid::detail::stats_of(g, p, q, s, block, threshold, tot.data(), hs);
            gat::detail::tiles(g, p.heads, 0, true, hs.baseline);
            print_stats("hybrid" + std::to_string(block) + "_t" + std::to_string(threshold), hs.baseline,
                        {uint64_t(hs.optimized), hs.ph_calls, hs.ph_physical_fma, hs.ph_useful_fma, hs.raw_H_bytes,
                         hs.packed_H_bytes, hs.projection_calls, hs.head_switch_store_bytes,
                         hs.head_switch_reload_bytes, hs.ub_scatter_bytes});
        }
    }
}

}  // namespace

int main(int argc, char** argv) {
    try {
        const std::string mode = argc > 1 ? argv[1] : "--host";
        const std::string dir = argc > 2 ? argv[2] : ".";
        if (mode == "--gpu")
            gpu_checks();
        else if (mode == "--gpu-online")
            online_checks();
        else if (mode == "--stats")
            stats_checks(dir);
        else
            host_checks(dir);
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "MIRROR FAIL " << e.what() << "\n";
        return 1;
    }
}
