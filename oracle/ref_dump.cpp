// Golden-vector harness (test infrastructure): links the reference's own
// sources, compiled in place by oracle/Makefile, calls the reference functions
// and writes their outputs as raw little-endian files for
// tests/golden/make_golden.py. Nothing here is part of libgat_b200.so.
//
//   ref_dump boundary OUTDIR          64 D/K/d cases of baseline/tests/boundaries.cpp
//   ref_dump chain GRAPH WEIGHTS OUTDIR   three-layer chains on a GATBIN1 graph;
//                                     WEIGHTS = GATWGT1 path or "seed:N" (random_model)
//   ref_dump counters GRAPH OUTDIR    icpp_online's exact counters (blocks 4/16/64),
//                                     icpp_block's and icpp_heads_hybrid's stats
//   ref_dump tfs OUTDIR               TFS aggregation variants (B1, icpp_online,
//                                     icpp_block, icpp_heads_hybrid) on the
//                                     boundary graphs, with their inputs
#include "gat.hpp"
#include "icpp_block.hpp"
#include "icpp_heads_hybrid.hpp"
#include "icpp_online.hpp"

#include <cstdio>
#include <iostream>
#include <random>

using namespace gat;

static void dump(const std::string& path, const void* data, size_t bytes) {
    std::ofstream f(path, std::ios::binary);
    f.write(static_cast<const char*>(data), std::streamsize(bytes));
    if (!f) throw std::runtime_error("cannot write " + path);
}
template <class T>
static void dumpv(const std::string& path, const std::vector<T>& v) { dump(path, v.data(), v.size() * sizeof(T)); }

// Test inputs of baseline/tests/boundaries.cpp:8-13 (restated: that file keeps
// them in static functions). 35 nodes, degrees cycling through
// {0,1,2,15,16,17,31,32,33,63,64,65,129}, x = 0.5 sin(0.17 i).
static Param boundary_params(int D, int K, int d) {
    Param p;
    p.in = D; p.heads = K; p.dim = d;
    p.w.resize(size_t(D) * K * d); p.al.resize(size_t(K) * d); p.ar.resize(size_t(K) * d);
    std::mt19937 rng(D + K + d);
    std::uniform_real_distribution<float> rnd(-.3, .3);
    for (auto& x : p.w) x = rnd(rng);
    for (auto& x : p.al) x = rnd(rng);
    for (auto& x : p.ar) x = rnd(rng);
    return p;
}
static Graph boundary_graph(int D) {
    Graph g;
    g.n = 35; g.din = D; g.classes = 40; g.row = {0};
    const int deg[] = {0, 1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 129};
    for (uint64_t i = 0; i < g.n; ++i) {
        int count = deg[i % 13];
        for (int e = 0; e < count; ++e) g.col.push_back(uint32_t((i * 3 + e * 7) % g.n));
        g.row.push_back(g.col.size());
    }
    g.e = g.col.size();
    g.x.resize(g.n * D);
    for (size_t i = 0; i < g.x.size(); ++i) g.x[i] = std::sin(float(i) * .17f) * .5f;
    g.validate();
    return g;
}

static int boundary(const std::string& out) {
    for (int D : {17, 33, 128, 256})
        for (int K : {1, 2, 4, 8})
            for (int d : {7, 32, 40, 47}) {
                Graph g = boundary_graph(D);
                Param p = boundary_params(D, K, d);
                Prepared q = prepare(p);
                Workspace r, b, f;
                r.allocate(g, p, "ref_fp32");
                b.allocate(g, p, "standard_bf16");
                f.allocate(g, p, "standard_fp32");
                Times t;
                ref_layer(g, p, g.x, r, false, t);
                standard_layer(g, p, q, g.x, b, false, t, false);
                standard_layer(g, p, q, g.x, f, false, t, true);
                std::string pre = out + "/bnd_" + std::to_string(D) + "_" + std::to_string(K) + "_" + std::to_string(d);
                dumpv(pre + "_ref.f32", r.out);
                dumpv(pre + "_b0bf16.f32", b.out);
                dumpv(pre + "_b0fp32.f32", f.out);
                dumpv(pre + "_w.f32", p.w);
                dumpv(pre + "_al.f32", p.al);
                dumpv(pre + "_ar.f32", p.ar);
            }
    Graph g = boundary_graph(17);
    Schedule s = degree_schedule(g);
    dumpv(out + "/bnd_perm.u32", s.perm);
    dump(out + "/bnd_steps.u64", &s.neighbor_steps, 8);
    dumpv(out + "/bnd_row.u64", g.row);
    dumpv(out + "/bnd_col.u32", g.col);
    std::cout << "BOUNDARY_DUMP cases=64\n";
    return 0;
}

// The TFS family on the boundary graphs. Inputs (BF16 X, L, R from the BF16
// lr policy, prescan max) come from the reference's own stages and are dumped
// with the outputs, so the restatement is checked on identical inputs.
static int tfs(const std::string& out) {
    int cases = 0;
    for (int D : {17, 33, 128, 256})
        for (int K : {1, 2, 4, 8})
            for (int d : {7, 32, 40, 47}) {
                Graph g = boundary_graph(D);
                Param p = boundary_params(D, K, d);
                Prepared q = prepare(p, true, true, true);
                Schedule s = degree_schedule(g);
                Workspace w;
                w.allocate(g, p, "tfs_bf16");
                convert(g.x.data(), w.xbf.data(), g.x.size());
                lr_reordered(g, p, q, g.x, w, "bf16");
                std::vector<float> lbf = w.left, rbf = w.right;
                lr_reordered(g, p, q, g.x, w, "fp32");
                std::vector<float> l32 = w.left, r32 = w.right;
                w.left = lbf;
                w.right = rbf;
                max_prescan(g, p, w);
                Times t;
                tfs_aggregate(g, p, q, s, w, 16, t);
                std::string pre = out + "/tfs_" + std::to_string(D) + "_" + std::to_string(K) + "_" + std::to_string(d);
                dumpv(pre + "_xbf.u16", w.xbf);
                dumpv(pre + "_w.f32", p.w);
                dumpv(pre + "_al.f32", p.al);
                dumpv(pre + "_ar.f32", p.ar);
                dumpv(pre + "_blr.f32", q.blr);
                dumpv(pre + "_lbf.f32", lbf);
                dumpv(pre + "_rbf.f32", rbf);
                dumpv(pre + "_l32.f32", l32);
                dumpv(pre + "_r32.f32", r32);
                dumpv(pre + "_max.f32", w.max);
                dumpv(pre + "_b1_out.f32", w.out);
                dumpv(pre + "_b1_den.f32", w.den);
                {
                    icpp_online::Workspace o;
                    o.allocate(g, p, true);  // with the exact counters (icpp_online.hpp:18-22)
                    o.base.xbf = w.xbf; o.base.left = lbf; o.base.right = rbf;
                    icpp_online::Stats st;
                    icpp_online::aggregate(g, p, q, s, o, 16, 16, st, 0, true);
                    dumpv(pre + "_online16_out.f32", o.base.out);
                    dumpv(pre + "_online16_den.f32", o.base.den);
                    dumpv(pre + "_online16_max.f32", o.base.max);
                    dumpv(pre + "_online16_rowblocks.u64", o.row_blocks);
                    dumpv(pre + "_online16_rowupdates.u64", o.row_max_updates);
                    dumpv(pre + "_online16_rowrescales.u64", o.row_rescales);
                    const std::vector<uint64_t> totals = {st.blocks, st.max_updates, st.rescales, st.rescale_events,
                                                          st.neighbor_steps, st.amx_calls, st.executed_fma,
                                                          st.rescaled_feature_elements,
                                                          st.rescaled_padded_feature_elements, st.spill_bytes,
                                                          st.reload_bytes};
                    dumpv(pre + "_online16_counters.u64", totals);
                }
                {
                    icpp_block::Workspace b;
                    b.allocate(g, p);
                    auto& bb = b.original.base;
                    bb.xbf = w.xbf; bb.left = lbf; bb.right = rbf;
                    icpp_block::Stats st;
                    icpp_block::aggregate(g, p, q, s, b, 32, 16, st);
                    dumpv(pre + "_block32_out.f32", bb.out);
                    dumpv(pre + "_block32_den.f32", bb.den);
                    dumpv(pre + "_block32_max.f32", bb.max);
                }
                {
                    icpp_heads_hybrid::Workspace hw;
                    hw.allocate(g, p);
                    auto& hb = hw.fallback.original.base;
                    hb.xbf = w.xbf; hb.left = lbf; hb.right = rbf;
                    icpp_heads_hybrid::Stats st;
                    icpp_heads_hybrid::aggregate(g, p, q, s, hw, 32, 16, st, 0, false, 16);
                    dumpv(pre + "_hybrid32_out.f32", hb.out);
                    dumpv(pre + "_hybrid32_den.f32", hb.den);
                    dumpv(pre + "_hybrid32_max.f32", hb.max);
                }
                ++cases;
            }
    std::cout << "TFS_DUMP cases=" << cases << "\n";
    return 0;
}

// icpp_online's exact counters (icpp_online.hpp:18-22) on a real graph, with
// attention scores that rise with the source id so later neighbour blocks
// raise the running maximum (the boundary graph's periodic sources never do).
static int counters(const std::string& graph, const std::string& out) {
    Graph g = load_graph(graph);
    const int K = 8, d = 32;
    Param p = boundary_params(g.din, K, d);
    Prepared q = prepare(p, true, true, true);
    Schedule s = degree_schedule(g);
    std::vector<float> left(g.n * K), right(g.n * K);
    for (uint64_t i = 0; i < g.n; ++i)
        for (int h = 0; h < K; ++h) {
            left[i * K + h] = std::sin(0.1f * float(i) + float(h));
            right[i * K + h] = 0.004f * float(i) * float(h + 1) + std::sin(0.7f * float(i) + float(h));
        }
    dumpv(out + "/counters_left.f32", left);
    dumpv(out + "/counters_right.f32", right);
    for (int block : {4, 16, 64}) {
        icpp_online::Workspace o;
        o.allocate(g, p, true);
        o.base.xbf.resize(g.x.size());
        convert(g.x.data(), o.base.xbf.data(), g.x.size());
        o.base.left = left;
        o.base.right = right;
        icpp_online::Stats st;
        icpp_online::aggregate(g, p, q, s, o, block, 16, st, 0, true);
        const std::string pre = out + "/counters_b" + std::to_string(block);
        dumpv(pre + "_rowblocks.u64", o.row_blocks);
        dumpv(pre + "_rowupdates.u64", o.row_max_updates);
        dumpv(pre + "_rowrescales.u64", o.row_rescales);
        const std::vector<uint64_t> totals = {st.blocks, st.max_updates, st.rescales, st.rescale_events,
                                              st.neighbor_steps, st.amx_calls, st.executed_fma,
                                              st.rescaled_feature_elements, st.rescaled_padded_feature_elements,
                                              st.spill_bytes, st.reload_bytes};
        dumpv(pre + "_totals.u64", totals);
    }
    // icpp_block's and icpp_heads_hybrid's statistics with exact counters on the
    // same inputs (icpp_block.hpp:17-26, icpp_heads.hpp:16-27)
    auto base_fields = [](const icpp_online::Stats& st) {
        return std::vector<uint64_t>{st.blocks, st.max_updates, st.rescales, st.rescale_events, st.neighbor_steps,
                                     st.amx_calls, st.executed_fma, st.rescaled_feature_elements,
                                     st.rescaled_padded_feature_elements, st.spill_bytes, st.reload_bytes,
                                     st.total_tiles};
    };
    for (int block : {16, 32}) {
        icpp_block::Workspace b;
        b.allocate(g, p, true);
        auto& bb = b.original.base;
        bb.xbf.resize(g.x.size());
        convert(g.x.data(), bb.xbf.data(), g.x.size());
        bb.left = left;
        bb.right = right;
        icpp_block::Stats st;
        icpp_block::aggregate(g, p, q, s, b, block, 16, st, 0, true);
        std::vector<uint64_t> v = base_fields(st.baseline);
        for (uint64_t x : {st.actual_input_feature_FMA, st.padded_input_feature_FMA, st.useful_projection_FMA,
                           st.logical_H_bytes, st.block_projection_calls, st.conversion_elements,
                           st.source_neighbor_steps})
            v.push_back(x);
        dumpv(out + "/counters_block" + std::to_string(block) + "_stats.u64", v);
        for (int threshold : {1, 16, 33}) {
            icpp_heads_hybrid::Workspace hw;
            hw.allocate(g, p, true);
            auto& hb = hw.fallback.original.base;
            hb.xbf = bb.xbf;
            hb.left = left;
            hb.right = right;
            icpp_heads_hybrid::Stats hs;
            icpp_heads_hybrid::aggregate(g, p, q, s, hw, block, 16, hs, 0, true, threshold);
            std::vector<uint64_t> u = base_fields(hs.baseline);
            for (uint64_t x : {uint64_t(hs.optimized), hs.ph_calls, hs.ph_physical_fma, hs.ph_useful_fma,
                               hs.raw_H_bytes, hs.packed_H_bytes, hs.projection_calls, hs.head_switch_store_bytes,
                               hs.head_switch_reload_bytes, hs.ub_scatter_bytes})
                u.push_back(x);
            dumpv(out + "/counters_hybrid" + std::to_string(block) + "_t" + std::to_string(threshold) + "_stats.u64",
                  u);
        }
    }
    std::cout << "COUNTERS_DUMP n=" << g.n << " e=" << g.e << "\n";
    return 0;
}

static int chain(const std::string& graph, const std::string& weights, const std::string& out) {
    Graph g = load_graph(graph);
    Model model;
    if (weights.rfind("seed:", 0) == 0) {
        model = random_model(g.din, g.classes, std::stoi(weights.substr(5)));
        save_model(model, out + "/weights.gatwgt");
    } else {
        model = load_model(weights, g.din, g.classes);
    }
    Schedule s = degree_schedule(g);
    dumpv(out + "/perm.u32", s.perm);
    dump(out + "/steps.u64", &s.neighbor_steps, 8);
    // R0 chain with per-layer intermediates.
    std::vector<float> input = g.x;
    for (int l = 0; l < 3; ++l) {
        Workspace w;
        w.allocate(g, model[l], "ref_fp32");
        Times t;
        ref_layer(g, model[l], input, w, l < 2, t);
        std::string pre = out + "/ref_l" + std::to_string(l + 1);
        dumpv(pre + "_left.f32", w.left);
        dumpv(pre + "_right.f32", w.right);
        dumpv(pre + "_max.f32", w.max);
        dumpv(pre + "_den.f32", w.den);
        dumpv(pre + "_out.f32", w.out);
        input = std::move(w.out);
    }
    // B0 chains (each path consumes its own previous output, bench/main.cpp:95-96).
    for (bool fp32 : {false, true}) {
        std::vector<Prepared> prep;
        for (const auto& p : model) prep.push_back(prepare(p));
        std::vector<float> in = g.x;
        for (int l = 0; l < 3; ++l) {
            Workspace w;
            w.allocate(g, model[l], fp32 ? "standard_fp32" : "standard_bf16");
            Times t;
            standard_layer(g, model[l], prep[l], in, w, l < 2, t, fp32);
            in = std::move(w.out);
        }
        dumpv(out + (fp32 ? "/b0fp32_out.f32" : "/b0bf16_out.f32"), in);
    }
    // TFS BF16 chain (bench/main.cpp:23 path tfs_bf16, lr policy bf16, panel 16).
    {
        std::vector<Prepared> prep;
        for (const auto& p : model) prep.push_back(prepare(p, true, true, true));
        std::vector<float> in = g.x;
        for (int l = 0; l < 3; ++l) {
            Workspace w;
            w.allocate(g, model[l], "tfs_bf16");
            Times t;
            tfs_layer(g, model[l], prep[l], s, in, w, l < 2, 16, t, "bf16");
            in = std::move(w.out);
        }
        dumpv(out + "/tfsbf16_out.f32", in);
    }
    std::cout << "CHAIN_DUMP n=" << g.n << " e=" << g.e << "\n";
    return 0;
}

int main(int argc, char** argv) {
    try {
        omp_set_num_threads(8);
        std::string mode = argc > 1 ? argv[1] : "";
        if (mode == "boundary" && argc == 3) return boundary(argv[2]);
        if (mode == "chain" && argc == 5) return chain(argv[2], argv[3], argv[4]);
        if (mode == "tfs" && argc == 3) return tfs(argv[2]);
        if (mode == "counters" && argc == 4) return counters(argv[2], argv[3]);
        std::cerr << "usage: ref_dump boundary OUTDIR | ref_dump chain GRAPH WEIGHTS OUTDIR | ref_dump tfs OUTDIR | "
                     "ref_dump counters GRAPH OUTDIR\n";
        return 2;
    } catch (const std::exception& e) {
        std::cerr << "FAIL " << e.what() << "\n";
        return 1;
    }
}
