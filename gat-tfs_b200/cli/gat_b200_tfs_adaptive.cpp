// gat_b200_tfs_adaptive: the reference's adaptive TFS experiment driver
// (baseline/tfs_online/adaptive_main.cpp) on the B200 library, through the C ABI.
//
//   gat_b200_tfs_adaptive GRAPH THREADS WARMUPS REPEATS PROFILE_PERIOD | --smoke
//
// Paths, as the reference names them:
//   B0_BF16                the standard BF16 layer in all three layers;
//   HYBRID_T16_B32         icpp_heads_hybrid in every layer (blocks of 32
//                          neighbours, PH from BF16 high/low p for blocks of at
//                          least 16), layer 3 outside heads 8 / dim 32 through
//                          icpp_block, as the reference falls back;
//   TFS_L12_B0_L3_MATCHED  the hybrid in layers 1-2, layer 3 the standard BF16
//                          layer with L/R from lr_reordered ("fp32").
// Same output lines: CONFIG, PATH_SEMANTICS, STATIC per layer; CHECK lines
// (the 0.003 absolute gate) of every path's chain against the B0 FP32 chain,
// of the hybrid layer 2 against the FP32 layer with the same contracted L/R on
// a common input, and of the matched layer 3 against the full hybrid layer 3;
// one JSON line per path, repeat and layer; PROFILE_IDENTITY, HYBRID_MIX,
// PROFILE, ONLINE_STATS and HEAD_WORK per hybrid layer with the counters exact
// (the Online units from gat_b200_tfs_online_counters, the work counts from
// the CSR and the degree order as the reference's own identities state them);
// ICPP_ADAPTIVE_COMPLETE / ICPP_HEADS_COMPLETE, or ICPP_HEADS_FAIL <message>
// and exit status 1. All layers run on the current CUDA device with
// device-resident buffers; a layer is timed on the host clock around the call
// and a device synchronisation. THREADS is validated and reported; the
// per-worker AMX timers of the reference's PROFILE line have no counterpart on
// the GPU and print as 0.
#include <algorithm>
#include <array>
#include <cmath>
#include <cstring>
#include <iomanip>
#include <iostream>
#include <string>
#include <vector>

#include "driver_common.hpp"
#include "gat_b200_online.hpp"

namespace gat = gat_b200;

namespace {

using gat::check;
using gat::Clock;
using gat::seconds;
using gat_b200_cli::boundary_graph;
using gat_b200_cli::difference;
using gat_b200_cli::fingerprint;

void report(const std::string& path, int layer, const std::string& ref, const gat::Error& e) {
    gat_b200_cli::report(path, layer, ref, e, "nonfinite output");
}

constexpr int kBlock = 32, kThreshold = 16;

enum Kind { kStandard, kHybrid, kMatchedL3 };
struct Path {
    std::string name;
    Kind kind;
};

bool optimized_shape(const gat::Param& p) { return p.heads == 8 && p.dim == 32 && p.in > 0 && p.in <= 256; }

// Device state of one (graph, model): the layers, the scratch tables and the
// output of every layer.
struct Runner {
    const gat::Graph& g;
    const gat::Model& model;
    gat::detail::GraphHandle graph;
    gat_b200_layer* layer[3] = {nullptr, nullptr, nullptr};
    gat::detail::DeviceBuffer x, xb, h, left, right, max, den, out[3], rows;
    double prepare_ms[3] = {0, 0, 0};
    Runner(const gat::Graph& g_, const gat::Model& m) : g(g_), model(m) {
        graph.of(g);
        for (int l = 0; l < 3; ++l) {
            const auto t0 = Clock::now();
            check(gat_b200_layer_create(m[l].in, m[l].heads, m[l].dim, m[l].w.data(), m[l].al.data(),
                                        m[l].ar.data(), &layer[l]));
            prepare_ms[l] = seconds(t0, Clock::now()) * 1000;
        }
    }
    ~Runner() {
        for (auto* p : layer) gat_b200_layer_destroy(p);
    }
    float* L(int l) { return static_cast<float*>(left.get(size_t(g.n) * model[l].heads * 4)); }
    float* R(int l) { return static_cast<float*>(right.get(size_t(g.n) * model[l].heads * 4)); }
    // The standard layer (baseline_standard.cpp:98-108) from FP32 device rows
    // `in` [n][in] into out[l]: BF16, or FP32 with fp32; with matched the L/R
    // come from lr_reordered "fp32" (the FP32 input times W a). Returns ms.
    double standard(int l, const float* in, bool hidden, bool fp32, bool matched) {
        const gat::Param& p = model[l];
        const uint64_t n = g.n;
        const int K = p.heads, W = p.width();
        float* o = static_cast<float*>(out[l].get(size_t(n) * W * 4));
        float *lp = L(l), *rp = R(l);
        const int hd = fp32 ? GAT_B200_F32 : GAT_B200_BF16;
        const int ldh = gat_b200_padded_ld(W, hd);
        void* hs = h.get(size_t(n) * ldh * (fp32 ? 4 : 2));
        const auto t0 = Clock::now();
        const void* xin = in;
        int ldx = p.in;
        if (!fp32) {
            ldx = gat_b200_padded_ld(p.in, GAT_B200_BF16);
            void* xs = xb.get(size_t(n) * ldx * 2);
            check(gat_b200_convert(n, p.in, in, p.in, static_cast<uint16_t*>(xs), ldx, nullptr));
            xin = xs;
        }
        if (!matched) {
            check(gat_b200_standard_layer(graph.g, layer[l], xin, ldx,
                                          fp32 ? GAT_B200_PATH_STANDARD_FP32 : GAT_B200_PATH_STANDARD_BF16, hidden, hs,
                                          lp, rp, o, GAT_B200_F32, W, nullptr));
        } else {
            check(gat_b200_projection(layer[l], n, xin, ldx, hd, hs, hd, ldh, lp, rp, nullptr));
            check(gat_b200_lr_reordered(layer[l], n, in, GAT_B200_F32, p.in, GAT_B200_LR_FP32, nullptr, 0, lp, rp,
                                        nullptr));
            check(gat_b200_aggregate_fused(graph.g, K, p.dim, hs, hd, ldh, lp, rp, hidden, o, GAT_B200_F32, W,
                                           nullptr));
        }
        check(gat_b200_check_device());
        return seconds(t0, Clock::now()) * 1000;
    }
    // icpp_heads_hybrid::layer (icpp_heads_hybrid.hpp:21-24, "fp32" LR): SPLIT
    // rounding with the running maximum for the optimized shape, else
    // icpp_block's BLOCK rounding. Returns ms.
    double hybrid(int l, const float* in, bool hidden) {
        const gat::Param& p = model[l];
        const uint64_t n = g.n;
        const int K = p.heads, W = p.width();
        const bool opt = optimized_shape(p);
        float* o = static_cast<float*>(out[l].get(size_t(n) * W * 4));
        const int ldb = gat_b200_padded_ld(p.in, GAT_B200_BF16);
        void* xs = xb.get(size_t(n) * ldb * 2);
        float* M = static_cast<float*>(max.get(size_t(n) * K * 4));
        float* D = static_cast<float*>(den.get(size_t(n) * K * 4));
        const auto t0 = Clock::now();
        check(gat_b200_tfs_layer(graph.g, layer[l], in, GAT_B200_F32, p.in, hidden, GAT_B200_LR_FP32,
                                 opt ? GAT_B200_TFS_SPLIT : GAT_B200_TFS_BLOCK, kBlock, opt ? kThreshold : 1, xs, L(l),
                                 R(l), M, D, o, GAT_B200_F32, W, nullptr));
        check(gat_b200_check_device());
        return seconds(t0, Clock::now()) * 1000;
    }
    double run_layer(const Path& path, int l, const float* in, bool hidden) {
        if (path.kind == kStandard || (path.kind == kMatchedL3 && l == 2))
            return standard(l, in, hidden, false, path.kind == kMatchedL3);
        return hybrid(l, in, hidden);
    }
    std::vector<float> output(int l) {
        std::vector<float> v(size_t(g.n) * model[l].width());
        out[l].download(v);
        return v;
    }
    const float* upload_input(const std::vector<float>& v) { return x.upload(v); }
    void chain(const Path& path, std::array<double, 3>& ms) {
        const float* in = upload_input(g.x);
        for (int l = 0; l < 3; ++l) {
            ms[l] = run_layer(path, l, in, l < 2);
            in = static_cast<const float*>(out[l].p);
        }
    }
};

// The exact counters of the hybrid layer just run (its L/R are in the
// runner's buffers), the reference's identities checked against them, and the
// PROFILE / ONLINE_STATS / HEAD_WORK / HYBRID_MIX lines (adaptive_main.cpp:36-77).
void profile(Runner& run, const gat::Schedule& sched, const std::string& name, int l, double layer_ms,
             int period) {
    const gat::Param& p = run.model[l];
    const gat::Graph& g = run.g;
    const uint64_t K = uint64_t(p.heads), nk = g.n * K;
    uint64_t* rows = static_cast<uint64_t*>(run.rows.get(3 * nk * 8));
    uint64_t tot[5];
    check(gat_b200_tfs_online_counters(run.graph.g, p.heads, run.L(l), run.R(l), kBlock, rows, rows + nk,
                                       rows + 2 * nk, tot, nullptr));
    std::vector<uint64_t> rb(nk), ru(nk), rr(nk);
    check(gat_b200_copy_to_host(rb.data(), rows, nk * 8));
    check(gat_b200_copy_to_host(ru.data(), rows + nk, nk * 8));
    check(gat_b200_copy_to_host(rr.data(), rows + 2 * nk, nk * 8));
    gat::Prepared q;
    q.padded_in = (p.in + 31) / 32 * 32;
    q.output_blocks = (p.dim + 15) / 16;
    gat::icpp_heads_hybrid::Stats st;
    const bool opt = optimized_shape(p);
    if (opt) {
        st.optimized = true;
        gat::icpp_heads_hybrid::detail::stats_of(g, p, q, sched, kBlock, kThreshold, tot, st);
    } else {
        gat::icpp_block::Stats bs;
        gat::detail::block_stats(g, p, q, sched, kBlock, tot, bs);
        st.baseline = bs.baseline;
        st.projection_calls = bs.block_projection_calls;
    }
    gat::detail::tiles(g, p.heads, period, true, st.baseline);
    const auto& s = st.baseline;
    uint64_t blocks = 0, updates = 0, rescales = 0;
    std::vector<double> ratios(nk);
    for (size_t i = 0; i < nk; ++i) {
        blocks += rb[i];
        updates += ru[i];
        rescales += rr[i];
        ratios[i] = rb[i] ? double(rr[i]) / rb[i] : 0;
    }
    if (blocks != s.blocks || updates != s.max_updates || rescales != s.rescales ||
        s.rescaled_feature_elements != rescales * uint64_t(p.dim))
        throw std::runtime_error("heads per-row identity");
    const uint64_t dp = uint64_t(q.padded_in), in16 = (uint64_t(p.in) + 15) / 16 * 16;
    if (opt) {
        uint64_t rowblocks = 0, groups = 0, nonempty = 0, avx = 0, amx = 0, avx_edges = 0;
        for (uint64_t i = 0; i < g.n; ++i) {
            const uint64_t deg = g.row[i + 1] - g.row[i];
            rowblocks += (deg + kBlock - 1) / kBlock;
            for (uint64_t b = 0; b < deg; b += kBlock) {
                const uint64_t len = std::min<uint64_t>(kBlock, deg - b);
                if (len < uint64_t(kThreshold)) {
                    ++avx;
                    avx_edges += len;
                } else {
                    ++amx;
                }
            }
        }
        for (uint64_t first = 0; first < g.n; first += 16) {
            uint64_t md = 0;
            for (uint64_t k = first; k < std::min<uint64_t>(g.n, first + 16); ++k) {
                const uint32_t r = sched.perm[k];
                md = std::max<uint64_t>(md, g.row[r + 1] - g.row[r]);
            }
            groups += (md + kBlock - 1) / kBlock;
            nonempty += md > 0;
        }
        if (blocks != rowblocks * K || st.ph_useful_fma != g.e * K * uint64_t(p.in) ||
            st.raw_H_bytes != g.e * uint64_t(p.in) * 2 || st.projection_calls != groups * K ||
            s.amx_calls != st.projection_calls * (dp / 32) * 2 || s.executed_fma != st.projection_calls * 16 * dp * 32 ||
            st.head_switch_store_bytes != groups * K * 2048 ||
            st.head_switch_reload_bytes != (groups - nonempty) * K * 2048 || s.spill_bytes || s.reload_bytes)
            throw std::runtime_error("heads work identity");
        if (avx + amx != rowblocks || st.ph_calls != amx * (dp / 16) * 2 ||
            st.ph_physical_fma != amx * K * 32 * dp * 2 + avx_edges * K * in16 ||
            st.packed_H_bytes != amx * 32 * dp * 2 || st.ub_scatter_bytes != amx * K * dp * 4 + avx * K * in16 * 4)
            throw std::runtime_error("hybrid PH work identity");
        std::cout << "HYBRID_MIX path=" << name << " layer=" << l + 1 << " threshold=" << kThreshold
                  << " avx_rowblocks=" << avx << " amx_rowblocks=" << amx << " avx_edges=" << avx_edges
                  << " AMX_P_tile_load_bytes=" << amx * 1024 << " physical_to_useful_PH_FMA="
                  << (st.ph_useful_fma ? double(st.ph_physical_fma) / st.ph_useful_fma : 0) << "\n";
    }
    std::sort(ratios.begin(), ratios.end());
    auto pct = [&](double f) {
        return ratios.empty() ? 0 : ratios[std::min(ratios.size() - 1, size_t(std::ceil(f * ratios.size())) - 1)];
    };
    std::cout << std::setprecision(12) << "PROFILE path=" << name << " layer=" << l + 1 << " optimized=" << opt
              << " layer_wall_ms=" << layer_ms << " kernel_wall_ms=" << layer_ms
              << " sampled_head_tiles=" << s.sampled_tiles
              << " worker_times_are_sampled_sums=true worker_times=unavailable_on_gpu\n";
    std::cout << "ONLINE_STATS path=" << name << " layer=" << l + 1 << " block=" << kBlock << " heads=" << p.heads
              << " D=" << p.in << " d=" << p.dim << " edges=" << g.e << " blocks=" << blocks
              << " max_updates_including_initial=" << updates << " rescales=" << rescales
              << " rescale_per_block=" << (blocks ? double(rescales) / blocks : 0) << " P50=" << pct(.5)
              << " P90=" << pct(.9) << " P95=" << pct(.95) << " P99=" << pct(.99)
              << " rescaled_feature_elements=" << s.rescaled_feature_elements << " rescale_events=" << s.rescale_events
              << " spill_bytes=" << s.spill_bytes << " reload_bytes=" << s.reload_bytes << " UW_calls=" << s.amx_calls
              << " UW_physical_FMA=" << s.executed_fma << " head_tiles=" << s.total_tiles
              << " projection_groups=" << st.projection_calls << " cpu_schedule_counters=modelled_not_measured_on_gpu\n";
    std::cout << "HEAD_WORK path=" << name << " layer=" << l + 1 << " optimized=" << opt << " PH_calls=" << st.ph_calls
              << " PH_physical_FMA=" << st.ph_physical_fma << " PH_useful_FMA=" << st.ph_useful_fma
              << " raw_H_bytes=" << st.raw_H_bytes << " packed_H_bytes=" << st.packed_H_bytes
              << " UB_scatter_bytes=" << st.ub_scatter_bytes << " head_switch_store_bytes="
              << st.head_switch_store_bytes << " head_switch_reload_bytes=" << st.head_switch_reload_bytes
              << " sparse_width_amplification=" << double(p.in) / p.dim
              << " traffic_is_logical_not_DRAM=true no_full_Z_U_e_alpha=true bounded_V_in_local_memory=true"
              << " cpu_schedule_counters=modelled_not_measured_on_gpu\n";
}


// --smoke: on the boundary graph, the hybrid with threshold 33 (every block on
// the FP32-p side) equals icpp_block, and thresholds 1 and 16 (high/low p on
// long blocks) stay within the split's rounding of it.
int smoke() {
    int cases = 0;
    for (int D : {17, 128}) {
        gat::Graph g = boundary_graph(D);
        gat::Model m = gat::random_model(D, 4, 11);
        gat::detail::GraphHandle graph;
        graph.of(g);
        gat_b200_layer* lay = nullptr;
        check(gat_b200_layer_create(m[0].in, m[0].heads, m[0].dim, m[0].w.data(), m[0].al.data(), m[0].ar.data(),
                                    &lay));
        const uint64_t n = g.n;
        const int K = m[0].heads, W = m[0].width(), ldb = gat_b200_padded_ld(D, GAT_B200_BF16);
        gat::detail::DeviceBuffer x, xb, l, r, mx, dn, o;
        const float* xin = x.upload(g.x);
        void* xs = xb.get(n * ldb * 2);
        float *lp = static_cast<float*>(l.get(n * K * 4)), *rp = static_cast<float*>(r.get(n * K * 4));
        float *mp = static_cast<float*>(mx.get(n * K * 4)), *dp = static_cast<float*>(dn.get(n * K * 4));
        float* op = static_cast<float*>(o.get(n * W * 4));
        auto layer = [&](int rounding, int threshold) {
            check(gat_b200_tfs_layer(graph.g, lay, xin, GAT_B200_F32, D, 0, GAT_B200_LR_FP32, rounding, kBlock,
                                     threshold, xs, lp, rp, mp, dp, op, GAT_B200_F32, W, nullptr));
            std::vector<float> v(n * W);
            o.download(v);
            return v;
        };
        const std::vector<float> block = layer(GAT_B200_TFS_BLOCK, 1);
        for (int t : {33, 16, 1}) {
            const gat::Error e = difference(block, layer(GAT_B200_TFS_SPLIT, t));
            const double tol = t == 33 ? 0 : 2e-3;  // a BF16 step of U flipped by the high/low split
            if (!e.finite || e.max_abs > tol)
                throw std::runtime_error("smoke: hybrid threshold " + std::to_string(t) + " differs from icpp_block");
            ++cases;
        }
        gat_b200_layer_destroy(lay);
    }
    std::cout << "SMOKE PASS cases=" << cases << " hybrid_thresholds=33,16,1_vs_icpp_block\n";
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        if (argc == 2 && std::string(argv[1]) == "--smoke") return smoke();
        if (argc != 6) throw std::runtime_error("usage: icpp_heads GRAPH THREADS WARMUPS REPEATS PROFILE_PERIOD | --smoke");
        const int threads = std::stoi(argv[2]), warm = std::stoi(argv[3]), reps = std::stoi(argv[4]),
                  period = std::stoi(argv[5]);
        if (threads < 1 || warm < 0 || reps < 1 || period < 1) throw std::runtime_error("invalid configuration");
        const gat::Graph g = gat::load_graph(argv[1]);
        const gat::Model model = gat::random_model(g.din, g.classes, 11);
        const gat::Schedule sched = gat::degree_schedule(g);
        Runner run(g, model);
        const std::vector<Path> paths = {
            {"B0_BF16", kStandard}, {"HYBRID_T16_B32", kHybrid}, {"TFS_L12_B0_L3_MATCHED", kMatchedL3}};
        std::cout << std::setprecision(12) << "CONFIG N=" << g.n << " E=" << g.e << " Din=" << g.din << " C=" << g.classes
                  << " threads=" << threads << " check_runs=1 warmups=" << warm << " repeats=" << reps
                  << " degree_sort_ms=" << sched.degree_sort_s * 1000
                  << " seed=11 untrained=true LR_policy=fp32 panel=64 tile_rows=16 attention_independent=true"
                  << " master_abs_gate=.003 performance=EXPLORATORY task_accuracy=UNVERIFIED device=sm_100a\n";
        std::cout << "PATH_SEMANTICS B0_BF16=standard_transform_first_all_layers"
                     " HYBRID_T16_B32=TFS_DegreeSort_TR16_Online_PH_UW_all_layers_with_L3_original_block_fallback"
                     " TFS_L12_B0_L3_MATCHED=TFS_hybrid_L1_L2_plus_standard_BF16_transform_first_L3_with_contracted_FP32_LR\n";
        // the B0 FP32 chain: the master of every CHECK
        std::array<std::vector<float>, 3> master;
        {
            const float* in = run.upload_input(g.x);
            for (int l = 0; l < 3; ++l) {
                run.standard(l, in, l < 2, true, false);
                master[l] = run.output(l);
                in = static_cast<const float*>(run.out[l].p);
            }
        }
        for (int l = 0; l < 3; ++l) {
            const gat::Param& p = model[l];
            const bool opt = optimized_shape(p);
            std::cout << "STATIC layer=" << l + 1 << " weight_and_bLR_prepare_ms=" << run.prepare_ms[l]
                      << " heads_workspace_bytes=" << g.n * uint64_t(p.heads) * 16 << " full_Z_bytes=0"
                      << " edge_score_bytes=0 alpha_bytes=0 optimized_U_bytes=0 local_V_bytes=0"
                      << " optimized=" << opt << "\n";
        }
        // timed three-layer chains, AB/BA order (adaptive_main.cpp:95-100)
        for (int rep = -warm - 1; rep < reps; ++rep) {
            auto order = paths;
            if (rep >= 0 && rep % 2) std::reverse(order.begin(), order.end());
            for (const auto& path : order) {
                std::array<double, 3> ms{};
                const auto begin = Clock::now();
                run.chain(path, ms);
                const double e2e = seconds(begin, Clock::now()) * 1000;
                if (rep == -warm - 1)
                    for (int l = 0; l < 3; ++l)
                        report(path.name, l + 1, "B0_FP32_own_output_3layer", difference(master[l], run.output(l)));
                if (rep >= 0) {
                    gat::require_finite(run.output(2), path.name);
                    for (int l = 0; l < 3; ++l) {
                        const bool online = path.kind != kStandard && !(path.kind == kMatchedL3 && l == 2);
                        std::cout << "{\"path\":\"" << path.name << "\",\"rep\":" << rep << ",\"layer\":" << l + 1
                                  << ",\"e2e_ms\":" << e2e << ",\"layer_ms\":" << ms[l]
                                  << ",\"projection_ms\":0,\"conversion_ms\":0,\"lr_ms\":0,\"max_prescan_ms\":0"
                                  << ",\"kernel_ms\":" << ms[l] << ",\"normalization_ms\":0,\"activation_ms\":0"
                                  << ",\"block\":" << (online ? kBlock : 0) << "}\n";
                    }
                }
            }
        }
        // common-input controls (adaptive_main.cpp:102-107): the hybrid layer 2
        // against the FP32 layer with the same contracted L/R, no ELU; the
        // matched layer 3 against the full hybrid's layer 3 on its input
        {
            const float* in = run.upload_input(master[0]);
            run.standard(1, in, false, true, true);
            const std::vector<float> fp32 = run.output(1);
            for (const auto& path : paths)
                if (path.kind != kStandard) {
                    run.hybrid(1, in, false);
                    report(path.name, 2, "FP32_same_input_same_contracted_LR_no_ELU", difference(fp32, run.output(1)));
                }
            std::array<double, 3> ms{};
            run.chain(paths[1], ms);
            const std::vector<float> full_l3 = run.output(2);
            run.standard(2, static_cast<const float*>(run.out[1].p), false, false, true);
            report("TFS_L12_B0_L3_MATCHED", 3, "same_input_full_TFS_L3", difference(full_l3, run.output(2)));
        }
        // profile identity and the exact counters of the hybrid (adaptive_main.cpp:108-111)
        {
            const Path& path = paths[1];
            std::array<double, 3> ms{};
            run.chain(path, ms);
            std::array<uint64_t, 3> hashes{};
            for (int l = 0; l < 3; ++l) hashes[l] = fingerprint(run.output(l));
            const float* in = run.upload_input(g.x);
            for (int l = 0; l < 3; ++l) {
                const double t = run.hybrid(l, in, l < 2);
                in = static_cast<const float*>(run.out[l].p);
                const bool same = hashes[l] == fingerprint(run.output(l));
                std::cout << "PROFILE_IDENTITY path=" << path.name << " layer=" << l + 1
                          << " bit_fingerprint_equal=" << same << "\n";
                if (!same) throw std::runtime_error("heads profile changed output");
                profile(run, sched, path.name, l, t, period);
            }
        }
        std::cout << "ICPP_ADAPTIVE_COMPLETE hybrid_smoke_and_same_input_L3_control=true\n";
        std::cout << "ICPP_HEADS_COMPLETE architecture=B200_TFS_heads_hybrid_in_L1_L2_for_mixed_path"
                     " no_global_U_Z_e_alpha_in_TFS_layers=true independent_heads=true"
                     " source_width_amplification_retained=true master_gate=SEE_PER_LAYER_ERRORS"
                     " performance=EXPLORATORY task_accuracy=UNVERIFIED\n";
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "ICPP_HEADS_FAIL " << e.what() << "\n";
        return 1;
    }
}
