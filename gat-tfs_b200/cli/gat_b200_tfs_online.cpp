// gat_b200_tfs_online: the reference's online-TFS experiment driver
// (baseline/tfs_online/main.cpp) on the B200 library, through the C ABI.
//
//   gat_b200_tfs_online GRAPH THREADS WARMUPS REPEATS BLOCKS_CSV PROFILE_PERIOD | --smoke
//
// Same arguments and the same output lines, so its summaries read unchanged:
//   CONFIG, STATIC per layer; CHECK lines (max/mean abs and relative L2 error,
//   the 0.003 absolute gate) of every online block size against B1 with the
//   prescan maximum on a common input, the FP64 oracle on selected complete
//   neighbourhoods (ORACLE_COVERAGE, the global maximum-degree row included),
//   and every path's three-layer chain against its B0 FP32 output; one JSON
//   line per path, repeat and layer; PROFILE_IDENTITY, PROFILE and
//   ONLINE_STATS per online block size and layer, the counters exact
//   (gat_b200_tfs_online_counters: blocks, max updates, rescales, rescale
//   events and neighbor steps; the others derived as the reference does);
//   ICPP_ONLINE_COMPLETE, or ICPP_ONLINE_FAIL <message> and exit status 1.
// Paths: B0_FP32, B0_BF16 (standard layer), B1_TFS_PREMAX (TFS, prescan max),
// ICPP_TFS_ONLINE_B<b> (TFS with the running maximum per block of b). All
// layers run on the current CUDA device with device-resident buffers; a layer
// is timed on the host clock around the call and a device synchronisation.
// THREADS is validated and reported; the per-worker AMX timers of the
// reference's PROFILE line have no counterpart on the GPU.
#include <algorithm>
#include <array>
#include <cmath>
#include <cstring>
#include <iomanip>
#include <iostream>
#include <set>
#include <sstream>
#include <string>
#include <vector>

#include "driver_common.hpp"
#include "gat_b200.hpp"

namespace gat = gat_b200;

namespace {

using gat::check;
using gat::Clock;
using gat::seconds;
using gat_b200_cli::boundary_graph;
using gat_b200_cli::difference;
using gat_b200_cli::fingerprint;

void report(const std::string& path, int layer, const std::string& ref, const gat::Error& e) {
    gat_b200_cli::report(path, layer, ref, e, "nonfinite comparison");
}

struct Path {
    std::string name;
    int block = 0;  // > 0: online TFS with this block
};

// Device state of one (graph, model) and the layer of every path.
struct Runner {
    const gat::Graph& g;
    const gat::Model& model;
    gat::detail::GraphHandle graph;
    gat_b200_layer* layer[3] = {nullptr, nullptr, nullptr};
    gat::detail::DeviceBuffer x, xb, h, left, right, max, den, out[3], rb, ru, rr;
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
    // One layer of `path` from FP32 device rows `in` [n][in] into out[l] (FP32 [n][width]); ms.
    double run_layer(const Path& path, int l, const float* in, bool hidden) {
        const gat::Param& p = model[l];
        const uint64_t n = g.n;
        const int K = p.heads, W = p.width();
        float* o = static_cast<float*>(out[l].get(size_t(n) * W * 4));
        float* L = static_cast<float*>(left.get(size_t(n) * K * 4));
        float* R = static_cast<float*>(right.get(size_t(n) * K * 4));
        const auto t0 = Clock::now();
        if (path.name == "B0_FP32") {
            void* hs = h.get(size_t(n) * gat_b200_padded_ld(W, GAT_B200_F32) * 4);
            check(gat_b200_standard_layer(graph.g, layer[l], in, p.in, GAT_B200_PATH_STANDARD_FP32, hidden, hs, L, R, o,
                                          GAT_B200_F32, W, nullptr));
        } else if (path.name == "B0_BF16") {
            const int ld = gat_b200_padded_ld(p.in, GAT_B200_BF16);
            void* xs = xb.get(size_t(n) * ld * 2);
            check(gat_b200_convert(n, p.in, in, p.in, static_cast<uint16_t*>(xs), ld, nullptr));
            void* hs = h.get(size_t(n) * gat_b200_padded_ld(W, GAT_B200_BF16) * 2);
            check(gat_b200_standard_layer(graph.g, layer[l], xs, ld, GAT_B200_PATH_STANDARD_BF16, hidden, hs, L, R, o,
                                          GAT_B200_F32, W, nullptr));
        } else {
            const int ld = gat_b200_padded_ld(p.in, GAT_B200_BF16);
            void* xs = xb.get(size_t(n) * ld * 2);
            float* M = static_cast<float*>(max.get(size_t(n) * K * 4));
            float* D = static_cast<float*>(den.get(size_t(n) * K * 4));
            check(gat_b200_tfs_layer(graph.g, layer[l], in, GAT_B200_F32, p.in, hidden, GAT_B200_LR_FP32,
                                     GAT_B200_TFS_EDGE, path.block, 1, xs, L, R, M, D, o, GAT_B200_F32, W, nullptr));
        }
        check(gat_b200_check_device());
        return seconds(t0, Clock::now()) * 1000;
    }
    std::vector<float> output(int l) {
        std::vector<float> v(size_t(g.n) * model[l].width());
        out[l].download(v);
        return v;
    }
    const float* upload_input(const std::vector<float>& v) { return x.upload(v); }
    // Three layers from the graph's features; per-layer ms in ms[].
    void chain(const Path& path, std::array<double, 3>& ms) {
        const float* in = upload_input(g.x);
        for (int l = 0; l < 3; ++l) {
            ms[l] = run_layer(path, l, in, l < 2);
            in = static_cast<const float*>(out[l].p);
        }
    }
};

// FP64 diagnostic of one online TFS layer on a sample of destination rows
// with their complete neighbourhoods. The sample is taken along the degree
// order: the rows at 0, 25, 50, 75, 90, 99 and 99.9 % of it and the row of
// largest degree (the longest softmax the kernels run). For every sampled row
// the attention weights of all heads come first, from the same L/R the device
// used (exp in FP64 after the FP32 leaky score, as the device scores them);
// then one pass over the neighbours accumulates the weighted input rows per
// head, both the master FP32 input and its BF16 rounding; the head outputs are
// those sums times the master W and times the BF16 W, over the head's weight
// sum. Only the log keys of the reference's diagnostic
// (baseline/tfs_online/main.cpp:45, ORACLE_COVERAGE and its two CHECK
// references) are kept, so its summaries read this output too.
struct SampleRows {
    std::vector<uint32_t> rows;
    uint32_t hub = 0;
    uint64_t hub_degree = 0;
};

SampleRows sample_by_degree(const gat::Graph& g) {
    SampleRows s;
    std::vector<uint64_t> deg(g.n);
    for (uint64_t i = 0; i < g.n; ++i) deg[i] = g.row[i + 1] - g.row[i];
    std::vector<uint32_t> order(g.n);
    for (uint64_t i = 0; i < g.n; ++i) order[i] = uint32_t(i);
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return deg[a] < deg[b]; });
    const auto top = std::max_element(deg.begin(), deg.end());
    s.hub = uint32_t(top - deg.begin());
    s.hub_degree = *top;
    for (double q : {0.0, 0.25, 0.5, 0.75, 0.9, 0.99, 0.999})
        s.rows.push_back(order[size_t(q * double(g.n - 1))]);
    s.rows.push_back(s.hub);
    std::sort(s.rows.begin(), s.rows.end());
    s.rows.erase(std::unique(s.rows.begin(), s.rows.end()), s.rows.end());
    return s;
}

void fp64_row_diagnostic(const gat::Graph& g, const gat::Param& p, const std::vector<float>& input,
                         const std::vector<float>& left, const std::vector<float>& right,
                         const std::vector<float>& actual, int layer, const std::string& name) {
    const SampleRows sample = sample_by_degree(g);
    const int K = p.heads, D = p.in, W = p.width();
    const std::vector<float> in_bf = gat::quantized(input), w_bf = gat::quantized(p.w);
    std::vector<float> want_master, want_bf16, have;
    uint64_t edges = 0;
    for (uint32_t r : sample.rows) {
        const uint64_t b = g.row[r], deg = g.row[r + 1] - b;
        edges += deg;
        // attention weights [deg][K] and their sums per head
        std::vector<double> wgt(deg * K), wsum(K, 0.0);
        for (int h = 0; h < K; ++h) {
            double top = -INFINITY;
            for (uint64_t j = 0; j < deg; ++j) {
                const double sc = gat::leak(left[size_t(r) * K + h] + right[size_t(g.col[b + j]) * K + h]);
                wgt[j * K + h] = sc;
                top = std::max(top, sc);
            }
            for (uint64_t j = 0; j < deg; ++j) {
                wgt[j * K + h] = std::exp(wgt[j * K + h] - top);
                wsum[h] += wgt[j * K + h];
            }
        }
        // weighted input sums per head: master and BF16-rounded input rows
        std::vector<double> sum_master(size_t(K) * D, 0.0), sum_bf16(size_t(K) * D, 0.0);
        for (uint64_t j = 0; j < deg; ++j) {
            const size_t src = size_t(g.col[b + j]) * D;
            for (int h = 0; h < K; ++h) {
                const double a = wgt[j * K + h];
                double* um = &sum_master[size_t(h) * D];
                double* ub = &sum_bf16[size_t(h) * D];
                for (int k = 0; k < D; ++k) {
                    um[k] += a * input[src + k];
                    ub[k] += a * in_bf[src + k];
                }
            }
        }
        for (int h = 0; h < K; ++h)
            for (int d = 0; d < p.dim; ++d) {
                const int c = h * p.dim + d;
                double vm = 0, vb = 0;
                for (int k = 0; k < D; ++k) {
                    vm += sum_master[size_t(h) * D + k] * p.w[size_t(k) * W + c];
                    vb += sum_bf16[size_t(h) * D + k] * w_bf[size_t(k) * W + c];
                }
                const double inv = wsum[h] > 0 ? 1.0 / wsum[h] : 0.0;
                want_master.push_back(float(vm * inv));
                want_bf16.push_back(float(vb * inv));
                have.push_back(actual[size_t(r) * W + c]);
            }
    }
    std::cout << "ORACLE_COVERAGE layer=" << layer << " rows=" << sample.rows.size() << " edges=" << edges
              << " global_max_degree_node=" << sample.hub << " global_max_degree=" << sample.hub_degree
              << " global_max_degree_included=true complete_neighborhoods=true activation=false"
              << " outputs_rounded_to_fp32=true\n";
    report(name, layer, "FP64_master_same_LR_selected_rows", difference(want_master, have));
    report(name, layer, "FP64_quantized_H_W_same_LR_without_pH_quantization", difference(want_bf16, have));
}

// ONLINE_STATS (tfs_online/main.cpp:52-66) from the exact counters.
void online_stats(Runner& run, int l, int block) {
    const gat::Param& p = run.model[l];
    const gat::Graph& g = run.g;
    const size_t nk = size_t(g.n) * p.heads;
    uint64_t* rb = static_cast<uint64_t*>(run.rb.get(nk * 8));
    uint64_t* ru = static_cast<uint64_t*>(run.ru.get(nk * 8));
    uint64_t* rr = static_cast<uint64_t*>(run.rr.get(nk * 8));
    uint64_t tot[5];
    check(gat_b200_tfs_online_counters(run.graph.g, p.heads, static_cast<const float*>(run.left.p),
                                       static_cast<const float*>(run.right.p), block, rb, ru, rr, tot, nullptr));
    std::vector<uint64_t> hb(nk), hr(nk), hu(nk);
    check(gat_b200_copy_to_host(hb.data(), rb, nk * 8));
    check(gat_b200_copy_to_host(hu.data(), ru, nk * 8));
    check(gat_b200_copy_to_host(hr.data(), rr, nk * 8));
    uint64_t nb = 0, nu = 0, nr = 0;
    std::vector<double> ratios(nk);
    for (size_t i = 0; i < nk; ++i) {
        nb += hb[i];
        nu += hu[i];
        nr += hr[i];
        ratios[i] = hb[i] ? double(hr[i]) / hb[i] : 0;
    }
    if (nb != tot[0] || nu != tot[1] || nr != tot[2]) throw std::runtime_error("row/worker counter mismatch");
    std::sort(ratios.begin(), ratios.end());
    auto pct = [&](double f) {
        return ratios.empty() ? 0 : ratios[std::min(ratios.size() - 1, size_t(std::ceil(f * ratios.size())) - 1)];
    };
    const uint64_t obs = uint64_t(p.dim + 15) / 16, dp = uint64_t(p.in + 31) / 32 * 32;
    const uint64_t events = tot[3], steps = tot[4], padded = nr * obs * 16;
    std::cout << std::setprecision(12) << "ONLINE_STATS layer=" << l + 1 << " block=" << block << " heads=" << p.heads
              << " D=" << p.in << " d=" << p.dim << " blocks=" << nb << " max_updates_including_initial=" << nu
              << " rescales=" << nr << " rescale_per_block=" << (nb ? double(nr) / nb : 0) << " P50=" << pct(.5)
              << " P90=" << pct(.9) << " P95=" << pct(.95) << " P99=" << pct(.99)
              << " rescaled_feature_elements=" << nr * uint64_t(p.dim) << " expected_elements=" << nr * uint64_t(p.dim)
              << " rescaled_padded_feature_elements=" << padded << " rescale_events=" << events
              << " spill_bytes=" << events * obs * 1024 << " reload_bytes=" << events * obs * 1024
              << " row_scale_load_bytes=" << padded * 4 << " row_scale_store_bytes=" << padded * 4
              << " amx_calls=" << steps * (dp / 32) * obs << " neighbor_steps=" << steps
              << " executed_fma=" << steps * 16 * dp * obs * 16
              << " total_tiles=" << uint64_t(p.heads) * ((g.n + 15) / 16)
              << " cpu_schedule_counters=modelled_not_measured_on_gpu\n";
}


// --smoke: the online variants against B1 with the prescan maximum on the
// boundary graph (they differ only through the rescale roundings).
int smoke() {
    int cases = 0;
    for (int D : {17, 128})
        for (int K : {1, 8})
            for (int d : {7, 32}) {
                gat::Graph g = boundary_graph(D);
                gat::Model m(3);
                gat::Model full = gat::random_model(D, d, 11);
                m[0] = full[0];
                m[0].heads = K;
                m[0].dim = d;
                m[0].w.resize(size_t(D) * K * d);
                m[0].al.resize(size_t(K) * d);
                m[0].ar.resize(size_t(K) * d);
                for (size_t i = 0; i < m[0].w.size(); ++i) m[0].w[i] = std::cos(0.31f * float(i)) / std::sqrt(float(D));
                for (size_t i = 0; i < m[0].al.size(); ++i) {
                    m[0].al[i] = std::sin(0.23f * float(i)) / std::sqrt(float(d));
                    m[0].ar[i] = std::cos(0.19f * float(i)) / std::sqrt(float(d));
                }
                m[1] = m[0];
                m[2] = m[0];
                Runner run(g, m);
                const float* in = run.upload_input(g.x);
                run.run_layer({"B1_TFS_PREMAX", 0}, 0, in, false);
                const std::vector<float> b1 = run.output(0);
                for (int block : {16, 32, 64}) {
                    run.run_layer({"ICPP_TFS_ONLINE_B" + std::to_string(block), block}, 0, in, false);
                    const gat::Error e = difference(b1, run.output(0));
                    if (!e.finite || e.relative_l2 > 1e-4 || e.max_abs > 1e-4)
                        throw std::runtime_error("smoke: online block " + std::to_string(block) + " differs from B1");
                }
                ++cases;
            }
    std::cout << "SMOKE PASS cases=" << cases << " blocks=16,32,64 online_vs_B1_premax\n";
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        if (argc == 2 && std::string(argv[1]) == "--smoke") return smoke();
        if (argc != 7)
            throw std::runtime_error("usage: icpp_online GRAPH THREADS WARMUPS REPEATS BLOCKS_CSV PROFILE_PERIOD | --smoke");
        const int threads = std::stoi(argv[2]), warm = std::stoi(argv[3]), reps = std::stoi(argv[4]),
                  period = std::stoi(argv[6]);
        if (threads < 1 || warm < 0 || reps < 1 || period < 1) throw std::runtime_error("invalid config");
        std::vector<Path> paths = {{"B0_FP32", 0}, {"B0_BF16", 0}, {"B1_TFS_PREMAX", 0}};
        std::stringstream csv(argv[5]);
        std::string word;
        while (std::getline(csv, word, ',')) {
            const int block = std::stoi(word);
            if (block < 1 || block > 64) throw std::runtime_error("invalid block");
            paths.push_back({"ICPP_TFS_ONLINE_B" + std::to_string(block), block});
        }
        if (paths.size() == 3) throw std::runtime_error("no Online path");
        const gat::Graph g = gat::load_graph(argv[1]);
        const gat::Model model = gat::random_model(g.din, g.classes, 11);
        const gat::Schedule sched = gat::degree_schedule(g);
        Runner run(g, model);
        std::cout << std::setprecision(12) << "CONFIG N=" << g.n << " E=" << g.e << " Din=" << g.din << " C=" << g.classes
                  << " threads=" << threads << " seed=11 untrained=true warmups=" << warm << " repeats=" << reps
                  << " degree_sort_ms=" << sched.degree_sort_s * 1000
                  << " panel=64 tile_rows=16 LR_policy=fp32 online_max_prescan=false output_accumulator=FP32_registers"
                  << " output_rescale_dim=d task_accuracy=UNVERIFIED performance=EXPLORATORY device=sm_100a\n";
        // B0 FP32 reference chain
        std::array<std::vector<float>, 3> ref;
        {
            std::array<double, 3> ms{};
            run.chain(paths[0], ms);
            for (int l = 0; l < 3; ++l) ref[l] = run.output(l);
        }
        for (int l = 0; l < 3; ++l)
            std::cout << "STATIC layer=" << l + 1 << " prepare_ms=" << run.prepare_ms[l]
                      << " online_workspace_bytes=" << g.n * size_t(model[l].heads) * 16
                      << " global_Z_bytes=0 global_edge_score_bytes=0 global_alpha_bytes=0\n";
        // common-input controls, outside the three-layer timer
        for (int l = 0; l < 3; ++l) {
            const std::vector<float>& input = l ? ref[l - 1] : g.x;
            const float* in = run.upload_input(input);
            run.run_layer(paths[2], l, in, false);
            const std::vector<float> b1 = run.output(l);
            for (const auto& path : paths)
                if (path.block) {
                    run.run_layer(path, l, in, false);
                    const std::vector<float> got = run.output(l);
                    report(path.name, l + 1, "B1_PREMAX_same_input_same_LR", difference(b1, got));
                    if (path.block == paths.back().block) {
                        std::vector<float> L(size_t(g.n) * model[l].heads), R(L.size());
                        run.left.download(L);
                        run.right.download(R);
                        fp64_row_diagnostic(g, model[l], input, L, R, got, l + 1, path.name);
                    }
                }
        }
        // timed three-layer chains
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
                        report(path.name, l + 1, "B0_FP32_own_output_3layer", difference(ref[l], run.output(l)));
                if (rep >= 0) {
                    gat::require_finite(run.output(2), path.name);
                    for (int l = 0; l < 3; ++l)
                        std::cout << "{\"path\":\"" << path.name << "\",\"rep\":" << rep << ",\"layer\":" << l + 1
                                  << ",\"e2e_ms\":" << e2e << ",\"layer_ms\":" << ms[l]
                                  << ",\"projection_ms\":0,\"conversion_ms\":0,\"lr_ms\":0,\"max_prescan_ms\":0"
                                  << ",\"kernel_ms\":" << ms[l] << ",\"normalization_ms\":0,\"activation_ms\":0"
                                  << ",\"block\":" << path.block << "}\n";
                }
            }
        }
        // profile identity and the exact counters of every online block size
        for (const auto& path : paths)
            if (path.block) {
                std::array<double, 3> ms{};
                run.chain(path, ms);
                std::array<uint64_t, 3> hashes{};
                for (int l = 0; l < 3; ++l) hashes[l] = fingerprint(run.output(l));
                const float* in = run.upload_input(g.x);
                for (int l = 0; l < 3; ++l) {
                    const double t = run.run_layer(path, l, in, l < 2);
                    in = static_cast<const float*>(run.out[l].p);
                    const bool equal = hashes[l] == fingerprint(run.output(l));
                    std::cout << "PROFILE_IDENTITY layer=" << l + 1 << " block=" << path.block
                              << " bit_fingerprint_equal=" << equal << "\n";
                    if (!equal) throw std::runtime_error("profile output changed");
                    std::cout << std::setprecision(12) << "PROFILE path=ICPP_TFS_ONLINE_B" << path.block
                              << " layer=" << l + 1 << " layer_wall_ms=" << t << " kernel_wall_ms=" << t
                              << " sampled_tiles=0 worker_times=unavailable_on_gpu profile_period=" << period << "\n";
                    online_stats(run, l, path.block);
                }
            }
        std::cout << "ICPP_ONLINE_COMPLETE architecture=B200_TFS_online_running_max master_gate=SEE_PER_LAYER_ERRORS"
                     " task_accuracy=UNVERIFIED performance=EXPLORATORY\n";
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "ICPP_ONLINE_FAIL " << e.what() << "\n";
        return 1;
    }
}
