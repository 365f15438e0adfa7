// gat_b200_bench: the reference's benchmark driver (baseline/bench/main.cpp)
// on the B200 library, through the C ABI only (include/gat_b200.h).
//
// Same arguments (--key value) and the same log lines, so the reference's
// summarize scripts read its output unchanged:
//   ENV / STATIC / CONFIG / MODEL / COLD lines, one JSON line per layer and
//   repeat with the keys of print_times (baseline/src/common.cpp:155-170),
//   E2E per repeat, SUMMARY; in correctness mode ERROR lines
//   (common.cpp:151-154) and a CORRECTNESS verdict.
//
// Paths: ref_fp32 (served by the FP32 path, which the test suite pins to the
// reference's R0 at max-abs <= 1e-5), standard_fp32, standard_bf16, tfs_bf16,
// matched_attention, and adaptive_bf16 (layer 1 through TFS aggregation).
// Modes: benchmark (the three-layer forward, or one layer with --layer N),
// correctness (with --dump-prefix), and the operator modes micro,
// export-fixture and fixed-p on one layer (--layer, default 2). A forward is
// timed end to end on the host clock: FP32 X from host memory in, FP32 logits
// to host memory out, as the reference times its forward over host buffers.
// A single layer and the operator modes time each stage on device-resident
// buffers.
// --init-policy and --diagnostics are accepted: they place the reference's CPU
// threads and report its NUMA maps, which have no device counterpart.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <iomanip>
#include <iostream>
#include <map>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "gat_b200.hpp"

namespace gat = gat_b200;

namespace {

using gat::check;
using gat::Clock;
using gat::seconds;

struct Args {
    std::map<std::string, std::string> v;
    Args(int argc, char** argv) {
        const std::vector<std::string> allowed = {
            "--graph",  "--weights",   "--seed",    "--save-weights", "--path",        "--mode",
            "--threads", "--panel-r",  "--repeats", "--warmups",      "--layer",       "--lr-policy",
            "--fixture", "--max-abs",  "--rel-l2",  "--dump-prefix",  "--output",      "--init-policy",
            "--diagnostics"};
        // bench/main.cpp:9-14: pairs first (duplicates rejected), then the names
        for (int i = 1; i < argc; ++i) {
            std::string k = argv[i];
            if (k.rfind("--", 0) != 0 || i + 1 == argc) throw std::runtime_error("arguments must be --key value");
            if (!v.emplace(k, argv[++i]).second) throw std::runtime_error("duplicate argument: " + k);
        }
        for (const auto& kv : v)
            if (std::find(allowed.begin(), allowed.end(), kv.first) == allowed.end())
                throw std::runtime_error("unknown option: " + kv.first);
    }
    std::string get(const std::string& k, const std::string& def = "") const {
        auto i = v.find(k);
        return i == v.end() ? def : i->second;
    }
    int num(const std::string& k, int def) const { return std::stoi(get(k, std::to_string(def))); }
};

double pct(std::vector<double> x, double q) {
    std::sort(x.begin(), x.end());
    return x[std::min(x.size() - 1, size_t(std::ceil(q * x.size()) - 1))];
}

int path_code(const std::string& p) {
    if (p == "ref_fp32" || p == "standard_fp32") return GAT_B200_PATH_STANDARD_FP32;
    if (p == "standard_bf16") return GAT_B200_PATH_STANDARD_BF16;
    if (p == "tfs_bf16") return GAT_B200_PATH_TFS_BF16;
    if (p == "matched_attention") return GAT_B200_PATH_MATCHED_ATTENTION;
    if (p == "adaptive_bf16") return GAT_B200_PATH_ADAPTIVE_BF16;
    throw std::runtime_error("bad path");
}

// Stage times (ms) and counts of one layer, the fields of the reference's
// Times (baseline/include/gat.hpp:68-76).
struct StageMs {
    double convert = 0, projection = 0, lr = 0, max_prescan = 0, aggregate = 0, normalize = 0, activation = 0,
           total = 0;
    uint64_t neighbor_steps = 0, executed_fma = 0, workspace_bytes = 0;
};

// One JSON line per layer and repeat with print_times' keys, in its order
// (baseline/src/common.cpp:155-170; the CPU worker sums of its profile build
// print as 0); `extra` appends keys of this backend.
void print_times(const std::string& path, const std::string& mode, int layer, int rep, const gat::Graph& g,
                 const gat::Param& p, int threads, bool fp32, const StageMs& t, double static_ms, int panel,
                 const std::string& extra = "") {
    const uint64_t useful = g.e * uint64_t(p.heads) * uint64_t(p.in) * uint64_t(p.dim);
    std::cout << std::setprecision(10) << "{\"path\":\"" << path << "\",\"mode\":\"" << mode
              << "\",\"layer\":" << layer << ",\"rep\":" << rep << ",\"N\":" << g.n << ",\"E\":" << g.e
              << ",\"D\":" << p.in << ",\"K\":" << p.heads << ",\"d\":" << p.dim << ",\"threads\":" << threads
              << ",\"profile\":false,\"precision\":\"" << (fp32 ? "FP32" : "BF16_RNE_FP32_state") << "\""
              << ",\"projection_ms\":" << t.projection << ",\"lr_ms\":" << t.lr
              << ",\"max_prescan_ms\":" << t.max_prescan << ",\"score_exp_aggregate_ms\":" << t.aggregate
              << ",\"normalize_ms\":" << t.normalize << ",\"activation_ms\":" << t.activation
              << ",\"convert_ms\":" << t.convert << ",\"total_ms\":" << t.total
              << ",\"workspace_bytes\":" << t.workspace_bytes << ",\"static_preprocess_ms\":" << static_ms
              << ",\"panel_R\":" << panel << ",\"tile_rows\":16";
    for (const char* k : {"score_exp_worker_ms", "gather_weight_convert_worker_ms", "tile_load_worker_ms",
                          "gather_load_worker_ms", "p_times_x_convert_worker_ms", "weighted_spmm_worker_ms",
                          "amx_compute_worker_ms", "tile_store_worker_ms", "tile_config_worker_ms",
                          "scheduling_worker_ms", "output_write_worker_ms"})
        std::cout << ",\"" << k << "\":0";
    std::cout << ",\"neighbor_steps\":" << t.neighbor_steps << ",\"executed_fma\":" << t.executed_fma
              << ",\"padding_executed_flops\":" << (t.executed_fma ? 2 * (t.executed_fma - useful) : 0) << extra
              << "}\n";
}

void dump(const std::string& path, const std::vector<float>& v) {
    std::ofstream f(path, std::ios::binary);
    f.write(reinterpret_cast<const char*>(v.data()), std::streamsize(v.size() * 4));
    if (!f) throw std::runtime_error("cannot write dump");
}

// Device objects of one (graph, checkpoint): the graph with its degree
// schedule, the three prepared layers, and one model per path.
struct Device {
    gat_b200_graph* g = nullptr;
    gat_b200_layer* layer[3] = {nullptr, nullptr, nullptr};
    std::map<int, gat_b200_model*> models;
    ~Device() {
        for (auto& kv : models) gat_b200_model_destroy(kv.second);
        for (auto* p : layer) gat_b200_layer_destroy(p);
        gat_b200_graph_destroy(g);
    }
    gat_b200_model* model(int path) {
        auto it = models.find(path);
        if (it != models.end()) return it->second;
        gat_b200_model* m = nullptr;
        const gat_b200_layer* const ls[3] = {layer[0], layer[1], layer[2]};
        check(gat_b200_model_create(g, ls, path, &m));
        models[path] = m;
        return m;
    }
};

std::vector<float> forward(gat_b200_model* m, const gat::Graph& g, const gat::Model& model) {
    std::vector<float> logits(g.n * size_t(model[2].width()));
    check(gat_b200_model_forward(m, g.x.data(), 1, logits.data(), 1, nullptr));
    return logits;
}

// Timing of one operation on the device: host clock around the call and a
// synchronization (so that a kernel's time lands in its own stage).
template <class F>
double timed_ms(F&& f) {
    const auto t0 = Clock::now();
    f();
    check(gat_b200_check_device());
    return seconds(t0, Clock::now()) * 1000;
}

// The input of layer `layer` (1-based): the R0 chain of the layers before it
// (bench/main.cpp:105-106,168).
std::vector<float> r0_input(const gat::Graph& g, const gat::Model& model, int layer) {
    std::vector<float> input = g.x;
    for (int l = 0; l < layer - 1; ++l) {
        gat::Workspace rw;
        rw.allocate(g, model[l], "standard_fp32");
        gat::Times t;
        gat::ref_layer(g, model[l], input, rw, true, t);
        input = std::move(rw.out);
    }
    return input;
}

// One layer of `pc` (0-based l) from FP32 device rows xf [n][in] into out
// (FP32 [n][width]), each stage timed alone (host clock and a device
// synchronisation): the single-layer benchmark of bench/main.cpp:166-180.
struct LayerBuffers {
    gat::detail::DeviceBuffer xb, h, left, right, max, den, out;
};
StageMs run_single_layer(Device& dev, const gat::Model& model, int pc, int l, const float* xf, uint64_t n,
                         LayerBuffers& b) {
    const gat::Param& p = model[l];
    const gat_b200_layer* lp = dev.layer[l];
    const int K = p.heads, d = p.dim, W = p.width(), D = p.in;
    const bool hidden = l < 2;
    const int ldb = gat_b200_padded_ld(D, GAT_B200_BF16);
    uint16_t* xb = static_cast<uint16_t*>(b.xb.get(n * size_t(ldb) * 2));
    float* L = static_cast<float*>(b.left.get(n * K * 4));
    float* R = static_cast<float*>(b.right.get(n * K * 4));
    float* out = static_cast<float*>(b.out.get(n * size_t(W) * 4));
    StageMs t;
    const bool tfs = pc == GAT_B200_PATH_TFS_BF16 || (pc == GAT_B200_PATH_ADAPTIVE_BF16 && l == 0);
    if (tfs) {
        // baseline_tfs.cpp:111-117: convert + lr_reordered ("bf16"), max_prescan,
        // TFS aggregation (B1 rounding; the adaptive path's layer 1 rounds as
        // heads_hybrid with one block per row), finish
        float* M = static_cast<float*>(b.max.get(n * K * 4));
        float* dn = static_cast<float*>(b.den.get(n * K * 4));
        t.lr = timed_ms([&] {
            check(gat_b200_lr_reordered(lp, n, xf, GAT_B200_F32, D, GAT_B200_LR_BF16, xb, ldb, L, R, nullptr));
        });
        t.max_prescan = timed_ms([&] { check(gat_b200_max_prescan(dev.g, K, L, R, M, nullptr)); });
        const int rounding = pc == GAT_B200_PATH_TFS_BF16 ? GAT_B200_TFS_EDGE : GAT_B200_TFS_SPLIT;
        t.aggregate = timed_ms([&] {
            check(gat_b200_tfs_aggregate(dev.g, lp, xb, ldb, L, R, M, nullptr, nullptr, rounding, 0, 1, out, W, dn,
                                         nullptr, nullptr));
        });
        t.normalize = timed_ms([&] { check(gat_b200_finish(n, K, d, dn, hidden, out, W, nullptr)); });
    } else {
        // baseline_standard.cpp:98-108: convert, projection with L/R (or
        // lr_reordered "bf16" on the matched path), the aggregation with max,
        // normalisation and ELU fused
        const bool fp32 = pc == GAT_B200_PATH_STANDARD_FP32;
        const int hd = fp32 ? GAT_B200_F32 : GAT_B200_BF16, ldh = gat_b200_padded_ld(W, hd);
        void* h = b.h.get(n * size_t(ldh) * (fp32 ? 4 : 2));
        const void* x = xf;
        int ldx = D;
        if (!fp32) {
            t.convert = timed_ms([&] { check(gat_b200_convert(n, D, xf, D, xb, ldb, nullptr)); });
            x = xb;
            ldx = ldb;
        }
        t.projection = timed_ms([&] { check(gat_b200_projection(lp, n, x, ldx, hd, h, hd, ldh, L, R, nullptr)); });
        if (pc == GAT_B200_PATH_MATCHED_ATTENTION)
            t.lr = timed_ms([&] {
                check(gat_b200_lr_reordered(lp, n, xb, GAT_B200_BF16, ldb, GAT_B200_LR_BF16, nullptr, 0, L, R,
                                            nullptr));
            });
        t.aggregate = timed_ms([&] {
            check(gat_b200_aggregate_fused(dev.g, K, d, h, hd, ldh, L, R, hidden, out, GAT_B200_F32, W, nullptr));
        });
    }
    t.total = t.convert + t.projection + t.lr + t.max_prescan + t.aggregate + t.normalize;
    return t;
}

// The operator modes of the reference's driver on one layer (bench/main.cpp:103-151):
//   micro           each stage of the layer timed alone (MICRO lines)
//   export-fixture  R0's weights p and den of the layer, written as GATFIX1
//   fixed-p         the standard (BF16 projection + aggregation with the
//                   fixture's p, den + finish) and TFS B1 (aggregate-first with
//                   the same p, den + finish) operators, alternated AB/BA, with
//                   the reference's error controls and FIXED_P summary
// The layer's input is the R0 chain of the earlier layers; the operators run
// on device-resident buffers (input conversion shared and untimed, as the
// reference excludes it).
int operator_modes(const Args& a, const std::string& mode, const gat::Graph& g, const gat::Model& model,
                   Device& dev, int layer_arg, int threads, int panel, int reps, int warmups, double static_ms,
                   uint64_t neighbor_steps) {
    const int layer = layer_arg ? layer_arg : 2;
    const gat::Param& p = model[layer - 1];
    const gat_b200_layer* lp = dev.layer[layer - 1];
    std::vector<float> input = r0_input(g, model, layer);
    const uint64_t n = g.n, e = g.e;
    const int K = p.heads, d = p.dim, W = p.width(), D = p.in;
    const int ldb = gat_b200_padded_ld(D, GAT_B200_BF16), ldz = gat_b200_padded_ld(W, GAT_B200_F32);
    gat::detail::DeviceBuffer bx, bxb, bz, bl, br, bm, bo, bd, bo2, bd2, bp, bpd;
    float* L = static_cast<float*>(bl.get(n * K * 4));
    float* R = static_cast<float*>(br.get(n * K * 4));
    float* z = static_cast<float*>(bz.get(n * size_t(ldz) * 4));
    float* out = static_cast<float*>(bo.get(n * size_t(W) * 4));
    float* den = static_cast<float*>(bd.get(n * K * 4));
    uint16_t* xb = static_cast<uint16_t*>(bxb.get(n * size_t(ldb) * 2));

    if (mode == "micro") {
        // bench/main.cpp:107-118
        const float* xf = bx.upload(input);
        float* mx = static_cast<float*>(bm.get(n * K * 4));
        auto bench = [&](const std::string& name, const std::function<void()>& fn) {
            std::vector<double> samples;
            for (int r = -warmups; r < reps; ++r) {
                const double ms = timed_ms(fn);
                if (r >= 0) samples.push_back(ms);
            }
            std::cout << "MICRO name=" << name << " layer=" << layer << " median_ms=" << pct(samples, .5)
                      << " p95_ms=" << pct(samples, .95) << "\n";
        };
        bench("convert_rne", [&] { check(gat_b200_convert(n, D, xf, D, xb, ldb, nullptr)); });
        bench("projection_bf16", [&] {
            check(gat_b200_projection(lp, n, xb, ldb, GAT_B200_BF16, z, GAT_B200_F32, ldz, L, R, nullptr));
        });
        // L and R from Z are computed in the projection's epilogue on this backend
        std::cout << "MICRO name=lr_z_avx layer=" << layer << " fused_into=projection_bf16\n";
        std::cout << "MICRO name=lr_z_sgemm_static_workspace layer=" << layer << " fused_into=projection_bf16\n";
        bench("lr_reordered_bf16", [&] {
            check(gat_b200_lr_reordered(lp, n, xb, GAT_B200_BF16, ldb, GAT_B200_LR_BF16, nullptr, 0, L, R, nullptr));
        });
        bench("lr_reordered_fp32", [&] {
            check(gat_b200_lr_reordered(lp, n, xf, GAT_B200_F32, D, GAT_B200_LR_FP32, nullptr, 0, L, R, nullptr));
        });
        // "avx" is the same FP32 product as "fp32" here
        std::cout << "MICRO name=lr_reordered_avx layer=" << layer << " same_as=lr_reordered_fp32\n";
        check(gat_b200_projection(lp, n, xb, ldb, GAT_B200_BF16, z, GAT_B200_F32, ldz, L, R, nullptr));
        bench("max_prescan", [&] { check(gat_b200_max_prescan(dev.g, K, L, R, mx, nullptr)); });
        bench("weighted_spmm_score_exp", [&] {
            check(gat_b200_standard_aggregate(dev.g, K, d, z, GAT_B200_F32, ldz, L, R, nullptr, nullptr, out, W, den,
                                              mx, nullptr));
        });
        return 0;
    }

    gat::Fixture fixture;
    if (mode == "export-fixture" || a.get("--fixture").empty()) {
        // R0's p and den (ref_fp32.cpp:3-14): FP32 projection, edge softmax
        const float* xf = bx.upload(input);
        check(gat_b200_projection(lp, n, xf, D, GAT_B200_F32, z, GAT_B200_F32, ldz, L, R, nullptr));
        float* pp = static_cast<float*>(bp.get(e * K * 4));
        check(gat_b200_edge_softmax(dev.g, K, L, R, nullptr, nullptr, pp, den, nullptr, nullptr));
        fixture.input = input;
        fixture.p.resize(e * K);
        fixture.den.resize(n * K);
        check(gat_b200_copy_to_host(fixture.p.data(), pp, e * K * 4));
        check(gat_b200_copy_to_host(fixture.den.data(), den, n * K * 4));
    } else {
        fixture = gat::load_fixture(g, p, a.get("--fixture"));
    }
    if (mode == "export-fixture") {
        gat::save_fixture(g, p, fixture, a.get("--fixture"));
        std::cout << "FIXTURE saved layer=" << layer << "\n";
        return 0;
    }

    // fixed-p: both operators on the identical fixture, input converted once
    input = std::move(fixture.input);
    const float* xf = bx.upload(input);
    check(gat_b200_convert(n, D, xf, D, xb, ldb, nullptr));
    const float* fp = bp.upload(fixture.p);
    const float* fd = bpd.upload(fixture.den);
    float* out2 = static_cast<float*>(bo2.get(n * size_t(W) * 4));
    float* den2 = static_cast<float*>(bd2.get(n * K * 4));
    auto standard_op = [&](StageMs& t) {
        t.projection = timed_ms([&] {
            check(gat_b200_projection(lp, n, xb, ldb, GAT_B200_BF16, z, GAT_B200_F32, ldz, L, R, nullptr));
        });
        t.aggregate = timed_ms([&] {
            check(gat_b200_standard_aggregate(dev.g, K, d, z, GAT_B200_F32, ldz, nullptr, nullptr, fp, fd, out, W,
                                              den, nullptr, nullptr));
        });
        t.normalize = timed_ms([&] { check(gat_b200_finish(n, K, d, den, 0, out, W, nullptr)); });
        t.total = t.projection + t.aggregate + t.normalize;
        t.workspace_bytes = n * (uint64_t(ldz) * 4 + uint64_t(W) * 4 + uint64_t(K) * 12 + uint64_t(ldb) * 2);
    };
    auto tfs_op = [&](StageMs& t) {
        t.aggregate = timed_ms([&] {
            check(gat_b200_tfs_aggregate(dev.g, lp, xb, ldb, nullptr, nullptr, nullptr, fp, fd, GAT_B200_TFS_EDGE, 0,
                                         1, out2, W, den2, nullptr, nullptr));
        });
        t.normalize = timed_ms([&] { check(gat_b200_finish(n, K, d, den2, 0, out2, W, nullptr)); });
        t.total = t.aggregate + t.normalize;
        t.workspace_bytes = n * (uint64_t(W) * 4 + uint64_t(K) * 4 + uint64_t(ldb) * 2);
    };
    auto host = [&](const float* dptr, size_t count) {
        std::vector<float> v(count);
        check(gat_b200_copy_to_host(v.data(), dptr, count * 4));
        return v;
    };
    StageMs st, tt;
    standard_op(st);
    tfs_op(tt);
    const std::vector<float> sw = host(out, n * W), tw = host(out2, n * W);
    gat::require_finite(sw, "fixed-p standard");
    gat::require_finite(tw, "fixed-p TFS");
    gat::print_error("tfs_fixed_p", layer, "vs_standard_bf16_extra_pX_quantization_and_reduction",
                     gat::errors(sw, tw));
    // the FP32 fixed-p operator (FP32 projection) as the master: separates the
    // cost of the pX rounding from that of BF16 X and W
    check(gat_b200_projection(lp, n, xf, D, GAT_B200_F32, z, GAT_B200_F32, ldz, L, R, nullptr));
    check(gat_b200_standard_aggregate(dev.g, K, d, z, GAT_B200_F32, ldz, nullptr, nullptr, fp, fd, out, W, den,
                                      nullptr, nullptr));
    check(gat_b200_finish(n, K, d, den, 0, out, W, nullptr));
    const std::vector<float> master = host(out, n * W);
    gat::print_error("standard_fixed_p", layer, "vs_master_fixed_p", gat::errors(master, sw));
    gat::print_error("tfs_fixed_p", layer, "vs_master_fixed_p", gat::errors(master, tw));
    // scalar emulation of the TFS edge projection: BF16(p x) times BF16 W in
    // neighbour order (bench/main.cpp:132-137), for small layers
    if (double(e) * K * D * d <= 2e7) {
        std::vector<float> emulated(n * size_t(W), 0.f);
        const std::vector<float> xq = gat::quantized(input), wq = gat::quantized(p.w);
        for (uint64_t i = 0; i < n; ++i)
            for (int h = 0; h < K; ++h) {
                float* o = emulated.data() + i * W + h * d;
                for (uint64_t ed = g.row[i]; ed < g.row[i + 1]; ++ed)
                    for (int k = 0; k < D; ++k) {
                        const float v = gat::expand(gat::rne(fixture.p[ed * K + h] * xq[size_t(g.col[ed]) * D + k]));
                        for (int c = 0; c < d; ++c) o[c] += v * wq[size_t(k) * W + h * d + c];
                    }
                const float dn = fixture.den[i * K + h];
                for (int c = 0; c < d; ++c) o[c] = dn > 0 ? o[c] / dn : 0.f;
            }
        gat::print_error("tfs_fixed_p", layer, "vs_pX_bf16_emulation_reduction_only", gat::errors(emulated, tw));
    } else {
        std::cout << "CONTROL pX_scalar_emulation=SKIPPED_TOO_LARGE validated_in_boundary_tests=true\n";
    }
    std::vector<double> ss, ts;
    const int dp = (D + 31) / 32 * 32, obs = (d + 15) / 16;
    for (int r = -warmups; r < reps; ++r) {
        StageMs s1, t1;
        if (r % 2 == 0) {
            standard_op(s1);
            tfs_op(t1);
        } else {
            tfs_op(t1);
            standard_op(s1);
        }
        if (r < 0) continue;
        ss.push_back(s1.total);
        ts.push_back(t1.total);
        t1.neighbor_steps = neighbor_steps * uint64_t(K);
        t1.executed_fma = t1.neighbor_steps * 16 * uint64_t(dp) * uint64_t(obs) * 16;
        print_times("standard_bf16", "fixed-p", layer, r, g, p, threads, false, s1, static_ms, panel);
        print_times("tfs_bf16", "fixed-p", layer, r, g, p, threads, false, t1, static_ms, panel);
    }
    std::cout << "FIXED_P median_standard_ms=" << pct(ss, .5) << " median_tfs_ms=" << pct(ts, .5)
              << " speedup=" << pct(ss, .5) / pct(ts, .5)
              << " conversion_excluded=true input_preparation=shared policy=AB_BA\n";
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        Args a(argc, argv);
        const std::string graph_path = a.get("--graph"), path = a.get("--path", "standard_bf16"),
                          mode = a.get("--mode", "correctness");
        if (graph_path.empty()) throw std::runtime_error("--graph is required");
        const int pc = path_code(path);
        const int threads = a.num("--threads", 16), panel = a.num("--panel-r", 64), reps = a.num("--repeats", 5),
                  warmups = a.num("--warmups", 2), layer_arg = a.num("--layer", 0);
        if (threads <= 0 || panel < 16 || panel % 16 || reps < 1 || warmups < 0 || layer_arg < 0 || layer_arg > 3)
            throw std::runtime_error("invalid benchmark controls");
        const bool operator_mode = mode == "export-fixture" || mode == "fixed-p" || mode == "micro";
        if (mode != "correctness" && mode != "benchmark" && mode != "profile" && !operator_mode)
            throw std::runtime_error("bad mode");
        // the profile mode needs the reference's counter build (GAT_PROFILE); this
        // backend's stage times come from CUDA events in every benchmark run
        if (mode == "profile") throw std::runtime_error("profile requires profile binary");
        if (mode == "export-fixture" && a.get("--fixture").empty())
            throw std::runtime_error("--fixture output is required");
        const std::string init = a.get("--init-policy", "original");
        if (init != "original" && init != "warm") throw std::runtime_error("bad init policy");
        const std::string policy =
            a.get("--lr-policy", path == "tfs_bf16" || path == "matched_attention" ? "bf16" : "z_avx");
        // bench/main.cpp:61-63 (checked here before any device work)
        if (policy != "bf16" && policy != "fp32" && policy != "avx" && policy != "z_avx" && policy != "z_mkl")
            throw std::runtime_error("bad LR policy");
        const bool reordered = path == "tfs_bf16" || path == "matched_attention";
        if (reordered && (policy == "z_avx" || policy == "z_mkl"))
            throw std::runtime_error("reordered LR path requires bf16/fp32/avx");
        // The device model takes the reordered L/R of these paths from the BF16
        // layer input ("bf16"); the standard paths take L/R from Z in the
        // projection epilogue, which serves every policy there (the reference
        // runs any policy but z_mkl as z_avx on them, bench/main.cpp:24).
        if (reordered && policy != "bf16")
            throw std::runtime_error("LR policy " + policy + " is not available for path " + path +
                                     " on this backend (bf16 only)");
        std::cout << "ENV backend=gat_b200 version=" << gat_b200_version() << " threads=" << threads
                  << " source_input=" << graph_path << " checkpoint="
                  << (a.get("--weights").empty() ? "random_fixture_not_trained" : a.get("--weights"))
                  << " profile=0 device=sm_100a\n";
        const auto cold_start = Clock::now();
        const gat::Graph g = gat::load_graph(graph_path);
        gat::Model model;
        if (!a.get("--weights").empty()) {
            model = gat::load_model(a.get("--weights"), g.din, g.classes);
        } else {
            if (a.get("--seed").empty())
                throw std::runtime_error("provide --weights checkpoint.bin or explicit --seed for synthetic fixture");
            model = gat::random_model(g.din, g.classes, a.num("--seed", 11));
        }
        if (!a.get("--save-weights").empty()) gat::save_model(model, a.get("--save-weights"));

        Device dev;
        auto t0 = Clock::now();
        check(gat_b200_graph_create(g.n, g.e, g.row.data(), g.col.data(), nullptr, &dev.g));
        check(gat_b200_check_device());
        const double degree_sort_s = seconds(t0, Clock::now());
        t0 = Clock::now();
        for (int l = 0; l < 3; ++l)
            check(gat_b200_layer_create(model[l].in, model[l].heads, model[l].dim, model[l].w.data(),
                                        model[l].al.data(), model[l].ar.data(), &dev.layer[l]));
        const double prepare_s = seconds(t0, Clock::now());
        uint64_t neighbor_steps = 0;
        check(gat_b200_graph_schedule(dev.g, nullptr, &neighbor_steps));
        std::cout << "STATIC degree_sort_ms=" << degree_sort_s * 1000 << " model_prepare_ms=" << prepare_s * 1000
                  << " bytes=" << g.n * 4 << " graph_policy=as_loaded_no_mutation\n";
        std::cout << "CONFIG mode=" << mode << " path=" << path << " lr_policy=" << policy << " panel_R=" << panel
                  << " layer=" << layer_arg << " warmups=" << warmups << " repeats=" << reps << "\n";

        if (mode == "correctness") {
            const bool have_abs = !a.get("--max-abs").empty(), have_rel = !a.get("--rel-l2").empty();
            if (have_abs != have_rel) throw std::runtime_error("set both --max-abs and --rel-l2");
            const double maxabs = have_abs ? std::stod(a.get("--max-abs")) : 0,
                         rel = have_rel ? std::stod(a.get("--rel-l2")) : 0;
            if (have_abs && (!std::isfinite(maxabs) || !std::isfinite(rel) || maxabs < 0 || rel < 0))
                throw std::runtime_error("invalid accuracy thresholds");
            bool pass = true, finite = true;
            auto check_e = [&](const std::string& name, int layer, const std::string& stage,
                               const std::vector<float>& r, const std::vector<float>& v, bool gate) {
                const gat::Error e = gat::errors(r, v);
                gat::print_error(name, layer, stage, e);
                pass &= e.finite;
                finite &= e.finite;
                if (gate && have_abs) pass &= e.max_abs <= maxabs && e.relative_l2 <= rel;
            };
            // Per layer, on R0's input (bench/main.cpp:70-92): R0 with its trace,
            // R0 on BF16-quantized X and W, every path's stages through the C++
            // mirror of the reference API, and the FP32 attention-reorder control.
            // --dump-prefix writes R0's per-layer trace and every path's logits as
            // raw FP32 files with the reference's names (bench/main.cpp:72-75,94-96).
            const std::string prefix = a.get("--dump-prefix");
            const gat::Schedule sched = gat::degree_schedule(g);
            std::vector<float> master = g.x;
            for (int l = 0; l < 3; ++l) {
                const gat::Param& p = model[l];
                const bool hidden = l < 2;
                const gat::Prepared q = gat::prepare(p);
                gat::Workspace rw;
                rw.allocate(g, p, "ref_fp32");
                gat::Times rt;
                gat::ref_layer(g, p, master, rw, hidden, rt);
                gat::require_finite(rw.out, "output");
                if (!prefix.empty()) {
                    const std::string pre = prefix + "_layer" + std::to_string(l + 1) + "_";
                    const std::pair<const char*, const std::vector<float>*> items[] = {
                        {"output", &rw.out}, {"z", &rw.z},     {"left", &rw.left}, {"right", &rw.right},
                        {"max", &rw.max},    {"den", &rw.den}, {"score", &rw.score}, {"p", &rw.p},
                        {"alpha", &rw.alpha}};
                    for (const auto& item : items) dump(pre + item.first + ".f32", *item.second);
                }
                gat::Param qp = p;
                qp.w = gat::quantized(p.w);
                gat::Workspace qr;
                qr.allocate(g, p, "ref_fp32");
                gat::Times qt;
                gat::ref_layer(g, qp, gat::quantized(master), qr, hidden, qt);
                check_e("quantized_XW_fp32_accum", l + 1, "Z", rw.z, qr.z, false);
                check_e("quantized_XW_fp32_accum", l + 1, "layer", rw.out, qr.out, false);
                for (const std::string test : {"standard_fp32", "standard_bf16", "tfs_bf16", "matched_attention"}) {
                    gat::Workspace w;
                    w.allocate(g, p, test);
                    gat::Times t;
                    if (test == "tfs_bf16") {
                        gat::tfs_layer(g, p, q, sched, master, w, hidden, panel, t, "bf16");
                    } else {
                        const auto t0 = Clock::now();
                        gat::projection(g, p, q, master, w, test != "standard_fp32");
                        t.projection = seconds(t0, Clock::now());
                        const auto t1 = Clock::now();
                        if (test == "matched_attention")
                            gat::lr_reordered(g, p, q, master, w, "bf16");
                        else
                            gat::lr_from_z(g, p, w);
                        t.lr = seconds(t1, Clock::now());
                        const auto t2 = Clock::now();
                        gat::max_prescan(g, p, w);
                        t.max_prescan = seconds(t2, Clock::now());
                        gat::standard_aggregate(g, p, w, nullptr, nullptr, &t);
                        gat::finish(g, p, w, hidden, t);
                        t.total = t.projection + t.lr + t.max_prescan + t.aggregate + t.normalize;
                    }
                    if (!w.z.empty()) {
                        check_e(test, l + 1, "Z", rw.z, w.z, false);
                        check_e(test, l + 1, "Z_accum_vs_quantized_fp32", qr.z, w.z, false);
                    }
                    check_e(test, l + 1, "L", rw.left, w.left, false);
                    check_e(test, l + 1, "R", rw.right, w.right, false);
                    check_e(test, l + 1, "row_max", rw.max, w.max, false);
                    check_e(test, l + 1, "denominator", rw.den, w.den, false);
                    check_e(test, l + 1, "layer", rw.out, w.out, true);
                    StageMs ms;
                    ms.projection = t.projection * 1000;
                    ms.lr = t.lr * 1000;
                    ms.max_prescan = t.max_prescan * 1000;
                    ms.aggregate = t.aggregate * 1000;
                    ms.normalize = t.normalize * 1000;
                    ms.total = t.total * 1000;
                    ms.workspace_bytes = w.bytes();
                    print_times(test, "correctness", l + 1, 0, g, p, threads, test == "standard_fp32", ms,
                                (degree_sort_s + prepare_s) * 1000, panel);
                }
                // FP32 contraction control: the attention reorder alone, without BF16
                gat::Workspace control;
                control.allocate(g, p, "tfs_bf16");
                gat::lr_reordered(g, p, q, master, control, "fp32");
                check_e("attention_reorder_fp32", l + 1, "L", rw.left, control.left, false);
                check_e("attention_reorder_fp32", l + 1, "R", rw.right, control.right, false);
                master = std::move(rw.out);
            }
            if (!prefix.empty()) dump(prefix + "_model_ref_fp32.f32", master);
            // every path's own three-layer chain against the R0 chain (bench/main.cpp:89-94)
            for (const std::string test : {"standard_fp32", "standard_bf16", "tfs_bf16", "matched_attention",
                                           "adaptive_bf16"}) {
                const std::vector<float> out = forward(dev.model(path_code(test)), g, model);
                if (!prefix.empty()) dump(prefix + "_model_" + test + ".f32", out);
                check_e(test, 3, "model_path_specific_chain", master, out, true);
            }
            std::cout << "CORRECTNESS finite=" << finite << " accuracy_gate="
                      << (have_abs ? (pass ? "PASS" : "FAIL") : "UNCONFIGURED_NOT_ACCEPTED")
                      << " task_metric=UNAVAILABLE\n";
            return pass ? 0 : 1;
        }
        if (operator_mode)
            return operator_modes(a, mode, g, model, dev, layer_arg, threads, panel, reps, warmups,
                                  (degree_sort_s + prepare_s) * 1000, neighbor_steps);

        if (layer_arg != 0) {
            // one layer on the R0 chain's input (bench/main.cpp:166-180), the
            // input resident on the device before the timer starts
            const int l = layer_arg - 1;
            const std::vector<float> input = r0_input(g, model, layer_arg);
            gat::detail::DeviceBuffer bx;
            const float* xf = bx.upload(input);
            LayerBuffers buf;
            std::cout << "MODEL workspace_bytes=" << g.n * size_t(model[l].in) * 4 << " static_bytes=" << g.n * 4
                      << " excludes_graph_and_master_weights=true\n";
            std::cout << "COLD startup_before_inference_ms=" << seconds(cold_start, Clock::now()) * 1000
                      << " includes_graph_load=true\n";
            std::vector<double> totals;
            double cold_forward = 0;
            const bool fp32 = pc == GAT_B200_PATH_STANDARD_FP32;
            for (int r = -warmups; r < reps; ++r) {
                StageMs t = run_single_layer(dev, model, pc, l, xf, g.n, buf);
                if (r == -warmups) cold_forward = t.total;
                if (r < 0) continue;
                totals.push_back(t.total);
                const bool tfs = pc == GAT_B200_PATH_TFS_BF16 || (pc == GAT_B200_PATH_ADAPTIVE_BF16 && l == 0);
                t.neighbor_steps = tfs ? neighbor_steps * model[l].heads : 0;
                print_times(path, mode, layer_arg, r, g, model[l], threads, fp32, t, (degree_sort_s + prepare_s) * 1000,
                            panel);
                std::cout << "E2E path=" << path << " rep=" << r << " layer=" << layer_arg << " total_ms=" << t.total
                          << " finite=1\n";
            }
            std::vector<float> o(g.n * size_t(model[l].width()));
            buf.out.download(o);
            gat::require_finite(o, "benchmark output");
            if (!a.get("--output").empty()) dump(a.get("--output"), o);
            std::cout << "SUMMARY path=" << path << " median_ms=" << pct(totals, .5) << " p95_ms=" << pct(totals, .95)
                      << " cold_forward_ms=" << cold_forward << " repeats=" << reps << " task_accuracy=UNVERIFIED\n";
            return 0;
        }
        gat_b200_model* m = dev.model(pc);
        check(gat_b200_model_enable_timing(m, 1));
        std::cout << "MODEL workspace_bytes=" << g.n * size_t(g.din) * 4 << " static_bytes=" << g.n * 4
                  << " excludes_graph_and_master_weights=true\n";
        std::cout << "COLD startup_before_inference_ms=" << seconds(cold_start, Clock::now()) * 1000
                  << " includes_graph_load=true\n";
        std::vector<double> totals;
        double cold_forward = 0;
        std::vector<float> logits;
        const bool tfs_layer1 = pc == GAT_B200_PATH_TFS_BF16 || pc == GAT_B200_PATH_ADAPTIVE_BF16;
        const bool fp32 = pc == GAT_B200_PATH_STANDARD_FP32;
        for (int r = -warmups; r < reps; ++r) {
            const auto begin = Clock::now();
            logits = forward(m, g, model);
            const double total = seconds(begin, Clock::now());
            if (r == -warmups) cold_forward = total;
            gat::require_finite(logits, "benchmark output");
            if (r < 0) continue;
            totals.push_back(total);
            float st[9];
            if (gat_b200_model_stage_times(m, st) < 1) throw std::runtime_error(gat_b200_last_error());
            for (int l = 0; l < 3; ++l) {
                const gat::Param& p = model[l];
                // stage slots: 1 convert, 2+2l projection (TFS: lr_reordered + max prescan), 3+2l aggregation
                const bool tfs = pc == GAT_B200_PATH_TFS_BF16 || (tfs_layer1 && l == 0);
                const double pre = st[2 + 2 * l], agg = st[3 + 2 * l], conv = l == 0 ? st[1] : 0.0;
                StageMs t;
                (tfs ? t.lr : t.projection) = pre;
                t.aggregate = agg;
                t.convert = conv;
                t.total = pre + agg + conv;
                t.neighbor_steps = tfs ? neighbor_steps * p.heads : 0;
                std::ostringstream extra;
                extra << std::setprecision(10) << ",\"h2d_ms\":" << (l == 0 ? st[0] : 0.0)
                      << ",\"d2h_ms\":" << (l == 2 ? st[8] : 0.0) << ",\"kernels\":" << gat_b200_model_launches(m);
                print_times(path, mode, l + 1, r, g, p, threads, fp32, t, (degree_sort_s + prepare_s) * 1000, panel,
                            extra.str());
            }
            std::cout << "E2E path=" << path << " rep=" << r << " layer=" << layer_arg << " total_ms=" << total * 1000
                      << " finite=1\n";
        }
        if (!a.get("--output").empty()) dump(a.get("--output"), logits);
        std::cout << "SUMMARY path=" << path << " median_ms=" << pct(totals, .5) * 1000
                  << " p95_ms=" << pct(totals, .95) * 1000 << " cold_forward_ms=" << cold_forward * 1000
                  << " repeats=" << reps << " task_accuracy=UNVERIFIED\n";
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "FAIL " << e.what() << "\n";
        return 1;
    }
}
