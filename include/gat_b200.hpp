// C++ mirror of the reference's host API (baseline/include/gat.hpp) over the
// C ABI of libgat_b200.so (include/gat_b200.h); the online TFS experiments of
// baseline/tfs_online/icpp_*.hpp are mirrored in gat_b200_online.hpp. A caller of the reference
// switches by including this header and aliasing the namespace:
//
//   #include "gat_b200.hpp"
//   namespace gat = gat_b200;
//
// Names, argument meaning and error behaviour follow gat.hpp: the same structs
// (Graph, Param, Prepared, Schedule, Workspace, Times, Error, Fixture), the same
// free functions and defaults, failures thrown as std::runtime_error with the
// reference's messages. Workspace keeps the reference's host vectors as the
// results: each compute call uploads what it reads from them, runs the
// library's kernels on the current CUDA device and writes its outputs back.
// There is no host arithmetic on the compute path. Differences, by design:
//   * projection() computes Z together with L and R (one tensor-core kernel);
//     lr_from_z() checks that they came from the preceding projection();
//   * ref_layer() (R0) takes its output from the FP32 path, which the
//     library's tests pin to R0 at max-abs <= 1e-5, and its trace (max, den,
//     score, p, alpha) from R0's edge softmax on the device;
//   * standard_layer() runs the stages one by one (one device call each) and
//     leaves the workspace as the reference does; the timed forward is the
//     model API;
//   * the panel argument of the TFS calls has no counterpart (the degree
//     schedule orders and balances the rows); it is accepted and ignored.
// Header-only; link with -lgat_b200.
#pragma once
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <iomanip>
#include <iostream>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "gat_b200.h"

namespace gat_b200 {

using BF16 = uint16_t;
using Clock = std::chrono::steady_clock;
inline double seconds(Clock::time_point a, Clock::time_point b) {
    return std::chrono::duration<double>(b - a).count();
}
// the reference's profile-build switches (gat.hpp:23-29): a speed build here
inline Clock::time_point tick() { return {}; }
inline constexpr bool profiling = false;

inline void check(int rc) {
    if (rc) throw std::runtime_error(gat_b200_last_error());
}

// baseline/src/common.cpp:6-13
inline size_t checked(uint64_t a, uint64_t b) {
    if (b && a > SIZE_MAX / b) throw std::runtime_error("size overflow");
    return size_t(a * b);
}
inline void require_finite(const std::vector<float>& a, const std::string& name) {
    for (size_t i = 0; i < a.size(); ++i)
        if (!std::isfinite(a[i])) throw std::runtime_error("nonfinite " + name + " index=" + std::to_string(i));
}

// ---- graph, parameters, files ---------------------------------------------
struct Graph {
    uint64_t n = 0, e = 0;
    int din = 0, classes = 0;
    std::vector<uint64_t> row;
    std::vector<uint32_t> col;
    std::vector<float> x;
    void validate() const {
        if (!n || n > INT32_MAX || din <= 0 || classes <= 0 || row.size() != n + 1 || col.size() != e ||
            x.size() != checked(n, uint64_t(din)))
            throw std::runtime_error("invalid graph sizes");
        check(gat_b200_validate_csr(n, e, row.data(), col.data()));
        require_finite(x, "graph input");
    }
};

inline Graph load_graph(const std::string& path) {
    Graph g;
    uint32_t din = 0, classes = 0;
    check(gat_b200_read_graph_header(path.c_str(), &g.n, &g.e, &din, &classes));
    g.din = int(din);
    g.classes = int(classes);
    g.row.resize(g.n + 1);
    g.col.resize(g.e);
    g.x.resize(checked(g.n, din));
    check(gat_b200_read_graph(path.c_str(), g.n, g.e, din, g.row.data(), g.col.data(), g.x.data()));
    return g;
}
inline void save_graph(const Graph& g, const std::string& path) {
    check(gat_b200_write_graph(path.c_str(), g.n, g.e, uint32_t(g.din), uint32_t(g.classes), g.row.data(),
                               g.col.data(), g.x.data()));
}

struct Param {
    int in = 0, heads = 0, dim = 0;
    std::vector<float> w, al, ar;  // W[in][heads*dim]; heads are independent.
    int width() const { return heads * dim; }
    void validate() const {  // baseline/src/common.cpp:45-49
        if (in <= 0 || heads <= 0 || heads > 8 || dim <= 0 || dim > 64 ||
            w.size() != checked(uint64_t(in), uint64_t(width())) || al.size() != size_t(width()) ||
            ar.size() != size_t(width()))
            throw std::runtime_error("invalid parameter shape (heads <=8, head_dim <=64)");
        require_finite(w, "W");
        require_finite(al, "aL");
        require_finite(ar, "aR");
    }
};
using Model = std::vector<Param>;

namespace detail {
inline Model model_storage(int din, int classes) {  // common.cpp:53: din -> 8x32 -> 8x32 -> 1xC
    Model m(3);
    for (int l = 0; l < 3; ++l) {
        m[l].in = l == 0 ? din : 256;
        m[l].heads = l < 2 ? 8 : 1;
        m[l].dim = l < 2 ? 32 : classes;
        m[l].w.resize(size_t(m[l].in) * m[l].width());
        m[l].al.resize(m[l].width());
        m[l].ar.resize(m[l].width());
    }
    return m;
}
struct Ptrs {
    float* w[3];
    float* al[3];
    float* ar[3];
    explicit Ptrs(Model& m) {
        for (int l = 0; l < 3; ++l) {
            w[l] = m[l].w.data();
            al[l] = m[l].al.data();
            ar[l] = m[l].ar.data();
        }
    }
};
}  // namespace detail

inline Model random_model(int din, int classes, int seed) {
    Model m = detail::model_storage(din, classes);
    detail::Ptrs p(m);
    check(gat_b200_random_model(din, classes, seed, p.w, p.al, p.ar));
    return m;
}
inline Model load_model(const std::string& path, int din, int classes) {
    Model m = detail::model_storage(din, classes);
    detail::Ptrs p(m);
    check(gat_b200_read_weights(path.c_str(), din, classes, p.w, p.al, p.ar));
    return m;
}
inline void save_model(const Model& m, const std::string& path) {
    if (m.size() != 3) throw std::runtime_error("model must have three layers");
    const float* w[3] = {m[0].w.data(), m[1].w.data(), m[2].w.data()};
    const float* al[3] = {m[0].al.data(), m[1].al.data(), m[2].al.data()};
    const float* ar[3] = {m[0].ar.data(), m[1].ar.data(), m[2].ar.data()};
    check(gat_b200_write_weights(path.c_str(), m[0].in, m[2].dim, w, al, ar));
}

// ---- BF16 -----------------------------------------------------------------
inline float leak(float x) { return x >= 0 ? x : 0.2f * x; }
inline float elu(float x) { return x >= 0 ? x : std::expm1(x); }
inline BF16 rne(float x) { return gat_b200_rne(x); }
inline float expand(BF16 x) {
    uint32_t u = uint32_t(x) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
inline void convert(const float* input, BF16* output, size_t count) {
    check(gat_b200_convert_host(input, output, count));
}
inline std::vector<float> quantized(const std::vector<float>& a) {
    std::vector<BF16> b(a.size());
    convert(a.data(), b.data(), a.size());
    std::vector<float> r(a.size());
    for (size_t i = 0; i < a.size(); ++i) r[i] = expand(b[i]);
    return r;
}

// ---- timing, errors --------------------------------------------------------
struct Times {
    double convert = 0, projection = 0, lr = 0, max_prescan = 0, aggregate = 0, normalize = 0, activation = 0,
           total = 0;
    // the reference's profile-build worker sums (CPU workers): kept at 0 here
    double score_exp_worker = 0, gather_weight_convert_worker = 0, tile_load_worker = 0;
    double gather_load_worker = 0, p_times_x_convert_worker = 0, weighted_spmm_worker = 0;
    double amx_compute_worker = 0, tile_store_worker = 0, normalize_worker = 0, activation_worker = 0;
    double tile_config_worker = 0, scheduling_worker = 0, output_write_worker = 0;
    uint64_t neighbor_steps = 0, executed_fma = 0;
};
struct Error {
    double max_abs = 0, mean_abs = 0, relative_l2 = 0, rmse = 0, p50 = 0, p90 = 0, p99 = 0;
    bool finite = true;
};
// baseline/src/common.cpp:141-150
inline Error errors(const std::vector<float>& ref, const std::vector<float>& actual) {
    if (ref.size() != actual.size()) throw std::runtime_error("error metric size mismatch");
    Error e;
    double num = 0, den = 0, sum = 0;
    std::vector<double> d(ref.size());
    for (size_t i = 0; i < ref.size(); ++i) {
        if (!std::isfinite(actual[i])) e.finite = false;
        d[i] = std::fabs(double(actual[i]) - double(ref[i]));
        e.max_abs = std::max(e.max_abs, d[i]);
        sum += d[i];
        num += d[i] * d[i];
        den += double(ref[i]) * ref[i];
    }
    if (!ref.empty()) {
        e.mean_abs = sum / ref.size();
        e.rmse = std::sqrt(num / ref.size());
        e.relative_l2 = std::sqrt(num) / std::max(std::sqrt(den), 1e-30);
        std::sort(d.begin(), d.end());
        auto q = [&](double p) { return d[std::min(d.size() - 1, size_t(std::ceil(p * d.size())) - 1)]; };
        e.p50 = q(.5);
        e.p90 = q(.9);
        e.p99 = q(.99);
    }
    return e;
}
inline void print_error(const std::string& path, int layer, const std::string& stage, const Error& e) {
    std::cout << std::setprecision(10) << "ERROR path=" << path << " layer=" << layer << " stage=" << stage
              << " finite=" << e.finite << " max_abs=" << e.max_abs << " mean_abs=" << e.mean_abs
              << " relative_l2=" << e.relative_l2 << " rmse=" << e.rmse << " p50=" << e.p50 << " p90=" << e.p90
              << " p99=" << e.p99 << "\n";
}

// The per-layer JSON line (common.cpp:155-170) with the reference's keys. The
// reference's OpenMP thread count has no counterpart: `threads` prints 1.
// (The overload taking the Workspace, as gat.hpp declares it, follows it.)
inline void print_times(const std::string& path, const std::string& mode, int layer, int rep, const Graph& g,
                        const Param& p, size_t workspace_bytes, const Times& t, double stat, int panel) {
    const uint64_t useful = g.e * uint64_t(p.heads) * uint64_t(p.in) * uint64_t(p.dim);
    std::cout << std::setprecision(10) << "{\"path\":\"" << path << "\",\"mode\":\"" << mode << "\",\"layer\":" << layer
              << ",\"rep\":" << rep << ",\"N\":" << g.n << ",\"E\":" << g.e << ",\"D\":" << p.in << ",\"K\":" << p.heads
              << ",\"d\":" << p.dim << ",\"threads\":1,\"profile\":false,\"precision\":\""
              << (path == "ref_fp32" || path == "standard_fp32" ? "FP32" : "BF16_RNE_FP32_state") << "\""
              << ",\"projection_ms\":" << t.projection * 1000 << ",\"lr_ms\":" << t.lr * 1000
              << ",\"max_prescan_ms\":" << t.max_prescan * 1000 << ",\"score_exp_aggregate_ms\":" << t.aggregate * 1000
              << ",\"normalize_ms\":" << t.normalize * 1000 << ",\"activation_ms\":" << t.activation * 1000
              << ",\"convert_ms\":" << t.convert * 1000 << ",\"total_ms\":" << t.total * 1000
              << ",\"workspace_bytes\":" << workspace_bytes << ",\"static_preprocess_ms\":" << stat * 1000
              << ",\"panel_R\":" << panel << ",\"tile_rows\":16,\"score_exp_worker_ms\":" << t.score_exp_worker * 1000
              << ",\"gather_weight_convert_worker_ms\":" << t.gather_weight_convert_worker * 1000
              << ",\"tile_load_worker_ms\":" << t.tile_load_worker * 1000
              << ",\"gather_load_worker_ms\":" << t.gather_load_worker * 1000
              << ",\"p_times_x_convert_worker_ms\":" << t.p_times_x_convert_worker * 1000
              << ",\"weighted_spmm_worker_ms\":" << t.weighted_spmm_worker * 1000
              << ",\"amx_compute_worker_ms\":" << t.amx_compute_worker * 1000
              << ",\"tile_store_worker_ms\":" << t.tile_store_worker * 1000
              << ",\"tile_config_worker_ms\":" << t.tile_config_worker * 1000
              << ",\"scheduling_worker_ms\":" << t.scheduling_worker * 1000
              << ",\"output_write_worker_ms\":" << t.output_write_worker * 1000
              << ",\"neighbor_steps\":" << t.neighbor_steps << ",\"executed_fma\":" << t.executed_fma
              << ",\"padding_executed_flops\":" << (t.executed_fma ? 2 * (t.executed_fma - useful) : 0) << "}\n";
}

// ---- device objects ---------------------------------------------------------
namespace detail {
struct DeviceBuffer {
    void* p = nullptr;
    size_t bytes = 0;
    DeviceBuffer() = default;
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    ~DeviceBuffer() { gat_b200_device_free(p); }
    void* get(size_t n) {  // at least n bytes (contents unspecified after growth)
        if (n > bytes) {
            gat_b200_device_free(p);
            p = nullptr;
            bytes = 0;
            check(gat_b200_device_alloc(n, &p));
            bytes = n;
        }
        return p;
    }
    template <class T>
    T* upload(const std::vector<T>& v) {
        void* d = get(v.size() * sizeof(T));
        check(gat_b200_copy_to_device(d, v.data(), v.size() * sizeof(T)));
        return static_cast<T*>(d);
    }
    template <class T>
    void download(std::vector<T>& v) const {
        check(gat_b200_copy_to_host(v.data(), p, v.size() * sizeof(T)));
    }
};
struct GraphHandle {
    gat_b200_graph* g = nullptr;
    uint64_t n = 0, e = 0;
    const uint64_t* row = nullptr;
    const uint32_t* col = nullptr;
    ~GraphHandle() { gat_b200_graph_destroy(g); }
    // the device graph of g (re-created when the caller passes another graph)
    gat_b200_graph* of(const Graph& gr) {
        if (!g || n != gr.n || e != gr.e || row != gr.row.data() || col != gr.col.data()) {
            gat_b200_graph_destroy(g);
            g = nullptr;
            check(gat_b200_graph_create(gr.n, gr.e, gr.row.data(), gr.col.data(), nullptr, &g));
            n = gr.n;
            e = gr.e;
            row = gr.row.data();
            col = gr.col.data();
        }
        return g;
    }
};
struct LayerHandle {
    gat_b200_layer* p = nullptr;
    ~LayerHandle() { gat_b200_layer_destroy(p); }
};
}  // namespace detail

// prepare(): the device copy of a layer (BF16 W^T, FP32 W, a, W.a).
struct Prepared {
    std::shared_ptr<detail::LayerHandle> layer;
    // w: the BF16 RNE copy of W, as the reference keeps it. Its other host
    // copies (W a in FP32 / BF16 / transposed, the AMX packing) live on the
    // device inside `layer`; those vectors stay empty.
    std::vector<BF16> w, blr_bf16, packed;
    std::vector<float> blr, blr_dot;
    int padded_in = 0, output_blocks = 0;
    double weight_prepare_s = 0;
};
inline Prepared prepare(const Param& p, bool = true, bool = true, bool = true) {
    p.validate();
    auto t0 = Clock::now();
    Prepared q;
    q.layer = std::make_shared<detail::LayerHandle>();
    check(gat_b200_layer_create(p.in, p.heads, p.dim, p.w.data(), p.al.data(), p.ar.data(), &q.layer->p));
    q.padded_in = (p.in + 31) / 32 * 32;
    q.output_blocks = (p.dim + 15) / 16;
    // the reference's BF16 copy of W (common.cpp:98-99), for callers that emulate
    // the BF16 arithmetic themselves (boundaries.cpp:44)
    q.w.resize(p.w.size());
    check(gat_b200_convert_host(p.w.data(), q.w.data(), p.w.size()));
    q.weight_prepare_s = seconds(t0, Clock::now());
    return q;
}

struct Schedule {
    std::vector<uint32_t> perm;
    uint64_t neighbor_steps = 0;
    double degree_sort_s = 0;
};
inline Schedule degree_schedule(const Graph& g) {
    detail::GraphHandle h;
    auto t0 = Clock::now();
    Schedule s;
    s.perm.resize(g.n);
    check(gat_b200_graph_schedule(h.of(g), s.perm.data(), &s.neighbor_steps));
    s.degree_sort_s = seconds(t0, Clock::now());
    return s;
}

struct Workspace {
    std::vector<BF16> xbf;
    std::vector<float> z, left, right, max, den, out;
    std::vector<float> score, p, alpha;  // R0 trace [e][heads] (ref_fp32 workspaces)
    // the reference's CPU scratch (L/R staging, per-thread tiles, the L/R SGEMM
    // operands): no counterpart on the device, kept empty
    std::vector<float> lr, thread_cbuf, lr_sgemm_weights, lr_sgemm_tmp;
    std::vector<BF16> thread_hbuf;
    // device state
    std::shared_ptr<detail::GraphHandle> graph = std::make_shared<detail::GraphHandle>();
    std::shared_ptr<detail::DeviceBuffer> d_x = std::make_shared<detail::DeviceBuffer>(),
                                          d_xb = std::make_shared<detail::DeviceBuffer>(),
                                          d_z = std::make_shared<detail::DeviceBuffer>(),
                                          d_left = std::make_shared<detail::DeviceBuffer>(),
                                          d_right = std::make_shared<detail::DeviceBuffer>(),
                                          d_max = std::make_shared<detail::DeviceBuffer>(),
                                          d_den = std::make_shared<detail::DeviceBuffer>(),
                                          d_out = std::make_shared<detail::DeviceBuffer>(),
                                          d_fp = std::make_shared<detail::DeviceBuffer>(),
                                          d_fd = std::make_shared<detail::DeviceBuffer>(),
                                          d_trace = std::make_shared<detail::DeviceBuffer>();
    bool lr_from_projection = false;
    // baseline/src/common.cpp:126-134: the buffers of each path
    void allocate(const Graph& g, const Param& p, const std::string& path) {
        const size_t nw = checked(g.n, uint64_t(p.width())), nk = checked(g.n, uint64_t(p.heads));
        if (path != "ref_fp32" && path != "standard_bf16" && path != "standard_fp32" && path != "tfs_bf16" &&
            path != "matched_attention")
            throw std::runtime_error("unknown workspace path " + path);
        z.assign(path == "tfs_bf16" ? 0 : nw, 0.f);
        left.assign(nk, 0.f);
        right.assign(nk, 0.f);
        max.assign(nk, 0.f);
        den.assign(nk, 0.f);
        out.assign(nw, 0.f);
        xbf.assign(path == "standard_fp32" || path == "ref_fp32" ? 0 : checked(g.n, uint64_t(p.in)), 0);
        const size_t ek = path == "ref_fp32" ? checked(g.e, uint64_t(p.heads)) : 0;
        score.assign(ek, 0.f);
        this->p.assign(ek, 0.f);
        alpha.assign(ek, 0.f);
        graph->of(g);
    }
    // common.cpp:135-138: L/R come from the projection's epilogue on every
    // policy, so there is no SGEMM operand to prepare
    void prepare_lr_sgemm(const Graph&, const Param&) {}
    size_t bytes() const {
        return (xbf.size() + thread_hbuf.size()) * 2 +
               (z.size() + left.size() + right.size() + max.size() + den.size() + out.size() + lr.size() +
                score.size() + p.size() + alpha.size() + thread_cbuf.size() + lr_sgemm_weights.size() +
                lr_sgemm_tmp.size()) *
                   4;
    }
};

inline void print_times(const std::string& path, const std::string& mode, int layer, int rep, const Graph& g,
                        const Param& p, const Workspace& w, const Times& t, double stat, int panel) {
    print_times(path, mode, layer, rep, g, p, w.bytes(), t, stat, panel);
}

namespace detail {
inline int padded(int width, int dtype) { return gat_b200_padded_ld(width, dtype); }
// lr_reordered's policies (baseline/src/baseline_standard.cpp:29-40): "bf16"
// multiplies the BF16 input by RNE(W a); "fp32" and "avx" multiply the FP32
// input by W a (one SGEMM, or one dot product per row and column).
inline int lr_policy(const std::string& policy) {
    if (policy == "bf16") return GAT_B200_LR_BF16;
    if (policy == "fp32" || policy == "avx") return GAT_B200_LR_FP32;
    throw std::runtime_error("unknown LR policy");
}
inline void need(const std::vector<float>& v, size_t n, const char* what) {
    if (v.size() != n) throw std::runtime_error(std::string("workspace ") + what + " has the wrong size");
}
// Dense [n][width] rows of a device buffer with row stride ld (FP32), into v.
inline void download_rows(const DeviceBuffer& b, uint64_t n, int width, int ld, std::vector<float>& v) {
    if (ld == width) {
        b.download(v);
        return;
    }
    std::vector<float> tmp(size_t(n) * ld);
    b.download(tmp);
    for (uint64_t i = 0; i < n; ++i)
        std::copy(tmp.begin() + i * ld, tmp.begin() + i * ld + width, v.begin() + i * width);
}
// FP32 input rows [n][in] -> device BF16 [n][padded] (the reference's convert, on the device).
inline const void* upload_bf16(Workspace& w, const std::vector<float>& input, uint64_t n, int in, int& ld) {
    ld = padded(in, GAT_B200_BF16);
    const float* x = w.d_x->upload(input);
    void* xb = w.d_xb->get(size_t(n) * ld * 2);
    check(gat_b200_convert(n, in, x, in, static_cast<uint16_t*>(xb), ld, nullptr));
    return xb;
}
}  // namespace detail

// ---- the layer functions (baseline/include/gat.hpp:107-117) -------------------
// Z = X W (BF16 inputs on tensor cores when bf16, else FP32), with L and R.
inline void projection(const Graph& g, const Param& p, const Prepared& q, const std::vector<float>& input,
                       Workspace& w, bool bf16) {
    detail::need(w.z, checked(g.n, uint64_t(p.width())), "z");
    if (input.size() != checked(g.n, uint64_t(p.in))) throw std::runtime_error("projection input size mismatch");
    const void* x;
    int ldx = p.in;
    if (bf16) {
        x = detail::upload_bf16(w, input, g.n, p.in, ldx);
    } else {
        x = w.d_x->upload(input);
    }
    const int ldz = detail::padded(p.width(), GAT_B200_F32);
    void* z = w.d_z->get(size_t(g.n) * ldz * 4);
    float* l = static_cast<float*>(w.d_left->get(w.left.size() * 4));
    float* r = static_cast<float*>(w.d_right->get(w.right.size() * 4));
    check(gat_b200_projection(q.layer->p, g.n, x, ldx, bf16 ? GAT_B200_BF16 : GAT_B200_F32, z, GAT_B200_F32, ldz,
                              l, r, nullptr));
    detail::download_rows(*w.d_z, g.n, p.width(), ldz, w.z);
    w.d_left->download(w.left);
    w.d_right->download(w.right);
    w.lr_from_projection = true;
}
inline void lr_from_z(const Graph&, const Param&, Workspace& w, bool = false) {
    if (!w.lr_from_projection) throw std::runtime_error("lr_from_z: L and R come from projection(); call it first");
}
// baseline_standard.cpp:21-28 (the same L and R through an SGEMM)
inline void lr_from_z_mkl(const Graph& g, const Param& p, Workspace& w) { lr_from_z(g, p, w); }
inline void lr_reordered(const Graph& g, const Param& p, const Prepared& q, const std::vector<float>& input,
                         Workspace& w, const std::string& policy) {
    const int pol = detail::lr_policy(policy);
    const float* x = w.d_x->upload(input);
    const int ldb = detail::padded(p.in, GAT_B200_BF16);
    void* xb = w.d_xb->get(size_t(g.n) * ldb * 2);
    float* l = static_cast<float*>(w.d_left->get(w.left.size() * 4));
    float* r = static_cast<float*>(w.d_right->get(w.right.size() * 4));
    check(gat_b200_lr_reordered(q.layer->p, g.n, x, GAT_B200_F32, p.in, pol, xb, ldb, l, r, nullptr));
    w.d_left->download(w.left);
    w.d_right->download(w.right);
    if (!w.xbf.empty()) {
        std::vector<BF16> tmp(size_t(g.n) * ldb);
        check(gat_b200_copy_to_host(tmp.data(), xb, tmp.size() * 2));
        for (uint64_t i = 0; i < g.n; ++i)
            std::copy(tmp.begin() + i * ldb, tmp.begin() + i * ldb + p.in, w.xbf.begin() + i * p.in);
    }
    w.lr_from_projection = false;
}
inline void max_prescan(const Graph& g, const Param& p, Workspace& w) {
    const size_t nk = checked(g.n, uint64_t(p.heads));
    detail::need(w.left, nk, "left");
    detail::need(w.right, nk, "right");
    detail::need(w.max, nk, "max");
    const float* l = w.d_left->upload(w.left);
    const float* r = w.d_right->upload(w.right);
    float* m = static_cast<float*>(w.d_max->get(w.max.size() * 4));
    check(gat_b200_max_prescan(w.graph->of(g), p.heads, l, r, m, nullptr));
    w.d_max->download(w.max);
}
// Unnormalised out and den (and max), from w.z (FP32 rows) and w.left / w.right,
// or from fixed_p [e][heads] / fixed_den [n][heads].
inline void standard_aggregate(const Graph& g, const Param& p, Workspace& w, const float* fixed_p = nullptr,
                               const float* fixed_den = nullptr, Times* times = nullptr) {
    auto t0 = Clock::now();
    const size_t nk = checked(g.n, uint64_t(p.heads)), nw = checked(g.n, uint64_t(p.width()));
    detail::need(w.z, nw, "z");
    detail::need(w.left, nk, "left");
    detail::need(w.right, nk, "right");
    detail::need(w.out, nw, "out");
    detail::need(w.den, nk, "den");
    detail::need(w.max, nk, "max");
    const int ldz = detail::padded(p.width(), GAT_B200_F32);
    std::vector<float> zp(size_t(g.n) * ldz, 0.f);
    for (uint64_t i = 0; i < g.n; ++i)
        std::copy(w.z.begin() + i * p.width(), w.z.begin() + (i + 1) * p.width(), zp.begin() + i * ldz);
    const float* z = w.d_z->upload(zp);
    const float* l = w.d_left->upload(w.left);
    const float* r = w.d_right->upload(w.right);
    const float *fp = nullptr, *fd = nullptr;
    if (fixed_p) {
        std::vector<float> a(fixed_p, fixed_p + checked(g.e, uint64_t(p.heads)));
        std::vector<float> b(fixed_den, fixed_den + checked(g.n, uint64_t(p.heads)));
        fp = w.d_fp->upload(a);
        fd = w.d_fd->upload(b);
    }
    float* o = static_cast<float*>(w.d_out->get(w.out.size() * 4));
    float* dn = static_cast<float*>(w.d_den->get(w.den.size() * 4));
    float* m = static_cast<float*>(w.d_max->get(w.max.size() * 4));
    check(gat_b200_standard_aggregate(w.graph->of(g), p.heads, p.dim, z, GAT_B200_F32, ldz, l, r, fp, fd, o,
                                      p.width(), dn, m, nullptr));
    w.d_out->download(w.out);
    w.d_den->download(w.den);
    w.d_max->download(w.max);
    if (times) times->aggregate += seconds(t0, Clock::now());
}
inline void finish(const Graph& g, const Param& p, Workspace& w, bool hidden, Times& t) {
    auto t0 = Clock::now();
    detail::need(w.out, checked(g.n, uint64_t(p.width())), "out");
    detail::need(w.den, checked(g.n, uint64_t(p.heads)), "den");
    float* o = w.d_out->upload(w.out);
    const float* dn = w.d_den->upload(w.den);
    check(gat_b200_finish(g.n, p.heads, p.dim, dn, hidden, o, p.width(), nullptr));
    w.d_out->download(w.out);
    t.normalize += seconds(t0, Clock::now());
}
// The B0 layer (baseline_standard.cpp:98-108), stage by stage as the reference
// runs it, so that the workspace holds what the reference leaves there: xbf
// (BF16 path), z (FP32), left and right (from Z, or from lr_reordered with the
// policies "bf16" / "fp32" / "avx": the matched-attention layer), max, den and
// the finished out. Each stage is one device call with its copies; the timed
// forward is the model API.
inline void standard_layer(const Graph& g, const Param& p, const Prepared& q, const std::vector<float>& input,
                           Workspace& w, bool hidden, Times& t, bool fp32 = false,
                           const std::string& lr_policy = "z_avx") {
    const bool matched = lr_policy != "z_avx" && lr_policy != "z_mkl";
    if (matched) detail::lr_policy(lr_policy);  // "unknown LR policy"
    if (input.size() != checked(g.n, uint64_t(p.in))) throw std::runtime_error("layer input size mismatch");
    const auto begin = Clock::now();
    auto a = begin;
    if (!fp32 && w.xbf.size() == input.size()) check(gat_b200_convert_host(input.data(), w.xbf.data(), input.size()));
    t.convert = seconds(a, Clock::now());
    a = Clock::now();
    projection(g, p, q, input, w, !fp32);
    t.projection = seconds(a, Clock::now());
    a = Clock::now();
    if (matched)
        lr_reordered(g, p, q, input, w, lr_policy);
    else
        lr_from_z(g, p, w);
    t.lr = seconds(a, Clock::now());
    a = Clock::now();
    max_prescan(g, p, w);
    t.max_prescan = seconds(a, Clock::now());
    a = Clock::now();
    standard_aggregate(g, p, w, nullptr, nullptr, &t);
    t.aggregate = seconds(a, Clock::now());
    finish(g, p, w, hidden, t);
    t.total = seconds(begin, Clock::now());
}
// R0 (baseline/src/ref_fp32.cpp:3-26): out from the FP32 path (FP32 projection,
// aggregation, finish), and the R0 trace from gat_b200_edge_softmax: z, left,
// right, and max, den in R0's order, with score, p and alpha when the workspace
// was allocated for ref_fp32.
inline void ref_layer(const Graph& g, const Param& p, const std::vector<float>& input, Workspace& w, bool hidden,
                      Times& t) {
    const auto begin = Clock::now();
    auto a = begin;
    const Prepared q = prepare(p);
    projection(g, p, q, input, w, false);
    t.projection += seconds(a, Clock::now());
    a = Clock::now();
    standard_aggregate(g, p, w);
    finish(g, p, w, hidden, t);
    t.aggregate += seconds(a, Clock::now());
    const size_t ek = checked(g.e, uint64_t(p.heads)), nk = checked(g.n, uint64_t(p.heads));
    const bool trace = w.score.size() == ek && w.p.size() == ek && w.alpha.size() == ek;
    float* buf = static_cast<float*>(w.d_trace->get(((trace ? 3 : 1) * ek + 2 * nk) * 4));
    float *pp = buf, *dn = buf + ek, *mx = dn + nk;
    float* sc = trace ? mx + nk : nullptr;
    float* al = trace ? sc + ek : nullptr;
    const float* l = w.d_left->upload(w.left);
    const float* r = w.d_right->upload(w.right);
    check(gat_b200_edge_softmax(w.graph->of(g), p.heads, l, r, sc, mx, pp, dn, al, nullptr));
    check(gat_b200_copy_to_host(w.den.data(), dn, nk * 4));
    check(gat_b200_copy_to_host(w.max.data(), mx, nk * 4));
    if (trace) {
        check(gat_b200_copy_to_host(w.score.data(), sc, ek * 4));
        check(gat_b200_copy_to_host(w.p.data(), pp, ek * 4));
        check(gat_b200_copy_to_host(w.alpha.data(), al, ek * 4));
    }
    t.total += seconds(begin, Clock::now());
}
// B1 (baseline/src/baseline_tfs.cpp:16-110) from w.xbf, w.left, w.right, w.max.
inline void tfs_aggregate(const Graph& g, const Param& p, const Prepared& q, const Schedule&, Workspace& w, int,
                          Times& t, const float* fixed_p = nullptr, const float* fixed_den = nullptr) {
    auto t0 = Clock::now();
    const size_t nk = checked(g.n, uint64_t(p.heads));
    if (w.xbf.size() != checked(g.n, uint64_t(p.in))) throw std::runtime_error("workspace xbf has the wrong size");
    detail::need(w.left, nk, "left");
    detail::need(w.right, nk, "right");
    if (!fixed_p) detail::need(w.max, nk, "max");
    detail::need(w.out, checked(g.n, uint64_t(p.width())), "out");
    detail::need(w.den, nk, "den");
    const int ldb = detail::padded(p.in, GAT_B200_BF16);
    std::vector<BF16> xp(size_t(g.n) * ldb, 0);
    for (uint64_t i = 0; i < g.n; ++i)
        std::copy(w.xbf.begin() + i * p.in, w.xbf.begin() + (i + 1) * p.in, xp.begin() + i * ldb);
    const void* xb = w.d_xb->upload(xp);
    const float* l = w.d_left->upload(w.left);
    const float* r = w.d_right->upload(w.right);
    const float* m = fixed_p ? nullptr : w.d_max->upload(w.max);
    const float *fp = nullptr, *fd = nullptr;
    if (fixed_p) {
        std::vector<float> a(fixed_p, fixed_p + checked(g.e, uint64_t(p.heads)));
        std::vector<float> b(fixed_den, fixed_den + checked(g.n, uint64_t(p.heads)));
        fp = w.d_fp->upload(a);
        fd = w.d_fd->upload(b);
    }
    float* o = static_cast<float*>(w.d_out->get(w.out.size() * 4));
    float* dn = static_cast<float*>(w.d_den->get(w.den.size() * 4));
    check(gat_b200_tfs_aggregate(w.graph->of(g), q.layer->p, xb, ldb, l, r, m, fp, fd, GAT_B200_TFS_EDGE, 0, 1, o,
                                 p.width(), dn, nullptr, nullptr));
    w.d_out->download(w.out);
    w.d_den->download(w.den);
    t.aggregate += seconds(t0, Clock::now());
}
// The B1 layer (baseline/src/baseline_tfs.cpp:111-117).
inline void tfs_layer(const Graph& g, const Param& p, const Prepared& q, const Schedule&,
                      const std::vector<float>& input, Workspace& w, bool hidden, int, Times& t,
                      const std::string& lr_policy) {
    auto t0 = Clock::now();
    const size_t nk = checked(g.n, uint64_t(p.heads));
    if (input.size() != checked(g.n, uint64_t(p.in))) throw std::runtime_error("layer input size mismatch");
    if (w.xbf.size() != checked(g.n, uint64_t(p.in))) throw std::runtime_error("workspace xbf has the wrong size");
    detail::need(w.left, nk, "left");
    detail::need(w.right, nk, "right");
    detail::need(w.max, nk, "max");
    detail::need(w.den, nk, "den");
    detail::need(w.out, checked(g.n, uint64_t(p.width())), "out");
    const float* x = w.d_x->upload(input);
    const int ldb = detail::padded(p.in, GAT_B200_BF16);
    void* xb = w.d_xb->get(size_t(g.n) * ldb * 2);
    float* l = static_cast<float*>(w.d_left->get(w.left.size() * 4));
    float* r = static_cast<float*>(w.d_right->get(w.right.size() * 4));
    float* m = static_cast<float*>(w.d_max->get(w.max.size() * 4));
    float* dn = static_cast<float*>(w.d_den->get(w.den.size() * 4));
    float* o = static_cast<float*>(w.d_out->get(w.out.size() * 4));
    check(gat_b200_tfs_layer(w.graph->of(g), q.layer->p, x, GAT_B200_F32, p.in, hidden,
                             detail::lr_policy(lr_policy), GAT_B200_TFS_EDGE, 0, 1, xb,
                             l, r, m, dn, o, GAT_B200_F32, p.width(), nullptr));
    // the workspace as the reference's tfs_layer leaves it: xbf, left, right,
    // max, den and the finished out
    w.d_out->download(w.out);
    w.d_left->download(w.left);
    w.d_right->download(w.right);
    w.d_max->download(w.max);
    w.d_den->download(w.den);
    std::vector<BF16> tmp(size_t(g.n) * ldb);
    check(gat_b200_copy_to_host(tmp.data(), xb, tmp.size() * 2));
    for (uint64_t i = 0; i < g.n; ++i)
        std::copy(tmp.begin() + i * ldb, tmp.begin() + i * ldb + p.in, w.xbf.begin() + i * p.in);
    t.total += seconds(t0, Clock::now());
}

struct Trace {
    std::vector<float> z, left, right, max, den, score, p, alpha;
};
inline Trace capture(const Workspace& w) { return Trace{w.z, w.left, w.right, w.max, w.den, w.score, w.p, w.alpha}; }

// ---- GATFIX1 fixed-p fixtures (baseline/src/common.cpp:171-194) -------------
struct Fixture {
    std::vector<float> input, p, den;
};
inline void save_fixture(const Graph& g, const Param& p, const Fixture& f, const std::string& path) {
    check(gat_b200_write_fixture(path.c_str(), g.n, g.e, p.in, p.heads, p.dim, g.row.data(), g.col.data(),
                                 p.w.data(), p.al.data(), p.ar.data(), f.input.data(), f.p.data(), f.den.data()));
}
inline Fixture load_fixture(const Graph& g, const Param& p, const std::string& path) {
    Fixture f;
    f.input.resize(checked(g.n, uint64_t(p.in)));
    f.p.resize(checked(g.e, uint64_t(p.heads)));
    f.den.resize(checked(g.n, uint64_t(p.heads)));
    check(gat_b200_read_fixture(path.c_str(), g.n, g.e, p.in, p.heads, p.dim, g.row.data(), g.col.data(),
                                p.w.data(), p.al.data(), p.ar.data(), f.input.data(), f.p.data(), f.den.data()));
    return f;
}

// ---- the model loop on N GPUs of one node -----------------------------------
// No counterpart in the reference (one CPU process). One process per GPU runs
// the reference's three-layer loop (baseline/bench/main.cpp:171-172) on its
// share of destination rows; the ranks exchange each layer's projected
// features over NVLink (gat_b200_part_model_*).
class Communicator {
public:
    // Rank `rank` of `world` on device `device`; rank 0 writes the NCCL id to
    // `id_path` (a path no earlier run used), the others wait for it.
    Communicator(const std::string& id_path, int world, int rank, int device, int timeout_ms = 120000) {
        check(gat_b200_set_device(device));
        check(gat_b200_comm_create_file(id_path.c_str(), world, rank, timeout_ms, &c_));
        world_ = world;
        rank_ = rank;
    }
    Communicator(const Communicator&) = delete;
    Communicator& operator=(const Communicator&) = delete;
    ~Communicator() { gat_b200_comm_destroy(c_); }
    void barrier() { check(gat_b200_comm_barrier(c_)); }
    int world() const { return world_; }
    int rank() const { return rank_; }
    gat_b200_comm* handle() const { return c_; }

private:
    gat_b200_comm* c_ = nullptr;
    int world_ = 1, rank_ = 0;
};

class PartitionedModel {
public:
    // Collective. g: the whole graph (every rank reads the same GATBIN1 file);
    // this rank keeps the sources and features of its own rows only.
    PartitionedModel(Communicator& comm, const Graph& g, const Model& model,
                     int exchange = GAT_B200_EXCHANGE_P2P, int chunks = 1)
        : comm_(comm) {
        for (int l = 0; l < 3; ++l) {
            model[l].validate();
            check(gat_b200_layer_create(model[l].in, model[l].heads, model[l].dim, model[l].w.data(),
                                        model[l].al.data(), model[l].ar.data(), &layers_[l]));
        }
        std::vector<uint64_t> cuts(comm.world() + 1);
        check(gat_b200_partition(g.n, g.row.data(), comm.world(), chunks, cuts.data(), nullptr, nullptr, nullptr));
        lo_ = cuts[comm.rank()];
        hi_ = cuts[comm.rank() + 1];
        const gat_b200_layer* ls[3] = {layers_[0], layers_[1], layers_[2]};
        check(gat_b200_part_model_create(comm.handle(), g.n, g.row.data(), g.col.data() + g.row[lo_], ls, exchange,
                                         chunks, nullptr, &m_));
        x_.assign(g.x.begin() + checked(lo_, g.din), g.x.begin() + checked(hi_, g.din));
        classes_ = model[2].width();
    }
    PartitionedModel(const PartitionedModel&) = delete;
    PartitionedModel& operator=(const PartitionedModel&) = delete;
    // Collective, like the constructor.
    ~PartitionedModel() {
        gat_b200_part_model_destroy(m_);
        for (auto* l : layers_) gat_b200_layer_destroy(l);
    }
    uint64_t first_row() const { return lo_; }
    uint64_t end_row() const { return hi_; }
    // Logits [end_row()-first_row()][classes] of this rank's rows.
    std::vector<float> forward() {
        std::vector<float> out(checked(hi_ - lo_, uint64_t(classes_)));
        check(gat_b200_part_model_forward(m_, x_.data(), 1, out.data(), 1, nullptr));
        return out;
    }
    // P2P exchange only: true (the default on more than one GPU) sends layer
    // 2's input rows from the layer-1 aggregation; false sends layer 2's
    // projected rows from its projection, like layers 1 and 3.
    void set_layer2_exchange(bool inputs) { check(gat_b200_part_model_set_layer2_exchange(m_, inputs ? 1 : 0)); }
    gat_b200_part_model* handle() const { return m_; }
    const std::vector<float>& input() const { return x_; }

private:
    Communicator& comm_;
    gat_b200_layer* layers_[3] = {nullptr, nullptr, nullptr};
    gat_b200_part_model* m_ = nullptr;
    uint64_t lo_ = 0, hi_ = 0;
    int classes_ = 0;
    std::vector<float> x_;
};

}  // namespace gat_b200
