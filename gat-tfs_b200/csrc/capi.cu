// Device-side C-ABI entry points of libgat_b200.so (see include/gat_b200.h).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "device.cuh"
#include "graph.cuh"

namespace gatb {
int aggregate_dispatch(const gat_b200_graph* g, int heads, int dim, const void* h, int h_dtype, int ldh,
                       const float* left, const float* right, const float* fixed_p, const float* fixed_den,
                       int unnorm, int hidden, void* out, int out_bf16, int ldo, float* den, float* max,
                       cudaStream_t st);
int convert_launch(uint64_t n, int width, const float* in, int ld_in, uint16_t* out, int ld_out, cudaStream_t st);
int max_prescan_launch(const gat_b200_graph* g, int heads, const float* left, const float* right, float* max,
                       cudaStream_t st);
int finish_launch(uint64_t n, int heads, int dim, const float* den, int hidden, float* out, int ldo, cudaStream_t st);
int edge_softmax_launch(const gat_b200_graph* g, int heads, const float* left, const float* right, float* score,
                        float* max, float* p, float* den, float* alpha, cudaStream_t st);
int projection_simt_launch(const gat_b200_layer* p, uint64_t n, const void* x, int x_bf16, int ldx, void* h,
                           int h_bf16, int ldh, float* left, float* right, cudaStream_t st);
int projection_tc_launch(const gat_b200_layer* p, uint64_t n, const uint16_t* x, int ldx, uint16_t* h, int ldh,
                         float* z, int ldz, float* left, float* right, cudaStream_t st, int npeer = 0,
                         uint16_t* const* h_peer = nullptr, float* const* r_peer = nullptr, int max_ctas = 0);
int projection_tc_check_error();
int peer_check_error();
int aggregate_check_error();
int tfs_tc_check_error();
int lr_reordered_launch(const gat_b200_layer* p, uint64_t n, const void* x, int x_dtype, int ldx, int policy,
                        uint16_t* xb, int ldb, float* left, float* right, cudaStream_t st);
int tfs_dispatch(const gat_b200_graph* g, const gat_b200_layer* p, const void* x, int ldx, const float* left,
                 const float* right, const float* max, const float* fixed_p, const float* fixed_den, int rounding,
                 int block, int threshold, int norm, int hidden, void* out, int out_bf16, int ldo, float* den,
                 float* max_out, cudaStream_t st, int* launches);
int device_check_errors() {
    int rc = projection_tc_check_error();
    int rc2 = aggregate_check_error();
    int rc3 = tfs_tc_check_error();
    int rc4 = peer_check_error();
    return rc ? rc : (rc2 ? rc2 : (rc3 ? rc3 : rc4));
}

namespace {
int dmalloc(void** p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    return e == cudaSuccess ? 0 : cuda_fail(e, "cudaMalloc");
}
}  // namespace

int projection_dispatch(const gat_b200_layer* p, uint64_t n, const void* x, int ldx, int precision, void* h,
                        int h_dtype, int ldh, float* left, float* right, cudaStream_t st) {
    if (!p || !x) return fail("projection: null argument");
    if (ldx < p->in) return fail("projection: X row stride smaller than the input width");
    if (precision == GAT_B200_BF16) {
        int rc = GAT_B200_EUNSUPPORTED;
        if (h_dtype == GAT_B200_BF16 || !h)
            rc = projection_tc_launch(p, n, static_cast<const uint16_t*>(x), ldx, static_cast<uint16_t*>(h), ldh,
                                      nullptr, 0, left, right, st);
        else
            rc = projection_tc_launch(p, n, static_cast<const uint16_t*>(x), ldx, nullptr, 0,
                                      static_cast<float*>(h), ldh, left, right, st);
        if (rc != GAT_B200_EUNSUPPORTED) return rc;
        // Shapes outside the tensor-core kernel (input width > 256): CUDA cores.
        return projection_simt_launch(p, n, x, 1, ldx, h, h_dtype == GAT_B200_BF16, ldh, left, right, st);
    }
    if (precision != GAT_B200_F32) return fail("projection: bad precision");
    return projection_simt_launch(p, n, x, 0, ldx, h, h_dtype == GAT_B200_BF16, ldh, left, right, st);
}

}  // namespace gatb

struct gat_b200_model {
    const gat_b200_graph* g = nullptr;
    const gat_b200_layer* layers[3] = {nullptr, nullptr, nullptr};
    int path = 0;
    int din = 0, classes = 0;
    float* x_f32 = nullptr;     // dense FP32 input [n][din] (device copy of the host input)
    void* x0 = nullptr;         // layer-1 input in the path's dtype [n][ld0]
    int ld0 = 0;
    void* h = nullptr;          // projected features [n][ldh_max]
    float* left = nullptr;      // [n][8]
    float* right = nullptr;     // [n][8]
    void* x1 = nullptr;         // layer outputs 1 and 2 [n][ld_hidden]
    void* x2 = nullptr;
    int ld_hidden = 0;
    float* logits = nullptr;    // [n][classes]
    float* max = nullptr;       // TFS paths: prescan maxima [n][8]
    // Optional per-stage CUDA events: `timing_steps` sets of kStageEvents,
    // one set per forward in a ring (no synchronisation inside forward).
    std::vector<cudaEvent_t> events;
    int timing_steps = 0;
    uint64_t forwards = 0;
    int launches_last = 0;  // kernels launched by the last forward
    // Pipelined host-to-host forwards (gat_b200_model_forward_async): two slots
    // of device input / logits, an upload and a download stream, and the events
    // that order slot reuse. Created by the first asynchronous call.
    float* ax[2] = {nullptr, nullptr};
    float* alog[2] = {nullptr, nullptr};
    cudaStream_t up = nullptr, down = nullptr;
    cudaEvent_t ev_up[2] = {}, ev_done[2] = {}, ev_down[2] = {};
    uint64_t submitted = 0;
};

namespace {
// Stage boundaries of one forward: h2d, convert, (projection, aggregation) x 3, d2h.
constexpr int kStages = 9;
constexpr int kStageEvents = kStages + 1;
// Stage boundaries of the forward: per-stage CUDA events when timing is on, and
// NVTX ranges (host side, one per stage inside a "gat_b200 forward" range) for
// Nsight timelines; NVTX calls cost nothing without a tool attached.
constexpr const char* kStageNames[kStages] = {"h2d",          "convert",      "projection L1",
                                              "aggregation L1", "projection L2", "aggregation L2",
                                              "projection L3", "aggregation L3", "d2h"};
inline void mark(gat_b200_model* m, int stage, cudaStream_t st) {
    if (stage == 0) nvtxRangePushA("gat_b200 forward");
    if (stage > 0) nvtxRangePop();
    if (stage < kStages) nvtxRangePushA(kStageNames[stage]);
    if (stage == kStages) nvtxRangePop();
    if (!m->timing_steps) return;
    const size_t set = size_t(m->forwards % uint64_t(m->timing_steps));
    cudaEventRecord(m->events[set * kStageEvents + stage], st);
}
}  // namespace

using namespace gatb;

namespace gatb {
// gat_b200_graph_create_part with the segment length of a graph of basis_e
// edges (0: e). The partitioned model passes the whole graph's edge count.
int graph_create_part_basis(uint64_t n, uint64_t n_src, uint64_t e, const uint64_t* row, const uint32_t* col,
                            void* stream, uint64_t basis_e, gat_b200_graph** out) {
    if (!out) return fail("graph_create_part: null output handle");
    *out = nullptr;
    if (!n || n > uint64_t(INT32_MAX) || !n_src || n_src > uint64_t(UINT32_MAX)) return fail("invalid graph sizes");
    if (!row || (e && !col)) return fail("invalid graph sizes");
    gat_b200_graph* g = new (std::nothrow) gat_b200_graph();
    if (!g) return fail("graph_create_part: out of host memory");
    g->n = n;
    g->e = e;
    g->n_src = n_src;
    g->seg_basis_e = basis_e;
    int rc = graph_build(g, row, col, as_stream(stream));
    if (rc) {
        graph_release(g);
        delete g;
        return rc;
    }
    *out = g;
    return 0;
}
}  // namespace gatb

extern "C" {

int gat_b200_graph_create(uint64_t n, uint64_t e, const uint64_t* row, const uint32_t* col, void* stream,
                          gat_b200_graph** out) {
    clear_error();
    if (!out) return fail("graph_create: null output handle");
    *out = nullptr;
    if (!n || n > uint64_t(INT32_MAX)) return fail("invalid graph sizes");
    if (!row || (e && !col)) return fail("invalid graph sizes");
    gat_b200_graph* g = new (std::nothrow) gat_b200_graph();
    if (!g) return fail("graph_create: out of host memory");
    g->n = n;
    g->e = e;
    int rc = graph_build(g, row, col, as_stream(stream));
    if (rc) {
        graph_release(g);
        delete g;
        return rc;
    }
    *out = g;
    return 0;
}


int gat_b200_graph_create_part(uint64_t n, uint64_t n_src, uint64_t e, const uint64_t* row, const uint32_t* col,
                               void* stream, gat_b200_graph** out) {
    clear_error();
    return graph_create_part_basis(n, n_src, e, row, col, stream, 0, out);
}

int gat_b200_graph_destroy(gat_b200_graph* g) {
    if (!g) return 0;
    graph_release(g);
    delete g;
    return 0;
}

int gat_b200_graph_schedule(const gat_b200_graph* g, uint32_t* perm, uint64_t* neighbor_steps) {
    if (!g) return fail("graph_schedule: null graph");
    if (perm) GATB_CUDA(cudaMemcpy(perm, g->perm, g->n * sizeof(uint32_t), cudaMemcpyDeviceToHost));
    if (neighbor_steps) *neighbor_steps = g->neighbor_steps;
    return 0;
}

int gat_b200_graph_device_csr(const gat_b200_graph* g, const uint64_t** row, const uint32_t** col) {
    if (!g) return fail("graph_device_csr: null graph");
    if (row) *row = g->row;
    if (col) *col = g->col;
    return 0;
}

int gat_b200_device_alloc(uint64_t bytes, void** ptr) {
    clear_error();
    if (!ptr) return fail("device_alloc: null output");
    *ptr = nullptr;
    void* p = nullptr;
    GATB_CUDA(cudaMalloc(&p, bytes ? bytes : 16));
    cudaError_t e = cudaMemset(p, 0, bytes ? bytes : 16);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e, "device_alloc");
    }
    *ptr = p;
    return 0;
}

int gat_b200_device_free(void* ptr) {
    clear_error();
    if (ptr) GATB_CUDA(cudaFree(ptr));
    return 0;
}

int gat_b200_copy_to_device(void* dst, const void* src, uint64_t bytes) {
    clear_error();
    if (!bytes) return 0;
    if (!dst || !src) return fail("copy_to_device: null pointer");
    GATB_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
    return 0;
}

int gat_b200_copy_to_host(void* dst, const void* src, uint64_t bytes) {
    clear_error();
    if (!bytes) return 0;
    if (!dst || !src) return fail("copy_to_host: null pointer");
    GATB_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost));
    return 0;
}

int gat_b200_graph_info(const gat_b200_graph* g, uint64_t* n, uint64_t* e, uint32_t* max_degree,
                        uint32_t* n_hub, uint32_t* n_seg, uint32_t* seg_edges) {
    if (!g) return fail("graph_info: null graph");
    if (n) *n = g->n;
    if (e) *e = g->e;
    if (max_degree) *max_degree = g->max_degree;
    if (n_hub) *n_hub = g->n_hub;
    if (n_seg) *n_seg = g->n_seg;
    if (seg_edges) *seg_edges = g->seg_edges;
    return 0;
}

int gat_b200_layer_create(int in, int heads, int dim, const float* w, const float* al, const float* ar,
                          gat_b200_layer** out) {
    clear_error();
    if (!out) return fail("layer_create: null output handle");
    *out = nullptr;
    // Param::validate (baseline/src/common.cpp:45-49)
    if (in <= 0 || heads <= 0 || heads > 8 || dim <= 0 || dim > 64 || !w || !al || !ar)
        return fail("invalid parameter shape (heads <=8, head_dim <=64)");
    const int width = heads * dim;
    const uint64_t nw = uint64_t(in) * width;
    for (uint64_t i = 0; i < nw; ++i)
        if (!std::isfinite(w[i])) return fail("nonfinite W index=" + std::to_string(i));
    for (int i = 0; i < width; ++i) {
        if (!std::isfinite(al[i])) return fail("nonfinite aL index=" + std::to_string(i));
        if (!std::isfinite(ar[i])) return fail("nonfinite aR index=" + std::to_string(i));
    }
    gat_b200_layer* p = new (std::nothrow) gat_b200_layer();
    if (!p) return fail("layer_create: out of host memory");
    p->in = in;
    p->heads = heads;
    p->dim = dim;
    p->width = width;
    p->kp = (in + 63) / 64 * 64;
    p->np = (width + 15) / 16 * 16;
    p->al_host.assign(al, al + width);
    p->ar_host.assign(ar, ar + width);
    // BF16 RNE(W) transposed to [np][kp] (K-major B operand), zero padded;
    // prepare() converts W with the same rounding (common.cpp:99).
    std::vector<uint16_t> wt(size_t(p->np) * p->kp, 0);
    for (int k = 0; k < in; ++k)
        for (int c = 0; c < width; ++c) wt[size_t(c) * p->kp + k] = gat_b200_rne(w[size_t(k) * width + c]);
    // blr[k][h] = sum_d W[k][h*dim+d] aL[h*dim+d], blr[k][heads+h] likewise with aR
    // (common.cpp:100-108): one FMA chain in ascending d, as the reference's
    // FMA-contracted build evaluates it (the TFS path's lr_reordered input).
    std::vector<float> blr(size_t(in) * 2 * heads);
    for (int k = 0; k < in; ++k)
        for (int h = 0; h < heads; ++h) {
            float l = 0, r = 0;
            for (int d = 0; d < dim; ++d) {
                const float wv = w[size_t(k) * width + h * dim + d];
                l = std::fma(wv, al[h * dim + d], l);
                r = std::fma(wv, ar[h * dim + d], r);
            }
            blr[size_t(k) * 2 * heads + h] = l;
            blr[size_t(k) * 2 * heads + heads + h] = r;
        }
    int rc = 0;
    do {
        if ((rc = dmalloc((void**)&p->wt_bf16, wt.size() * 2))) break;
        if ((rc = dmalloc((void**)&p->w, nw * 4))) break;
        if ((rc = dmalloc((void**)&p->al, size_t(width) * 4))) break;
        if ((rc = dmalloc((void**)&p->ar, size_t(width) * 4))) break;
        if ((rc = dmalloc((void**)&p->blr, blr.size() * 4))) break;
        cudaError_t e;
        if ((e = cudaMemcpy(p->wt_bf16, wt.data(), wt.size() * 2, cudaMemcpyHostToDevice)) ||
            (e = cudaMemcpy(p->w, w, nw * 4, cudaMemcpyHostToDevice)) ||
            (e = cudaMemcpy(p->al, al, size_t(width) * 4, cudaMemcpyHostToDevice)) ||
            (e = cudaMemcpy(p->ar, ar, size_t(width) * 4, cudaMemcpyHostToDevice)) ||
            (e = cudaMemcpy(p->blr, blr.data(), blr.size() * 4, cudaMemcpyHostToDevice))) {
            rc = cuda_fail(e, "layer upload");
            break;
        }
    } while (0);
    if (rc) {
        gat_b200_layer_destroy(p);
        return rc;
    }
    *out = p;
    return 0;
}

int gat_b200_layer_destroy(gat_b200_layer* p) {
    if (!p) return 0;
    cudaFree(p->wt_bf16);
    cudaFree(p->w);
    cudaFree(p->al);
    cudaFree(p->ar);
    cudaFree(p->blr);
    delete p;
    return 0;
}

int gat_b200_convert(uint64_t n, int width, const float* in, int ld_in, uint16_t* out, int ld_out, void* stream) {
    clear_error();
    return convert_launch(n, width, in, ld_in, out, ld_out, as_stream(stream));
}

int gat_b200_projection(const gat_b200_layer* p, uint64_t n, const void* x, int ldx, int precision, void* h,
                        int h_dtype, int ldh, float* left, float* right, void* stream) {
    clear_error();
    return projection_dispatch(p, n, x, ldx, precision, h, h_dtype, ldh, left, right, as_stream(stream));
}

int gat_b200_projection_scatter(const gat_b200_layer* p, uint64_t n, const void* x, int ldx, void* h, int ldh,
                                float* left, float* right, int npeer, void* const* h_peer, float* const* r_peer,
                                void* stream) {
    clear_error();
    if (!p || !x || !h || !right) return fail("projection_scatter: null argument");
    if (ldx < p->in) return fail("projection_scatter: X row stride smaller than the input width");
    if (npeer < 0 || npeer > 7) return fail("projection_scatter: npeer must be 0..7");
    if (npeer && (!h_peer || !r_peer)) return fail("projection_scatter: null peer table");
    int rc = projection_tc_launch(p, n, static_cast<const uint16_t*>(x), ldx, static_cast<uint16_t*>(h), ldh,
                                  nullptr, 0, left, right, as_stream(stream), npeer,
                                  reinterpret_cast<uint16_t* const*>(h_peer), r_peer);
    if (rc == GAT_B200_EUNSUPPORTED)
        return fail_code(rc, "projection_scatter: layer outside the tensor-core kernel (input or width > 256)");
    return rc;
}

int gat_b200_edge_softmax(const gat_b200_graph* g, int heads, const float* left, const float* right, float* score,
                          float* max, float* p, float* den, float* alpha, void* stream) {
    clear_error();
    return edge_softmax_launch(g, heads, left, right, score, max, p, den, alpha, as_stream(stream));
}

int gat_b200_max_prescan(const gat_b200_graph* g, int heads, const float* left, const float* right, float* max,
                         void* stream) {
    clear_error();
    return max_prescan_launch(g, heads, left, right, max, as_stream(stream));
}

int gat_b200_standard_aggregate(const gat_b200_graph* g, int heads, int dim, const void* h, int h_dtype, int ldh,
                                const float* left, const float* right, const float* fixed_p,
                                const float* fixed_den, float* out, int ldo, float* den, float* max,
                                void* stream) {
    clear_error();
    return aggregate_dispatch(g, heads, dim, h, h_dtype, ldh, left, right, fixed_p, fixed_den, 1, 0, out, 0, ldo,
                              den, max, as_stream(stream));
}

int gat_b200_finish(uint64_t n, int heads, int dim, const float* den, int hidden, float* out, int ldo,
                    void* stream) {
    clear_error();
    return finish_launch(n, heads, dim, den, hidden, out, ldo, as_stream(stream));
}

int gat_b200_aggregate_fused(const gat_b200_graph* g, int heads, int dim, const void* h, int h_dtype, int ldh,
                             const float* left, const float* right, int hidden, void* out, int out_dtype, int ldo,
                             void* stream) {
    clear_error();
    if (out_dtype != GAT_B200_BF16 && out_dtype != GAT_B200_F32) return fail("aggregate_fused: bad output dtype");
    return aggregate_dispatch(g, heads, dim, h, h_dtype, ldh, left, right, nullptr, nullptr, 0, hidden, out,
                              out_dtype == GAT_B200_BF16, ldo, nullptr, nullptr, as_stream(stream));
}

int gat_b200_standard_layer(const gat_b200_graph* g, const gat_b200_layer* p, const void* x, int ldx, int path,
                            int hidden, void* h, float* left, float* right, void* out, int out_dtype, int ldo,
                            void* stream) {
    clear_error();
    if (!g || !p) return fail("standard_layer: null handle");
    cudaStream_t st = as_stream(stream);
    const int hd = path == GAT_B200_PATH_STANDARD_BF16 ? GAT_B200_BF16 : GAT_B200_F32;
    if (path != GAT_B200_PATH_STANDARD_BF16 && path != GAT_B200_PATH_STANDARD_FP32)
        return fail("standard_layer: bad path");
    if (out_dtype != GAT_B200_BF16 && out_dtype != GAT_B200_F32) return fail("standard_layer: bad output dtype");
    const int ldh = gat_b200_padded_ld(p->width, hd);
    int rc = projection_dispatch(p, g->n, x, ldx, hd, h, hd, ldh, left, right, st);
    if (rc) return rc;
    return aggregate_dispatch(g, p->heads, p->dim, h, hd, ldh, left, right, nullptr, nullptr, 0, hidden, out,
                              out_dtype == GAT_B200_BF16, ldo, nullptr, nullptr, st);
}

int gat_b200_device_count(int* count) {
    clear_error();
    if (!count) return fail("device_count: null output");
    *count = 0;
    GATB_CUDA(cudaGetDeviceCount(count));
    return 0;
}

int gat_b200_set_device(int device) {
    clear_error();
    GATB_CUDA(cudaSetDevice(device));
    return 0;
}

int gat_b200_check_device(void) {
    clear_error();
    return device_check_errors();
}

int gat_b200_model_create(const gat_b200_graph* g, const gat_b200_layer* const* layers, int path,
                          gat_b200_model** out) {
    clear_error();
    if (!out) return fail("model_create: null output handle");
    *out = nullptr;
    if (!g || !layers || !layers[0] || !layers[1] || !layers[2]) return fail("model_create: null handle");
    if (path < GAT_B200_PATH_STANDARD_BF16 || path > GAT_B200_PATH_MATCHED_ATTENTION)
        return fail("model_create: bad path");
    for (int l = 0; l < 2; ++l)
        if (layers[l + 1]->in != layers[l]->width) return fail("model_create: layer widths do not chain");
    gat_b200_model* m = new (std::nothrow) gat_b200_model();
    if (!m) return fail("model_create: out of host memory");
    m->g = g;
    for (int l = 0; l < 3; ++l) m->layers[l] = layers[l];
    m->path = path;
    m->din = layers[0]->in;
    m->classes = layers[2]->width;
    const uint64_t n = g->n;
    const int hd = path == GAT_B200_PATH_STANDARD_FP32 ? GAT_B200_F32 : GAT_B200_BF16;
    const int es = hd == GAT_B200_BF16 ? 2 : 4;
    const bool tfs = path == GAT_B200_PATH_TFS_BF16 || path == GAT_B200_PATH_ADAPTIVE_BF16;
    int wmax = 0;
    for (int l = 0; l < 3; ++l) wmax = std::max(wmax, layers[l]->width);
    m->ld0 = gat_b200_padded_ld(m->din, hd);
    m->ld_hidden = gat_b200_padded_ld(std::max(layers[0]->width, layers[1]->width), hd);
    const int ldh = gat_b200_padded_ld(wmax, hd);
    int rc = 0;
    do {
        if ((rc = dmalloc((void**)&m->x_f32, n * size_t(m->din) * 4))) break;
        if (hd == GAT_B200_BF16 && (rc = dmalloc(&m->x0, n * size_t(m->ld0) * es))) break;
        if ((rc = dmalloc(&m->h, n * size_t(ldh) * es))) break;
        if ((rc = dmalloc((void**)&m->left, n * 8 * 4))) break;
        if ((rc = dmalloc((void**)&m->right, n * 8 * 4))) break;
        if ((rc = dmalloc(&m->x1, n * size_t(m->ld_hidden) * es))) break;
        if ((rc = dmalloc(&m->x2, n * size_t(m->ld_hidden) * es))) break;
        if ((rc = dmalloc((void**)&m->logits, n * size_t(m->classes) * 4))) break;
        if (tfs && (rc = dmalloc((void**)&m->max, n * 8 * 4))) break;
        // Padding columns of every feature buffer start (and stay) zero.
        cudaError_t e;
        if ((e = cudaMemset(m->h, 0, n * size_t(ldh) * es)) ||
            (e = cudaMemset(m->x1, 0, n * size_t(m->ld_hidden) * es)) ||
            (e = cudaMemset(m->x2, 0, n * size_t(m->ld_hidden) * es)) ||
            (m->x0 && (e = cudaMemset(m->x0, 0, n * size_t(m->ld0) * es)))) {
            rc = cuda_fail(e, "model buffers");
            break;
        }
    } while (0);
    if (rc) {
        gat_b200_model_destroy(m);
        return rc;
    }
    *out = m;
    return 0;
}

int gat_b200_model_destroy(gat_b200_model* m) {
    if (!m) return 0;
    for (cudaEvent_t e : m->events) cudaEventDestroy(e);
    cudaFree(m->x_f32);
    cudaFree(m->x0);
    cudaFree(m->h);
    cudaFree(m->left);
    cudaFree(m->right);
    cudaFree(m->x1);
    cudaFree(m->x2);
    cudaFree(m->logits);
    cudaFree(m->max);
    for (int b = 0; b < 2; ++b) {
        cudaFree(m->ax[b]);
        cudaFree(m->alog[b]);
        if (m->ev_up[b]) cudaEventDestroy(m->ev_up[b]);
        if (m->ev_done[b]) cudaEventDestroy(m->ev_done[b]);
        if (m->ev_down[b]) cudaEventDestroy(m->ev_down[b]);
    }
    if (m->up) cudaStreamDestroy(m->up);
    if (m->down) cudaStreamDestroy(m->down);
    delete m;
    return 0;
}

int gat_b200_model_forward(gat_b200_model* m, const float* x, int x_on_host, float* logits, int logits_on_host,
                           void* stream) {
    clear_error();
    if (!m || !x || !logits) return fail("model_forward: null argument");
    cudaStream_t st = as_stream(stream);
    const uint64_t n = m->g->n;
    const float* xin = x;
    int launches = 0;
    mark(m, 0, st);
    if (x_on_host) {
        GATB_CUDA(cudaMemcpyAsync(m->x_f32, x, n * size_t(m->din) * 4, cudaMemcpyHostToDevice, st));
        xin = m->x_f32;
    }
    mark(m, 1, st);
    const bool bf16 = m->path != GAT_B200_PATH_STANDARD_FP32;
    const int hd = bf16 ? GAT_B200_BF16 : GAT_B200_F32;
    const void* lin = xin;
    int ldin = m->din;
    int rc;
    // Layer l runs TFS (lr_reordered + max_prescan, then TFS aggregation with
    // finish fused) on the TFS path, and on layer 1 of the adaptive path.
    auto tfs_layer = [&](int l) {
        return m->path == GAT_B200_PATH_TFS_BF16 || (m->path == GAT_B200_PATH_ADAPTIVE_BF16 && l == 0);
    };
    if (bf16 && !tfs_layer(0)) {
        // Layer-1 input conversion (standard_layer's convert, baseline_standard.cpp:127).
        if ((rc = convert_launch(n, m->din, xin, m->din, static_cast<uint16_t*>(m->x0), m->ld0, st))) return rc;
        ++launches;
        lin = m->x0;
        ldin = m->ld0;
    }
    void* outs[2] = {m->x1, m->x2};
    for (int l = 0; l < 3; ++l) {
        const gat_b200_layer* p = m->layers[l];
        const bool last = l == 2;
        float* dst_logits = (last && !logits_on_host) ? logits : m->logits;
        void* dst = last ? static_cast<void*>(dst_logits) : outs[l];
        const int ldo = last ? p->width : m->ld_hidden;
        mark(m, 2 + 2 * l, st);
        if (tfs_layer(l)) {
            // baseline_tfs.cpp:111-117: convert + lr_reordered ("bf16" policy), max_prescan
            if (l == 0) {
                if ((rc = lr_reordered_launch(p, n, lin, GAT_B200_F32, ldin, GAT_B200_LR_BF16,
                                              static_cast<uint16_t*>(m->x0), m->ld0, m->left, m->right, st)))
                    return rc;
                lin = m->x0;
                ldin = m->ld0;
            } else if ((rc = lr_reordered_launch(p, n, lin, GAT_B200_BF16, ldin, GAT_B200_LR_BF16, nullptr, 0,
                                                  m->left, m->right, st))) {
                return rc;
            }
            if ((rc = max_prescan_launch(m->g, p->heads, m->left, m->right, m->max, st))) return rc;
            launches += 2;
            mark(m, 3 + 2 * l, st);
            // The TFS path keeps the reference's B1 rounding (per neighbour); the
            // adaptive path takes heads_hybrid's high/low rounding, one block per row.
            const int rounding = m->path == GAT_B200_PATH_TFS_BF16 ? GAT_B200_TFS_EDGE : GAT_B200_TFS_SPLIT;
            int k = 0;
            if ((rc = tfs_dispatch(m->g, p, lin, ldin, m->left, m->right, m->max, nullptr, nullptr, rounding, 0, 1, 1,
                                   last ? 0 : 1, dst, last ? 0 : 1, ldo, nullptr, nullptr, st, &k)))
                return rc;
            launches += k;
        } else {
            const int ldh = gat_b200_padded_ld(p->width, hd);
            if ((rc = projection_dispatch(p, n, lin, ldin, hd, m->h, hd, ldh, m->left, m->right, st))) return rc;
            if (m->path == GAT_B200_PATH_MATCHED_ATTENTION) {
                // L/R from the BF16 layer input and W.a (lr_reordered, "bf16" policy)
                if ((rc = lr_reordered_launch(p, n, lin, GAT_B200_BF16, ldin, GAT_B200_LR_BF16, nullptr, 0, m->left,
                                              m->right, st)))
                    return rc;
                ++launches;
            }
            mark(m, 3 + 2 * l, st);
            if ((rc = aggregate_dispatch(m->g, p->heads, p->dim, m->h, hd, ldh, m->left, m->right, nullptr, nullptr,
                                         0, last ? 0 : 1, dst, (!last && bf16) ? 1 : 0, ldo, nullptr, nullptr, st)))
                return rc;
            launches += 2 + (m->g->n_hub ? 1 : 0);
        }
        lin = dst;
        ldin = ldo;
    }
    mark(m, 8, st);
    if (logits_on_host)
        GATB_CUDA(cudaMemcpyAsync(logits, m->logits, n * size_t(m->classes) * 4, cudaMemcpyDeviceToHost, st));
    mark(m, 9, st);
    m->launches_last = launches;
    ++m->forwards;
    if (logits_on_host) {
        GATB_CUDA(cudaStreamSynchronize(st));
        return device_check_errors();
    }
    return 0;
}

int gat_b200_model_enable_timing(gat_b200_model* m, int steps) {
    clear_error();
    if (!m || steps < 0) return fail("model_enable_timing: bad argument");
    for (cudaEvent_t e : m->events) cudaEventDestroy(e);
    m->events.assign(size_t(steps) * kStageEvents, nullptr);
    for (auto& e : m->events) GATB_CUDA(cudaEventCreate(&e));
    m->timing_steps = steps;
    m->forwards = 0;
    return 0;
}

int gat_b200_model_stage_times(gat_b200_model* m, float* ms) {
    clear_error();
    if (!m || !ms) return fail("model_stage_times: bad argument");
    const int sets = int(std::min<uint64_t>(m->forwards, uint64_t(m->timing_steps)));
    for (int s = 0; s < sets; ++s)
        for (int k = 0; k < kStages; ++k) {
            GATB_CUDA(cudaEventSynchronize(m->events[size_t(s) * kStageEvents + k + 1]));
            float t = 0;
            GATB_CUDA(cudaEventElapsedTime(&t, m->events[size_t(s) * kStageEvents + k],
                                           m->events[size_t(s) * kStageEvents + k + 1]));
            ms[s * kStages + k] = t;
        }
    return sets;
}

int gat_b200_model_launches(const gat_b200_model* m) { return m ? m->launches_last : 0; }

int gat_b200_model_forward_async(gat_b200_model* m, const float* x, float* logits, void* stream) {
    clear_error();
    if (!m || !x || !logits) return fail("model_forward_async: null argument");
    cudaStream_t st = as_stream(stream);
    const uint64_t n = m->g->n;
    const size_t xb = n * size_t(m->din) * 4, lb = n * size_t(m->classes) * 4;
    if (!m->up) {
        for (int b = 0; b < 2; ++b) {
            int rc;
            if ((rc = dmalloc((void**)&m->ax[b], xb)) || (rc = dmalloc((void**)&m->alog[b], lb))) return rc;
            GATB_CUDA(cudaEventCreateWithFlags(&m->ev_up[b], cudaEventDisableTiming));
            GATB_CUDA(cudaEventCreateWithFlags(&m->ev_done[b], cudaEventDisableTiming));
            GATB_CUDA(cudaEventCreateWithFlags(&m->ev_down[b], cudaEventDisableTiming));
        }
        GATB_CUDA(cudaStreamCreateWithFlags(&m->up, cudaStreamNonBlocking));
        GATB_CUDA(cudaStreamCreateWithFlags(&m->down, cudaStreamNonBlocking));
    }
    const int b = int(m->submitted & 1);
    // upload once the forward that last read this slot is done
    if (m->submitted >= 2) GATB_CUDA(cudaStreamWaitEvent(m->up, m->ev_done[b], 0));
    GATB_CUDA(cudaMemcpyAsync(m->ax[b], x, xb, cudaMemcpyHostToDevice, m->up));
    GATB_CUDA(cudaEventRecord(m->ev_up[b], m->up));
    // compute once the input is in and the slot's previous logits are downloaded
    GATB_CUDA(cudaStreamWaitEvent(st, m->ev_up[b], 0));
    if (m->submitted >= 2) GATB_CUDA(cudaStreamWaitEvent(st, m->ev_down[b], 0));
    int rc = gat_b200_model_forward(m, m->ax[b], 0, m->alog[b], 0, stream);
    if (rc) return rc;
    GATB_CUDA(cudaEventRecord(m->ev_done[b], st));
    GATB_CUDA(cudaStreamWaitEvent(m->down, m->ev_done[b], 0));
    GATB_CUDA(cudaMemcpyAsync(logits, m->alog[b], lb, cudaMemcpyDeviceToHost, m->down));
    GATB_CUDA(cudaEventRecord(m->ev_down[b], m->down));
    ++m->submitted;
    return 0;
}

int gat_b200_model_join(gat_b200_model* m, void* stream) {
    clear_error();
    if (!m) return fail("model_join: null argument");
    if (!m->submitted) return 0;
    const int b = int((m->submitted - 1) & 1);
    GATB_CUDA(cudaStreamWaitEvent(as_stream(stream), m->ev_down[b], 0));
    return 0;
}

}  // extern "C"
