// Host-side C-ABI entry points of libgat_b200.so: error reporting, BF16 RNE,
// CSR validation, GATBIN1/GATWGT1 files, the reference's seeded random model
// and the synthetic-input generators. No GPU is touched here.
#include "gat_b200_internal.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <fstream>
#include <limits>
#include <vector>

namespace gatb {
namespace {
thread_local std::string g_last_error;
}
int fail(const std::string& msg) { return fail_code(GAT_B200_EINVAL, msg); }
int fail_code(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}
void clear_error() { g_last_error.clear(); }
const char* last_error() { return g_last_error.c_str(); }

namespace {
template <class T>
bool read_n(std::ifstream& f, T* data, uint64_t n) {
    if (n > uint64_t(std::numeric_limits<std::streamsize>::max()) / sizeof(T)) return false;
    f.read(reinterpret_cast<char*>(data), std::streamsize(n * sizeof(T)));
    return bool(f);
}
template <class T>
bool write_n(std::ofstream& f, const T* data, uint64_t n) {
    f.write(reinterpret_cast<const char*>(data), std::streamsize(n * sizeof(T)));
    return bool(f);
}
// Layer shapes of the reference's fixed model (baseline/src/common.cpp:53).
void layer_shape(int l, int din, int classes, int* in, int* heads, int* dim) {
    *in = l ? 256 : din;
    *heads = l < 2 ? 8 : 1;
    *dim = l < 2 ? 32 : classes;
}
}  // namespace
}  // namespace gatb

using namespace gatb;

extern "C" {

const char* gat_b200_last_error(void) { return gatb::last_error(); }
int gat_b200_version(void) { return 100; }
int gat_b200_padded_ld(int width, int elem_dtype) {
    return gatb::padded_ld(width, elem_dtype == GAT_B200_BF16 ? 2 : 4);
}

uint16_t gat_b200_rne(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) return uint16_t((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return uint16_t(u >> 16);
}

int gat_b200_convert_host(const float* in, uint16_t* out, uint64_t count) {
    if (!in || !out) return fail("convert_host: null pointer");
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)count; ++i) out[i] = gat_b200_rne(in[i]);
    return 0;
}

int gat_b200_validate_csr(uint64_t n, uint64_t e, const uint64_t* row, const uint32_t* col) {
    if (!n || n > uint64_t(INT32_MAX)) return fail("invalid graph sizes");
    if (!row || (e && !col)) return fail("invalid graph sizes");
    if (row[0] != 0 || row[n] != e) return fail("bad CSR bounds");
    for (uint64_t i = 0; i < n; ++i)
        if (row[i] > row[i + 1]) return fail("nonmonotone CSR");
    for (uint64_t k = 0; k < e; ++k)
        if (col[k] >= n) return fail("source index out of bounds");
    return 0;
}

int gat_b200_read_graph_header(const char* path, uint64_t* n, uint64_t* e, uint32_t* din,
                               uint32_t* classes) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return fail_code(GAT_B200_EIO, "cannot open graph");
    char magic[8];
    if (!read_n(f, magic, 8)) return fail_code(GAT_B200_EIO, "truncated file");
    if (std::memcmp(magic, "GATBIN1", 7)) return fail("bad graph magic");
    uint64_t nn, ee;
    uint32_t d, c;
    if (!read_n(f, &nn, 1) || !read_n(f, &ee, 1) || !read_n(f, &d, 1) || !read_n(f, &c, 1))
        return fail_code(GAT_B200_EIO, "truncated file");
    if (!nn || nn > uint64_t(INT32_MAX) || d > uint32_t(INT32_MAX) || c > uint32_t(INT32_MAX) || !d || !c)
        return fail("bad graph dimensions");
    *n = nn;
    *e = ee;
    *din = d;
    *classes = c;
    return 0;
}

int gat_b200_read_graph(const char* path, uint64_t n, uint64_t e, uint32_t din, uint64_t* row,
                        uint32_t* col, float* x) {
    uint64_t nn, ee;
    uint32_t d, c;
    int rc = gat_b200_read_graph_header(path, &nn, &ee, &d, &c);
    if (rc) return rc;
    if (nn != n || ee != e || d != din) return fail("graph header does not match the buffers");
    std::ifstream f(path, std::ios::binary);
    f.seekg(32);
    if (!read_n(f, row, n + 1) || !read_n(f, col, e) || !read_n(f, x, n * uint64_t(din)))
        return fail_code(GAT_B200_EIO, "truncated file");
    rc = gat_b200_validate_csr(n, e, row, col);
    if (rc) return rc;
    for (uint64_t i = 0; i < n * uint64_t(din); ++i)
        if (!std::isfinite(x[i])) return fail("nonfinite graph input index=" + std::to_string(i));
    return 0;
}

int gat_b200_write_graph(const char* path, uint64_t n, uint64_t e, uint32_t din, uint32_t classes,
                         const uint64_t* row, const uint32_t* col, const float* x) {
    int rc = gat_b200_validate_csr(n, e, row, col);
    if (rc) return rc;
    std::ofstream f(path, std::ios::binary);
    const char magic[8] = "GATBIN1";
    if (!f || !write_n(f, magic, 8) || !write_n(f, &n, 1) || !write_n(f, &e, 1) || !write_n(f, &din, 1) ||
        !write_n(f, &classes, 1) || !write_n(f, row, n + 1) || !write_n(f, col, e) ||
        !write_n(f, x, n * uint64_t(din)))
        return fail_code(GAT_B200_EIO, "write failed");
    return 0;
}

int gat_b200_read_weights(const char* path, int din, int classes, float* const* w, float* const* al,
                          float* const* ar) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return fail_code(GAT_B200_EIO, "cannot open weights");
    char magic[8];
    uint32_t count;
    if (!read_n(f, magic, 8)) return fail_code(GAT_B200_EIO, "truncated file");
    if (std::memcmp(magic, "GATWGT1", 7)) return fail("bad weights magic");
    if (!read_n(f, &count, 1)) return fail_code(GAT_B200_EIO, "truncated file");
    if (count != 3) return fail("model must have 3 layers");
    for (int l = 0; l < 3; ++l) {
        uint32_t s[3];
        int in, heads, dim;
        layer_shape(l, din, classes, &in, &heads, &dim);
        if (!read_n(f, s, 3)) return fail_code(GAT_B200_EIO, "truncated file");
        if (s[0] != uint32_t(in) || s[1] != uint32_t(heads) || s[2] != uint32_t(dim))
            return fail("checkpoint model shape mismatch");
        uint64_t width = uint64_t(heads) * dim;
        if (!read_n(f, w[l], uint64_t(in) * width) || !read_n(f, al[l], width) || !read_n(f, ar[l], width))
            return fail_code(GAT_B200_EIO, "truncated file");
        for (uint64_t i = 0; i < uint64_t(in) * width; ++i)
            if (!std::isfinite(w[l][i])) return fail("nonfinite W");
        for (uint64_t i = 0; i < width; ++i)
            if (!std::isfinite(al[l][i]) || !std::isfinite(ar[l][i])) return fail("nonfinite aL/aR");
    }
    return 0;
}

int gat_b200_write_weights(const char* path, int din, int classes, const float* const* w,
                           const float* const* al, const float* const* ar) {
    std::ofstream f(path, std::ios::binary);
    const char magic[8] = "GATWGT1";
    uint32_t count = 3;
    if (!f || !write_n(f, magic, 8) || !write_n(f, &count, 1)) return fail_code(GAT_B200_EIO, "write failed");
    for (int l = 0; l < 3; ++l) {
        int in, heads, dim;
        layer_shape(l, din, classes, &in, &heads, &dim);
        uint32_t s[3] = {uint32_t(in), uint32_t(heads), uint32_t(dim)};
        uint64_t width = uint64_t(heads) * dim;
        if (!write_n(f, s, 3) || !write_n(f, w[l], uint64_t(in) * width) || !write_n(f, al[l], width) ||
            !write_n(f, ar[l], width))
            return fail_code(GAT_B200_EIO, "write failed");
    }
    return 0;
}

int gat_b200_synth_uniform_graph(uint64_t n, uint32_t sources, uint64_t seed, uint64_t* row, uint32_t* col) {
    if (!row || !col) return fail("synth: null pointer");
    return synth_uniform_graph(n, sources, seed, row, col);
}
int gat_b200_synth_powerlaw_graph(uint64_t n, uint64_t e, uint64_t max_degree, double gamma, uint64_t seed,
                                  uint64_t* row, uint32_t* col) {
    if (!row || !col) return fail("synth: null pointer");
    return synth_powerlaw_graph(n, e, max_degree, gamma, seed, row, col);
}
int gat_b200_synth_normal(uint64_t count, double scale, uint64_t seed, uint64_t stream, float* out) {
    if (!out) return fail("synth: null pointer");
    return synth_normal(count, scale, seed, stream, out, 0);
}
int gat_b200_synth_normal_range(uint64_t offset, uint64_t count, double scale, uint64_t seed, uint64_t stream,
                                float* out) {
    if (!out) return fail("synth: null pointer");
    return synth_normal(count, scale, seed, stream, out, offset);
}
int gat_b200_synth_powerlaw_rows(uint64_t n, uint64_t e, uint64_t max_degree, double gamma, uint64_t seed,
                                 uint64_t r_lo, uint64_t r_hi, uint64_t* row, uint32_t* col) {
    if (!row) return fail("synth: null pointer");
    return synth_powerlaw_rows(n, e, max_degree, gamma, seed, r_lo, r_hi, row, col);
}
int gat_b200_synth_uniform(uint64_t count, double lo, double hi, uint64_t seed, uint64_t stream, float* out) {
    if (!out) return fail("synth: null pointer");
    return synth_uniform(count, lo, hi, seed, stream, out);
}

// GATFIX1 fixed-p fixture (baseline/src/common.cpp:171-194): magic, u64
// {n, e, in, heads, dim}, the CSR (to reject a different graph of equal shape),
// the layer's W/aL/aR (checkpoint), the layer input [n][in], p [e][heads] and
// den [n][heads].
int gat_b200_write_fixture(const char* path, uint64_t n, uint64_t e, int in, int heads, int dim,
                           const uint64_t* row, const uint32_t* col, const float* w, const float* al,
                           const float* ar, const float* input, const float* p, const float* den) {
    clear_error();
    if (!path || !row || !col || !w || !al || !ar || !input || !p || !den) return fail("write_fixture: null argument");
    if (in <= 0 || heads <= 0 || dim <= 0) return fail("bad fixture sizes");
    std::ofstream f(path, std::ios::binary);
    const char magic[8] = "GATFIX1";
    const uint64_t sizes[5] = {n, e, uint64_t(in), uint64_t(heads), uint64_t(dim)};
    const uint64_t width = uint64_t(heads) * dim;
    if (!f || !write_n(f, magic, 8) || !write_n(f, sizes, 5) || !write_n(f, row, n + 1) || !write_n(f, col, e) ||
        !write_n(f, w, uint64_t(in) * width) || !write_n(f, al, width) || !write_n(f, ar, width) ||
        !write_n(f, input, n * uint64_t(in)) || !write_n(f, p, e * uint64_t(heads)) ||
        !write_n(f, den, n * uint64_t(heads)))
        return fail_code(GAT_B200_EIO, "write failed");
    return 0;
}

int gat_b200_read_fixture(const char* path, uint64_t n, uint64_t e, int in, int heads, int dim,
                          const uint64_t* row, const uint32_t* col, const float* w, const float* al,
                          const float* ar, float* input, float* p, float* den) {
    clear_error();
    if (!path || !row || !col || !w || !al || !ar || !input || !p || !den) return fail("read_fixture: null argument");
    std::ifstream f(path, std::ios::binary);
    if (!f) return fail_code(GAT_B200_EIO, "cannot open fixture");
    char magic[8];
    if (!read_n(f, magic, 8)) return fail_code(GAT_B200_EIO, "truncated file");
    if (std::memcmp(magic, "GATFIX1", 7)) return fail("bad fixture magic");
    uint64_t s[5];
    if (!read_n(f, s, 5)) return fail_code(GAT_B200_EIO, "truncated file");
    if (s[0] != n || s[1] != e || s[2] != uint64_t(in) || s[3] != uint64_t(heads) || s[4] != uint64_t(dim))
        return fail("fixture shape mismatch");
    const uint64_t width = uint64_t(heads) * dim;
    std::vector<uint64_t> frow(n + 1);
    std::vector<uint32_t> fcol(e);
    if (!read_n(f, frow.data(), n + 1) || !read_n(f, fcol.data(), e)) return fail_code(GAT_B200_EIO, "truncated file");
    if (std::memcmp(frow.data(), row, (n + 1) * 8) || (e && std::memcmp(fcol.data(), col, e * 4)))
        return fail("fixture CSR mismatch");
    const float* masters[3] = {w, al, ar};
    const uint64_t counts[3] = {uint64_t(in) * width, width, width};
    for (int k = 0; k < 3; ++k) {
        std::vector<float> v(counts[k]);
        if (!read_n(f, v.data(), counts[k])) return fail_code(GAT_B200_EIO, "truncated file");
        if (std::memcmp(v.data(), masters[k], counts[k] * 4)) return fail("fixture checkpoint mismatch");
    }
    if (!read_n(f, input, n * uint64_t(in)) || !read_n(f, p, e * uint64_t(heads)) || !read_n(f, den, n * uint64_t(heads)))
        return fail_code(GAT_B200_EIO, "truncated file");
    for (uint64_t i = 0; i < n * uint64_t(in); ++i)
        if (!std::isfinite(input[i])) return fail("nonfinite fixture input index=" + std::to_string(i));
    for (uint64_t i = 0; i < e * uint64_t(heads); ++i)
        if (!std::isfinite(p[i])) return fail("nonfinite fixture p index=" + std::to_string(i));
    for (uint64_t i = 0; i < n * uint64_t(heads); ++i)
        if (!std::isfinite(den[i])) return fail("nonfinite fixture denominator index=" + std::to_string(i));
    for (uint64_t i = 0; i < n; ++i)
        for (int h = 0; h < heads; ++h) {
            float sum = 0.f;
            for (uint64_t k = row[i]; k < row[i + 1]; ++k) {
                const float x = p[k * heads + h];
                if (x < 0.f || x > 1.f) return fail("fixture p outside [0,1]");
                sum += x;
            }
            const float d = den[i * heads + h];
            if (std::fabs(sum - d) > 1e-5f * std::max(1.f, sum) || (row[i] != row[i + 1] && d <= 0.f))
                return fail("fixture denominator mismatch");
        }
    return 0;
}

}  // extern "C"
