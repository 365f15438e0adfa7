// Aggregation entry point that allocates no memory (gat_b200_aggregate_fused_noalloc).
//
// Some callers cannot allocate device memory on their own: a plugin running
// inside another framework whose caching allocator owns all of the GPU's
// memory, a real-time or serving loop where cudaMalloc would synchronize the
// device and stall every other stream, or a host binding that has no access
// to the framework's allocator at all. The regular entry points need a
// gat_b200_graph handle, whose creation allocates the degree schedule and the
// scratch of the hub-row segments. This variant takes the caller's device CSR
// directly and keeps its scratch in a file-scope __device__ array instead.
//
// Work split: the edge list is cut into W equal ranges of SEG edges (natural
// row order, balanced by edge count, no schedule to build). One warp handles
// one range: rows inside it are finished and written; a row that crosses a
// range boundary leaves a partial state (running max, sum, weighted sum) per
// range in the scratch array, and a second kernel merges those per row.
//
// The scratch array is shared by every call in the process: calls whose
// kernels overlap on the GPU (different streams, or several host threads)
// race on it and must be serialized by the caller. Nothing in it needs to start
// at zero: every slot a merge reads was written by the same call.
#include "device.cuh"
#include "graph.cuh"

namespace gatb {
namespace {

constexpr int kSlotFloats = kSegStateFloats;           // 16 + 512 floats per partial state
constexpr uint64_t kMaxRanges = 7936;                   // 2 slots each
constexpr uint64_t kScratchFloats = kMaxRanges * 2 * kSlotFloats;  // 8,380,416 floats = 31.97 MiB
constexpr uint64_t kMaxSeg = 65536;                     // edges per range
constexpr uint64_t kMinSeg = 1024;

// The scratch: every GPU that loads the library holds it until exit.
static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

struct NaArgs {
    const uint64_t* row;
    const uint32_t* col;
    uint64_t n, e, seg;
    uint32_t ranges;
    int heads, dim, width;
    const void* h;
    int ldh;
    const float* left;
    const float* right;
    int hidden;
    void* out;
    int out_bf16;
    int ldo;
    float* scratch;
};

// First index r in [0, n] with row[r] >= x (row is non-decreasing).
__device__ __forceinline__ uint64_t lower_bound_rows(const uint64_t* row, uint64_t n, uint64_t x) {
    uint64_t lo = 0, hi = n + 1;
    while (lo < hi) {
        uint64_t mid = (lo + hi) / 2;
        if (row[mid] < x) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// Normalisation and, for hidden layers, ELU as exp(v) - 1: the activation of
// the reference's B0 finish (baseline/include/gat.hpp:57-62), which the
// regular fused kernel also uses.
__device__ __forceinline__ float na_finalize(const NaArgs& a, int c, float acc, float den) {
    if (c >= a.width) return 0.f;
    float v = acc * (den > 0.f ? 1.f / den : 0.f);
    return (a.hidden && v < 0.f) ? __expf(v) - 1.f : v;
}

__device__ __forceinline__ void na_store(const NaArgs& a, uint64_t r, int c, float v) {
    if (a.out_bf16)
        static_cast<uint16_t*>(a.out)[r * a.ldo + c] = uint16_t(pack_bf16x2(v, 0.f) & 0xffffu);
    else
        static_cast<float*>(a.out)[r * a.ldo + c] = v;
}

// One warp: edges [b, e) of row r. Online softmax over chunks of 32 edges,
// lane = edge for the scores, lanes stride over the row's 16-byte vectors for
// the weighted sum. VEC elements per vector, up to NVP vectors per lane.
template <class HT, int VEC, int NVP>
__device__ void na_part(const NaArgs& a, uint64_t r, uint64_t b, uint64_t e, float* sp, float (&m)[8],
                        float (&den)[8], float (&acc)[NVP][VEC]) {
    const int lane = threadIdx.x & 31;
    const int K = a.heads;
    const int nvec = (a.width + VEC - 1) / VEC;
    float L[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) {
        L[h] = h < K ? a.left[r * K + h] : 0.f;
        m[h] = -INFINITY;
        den[h] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < NVP; ++j)
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[j][k] = 0.f;
    const HT* H = static_cast<const HT*>(a.h);
    for (uint64_t c0 = b; c0 < e; c0 += 32) {
        const int cnt = int(e - c0 < 32 ? e - c0 : 32);
        const uint32_t src = lane < cnt ? a.col[c0 + lane] : 0u;
        float s[8];
#pragma unroll
        for (int h = 0; h < 8; ++h)
            s[h] = (lane < cnt && h < K) ? leaky(L[h] + a.right[uint64_t(src) * K + h]) : -INFINITY;
        float sc[8];
#pragma unroll
        for (int h = 0; h < 8; ++h) {
            const float nm = fmaxf(m[h], warp_max(s[h]));
            const float nms = nm == -INFINITY ? 0.f : nm;
            sc[h] = __expf(m[h] - nms);
            m[h] = nm;
            const float p = __expf(s[h] - nms);
            den[h] = den[h] * sc[h] + warp_sum(p);
            sp[lane * 8 + h] = p;
        }
        sp[256 + lane] = __uint_as_float(src);
        __syncwarp();
#pragma unroll
        for (int j = 0; j < NVP; ++j)
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
                const int c = (lane + 32 * j) * VEC + k;
                float f = sc[0];
#pragma unroll
                for (int h = 1; h < 8; ++h) f = (c / a.dim == h) ? sc[h] : f;
                acc[j][k] *= f;
            }
        for (int t = 0; t < cnt; ++t) {
            const uint32_t st = __float_as_uint(sp[256 + t]);
#pragma unroll
            for (int j = 0; j < NVP; ++j) {
                const int v = lane + 32 * j;
                if (v >= nvec) continue;
                float f[VEC];
                const uint4 raw = ldg_nc_v4(H + uint64_t(st) * a.ldh + v * VEC);
                if constexpr (VEC == 8) {
                    f[0] = bf16lo(raw.x); f[1] = bf16hi(raw.x); f[2] = bf16lo(raw.y); f[3] = bf16hi(raw.y);
                    f[4] = bf16lo(raw.z); f[5] = bf16hi(raw.z); f[6] = bf16lo(raw.w); f[7] = bf16hi(raw.w);
                } else {
                    f[0] = __uint_as_float(raw.x); f[1] = __uint_as_float(raw.y);
                    f[2] = __uint_as_float(raw.z); f[3] = __uint_as_float(raw.w);
                }
#pragma unroll
                for (int k = 0; k < VEC; ++k) {
                    const int c = v * VEC + k;
                    const int hh = min(c / a.dim, K - 1);
                    acc[j][k] = fmaf(sp[t * 8 + hh], f[k], acc[j][k]);
                }
            }
        }
        __syncwarp();
    }
}

template <class HT, int VEC, int NVP>
__global__ void __launch_bounds__(128) na_range_kernel(const NaArgs a) {
    __shared__ float s_p[4][288];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    float* sp = s_p[wib];
    const uint64_t G = uint64_t(gridDim.x) * 4;
    for (uint64_t w = blockIdx.x * 4ull + wib; w < a.ranges; w += G) {
        const uint64_t lo = w * a.seg;
        const uint64_t hi = lo + a.seg < a.e ? lo + a.seg : a.e;
        const bool last = w + 1 == a.ranges;
        const uint64_t r0 = lower_bound_rows(a.row, a.n, lo);
        float m[8] = {}, den[8] = {}, acc[NVP][VEC] = {};
        auto emit = [&](uint64_t r, bool partial, int side) {
            if (partial) {
                float* st = a.scratch + (2 * w + side) * kSlotFloats;
                if (lane < 8) {
                    float mv = m[0], dv = den[0];
#pragma unroll
                    for (int h = 1; h < 8; ++h) {
                        mv = lane == h ? m[h] : mv;
                        dv = lane == h ? den[h] : dv;
                    }
                    st[lane] = mv;
                    st[8 + lane] = dv;
                }
#pragma unroll
                for (int j = 0; j < NVP; ++j)
#pragma unroll
                    for (int k = 0; k < VEC; ++k) {
                        const int c = (lane + 32 * j) * VEC + k;
                        if (c < a.width) st[16 + c] = acc[j][k];
                    }
                return;
            }
#pragma unroll
            for (int j = 0; j < NVP; ++j)
#pragma unroll
                for (int k = 0; k < VEC; ++k) {
                    const int c = (lane + 32 * j) * VEC + k;
                    if (c >= a.ldo) continue;
                    const int hh = min(c / a.dim, a.heads - 1);
                    float d = den[0];
#pragma unroll
                    for (int h = 1; h < 8; ++h) d = hh == h ? den[h] : d;
                    na_store(a, r, c, na_finalize(a, c, acc[j][k], d));
                }
            // padding columns beyond the vectors a lane holds (ldo > 512):
            // zeros, as the merge kernel writes them
            for (int c = NVP * 32 * VEC + lane; c < a.ldo; c += 32) na_store(a, r, c, 0.f);
        };
        // The row that started before lo and continues into this range.
        if (r0 > 0 && (r0 > a.n || a.row[r0] > lo) && lo < a.e) {
            const uint64_t rc = r0 - 1;
            const uint64_t end = a.row[rc + 1] < hi ? a.row[rc + 1] : hi;
            na_part<HT, VEC, NVP>(a, rc, lo, end, sp, m, den, acc);
            emit(rc, true, 0);
        }
        // Rows that start in [lo, hi) (the last range also takes the empty
        // rows at the very end of the edge list).
        for (uint64_t r = r0; r < a.n && (a.row[r] < hi || last); ++r) {
            const uint64_t b = a.row[r], en = a.row[r + 1];
            const bool partial = en > hi;
            na_part<HT, VEC, NVP>(a, r, b, partial ? hi : en, sp, m, den, acc);
            emit(r, partial, 1);
        }
    }
}

// One warp per range boundary x = w*SEG: merges the row that crosses x if it
// starts in range w-1 (so each crossing row is merged exactly once).
template <int VEC, int NVP>
__global__ void __launch_bounds__(128) na_merge_kernel(const NaArgs a) {
    const int lane = threadIdx.x & 31;
    const uint64_t w = blockIdx.x * 4ull + (threadIdx.x >> 5) + 1;
    if (w >= a.ranges) return;
    const uint64_t x = w * a.seg;
    const uint64_t r0 = lower_bound_rows(a.row, a.n, x);
    if (r0 <= a.n && a.row[r0] == x) return;  // x is a row start: nothing crosses
    const uint64_t r = r0 - 1;
    const uint64_t b = a.row[r], en = a.row[r + 1];
    if (b + a.seg < x) return;                // crosses an earlier boundary too
    const uint64_t w1 = (en - 1) / a.seg;
    const int K = a.heads;
    float M[8], den[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) { M[h] = -INFINITY; den[h] = 0.f; }
    // slots: (w-1, side 1), then (v, side 0) for v in [w, w1]
    for (uint64_t v = w - 1; v <= w1; ++v) {
        const float* st = a.scratch + (2 * v + (v == w - 1 ? 1 : 0)) * kSlotFloats;
#pragma unroll
        for (int h = 0; h < 8; ++h) if (h < K) M[h] = fmaxf(M[h], st[h]);
    }
    for (uint64_t v = w - 1; v <= w1; ++v) {
        const float* st = a.scratch + (2 * v + (v == w - 1 ? 1 : 0)) * kSlotFloats;
#pragma unroll
        for (int h = 0; h < 8; ++h) if (h < K) den[h] += st[8 + h] * __expf(st[h] - M[h]);
    }
    for (int c = lane; c < a.ldo; c += 32) {
        float accv = 0.f, d = 0.f;
        if (c < a.width) {
            const int hh = min(c / a.dim, K - 1);
            float Mh = M[0];
#pragma unroll
            for (int h = 1; h < 8; ++h) Mh = hh == h ? M[h] : Mh;
            for (uint64_t v = w - 1; v <= w1; ++v) {
                const float* st = a.scratch + (2 * v + (v == w - 1 ? 1 : 0)) * kSlotFloats;
                accv += st[16 + c] * __expf(st[hh] - Mh);
            }
            d = den[0];
#pragma unroll
            for (int h = 1; h < 8; ++h) d = hh == h ? den[h] : d;
        }
        na_store(a, r, c, na_finalize(a, c, accv, d));
    }
}

// Device address of the scratch array in the current device's context. It is
// looked up on every call (a host-side table lookup once the module is loaded),
// so a context that was reset and reloaded the module never sees a stale
// address. The first lookup on a device loads the module; that first call must
// come before any stream capture.
int scratch_for_current_device(float** out) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    *out = static_cast<float*>(p);
    return 0;
}

template <class HT, int VEC, int NVP>
int na_launch(const NaArgs& a, cudaStream_t st) {
    const unsigned blocks = unsigned((a.ranges + 3) / 4);
    na_range_kernel<HT, VEC, NVP><<<blocks, 128, 0, st>>>(a);
    GATB_LAUNCH("no-allocation aggregation kernel");
    if (a.ranges > 1) {
        na_merge_kernel<VEC, NVP><<<unsigned((a.ranges - 1 + 3) / 4), 128, 0, st>>>(a);
        GATB_LAUNCH("no-allocation merge kernel");
    }
    return 0;
}

}  // namespace
}  // namespace gatb

using namespace gatb;

extern "C" int gat_b200_aggregate_fused_noalloc(uint64_t n, uint64_t e, const uint64_t* row, const uint32_t* col,
                                                int heads, int dim, const void* h, int h_dtype, int ldh,
                                                const float* left, const float* right, int hidden, void* out,
                                                int out_dtype, int ldo, void* stream) {
    clear_error();
    if (!n || n > uint64_t(INT32_MAX)) return fail("invalid graph sizes");
    if (!row || (e && !col) || !h || !left || !right || !out) return fail("aggregate_fused_noalloc: null buffer");
    if (heads < 1 || heads > 8 || dim < 1 || dim > 64) return fail("invalid parameter shape (heads <=8, head_dim <=64)");
    if (h_dtype != GAT_B200_BF16 && h_dtype != GAT_B200_F32) return fail("aggregate_fused_noalloc: bad feature dtype");
    if (out_dtype != GAT_B200_BF16 && out_dtype != GAT_B200_F32) return fail("aggregate_fused_noalloc: bad output dtype");
    const int width = heads * dim;
    const int elem = h_dtype == GAT_B200_BF16 ? 2 : 4;
    if (ldh < padded_ld(width, elem) || ldo < width) return fail("aggregate_fused_noalloc: row stride smaller than the width");
    if ((reinterpret_cast<uintptr_t>(h) & 15) || (uint64_t(ldh) * elem) % 16)
        return fail("aggregate_fused_noalloc: feature rows must start on 16-byte boundaries");
    // Ranges of SEG edges: enough ranges to balance the warps, at most
    // kMaxRanges (the scratch holds two partial states per range).
    uint64_t ranges = (e + kMinSeg - 1) / kMinSeg;
    if (ranges > kMaxRanges) ranges = kMaxRanges;
    if (ranges == 0) ranges = 1;
    const uint64_t seg = e ? (e + ranges - 1) / ranges : 1;
    if (seg > kMaxSeg)
        return fail_code(GAT_B200_EUNSUPPORTED,
                         "aggregate_fused_noalloc: " + std::to_string(e) + " edges exceed the maximum of " +
                             std::to_string(kMaxRanges * kMaxSeg) +
                             " (32 MiB static scratch: 7936 ranges of at most 65536 edges)");
    float* scratch = nullptr;
    int rc = scratch_for_current_device(&scratch);
    if (rc) return rc;
    NaArgs a{};
    a.row = row;
    a.col = col;
    a.n = n;
    a.e = e;
    a.seg = seg;
    a.ranges = uint32_t((e + seg - 1) / seg ? (e + seg - 1) / seg : 1);
    a.heads = heads;
    a.dim = dim;
    a.width = width;
    a.h = h;
    a.ldh = ldh;
    a.left = left;
    a.right = right;
    a.hidden = hidden;
    a.out = out;
    a.out_bf16 = out_dtype == GAT_B200_BF16;
    a.ldo = ldo;
    a.scratch = scratch;
    cudaStream_t st = as_stream(stream);
    if (h_dtype == GAT_B200_BF16) return na_launch<uint16_t, 8, 2>(a, st);
    return na_launch<float, 4, 4>(a, st);
}
