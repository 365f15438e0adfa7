// Edge-softmax SpMM: the GAT aggregation (hot kernel).
//
// Replaces max_prescan + standard_aggregate + finish of the reference's B0 path
// (baseline/src/baseline_standard.cpp:44-97). For destination row i and head h:
//   s_ij = leaky(L_ih + R_jh),  m_ih = max_j s_ij,  p_ij = exp(s_ij - m_ih),
//   den_ih = sum_j p_ij,        out_ih = (sum_j p_ij H_j,h) / den_ih  (ELU if hidden).
//
// B200 design:
//  * One warp owns one work item (a row, or a <= seg_edges slice of a hub row).
//    Items are visited from the largest degree down (degree-sorted permutation
//    read backwards) and dealt round-robin to all resident warps, so every warp
//    gets the same mix of degrees and no item exceeds seg_edges edges.
//  * Edges are processed in chunks of 32: lane t computes the K scores of edge t
//    (one coalesced col load, a 4*K-byte R gather), the warp reduces the chunk
//    max per head, updates the running max and rescales the running sums once
//    per chunk (online softmax; the final max equals the reference's exact
//    max, because leaky is monotone). p and the source ids go through shared
//    memory.
//  * The feature gather: a row of H (K*d BF16 = 512 B for 8x32) is read by
//    LPE lanes with one 16-byte load each; 32/LPE edges are in flight per warp
//    step and the loop is unrolled so each lane keeps 8 loads outstanding.
//  * Epilogue fused: divide by den, ELU, and BF16 RNE store = the next layer's
//    input; or FP32 logits; or the reference's unnormalised out/den/max.
//  * Hub slices write partial (max, sum, acc) states to scratch; a second small
//    kernel merges them per hub row.
#include "device.cuh"
#include "graph.cuh"

namespace gatb {
namespace {

constexpr int kWarps = 8;  // warps per block
constexpr unsigned kFull = 0xffffffffu;

struct AggArgs {
    const uint64_t* row;
    const uint32_t* col;
    const uint32_t* perm;
    uint64_t n;
    uint32_t n_hub, n_seg;
    const Segment* segs;
    const uint32_t* hub_seg_offset;
    float* seg_state;
    int heads, dim, width;
    const void* h;
    int ldh;
    const float* left;
    const float* right;
    const float* fixed_p;    // [e][heads] or null
    const float* fixed_den;  // [n][heads] or null
    int unnorm;              // 1: write unnormalised FP32 out + den (+max)
    int hidden;              // ELU in the fused epilogue
    void* out;
    int out_bf16;
    int out_vec;             // out base and row stride allow 16-byte stores
    int ldo;
    float* den_out;
    float* max_out;
};

template <class HT>
struct Vec;
template <>
struct Vec<uint16_t> {  // BF16
    static constexpr int N = 8;
    __device__ static __forceinline__ void unpack(const uint4& r, float* f) {
        f[0] = bf16lo(r.x); f[1] = bf16hi(r.x); f[2] = bf16lo(r.y); f[3] = bf16hi(r.y);
        f[4] = bf16lo(r.z); f[5] = bf16hi(r.z); f[6] = bf16lo(r.w); f[7] = bf16hi(r.w);
    }
};
template <>
struct Vec<float> {
    static constexpr int N = 4;
    __device__ static __forceinline__ void unpack(const uint4& r, float* f) {
        f[0] = __uint_as_float(r.x); f[1] = __uint_as_float(r.y);
        f[2] = __uint_as_float(r.z); f[3] = __uint_as_float(r.w);
    }
};

template <int KM>
__device__ __forceinline__ float pick(const float (&a)[KM], int h) {
    float v = a[0];
#pragma unroll
    for (int k = 1; k < KM; ++k) v = (h == k) ? a[k] : v;
    return v;
}

// Writes VECN consecutive output values starting at column c0 of row r.
template <int VECN>
__device__ __forceinline__ void store_out(const AggArgs& a, uint64_t r, int c0, const float* v) {
    if (a.out_bf16) {
        uint16_t* o = static_cast<uint16_t*>(a.out) + r * uint64_t(a.ldo) + c0;
        if (a.out_vec && c0 + VECN <= a.ldo) {
            uint32_t w[VECN / 2];
#pragma unroll
            for (int k = 0; k < VECN / 2; ++k) w[k] = pack_bf16x2(v[2 * k], v[2 * k + 1]);
            if constexpr (VECN == 8) {
                *reinterpret_cast<uint4*>(o) = make_uint4(w[0], w[1], w[2], w[3]);
            } else {
                *reinterpret_cast<uint2*>(o) = make_uint2(w[0], w[1]);
            }
        } else {
#pragma unroll
            for (int k = 0; k < VECN; ++k)
                if (c0 + k < a.ldo) o[k] = uint16_t(pack_bf16x2(v[k], 0.f) & 0xffffu);
        }
    } else {
        float* o = static_cast<float*>(a.out) + r * uint64_t(a.ldo) + c0;
        if (a.out_vec && c0 + VECN <= a.ldo) {
#pragma unroll
            for (int k = 0; k < VECN; k += 4)
                *reinterpret_cast<float4*>(o + k) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
        } else {
#pragma unroll
            for (int k = 0; k < VECN; ++k)
                if (c0 + k < a.ldo) o[k] = v[k];
        }
    }
}

// Final value of one output element from its accumulated sum.
__device__ __forceinline__ float finalize(const AggArgs& a, int c, float acc, float den) {
    if (c >= a.width) return 0.f;  // padding columns stay zero
    if (a.unnorm) return acc;
    float v = acc * (den > 0.f ? 1.f / den : 0.f);  // baseline_standard.cpp:115-117
    return a.hidden ? elu(v) : v;
}

// KT: heads known at compile time (1 or 8), 0 = runtime heads <= 8.
// LPE lanes share one edge's feature row; VPL 16-byte vectors per lane.
// MIXED: a vector may straddle heads (dim not a multiple of the vector width).
template <class HT, int KT, int LPE, int VPL, bool MIXED>
__global__ void __launch_bounds__(kWarps * 32) agg_kernel(const AggArgs a) {
    using V = Vec<HT>;
    constexpr int VEC = V::N;
    constexpr int KM = KT ? KT : 8;
    constexpr int EPS = 32 / LPE;               // edges per warp step
    constexpr int U = (VPL == 1) ? 8 : (VPL == 2 ? 4 : 2);  // unroll: 8 loads in flight per lane
    __shared__ float s_p[kWarps][32 * KM];
    __shared__ uint32_t s_src[kWarps][32];

    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int K = KT ? KT : a.heads;
    const int es = lane / LPE, vl = lane % LPE;
    const int nvec = (a.width + VEC - 1) / VEC;
    float* sp = s_p[wib];
    uint32_t* ss = s_src[wib];
    const HT* H = static_cast<const HT*>(a.h);

    // Head owning each of this lane's vectors (or elements when MIXED).
    int hv[VPL];
    int hk[VPL][MIXED ? VEC : 1];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
        int v = vl + j * LPE;
        hv[j] = KT == 1 ? 0 : min((v * VEC) / a.dim, K - 1);
#pragma unroll
        for (int k = 0; k < (MIXED ? VEC : 1); ++k) hk[j][k] = min((v * VEC + k) / a.dim, K - 1);
    }

    const uint64_t total = uint64_t(a.n_seg) + (a.n - a.n_hub);
    const uint64_t gw = blockIdx.x * uint64_t(kWarps) + wib;
    const uint64_t G = uint64_t(gridDim.x) * kWarps;
    for (uint64_t item = gw; item < total; item += G) {
        uint64_t beg, end, r;
        bool partial = item < a.n_seg;
        if (partial) {
            Segment sg = a.segs[item];
            r = sg.row;
            beg = sg.beg;
            end = sg.end;
        } else {
            r = a.perm[a.n - 1 - a.n_hub - (item - a.n_seg)];
            beg = a.row[r];
            end = a.row[r + 1];
        }
        float Lr[KM], m[KM], ls[KM];
        bool have_l = false;
        if constexpr (KT == 8) {
            if (!a.fixed_p) {
                float4 l0 = *reinterpret_cast<const float4*>(a.left + r * 8);
                float4 l1 = *reinterpret_cast<const float4*>(a.left + r * 8 + 4);
                Lr[0] = l0.x; Lr[1] = l0.y; Lr[2] = l0.z; Lr[3] = l0.w;
                Lr[4] = l1.x; Lr[5] = l1.y; Lr[6] = l1.z; Lr[7] = l1.w;
                have_l = true;
            }
        }
        if (!have_l) {
#pragma unroll
            for (int h = 0; h < KM; ++h) Lr[h] = (h < K && !a.fixed_p) ? a.left[r * K + h] : 0.f;
        }
#pragma unroll
        for (int h = 0; h < KM; ++h) {
            m[h] = a.fixed_p ? 0.f : -INFINITY;
            ls[h] = 0.f;
        }
        float acc[VPL][VEC];
#pragma unroll
        for (int j = 0; j < VPL; ++j)
#pragma unroll
            for (int k = 0; k < VEC; ++k) acc[j][k] = 0.f;

        for (uint64_t c0 = beg; c0 < end; c0 += 32) {
            const int cnt = int(end - c0 < 32 ? end - c0 : 32);
            // ---- scores of up to 32 edges, one per lane ----
            float s[KM];
            uint32_t src = 0;
            if (lane < cnt) {
                src = ldg_stream_u32(a.col + c0 + lane);
                if (a.fixed_p) {
#pragma unroll
                    for (int h = 0; h < KM; ++h) s[h] = h < K ? a.fixed_p[(c0 + lane) * K + h] : 0.f;
                } else if constexpr (KT == 8) {
                    float4 r0 = __ldg(reinterpret_cast<const float4*>(a.right + uint64_t(src) * 8));
                    float4 r1 = __ldg(reinterpret_cast<const float4*>(a.right + uint64_t(src) * 8 + 4));
                    float rr[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
                    for (int h = 0; h < 8; ++h) s[h] = leaky(Lr[h] + rr[h]);
                } else {
#pragma unroll
                    for (int h = 0; h < KM; ++h)
                        s[h] = h < K ? leaky(Lr[h] + __ldg(a.right + uint64_t(src) * K + h)) : 0.f;
                }
            } else {
#pragma unroll
                for (int h = 0; h < KM; ++h) s[h] = a.fixed_p ? 0.f : -INFINITY;
            }
            float sc[KM];
            if (a.fixed_p) {
#pragma unroll
                for (int h = 0; h < KM; ++h) {
                    sc[h] = 1.f;
                    ls[h] += s[h];
                    sp[lane * KM + h] = s[h];
                }
            } else {
#pragma unroll
                for (int h = 0; h < KM; ++h) {
                    float nm = fmaxf(m[h], warp_max(s[h]));
                    sc[h] = expf(m[h] - nm);  // exp(-inf) = 0 on the first chunk
                    m[h] = nm;
                    float p = lane < cnt ? expf(s[h] - nm) : 0.f;
                    ls[h] = ls[h] * sc[h] + p;
                    sp[lane * KM + h] = p;
                }
#pragma unroll
                for (int j = 0; j < VPL; ++j) {
                    if constexpr (MIXED) {
#pragma unroll
                        for (int k = 0; k < VEC; ++k) acc[j][k] *= pick(sc, hk[j][k]);
                    } else {
                        float f = pick(sc, hv[j]);
#pragma unroll
                        for (int k = 0; k < VEC; ++k) acc[j][k] *= f;
                    }
                }
            }
            ss[lane] = src;
            __syncwarp();
            // ---- weighted gather of the feature rows ----
            for (int t0 = 0; t0 < cnt; t0 += EPS * U) {
                uint4 raw[U][VPL];
                float pw[U][VPL][MIXED ? VEC : 1];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int t = t0 + u * EPS + es;
                    const bool ok = t < cnt;
                    const uint32_t sidx = ok ? ss[t] : 0u;
#pragma unroll
                    for (int j = 0; j < VPL; ++j) {
                        const int v = vl + j * LPE;
                        if (ok && v < nvec)
                            raw[u][j] = ldg_nc_v4(H + uint64_t(sidx) * a.ldh + v * VEC);
                        else
                            raw[u][j] = make_uint4(0, 0, 0, 0);
#pragma unroll
                        for (int k = 0; k < (MIXED ? VEC : 1); ++k)
                            pw[u][j][k] = ok ? sp[t * KM + (MIXED ? hk[j][k] : hv[j])] : 0.f;
                    }
                }
#pragma unroll
                for (int u = 0; u < U; ++u)
#pragma unroll
                    for (int j = 0; j < VPL; ++j) {
                        float f[VEC];
                        V::unpack(raw[u][j], f);
#pragma unroll
                        for (int k = 0; k < VEC; ++k) acc[j][k] = fmaf(pw[u][j][MIXED ? k : 0], f[k], acc[j][k]);
                    }
            }
            __syncwarp();
        }
        // ---- combine edge slots and lanes ----
#pragma unroll
        for (int o = LPE; o < 32; o <<= 1)
#pragma unroll
            for (int j = 0; j < VPL; ++j)
#pragma unroll
                for (int k = 0; k < VEC; ++k) acc[j][k] += __shfl_xor_sync(kFull, acc[j][k], o);
        float den[KM];
#pragma unroll
        for (int h = 0; h < KM; ++h) den[h] = warp_sum(ls[h]);

        if (partial) {
            float* st = a.seg_state + item * kSegStateFloats;
            if (lane < K) {
                st[lane] = pick(m, lane);
                st[8 + lane] = pick(den, lane);
            }
            if (es == 0)
#pragma unroll
                for (int j = 0; j < VPL; ++j) {
                    const int v = vl + j * LPE;
                    if (v < nvec)
#pragma unroll
                        for (int k = 0; k < VEC; ++k) st[16 + v * VEC + k] = acc[j][k];
                }
            continue;
        }
        const bool empty = beg == end;
        if (a.unnorm && lane < K) {
            a.den_out[r * K + lane] = a.fixed_den ? a.fixed_den[r * K + lane] : pick(den, lane);
            if (a.max_out && !a.fixed_p) a.max_out[r * K + lane] = empty ? 0.f : pick(m, lane);
        }
        if (es == 0) {
#pragma unroll
            for (int j = 0; j < VPL; ++j) {
                const int v = vl + j * LPE;
                if (v * VEC >= a.ldo) continue;
                float o[VEC];
#pragma unroll
                for (int k = 0; k < VEC; ++k) {
                    int hh = MIXED ? hk[j][k] : hv[j];
                    o[k] = finalize(a, v * VEC + k, acc[j][k], pick(den, hh));
                }
                store_out<VEC>(a, r, v * VEC, o);
            }
        }
    }
}

// Merges the partial states of each hub row's segments (one warp per hub row).
__global__ void __launch_bounds__(kWarps * 32) hub_merge_kernel(const AggArgs a) {
    const int lane = threadIdx.x & 31;
    const uint64_t k = blockIdx.x * uint64_t(kWarps) + (threadIdx.x >> 5);
    if (k >= a.n_hub) return;
    const uint32_t s0 = a.hub_seg_offset[k], s1 = a.hub_seg_offset[k + 1];
    const uint64_t r = a.perm[a.n - 1 - k];
    const int K = a.heads;
    float M[8], den[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) { M[h] = -INFINITY; den[h] = 0.f; }
    for (uint32_t s = s0; s < s1; ++s) {
        const float* st = a.seg_state + uint64_t(s) * kSegStateFloats;
#pragma unroll
        for (int h = 0; h < 8; ++h) if (h < K) M[h] = fmaxf(M[h], st[h]);
    }
    for (uint32_t s = s0; s < s1; ++s) {
        const float* st = a.seg_state + uint64_t(s) * kSegStateFloats;
#pragma unroll
        for (int h = 0; h < 8; ++h) if (h < K) den[h] += st[8 + h] * expf(st[h] - M[h]);
    }
    if (a.unnorm && lane < K) {
        a.den_out[r * K + lane] = a.fixed_den ? a.fixed_den[r * K + lane] : pick(den, lane);
        if (a.max_out && !a.fixed_p) a.max_out[r * K + lane] = pick(M, lane);
    }
    for (int c = lane; c < a.ldo; c += 32) {
        float accv = 0.f, d = 0.f;
        if (c < a.width) {
            const int hh = min(c / a.dim, K - 1);
            const float Mh = pick(M, hh);
            for (uint32_t s = s0; s < s1; ++s) {
                const float* st = a.seg_state + uint64_t(s) * kSegStateFloats;
                accv += st[16 + c] * expf(st[hh] - Mh);
            }
            d = pick(den, hh);
        }
        float v = finalize(a, c, accv, d);
        if (a.out_bf16)
            static_cast<uint16_t*>(a.out)[r * a.ldo + c] = uint16_t(pack_bf16x2(v, 0.f) & 0xffffu);
        else
            static_cast<float*>(a.out)[r * a.ldo + c] = v;
    }
}

template <class HT, int KT, int LPE, int VPL, bool MIXED>
int launch_agg(const AggArgs& a, cudaStream_t st) {
    static int grid = 0;  // resident blocks (per process; all B200s are alike)
    if (!grid) {
        int dev = 0, sms = 0, per_sm = 0;
        GATB_CUDA(cudaGetDevice(&dev));
        GATB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        GATB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, agg_kernel<HT, KT, LPE, VPL, MIXED>,
                                                                kWarps * 32, 0));
        grid = sms * (per_sm > 0 ? per_sm : 1);
    }
    uint64_t items = uint64_t(a.n_seg) + (a.n - a.n_hub);
    uint64_t need = (items + kWarps - 1) / kWarps;
    unsigned blocks = unsigned(need < uint64_t(grid) ? need : uint64_t(grid));
    if (blocks == 0) blocks = 1;
    agg_kernel<HT, KT, LPE, VPL, MIXED><<<blocks, kWarps * 32, 0, st>>>(a);
    GATB_LAUNCH("edge-softmax aggregation kernel");
    if (a.n_hub) {
        hub_merge_kernel<<<(a.n_hub + kWarps - 1) / kWarps, kWarps * 32, 0, st>>>(a);
        GATB_LAUNCH("hub merge kernel");
    }
    return 0;
}

}  // namespace

int aggregate_dispatch(const gat_b200_graph* g, int heads, int dim, const void* h, int h_dtype, int ldh,
                       const float* left, const float* right, const float* fixed_p, const float* fixed_den,
                       int unnorm, int hidden, void* out, int out_bf16, int ldo, float* den, float* max,
                       cudaStream_t st) {
    if (!g) return fail("aggregate: null graph");
    if (heads < 1 || heads > 8 || dim < 1 || dim > 64) return fail("invalid parameter shape (heads <=8, head_dim <=64)");
    const int width = heads * dim;
    const int elem = h_dtype == GAT_B200_BF16 ? 2 : 4;
    if (h_dtype != GAT_B200_BF16 && h_dtype != GAT_B200_F32) return fail("aggregate: bad feature dtype");
    if (!h || !out || (!fixed_p && (!left || !right))) return fail("aggregate: null buffer");
    if (ldh < padded_ld(width, elem) || ldo < width) return fail("aggregate: row stride smaller than the width");
    if (unnorm && !den) return fail("aggregate: den output required");
    if ((reinterpret_cast<uintptr_t>(h) & 15) || (uint64_t(ldh) * elem) % 16)
        return fail("aggregate: feature rows must start on 16-byte boundaries");
    if ((fixed_p == nullptr) != (fixed_den == nullptr)) return fail("aggregate: fixed_p and fixed_den go together");
    AggArgs a{};
    a.row = g->row;
    a.col = g->col;
    a.perm = g->perm;
    a.n = g->n;
    a.n_hub = g->n_hub;
    a.n_seg = g->n_seg;
    a.segs = g->segs;
    a.hub_seg_offset = g->hub_seg_offset;
    a.seg_state = g->seg_state;
    a.heads = heads;
    a.dim = dim;
    a.width = width;
    a.h = h;
    a.ldh = ldh;
    a.left = left;
    a.right = right;
    a.fixed_p = fixed_p;
    a.fixed_den = fixed_den;
    a.unnorm = unnorm;
    a.hidden = hidden;
    a.out = out;
    a.out_bf16 = out_bf16;
    a.ldo = ldo;
    {
        const int oe = out_bf16 ? 2 : 4;
        a.out_vec = (reinterpret_cast<uintptr_t>(out) % 16 == 0) && (uint64_t(ldo) * oe) % 16 == 0;
    }
    a.den_out = den;
    a.max_out = max;
    if (h_dtype == GAT_B200_BF16) {
        if (heads == 8 && dim == 32 && (reinterpret_cast<uintptr_t>(left) & 15) == 0 &&
            (reinterpret_cast<uintptr_t>(right) & 15) == 0)
            return launch_agg<uint16_t, 8, 32, 1, false>(a, st);
        if (heads == 1 && width <= 64) return launch_agg<uint16_t, 1, 8, 1, false>(a, st);
        return launch_agg<uint16_t, 0, 32, 2, true>(a, st);
    }
    if (heads == 8 && dim == 32 && (reinterpret_cast<uintptr_t>(left) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(right) & 15) == 0)
        return launch_agg<float, 8, 32, 2, false>(a, st);
    if (heads == 1 && width <= 64) return launch_agg<float, 1, 16, 1, false>(a, st);
    return launch_agg<float, 0, 32, 4, true>(a, st);
}

}  // namespace gatb
