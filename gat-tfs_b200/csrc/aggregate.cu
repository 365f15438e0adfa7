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

// Packed FP32 pair (sm_100 f32x2 arithmetic; each half rounds like the scalar op).
struct F2 {
    unsigned long long v;
};
__device__ __forceinline__ F2 f2make(float lo, float hi) {
    F2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ F2 f2zero() { return F2{0ull}; }
__device__ __forceinline__ F2 f2fma(F2 a, F2 b, F2 c) {
    F2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v));
    return r;
}
__device__ __forceinline__ F2 f2mul(F2 a, F2 b) {
    F2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
    return r;
}
__device__ __forceinline__ float f2get(F2 a, int hi) {
    float lo_f, hi_f;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo_f), "=f"(hi_f) : "l"(a.v));
    return hi ? hi_f : lo_f;
}

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
    // ELU (gat.hpp:53): exp(x)-1 for x < 0, |error| < 3e-7 (values are >= -1).
    return (a.hidden && v < 0.f) ? __expf(v) - 1.f : v;
}

// ---- asynchronous pipeline -------------------------------------------------
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

enum : int { kValid = 1, kFirst = 2, kLast = 4, kPartial = 8 };

// One chunk (at most C edges) of a work item, identical in every lane.
struct Rec {
    uint64_t item;  // work item: segment index (< n_seg) or row item
    uint64_t pos;   // first edge of the chunk
    uint32_t r;     // destination row
    int cnt;        // edges in the chunk (0 for an empty row)
    int flags;
};

// Per-chunk record handed from the scoring stage to the consuming stage.
template <int C, int KM>
struct __align__(16) Slot {
    float p[KM * (C + 1)];  // p[h*(C+1) + t]: conflict-free stores and reads
    float sc[8];      // rescale of the running sums before this chunk
    float den[8];     // final sums (last chunk of an item)
    float m[8];       // final maxima (last chunk of an item)
    uint64_t item;
    uint32_t r;
    int cnt;
    int flags;
};

// Walks this warp's work items (gw, gw+G, ...) chunk by chunk. Item metadata
// is fetched two items ahead (segment or permutation entry) and one item
// ahead (row pointers), so a new item's bounds are in registers when needed.
template <int C>
struct Gen {
    uint64_t total, G;
    uint64_t item, beg, pos, end;
    uint32_t r;
    bool partial, have;
    uint64_t n_item, n_beg, n_end;  // next item
    uint32_t n_r;
    bool n_partial, n_have;
    uint64_t nn_item, nn_beg, nn_end;  // item after next (stage 1 only for rows)
    uint32_t nn_r;
    bool nn_partial, nn_have;

    __device__ __forceinline__ void stage1(const AggArgs& a, uint64_t it, uint32_t& rr, uint64_t& b, uint64_t& e,
                                           bool& part, bool& hv) {
        hv = it < total;
        part = false;
        b = e = 0;
        rr = 0;
        if (!hv) return;
        if (it < a.n_seg) {
            const Segment* sg = a.segs + it;
            rr = sg->row;
            b = sg->beg;
            e = sg->end;
            part = true;
        } else {
            rr = a.perm[a.n - 1 - a.n_hub - (it - a.n_seg)];
        }
    }
    __device__ __forceinline__ void stage2(const AggArgs& a, uint32_t rr, uint64_t& b, uint64_t& e, bool part,
                                           bool hv) {
        if (hv && !part) {
            b = a.row[rr];
            e = a.row[rr + 1];
        }
    }
    __device__ __forceinline__ void init(const AggArgs& a, uint64_t gw, uint64_t g_, uint64_t tot) {
        total = tot;
        G = g_;
        item = gw;
        stage1(a, item, r, beg, end, partial, have);
        stage2(a, r, beg, end, partial, have);
        pos = beg;
        n_item = gw + G;
        stage1(a, n_item, n_r, n_beg, n_end, n_partial, n_have);
        stage2(a, n_r, n_beg, n_end, n_partial, n_have);
        nn_item = gw + 2 * G;
        stage1(a, nn_item, nn_r, nn_beg, nn_end, nn_partial, nn_have);
    }
    __device__ __forceinline__ Rec next(const AggArgs& a) {
        Rec rec;
        rec.flags = 0;
        rec.cnt = 0;
        rec.item = item;
        rec.pos = pos;
        rec.r = r;
        if (!have) return rec;
        const uint64_t rem = end - pos;
        rec.cnt = int(rem < uint64_t(C) ? rem : uint64_t(C));
        rec.flags = kValid | (pos == beg ? kFirst : 0) | (rem <= uint64_t(C) ? kLast : 0) | (partial ? kPartial : 0);
        pos += C;
        if (pos >= end) {  // move to the next item
            item = n_item; r = n_r; beg = n_beg; end = n_end; partial = n_partial; have = n_have;
            pos = beg;
            n_item = nn_item; n_r = nn_r; n_beg = nn_beg; n_end = nn_end; n_partial = nn_partial; n_have = nn_have;
            stage2(a, n_r, n_beg, n_end, n_partial, n_have);
            nn_item = n_item + G;
            stage1(a, nn_item, nn_r, nn_beg, nn_end, nn_partial, nn_have);
        }
        return rec;
    }
};

// KT: heads known at compile time (1 or 8), 0 = runtime heads <= 8.
// C: edges per chunk. LPE lanes share one feature row in the gather; VPL
// 16-byte vectors per lane. MIXED: a vector may straddle two heads.
//
// Per warp, per loop iteration (one chunk k):
//   1. scores of chunk k (col and R were prefetched one and two iterations
//      earlier), running max / sum update, p and the rescale factor to shared
//      memory;
//   2. cp.async of chunk k's feature rows into shared-memory buffer k%2;
//   3. prefetch: R of chunk k+1, col of chunk k+2, metadata of later items;
//   4. consume chunk k-1 from buffer (k-1)%2 (waiting only for that group).
// Each lane copies exactly the 16-byte vectors it later consumes, so a lane
// waits only for its own copies.
template <class HT, int KT, int C, int LPE, int VPL, bool MIXED, int NVC>
__global__ void __launch_bounds__(256) agg_kernel(const AggArgs a) {
    using V = Vec<HT>;
    constexpr int VEC = V::N;
    constexpr int KM = KT ? KT : 8;
    constexpr int SPL = 32 / C;                 // score lanes per edge
    constexpr int KS = (KM + SPL - 1) / SPL;    // heads per score lane
    constexpr int EPS = 32 / LPE;               // edges per consume step
    constexpr int RV = LPE * VPL;               // 16-byte vectors per buffered row
    constexpr int NT = C / EPS;                 // consume steps per chunk
    constexpr int CPL = (RV + SPL - 1) / SPL;   // vectors each lane copies per edge
    constexpr int PS = C + 1;                   // p row stride (padding)
    static_assert(C * SPL == 32 && EPS * LPE == 32 && C % EPS == 0, "bad tiling");
    static_assert(VEC % 2 == 0, "packed pairs");
    using SlotT = Slot<C, KM>;

    extern __shared__ __align__(16) uint8_t agg_smem[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const size_t warp_bytes = 2 * sizeof(SlotT) + size_t(2) * C * RV * 16;
    uint8_t* wbase = agg_smem + wib * warp_bytes;
    SlotT* slots = reinterpret_cast<SlotT*>(wbase);
    uint4* bufs = reinterpret_cast<uint4*>(wbase + 2 * sizeof(SlotT));
    const uint32_t bufs_s = static_cast<uint32_t>(__cvta_generic_to_shared(bufs));

    const int K = KT ? KT : a.heads;
    const int t = lane % C, hs = lane / C;      // scoring role
    const int es = lane / LPE, vl = lane % LPE; // gather / consume role
    const int nvec = NVC ? NVC : (a.width + VEC - 1) / VEC;
    const HT* H = static_cast<const HT*>(a.h);
    const bool fixed = a.fixed_p != nullptr;

    int hv[VPL];
    int hk[VPL][MIXED ? VEC : 1];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
        const int v = vl + j * LPE;
        hv[j] = KT == 1 ? 0 : min((v * VEC) / a.dim, K - 1);
#pragma unroll
        for (int k = 0; k < (MIXED ? VEC : 1); ++k) hk[j][k] = min((v * VEC + k) / a.dim, K - 1);
    }

    const uint64_t total = uint64_t(a.n_seg) + (a.n - a.n_hub);
    const uint64_t G = uint64_t(gridDim.x) * (blockDim.x >> 5);
    const uint64_t gw = blockIdx.x * uint64_t(blockDim.x >> 5) + wib;
    Gen<C> gen;
    gen.init(a, gw, G, total);

    // Prefetch helpers (lane t of chunk rec).
    auto load_col = [&](const Rec& rc) -> uint32_t {
        return (rc.flags & kValid) && t < rc.cnt ? ldg_stream_u32(a.col + rc.pos + t) : 0u;
    };
    auto load_r = [&](const Rec& rc, uint32_t src, float (&o)[KS]) {
        const bool ok = (rc.flags & kValid) && t < rc.cnt;
        if (fixed) {
#pragma unroll
            for (int j = 0; j < KS; ++j) {
                const int h = hs * KS + j;
                o[j] = ok && h < K ? a.fixed_p[(rc.pos + t) * K + h] : 0.f;
            }
            return;
        }
        if constexpr (KT == 8 && KS == 4) {
            if (ok) {
                const float4 v = __ldg(reinterpret_cast<const float4*>(a.right + uint64_t(src) * 8 + hs * 4));
                o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
            } else {
#pragma unroll
                for (int j = 0; j < KS; ++j) o[j] = 0.f;
            }
        } else {
#pragma unroll
            for (int j = 0; j < KS; ++j) {
                const int h = hs * KS + j;
                o[j] = ok && h < K ? __ldg(a.right + uint64_t(src) * K + h) : 0.f;
            }
        }
    };
    auto load_l = [&](const Rec& rc, float (&o)[KS]) {
        const bool ok = (rc.flags & kValid) && (rc.flags & kFirst) && !fixed;
#pragma unroll
        for (int j = 0; j < KS; ++j) {
            const int h = hs * KS + j;
            o[j] = ok && h < K ? a.left[uint64_t(rc.r) * K + h] : 0.f;
        }
    };

    Rec P1 = gen.next(a);
    Rec P2 = gen.next(a);
    uint32_t colP1 = load_col(P1);
    float RP1[KS], LP1[KS];
    load_r(P1, colP1, RP1);
    load_l(P1, LP1);
    uint32_t colP2 = load_col(P2);

    float m[KS], ls[KS], Lr[KS];
#pragma unroll
    for (int j = 0; j < KS; ++j) { m[j] = -INFINITY; ls[j] = 0.f; Lr[j] = 0.f; }
    // Accumulators as packed FP32 pairs (fma.rn.f32x2 rounds each half like fmaf).
    F2 acc[VPL][VEC / 2];
#pragma unroll
    for (int j = 0; j < VPL; ++j)
#pragma unroll
        for (int k = 0; k < VEC / 2; ++k) acc[j][k] = f2zero();

    // Consumes the chunk in slot `sl` (its copies must be complete and visible).
    auto consume = [&](int sl) {
        const SlotT& S = slots[sl];
        const int flags = S.flags, cnt = S.cnt;
        if (flags & kFirst) {
#pragma unroll
            for (int j = 0; j < VPL; ++j)
#pragma unroll
                for (int k = 0; k < VEC / 2; ++k) acc[j][k] = f2zero();
        } else if (!fixed) {
#pragma unroll
            for (int j = 0; j < VPL; ++j)
#pragma unroll
                for (int k = 0; k < VEC / 2; ++k) {
                    const float s0 = S.sc[MIXED ? hk[j][2 * k] : hv[j]];
                    const float s1 = S.sc[MIXED ? hk[j][2 * k + 1] : hv[j]];
                    acc[j][k] = f2mul(acc[j][k], f2make(s0, s1));
                }
        }
        const uint4* buf = bufs + size_t(sl) * C * RV;
#pragma unroll
        for (int i = 0; i < NT; ++i) {
            const int tt = es + i * EPS;
            if (tt < cnt) {
#pragma unroll
                for (int j = 0; j < VPL; ++j) {
                    const int v = vl + j * LPE;
                    if (NVC == 0 && v >= nvec) continue;
                    float f[VEC];
                    V::unpack(buf[tt * RV + v], f);
                    if constexpr (MIXED) {
#pragma unroll
                        for (int k = 0; k < VEC / 2; ++k)
                            acc[j][k] = f2fma(f2make(f[2 * k], f[2 * k + 1]),
                                              f2make(S.p[hk[j][2 * k] * PS + tt], S.p[hk[j][2 * k + 1] * PS + tt]),
                                              acc[j][k]);
                    } else {
                        const float pw = S.p[hv[j] * PS + tt];
                        const F2 pp = f2make(pw, pw);
#pragma unroll
                        for (int k = 0; k < VEC / 2; ++k) acc[j][k] = f2fma(f2make(f[2 * k], f[2 * k + 1]), pp, acc[j][k]);
                    }
                }
            }
        }
        if (!(flags & kLast)) return;
        // ---- item complete: combine edge slots, then store ----
        float out[VPL][VEC];
#pragma unroll
        for (int j = 0; j < VPL; ++j)
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
                float v = f2get(acc[j][k / 2], k & 1);
#pragma unroll
                for (int o = LPE; o < 32; o <<= 1) v += __shfl_xor_sync(kFull, v, o);
                out[j][k] = v;
            }
        if (flags & kPartial) {
            float* st = a.seg_state + S.item * kSegStateFloats;
            if (lane < K) {
                st[lane] = S.m[lane];
                st[8 + lane] = S.den[lane];
            }
            if (es == 0)
#pragma unroll
                for (int j = 0; j < VPL; ++j) {
                    const int v = vl + j * LPE;
                    if (NVC != 0 || v < nvec)
#pragma unroll
                        for (int k = 0; k < VEC; ++k) st[16 + v * VEC + k] = out[j][k];
                }
            return;
        }
        const uint64_t r = S.r;
        if (a.unnorm && lane < K) {
            a.den_out[r * K + lane] = a.fixed_den ? a.fixed_den[r * K + lane] : S.den[lane];
            if (a.max_out && !fixed) a.max_out[r * K + lane] = S.m[lane];
        }
        if (es == 0) {
#pragma unroll
            for (int j = 0; j < VPL; ++j) {
                const int v = vl + j * LPE;
                if (v * VEC >= a.ldo) continue;
                float o[VEC];
#pragma unroll
                for (int k = 0; k < VEC; ++k) {
                    const int hh = MIXED ? hk[j][k] : hv[j];
                    o[k] = finalize(a, v * VEC + k, out[j][k], S.den[hh]);
                }
                store_out<VEC>(a, r, v * VEC, o);
            }
        }
    };

    int prev = -1;
    for (int k = 0;; ++k) {
        const Rec S = P1;
        if (!(S.flags & kValid)) break;
        const uint32_t colS = colP1;
        float RS[KS], LS[KS];
#pragma unroll
        for (int j = 0; j < KS; ++j) { RS[j] = RP1[j]; LS[j] = LP1[j]; }
        // ---- advance the prefetch pipeline ----
        P1 = P2;
        colP1 = colP2;
        load_r(P1, colP1, RP1);
        load_l(P1, LP1);
        P2 = gen.next(a);
        colP2 = load_col(P2);

        // ---- 1. scores of chunk k ----
        const int sl = k & 1;
        SlotT& SL = slots[sl];
        __syncwarp();
        if (S.flags & kFirst) {
#pragma unroll
            for (int j = 0; j < KS; ++j) {
                m[j] = fixed ? 0.f : -INFINITY;
                ls[j] = 0.f;
                Lr[j] = LS[j];
            }
        }
        const bool ok = t < S.cnt;
#pragma unroll
        for (int j = 0; j < KS; ++j) {
            const int h = hs * KS + j;
            float p, sc;
            if (fixed) {
                p = ok ? RS[j] : 0.f;
                sc = 1.f;
            } else {
                const float s = ok ? leaky(Lr[j] + RS[j]) : -INFINITY;
                float cm = s;
#pragma unroll
                for (int o = 1; o < C; o <<= 1) cm = fmaxf(cm, __shfl_xor_sync(kFull, cm, o));
                const float nm = fmaxf(m[j], cm);
                sc = nm == -INFINITY ? 1.f : __expf(m[j] - nm);
                p = ok ? __expf(s - nm) : 0.f;
                m[j] = nm;
            }
            ls[j] = ls[j] * sc + p;
            if (h < KM) SL.p[h * PS + t] = p;
            if (t == 0 && h < 8) SL.sc[h] = sc;
        }
        if (S.flags & kLast) {
#pragma unroll
            for (int j = 0; j < KS; ++j) {
                const int h = hs * KS + j;
                float d = ls[j];
#pragma unroll
                for (int o = 1; o < C; o <<= 1) d += __shfl_xor_sync(kFull, d, o);
                if (t == 0 && h < 8) {
                    SL.den[h] = d;
                    SL.m[h] = (S.cnt == 0 || fixed) ? 0.f : m[j];
                }
            }
        }
        if (lane == 0) {
            SL.item = S.item;
            SL.r = S.r;
            SL.cnt = S.cnt;
            SL.flags = S.flags;
        }
        // ---- 2. gather chunk k's feature rows: lane (t, hs) copies vectors
        // hs, hs+SPL, ... of edge t's row into buffer k%2 ----
        if (ok) {
            const HT* row = H + uint64_t(colS) * a.ldh;
            const uint32_t dst = bufs_s + uint32_t(sl) * C * RV * 16 + uint32_t(t) * RV * 16;
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
                const int v = hs + i * SPL;
                if (v < RV && (NVC != 0 || v < nvec)) cp_async16(dst + uint32_t(v) * 16, row + v * VEC);
            }
        }
        cp_commit();
        // ---- 4. consume chunk k-1 ----
        if (prev >= 0) {
            cp_wait<1>();
            __syncwarp();
            consume(prev);
        }
        prev = sl;
    }
    if (prev >= 0) {
        cp_wait<0>();
        __syncwarp();
        consume(prev);
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

template <class HT, int KT, int C, int LPE, int VPL, bool MIXED, int NVC>
int launch_agg(const AggArgs& a, cudaStream_t st) {
    constexpr int KM = KT ? KT : 8;
    constexpr size_t warp_bytes = 2 * sizeof(Slot<C, KM>) + size_t(2) * C * LPE * VPL * 16;
    // Warps per block: up to 8 within ~100 KB of shared memory per block.
    constexpr int wpb = warp_bytes * 8 <= 100 * 1024 ? 8 : (warp_bytes * 4 <= 100 * 1024 ? 4 : 2);
    constexpr size_t smem = warp_bytes * wpb;
    auto kern = agg_kernel<HT, KT, C, LPE, VPL, MIXED, NVC>;
    static int grid = 0;  // resident blocks (per process; all B200s are alike)
    if (!grid) {
        int dev = 0, sms = 0, per_sm = 0;
        GATB_CUDA(cudaGetDevice(&dev));
        GATB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        GATB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
        GATB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, wpb * 32, smem));
        grid = sms * (per_sm > 0 ? per_sm : 1);
    }
    uint64_t items = uint64_t(a.n_seg) + (a.n - a.n_hub);
    uint64_t need = (items + wpb - 1) / wpb;
    unsigned blocks = unsigned(need < uint64_t(grid) ? need : uint64_t(grid));
    if (blocks == 0) blocks = 1;
    kern<<<blocks, wpb * 32, smem, st>>>(a);
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
            return launch_agg<uint16_t, 8, 16, 32, 1, false, 32>(a, st);
        if (heads == 1 && width <= 64) return launch_agg<uint16_t, 1, 32, 8, 1, false, 0>(a, st);
        return launch_agg<uint16_t, 0, 16, 32, 2, true, 0>(a, st);
    }
    if (heads == 8 && dim == 32 && (reinterpret_cast<uintptr_t>(left) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(right) & 15) == 0)
        return launch_agg<float, 8, 16, 32, 2, false, 64>(a, st);
    if (heads == 1 && width <= 64) return launch_agg<float, 1, 32, 16, 1, false, 0>(a, st);
    return launch_agg<float, 0, 16, 32, 4, true, 0>(a, st);
}

}  // namespace gatb
