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
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include <cuda.h>

#include "device.cuh"
#include "graph.cuh"
#include "tc.cuh"

namespace gatb {
int make_row_gather_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t ld,
                        uint32_t box_cols);
namespace {

constexpr int kWarps = 8;  // warps per block
constexpr unsigned kFull = 0xffffffffu;

struct AggArgs {
    const uint64_t* row;
    const uint32_t* col;
    const uint32_t* perm;
    uint64_t n;
    uint64_t n_src;          // rows of the feature table the source ids index
    uint32_t n_hub, n_seg;
    uint32_t n_wide;         // rows after the hubs with more than kWideRowEdges edges
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
    // BF16 outputs only: every output row is also stored, at the same row and
    // stride, into out_peer[j], j < npeer (other GPUs' tables mapped over
    // NVLink; the multi-GPU forward's layer-2 input exchange)
    int npeer;
    uint16_t* out_peer[7];
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
        const uint64_t off = r * uint64_t(a.ldo) + c0;
        uint16_t* o = static_cast<uint16_t*>(a.out) + off;
        if (a.out_vec && c0 + VECN <= a.ldo) {
            uint32_t w[VECN / 2];
#pragma unroll
            for (int k = 0; k < VECN / 2; ++k) w[k] = pack_bf16x2(v[2 * k], v[2 * k + 1]);
            if constexpr (VECN == 8) {
                const uint4 q = make_uint4(w[0], w[1], w[2], w[3]);
                *reinterpret_cast<uint4*>(o) = q;
                for (int j = 0; j < a.npeer; ++j) *reinterpret_cast<uint4*>(a.out_peer[j] + off) = q;
            } else if constexpr (VECN == 4) {
                const uint2 q = make_uint2(w[0], w[1]);
                *reinterpret_cast<uint2*>(o) = q;
                for (int j = 0; j < a.npeer; ++j) *reinterpret_cast<uint2*>(a.out_peer[j] + off) = q;
            } else {
                static_assert(VECN == 2, "2, 4 or 8 values");
                *reinterpret_cast<uint32_t*>(o) = w[0];
                for (int j = 0; j < a.npeer; ++j) *reinterpret_cast<uint32_t*>(a.out_peer[j] + off) = w[0];
            }
        } else {
#pragma unroll
            for (int k = 0; k < VECN; ++k)
                if (c0 + k < a.ldo) {
                    const uint16_t b = uint16_t(pack_bf16x2(v[k], 0.f) & 0xffffu);
                    o[k] = b;
                    for (int j = 0; j < a.npeer; ++j) a.out_peer[j][off + k] = b;
                }
        }
    } else {
        float* o = static_cast<float*>(a.out) + r * uint64_t(a.ldo) + c0;
        if (a.out_vec && c0 + VECN <= a.ldo) {
            if constexpr (VECN % 4 == 0) {
#pragma unroll
                for (int k = 0; k < VECN; k += 4)
                    *reinterpret_cast<float4*>(o + k) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
            } else {
                static_assert(VECN == 2, "2 or a multiple of 4 values");
                *reinterpret_cast<float2*>(o) = make_float2(v[0], v[1]);
            }
        } else {
#pragma unroll
            for (int k = 0; k < VECN; ++k)
                if (c0 + k < a.ldo) o[k] = v[k];
        }
    }
}

// Sum of n values over the lanes lane ^ O, lane ^ 2O, ... < 32 (the edge groups
// of a warp that share a feature vector), scattered: each lane ends with n /
// (32 / O) of the sums, starting at value k0. Each step adds the partner's
// half to the half this lane keeps, own value first, so every sum has the
// same operands in the same order as a butterfly over all n values.
template <int N, int O>
__device__ __forceinline__ void reduce_scatter(const float* in, float* out, int lane, int& k0) {
    if constexpr (O >= 32) {
#pragma unroll
        for (int i = 0; i < N; ++i) out[i] = in[i];
    } else {
        static_assert(N % 2 == 0, "values must halve at every step");
        const bool hi = (lane & O) != 0;
        float t[N / 2];
#pragma unroll
        for (int i = 0; i < N / 2; ++i) {
            const float keep = hi ? in[N / 2 + i] : in[i];
            const float send = hi ? in[i] : in[N / 2 + i];
            t[i] = keep + __shfl_xor_sync(0xffffffffu, send, O);
        }
        if (hi) k0 += N / 2;
        reduce_scatter<N / 2, 2 * O>(t, out, lane, k0);
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

// Kept for gat_b200_check_device (this kernel has no waits that can time out).
__device__ unsigned g_agg_error = 0;

// 16-byte cp.async; src_bytes = 0 reads nothing and zero-fills the slot.
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr), "l"(g), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Packed FP32 pair: sm_100 f32x2 arithmetic, each half rounded like fmaf.
__device__ __forceinline__ unsigned long long pk(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ unsigned long long ffma2(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ unsigned long long fmul2(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ float2 upk(unsigned long long a) {
    float2 f;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(f.x), "=f"(f.y) : "l"(a));
    return f;
}

enum : int { kValid = 1, kFirst = 2, kLast = 4, kPartial = 8 };

// One chunk of at most C edges of a work item (identical in every lane).
struct Rec {
    uint32_t item, r, pos;
    int cnt, flags;
};

// Chunk record handed from scoring to consuming through shared memory.
template <int C, int KM>
struct __align__(16) Slot {
    float p[KM * (C + 4)];  // p[h*(C+4) + t]: conflict-free stores and reads
    float sc[8];            // rescale of the running sums before this chunk
    float den[8];           // final sums (last chunk of an item)
    float m[8];             // final maxima (last chunk of an item)
    uint32_t item, r;
    int cnt, flags;
};

// Walks this warp's work items (gw, gw+G, ...) chunk by chunk: items below
// n_seg are hub-row segments, the rest rows in descending degree order. The
// bounds of the next item are prefetched one item ahead and the permutation
// entry of the item after it two items ahead. Edge positions fit 32 bits.
template <int C>
struct Gen {
    uint32_t total, G;
    uint32_t item, r, beg, pos, end;
    bool partial, have;
    uint32_t n_item, n_r, n_beg, n_end;
    bool n_partial, n_have;
    uint32_t nn_item, nn_r, nn_beg, nn_end;
    bool nn_partial, nn_have;

    __device__ __forceinline__ void stage1(const AggArgs& a, uint32_t it, uint32_t& rr, uint32_t& b, uint32_t& e,
                                           bool& part, bool& hv) const {
        hv = it < total;
        part = false;
        b = e = 0;
        rr = 0;
        if (!hv) return;
        if (it < a.n_seg) {
            const Segment* sg = a.segs + it;
            rr = sg->row;
            b = uint32_t(sg->beg);
            e = uint32_t(sg->end);
            part = true;
        } else {
            rr = a.perm[a.n - 1 - a.n_hub - (it - a.n_seg)];
        }
    }
    __device__ __forceinline__ void stage2(const AggArgs& a, uint32_t rr, uint32_t& b, uint32_t& e, bool part,
                                           bool hv) const {
        if (hv && !part) {
            b = uint32_t(a.row[rr]);
            e = uint32_t(a.row[rr + 1]);
        }
    }
    __device__ __forceinline__ void init(const AggArgs& a, uint32_t gw, uint32_t g_, uint32_t tot) {
        total = tot;
        G = g_;
        item = gw;
        stage1(a, item, r, beg, end, partial, have);
        stage2(a, r, beg, end, partial, have);
        pos = beg;
        n_item = gw + G;
        stage1(a, n_item, n_r, n_beg, n_end, n_partial, n_have);
        stage2(a, n_r, n_beg, n_end, n_partial, n_have);
        nn_item = n_item + G;
        stage1(a, nn_item, nn_r, nn_beg, nn_end, nn_partial, nn_have);
    }
    __device__ __forceinline__ Rec next(const AggArgs& a) {
        Rec rec;
        rec.item = item;
        rec.r = r;
        rec.pos = pos;
        rec.cnt = 0;
        rec.flags = 0;
        if (!have) return rec;
        const uint32_t rem = end - pos;
        rec.cnt = int(rem < uint32_t(C) ? rem : uint32_t(C));
        rec.flags = kValid | (pos == beg ? kFirst : 0) | (rem <= uint32_t(C) ? kLast : 0) | (partial ? kPartial : 0);
        pos += C;
        if (rem <= uint32_t(C)) {  // item finished: move to the next one
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
// C: edges per chunk. LPE lanes share a feature row when copying and
// consuming it, VPL 16-byte vectors each. MIXED: a vector may straddle heads.
//
// Scoring layout: lane = (edge offset eo, head slot h). With 8 head slots 4
// edges are scored per group (C/4 groups), so a head's chunk max and its row
// sum need 2 shuffle steps; with one head every lane scores its own edge.
//
// Per warp and loop iteration (chunk k):
//   1. scores of chunk k from col/R prefetched one and two iterations ago;
//      running max, rescale factor and p to the chunk's shared-memory slot;
//   2. cp.async of chunk k's feature rows into buffer k%2: lane (es, vl)
//      copies vector vl (+LPE...) of edges es, es+32/LPE, ..., the source id
//      arriving by shuffle from the scoring lane;
//   3. prefetch R of chunk k+1 and col of chunk k+2;
//   4. consume chunk k-1 (waiting only for this lane's own copies: a lane
//      consumes exactly the vectors it copied).
// Shared memory of one warp: the two chunk slots, the two row buffers and,
// with TG, the buffers' two mbarriers (128-byte aligned regions). A buffer
// holds C rows of RP 16-byte vectors in groups of four rows; with TG each
// group (one tile::gather4) starts on a 128-byte boundary.
template <int RP, bool TG>
__host__ __device__ constexpr int agg_group_bytes() {
    return TG ? (64 * RP + 127) / 128 * 128 : 64 * RP;
}
template <int C, int RP, bool TG>
__host__ __device__ constexpr size_t agg_buf_bytes() {
    return size_t(C / 4) * agg_group_bytes<RP, TG>();
}
template <int C, int KM, bool TG>
__host__ __device__ constexpr size_t agg_slot_bytes() {
    return TG ? (2 * sizeof(Slot<C, KM>) + 127) / 128 * 128 : 2 * sizeof(Slot<C, KM>);
}
template <int C, int KM, int RP, bool TG>
__host__ __device__ constexpr size_t agg_warp_bytes() {
    return TG ? (agg_slot_bytes<C, KM, TG>() + 2 * agg_buf_bytes<C, RP, TG>() + 16 + 127) / 128 * 128
              : agg_slot_bytes<C, KM, TG>() + 2 * agg_buf_bytes<C, RP, TG>();
}

// Bounded wait on a row buffer's mbarrier (TG): false after ~1 s, with the
// error flag raised.
__device__ __forceinline__ bool agg_wait(uint64_t* bar, uint32_t parity) {
    if (tc::mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
        if (tc::mbar_try(bar, parity)) return true;
        if ((it & 63) == 63) {
            __nanosleep(32);
            if (clock64() - t0 > (1ll << 31)) {
                atomicOr(&g_agg_error, 1u);
                return false;
            }
        }
    }
}

// TG (BF16 rows: the hidden layers' 8 heads x 32, 512 bytes, or a single
// head of NVC 16-byte vectors): each chunk's rows are fetched by the tensor
// memory accelerator instead of per-lane cp.async -- lane q issues one
// tile::gather4 of rows 4q..4q+3 (source ids past the chunk's end point
// outside the table and read as zeros, up to the consumer's granule of 4
// steps), the buffer's mbarrier counts the bytes, and the consumer waits on
// it (bounded).
template <class HT, int KT, int C, int LPE, int VPL, bool MIXED, int NVC, int MAXT, bool TG>
__global__ void __launch_bounds__(MAXT) agg_kernel(const AggArgs a, const __grid_constant__ CUtensorMap tmh) {
    using V = Vec<HT>;
    constexpr int VEC = V::N;
    constexpr int KM = KT ? KT : 8;
    constexpr int HS = KT == 1 ? 1 : 8;  // score lanes per edge
    constexpr int EG = 32 / HS;          // edges per score group
    constexpr int NG = C / EG;           // score groups per chunk
    constexpr int EPS = 32 / LPE;        // edges per copy/consume step
    constexpr int NT = C / EPS;          // copy/consume steps per chunk
    constexpr int RV = LPE * VPL;        // 16-byte vectors a lane group covers
    constexpr int RP = TG ? NVC : RV;    // 16-byte vectors per buffered row
    constexpr int GPB = agg_group_bytes<RP, TG>();
    constexpr int BUFV = int(agg_buf_bytes<C, RP, TG>() / 16);  // vectors per row buffer
    constexpr int PS = C + 4;            // p row stride (Slot::p): conflict-free for 8 heads x 4 offsets
    static_assert(NG >= 1 && NG * EG == C && NT * EPS == C, "bad tiling");
    static_assert(HS == 1 || LPE == 32, "8 head slots need whole-warp rows");
    using SlotT = Slot<C, KM>;

    static_assert(!TG || (sizeof(HT) == 2 && VPL == 1 &&
                          ((KT == 8 && C == 16 && LPE == 32 && NVC == 32) ||
                           (KT == 1 && C == 32 && LPE == 8 && NVC >= 1 && NVC <= 8))),
                  "the row gather serves BF16 rows of 8 x 32 or of one head up to 64 columns");
    // first vector of buffered row tt
    auto row_vec = [](int tt) { return ((tt >> 2) * GPB + (tt & 3) * RP * 16) / 16; };
    extern __shared__ __align__(128) uint8_t agg_smem[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    constexpr size_t kSlotBytes = agg_slot_bytes<C, KM, TG>();
    constexpr size_t kWarpBytes = agg_warp_bytes<C, KM, RP, TG>();
    uint8_t* wbase = agg_smem + wib * kWarpBytes;
    SlotT* slots = reinterpret_cast<SlotT*>(wbase);
    const uint4* bufs = reinterpret_cast<const uint4*>(wbase + kSlotBytes);
    const uint32_t bufs_s = static_cast<uint32_t>(__cvta_generic_to_shared(bufs));
    uint64_t* bars = reinterpret_cast<uint64_t*>(wbase + kSlotBytes + size_t(2) * BUFV * 16);
    uint32_t par = 0;  // TG: phase parity of the two buffers' barriers
    if constexpr (TG) {
        if (lane == 0) {
            tc::mbar_init(bars, 1);
            tc::mbar_init(bars + 1, 1);
            tc::fence_mbarrier_init();
        }
        __syncwarp();
    }

    const int K = KT ? KT : a.heads;
    const int eo = lane / HS, hh = lane % HS;    // scoring role
    const bool hok = KT == 8 || hh < K;
    const int es = lane / LPE, vl = lane % LPE;  // copy / consume role
    const int nvec = NVC ? NVC : (a.width + VEC - 1) / VEC;
    const uint64_t row_bytes = uint64_t(a.ldh) * sizeof(HT);
    const char* hbase = reinterpret_cast<const char*>(a.h) + vl * 16;
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

    const uint32_t total = uint32_t(a.n_seg + (a.n - a.n_hub));
    const uint32_t G = gridDim.x * (blockDim.x >> 5);
    Gen<C> gen;
    gen.init(a, blockIdx.x * (blockDim.x >> 5) + wib, G, total);

    auto load_col = [&](const Rec& rc, uint32_t (&o)[NG]) {
#pragma unroll
        for (int g = 0; g < NG; ++g) {
            const int e = g * EG + eo;
            o[g] = (rc.flags & kValid) && e < rc.cnt ? ldg_stream_u32(a.col + rc.pos + e) : 0u;
        }
    };
    auto load_r = [&](const Rec& rc, const uint32_t (&c)[NG], float (&o)[NG]) {
#pragma unroll
        for (int g = 0; g < NG; ++g) {
            const int e = g * EG + eo;
            const bool ok = (rc.flags & kValid) && e < rc.cnt && hok;
            if (fixed)
                o[g] = ok ? a.fixed_p[(uint64_t(rc.pos) + e) * K + hh] : 0.f;
            else
                o[g] = ok ? __ldg(a.right + uint64_t(c[g]) * K + hh) : 0.f;
        }
    };
    auto load_l = [&](const Rec& rc) -> float {
        return (rc.flags & kValid) && (rc.flags & kFirst) && hok && !fixed ? a.left[uint64_t(rc.r) * K + hh] : 0.f;
    };

    Rec P1 = gen.next(a);
    Rec P2 = gen.next(a);
    uint32_t colP1[NG], colP2[NG];
    float RP1[NG];
    load_col(P1, colP1);
    load_r(P1, colP1, RP1);
    float LP1 = load_l(P1);
    load_col(P2, colP2);

    float m = fixed ? 0.f : -INFINITY, ls = 0.f, Lr = 0.f;
    unsigned long long acc[VPL][VEC / 2];
#pragma unroll
    for (int j = 0; j < VPL; ++j)
#pragma unroll
        for (int k = 0; k < VEC / 2; ++k) acc[j][k] = 0ull;

    auto consume = [&](int sl) {
        const SlotT& S = slots[sl];
        const int flags = S.flags, cnt = S.cnt;
        if (flags & kFirst) {
#pragma unroll
            for (int j = 0; j < VPL; ++j)
#pragma unroll
                for (int k = 0; k < VEC / 2; ++k) acc[j][k] = 0ull;
        } else if (!fixed) {
#pragma unroll
            for (int j = 0; j < VPL; ++j)
#pragma unroll
                for (int k = 0; k < VEC / 2; ++k)
                    acc[j][k] = fmul2(acc[j][k], pk(S.sc[MIXED ? hk[j][2 * k] : hv[j]],
                                                    S.sc[MIXED ? hk[j][2 * k + 1] : hv[j]]));
        }
        const uint4* buf = bufs + size_t(sl) * BUFV;
        // Slots past cnt hold zero rows and p = 0, so groups of 4 steps run
        // without per-edge predicates.
#pragma unroll
        for (int i0 = 0; i0 < NT; i0 += 4) {
            if (i0 * EPS >= cnt) break;
#pragma unroll
            for (int u = 0; u < 4 && i0 + u < NT; ++u) {
                const int tt = es + (i0 + u) * EPS;
#pragma unroll
                for (int j = 0; j < VPL; ++j) {
                    const int v = vl + j * LPE;
                    if ((NVC == 0 || NVC < RV) && v >= nvec) continue;
                    float f[VEC];
                    V::unpack(buf[row_vec(tt) + v], f);
                    if constexpr (MIXED) {
#pragma unroll
                        for (int k = 0; k < VEC / 2; ++k)
                            acc[j][k] = ffma2(pk(f[2 * k], f[2 * k + 1]),
                                              pk(S.p[hk[j][2 * k] * PS + tt], S.p[hk[j][2 * k + 1] * PS + tt]),
                                              acc[j][k]);
                    } else {
                        const float pw = S.p[hv[j] * PS + tt];
                        const unsigned long long pp = pk(pw, pw);
#pragma unroll
                        for (int k = 0; k < VEC / 2; ++k) acc[j][k] = ffma2(pk(f[2 * k], f[2 * k + 1]), pp, acc[j][k]);
                    }
                }
            }
        }
        if (!(flags & kLast)) return;
        // ---- item complete ----
        float out[VPL][VEC];
#pragma unroll
        for (int j = 0; j < VPL; ++j)
#pragma unroll
            for (int k = 0; k < VEC / 2; ++k) {
                const float2 f = upk(acc[j][k]);
                out[j][2 * k] = f.x;
                out[j][2 * k + 1] = f.y;
            }
        if constexpr (EPS > 1) {
            // Narrow rows (EPS edge groups): the groups' sums are reduced and
            // scattered so that each lane finishes and stores VEC / EPS values
            // of its vector (the butterfly's sums, without its redundant copies).
            static_assert(!MIXED && VEC % EPS == 0, "narrow rows hold one head per vector");
            constexpr int VR = VEC / EPS;
            float red[VPL][VR];
            int k0 = 0;
#pragma unroll
            for (int j = 0; j < VPL; ++j) {
                k0 = 0;
                reduce_scatter<VEC, LPE>(out[j], red[j], lane, k0);
            }
            if (flags & kPartial) {
                float* st = a.seg_state + uint64_t(S.item) * kSegStateFloats;
                if (lane < K) {
                    st[lane] = S.m[lane];
                    st[8 + lane] = S.den[lane];
                }
#pragma unroll
                for (int j = 0; j < VPL; ++j) {
                    const int v = vl + j * LPE;
                    if (v < nvec)
#pragma unroll
                        for (int i = 0; i < VR; ++i) st[16 + v * VEC + k0 + i] = red[j][i];
                }
                return;
            }
            const uint64_t r = S.r;
            if (a.unnorm && lane < K) {
                a.den_out[r * K + lane] = a.fixed_den ? a.fixed_den[r * K + lane] : S.den[lane];
                if (a.max_out && !fixed) a.max_out[r * K + lane] = S.m[lane];
            }
#pragma unroll
            for (int j = 0; j < VPL; ++j) {
                const int v = vl + j * LPE;
                if (v * VEC >= a.ldo) continue;
                float o[VR];
#pragma unroll
                for (int i = 0; i < VR; ++i) o[i] = finalize(a, v * VEC + k0 + i, red[j][i], S.den[hv[j]]);
                store_out<VR>(a, r, v * VEC + k0, o);
            }
            return;
        }
        // whole-warp rows (EPS == 1): every lane holds its vector's sums
        if (flags & kPartial) {
            float* st = a.seg_state + uint64_t(S.item) * kSegStateFloats;
            if (lane < K) {
                st[lane] = S.m[lane];
                st[8 + lane] = S.den[lane];
            }
            if (es == 0)
#pragma unroll
                for (int j = 0; j < VPL; ++j) {
                    const int v = vl + j * LPE;
                    if (v < nvec)
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
                for (int k = 0; k < VEC; ++k)
                    o[k] = finalize(a, v * VEC + k, out[j][k], S.den[MIXED ? hk[j][k] : hv[j]]);
                store_out<VEC>(a, r, v * VEC, o);
            }
        }
    };

    int prev = -1;
    for (int k = 0;; ++k) {
        const Rec S = P1;
        if (!(S.flags & kValid)) break;
        uint32_t colS[NG];
        float RS[NG];
#pragma unroll
        for (int g = 0; g < NG; ++g) { colS[g] = colP1[g]; RS[g] = RP1[g]; }
        const float LS = LP1;
        // ---- advance the prefetch pipeline ----
        P1 = P2;
#pragma unroll
        for (int g = 0; g < NG; ++g) colP1[g] = colP2[g];
        load_r(P1, colP1, RP1);
        LP1 = load_l(P1);
        P2 = gen.next(a);
        load_col(P2, colP2);

        // ---- 1. scores of chunk k ----
        const int sl = k & 1;
        SlotT& SL = slots[sl];
        __syncwarp();
        if (S.flags & kFirst) {
            m = fixed ? 0.f : -INFINITY;
            ls = 0.f;
            Lr = LS;
        }
        float p[NG];
        float sc = 1.f;
        if (fixed) {
#pragma unroll
            for (int g = 0; g < NG; ++g) p[g] = RS[g];
        } else {
            float s[NG];
            float mx = -INFINITY;
#pragma unroll
            for (int g = 0; g < NG; ++g) {
                const bool ok = g * EG + eo < S.cnt && hok;
                const float x = Lr + RS[g];
                s[g] = ok ? fmaxf(x, 0.2f * x) : -INFINITY;  // leaky (gat.hpp:52), exactly
                mx = fmaxf(mx, s[g]);
            }
#pragma unroll
            for (int o = HS; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
            const float nm = fmaxf(m, mx);
            const float nms = nm == -INFINITY ? 0.f : nm;  // a chunk without edges
            sc = __expf(m - nms);  // 0 on an item's first chunk
            m = nm;
#pragma unroll
            for (int g = 0; g < NG; ++g) p[g] = __expf(s[g] - nms);  // exp(-inf) = 0 for empty slots
        }
        ls *= sc;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
            ls += p[g];
            if (hh < KM) SL.p[hh * PS + g * EG + eo] = p[g];
        }
        if (eo == 0 && hh < 8) SL.sc[hh] = sc;
        if (S.flags & kLast) {
            float d = ls;
#pragma unroll
            for (int o = HS; o < 32; o <<= 1) d += __shfl_xor_sync(kFull, d, o);
            if (eo == 0 && hh < 8) {
                SL.den[hh] = d;
                SL.m[hh] = (S.cnt == 0 || fixed) ? 0.f : m;
            }
        }
        if (lane == 0) {
            SL.item = S.item;
            SL.r = S.r;
            SL.cnt = S.cnt;
            SL.flags = S.flags;
        }
        // ---- 2. copy chunk k's feature rows (every slot: rows past cnt are
        // zero-filled without reading memory) ----
        // Groups of 4 steps, as in consume: slots up to the end of the last
        // group holding an edge are written, later groups are skipped.
        if constexpr (TG) {
            // lane q gathers edges 4q..4q+3; rows are fetched up to the end
            // of the consumer's last granule of 4 steps (4*EPS edges), those
            // past cnt as zeros from outside the table
            const uint32_t oob = uint32_t(a.n_src);
            uint32_t y[4] = {oob, oob, oob, oob};
            if constexpr (HS == 1) {
                // edge e is held by lane e in colS[0]
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int e = 4 * lane + j;
                    const uint32_t v = __shfl_sync(kFull, colS[0], e & 31);
                    if (e < S.cnt) y[j] = v;
                }
            } else {
                // edge g*4+j is held by lane j*HS in colS[g]
#pragma unroll
                for (int g = 0; g < NG; ++g)
#pragma unroll
                    for (int j = 0; j < EG; ++j) {
                        const uint32_t v = __shfl_sync(kFull, colS[g], j * HS);
                        if (g == lane && g * EG + j < S.cnt) y[j] = v;
                    }
            }
            const int ngrp = (S.cnt + 4 * EPS - 1) / (4 * EPS) * EPS;
            if (lane == 0) tc::mbar_expect_tx(bars + sl, uint32_t(ngrp) * 4u * RP * 16u);
            __syncwarp();
            if (lane < ngrp) {
                tc::fence_proxy_async_smem();
                tc::tma_gather4(const_cast<uint4*>(bufs) + size_t(sl) * BUFV + size_t(lane) * (GPB / 16), &tmh,
                                bars + sl, 0, int(y[0]), int(y[1]), int(y[2]), int(y[3]));
            }
        } else {
            const uint32_t bs = bufs_s + uint32_t(sl) * BUFV * 16 + uint32_t(vl) * 16;
#pragma unroll
            for (int i0 = 0; i0 < NT; i0 += 4) {
                if (i0 * EPS >= S.cnt) break;
#pragma unroll
                for (int u = 0; u < 4 && i0 + u < NT; ++u) {
                    const int i = i0 + u;
                    const int tt = es + i * EPS;
                    const int g = (i * EPS) / EG;  // static: EPS == 1 or NG == 1
                    const uint32_t c = __shfl_sync(kFull, colS[g], (tt % EG) * HS);
                    const uint32_t nb = tt < S.cnt ? 16u : 0u;
                    const char* src = hbase + uint64_t(c) * row_bytes;
#pragma unroll
                    for (int j = 0; j < VPL; ++j) {
                        const int v = vl + j * LPE;
                        if (NVC != 0 || v < nvec)
                            cp_async16(bs + uint32_t(tt * RV + j * LPE) * 16, src + j * LPE * 16, nb);
                    }
                }
            }
            cp_commit();
        }
        __syncwarp();
        // ---- 4. consume chunk k-1 ----
        if (prev >= 0) {
            if constexpr (TG) {
                if (!agg_wait(bars + prev, (par >> prev) & 1u)) return;
                par ^= 1u << prev;
            } else {
                cp_wait<1>();
            }
            consume(prev);
        }
        prev = sl;
    }
    if (prev >= 0) {
        if constexpr (TG) {
            if (!agg_wait(bars + prev, (par >> prev) & 1u)) return;
        } else {
            cp_wait<0>();
        }
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
        if (a.out_bf16) {
            const uint16_t b = uint16_t(pack_bf16x2(v, 0.f) & 0xffffu);
            static_cast<uint16_t*>(a.out)[r * a.ldo + c] = b;
            for (int j = 0; j < a.npeer; ++j) a.out_peer[j][r * a.ldo + c] = b;
        } else {
            static_cast<float*>(a.out)[r * a.ldo + c] = v;
        }
    }
}

// ---- narrow single-head layers: two lanes per row -------------------------
// For heads == 1 with a BF16 row of at most 64 features (layer 3, 1 x C with
// C <= 64: 96 bytes on c4) a whole warp per row and chunk spends most of its
// issue slots on chunk and row bookkeeping. Here a pair of lanes walks a
// row's edges in blocks of 4, each lane accumulating its half of the row's
// 16-byte vectors (NVH of them) in registers:
//  * the block's four source ids and scores arrive one block ahead;
//  * the running maximum moves once per block (the sums are rescaled then,
//    as the warp kernel does per chunk);
//  * the four rows' half-vectors (4 * NVH loads) are issued together and
//    consumed in edge order with FP32 FMAs.
// Work units, dealt round-robin to warps in the warp kernel's order (largest
// first): a "wide" item -- a hub segment, or a row of more than
// kWideRowEdges edges -- takes a whole warp, its 16 pairs taking every 16th
// block and combining their (max, sum, acc) states by shuffles at the end;
// the remaining rows go 16 to a warp, one pair each (their degrees are nearly
// equal in that order). Hub segments leave their state for hub_merge_kernel,
// as the warp kernel does. No shared memory.
template <int NVH>
__device__ __forceinline__ void pair_walk(const AggArgs& a, const char* hb, uint64_t rowb, int nvec, int v0,
                                          float L, uint64_t first, uint64_t end, uint64_t step, float& m,
                                          float& den, unsigned long long (&acc)[NVH * 4]) {
    uint32_t src[4];
    float sco[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const bool ok = first + k < end;
        src[k] = ok ? __ldg(a.col + first + k) : 0u;
        const float x = ok ? L + __ldg(a.right + src[k]) : 0.f;
        sco[k] = ok ? fmaxf(x, 0.2f * x) : -INFINITY;
    }
    for (uint64_t e = first; e < end; e += step) {
        uint4 rows[4][NVH];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const char* sp = hb + uint64_t(src[k]) * rowb;
            const bool ok = e + k < end;
#pragma unroll
            for (int j = 0; j < NVH; ++j)
                rows[k][j] = (ok && v0 + j < nvec) ? ldg_nc_v4(sp + j * 16) : make_uint4(0, 0, 0, 0);
        }
        uint32_t nsrc[4];
        float nsco[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const bool ok = e + step + k < end;
            nsrc[k] = ok ? __ldg(a.col + e + step + k) : 0u;
            const float x = ok ? L + __ldg(a.right + nsrc[k]) : 0.f;
            nsco[k] = ok ? fmaxf(x, 0.2f * x) : -INFINITY;
        }
        const float bm = fmaxf(fmaxf(sco[0], sco[1]), fmaxf(sco[2], sco[3]));
        if (bm > m) {
            const float sc = __expf(m - bm);  // 0 before the first block
            den *= sc;
            const unsigned long long ss = pk(sc, sc);
#pragma unroll
            for (int k = 0; k < NVH * 4; ++k) acc[k] = fmul2(acc[k], ss);
            m = bm;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float p = __expf(sco[k] - m);  // 0 past the end
            den += p;
            const unsigned long long pp = pk(p, p);
#pragma unroll
            for (int j = 0; j < NVH; ++j) {
                float f[8];
                Vec<uint16_t>::unpack(rows[k][j], f);
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[j * 4 + q] = ffma2(pk(f[2 * q], f[2 * q + 1]), pp, acc[j * 4 + q]);
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            src[k] = nsrc[k];
            sco[k] = nsco[k];
        }
    }
}

// Item `it` of the warp kernel's order: a hub segment (it < n_seg) or a row.
__device__ __forceinline__ void pair_item(const AggArgs& a, uint64_t it, uint64_t& r, uint64_t& beg, uint64_t& end,
                                          bool& partial) {
    if (it < a.n_seg) {
        const Segment sg = a.segs[it];
        r = sg.row;
        beg = sg.beg;
        end = sg.end;
        partial = true;
    } else {
        r = a.perm[a.n - 1 - a.n_hub - (it - a.n_seg)];
        beg = a.row[r];
        end = a.row[r + 1];
        partial = false;
    }
}

template <int NVH>
__device__ __forceinline__ void pair_emit(const AggArgs& a, uint64_t it, uint64_t r, bool partial, int half, int v0,
                                          float m, float den, const unsigned long long (&acc)[NVH * 4]) {
    constexpr int NF = NVH * 8;
    const int c0 = v0 * 8;
    if (partial) {
        float* st = a.seg_state + it * kSegStateFloats;
        if (half == 0) {
            st[0] = m;
            st[8] = den;
        }
#pragma unroll
        for (int k = 0; k < NF / 2; ++k) {
            const float2 f = upk(acc[k]);
            if (c0 + 2 * k < a.width) st[16 + c0 + 2 * k] = f.x;
            if (c0 + 2 * k + 1 < a.width) st[16 + c0 + 2 * k + 1] = f.y;
        }
        return;
    }
    const float inv = den > 0.f ? 1.f / den : 0.f;
#pragma unroll
    for (int k = 0; k < NF / 2; ++k) {
        const float2 f = upk(acc[k]);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int c = c0 + 2 * k + t;
            if (c >= a.ldo) continue;
            float v = c < a.width ? (t ? f.y : f.x) * inv : 0.f;
            if (a.hidden && v < 0.f) v = __expf(v) - 1.f;  // the B0 activation (gat.hpp:57-62)
            if (a.out_bf16)
                static_cast<uint16_t*>(a.out)[r * a.ldo + c] = uint16_t(pack_bf16x2(v, 0.f) & 0xffffu);
            else
                static_cast<float*>(a.out)[r * a.ldo + c] = v;
        }
    }
    if (half == 1)  // padding columns past both lanes' vectors
        for (int c = 2 * NF; c < a.ldo; ++c) {
            if (a.out_bf16)
                static_cast<uint16_t*>(a.out)[r * a.ldo + c] = 0;
            else
                static_cast<float*>(a.out)[r * a.ldo + c] = 0.f;
        }
}

template <int NVH>
__global__ void __launch_bounds__(128) agg_pair_kernel(const AggArgs a) {
    const int lane = threadIdx.x & 31, half = lane & 1, pair = lane >> 1;
    const uint64_t total = uint64_t(a.n_seg) + (a.n - a.n_hub);
    const uint64_t n_big = uint64_t(a.n_seg) + a.n_wide;
    const uint64_t units = n_big + (total - n_big + 15) / 16;
    const uint64_t G = uint64_t(gridDim.x) * (blockDim.x >> 5);
    const int nvec = (a.width + 7) / 8;
    const int v0 = half * NVH;  // first vector of this lane
    const char* hb = static_cast<const char*>(a.h) + v0 * 16;
    const uint64_t rowb = uint64_t(a.ldh) * 2;
    for (uint64_t u = blockIdx.x * uint64_t(blockDim.x >> 5) + (threadIdx.x >> 5); u < units; u += G) {
        unsigned long long acc[NVH * 4];
#pragma unroll
        for (int k = 0; k < NVH * 4; ++k) acc[k] = 0ull;
        float m = -INFINITY, den = 0.f;
        uint64_t r, beg, end;
        bool partial;
        if (u < n_big) {
            // a wide item: pair q takes blocks q, q+16, ... of its edges
            pair_item(a, u, r, beg, end, partial);
            const float L = a.left[r];
            pair_walk<NVH>(a, hb, rowb, nvec, v0, L, beg + 4 * uint64_t(pair), end, 64, m, den, acc);
#pragma unroll
            for (int o = 2; o < 32; o <<= 1) {  // combine the 16 pairs' states (same half)
                const float mo = __shfl_xor_sync(kFull, m, o);
                const float dn = __shfl_xor_sync(kFull, den, o);
                const float M = fmaxf(m, mo);
                const float fa = m == -INFINITY ? 0.f : __expf(m - M);
                const float fb = mo == -INFINITY ? 0.f : __expf(mo - M);
                den = den * fa + dn * fb;
                const unsigned long long pa = pk(fa, fa), pb = pk(fb, fb);
#pragma unroll
                for (int k = 0; k < NVH * 4; ++k) {
                    const float2 x = upk(acc[k]);
                    const unsigned long long other =
                        pk(__shfl_xor_sync(kFull, x.x, o), __shfl_xor_sync(kFull, x.y, o));
                    acc[k] = ffma2(other, pb, fmul2(acc[k], pa));
                }
                m = M;
            }
            if (pair == 0) pair_emit<NVH>(a, u, r, partial, half, v0, m, den, acc);
        } else {
            const uint64_t it = n_big + (u - n_big) * 16 + pair;
            if (it >= total) continue;
            pair_item(a, it, r, beg, end, partial);
            const float L = a.left[r];
            pair_walk<NVH>(a, hb, rowb, nvec, v0, L, beg, end, 4, m, den, acc);
            pair_emit<NVH>(a, it, r, partial, half, v0, m, den, acc);
        }
    }
}

template <int NVH>
int launch_agg_pair(const AggArgs& a, cudaStream_t st, int reserve_sms) {
    int dev = 0, sms = 0;
    GATB_CUDA(cudaGetDevice(&dev));
    GATB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    static int per_sm = 0;
    if (!per_sm) {
        GATB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, agg_pair_kernel<NVH>, 128, 0));
        if (per_sm < 1) per_sm = 1;
    }
    const int usable = reserve_sms > 0 && reserve_sms < sms ? sms - reserve_sms : sms;
    const uint64_t items = uint64_t(a.n_seg) + (a.n - a.n_hub);
    const uint64_t n_big = uint64_t(a.n_seg) + a.n_wide;
    const uint64_t need = (n_big + (items - n_big + 15) / 16 + 3) / 4;  // 4 warps per block
    const uint64_t cap = uint64_t(usable) * per_sm;
    const unsigned blocks = unsigned(std::max<uint64_t>(1, std::min(need, cap)));
    agg_pair_kernel<NVH><<<blocks, 128, 0, st>>>(a);
    GATB_LAUNCH("edge-softmax aggregation kernel (lane pair per row)");
    if (a.n_hub) {
        hub_merge_kernel<<<(a.n_hub + kWarps - 1) / kWarps, kWarps * 32, 0, st>>>(a);
        GATB_LAUNCH("hub merge kernel");
    }
    return 0;
}

// Narrow single-head layers (heads == 1, width <= 64, BF16) run on the warp
// kernel (eight lanes per gathered row, one 16-byte vector each);
// GAT_B200_NARROW_AGG=pair selects the lane-pair kernel above instead (both
// compute the whole layer). Measured on c4 layer 3 (1 x 47, one B200): warp
// kernel 3.76-4.06 ms, lane pair 4.02-4.21 ms. Two other layouts were
// measured and dropped: one lane per row (8.2 ms: each lane's chain of
// dependent loads -- source id, then score and row -- leaves it
// latency-bound at 14 % issue activity) and the warp kernel with two lanes
// per row and three vectors each (7.6 ms: 166 registers, 12 warps per SM).
// Hidden layers (8 x 32 BF16) fetch their rows with per-lane cp.async; with
// GAT_B200_HIDDEN_AGG=gather4 the tensor memory accelerator's row gather
// (tile::gather4) does it. Both compute the whole layer.
bool hidden_row_gather() {
    static const bool v = [] {
        const char* e = std::getenv("GAT_B200_HIDDEN_AGG");
        return e && std::strcmp(e, "gather4") == 0;
    }();
    return v;
}

bool narrow_on_pairs() {
    static const bool v = [] {
        const char* e = std::getenv("GAT_B200_NARROW_AGG");
        return e && std::strcmp(e, "pair") == 0;
    }();
    return v;
}

bool narrow_row_gather() {
    static const bool v = [] {
        const char* e = std::getenv("GAT_B200_NARROW_AGG");
        return e && std::strcmp(e, "gather4") == 0;
    }();
    return v;
}

// reserve_sms = 0: blocks of up to 4 warps, as many resident blocks as fit
// on every SM. reserve_sms > 0 (the multi-GPU forward, where a projection
// kernel on another stream runs beside the aggregation): one block per SM
// with as many warps as fit in its shared memory (so no other kernel's CTA
// can share the SM), on all but reserve_sms SMs, which stay free for the
// other kernel.
template <class HT, int KT, int C, int LPE, int VPL, bool MIXED, int NVC, bool TG = false>
int launch_agg(const AggArgs& a, cudaStream_t st, int reserve_sms) {
    constexpr int KM = KT ? KT : 8;
    constexpr int RP = TG ? NVC : LPE * VPL;  // 16-byte vectors per buffered row
    constexpr size_t warp_bytes = agg_warp_bytes<C, KM, RP, TG>();
    CUtensorMap tmh;
    std::memset(&tmh, 0, sizeof(tmh));
    if constexpr (TG) {
        // boxes of one row of RP vectors (8 BF16 each)
        int rc = make_row_gather_map(&tmh, a.h, uint64_t(a.ldh), a.n_src, uint64_t(a.ldh), uint32_t(RP * 8));
        if (rc) return rc;
    }
    // Up to 4 warps per block within 200 KB of shared memory.
    constexpr int wpb = warp_bytes * 4 <= 200 * 1024 ? 4 : (warp_bytes * 2 <= 200 * 1024 ? 2 : 1);
    constexpr int wbig_fit = int((220 * 1024) / warp_bytes);
    constexpr int wbig = wbig_fit > 16 ? 16 : (wbig_fit < 1 ? 1 : wbig_fit);
    static_assert(warp_bytes * wbig > 114 * 1024 || wbig == 16, "one block per SM needs most of its shared memory");
    uint64_t items = uint64_t(a.n_seg) + (a.n - a.n_hub);
    int dev = 0, sms = 0;
    GATB_CUDA(cudaGetDevice(&dev));
    GATB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if (reserve_sms > 0 && reserve_sms < sms) {
        constexpr size_t smem = warp_bytes * wbig;
        auto kern = agg_kernel<HT, KT, C, LPE, VPL, MIXED, NVC, wbig * 32, TG>;
        static bool attr = false;
        if (!attr) {
            GATB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
            attr = true;
        }
        uint64_t need = (items + wbig - 1) / wbig;
        unsigned blocks = unsigned(need < uint64_t(sms - reserve_sms) ? need : uint64_t(sms - reserve_sms));
        if (blocks == 0) blocks = 1;
        kern<<<blocks, wbig * 32, smem, st>>>(a, tmh);
        GATB_LAUNCH("edge-softmax aggregation kernel");
    } else {
        constexpr size_t smem = warp_bytes * wpb;
        auto kern = agg_kernel<HT, KT, C, LPE, VPL, MIXED, NVC, 128, TG>;
        static int grid = 0;  // resident blocks (per process; all B200s are alike)
        if (!grid) {
            int per_sm = 0;
            GATB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
            GATB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, wpb * 32, smem));
            grid = sms * (per_sm > 0 ? per_sm : 1);
        }
        uint64_t need = (items + wpb - 1) / wpb;
        unsigned blocks = unsigned(need < uint64_t(grid) ? need : uint64_t(grid));
        if (blocks == 0) blocks = 1;
        kern<<<blocks, wpb * 32, smem, st>>>(a, tmh);
        GATB_LAUNCH("edge-softmax aggregation kernel");
    }
    if (a.n_hub) {
        hub_merge_kernel<<<(a.n_hub + kWarps - 1) / kWarps, kWarps * 32, 0, st>>>(a);
        GATB_LAUNCH("hub merge kernel");
    }
    return 0;
}

}  // namespace

int aggregate_check_error() {
    unsigned e = 0;
    GATB_CUDA(cudaMemcpyFromSymbol(&e, g_agg_error, sizeof(e)));
    if (e) {
        unsigned z = 0;
        cudaMemcpyToSymbol(g_agg_error, &z, sizeof(z));
        return fail_code(GAT_B200_ETIMEOUT, "aggregation kernel: a bounded wait on a row copy timed out");
    }
    return 0;
}

int aggregate_dispatch_reserved(const gat_b200_graph* g, int heads, int dim, const void* h, int h_dtype, int ldh,
                                const float* left, const float* right, const float* fixed_p, const float* fixed_den,
                                int unnorm, int hidden, void* out, int out_bf16, int ldo, float* den, float* max,
                                cudaStream_t st, int reserve_sms, int npeer = 0, uint16_t* const* out_peer = nullptr);

int aggregate_dispatch(const gat_b200_graph* g, int heads, int dim, const void* h, int h_dtype, int ldh,
                       const float* left, const float* right, const float* fixed_p, const float* fixed_den,
                       int unnorm, int hidden, void* out, int out_bf16, int ldo, float* den, float* max,
                       cudaStream_t st) {
    return aggregate_dispatch_reserved(g, heads, dim, h, h_dtype, ldh, left, right, fixed_p, fixed_den, unnorm, hidden,
                                       out, out_bf16, ldo, den, max, st, 0);
}

// npeer > 0 (BF16 hidden outputs only): every output row is also stored into
// out_peer[j] (other GPUs' tables, each offset like out), by the warp kernel.
int aggregate_dispatch_reserved(const gat_b200_graph* g, int heads, int dim, const void* h, int h_dtype, int ldh,
                                const float* left, const float* right, const float* fixed_p, const float* fixed_den,
                                int unnorm, int hidden, void* out, int out_bf16, int ldo, float* den, float* max,
                                cudaStream_t st, int reserve_sms, int npeer, uint16_t* const* out_peer) {
    if (npeer < 0 || npeer > 7) return fail("aggregate: at most 7 peer outputs");
    if (npeer && (!out_bf16 || unnorm || !out_peer)) return fail("aggregate: peer outputs need BF16 output rows");
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
    if (g->e >= (1ull << 32) - 64) return fail_code(GAT_B200_EUNSUPPORTED, "aggregate: more than 2^32 edges");
    AggArgs a{};
    a.row = g->row;
    a.col = g->col;
    a.perm = g->perm;
    a.n = g->n;
    a.n_src = g->n_src ? g->n_src : g->n;
    a.n_hub = g->n_hub;
    a.n_seg = g->n_seg;
    a.n_wide = g->n_wide;
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
    a.npeer = npeer;
    for (int j = 0; j < npeer; ++j) {
        if (!out_peer[j]) return fail("aggregate: null peer output");
        a.out_peer[j] = static_cast<uint16_t*>(out_peer[j]);
    }
    if (h_dtype == GAT_B200_BF16) {
        if (heads == 8 && dim == 32 && (reinterpret_cast<uintptr_t>(left) & 15) == 0 &&
            (reinterpret_cast<uintptr_t>(right) & 15) == 0) {
            if (ldh >= 256 && a.n_src < (1ull << 31) && hidden_row_gather())
                return launch_agg<uint16_t, 8, 16, 32, 1, false, 32, true>(a, st, reserve_sms);
            return launch_agg<uint16_t, 8, 16, 32, 1, false, 32>(a, st, reserve_sms);
        }
        if (heads == 1 && width <= 64) {
            const int nv = (width + 7) / 8;
            if (narrow_on_pairs() && !fixed_p && !unnorm && npeer == 0) {
                // the lane-pair kernel serves the fused epilogue only
                const int nvh = (nv + 1) / 2;
                if (nvh <= 1) return launch_agg_pair<1>(a, st, reserve_sms);
                if (nvh <= 2) return launch_agg_pair<2>(a, st, reserve_sms);
                if (nvh <= 3) return launch_agg_pair<3>(a, st, reserve_sms);
                return launch_agg_pair<4>(a, st, reserve_sms);
            }
            if (narrow_row_gather() && ldh >= nv * 8 && a.n_src < (1ull << 31)) {
                // rows of nv vectors through the TMA row gather
                switch (nv) {
                    case 1: return launch_agg<uint16_t, 1, 32, 8, 1, false, 1, true>(a, st, reserve_sms);
                    case 2: return launch_agg<uint16_t, 1, 32, 8, 1, false, 2, true>(a, st, reserve_sms);
                    case 3: return launch_agg<uint16_t, 1, 32, 8, 1, false, 3, true>(a, st, reserve_sms);
                    case 4: return launch_agg<uint16_t, 1, 32, 8, 1, false, 4, true>(a, st, reserve_sms);
                    case 5: return launch_agg<uint16_t, 1, 32, 8, 1, false, 5, true>(a, st, reserve_sms);
                    case 6: return launch_agg<uint16_t, 1, 32, 8, 1, false, 6, true>(a, st, reserve_sms);
                    case 7: return launch_agg<uint16_t, 1, 32, 8, 1, false, 7, true>(a, st, reserve_sms);
                    default: return launch_agg<uint16_t, 1, 32, 8, 1, false, 8, true>(a, st, reserve_sms);
                }
            }
            return launch_agg<uint16_t, 1, 32, 8, 1, false, 0>(a, st, reserve_sms);
        }
        return launch_agg<uint16_t, 0, 16, 32, 2, true, 0>(a, st, reserve_sms);
    }
    if (heads == 8 && dim == 32 && (reinterpret_cast<uintptr_t>(left) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(right) & 15) == 0)
        return launch_agg<float, 8, 16, 32, 2, false, 64>(a, st, reserve_sms);
    if (heads == 1 && width <= 64) return launch_agg<float, 1, 32, 16, 1, false, 0>(a, st, reserve_sms);
    return launch_agg<float, 0, 16, 32, 4, true, 0>(a, st, reserve_sms);
}

}  // namespace gatb
