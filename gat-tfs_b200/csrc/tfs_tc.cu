// Tensor-core TFS aggregation (sm_100a: tcgen05 + TMEM, cp.async gathers).
//
// Semantics: baseline/tfs_online/icpp_heads_hybrid.cpp with one block per
// destination row (hub rows: one block per segment) and the prescan maximum:
//   p_ij  = exp(leaky(L_ih + R_jh) - m_ih),   p = p_hi + p_lo (two BF16 values)
//   U_ih  = sum_j p_hi x_j + sum_j p_lo x_j   (FP32 accumulation, tensor cores)
//   V_ih  = RNE(U_ih) . RNE(W_h)              (FP32 accumulation, tensor cores)
//   den_ih = sum_j p_ij   (the same tensor-core sum: feature row 127 of the
//                         gathered tile holds 1.0 for every neighbour)
// then finish (V/den, ELU) and the BF16 or FP32 store, or the unnormalized V
// and den of gat_b200_tfs_aggregate.
//
// Work: the degree-sorted items of the aggregation (hub segments, then rows in
// descending degree) in groups of 8; CTA b takes groups b, b+grid, ... Every
// item is cut into chunks of 16 neighbours; a chunk is one K=16 step of
//   PH:  D[f][(hi|lo, h)] += X^T[f][j] . P[j][(hi|lo, h)]   M=128 (features),
//        N=16, A = gathered X rows (MN-major), B = the chunk's p split (K-major)
// into the item's 16 TMEM columns. When a group's chunks are done, U (high +
// low columns) is rounded to BF16 into shared memory and
//   UW:  D[(h',c)][(slot, h)] += W^T[(h',c)][f] . U[f][(slot, h)]  M=128, N=64
// projects all 8 items at once (only the h == h' columns are kept).
//
// Warps: 0-7 producers (neighbour ids, R gathers, p, P tiles, cp.async of X
// rows into a 6-stage ring of 64 neighbours; warp w fills position w%4 of the
// stages of parity w/4), 8 TMEM owner and MMA issuer, 9-12 epilogue (U
// rounding, den, UW readout, output). TMEM: two group buffers of 256 columns (8 x 16 PH
// columns + 2 x 64 UW columns). Every wait is bounded (about 1 s) and records
// GAT_B200_ETIMEOUT. No cluster launch and no multicast.
#include <algorithm>

#include "device.cuh"
#include "graph.cuh"
#include "tc.cuh"

namespace gatb {

__device__ unsigned g_tfs_error = 0;

namespace {

using namespace tc;

constexpr int kStages = 6;
constexpr int kABytes = 16384;  // X^T stage: 2 M-atoms (features 0-63, 64-127) x 8 K-atoms (64 neighbours)
constexpr int kPBytes = 2048;   // P stage: 16 rows (8 high, 8 low) x 64 neighbours
constexpr int kDescBytes = 16;  // per stage: the flags of its 4 chunks
constexpr int kOnesRow = 127;   // feature row of the gathered tile that holds 1.0 (den)
constexpr int kWBytes = 32768;  // W^T half: 128 rows x 128 features
constexpr int kUBytes = 16384;  // U tile: 128 features x 64 columns (8 slots x 8 heads)
constexpr int kProd = 8;                    // producer warps 0-7
constexpr int kMma0 = kProd;                // MMA warps 8-11 (warp 8 also owns TMEM)
constexpr int kMmaWarps = 4;
constexpr int kEpi0 = kMma0 + kMmaWarps;    // epilogue warps 12-15
constexpr int kThreads = (kEpi0 + 4) * 32;  // 512
constexpr int kSegFloats = 8 * 64 + 16;

// chunk flag bits
constexpr uint32_t F_SLOT = 7u;
constexpr uint32_t F_FIRST_ITEM = 1u << 3;
constexpr uint32_t F_VALID = 1u << 4;
constexpr uint32_t F_LAST_GROUP = 1u << 5;
constexpr uint32_t F_GB = 1u << 6;
constexpr uint32_t F_FIRST_GROUP = 1u << 7;
constexpr uint32_t F_END = 1u << 8;   // last chunk of the CTA's stream
constexpr uint32_t F_NONE = 1u << 9;  // position past the end of the stream

struct TcArgs {
    const uint64_t* row;
    const uint32_t* col;
    const uint32_t* perm;
    const Segment* segs;
    uint64_t n;
    uint32_t n_hub, n_seg;
    uint64_t n_items, n_groups;
    int in, heads, dim, width, ch, mh, ksteps;
    const uint16_t* x;
    int ldx;
    const uint16_t* wt;
    int kp, np;
    const float* left;
    const float* right;
    const float* max;
    int norm, hidden, out_bf16;
    void* out;
    int ldo;
    float* den_out;
    float* seg_state;
    int uniform_head;  // dim divides 32: each warp's output rows belong to one head
};

struct Item {
    uint64_t beg, end;
    uint32_t row;
    int seg;  // segment index, -1 for a whole row
};

__device__ __forceinline__ Item item_info(const TcArgs& a, uint64_t it) {
    Item r;
    if (it < a.n_seg) {
        const Segment s = a.segs[it];
        r.row = s.row;
        r.beg = s.beg;
        r.end = s.end;
        r.seg = int(it);
    } else {
        const uint32_t rr = a.perm[a.n - 1 - a.n_hub - (it - a.n_seg)];
        r.row = rr;
        r.beg = a.row[rr];
        r.end = a.row[rr + 1];
        r.seg = -1;
    }
    return r;
}

__device__ __forceinline__ uint16_t rne16(float x) {
    uint16_t r;
    asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ float bf(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

__global__ void __launch_bounds__(kThreads, 1) tfs_tc_kernel(const TcArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a_s = smem;                                  // kStages x 16 KB
    uint8_t* p_s = a_s + kStages * kABytes;               // kStages x 2 KB
    uint8_t* w_s = p_s + kStages * kPBytes;               // 2 x 32 KB
    uint8_t* u_s = w_s + 2 * kWBytes;                     // 2 x 16 KB
    uint8_t* d_s = u_s + 2 * kUBytes;                     // kStages x kDescBytes
    float* den_epi = reinterpret_cast<float*>(d_s + kStages * kDescBytes);  // [2][8 slots][8 heads]
    uint64_t* bars = reinterpret_cast<uint64_t*>(den_epi + 128);
    uint64_t* full = bars;                 // [kStages]
    uint64_t* empty = full + kStages;      // [kStages]
    uint64_t* ph_full = empty + kStages;   // [2]
    uint64_t* u_full = ph_full + 2;        // [2]
    uint64_t* uw_full = u_full + 2;        // [2]
    uint64_t* uw_empty = uw_full + 2;      // [2]
    uint64_t* mma_done = uw_empty + 2;     // 1
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = a.heads;

    // ---- setup: zero the X ring (feature columns past the row stay zero), load W^T
    for (int i = threadIdx.x; i < kStages * kABytes / 16; i += kThreads)
        reinterpret_cast<uint4*>(a_s)[i] = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < a.mh * 128 * 16; i += kThreads) {
        const int r = i >> 4, kc = i & 15;  // W^T row r (= output column h'*dim+c), 8-feature chunk kc
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < a.np && kc * 8 < a.kp) v = *reinterpret_cast<const uint4*>(a.wt + size_t(r) * a.kp + kc * 8);
        const int rr = r & 127, hf = r >> 7;
        uint8_t* dst = w_s + hf * kWBytes + (kc >> 3) * 16384 + (rr >> 3) * 1024 + (rr & 7) * 128 +
                       (((kc & 7) ^ (rr & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = v;
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full + s, 256);  // per producer thread: its copies landed + its stores done
            mbar_init(empty + s, kMmaWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(ph_full + b, kMmaWarps);
            mbar_init(u_full + b, 128);
            mbar_init(uw_full + b, a.mh);
            mbar_init(uw_empty + b, 128);
        }
        mbar_init(mma_done, kMmaWarps);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMma0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_proxy_async_smem();
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_holder;
    unsigned* err = &g_tfs_error;

    if (warp < kProd) {
        // ================= producers =================
        // Warp w fills position w%4 (16 neighbours) of the 64-neighbour stages q
        // with q%2 == w/4, so each warp has two stages' time to cover its loads.
        // Loads are pipelined along the warp's chunks: neighbour ids three ahead,
        // R / L / max two ahead, X rows by cp.async up to kStages stages ahead.
        const int w = warp & 3, par = warp >> 2;
        const int j = lane & 15, hb = (lane >> 4) * 4;
        const bool vec8 = K == 8;  // L, max, R rows of 8 heads: two float4 per row  // scoring lane: neighbour j, heads hb..hb+3
        uint64_t G = blockIdx.x;  // global group index of the group table
        uint64_t t = 0;           // its local index
        bool have = G < a.n_groups;
        uint64_t gstart = 0;      // stream chunk index where group t starts
        int gtotal = 0, gchunks = 1;
        uint64_t ibeg = 0, iend = 0, pbeg = 0, pend = 0;
        uint32_t irow = 0, prow = 0;
        int nch = 0, pre = 0;
        // item table of group Gx into (b, e, r) on lanes 0..7
        auto fetch = [&](uint64_t Gx, uint64_t& b, uint64_t& e, uint32_t& r) {
            const uint64_t it = Gx * 8 + uint64_t(lane);
            b = e = 0;
            r = 0;
            if (lane < 8 && Gx < a.n_groups && it < a.n_items) {
                const Item m = item_info(a, it);
                b = m.beg;
                e = m.end;
                r = m.row;
            }
        };
        auto take = [&]() {  // the prefetched table becomes group G's; prefetch the next one
            ibeg = pbeg;
            iend = pend;
            irow = prow;
            nch = int((iend - ibeg + 15) / 16);
            int x = nch;
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            pre = x - nch;
            gtotal = __shfl_sync(0xffffffffu, x, 7);
            gchunks = gtotal > 0 ? gtotal : 1;
            fetch(G + gridDim.x, pbeg, pend, prow);
        };
        fetch(G, pbeg, pend, prow);
        if (have) take();
        struct Chunk {
            uint32_t flags, row;
            uint64_t cb;
            int ne;
        };
        // description of stream chunk cc (called with increasing cc)
        auto chunk_at = [&](uint64_t cc) -> Chunk {
            while (have && cc >= gstart + uint64_t(gchunks)) {
                gstart += uint64_t(gchunks);
                ++t;
                G += gridDim.x;
                have = G < a.n_groups;
                if (have) take();
            }
            Chunk c{F_NONE, 0, 0, 0};
            if (!have) return c;
            const int loc = int(cc - gstart);
            const bool last_group = loc == gchunks - 1;
            c.flags = ((t & 1) ? F_GB : 0u) | (loc == 0 ? F_FIRST_GROUP : 0u) | (last_group ? F_LAST_GROUP : 0u) |
                      (last_group && G + gridDim.x >= a.n_groups ? F_END : 0u);
            if (gtotal > 0) {
                const unsigned m = __ballot_sync(0xffffffffu, lane < 8 && nch > 0 && pre <= loc);
                const int i = 31 - __clz(int(m));
                const uint64_t b_i = __shfl_sync(0xffffffffu, ibeg, i);
                const uint64_t e_i = __shfl_sync(0xffffffffu, iend, i);
                const int pre_i = __shfl_sync(0xffffffffu, pre, i);
                c.row = __shfl_sync(0xffffffffu, irow, i);
                const int k = loc - pre_i;
                c.cb = b_i + uint64_t(k) * 16;
                c.ne = int((e_i - c.cb) < 16 ? (e_i - c.cb) : 16);
                c.flags |= uint32_t(i) | F_VALID | (k == 0 ? F_FIRST_ITEM : 0u);
            }
            return c;
        };
        auto load_src = [&](const Chunk& c) -> uint32_t {
            return (c.ne > 0 && lane < c.ne) ? a.col[c.cb + lane] : 0u;
        };
        struct Score {
            float L[4], M[4], R[4];
        };
        auto load_score = [&](const Chunk& c, uint32_t src, Score& sc) {
            const uint32_t sj = __shfl_sync(0xffffffffu, src, j);
#pragma unroll
            for (int hh = 0; hh < 4; ++hh) sc.L[hh] = sc.M[hh] = sc.R[hh] = 0.f;
            if (j < c.ne) {
                if (vec8) {
                    const float4 l = *reinterpret_cast<const float4*>(a.left + uint64_t(c.row) * 8 + hb);
                    const float4 m = *reinterpret_cast<const float4*>(a.max + uint64_t(c.row) * 8 + hb);
                    const float4 r = *reinterpret_cast<const float4*>(a.right + uint64_t(sj) * 8 + hb);
                    sc.L[0] = l.x; sc.L[1] = l.y; sc.L[2] = l.z; sc.L[3] = l.w;
                    sc.M[0] = m.x; sc.M[1] = m.y; sc.M[2] = m.z; sc.M[3] = m.w;
                    sc.R[0] = r.x; sc.R[1] = r.y; sc.R[2] = r.z; sc.R[3] = r.w;
                } else {
#pragma unroll
                    for (int hh = 0; hh < 4; ++hh) {
                        const int h = hb + hh;
                        if (h < K) {
                            sc.L[hh] = a.left[uint64_t(c.row) * K + h];
                            sc.M[hh] = a.max[uint64_t(c.row) * K + h];
                            sc.R[hh] = a.right[uint64_t(sj) * K + h];
                        }
                    }
                }
            }
        };
        // chunk i of this warp's sequence is stream chunk (par + 2i)*4 + w
        Chunk c0 = chunk_at(uint64_t(par) * 4 + w);
        Chunk c1 = chunk_at(uint64_t(par + 2) * 4 + w);
        Chunk c2 = chunk_at(uint64_t(par + 4) * 4 + w);
        uint32_t src0 = load_src(c0), src1 = load_src(c1), src2 = load_src(c2);
        Score s0, s1;
        load_score(c0, src0, s0);
        load_score(c1, src1, s1);
        uint64_t q = uint64_t(par);
        bool ok = true;
        for (;; q += 2) {
            const Chunk c3 = chunk_at((q + 6) * 4 + uint64_t(w));
            // stage q belongs to the stream while chunk 4q exists
            if (!(have || q * 4 < gstart)) break;
            const uint32_t src3 = load_src(c3);  // used three iterations ahead
            Score s2;
            load_score(c2, src2, s2);            // used two iterations ahead
            const int s = int(q % kStages);
            if (!mbar_wait(empty + s, (uint32_t(q / kStages) & 1u) ^ 1u, abort_flag, err)) { ok = false; break; }
            uint8_t* dsc = d_s + s * kDescBytes;
            if (c0.flags & F_VALID) {
                const int ne = c0.ne;
                float p[4];
#pragma unroll
                for (int hh = 0; hh < 4; ++hh)
                    p[hh] = (j < ne && hb + hh < K) ? __expf(leaky(s0.L[hh] + s0.R[hh]) - s0.M[hh]) : 0.f;
                // P tile: row h (high), 8+h (low), column 16w+j
                const int e = 16 * w + j;
#pragma unroll
                for (int hh = 0; hh < 4; ++hh) {
                    const int nh = hb + hh, nl = 8 + hb + hh;
                    const uint16_t hi = rne16(p[hh]);
                    const uint16_t lo = rne16(p[hh] - bf(hi));
                    *reinterpret_cast<uint16_t*>(p_s + s * kPBytes + (nh >> 3) * 1024 + (nh & 7) * 128 +
                                                 ((((e >> 3) ^ (nh & 7))) << 4) + (e & 7) * 2) = hi;
                    *reinterpret_cast<uint16_t*>(p_s + s * kPBytes + (nl >> 3) * 1024 + (nl & 7) * 128 +
                                                 ((((e >> 3) ^ (nl & 7))) << 4) + (e & 7) * 2) = lo;
                }
                // feature row 127: 1.0 for the chunk's neighbours, 0 past its end (den)
                if (lane < 16) {
                    const int kk = 16 * w + lane;
                    *reinterpret_cast<uint16_t*>(a_s + s * kABytes + 8192 + (kk >> 3) * 1024 + (kk & 7) * 128 +
                                                 ((7 ^ (kk & 7)) << 4) + 14) = lane < ne ? 0x3F80 : 0;
                }
                // gathered X rows -> X^T tile (MN-major): lane = (16-byte chunk c, neighbour parity),
                // neighbours 16w + ee
                const uint32_t a_base = smem_u32(a_s + s * kABytes);
                const int c = lane & 15;
                const int rem = (a.in - c * 8) * 2;
                const uint32_t cbytes = c < a.ch ? uint32_t(rem < 16 ? rem : 16) : 0u;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int ee = (lane >> 4) + 2 * i;
                    const uint32_t se = __shfl_sync(0xffffffffu, src0, ee);
                    if (c < a.ch) {
                        const bool v = ee < ne;
                        const uint16_t* g = v ? a.x + uint64_t(se) * a.ldx + c * 8 : a.x;
                        const int kk = 16 * w + ee;
                        const uint32_t dst = a_base + (c >> 3) * 8192 + (kk >> 3) * 1024 + (kk & 7) * 128 +
                                             (((c & 7) ^ (kk & 7)) << 4);
                        cp_async16(dst, g, v ? cbytes : 0u);
                    }
                }
            }
            if (lane == 0) *reinterpret_cast<uint32_t*>(dsc + 4 * w) = c0.flags;
            // Stage q is complete for this thread when its copies have landed
            // (asynchronous arrival) and its shared-memory stores are released
            // (plain arrival). The MMA thread fences the async proxy after its
            // wait, so the producer never waits on its own copies.
            cp_async_arrive_noinc(full + s);
            mbar_arrive(full + s);
            c0 = c1;
            c1 = c2;
            c2 = c3;
            src0 = src1;
            src1 = src2;
            src2 = src3;
            s0 = s1;
            s1 = s2;
        }
        cp_async_wait<0>();
    } else if (warp < kEpi0) {
        // ================= MMA issuers (lane 0 of warps 8-11) =================
        // Warp k issues the PH MMAs of slots k and k+4 (an item's chunks stay on
        // one thread, so its accumulation order is fixed); warps 8 and 9 issue
        // the UW MMAs of W^T halves 0 and 1. One thread can have one MMA in
        // flight at a time, so the issue is spread over four threads.
        const int mk = warp - kMma0;
        if (lane == 0 && blockIdx.x < a.n_groups) {
            constexpr uint32_t idesc_ph = idesc_bf16(128, 16, 1, 0);
            constexpr uint32_t idesc_uw = idesc_bf16(128, 64, 0, 1);
            uint64_t t = 0;  // groups completed
            bool ok = true, done = false;
            // Group t's PH accumulators reuse the TMEM columns of group t-2: every
            // MMA warp first waits until the epilogue has read them (u_full of t-2).
            auto ph_free = [&](uint64_t tt) -> bool {
                const uint32_t gb = uint32_t(tt & 1), u = uint32_t(tt >> 1);
                return mbar_wait(u_full + gb, u & 1u, abort_flag, err);
            };
            auto issue_uw = [&](uint64_t tt) -> bool {
                const uint32_t gb = uint32_t(tt & 1), u = uint32_t(tt >> 1);
                if (!mbar_wait(u_full + gb, u & 1u, abort_flag, err)) return false;
                if (!mbar_wait(uw_empty + gb, (u & 1u) ^ 1u, abort_flag, err)) return false;
                fence_after();
                const uint32_t ub = smem_u32(u_s + gb * kUBytes);
                const uint32_t wb = smem_u32(w_s + mk * kWBytes);
                const uint32_t d = tmem + gb * 256 + 128 + mk * 64;
                for (int ks = 0; ks < a.ksteps; ++ks)
                    mma_bf16(d, desc_sw128(wb + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024),
                             desc_sw128(ub + ks * 2048, 16384, 1024), idesc_uw, ks > 0);
                mma_commit(uw_full + gb);
                return true;
            };
            const bool uw = mk < a.mh;
            const uint32_t a0 = smem_u32(a_s), p0 = smem_u32(p_s);
            for (uint64_t q = 0; !done && ok; ++q) {
                const int s = int(q % kStages);
                if (!mbar_wait(full + s, uint32_t(q / kStages) & 1u, abort_flag, err)) { ok = false; break; }
                // the X tiles were written by cp.async and st.shared (generic proxy); the
                // MMA reads them through the async proxy
                fence_proxy_async_smem();
                fence_after();
                const uint4 fl = *reinterpret_cast<const uint4*>(d_s + s * kDescBytes);
                const uint32_t fs[4] = {fl.x, fl.y, fl.z, fl.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t f = fs[j];
                    if (f & F_NONE) continue;
                    const uint32_t gb = (f & F_GB) ? 1u : 0u;
                    if ((f & F_FIRST_GROUP) && t >= 2 && !(uw ? issue_uw(t - 2) : ph_free(t - 2))) {
                        ok = false;
                        break;
                    }
                    if ((f & F_VALID) && int(f & 3u) == mk)
                        mma_bf16(tmem + gb * 256 + (f & F_SLOT) * 16,
                                 desc_sw128(a0 + uint32_t(s * kABytes + j * 2048), 8192, 1024),
                                 desc_sw128(p0 + uint32_t(s * kPBytes + j * 32), 16, 1024), idesc_ph,
                                 (f & F_FIRST_ITEM) ? 0u : 1u);
                    if (f & F_LAST_GROUP) {
                        mma_commit(ph_full + gb);
                        ++t;
                    }
                    if (f & F_END) done = true;
                }
                mma_commit(empty + s);
            }
            // the projections of the last two groups
            if (uw && ok && t >= 2 && !issue_uw(t - 2)) ok = false;
            if (uw && ok && t >= 1) issue_uw(t - 1);
            mma_commit(mma_done);
            mbar_wait(mma_done, 0, abort_flag, err);
        }
        __syncwarp();
    } else {
        // ================= epilogue =================
        const int q4 = warp & 3;              // TMEM lane quarter
        const int et = threadIdx.x - kEpi0 * 32;  // 0..127
        const int kf = q4 * 32 + lane;        // feature row of the PH accumulators
        // item table of a group on lanes 0..7: row, segment (-1: whole row), live (has neighbours)
        struct Tab {
            uint32_t row;
            int seg;
            int live;
        };
        auto fetch = [&](uint64_t G) -> Tab {
            Tab tb{0, -1, 0};
            const uint64_t it = G * 8 + uint64_t(lane);
            if (lane < 8 && it < a.n_items) {
                const Item m = item_info(a, it);
                tb.row = m.row;
                tb.seg = m.seg;
                tb.live = m.end > m.beg ? 1 : 2;  // 2: an item without neighbours
            }
            return tb;
        };
        auto outputs = [&](uint64_t tt, const Tab& tb) -> bool {
            const uint32_t gb = uint32_t(tt & 1), u = uint32_t(tt >> 1);
            if (!mbar_wait(uw_full + gb, u & 1u, abort_flag, err)) return false;
            fence_after();
            for (int hf = 0; hf < a.mh; ++hf) {
                const int r = hf * 128 + kf;  // W^T row = output column h'*dim + c
                const int hh = r < a.width ? r / a.dim : 0;
                float v8[8];                  // the 8 slots of head hh
                if (a.uniform_head) {
                    // dim divides 32: the warp's 32 rows share one head
                    const int hw = (hf * 128 + q4 * 32) / a.dim;
                    __syncwarp();
                    tmem_ld8(tmem + (uint32_t(q4 * 32) << 16) + gb * 256 + 128 + hf * 64 + hw * 8, v8);
                } else {
                    float v64[64];
                    __syncwarp();
                    tmem_ld64(tmem + (uint32_t(q4 * 32) << 16) + gb * 256 + 128 + hf * 64, v64);
#pragma unroll
                    for (int sl = 0; sl < 8; ++sl) {
                        float v = v64[sl];
#pragma unroll
                        for (int i = 1; i < 8; ++i) v = hh == i ? v64[i * 8 + sl] : v;
                        v8[sl] = v;
                    }
                }
#pragma unroll
                for (int sl = 0; sl < 8; ++sl) {
                    const int have = __shfl_sync(0xffffffffu, tb.live, sl);
                    const uint32_t mrow = __shfl_sync(0xffffffffu, tb.row, sl);
                    const int mseg = __shfl_sync(0xffffffffu, tb.seg, sl);
                    if (have && r < a.width) {
                        const float v = v8[sl];
                        const float dn = den_epi[gb * 64 + sl * 8 + hh];
                        if (mseg >= 0) {
                            float* st = a.seg_state + uint64_t(mseg) * kSegFloats;
                            st[16 + r] = v;
                            if (r % a.dim == 0) {
                                st[8 + hh] = dn;
                                st[hh] = a.max[uint64_t(mrow) * K + hh];
                            }
                        } else if (a.norm) {
                            float o = dn > 0.f ? v * (1.f / dn) : 0.f;
                            if (a.hidden && o < 0.f) o = __expf(o) - 1.f;
                            const uint64_t at = uint64_t(mrow) * a.ldo + r;
                            if (a.out_bf16) static_cast<uint16_t*>(a.out)[at] = rne16(o);
                            else static_cast<float*>(a.out)[at] = o;
                        } else {
                            static_cast<float*>(a.out)[uint64_t(mrow) * a.ldo + r] = v;
                            if (r % a.dim == 0) a.den_out[uint64_t(mrow) * K + hh] = dn;
                        }
                    }
                }
            }
            if (a.norm && a.out_bf16 && a.width < a.ldo)
                for (int sl = 0; sl < 8; ++sl) {
                    const int have = __shfl_sync(0xffffffffu, tb.live, sl);
                    const uint32_t mrow = __shfl_sync(0xffffffffu, tb.row, sl);
                    const int mseg = __shfl_sync(0xffffffffu, tb.seg, sl);
                    if (have && mseg < 0)
                        for (int c = a.width + et; c < a.ldo; c += 128)
                            static_cast<uint16_t*>(a.out)[uint64_t(mrow) * a.ldo + c] = 0;
                }
            fence_before();
            mbar_arrive(uw_empty + gb);
            return true;
        };
        uint64_t t = 0;
        bool ok = true;
        Tab tab2{0, -1, 0}, tab1{0, -1, 0};  // tables of groups t-2 and t-1
        for (uint64_t G = blockIdx.x; G < a.n_groups; G += gridDim.x, ++t) {
            const uint32_t gb = uint32_t(t & 1), u = uint32_t(t >> 1);
            const Tab tab0 = fetch(G);  // in flight while waiting for the group's accumulators
            if (!mbar_wait(ph_full + gb, u & 1u, abort_flag, err)) { ok = false; break; }
            fence_after();
            if (t >= 2 && !outputs(t - 2, tab2)) { ok = false; break; }
            // den_epi[gb] is free once every epilogue thread finished outputs(t-2)
            asm volatile("bar.sync 1, 128;" ::: "memory");
            // U = high + low columns, BF16 RNE, into the UW operand (MN-major) with
            // column n = head*8 + slot: the 16-byte chunk of head h holds the 8 slots.
            uint8_t* ub = u_s + gb * kUBytes + (kf >> 3) * 1024 + (kf & 7) * 128;
            float uv[64];  // U[slot][head] of this feature row
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float v[64];  // slots 4*half .. 4*half+3: 16 columns each (8 high, 8 low)
                __syncwarp();
                tmem_ld64(tmem + (uint32_t(q4 * 32) << 16) + gb * 256 + half * 64, v);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const bool live = __shfl_sync(0xffffffffu, tab0.live, half * 4 + k) == 1;
#pragma unroll
                    for (int h = 0; h < 8; ++h) uv[(half * 4 + k) * 8 + h] = live ? v[k * 16 + h] + v[k * 16 + 8 + h] : 0.f;
                }
            }
#pragma unroll
            for (int h = 0; h < 8; ++h) {
                const uint32_t p0 = pack_bf16x2(uv[0 * 8 + h], uv[1 * 8 + h]), p1 = pack_bf16x2(uv[2 * 8 + h], uv[3 * 8 + h]);
                const uint32_t p2 = pack_bf16x2(uv[4 * 8 + h], uv[5 * 8 + h]), p3 = pack_bf16x2(uv[6 * 8 + h], uv[7 * 8 + h]);
                *reinterpret_cast<uint4*>(ub + ((h ^ (kf & 7)) << 4)) = make_uint4(p0, p1, p2, p3);
            }
            if (kf == kOnesRow)  // den[slot][head] (0 for an item without neighbours)
#pragma unroll
                for (int i = 0; i < 64; ++i) den_epi[gb * 64 + i] = uv[i];
            fence_before();
            fence_proxy_async_smem();
            mbar_arrive(u_full + gb);
            tab2 = tab1;
            tab1 = tab0;
        }
        if (ok && t >= 2) ok = outputs(t - 2, tab2);
        if (ok && t >= 1) outputs(t - 1, tab1);
    }

    fence_before();
    __syncthreads();
    if (warp == kMma0) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

// Sums the segments of each hub row (one warp per hub row) and finishes it.
__global__ void tfs_hub_merge_kernel(const TcArgs a, const uint32_t* __restrict__ hub_seg_offset) {
    const int lane = threadIdx.x & 31;
    const uint64_t k = blockIdx.x * uint64_t(blockDim.x / 32) + (threadIdx.x >> 5);
    if (k >= a.n_hub) return;
    const uint32_t s0 = hub_seg_offset[k], s1 = hub_seg_offset[k + 1];
    const uint64_t r = a.perm[a.n - 1 - k];
    const int K = a.heads;
    for (int c = lane; c < a.ldo; c += 32) {
        float v = 0.f, d = 0.f;
        const int hh = c < a.width ? c / a.dim : 0;
        if (c < a.width)
            for (uint32_t s = s0; s < s1; ++s) {
                const float* st = a.seg_state + uint64_t(s) * kSegFloats;
                v += st[16 + c];
                d += st[8 + hh];
            }
        if (a.norm) {
            const float scale = d > 0.f ? 1.f / d : 0.f;
            float o = c < a.width ? v * scale : 0.f;
            if (a.hidden && o < 0.f) o = expf(o) - 1.f;
            if (a.out_bf16) static_cast<uint16_t*>(a.out)[r * a.ldo + c] = rne16(o);
            else if (c < a.width) static_cast<float*>(a.out)[r * a.ldo + c] = o;
        } else if (c < a.width) {
            static_cast<float*>(a.out)[r * a.ldo + c] = v;
            if (c % a.dim == 0) a.den_out[r * K + hh] = d;
        }
    }
}

constexpr size_t kSmem = 1024 + kStages * (kABytes + kPBytes + kDescBytes) + 2 * kWBytes + 2 * kUBytes +
                         128 * sizeof(float) + (2 * kStages + 9) * 8 + 16;

}  // namespace

// in <= 120: feature row 127 of the gathered tile carries den, and no row copy
// may touch its 16-byte chunk (features 120-127).
bool tfs_tc_supported(const gat_b200_layer* p) {
    return p->in <= 120 && p->heads <= 8 && p->width <= 256 && p->np <= 256 && p->kp <= 128;
}

int tfs_tc_dispatch(const gat_b200_graph* g, const gat_b200_layer* p, const uint16_t* x, int ldx, const float* left,
                    const float* right, const float* max, int norm, int hidden, void* out, int out_bf16, int ldo,
                    float* den, cudaStream_t st, int* launches) {
    if ((reinterpret_cast<uintptr_t>(x) & 15) || ldx % 8) return fail("tfs: BF16 X rows must be 16-byte aligned");
    if (!norm && !den) return fail("tfs: null den");
    if (p->heads == 8 && ((reinterpret_cast<uintptr_t>(left) | reinterpret_cast<uintptr_t>(right) |
                           reinterpret_cast<uintptr_t>(max)) & 15))
        return fail("tfs: left/right/max must be 16-byte aligned");
    TcArgs a{};
    a.row = g->row;
    a.col = g->col;
    a.perm = g->perm;
    a.segs = g->segs;
    a.n = g->n;
    a.n_hub = g->n_hub;
    a.n_seg = g->n_seg;
    a.n_items = uint64_t(g->n_seg) + (g->n - g->n_hub);
    a.n_groups = (a.n_items + 7) / 8;
    a.in = p->in;
    a.heads = p->heads;
    a.dim = p->dim;
    a.width = p->width;
    a.ch = (p->in + 7) / 8;
    a.mh = p->width > 128 ? 2 : 1;
    a.ksteps = (p->in + 15) / 16;
    a.x = x;
    a.ldx = ldx;
    a.wt = p->wt_bf16;
    a.kp = p->kp;
    a.np = p->np;
    a.left = left;
    a.right = right;
    a.max = max;
    a.norm = norm;
    a.hidden = hidden;
    a.out_bf16 = out_bf16;
    a.out = out;
    a.ldo = ldo;
    a.den_out = den;
    a.seg_state = g->seg_state;
    a.uniform_head = 32 % p->dim == 0;
    *launches = 0;
    if (a.n_groups == 0) return 0;
    static_assert(kSmem <= 227 * 1024, "TFS tensor-core kernel exceeds shared memory");
    int dev = 0, sms = 0;
    GATB_CUDA(cudaGetDevice(&dev));
    GATB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    GATB_CUDA(cudaFuncSetAttribute(tfs_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmem)));
    const unsigned grid = unsigned(a.n_groups < uint64_t(sms) ? a.n_groups : uint64_t(sms));
    tfs_tc_kernel<<<grid, kThreads, kSmem, st>>>(a);
    GATB_LAUNCH("TFS aggregation (tcgen05) kernel");
    *launches = 1;
    if (g->n_hub) {
        tfs_hub_merge_kernel<<<(g->n_hub + 3) / 4, 128, 0, st>>>(a, g->hub_seg_offset);
        GATB_LAUNCH("TFS hub merge kernel");
        *launches = 2;
    }
    return 0;
}

int tfs_tc_check_error() {
    unsigned e = 0;
    GATB_CUDA(cudaMemcpyFromSymbol(&e, g_tfs_error, sizeof(e)));
    if (e) {
        unsigned z = 0;
        cudaMemcpyToSymbol(g_tfs_error, &z, sizeof(z));
        return fail_code(GAT_B200_ETIMEOUT, "TFS kernel: a bounded wait timed out");
    }
    return 0;
}

}  // namespace gatb
