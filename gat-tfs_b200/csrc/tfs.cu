// TFS ("transform from sum") path: aggregate the layer INPUT features first,
// then project, as the reference's TFS kernels do:
//
//   baseline/src/baseline_tfs.cpp:16-117         tfs_aggregate / tfs_layer (B1)
//   baseline/tfs_online/icpp_online.cpp:40-215   running-max B1
//   baseline/tfs_online/icpp_block.cpp:36-210    block-rounded U_B . W
//   baseline/tfs_online/icpp_heads_hybrid.cpp    U_B from a BF16 high/low split of p
//   baseline/src/baseline_standard.cpp:29-43     lr_reordered: [L|R] = X . (W a)
//
// For destination i and head h, with p_ij = exp(leaky(L_ih + R_jh) - m_ih):
//   rounding EDGE   V_ih = sum_j RNE(p_ij x_j) . W_h           (per neighbour)
//   rounding BLOCK  V_ih = sum_B RNE(sum_{j in B} p_ij x_j) . W_h (per block)
//   rounding SPLIT  as BLOCK with sum_{j in B} p_hi x_j + sum p_lo x_j,
//                   p = p_hi + p_lo two BF16 values, for blocks holding at
//                   least `threshold` neighbours (FP32 FMA below that)
// and den_ih = sum_j p_ij. V is the UNNORMALIZED output (finish divides by den).
//
// This file holds the fused convert + lr_reordered kernel and the CUDA-core
// TFS kernel, which implements every variant for any layer shape. It is the
// reference-semantics path: each lane runs the restatement's arithmetic in
// the same order (sequential FP32 over features, FMA chains where the
// reference uses FMA), so it differs from the CPU oracle only through expf.
// The tensor-core kernel for the layer-1 shapes is in tfs_tc.cu.
#include <algorithm>

#include "device.cuh"
#include "graph.cuh"

namespace gatb {

int tfs_tc_dispatch(const gat_b200_graph* g, const gat_b200_layer* p, const uint16_t* x, int ldx,
                    const float* left, const float* right, const float* max, int norm, int hidden, void* out,
                    int out_bf16, int ldo, float* den, cudaStream_t st, int* launches);
bool tfs_tc_supported(const gat_b200_layer* p);
int max_prescan_launch(const gat_b200_graph* g, int heads, const float* left, const float* right, float* max,
                       cudaStream_t st);

namespace {

__device__ __forceinline__ uint16_t rne16(float x) {
    uint16_t r;
    asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ float bf(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

// ---- convert + lr_reordered ------------------------------------------------
constexpr int kLrRows = 128;   // rows per block (one per thread)
constexpr int kLrChunk = 32;   // features staged per step

// Thread t of the block owns row r0+t: acc[c] = sum_k x[r][k] * blr[k][c] as
// one FMA chain in ascending k (the oracle's order). Rows are staged through
// shared memory in 32-feature chunks with coalesced loads; the BF16 copy of X
// (convert, common.cpp:85-93) is written on the way.
template <typename TX>
__global__ void __launch_bounds__(kLrRows)
    lr_kernel(uint64_t n, int in, int heads, const TX* __restrict__ x, int ldx, int policy,
              const float* __restrict__ blr, uint16_t* __restrict__ xb, int ldb, float* __restrict__ left,
              float* __restrict__ right) {
    extern __shared__ float lr_smem[];
    const int cols = 2 * heads;
    float* tile = lr_smem;                         // [kLrRows][kLrChunk + 1]
    float* bs = tile + kLrRows * (kLrChunk + 1);   // [in][cols]
    for (int i = threadIdx.x; i < in * cols; i += blockDim.x) {
        const float b = blr[i];
        bs[i] = policy == 0 ? bf(rne16(b)) : b;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kend = xb && ldb > in ? ldb : in;
    for (uint64_t r0 = uint64_t(blockIdx.x) * kLrRows; r0 < n; r0 += uint64_t(gridDim.x) * kLrRows) {
        float acc[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) acc[c] = 0.f;
        for (int k0 = 0; k0 < kend; k0 += kLrChunk) {
            __syncthreads();
            for (int rr = warp; rr < kLrRows; rr += kLrRows / 32) {
                const uint64_t r = r0 + rr;
                const int k = k0 + lane;
                float v = 0.f;
                uint16_t q = 0;
                if (r < n && k < in) {
                    if constexpr (sizeof(TX) == 4) {
                        v = x[r * uint64_t(ldx) + k];
                        q = rne16(v);
                    } else {
                        q = x[r * uint64_t(ldx) + k];
                        v = bf(q);
                    }
                }
                if (xb && r < n && k < ldb) xb[r * uint64_t(ldb) + k] = q;
                tile[rr * (kLrChunk + 1) + lane] = policy == 0 ? bf(q) : v;
            }
            __syncthreads();
            const int kk_end = in - k0 < kLrChunk ? in - k0 : kLrChunk;
            for (int kk = 0; kk < kk_end; ++kk) {
                const float xv = tile[threadIdx.x * (kLrChunk + 1) + kk];
                const float* b = bs + (k0 + kk) * cols;
#pragma unroll
                for (int c = 0; c < 16; ++c)
                    if (c < cols) acc[c] = fmaf(xv, b[c], acc[c]);
            }
        }
        const uint64_t r = r0 + threadIdx.x;
        if (r < n) {
#pragma unroll
            for (int c = 0; c < 16; ++c)
                if (c < heads) left[r * heads + c] = acc[c];
                else if (c < cols) right[r * heads + (c - heads)] = acc[c];
        }
    }
}

// ---- CUDA-core TFS aggregation ----------------------------------------------
struct TfsArgs {
    const uint64_t* row;
    const uint32_t* col;
    const uint32_t* perm;  // degree order (ascending); rows are taken from its end
    uint64_t n;
    int in, heads, dim, width, in_pad;
    const uint16_t* x;
    int ldx;
    const uint16_t* wt;  // RNE(W)^T [np][kp]
    int kp;
    const float* left;
    const float* right;
    const float* max_in;
    const float* fixed_p;
    const float* fixed_den;
    int rounding, block, threshold;
    uint64_t seg;                // the graph's segment length (block 0 with BLOCK/SPLIT)
    int norm, hidden, out_bf16;  // norm: write finish()ed out (BF16 or FP32) instead of V
    void* out;
    int ldo;
    float* den;
    float* max_out;
};

constexpr int kGenWarps = 4;    // warps per block, W read from global memory
constexpr int kGenWarpsWs = 16;  // warps per block with W staged in shared memory

// V[c] (lane owns c = lane, lane+32) += sum_k a[k] * W[k][h*dim+c], sequential
// FP32 over k with exact BF16 x BF16 products (the order of AMX tdpbf16ps).
// WS: W read from the block's shared copy w_s[k][col] (consecutive lanes read
// consecutive columns), else from the global W^T rows. Same products, same
// order: the two give identical bits.
template <bool WS>
__device__ __forceinline__ void gen_accumulate(const TfsArgs& a, int h, const float* s_a, float* v, int lane,
                                               const uint16_t* w_s) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int c = lane + 32 * j;
        if (c < a.dim) {
            float acc = v[j];
            if constexpr (WS) {
                // W in shared memory as groups of four features per column
                // (w_s viewed as uint2 [in/4][width]: W[4g..4g+3][col] in one
                // 8-byte word); eight features at a time, their s_a and W values
                // loaded together, the FMAs in feature order
                const uint2* w4 = reinterpret_cast<const uint2*>(w_s) + h * a.dim + c;
                const int ws = a.width;
                int k = 0;
                for (; k + 8 <= a.in; k += 8) {
                    const float4 s0 = *reinterpret_cast<const float4*>(s_a + k);
                    const float4 s1 = *reinterpret_cast<const float4*>(s_a + k + 4);
                    const uint2 wa = w4[size_t(k / 4) * ws];
                    const uint2 wb = w4[size_t(k / 4 + 1) * ws];
                    acc = fmaf(s0.x, bf16lo(wa.x), acc);
                    acc = fmaf(s0.y, bf16hi(wa.x), acc);
                    acc = fmaf(s0.z, bf16lo(wa.y), acc);
                    acc = fmaf(s0.w, bf16hi(wa.y), acc);
                    acc = fmaf(s1.x, bf16lo(wb.x), acc);
                    acc = fmaf(s1.y, bf16hi(wb.x), acc);
                    acc = fmaf(s1.z, bf16lo(wb.y), acc);
                    acc = fmaf(s1.w, bf16hi(wb.y), acc);
                }
                for (; k < a.in; ++k) {
                    const uint2 wq = w4[size_t(k / 4) * ws];
                    const uint32_t word = (k & 2) ? wq.y : wq.x;
                    acc = fmaf(s_a[k], (k & 1) ? bf16hi(word) : bf16lo(word), acc);
                }
            } else {
                const uint16_t* w = a.wt + size_t(h * a.dim + c) * a.kp;
                for (int k = 0; k < a.in; ++k) acc = fmaf(s_a[k], bf(w[k]), acc);
            }
            v[j] = acc;
        }
    }
}

// One warp per destination row, heads in turn, neighbours in CSR order. With
// WS the block first copies RNE(W) (in x width BF16, row-major) into shared
// memory, so the FMA chains read W from there.
template <int NW, bool WS>
__global__ void __launch_bounds__(32 * NW, 1) tfs_generic_kernel(const TfsArgs a) {
    extern __shared__ float gen_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint16_t* w_s = nullptr;
    float* wbase = gen_smem;
    if constexpr (WS) {
        // element (k, col) at uint16 index ((k/4) * width + col) * 4 + k%4;
        // features past `in` (up to a multiple of 4) hold zeros and are never used
        uint16_t* ws = reinterpret_cast<uint16_t*>(gen_smem);
        const int in4 = (a.in + 3) / 4 * 4;
        const size_t wcount = size_t(in4) * a.width;
        for (size_t t = threadIdx.x; t < wcount; t += blockDim.x) {
            const int g = int(t / (size_t(a.width) * 4)), rem = int(t % (size_t(a.width) * 4));
            const int c = rem / 4, k = g * 4 + rem % 4;
            ws[t] = k < a.in ? a.wt[size_t(c) * a.kp + k] : uint16_t(0);
        }
        __syncthreads();
        w_s = ws;
        wbase = gen_smem + (wcount * 2 + 15) / 16 * 4;  // past W, 16-byte aligned
    }
    float* s_a = wbase + size_t(warp) * (2 * a.in_pad + 64);  // RNE(.) vector [in_pad]
    float* s_u = s_a + a.in_pad;                                 // U accumulator [in_pad]
    float* s_p = s_u + a.in_pad;                                 // weights of a 32-neighbour chunk
    uint32_t* s_src = reinterpret_cast<uint32_t*>(s_p + 32);     // their sources
    // Work items are (row, head) pairs, rows from the largest degree down (the
    // degree order), so the heads of a hub row run on different warps at once;
    // every (row, head) keeps its neighbour order, so the sums are unchanged.
    const uint64_t items = a.n * uint64_t(a.heads);
    // rows of at most 256 features, 8-feature aligned, in 16-byte pieces
    const bool vec_rows = a.in <= 256 && a.in % 8 == 0 && a.ldx % 8 == 0 &&
                          (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
    for (uint64_t item = (uint64_t(blockIdx.x) * NW + warp); item < items; item += uint64_t(gridDim.x) * NW) {
        const uint64_t ri = item / uint64_t(a.heads);
        const int h = int(item % uint64_t(a.heads));
        const uint64_t i = a.perm ? a.perm[a.n - 1 - ri] : ri;
        const uint64_t beg = a.row[i], deg = a.row[i + 1] - beg;
        // block 0: one block per row; with BLOCK/SPLIT rounding a row longer than
        // the graph's segment length takes one block per segment, as the
        // tensor-core kernel does (it rounds U once per segment).
        const uint64_t B = a.block > 0 ? uint64_t(a.block)
                                       : (a.rounding != 0 && deg > a.seg ? a.seg : (deg ? deg : 1));
        {
            const float L = a.left ? a.left[i * a.heads + h] : 0.f;
            float v[2] = {0.f, 0.f};
            float den = 0.f, m = -INFINITY;
            for (uint64_t b0 = 0; b0 < deg; b0 += B) {
                const uint64_t cnt = deg - b0 < B ? deg - b0 : B;
                // block maximum, running maximum and rescale (icpp_online.cpp:75-135)
                if (!a.fixed_p) {
                    if (a.max_in) {
                        m = a.max_in[i * a.heads + h];
                    } else {
                        float bm = -INFINITY;
                        for (uint64_t b = lane; b < cnt; b += 32) {
                            const uint32_t s = a.col[beg + b0 + b];
                            bm = fmaxf(bm, leaky(L + a.right[uint64_t(s) * a.heads + h]));
                        }
                        bm = warp_max(bm);
                        const float prev = m;
                        m = fmaxf(m, bm);
                        const bool changed = m > prev && den > 0.f;
                        const float r = expf(changed ? prev - m : 0.f);
                        den = den * r;
                        if (changed) { v[0] *= r; v[1] *= r; }
                    }
                }
                const bool split = a.rounding == 2 && int64_t(cnt) >= int64_t(a.threshold);
                if (a.rounding != 0)
                    for (int k = lane; k < a.in_pad; k += 32) s_u[k] = 0.f;
                for (int pass = 0; pass < (split ? 2 : 1); ++pass) {
                    for (uint64_t c0 = 0; c0 < cnt; c0 += 32) {
                        const int cn = cnt - c0 < 32 ? int(cnt - c0) : 32;
                        __syncwarp();
                        if (lane < cn) {
                            const uint64_t e = beg + b0 + c0 + lane;
                            const uint32_t s = a.col[e];
                            float p;
                            if (a.fixed_p) p = a.fixed_p[e * a.heads + h];
                            else p = expf(leaky(L + a.right[uint64_t(s) * a.heads + h]) - m);
                            s_p[lane] = p;
                            s_src[lane] = s;
                        }
                        __syncwarp();
                        if (pass == 0) {
                            // den += p in neighbour order (one lane keeps the sum sequential,
                            // then every lane takes it: the rescale test reads den)
                            if (lane == 0)
                                for (int b = 0; b < cn; ++b) den = den + s_p[b];
                            den = __shfl_sync(0xffffffffu, den, 0);
                        }
                        if (a.rounding == 0 && vec_rows) {
                            // per-edge rounding with the rows read as one 16-byte piece
                            // per lane (8 features), the next neighbour's row in flight
                            // while this one's FMA chains run
                            const int k0 = lane * 8;
                            const bool mine = k0 < a.in;
                            uint4 cur = mine ? ldg_nc_v4(a.x + uint64_t(s_src[0]) * a.ldx + k0)
                                             : make_uint4(0, 0, 0, 0);
                            for (int b = 0; b < cn; ++b) {
                                uint4 nxt = make_uint4(0, 0, 0, 0);
                                if (b + 1 < cn && mine) nxt = ldg_nc_v4(a.x + uint64_t(s_src[b + 1]) * a.ldx + k0);
                                const float p = s_p[b];
                                if (mine) {
                                    const uint32_t xw[4] = {cur.x, cur.y, cur.z, cur.w};
                                    float o[8];
#pragma unroll
                                    for (int q = 0; q < 4; ++q) {
                                        o[2 * q] = bf(rne16(__fmul_rn(bf16lo(xw[q]), p)));
                                        o[2 * q + 1] = bf(rne16(__fmul_rn(bf16hi(xw[q]), p)));
                                    }
                                    *reinterpret_cast<float4*>(s_a + k0) = make_float4(o[0], o[1], o[2], o[3]);
                                    *reinterpret_cast<float4*>(s_a + k0 + 4) = make_float4(o[4], o[5], o[6], o[7]);
                                }
                                __syncwarp();
                                gen_accumulate<WS>(a, h, s_a, v, lane, w_s);
                                __syncwarp();
                                cur = nxt;
                            }
                            continue;
                        }
                        for (int b = 0; b < cn; ++b) {
                            const float p = s_p[b];
                            const uint16_t* xr = a.x + uint64_t(s_src[b]) * a.ldx;
                            if (a.rounding == 0) {
                                // hbuf = RNE(x * p) (baseline_tfs.cpp:67-69), then V += hbuf . W
                                for (int k = lane; k < a.in; k += 32) s_a[k] = bf(rne16(__fmul_rn(bf(xr[k]), p)));
                                __syncwarp();
                                gen_accumulate<WS>(a, h, s_a, v, lane, w_s);
                                __syncwarp();
                            } else if (!split) {
                                for (int k = lane; k < a.in; k += 32) s_u[k] = fmaf(p, bf(xr[k]), s_u[k]);
                            } else {
                                const float hi = bf(rne16(p));
                                const float f = pass == 0 ? hi : bf(rne16(p - hi));
                                for (int k = lane; k < a.in; k += 32) s_u[k] = fmaf(f, bf(xr[k]), s_u[k]);
                            }
                        }
                    }
                }
                if (a.rounding != 0) {
                    __syncwarp();
                    for (int k = lane; k < a.in; k += 32) s_a[k] = bf(rne16(s_u[k]));
                    __syncwarp();
                    gen_accumulate<WS>(a, h, s_a, v, lane, w_s);
                }
            }
            if (a.fixed_den) den = a.fixed_den[i * a.heads + h];
            if (a.norm) {
                const float scale = den > 0.f ? 1.f / den : 0.f;
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int c = lane + 32 * j;
                    if (c < a.dim) {
                        float o = v[j] * scale;
                        if (a.hidden && o < 0.f) o = expf(o) - 1.f;
                        const uint64_t at = i * uint64_t(a.ldo) + h * a.dim + c;
                        if (a.out_bf16) static_cast<uint16_t*>(a.out)[at] = rne16(o);
                        else static_cast<float*>(a.out)[at] = o;
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int c = lane + 32 * j;
                    if (c < a.dim) static_cast<float*>(a.out)[i * uint64_t(a.ldo) + h * a.dim + c] = v[j];
                }
            }
            if (lane == 0) {
                if (a.den) a.den[i * a.heads + h] = den;
                if (a.max_out) a.max_out[i * a.heads + h] = m;
            }
        }
        if (a.norm && a.out_bf16 && h == 0) {
            // zero the padding columns of a BF16 row (the next layer gathers whole rows)
            uint16_t* o = static_cast<uint16_t*>(a.out) + i * uint64_t(a.ldo);
            for (int c = a.width + lane; c < a.ldo; c += 32) o[c] = 0;
        }
    }
}

// icpp_online's exact counters (baseline/tfs_online/icpp_online.cpp:50-116,
// 146-164, 229-233, 330-346): one warp per (batch of 16 consecutive rows of the
// degree order, head); lane k < 16 follows row perm[16*batch + k] through
// neighbour blocks of `block` up to the batch's largest degree, exactly as the
// reference's tile does: block maximum of leaky(L + R) (same FP32 sum and
// leaky), a strict raise of the running maximum is a max update, an update
// after the row's first block (den > 0) a rescale; a batch block with any
// rescale is one rescale event (warp ballot).
__global__ void online_counters_kernel(const uint64_t* __restrict__ row, const uint32_t* __restrict__ col,
                                       const uint32_t* __restrict__ perm, uint64_t n, int heads,
                                       const float* __restrict__ left, const float* __restrict__ right, int block,
                                       unsigned long long* row_blocks, unsigned long long* row_updates,
                                       unsigned long long* row_rescales, unsigned long long* totals) {
    const uint64_t batches = (n + 15) / 16;
    const uint64_t warp = (blockIdx.x * uint64_t(blockDim.x) + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= batches * uint64_t(heads)) return;
    const int h = int(warp / batches);
    const uint64_t base = (warp % batches) * 16;
    const bool live = lane < 16 && base + lane < n;
    uint32_t r = 0;
    uint64_t beg = 0, deg = 0;
    float l = 0.f;
    if (live) {
        r = perm[base + lane];
        beg = row[r];
        deg = row[r + 1] - beg;
        l = left[uint64_t(r) * heads + h];
    }
    uint64_t maxdeg = deg;
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t v = __shfl_xor_sync(0xffffffffu, maxdeg, o);
        maxdeg = v > maxdeg ? v : maxdeg;
    }
    float run = -INFINITY;
    bool seen = false;
    unsigned long long nb = 0, nu = 0, nr = 0, events = 0;
    for (uint64_t b0 = 0; b0 < maxdeg; b0 += uint64_t(block)) {
        bool rescale = false;
        if (live && b0 < deg) {
            const uint64_t end = b0 + uint64_t(block) < deg ? b0 + uint64_t(block) : deg;
            float bm = -INFINITY;
            for (uint64_t s = b0; s < end; ++s) {
                const float sc = leaky(l + right[uint64_t(col[beg + s]) * heads + h]);
                bm = sc > bm ? sc : bm;
            }
            const float prev = run;
            run = bm > run ? bm : run;
            const bool update = run > prev;
            rescale = update && seen;
            seen = true;
            ++nb;
            nu += update ? 1u : 0u;
            nr += rescale ? 1u : 0u;
        }
        if (__ballot_sync(0xffffffffu, rescale)) ++events;
    }
    if (live) {
        const uint64_t idx = uint64_t(r) * heads + h;
        if (row_blocks) row_blocks[idx] = nb;
        if (row_updates) row_updates[idx] = nu;
        if (row_rescales) row_rescales[idx] = nr;
    }
    for (int o = 16; o > 0; o >>= 1) {
        nb += __shfl_xor_sync(0xffffffffu, nb, o);
        nu += __shfl_xor_sync(0xffffffffu, nu, o);
        nr += __shfl_xor_sync(0xffffffffu, nr, o);
    }
    if (lane == 0) {
        atomicAdd(totals + 0, nb);
        atomicAdd(totals + 1, nu);
        atomicAdd(totals + 2, nr);
        atomicAdd(totals + 3, events);
        atomicAdd(totals + 4, (unsigned long long)maxdeg);
    }
}

}  // namespace

int online_counters_launch(const gat_b200_graph* g, int heads, const float* left, const float* right, int block,
                           uint64_t* row_blocks, uint64_t* row_updates, uint64_t* row_rescales, uint64_t* totals,
                           cudaStream_t st) {
    if (!g || !left || !right || !totals) return fail("tfs_online_counters: null argument");
    if (heads < 1 || heads > 8) return fail("invalid parameter shape (heads <=8, head_dim <=64)");
    if (block < 1) return fail("tfs_online_counters: block must be positive");
    unsigned long long* d = nullptr;
    GATB_CUDA(cudaMalloc(&d, 5 * sizeof(unsigned long long)));
    cudaError_t e = cudaMemsetAsync(d, 0, 5 * sizeof(unsigned long long), st);
    const uint64_t warps = (g->n + 15) / 16 * uint64_t(heads);
    if (e == cudaSuccess && warps) {
        online_counters_kernel<<<unsigned((warps + 7) / 8), 256, 0, st>>>(
            g->row, g->col, g->perm, g->n, heads, left, right, block,
            reinterpret_cast<unsigned long long*>(row_blocks), reinterpret_cast<unsigned long long*>(row_updates),
            reinterpret_cast<unsigned long long*>(row_rescales), d);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(totals, d, 5 * sizeof(unsigned long long), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaFree(d);
    return e == cudaSuccess ? 0 : cuda_fail(e, "tfs_online_counters");
}

int lr_reordered_launch(const gat_b200_layer* p, uint64_t n, const void* x, int x_dtype, int ldx, int policy,
                        uint16_t* xb, int ldb, float* left, float* right, cudaStream_t st) {
    if (!p || !x || !left || !right) return fail("lr_reordered: null buffer");
    if (policy != GAT_B200_LR_BF16 && policy != GAT_B200_LR_FP32) return fail("unknown LR policy");
    if (x_dtype != GAT_B200_F32 && x_dtype != GAT_B200_BF16) return fail("lr_reordered: bad x dtype");
    if (ldx < p->in) return fail("lr_reordered: row stride smaller than the width");
    if (xb && ldb < p->in) return fail("lr_reordered: BF16 row stride smaller than the width");
    if (n == 0) return 0;
    const size_t smem = (size_t(kLrRows) * (kLrChunk + 1) + size_t(p->in) * 2 * p->heads) * sizeof(float);
    if (smem > 200 * 1024) return fail_code(GAT_B200_EUNSUPPORTED, "lr_reordered: input width too large");
    unsigned blocks = unsigned(std::min<uint64_t>((n + kLrRows - 1) / kLrRows, 148ull * 16));
    if (x_dtype == GAT_B200_F32) {
        GATB_CUDA(cudaFuncSetAttribute(lr_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
        lr_kernel<float><<<blocks, kLrRows, smem, st>>>(n, p->in, p->heads, static_cast<const float*>(x), ldx, policy,
                                                        p->blr, xb, ldb, left, right);
    } else {
        GATB_CUDA(cudaFuncSetAttribute(lr_kernel<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
        lr_kernel<uint16_t><<<blocks, kLrRows, smem, st>>>(n, p->in, p->heads, static_cast<const uint16_t*>(x), ldx,
                                                           policy, p->blr, xb, ldb, left, right);
    }
    GATB_LAUNCH("lr_reordered kernel");
    return 0;
}

// Validates the arguments shared by the TFS entry points.
static int tfs_check(const gat_b200_graph* g, const gat_b200_layer* p, const void* x, int ldx, int rounding,
                     int block, int threshold) {
    if (!g || !p) return fail("tfs: null handle");
    if (!x) return fail("tfs: null feature table");
    if (ldx < p->in) return fail("tfs: row stride smaller than the input width");
    if (rounding < GAT_B200_TFS_EDGE || rounding > GAT_B200_TFS_SPLIT) return fail("tfs: unknown rounding");
    if (block < 0) return fail("tfs: block must be >= 0");
    if (threshold < 1 || threshold > 33) return fail("ICPP heads hybrid threshold must be in [1,33]");
    return 0;
}

int tfs_generic_launch(const gat_b200_graph* g, const gat_b200_layer* p, const uint16_t* x, int ldx,
                       const float* left, const float* right, const float* max, const float* fixed_p,
                       const float* fixed_den, int rounding, int block, int threshold, int norm, int hidden,
                       void* out, int out_bf16, int ldo, float* den, float* max_out, cudaStream_t st) {
    TfsArgs a{};
    a.row = g->row;
    a.col = g->col;
    a.perm = g->perm;
    a.n = g->n;
    a.in = p->in;
    a.heads = p->heads;
    a.dim = p->dim;
    a.width = p->width;
    a.in_pad = (p->in + 31) / 32 * 32;
    a.x = x;
    a.ldx = ldx;
    a.wt = p->wt_bf16;
    a.kp = p->kp;
    a.left = left;
    a.right = right;
    a.max_in = max;
    a.fixed_p = fixed_p;
    a.fixed_den = fixed_den;
    a.rounding = rounding;
    a.block = block;
    a.threshold = threshold;
    a.seg = g->seg_edges ? g->seg_edges : ~0ull;
    a.norm = norm;
    a.hidden = hidden;
    a.out_bf16 = out_bf16;
    a.out = out;
    a.ldo = ldo;
    a.den = den;
    a.max_out = max_out;
    if (g->n == 0) return 0;
    // W staged in shared memory when it fits beside 16 warps' vectors: one
    // block per SM, four FMA chains per scheduler
    const size_t w_bytes = (size_t((a.in + 3) / 4 * 4) * a.width * 2 + 15) / 16 * 16;
    const size_t smem_ws = w_bytes + size_t(kGenWarpsWs) * (2 * a.in_pad + 64) * sizeof(float);
    if (smem_ws <= 200 * 1024) {
        auto k = tfs_generic_kernel<kGenWarpsWs, true>;
        GATB_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem_ws)));
        int dev = 0, sms = 0;
        GATB_CUDA(cudaGetDevice(&dev));
        GATB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        const uint64_t items = g->n * uint64_t(p->heads);
        unsigned blocks = unsigned(std::min<uint64_t>((items + kGenWarpsWs - 1) / kGenWarpsWs, uint64_t(sms)));
        k<<<blocks, 32 * kGenWarpsWs, smem_ws, st>>>(a);
        GATB_LAUNCH("TFS aggregation kernel");
        return 0;
    }
    const size_t smem = size_t(kGenWarps) * (2 * a.in_pad + 64) * sizeof(float);
    if (smem > 200 * 1024) return fail_code(GAT_B200_EUNSUPPORTED, "tfs: input width too large");
    auto k = tfs_generic_kernel<kGenWarps, false>;
    GATB_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    unsigned blocks =
        unsigned(std::min<uint64_t>((g->n * uint64_t(p->heads) + kGenWarps - 1) / kGenWarps, 148ull * 32));
    k<<<blocks, 32 * kGenWarps, smem, st>>>(a);
    GATB_LAUNCH("TFS aggregation kernel");
    return 0;
}

// Chooses the kernel: the tensor-core kernel implements SPLIT rounding with one
// block per row (hub rows: one block per segment) and the prescan maximum;
// everything else runs on the CUDA-core kernel.
int tfs_dispatch(const gat_b200_graph* g, const gat_b200_layer* p, const void* x, int ldx, const float* left,
                 const float* right, const float* max, const float* fixed_p, const float* fixed_den, int rounding,
                 int block, int threshold, int norm, int hidden, void* out, int out_bf16, int ldo, float* den,
                 float* max_out, cudaStream_t st, int* launches) {
    int dummy = 0;
    if (!launches) launches = &dummy;
    *launches = 0;
    int rc = tfs_check(g, p, x, ldx, rounding, block, threshold);
    if (rc) return rc;
    if (!out) return fail("tfs: null output");
    if (ldo < p->width) return fail("tfs: output row stride smaller than the width");
    if (!fixed_p && (!left || !right)) return fail("tfs: null left/right");
    if (fixed_p && !fixed_den) return fail("tfs: fixed_p needs fixed_den");
    if (g->n_src && g->n_src != g->n) return fail("tfs: partitioned graphs are not supported");
    if (rounding == GAT_B200_TFS_SPLIT && block == 0 && threshold <= 1 && !fixed_p && max && !max_out &&
        tfs_tc_supported(p))
        return tfs_tc_dispatch(g, p, static_cast<const uint16_t*>(x), ldx, left, right, max, norm, hidden, out,
                               out_bf16, ldo, den, st, launches);
    *launches = 1;
    return tfs_generic_launch(g, p, static_cast<const uint16_t*>(x), ldx, left, right, max, fixed_p, fixed_den,
                              rounding, block, threshold, norm, hidden, out, out_bf16, ldo, den, max_out, st);
}

}  // namespace gatb

using namespace gatb;

extern "C" {

int gat_b200_lr_reordered(const gat_b200_layer* p, uint64_t n, const void* x, int x_dtype, int ldx, int policy,
                          void* x_bf16, int ld_bf16, float* left, float* right, void* stream) {
    clear_error();
    return lr_reordered_launch(p, n, x, x_dtype, ldx, policy, static_cast<uint16_t*>(x_bf16), ld_bf16, left, right,
                               as_stream(stream));
}

int gat_b200_tfs_online_counters(const gat_b200_graph* g, int heads, const float* left, const float* right,
                                 int block, uint64_t* row_blocks, uint64_t* row_updates, uint64_t* row_rescales,
                                 uint64_t* totals, void* stream) {
    clear_error();
    return online_counters_launch(g, heads, left, right, block, row_blocks, row_updates, row_rescales, totals,
                                  as_stream(stream));
}

int gat_b200_tfs_aggregate(const gat_b200_graph* g, const gat_b200_layer* p, const void* x, int ldx,
                           const float* left, const float* right, const float* max, const float* fixed_p,
                           const float* fixed_den, int rounding, int block, int threshold, float* out, int ldo,
                           float* den, float* max_out, void* stream) {
    clear_error();
    if (!den) return fail("tfs_aggregate: null den");
    if (rounding == GAT_B200_TFS_EDGE && block == 0 && !max && !fixed_p)
        return fail("tfs_aggregate: B1 (block 0) needs the prescan maximum");
    return tfs_dispatch(g, p, x, ldx, left, right, max, fixed_p, fixed_den, rounding, block, threshold, 0, 0, out, 0,
                        ldo, den, max_out, as_stream(stream), nullptr);
}

int gat_b200_tfs_layer(const gat_b200_graph* g, const gat_b200_layer* p, const void* x, int x_dtype, int ldx,
                       int hidden, int policy, int rounding, int block, int threshold, void* x_bf16, float* left,
                       float* right, float* max, float* den, void* out, int out_dtype, int ldo, void* stream) {
    clear_error();
    if (!g || !p) return fail("tfs_layer: null handle");
    if (!x_bf16 || !left || !right || !max || !den) return fail("tfs_layer: null scratch buffer");
    cudaStream_t st = as_stream(stream);
    const int ldb = gat_b200_padded_ld(p->in, GAT_B200_BF16);
    int rc = lr_reordered_launch(p, g->n, x, x_dtype, ldx, policy, static_cast<uint16_t*>(x_bf16), ldb, left, right, st);
    if (rc) return rc;
    if ((rc = max_prescan_launch(g, p->heads, left, right, max, st))) return rc;
    // Online-max variants (block > 0) start from the row's running maximum;
    // with the prescan maximum every block already uses the final one, which
    // differs from the running maximum only through the rescale roundings.
    const float* mx = block == 0 ? max : nullptr;
    return tfs_dispatch(g, p, x_bf16, ldb, left, right, mx, nullptr, nullptr, rounding, block, threshold, 1, hidden,
                        out, out_dtype == GAT_B200_BF16, ldo, den, nullptr, st, nullptr);
}

}  // extern "C"
