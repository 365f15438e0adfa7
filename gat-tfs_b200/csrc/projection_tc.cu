// Tensor-core projection with fused attention dots (sm_100a tcgen05 + TMA).
//
// Replaces gat::projection + gat::lr_from_z of the B0 BF16 path
// (baseline/src/baseline_standard.cpp:3-20):
//   Z = BF16(X) . BF16(W)  (FP32 accumulate)
//   left[i][h] = Z_ih . aL_h,  right[i][h] = Z_ih . aR_h   (from the FP32 Z)
//   H = BF16 RNE(Z)        (the gathered feature rows of the aggregation)
//
// Persistent kernel, one CTA per SM, 10 warps with fixed roles:
//   warp 0  TMA producer: W^T once (resident in shared memory for the whole
//           kernel), then 128-row x 64-column tiles of X through an S-stage ring.
//   warp 1  TMEM owner and MMA issuer: 128 x NP x 16 tcgen05.mma (kind::f16,
//           BF16 x BF16 -> FP32) into one of two TMEM accumulators, so the
//           epilogue of tile t overlaps the MMAs of tile t+1.
//   warps 2-9 epilogue, two sets of four: set b drains accumulator b (the
//           CTA's even / odd tiles), so two tiles' epilogues run at once and
//           every SM sub-partition holds two epilogue warps. tcgen05.ld of 64
//           columns at a time (thread = row), L/R dot products in FP32, BF16
//           pack into a 128B-swizzled staging buffer, TMA store of 32 x 64
//           boxes (two staging buffers per warp where shared memory allows,
//           else one).
// No cluster launch, no multicast: every CTA loads its own tiles.
//
// Every mbarrier wait is bounded: after ~1 s without progress the CTA records
// GAT_B200_ETIMEOUT in a device flag, waits (bounded) for its own copies and
// MMAs in flight, frees its TMEM and exits.
#include <cuda.h>

#include "device.cuh"
#include "graph.cuh"
#include "tc.cuh"

namespace gatb {

__device__ unsigned g_proj_error = 0;

namespace {

constexpr int kTileM = 128;
constexpr int kKBlock = 64;                       // BF16 elements per 128-byte swizzle row
constexpr int kABytes = kTileM * kKBlock * 2;     // 16 KB per A stage
constexpr int kStageRows = 32;                    // epilogue store box rows (one warp)
constexpr int kStageBytes = kStageRows * 128;     // 4 KB
constexpr int kThreads = 320;
constexpr int kEpiWarps = 8;
constexpr int kMaxPeers = 7;
constexpr int kMaxCoef = 256;  // attention coefficients carried in the launch parameters

struct ProjArgs {
    uint64_t n;
    int heads, dim, width, np, kb;
    int stages;
    uint32_t tmem_cols;  // two accumulators, tmem_cols/2 columns apart
    float* left;
    float* right;
    float* z;       // optional FP32 Z [n][ldz]
    int ldz;
    int lr_vec;     // left/right allow float4 stores (heads == 8, aligned)
    int store_h;    // 1: BF16 H through TMA stores (0: only z / left / right)
    int sb;         // staging buffers per epilogue warp (1 or 2)
    const float* al;
    const float* ar;
    // Extra destinations (other GPUs' tables, mapped peer memory): every H row
    // and R row is also stored to hp[i] / rp[i], i < npeer, with the same row
    // index and row stride ldh (R: heads floats per row).
    int npeer;
    int ldh;
    uint16_t* hp[kMaxPeers];
    float* rp[kMaxPeers];
    // aL / aR (zero past the width) for the shape-specialised epilogues, which
    // read them as constant operands instead of from shared memory
    float alc[kMaxCoef];
    float arc[kMaxCoef];
};

// ---- PTX wrappers (tc.cuh) -------------------------------------------------
using tc::bulk_commit;
using tc::bulk_wait_all;
using tc::bulk_wait_read;
using tc::fence_proxy_async_smem;
using tc::mbar_arrive;
using tc::mbar_expect_tx;
using tc::mbar_init;
using tc::mbar_try;
using tc::mma_bf16;
using tc::mma_commit;
using tc::smem_u32;
using tc::tma_load_2d;
using tc::tma_store_2d;
using tc::tmem_ld16;
// Bounded wait recording a timeout in this kernel's error flag.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    return tc::mbar_wait(bar, parity, abort_flag, &g_proj_error);
}
// K-major operand in the 128-byte swizzle layout: 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) { return tc::desc_sw128(saddr, 16, 1024); }

// ALIGNED16: every 16-column block lies in one head. NPT / KT: the padded
// width and the head count at compile time (0 = read from the arguments);
// with both known the epilogue's loops unroll completely, the coefficients
// are constant operands and each block's head is a constant.
template <bool ALIGNED16, int NPT, int KT>
__global__ void __launch_bounds__(kThreads, 1)
    proj_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_h, const __grid_constant__ ProjArgs a) {
    static_assert(NPT == 0 || (ALIGNED16 && KT != 0 && NPT <= kMaxCoef && NPT % 16 == 0), "bad specialisation");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled tiles.
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = a.stages, NP = NPT ? NPT : a.np, KB = a.kb;
    uint8_t* w_s = smem;                                         // KB x [NP x 128 B]
    uint8_t* a_s = w_s + size_t(KB) * NP * 128;                   // S x 16 KB
    uint8_t* st_s = a_s + size_t(S) * kABytes;                    // 8 warps x sb x 4 KB
    float* al_s = reinterpret_cast<float*>(st_s + size_t(kEpiWarps) * a.sb * kStageBytes);  // [NP]
    float* ar_s = al_s + NP;                                      // [NP]
    uint64_t* bars = reinterpret_cast<uint64_t*>(ar_s + NP);
    uint64_t* full = bars;              // [S]
    uint64_t* empty = bars + S;         // [S]
    uint64_t* w_full = bars + 2 * S;    // 1
    uint64_t* acc_full = w_full + 1;    // [2]
    uint64_t* acc_empty = acc_full + 2; // [2]
    uint64_t* mma_done = acc_empty + 2; // 1
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t ntiles = (a.n + kTileM - 1) / kTileM;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        mbar_init(w_full, 1);
        mbar_init(acc_full + 0, 1);
        mbar_init(acc_full + 1, 1);
        mbar_init(acc_empty + 0, 4);
        mbar_init(acc_empty + 1, 4);
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int c = threadIdx.x; c < NP; c += kThreads) {
        al_s[c] = c < a.width ? a.al[c] : 0.f;
        ar_s[c] = c < a.width ? a.ar[c] : 0.f;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                     "r"(a.tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer ----
            mbar_expect_tx(w_full, uint32_t(KB) * NP * 128);
            for (int k = 0; k < KB; ++k) tma_load_2d(w_s + size_t(k) * NP * 128, &tm_w, w_full, k * kKBlock, 0);
            uint64_t kc = 0;
            bool ok = true;
            for (uint64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                for (int k = 0; k < KB; ++k, ++kc) {
                    const int s = int(kc % S);
                    const uint32_t ph = uint32_t(kc / S) & 1u;
                    if (!mbar_wait(empty + s, ph ^ 1u, abort_flag)) { ok = false; break; }
                    mbar_expect_tx(full + s, kABytes);
                    tma_load_2d(a_s + size_t(s) * kABytes, &tm_x, full + s, k * kKBlock, int(t * kTileM));
                }
            }
            // Wait (bounded) until every load this thread issued has landed.
            mbar_wait(w_full, 0, abort_flag);
            for (int s = 0; s < S; ++s) {
                if (kc > uint64_t(s)) {
                    uint64_t last = kc - 1 - ((kc - 1 - s) % S);  // last k-block index that used stage s
                    mbar_wait(full + s, uint32_t(last / S) & 1u, abort_flag);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer ----
            const uint32_t idesc = (1u << 4)            // D = F32
                                   | (1u << 7)          // A = BF16
                                   | (1u << 10)         // B = BF16
                                   | (uint32_t(NP >> 3) << 17)  // N
                                   | (uint32_t(kTileM >> 4) << 24);  // M
            bool ok = mbar_wait(w_full, 0, abort_flag);
            tc::fence_after();
            uint64_t kc = 0;
            uint32_t t_local = 0;
            for (uint64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++t_local) {
                const uint32_t buf = t_local & 1u, use = t_local >> 1;
                if (!mbar_wait(acc_empty + buf, (use & 1u) ^ 1u, abort_flag)) { ok = false; break; }
                tc::fence_after();
                const uint32_t d_tmem = tmem_base + buf * (a.tmem_cols / 2);
                for (int k = 0; k < KB; ++k, ++kc) {
                    const int s = int(kc % S);
                    if (!mbar_wait(full + s, uint32_t(kc / S) & 1u, abort_flag)) { ok = false; break; }
                    tc::fence_after();
                    const uint32_t a_addr = smem_u32(a_s + size_t(s) * kABytes);
                    const uint32_t b_addr = smem_u32(w_s + size_t(k) * NP * 128);
#pragma unroll
                    for (int kk = 0; kk < kKBlock / 16; ++kk)
                        mma_bf16(d_tmem, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), idesc,
                                 (k | kk) ? 1u : 0u);
                    mma_commit(empty + s);
                }
                if (!ok) break;
                mma_commit(acc_full + buf);
            }
            // All MMAs issued so far complete before this barrier fires.
            mma_commit(mma_done);
            mbar_wait(mma_done, 0, abort_flag);
        }
    } else {
        // ---- epilogue: warps 2..9, TMEM lane quarter = warp % 4; set b = (warp-2)/4
        // takes the CTA's tiles of parity b, i.e. accumulator b ----
        const int q = warp & 3;
        const int ew = warp - 2;  // staging slot
        const uint32_t buf = uint32_t(ew >> 2);
        uint8_t* stage0 = st_s + size_t(ew) * a.sb * kStageBytes;
        uint32_t toggle = 0;
        uint32_t use = 0;
        for (uint64_t t = blockIdx.x + buf * gridDim.x; t < ntiles; t += 2ull * gridDim.x, ++use) {
            if (!mbar_wait(acc_full + buf, use & 1u, abort_flag)) break;
            tc::fence_after();
            const uint64_t row = t * kTileM + uint64_t(q) * 32 + lane;
            const uint32_t taddr = tmem_base + (uint32_t(q * 32) << 16) + buf * (a.tmem_cols / 2);
            float L[8], R[8];
#pragma unroll
            for (int h = 0; h < 8; ++h) { L[h] = 0.f; R[h] = 0.f; }
#pragma unroll
            for (int g = 0; g < NP; g += 64) {
                uint8_t* sb = stage0 + toggle * kStageBytes;
                if (lane == 0 && a.store_h) {
                    if (a.sb == 2)
                        bulk_wait_read<1>();  // the store that last used this buffer has read it
                    else
                        bulk_wait_read<0>();
                }
                __syncwarp();
                // 16 accumulator columns c..c+15 of this row (sub-block cc of the group)
                auto col16 = [&](int cc, const float* v) {
                    const int c = g + cc * 16;
                    if constexpr (ALIGNED16 && NPT != 0) {
                        // c is a constant here: the same FMA chains as below
                        float pl = 0.f, pr = 0.f;
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            pl = fmaf(v[j], a.alc[c + j], pl);
                            pr = fmaf(v[j], a.arc[c + j], pr);
                        }
                        const int hh = KT == 1 ? 0 : c / (NPT / KT);
                        L[hh] += pl;
                        R[hh] += pr;
                    } else if constexpr (ALIGNED16) {
                        // the block's 16 coefficients as four 16-byte reads
                        const float4* l4 = reinterpret_cast<const float4*>(al_s + c);
                        const float4* r4 = reinterpret_cast<const float4*>(ar_s + c);
                        float pl = 0.f, pr = 0.f;
#pragma unroll
                        for (int j4 = 0; j4 < 4; ++j4) {
                            const float4 x = l4[j4], y = r4[j4];
                            const float* vv = v + 4 * j4;
                            pl = fmaf(vv[0], x.x, pl);
                            pl = fmaf(vv[1], x.y, pl);
                            pl = fmaf(vv[2], x.z, pl);
                            pl = fmaf(vv[3], x.w, pl);
                            pr = fmaf(vv[0], y.x, pr);
                            pr = fmaf(vv[1], y.y, pr);
                            pr = fmaf(vv[2], y.z, pr);
                            pr = fmaf(vv[3], y.w, pr);
                        }
                        const int hh = c / a.dim;
#pragma unroll
                        for (int h = 0; h < 8; ++h)
                            if (h == hh) { L[h] += pl; R[h] += pr; }
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int hh = (c + j) / a.dim;
                            const float xl = v[j] * al_s[c + j], xr = v[j] * ar_s[c + j];
#pragma unroll
                            for (int h = 0; h < 8; ++h)
                                if (h == hh) { L[h] += xl; R[h] += xr; }
                        }
                    }
                    if (a.z && row < a.n) {
                        float* zr = a.z + row * uint64_t(a.ldz) + c;
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (c + j < a.width) zr[j] = v[j];
                    }
                    if (!a.store_h) return;
                    uint32_t pk[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) pk[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
                    // 16-byte chunks 2cc and 2cc+1 of this row, 128B swizzle.
                    const int c0 = (2 * cc) ^ (lane & 7), c1 = (2 * cc + 1) ^ (lane & 7);
                    *reinterpret_cast<uint4*>(sb + lane * 128 + c0 * 16) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    *reinterpret_cast<uint4*>(sb + lane * 128 + c1 * 16) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                };
                if (g + 64 <= NP) {
                    // one TMEM read (and one wait) for the group's 64 columns
                    float v64[64];
                    tc::tmem_ld64(taddr + uint32_t(g), v64);
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) col16(cc, v64 + cc * 16);
                } else {
#pragma unroll
                    for (int cc = 0; cc < 4 && g + cc * 16 < NP; ++cc) {
                        float v[16];
                        tmem_ld16(taddr + uint32_t(g + cc * 16), v);
                        col16(cc, v);
                    }
                }
                if (!a.store_h) continue;
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tm_h, sb, g, int(t * kTileM) + q * 32);
                    bulk_commit();
                }
                if (a.npeer) {
                    // the same 32 x 64 box to every peer table: 16-byte stores,
                    // lanes 8 at a time along a 128-byte row segment
                    const uint64_t r0 = t * kTileM + uint64_t(q) * 32;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int rr = i * 4 + (lane >> 3), ch = lane & 7;
                        const int col = g + ch * 8;
                        if (r0 + rr < a.n && col < a.ldh) {
                            const uint4 v = *reinterpret_cast<const uint4*>(sb + rr * 128 + ((ch ^ (rr & 7)) * 16));
                            const uint64_t off = (r0 + rr) * uint64_t(a.ldh) + col;
#pragma unroll
                            for (int pi = 0; pi < kMaxPeers; ++pi)
                                if (pi < a.npeer) *reinterpret_cast<uint4*>(a.hp[pi] + off) = v;
                        }
                    }
                }
                if (a.sb == 2) toggle ^= 1u;
            }
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + buf);
            if (row < a.n) {
                if (a.lr_vec) {
                    float4* lp = reinterpret_cast<float4*>(a.left + row * 8);
                    float4* rp = reinterpret_cast<float4*>(a.right + row * 8);
                    const float4 r0 = make_float4(R[0], R[1], R[2], R[3]), r1 = make_float4(R[4], R[5], R[6], R[7]);
                    if (a.left) { lp[0] = make_float4(L[0], L[1], L[2], L[3]); lp[1] = make_float4(L[4], L[5], L[6], L[7]); }
                    if (a.right) { rp[0] = r0; rp[1] = r1; }
#pragma unroll
                    for (int pi = 0; pi < kMaxPeers; ++pi)
                        if (pi < a.npeer) {
                            float4* pp = reinterpret_cast<float4*>(a.rp[pi] + row * 8);
                            pp[0] = r0;
                            pp[1] = r1;
                        }
                } else {
#pragma unroll
                    for (int h = 0; h < 8; ++h)
                        if (h < a.heads) {
                            if (a.left) a.left[row * a.heads + h] = L[h];
                            if (a.right) a.right[row * a.heads + h] = R[h];
#pragma unroll
                            for (int pi = 0; pi < kMaxPeers; ++pi)
                                if (pi < a.npeer) a.rp[pi][row * a.heads + h] = R[h];
                        }
                }
            }
        }
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(a.tmem_cols));
    }
}

// ---- host side -------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D BF16 tensor map: inner extent `cols`, `rows` rows, row pitch `ld` elements.
int make_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_cols,
             uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail_code(GAT_B200_ECUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail_code(GAT_B200_ECUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return 0;
}

}  // namespace

// Row-gather map of a BF16 feature table (the aggregation's tile::gather4
// loads): `rows` rows of `cols` elements at a pitch of `ld` elements, boxes of
// one row of box_cols elements, no swizzle, zeros outside the table.
int make_row_gather_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t ld,
                        uint32_t box_cols) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail_code(GAT_B200_ECUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {box_cols, 1};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail_code(GAT_B200_ECUDA, "cuTensorMapEncodeTiled (row gather) failed (" + std::to_string(int(r)) + ")");
    return 0;
}

// Returns GAT_B200_EUNSUPPORTED when the shape is outside the kernel (the
// caller then uses the CUDA-core projection).
// max_ctas > 0 caps the persistent grid (the multi-GPU forward runs this
// kernel beside an aggregation that leaves that many SMs free).
int projection_tc_launch(const gat_b200_layer* p, uint64_t n, const uint16_t* x, int ldx, uint16_t* h, int ldh,
                         float* z, int ldz, float* left, float* right, cudaStream_t st, int npeer,
                         uint16_t* const* h_peer, float* const* r_peer, int max_ctas) {
    if (p->np > 256 || p->kp > 256) return GAT_B200_EUNSUPPORTED;
    if (n == 0) return 0;
    if (n > uint64_t(INT32_MAX)) return fail("projection: too many rows");
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (uint64_t(ldx) * 2) % 16) return fail("projection: X rows must be 16-byte aligned");
    if (h && ((reinterpret_cast<uintptr_t>(h) & 15) || (uint64_t(ldh) * 2) % 16 || ldh < p->width))
        return fail("projection: H rows must be 16-byte aligned and hold the width");
    if (z && ldz < p->width) return fail("projection: Z row stride smaller than the width");
    ProjArgs a{};
    a.n = n;
    a.heads = p->heads;
    a.dim = p->dim;
    a.width = p->width;
    a.np = p->np;
    a.kb = p->kp / kKBlock;
    a.left = left;
    a.right = right;
    a.z = z;
    a.ldz = ldz;
    a.al = p->al;
    a.ar = p->ar;
    a.store_h = h != nullptr;
    a.lr_vec = p->heads == 8 && (reinterpret_cast<uintptr_t>(left) & 15) == 0 &&
               (reinterpret_cast<uintptr_t>(right) & 15) == 0;
    if (npeer < 0 || npeer > kMaxPeers) return fail("projection: at most 7 peer destinations");
    if (npeer && (!h || !right)) return fail("projection: peer destinations need H and R");
    a.npeer = npeer;
    a.ldh = ldh;
    for (int i = 0; i < npeer; ++i) {
        if (!h_peer[i] || !r_peer[i]) return fail("projection: null peer destination");
        if (reinterpret_cast<uintptr_t>(h_peer[i]) & 15) return fail("projection: peer H rows must be 16-byte aligned");
        if (reinterpret_cast<uintptr_t>(r_peer[i]) & 15) a.lr_vec = 0;  // R rows then go out as scalars
        a.hp[i] = h_peer[i];
        a.rp[i] = r_peer[i];
    }
    uint32_t cols = 32;
    while (cols < uint32_t(2 * p->np)) cols <<= 1;
    a.tmem_cols = cols;
    // Two staging buffers per epilogue warp unless that leaves fewer than 4
    // stages for X (layers with a 256-row W^T), then one.
    const size_t limit = 227 * 1024;
    int S = 0;
    for (a.sb = 2; a.sb >= 1; --a.sb) {
        const size_t fixed_sb = size_t(a.kb) * p->np * 128 + size_t(kEpiWarps) * a.sb * kStageBytes +
                                2 * size_t(p->np) * 4 + 512 + 1024;
        S = fixed_sb < limit ? int((limit - fixed_sb) / kABytes) : 0;
        if (S >= 4 || a.sb == 1) break;
    }
    S = S > 8 ? 8 : S;
    if (S < 2) return GAT_B200_EUNSUPPORTED;
    const size_t fixed = size_t(a.kb) * p->np * 128 + size_t(kEpiWarps) * a.sb * kStageBytes +
                         2 * size_t(p->np) * 4 + 512 + 1024;
    a.stages = S;
    size_t smem = fixed + size_t(S) * kABytes;
    // 512 TMEM columns are only safe with one CTA per SM: make the shared
    // memory request rule out a second resident CTA.
    if (cols > 256 && smem < 120 * 1024) smem = 120 * 1024;

    CUtensorMap tm_x, tm_w, tm_h;
    int rc;
    if ((rc = make_map(&tm_x, x, uint64_t(p->in), n, uint64_t(ldx), kKBlock, kTileM))) return rc;
    if ((rc = make_map(&tm_w, p->wt_bf16, uint64_t(p->kp), uint64_t(p->np), uint64_t(p->kp), kKBlock, uint32_t(p->np)))) return rc;
    if (h) {
        if ((rc = make_map(&tm_h, h, uint64_t(ldh), n, uint64_t(ldh), 64, kStageRows))) return rc;
    } else {
        tm_h = tm_x;  // never used when store_h == 0
    }

    int dev = 0, sms = 0;
    GATB_CUDA(cudaGetDevice(&dev));
    GATB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const uint64_t ntiles = (n + kTileM - 1) / kTileM;
    const uint64_t cap = max_ctas > 0 && max_ctas < sms ? uint64_t(max_ctas) : uint64_t(sms);
    const unsigned grid = unsigned(ntiles < cap ? ntiles : cap);
    // Heads aligned to 16 columns (or a single head, whose columns past the
    // width carry zero coefficients): one head per 16-column block.
    // Shape-specialised epilogues: 8 heads x 32 (the hidden layers) and one
    // head of 48 or 64 padded columns (class logits).
    for (int c = 0; c < kMaxCoef; ++c) {
        a.alc[c] = c < p->width && c < int(p->al_host.size()) ? p->al_host[c] : 0.f;
        a.arc[c] = c < p->width && c < int(p->ar_host.size()) ? p->ar_host[c] : 0.f;
    }
    const bool coef = int(p->al_host.size()) == p->width && int(p->ar_host.size()) == p->width;
    auto launch = [&](auto kern) -> int {
        GATB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
        kern<<<grid, kThreads, smem, st>>>(tm_x, tm_w, tm_h, a);
        return 0;
    };
    if (coef && p->heads == 8 && p->dim == 32 && p->np == 256)
        rc = launch(proj_tc_kernel<true, 256, 8>);
    else if (coef && p->heads == 1 && p->np == 48)
        rc = launch(proj_tc_kernel<true, 48, 1>);
    else if (coef && p->heads == 1 && p->np == 64)
        rc = launch(proj_tc_kernel<true, 64, 1>);
    else if (p->dim % 16 == 0 || p->heads == 1)
        rc = launch(proj_tc_kernel<true, 0, 0>);
    else
        rc = launch(proj_tc_kernel<false, 0, 0>);
    if (rc) return rc;
    GATB_LAUNCH("projection (tcgen05) kernel");
    return 0;
}

int projection_tc_check_error() {
    unsigned e = 0;
    GATB_CUDA(cudaMemcpyFromSymbol(&e, g_proj_error, sizeof(e)));
    if (e) {
        unsigned z = 0;
        cudaMemcpyToSymbol(g_proj_error, &z, sizeof(z));
        return fail_code(GAT_B200_ETIMEOUT, "projection kernel: a bounded wait timed out");
    }
    return 0;
}

}  // namespace gatb
