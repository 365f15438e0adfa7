// Small stage kernels: FP32->BF16 convert, max prescan, finish, and the
// CUDA-core projection (FP32 path, and the BF16 path for shapes outside the
// tensor-core kernel).
#include "device.cuh"
#include "graph.cuh"

namespace gatb {
namespace {

// Two FP32 -> BF16 RNE conversions (low, high) with the reference's NaN rule
// (baseline/src/common.cpp:80-84): a NaN keeps its sign and payload bits and
// gets the quiet bit, instead of the hardware's canonical NaN.
__device__ __forceinline__ uint32_t rne_pair(float lo, float hi) {
    uint32_t r = pack_bf16x2(lo, hi);
    if (lo != lo) r = (r & 0xffff0000u) | ((__float_as_uint(lo) >> 16) | 0x40u);
    if (hi != hi) r = (r & 0x0000ffffu) | (((__float_as_uint(hi) >> 16) | 0x40u) << 16);
    return r;
}

// baseline/src/common.cpp:85-93: FP32 -> BF16 RNE, here with a padded output
// stride whose padding columns are written as zero.
__global__ void convert_kernel(uint64_t n, int width, const float* __restrict__ in, int ld_in,
                               uint16_t* __restrict__ out, int ld_out) {
    const uint64_t total = n * uint64_t(ld_out / 2);  // pairs of output columns
    for (uint64_t t = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; t < total;
         t += uint64_t(gridDim.x) * blockDim.x) {
        uint64_t r = t / uint64_t(ld_out / 2);
        int c = int(t % uint64_t(ld_out / 2)) * 2;
        const float* src = in + r * uint64_t(ld_in);
        float a = c < width ? src[c] : 0.f;
        float b = c + 1 < width ? src[c + 1] : 0.f;
        reinterpret_cast<uint32_t*>(out + r * uint64_t(ld_out))[c / 2] = rne_pair(a, b);
    }
}

// The same conversion, 8 output columns (one 16-byte store) per thread, for
// 16-byte aligned rows in and out (ld_in % 4 == 0, ld_out % 8 == 0).
__global__ void convert_vec_kernel(uint64_t n, int width, const float* __restrict__ in, int ld_in,
                                   uint16_t* __restrict__ out, int ld_out) {
    const int chunks = ld_out / 8;
    const uint64_t total = n * uint64_t(chunks);
    for (uint64_t t = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; t < total;
         t += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t r = t / uint64_t(chunks);
        const int c = int(t % uint64_t(chunks)) * 8;
        const float* src = in + r * uint64_t(ld_in) + c;
        float v[8];
        if (c + 8 <= width) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(src));
            const float4 b = __ldg(reinterpret_cast<const float4*>(src + 4));
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = c + k < width ? src[k] : 0.f;
        }
        *reinterpret_cast<uint4*>(out + r * uint64_t(ld_out) + c) =
            make_uint4(rne_pair(v[0], v[1]), rne_pair(v[2], v[3]), rne_pair(v[4], v[5]), rne_pair(v[6], v[7]));
    }
}

// The layer-1 input exchange of the partitioned multi-GPU forward: the
// conversion of convert_vec_kernel (any input alignment), each 16-byte result
// stored to `ndst` destinations -- this rank's block of its input table and
// the same block of every peer's table, mapped over NVLink. Consecutive
// threads store consecutive 16-byte pieces, so each destination receives
// whole contiguous rows.
struct ConvertDst {
    uint16_t* d[8];
};
__global__ void convert_scatter_kernel(uint64_t n, int width, const float* __restrict__ in, int ld_in, bool vec_in,
                                       ConvertDst dst, int ndst, int ld_out) {
    const int chunks = ld_out / 8;
    const uint64_t total = n * uint64_t(chunks);
    for (uint64_t t = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; t < total;
         t += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t r = t / uint64_t(chunks);
        const int c = int(t % uint64_t(chunks)) * 8;
        const float* src = in + r * uint64_t(ld_in) + c;
        float v[8];
        if (vec_in && c + 8 <= width) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(src));
            const float4 b = __ldg(reinterpret_cast<const float4*>(src + 4));
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = c + k < width ? src[k] : 0.f;
        }
        const uint4 o = make_uint4(rne_pair(v[0], v[1]), rne_pair(v[2], v[3]), rne_pair(v[4], v[5]),
                                   rne_pair(v[6], v[7]));
        const uint64_t off = r * uint64_t(ld_out) + c;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (j < ndst) *reinterpret_cast<uint4*>(dst.d[j] + off) = o;
    }
}

// baseline/src/baseline_standard.cpp:44-51 (one warp per row).
__global__ void max_prescan_kernel(const uint64_t* __restrict__ row, const uint32_t* __restrict__ col,
                                   uint64_t n, int heads, const float* __restrict__ left,
                                   const float* __restrict__ right, float* __restrict__ max) {
    const int lane = threadIdx.x & 31;
    for (uint64_t i = (blockIdx.x * uint64_t(blockDim.x) + threadIdx.x) >> 5; i < n;
         i += (uint64_t(gridDim.x) * blockDim.x) >> 5) {
        float mr[8];
#pragma unroll
        for (int h = 0; h < 8; ++h) mr[h] = -INFINITY;
        for (uint64_t e = row[i] + lane; e < row[i + 1]; e += 32) {
            uint32_t s = col[e];
#pragma unroll
            for (int h = 0; h < 8; ++h)
                if (h < heads) mr[h] = fmaxf(mr[h], right[uint64_t(s) * heads + h]);
        }
#pragma unroll
        for (int h = 0; h < 8; ++h) mr[h] = warp_max(mr[h]);
        const bool empty = row[i] == row[i + 1];
#pragma unroll
        for (int h = 0; h < 8; ++h)
            if (h < heads && lane == h) max[i * heads + h] = empty ? 0.f : leaky(mr[h] + left[i * heads + h]);
    }
}

// R0's edge softmax (baseline/src/ref_fp32.cpp:7-14), one thread per (row,
// head) so that the maximum and the FP32 sum of p run over the row's edges in
// the reference's order: score = leaky(L_ih + R_jh), m = the row maximum (0 for
// an empty row), p = exp(score - m), den = sum p, alpha = p / den.
__global__ void edge_softmax_kernel(const uint64_t* __restrict__ row, const uint32_t* __restrict__ col, uint64_t n,
                                    int heads, const float* __restrict__ left, const float* __restrict__ right,
                                    float* __restrict__ score, float* __restrict__ max, float* __restrict__ p,
                                    float* __restrict__ den, float* __restrict__ alpha) {
    const uint64_t total = n * uint64_t(heads);
    for (uint64_t t = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; t < total;
         t += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t i = t / uint64_t(heads);
        const int h = int(t - i * uint64_t(heads));
        const uint64_t b = row[i], e_end = row[i + 1];
        const float l = left[t];
        float m = -INFINITY;
        for (uint64_t e = b; e < e_end; ++e) m = fmaxf(m, leaky(l + right[uint64_t(col[e]) * heads + h]));
        float sum = 0.f;
        for (uint64_t e = b; e < e_end; ++e) {
            const float sc = leaky(l + right[uint64_t(col[e]) * heads + h]);
            const float v = expf(sc - m);
            if (score) score[e * heads + h] = sc;
            p[e * heads + h] = v;
            sum += v;
        }
        den[t] = sum;
        if (max) max[t] = b == e_end ? 0.f : m;
        if (alpha)
            for (uint64_t e = b; e < e_end; ++e) alpha[e * heads + h] = p[e * heads + h] / sum;
    }
}

// baseline/src/baseline_standard.cpp:85-97
__global__ void finish_kernel(uint64_t n, int heads, int dim, const float* __restrict__ den, int hidden,
                              float* __restrict__ out, int ldo) {
    const int width = heads * dim;
    const uint64_t total = n * uint64_t(width);
    for (uint64_t t = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; t < total;
         t += uint64_t(gridDim.x) * blockDim.x) {
        uint64_t r = t / width;
        int c = int(t % width);
        float d = den[r * heads + c / dim];
        float v = out[r * ldo + c] * (d > 0.f ? 1.f / d : 0.f);
        if (hidden) v = elu(v);
        out[r * ldo + c] = v;
    }
}

// CUDA-core projection: Z = X W (FP32 accumulate over k ascending in blocks of
// 32), left/right = Z_h . aL_h / aR_h, Z stored as FP32 or BF16 RNE.
// Block: kRows rows x all `width` columns, 256 threads.
constexpr int kRows = 32;
constexpr int kKb = 32;
template <class XT>
__global__ void __launch_bounds__(256) projection_simt_kernel(
    uint64_t n, int in, int heads, int dim, const XT* __restrict__ x, int ldx, const float* __restrict__ w,
    int quantize_w, const float* __restrict__ al, const float* __restrict__ ar, void* __restrict__ h,
    int h_bf16, int ldh, float* __restrict__ left, float* __restrict__ right) {
    extern __shared__ float smem[];
    const int width = heads * dim;
    float* xs = smem;                 // [kRows][kKb]
    float* ws = xs + kRows * kKb;     // [kKb][width]
    float* zs = ws + kKb * width;     // [kRows][width+1]
    const int zld = width + 1;
    const uint64_t r0 = blockIdx.x * uint64_t(kRows);
    const int tid = threadIdx.x;
    constexpr int CPT = 2;  // columns per thread (width <= 512)
    float acc[CPT][kRows];
#pragma unroll
    for (int j = 0; j < CPT; ++j)
#pragma unroll
        for (int r = 0; r < kRows; ++r) acc[j][r] = 0.f;
    for (int k0 = 0; k0 < in; k0 += kKb) {
        for (int t = tid; t < kRows * kKb; t += 256) {
            int r = t / kKb, k = t % kKb;
            float v = 0.f;
            if (r0 + r < n && k0 + k < in) {
                if constexpr (sizeof(XT) == 2)
                    v = __uint_as_float(uint32_t(x[(r0 + r) * ldx + k0 + k]) << 16);
                else
                    v = x[(r0 + r) * ldx + k0 + k];
            }
            xs[t] = v;
        }
        for (int t = tid; t < kKb * width; t += 256) {
            int k = t / width, c = t % width;
            float v = k0 + k < in ? w[uint64_t(k0 + k) * width + c] : 0.f;
            if (quantize_w) v = __uint_as_float((pack_bf16x2(v, 0.f) & 0xffffu) << 16);
            ws[t] = v;
        }
        __syncthreads();
        const int kmax = min(kKb, in - k0);
        for (int k = 0; k < kmax; ++k) {
            float wv[CPT];
#pragma unroll
            for (int j = 0; j < CPT; ++j) {
                int c = tid + j * 256;
                wv[j] = c < width ? ws[k * width + c] : 0.f;
            }
#pragma unroll
            for (int r = 0; r < kRows; ++r) {
                float xv = xs[r * kKb + k];
#pragma unroll
                for (int j = 0; j < CPT; ++j) acc[j][r] = fmaf(xv, wv[j], acc[j][r]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
        int c = tid + j * 256;
        if (c < width)
#pragma unroll
            for (int r = 0; r < kRows; ++r) zs[r * zld + c] = acc[j][r];
    }
    __syncthreads();
    // Attention dots, sequential over the head's columns (lr_from_z scalar form).
    for (int t = tid; t < kRows * heads; t += 256) {
        int r = t / heads, hh = t % heads;
        if (r0 + r >= n) continue;
        float l = 0.f, rr = 0.f;
        for (int d = 0; d < dim; ++d) {
            float z = zs[r * zld + hh * dim + d];
            l = fmaf(z, al[hh * dim + d], l);
            rr = fmaf(z, ar[hh * dim + d], rr);
        }
        if (left) left[(r0 + r) * heads + hh] = l;
        if (right) right[(r0 + r) * heads + hh] = rr;
    }
    if (h) {
        for (int t = tid; t < kRows * ldh; t += 256) {
            int r = t / ldh, c = t % ldh;
            if (r0 + r >= n) continue;
            float z = c < width ? zs[r * zld + c] : 0.f;
            if (h_bf16)
                static_cast<uint16_t*>(h)[(r0 + r) * ldh + c] = uint16_t(pack_bf16x2(z, 0.f) & 0xffffu);
            else
                static_cast<float*>(h)[(r0 + r) * ldh + c] = z;
        }
    }
}

unsigned grid_for(uint64_t work, int per_block) {
    uint64_t b = (work + per_block - 1) / per_block;
    if (b > 148ull * 64) b = 148ull * 64;
    return unsigned(b ? b : 1);
}

}  // namespace

int convert_launch(uint64_t n, int width, const float* in, int ld_in, uint16_t* out, int ld_out, cudaStream_t st) {
    if (!in || !out) return fail("convert: null buffer");
    if (ld_in < width || ld_out < width || (ld_out & 1)) return fail("convert: bad row strides");
    if ((reinterpret_cast<uintptr_t>(in) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
        ld_in % 4 == 0 && ld_out % 8 == 0)
        convert_vec_kernel<<<grid_for(n * uint64_t(ld_out / 8), 256), 256, 0, st>>>(n, width, in, ld_in, out,
                                                                                     ld_out);
    else
        convert_kernel<<<grid_for(n * uint64_t(ld_out / 2), 256), 256, 0, st>>>(n, width, in, ld_in, out, ld_out);
    GATB_LAUNCH("convert kernel");
    return 0;
}

int convert_scatter_launch(uint64_t n, int width, const float* in, int ld_in, int ndst, uint16_t* const* dst,
                           int ld_out, cudaStream_t st) {
    if (!in || !dst) return fail("convert_scatter: null buffer");
    if (ndst < 1 || ndst > 8) return fail("convert_scatter: 1..8 destinations");
    if (ld_in < width || ld_out < width || ld_out % 8) return fail("convert_scatter: bad row strides");
    ConvertDst d{};
    for (int j = 0; j < ndst; ++j) {
        if (!dst[j] || (reinterpret_cast<uintptr_t>(dst[j]) & 15)) return fail("convert_scatter: destinations must be 16-byte aligned");
        d.d[j] = dst[j];
    }
    if (n == 0) return 0;
    const bool vec_in = (reinterpret_cast<uintptr_t>(in) & 15) == 0 && ld_in % 4 == 0;
    convert_scatter_kernel<<<grid_for(n * uint64_t(ld_out / 8), 256), 256, 0, st>>>(n, width, in, ld_in, vec_in, d,
                                                                                    ndst, ld_out);
    GATB_LAUNCH("convert scatter kernel");
    return 0;
}

int max_prescan_launch(const gat_b200_graph* g, int heads, const float* left, const float* right, float* max,
                       cudaStream_t st) {
    if (!g || !left || !right || !max) return fail("max_prescan: null buffer");
    if (heads < 1 || heads > 8) return fail("invalid parameter shape (heads <=8, head_dim <=64)");
    max_prescan_kernel<<<grid_for(g->n * 32, 256), 256, 0, st>>>(g->row, g->col, g->n, heads, left, right, max);
    GATB_LAUNCH("max prescan kernel");
    return 0;
}

int edge_softmax_launch(const gat_b200_graph* g, int heads, const float* left, const float* right, float* score,
                        float* max, float* p, float* den, float* alpha, cudaStream_t st) {
    if (!g || !left || !right || !p || !den) return fail("edge_softmax: null buffer");
    if (heads < 1 || heads > 8) return fail("invalid parameter shape (heads <=8, head_dim <=64)");
    if (g->n == 0) return 0;
    edge_softmax_kernel<<<grid_for(g->n * uint64_t(heads), 256), 256, 0, st>>>(g->row, g->col, g->n, heads, left,
                                                                               right, score, max, p, den, alpha);
    GATB_LAUNCH("edge softmax kernel");
    return 0;
}

int finish_launch(uint64_t n, int heads, int dim, const float* den, int hidden, float* out, int ldo, cudaStream_t st) {
    if (!den || !out) return fail("finish: null buffer");
    if (heads < 1 || heads > 8 || dim < 1 || dim > 64) return fail("invalid parameter shape (heads <=8, head_dim <=64)");
    if (ldo < heads * dim) return fail("finish: row stride smaller than the width");
    finish_kernel<<<grid_for(n * uint64_t(heads * dim), 256), 256, 0, st>>>(n, heads, dim, den, hidden, out, ldo);
    GATB_LAUNCH("finish kernel");
    return 0;
}

int projection_simt_launch(const gat_b200_layer* p, uint64_t n, const void* x, int x_bf16, int ldx, void* h,
                           int h_bf16, int ldh, float* left, float* right, cudaStream_t st) {
    const size_t smem = (size_t(kRows) * kKb + size_t(kKb) * p->width + size_t(kRows) * (p->width + 1)) * sizeof(float);
    unsigned blocks = unsigned((n + kRows - 1) / kRows);
    if (x_bf16) {
        auto k = projection_simt_kernel<uint16_t>;
        GATB_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
        k<<<blocks, 256, smem, st>>>(n, p->in, p->heads, p->dim, static_cast<const uint16_t*>(x), ldx, p->w, 1,
                                     p->al, p->ar, h, h_bf16, ldh, left, right);
    } else {
        auto k = projection_simt_kernel<float>;
        GATB_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
        k<<<blocks, 256, smem, st>>>(n, p->in, p->heads, p->dim, static_cast<const float*>(x), ldx, p->w, 0,
                                     p->al, p->ar, h, h_bf16, ldh, left, right);
    }
    GATB_LAUNCH("projection (CUDA cores) kernel");
    return 0;
}

}  // namespace gatb
