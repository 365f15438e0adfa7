// RMAT stress graph, generated on the current CUDA device.
//
// Edge k (k < edges) picks one quadrant per level of the 2^lg x 2^lg
// adjacency matrix with probabilities (a, b, c, 1-a-b-c): a = (0,0),
// b = (0,1), c = (1,0), d = (1,1), the first bit being the source's and the
// second the destination's, most significant level first. The draw of level l
// is unit(rng(seed, 7, k*lg + l)), the same counter-based stream as the host
// generators, so the graph is identical on every device and for every launch
// shape. Every node also gets a self loop. The destination-row CSR keeps each
// (destination, source) pair once (generated self edges merge with the self
// loop) with sources ascending:
//   keys = (dst << lg) | src for all edges and self loops -> radix sort ->
//   unique -> row[i] = first key >= (i << lg), col = key & (2^lg - 1).
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_select.cuh>

#include "device.cuh"

namespace gatb {
namespace {

__device__ __forceinline__ uint64_t splitmix64_d(uint64_t x) {
    x += 0x9e3779b97f4a7c15ULL;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
    return x ^ (x >> 31);
}

// base = splitmix64(seed ^ splitmix64(stream + c)): rng(seed, stream, i) = splitmix64(base + i).
uint64_t splitmix64_h(uint64_t x) {
    x += 0x9e3779b97f4a7c15ULL;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
    return x ^ (x >> 31);
}

__global__ void rmat_keys(uint64_t edges, uint64_t nodes, int lg, uint64_t base, double ta, double tab,
                          double tabc, uint64_t* __restrict__ keys) {
    const uint64_t total = edges + nodes;
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t k = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; k < total; k += stride) {
        if (k >= edges) {
            const uint64_t i = k - edges;
            keys[k] = (i << lg) | i;
            continue;
        }
        uint64_t src = 0, dst = 0;
        for (int l = 0; l < lg; ++l) {
            const double u = double(splitmix64_d(base + k * uint64_t(lg) + uint64_t(l)) >> 11) *
                             (1.0 / 9007199254740992.0);
            const uint64_t bs = u >= tab ? 1u : 0u;              // c or d
            const uint64_t bd = (u >= ta && u < tab) || u >= tabc ? 1u : 0u;  // b or d
            src = (src << 1) | bs;
            dst = (dst << 1) | bd;
        }
        keys[k] = (dst << lg) | src;
    }
}

__global__ void rmat_rowptr(const uint64_t* __restrict__ keys, uint64_t e, uint64_t nodes, int lg,
                            uint64_t* __restrict__ row) {
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i <= nodes; i += stride) {
        const uint64_t want = i << lg;
        uint64_t lo = 0, hi = e;  // first key >= want
        while (lo < hi) {
            const uint64_t mid = (lo + hi) >> 1;
            if (keys[mid] < want) lo = mid + 1; else hi = mid;
        }
        row[i] = lo;
    }
}

__global__ void rmat_cols(const uint64_t* __restrict__ keys, uint64_t beg, uint64_t count, uint64_t mask,
                          uint32_t* __restrict__ col) {
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t k = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; k < count; k += stride)
        col[k] = uint32_t(keys[beg + k] & mask);
}

}  // namespace
}  // namespace gatb

extern "C" int gat_b200_synth_rmat(int log2_nodes, uint64_t edges, double a, double b, double c, uint64_t seed,
                                   uint64_t r_lo, uint64_t r_hi, uint64_t* row, uint32_t* col, uint64_t* e_total) {
    using namespace gatb;
    clear_error();
    if (log2_nodes < 1 || log2_nodes > 31) return fail("rmat: log2_nodes must be 1..31");
    if (!(a > 0 && b >= 0 && c >= 0 && a + b + c < 1.0)) return fail("rmat: need a > 0, b, c >= 0, a+b+c < 1");
    const uint64_t nodes = uint64_t(1) << log2_nodes;
    if (!row) return fail("rmat: null row output");
    if (r_lo > r_hi || r_hi > nodes) return fail("rmat: bad row range");
    const uint64_t total = edges + nodes;
    if (total >= (uint64_t(1) << 31)) return fail("rmat: edges + nodes must stay below 2^31");
    const int items = int(total);
    uint64_t *k0 = nullptr, *k1 = nullptr, *rowd = nullptr;
    int* nsel = nullptr;
    uint32_t* cold = nullptr;
    void* temp = nullptr;
    int rc = 0;
    cudaStream_t st = 0;
    auto cleanup = [&] {
        cudaFree(k0);
        cudaFree(k1);
        cudaFree(rowd);
        cudaFree(nsel);
        cudaFree(cold);
        cudaFree(temp);
    };
    do {
        cudaError_t ce;
        if ((ce = cudaMalloc(&k0, total * 8)) != cudaSuccess) { rc = cuda_fail(ce, "rmat keys"); break; }
        if ((ce = cudaMalloc(&k1, total * 8)) != cudaSuccess) { rc = cuda_fail(ce, "rmat keys"); break; }
        if ((ce = cudaMalloc(&nsel, sizeof(int))) != cudaSuccess) { rc = cuda_fail(ce, "rmat count"); break; }
        const uint64_t base = splitmix64_h(seed ^ splitmix64_h(uint64_t(7) + 0x632be59bd9b4e019ULL));
        rmat_keys<<<148 * 16, 256, 0, st>>>(edges, nodes, log2_nodes, base, a, a + b, a + b + c, k0);
        size_t tb_sort = 0, tb_uniq = 0;
        cub::DeviceRadixSort::SortKeys(nullptr, tb_sort, k0, k1, items, 0, 2 * log2_nodes, st);
        cub::DeviceSelect::Unique(nullptr, tb_uniq, k1, k0, nsel, items, st);
        if ((ce = cudaMalloc(&temp, tb_sort > tb_uniq ? tb_sort : tb_uniq)) != cudaSuccess) {
            rc = cuda_fail(ce, "rmat temp");
            break;
        }
        if ((ce = cub::DeviceRadixSort::SortKeys(temp, tb_sort, k0, k1, items, 0, 2 * log2_nodes, st)) !=
            cudaSuccess) { rc = cuda_fail(ce, "rmat sort"); break; }
        if ((ce = cub::DeviceSelect::Unique(temp, tb_uniq, k1, k0, nsel, items, st)) != cudaSuccess) {
            rc = cuda_fail(ce, "rmat unique");
            break;
        }
        int e_sel = 0;
        cudaMemcpyAsync(&e_sel, nsel, sizeof(int), cudaMemcpyDeviceToHost, st);
        if ((ce = cudaStreamSynchronize(st)) != cudaSuccess) { rc = cuda_fail(ce, "rmat"); break; }
        const uint64_t e = uint64_t(e_sel);
        if ((ce = cudaMalloc(&rowd, (nodes + 1) * 8)) != cudaSuccess) { rc = cuda_fail(ce, "rmat rows"); break; }
        rmat_rowptr<<<148 * 8, 256, 0, st>>>(k0, e, nodes, log2_nodes, rowd);
        if ((ce = cudaMemcpyAsync(row, rowd, (nodes + 1) * 8, cudaMemcpyDeviceToHost, st)) != cudaSuccess) {
            rc = cuda_fail(ce, "rmat rows copy");
            break;
        }
        if ((ce = cudaStreamSynchronize(st)) != cudaSuccess) { rc = cuda_fail(ce, "rmat rows"); break; }
        if (e_total) *e_total = e;
        if (col && r_hi > r_lo) {
            const uint64_t beg = row[r_lo], count = row[r_hi] - row[r_lo];
            if ((ce = cudaMalloc(&cold, count * 4 + 4)) != cudaSuccess) { rc = cuda_fail(ce, "rmat cols"); break; }
            rmat_cols<<<148 * 8, 256, 0, st>>>(k0, beg, count, nodes - 1, cold);
            if ((ce = cudaMemcpyAsync(col, cold, count * 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess) {
                rc = cuda_fail(ce, "rmat cols copy");
                break;
            }
            if ((ce = cudaStreamSynchronize(st)) != cudaSuccess) { rc = cuda_fail(ce, "rmat cols"); break; }
        }
        if ((ce = cudaGetLastError()) != cudaSuccess) { rc = cuda_fail(ce, "rmat kernels"); break; }
    } while (0);
    cleanup();
    return rc;
}
