// Graph upload, device-side CSR validation and the degree schedule.
//
// Degree schedule (replaces gat::degree_schedule, baseline/src/common.cpp:120-125):
// perm = rows sorted by (degree ascending, row id ascending). A stable LSD radix
// sort of (degree -> row id) pairs that starts from the identity order gives
// exactly that order, so the permutation is bit-identical to the reference's
// std::sort with its (degree, id) comparator. neighbor_steps is the sum over
// consecutive 16-row tiles of perm of the last row's degree (common.cpp:123).
//
// Work list for the aggregation kernels: rows are visited from the largest
// degree down (perm read backwards). A row with more than `seg_edges` edges is
// cut into segments of at most seg_edges edges, each handled by its own warp
// and merged afterwards, so no warp owns more than seg_edges edges and a
// 17k-edge hub cannot become the tail of the kernel.
#include <cub/device/device_radix_sort.cuh>

#include <vector>

#include "device.cuh"
#include "graph.cuh"

namespace gatb {

int cuda_fail(cudaError_t e, const char* what) {
    return fail_code(GAT_B200_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

namespace {

int dalloc(void** p, size_t bytes, const char* what) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 1);
    return e == cudaSuccess ? 0 : cuda_fail(e, what);
}

// Error bits of the device validation.
enum : unsigned { kBadBounds = 1, kNonMonotone = 2, kSourceRange = 4, kDegreeRange = 8 };

__global__ void validate_rows(const uint64_t* __restrict__ row, uint64_t n, uint64_t e,
                              uint32_t* __restrict__ deg, uint32_t* __restrict__ ids,
                              unsigned* __restrict__ flags) {
    uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x;
    if (i == 0 && (row[0] != 0 || row[n] != e)) atomicOr(flags, kBadBounds);
    if (i >= n) return;
    uint64_t a = row[i], b = row[i + 1];
    if (a > b) {
        atomicOr(flags, kNonMonotone);
        deg[i] = 0;
    } else {
        uint64_t d = b - a;
        if (d > 0xffffffffull) atomicOr(flags, kDegreeRange);
        deg[i] = uint32_t(d);
    }
    ids[i] = uint32_t(i);
}

__global__ void validate_cols(const uint32_t* __restrict__ col, uint64_t e, uint64_t n,
                              unsigned* __restrict__ flags) {
    uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    bool bad = false;
    for (uint64_t k = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; k < e; k += stride)
        bad |= col[k] >= n;
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(flags, kSourceRange);
}

// neighbor_steps and the hub statistics from the sorted degrees.
__global__ void schedule_stats(const uint32_t* __restrict__ sorted_deg, uint64_t n, uint32_t seg_edges,
                               unsigned long long* __restrict__ steps,
                               unsigned long long* __restrict__ n_hub,
                               unsigned long long* __restrict__ n_seg,
                               unsigned long long* __restrict__ n_wide) {
    uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    unsigned long long s = 0, h = 0, g = 0, w = 0;
    for (uint64_t t = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; t < n; t += stride) {
        uint32_t d = sorted_deg[t];
        if (t % 16 == 15 || t == n - 1) s += d;  // last row of each 16-row tile
        if (d > seg_edges) {
            ++h;
            g += (d + seg_edges - 1) / seg_edges;
        } else if (d > kWideRowEdges) {
            ++w;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, o);
        h += __shfl_xor_sync(0xffffffffu, h, o);
        g += __shfl_xor_sync(0xffffffffu, g, o);
        w += __shfl_xor_sync(0xffffffffu, w, o);
    }
    if ((threadIdx.x & 31) == 0) {
        atomicAdd(steps, s);
        atomicAdd(n_hub, h);
        atomicAdd(n_seg, g);
        atomicAdd(n_wide, w);
    }
}

// Segment table for the hub rows: the top n_hub entries of perm, largest first.
// One thread per hub row writes its segments at the exclusive prefix offset.
__global__ void build_segments(const uint64_t* __restrict__ row, const uint32_t* __restrict__ perm,
                               uint64_t n, uint32_t n_hub, uint32_t seg_edges,
                               const uint32_t* __restrict__ seg_offset,  // [n_hub+1]
                               Segment* __restrict__ segs) {
    uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= n_hub) return;
    uint32_t r = perm[n - 1 - k];
    uint64_t a = row[r], b = row[r + 1];
    uint32_t s = seg_offset[k];
    for (uint64_t x = a; x < b; x += seg_edges, ++s) {
        segs[s].row = r;
        segs[s].hub = k;
        segs[s].beg = x;
        segs[s].end = x + seg_edges < b ? x + seg_edges : b;
    }
}

}  // namespace

int graph_build(gat_b200_graph* g, const uint64_t* row_h, const uint32_t* col_h, cudaStream_t st) {
    const uint64_t n = g->n, e = g->e;
    GATB_CUDA(cudaGetDevice(&g->device));
    GATB_CUDA(cudaMalloc(&g->row, (n + 1) * sizeof(uint64_t)));
    GATB_CUDA(cudaMalloc(&g->col, (e ? e : 1) * sizeof(uint32_t)));
    GATB_CUDA(cudaMalloc(&g->perm, n * sizeof(uint32_t)));
    GATB_CUDA(cudaMemcpyAsync(g->row, row_h, (n + 1) * sizeof(uint64_t), cudaMemcpyHostToDevice, st));
    if (e) GATB_CUDA(cudaMemcpyAsync(g->col, col_h, e * sizeof(uint32_t), cudaMemcpyHostToDevice, st));

    uint32_t *deg = nullptr, *ids = nullptr, *sorted_deg = nullptr;
    unsigned* flags = nullptr;
    unsigned long long* stats = nullptr;
    void* temp = nullptr;
    size_t temp_bytes = 0;
    auto cleanup = [&] {
        cudaFree(deg);
        cudaFree(ids);
        cudaFree(sorted_deg);
        cudaFree(flags);
        cudaFree(stats);
        cudaFree(temp);
    };
    int rc = 0;
    do {
        if ((rc = dalloc((void**)&deg, n * sizeof(uint32_t), "cudaMalloc deg"))) break;
        if ((rc = dalloc((void**)&ids, n * sizeof(uint32_t), "cudaMalloc ids"))) break;
        if ((rc = dalloc((void**)&sorted_deg, n * sizeof(uint32_t), "cudaMalloc sorted"))) break;
        if ((rc = dalloc((void**)&flags, sizeof(unsigned), "cudaMalloc flags"))) break;
        if ((rc = dalloc((void**)&stats, 4 * sizeof(unsigned long long), "cudaMalloc stats"))) break;
        cudaMemsetAsync(flags, 0, sizeof(unsigned), st);
        cudaMemsetAsync(stats, 0, 4 * sizeof(unsigned long long), st);
        validate_rows<<<unsigned((n + 255) / 256), 256, 0, st>>>(g->row, n, e, deg, ids, flags);
        if (e) validate_cols<<<1184, 256, 0, st>>>(g->col, e, g->n_src ? g->n_src : n, flags);
        unsigned hflags = 0;
        cudaMemcpyAsync(&hflags, flags, sizeof(unsigned), cudaMemcpyDeviceToHost, st);
        cudaError_t ce = cudaStreamSynchronize(st);
        if (ce != cudaSuccess) { rc = cuda_fail(ce, "graph validation"); break; }
        // Same messages as the reference's Graph::validate (common.cpp:26-28).
        if (hflags & kBadBounds) { rc = fail("bad CSR bounds"); break; }
        if (hflags & kNonMonotone) { rc = fail("nonmonotone CSR"); break; }
        if (hflags & kSourceRange) { rc = fail("source index out of bounds"); break; }
        if (hflags & kDegreeRange) { rc = fail("row degree exceeds 2^32-1"); break; }

        // Segment length: about 1/8 of the edges one resident warp processes
        // (148 SMs x 24 warps), as a power of two in [128, 8192].
        {
            int sms = 148;
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, g->device);
            uint64_t per = (g->seg_basis_e ? g->seg_basis_e : e) / (uint64_t(sms) * 24 * 8);
            uint32_t seg = 128;
            while (seg < 8192 && uint64_t(seg) * 2 <= per) seg *= 2;
            g->seg_edges = seg;
        }
        // Stable radix sort over the significant key bits only.
        int end_bit = 1;
        while (end_bit < 32 && (e >> end_bit)) ++end_bit;
        cub::DeviceRadixSort::SortPairs(nullptr, temp_bytes, deg, sorted_deg, ids, g->perm, int(n), 0,
                                        end_bit, st);
        if ((rc = dalloc((void**)&temp, temp_bytes, "cudaMalloc sort temp"))) break;
        ce = cub::DeviceRadixSort::SortPairs(temp, temp_bytes, deg, sorted_deg, ids, g->perm, int(n), 0, end_bit, st);
        if (ce != cudaSuccess) { rc = cuda_fail(ce, "degree sort"); break; }
        schedule_stats<<<592, 256, 0, st>>>(sorted_deg, n, g->seg_edges, stats, stats + 1, stats + 2, stats + 3);
        unsigned long long hs[4];
        cudaMemcpyAsync(hs, stats, sizeof(hs), cudaMemcpyDeviceToHost, st);
        cudaMemcpyAsync(&g->max_degree, sorted_deg + (n - 1), sizeof(uint32_t), cudaMemcpyDeviceToHost, st);
        ce = cudaStreamSynchronize(st);
        if (ce != cudaSuccess) { rc = cuda_fail(ce, "degree schedule"); break; }
        g->neighbor_steps = hs[0];
        g->n_hub = uint32_t(hs[1]);
        g->n_seg = uint32_t(hs[2]);
        g->n_wide = uint32_t(hs[3]);
        if (g->n_hub) {
            // Segment offsets: exclusive prefix over the hub rows (host side; few rows).
            std::vector<uint32_t> hub_deg(g->n_hub), off(g->n_hub + 1);
            cudaMemcpyAsync(hub_deg.data(), sorted_deg + (n - g->n_hub), g->n_hub * sizeof(uint32_t),
                            cudaMemcpyDeviceToHost, st);
            ce = cudaStreamSynchronize(st);
            if (ce != cudaSuccess) { rc = cuda_fail(ce, "hub degrees"); break; }
            off[0] = 0;
            // Hub k is perm[n-1-k], i.e. hub_deg[n_hub-1-k].
            for (uint32_t k = 0; k < g->n_hub; ++k)
                off[k + 1] = off[k] + (hub_deg[g->n_hub - 1 - k] + g->seg_edges - 1) / g->seg_edges;
            uint32_t* off_d = nullptr;
            if ((rc = dalloc((void**)&off_d, off.size() * sizeof(uint32_t), "cudaMalloc seg offsets"))) break;
            if ((rc = dalloc((void**)&g->segs, size_t(g->n_seg) * sizeof(Segment), "cudaMalloc segments"))) { cudaFree(off_d); break; }
            if ((rc = dalloc((void**)&g->seg_state, size_t(g->n_seg) * kSegStateFloats * sizeof(float), "cudaMalloc segment state"))) { cudaFree(off_d); break; }
            cudaMemcpyAsync(off_d, off.data(), off.size() * sizeof(uint32_t), cudaMemcpyHostToDevice, st);
            build_segments<<<(g->n_hub + 127) / 128, 128, 0, st>>>(g->row, g->perm, n, g->n_hub, g->seg_edges,
                                                                   off_d, g->segs);
            g->hub_seg_offset = off_d;
            ce = cudaStreamSynchronize(st);
            if (ce != cudaSuccess) { rc = cuda_fail(ce, "segment table"); break; }
        }
    } while (0);
    cleanup();
    return rc;
}

void graph_release(gat_b200_graph* g) {
    cudaFree(g->row);
    cudaFree(g->col);
    cudaFree(g->perm);
    cudaFree(g->segs);
    cudaFree(g->hub_seg_offset);
    cudaFree(g->seg_state);
    g->seg_state = nullptr;
    g->row = nullptr;
    g->col = nullptr;
    g->perm = nullptr;
    g->segs = nullptr;
    g->hub_seg_offset = nullptr;
}

}  // namespace gatb
