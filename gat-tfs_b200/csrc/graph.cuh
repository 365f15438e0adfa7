// Device-resident graph, prepared layer and model objects behind the opaque
// handles of include/gat_b200.h.
#pragma once
#include <vector>
#include <cuda_runtime.h>
#include <cstdint>

#include "gat_b200_internal.h"

namespace gatb {
// One segment of a high-degree ("hub") row: edges [beg, end) of row `row`,
// which is hub number `hub` (0 = largest degree).
struct Segment {
    uint32_t row;
    uint32_t hub;
    uint64_t beg;
    uint64_t end;
};
}  // namespace gatb

struct gat_b200_graph {
    uint64_t n = 0, e = 0;
    uint64_t n_src = 0;       // source ids are < n_src (n for a square graph)
    int device = 0;
    uint64_t* row = nullptr;  // device [n+1]
    uint32_t* col = nullptr;  // device [e]
    uint32_t* perm = nullptr; // device [n], (degree, id) ascending
    uint64_t neighbor_steps = 0;
    uint32_t max_degree = 0;
    // Rows with degree > seg_edges are hubs; they are perm[n-1-k], k < n_hub,
    // cut into n_seg segments (segs, ordered by hub then edge position).
    uint32_t seg_edges = 256;
    // Edge count the segment length is derived from (0: this graph's e). The
    // slices of a partitioned graph take the whole graph's, so their hub rows
    // are cut where the one-GPU graph cuts them and the sums run in the same
    // order on any number of GPUs.
    uint64_t seg_basis_e = 0;
    uint32_t n_hub = 0, n_seg = 0;
    // Rows with more than kWideRowEdges edges that are not hubs: in the degree
    // order they follow the hubs, perm[n-1-n_hub-k] for k < n_wide.
    uint32_t n_wide = 0;
    gatb::Segment* segs = nullptr;       // device [n_seg]
    uint32_t* hub_seg_offset = nullptr;  // device [n_hub+1]
    // Device scratch for the segments' partial softmax states: kSegStateFloats
    // floats per segment (max row width 8*64 plus running max and sum per head).
    float* seg_state = nullptr;
};

struct gat_b200_layer {
    int in = 0, heads = 0, dim = 0, width = 0;
    int kp = 0;                 // in padded to 64 (tensor-core K blocks)
    int np = 0;                 // width padded to 16 (tensor-core N)
    uint16_t* wt_bf16 = nullptr; // device [np][kp] BF16 RNE(W)^T, zero padded
    float* w = nullptr;          // device [in][width] FP32 W
    float* al = nullptr;         // device [width]
    float* ar = nullptr;         // device [width]
    float* blr = nullptr;        // device [in][2*heads] = W.a (common.cpp:100-108)
    std::vector<float> al_host, ar_host;  // host copies of aL / aR [width]
};

namespace gatb {
int graph_build(gat_b200_graph* g, const uint64_t* row_h, const uint32_t* col_h, cudaStream_t st);
void graph_release(gat_b200_graph* g);
constexpr int kSegStateFloats = 8 * 64 + 2 * 8;
// Rows above this many edges get a whole warp in the narrow-layer kernel.
constexpr uint32_t kWideRowEdges = 64;
}  // namespace gatb
