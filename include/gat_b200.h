/*
 * gat_b200.h -- C-ABI of libgat_b200.so, the B200 (sm_100a) implementation of
 * the three-layer multi-head GAT forward of huamiao123/GAT-TFS.
 *
 * Plain C: opaque handles, plain pointers and sizes, int status codes. No C++
 * exceptions cross this boundary; gat_b200_last_error() returns the message of
 * the calling thread's last failure (the reference throws std::runtime_error
 * with the same kind of message, e.g. baseline/src/common.cpp:24-28).
 *
 * Each entry point names the reference interface it replaces (file:line inside
 * the reference project). Reference layouts are kept: destination-row CSR with
 * u64 row pointers and u32 source ids, row-major features, W[in][heads*dim]
 * with head-major columns, per-row/head arrays [n][heads], per-edge arrays
 * [e][heads]. Device feature buffers use a row stride `ld` (elements) that the
 * caller passes; gat_b200_padded_ld() gives the stride the library uses itself
 * (rows start on 16-byte boundaries, padding columns hold zeros).
 *
 * Streams are passed as `void*` (a cudaStream_t; NULL = legacy default stream).
 * Device-pointer arguments must be device memory of the current device.
 */
#ifndef GAT_B200_H
#define GAT_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define GAT_B200_OK 0
#define GAT_B200_EINVAL 1       /* bad argument, shape or input data */
#define GAT_B200_ECUDA 2        /* CUDA runtime / driver error */
#define GAT_B200_EUNSUPPORTED 3 /* shape outside what the kernels implement */
#define GAT_B200_ETIMEOUT 4     /* a bounded device-side wait gave up */
#define GAT_B200_EIO 5          /* file open/read/write failure */

/* ---- element types, paths ---------------------------------------------- */
#define GAT_B200_F32 0
#define GAT_B200_BF16 1

/* Layer paths, named after the reference's --path values
 * (baseline/bench/main.cpp:30, baseline/src/common.cpp:126-134). */
#define GAT_B200_PATH_STANDARD_BF16 0 /* B0: BF16 X/W on tcgen05, FP32 softmax state */
#define GAT_B200_PATH_STANDARD_FP32 1 /* B0 FP32 projection, FP32 features         */
#define GAT_B200_PATH_TFS_BF16 2      /* tfs_bf16: B1 TFS layers (baseline_tfs.cpp:111-117) */
/* No --path of that name in the reference: layer 1 through TFS aggregation
 * (tensor cores, heads_hybrid rounding with one block per row), layers 2-3 as
 * STANDARD_BF16 -- the per-layer choice of the reference's adaptive driver
 * (baseline/tfs_online/adaptive_main.cpp:86-101), where TFS wins on layer 1. */
#define GAT_B200_PATH_ADAPTIVE_BF16 3
/* matched_attention: STANDARD_BF16 with L/R from lr_reordered ("bf16" policy,
 * the TFS attention contraction) instead of from Z
 * (baseline/bench/main.cpp:22-25, baseline/src/baseline_standard.cpp:98-108). */
#define GAT_B200_PATH_MATCHED_ATTENTION 4

/* TFS rounding variants (gat_b200_tfs_aggregate). */
#define GAT_B200_TFS_EDGE 0  /* V += RNE(p x) . W per neighbour: B1, icpp_online  */
#define GAT_B200_TFS_BLOCK 1 /* V += RNE(sum_B p x) . W per block: icpp_block     */
#define GAT_B200_TFS_SPLIT 2 /* as BLOCK, sum from BF16 high/low p: heads_hybrid */

/* lr_reordered policies (baseline_standard.cpp:29-43). */
#define GAT_B200_LR_BF16 0 /* BF16 X times RNE(W a)  ("bf16") */
#define GAT_B200_LR_FP32 1 /* FP32 X times W a        ("fp32") */

/* Message of this thread's last failure ("" if none). */
const char* gat_b200_last_error(void);
/* Library version: major*10000 + minor*100 + patch. */
int gat_b200_version(void);
/* Row stride (elements) the library uses for `width` columns of elem_dtype. */
int gat_b200_padded_ld(int width, int elem_dtype);

/* ======================================================================== *
 *  Host utilities (no GPU needed)                                          *
 * ======================================================================== */

/* FP32 -> BF16 round-to-nearest-even, NaN quieted.
 * Replaces gat::rne (baseline/src/common.cpp:80-83). */
uint16_t gat_b200_rne(float x);
/* Replaces gat::convert (baseline/src/common.cpp:85-93), host side. */
int gat_b200_convert_host(const float* in, uint16_t* out, uint64_t count);

/* Replaces gat::Graph::validate (baseline/src/common.cpp:23-30) for the CSR
 * part: row[0]==0, row[n]==e, monotone rows, col < n, 0 < n <= INT32_MAX. */
int gat_b200_validate_csr(uint64_t n, uint64_t e, const uint64_t* row, const uint32_t* col);

/* GATBIN1 graph files. Replaces gat::load_graph / save_graph
 * (baseline/src/common.cpp:31-44). Read the header first, then the arrays into
 * caller buffers of row[n+1], col[e], x[n*din]. */
int gat_b200_read_graph_header(const char* path, uint64_t* n, uint64_t* e, uint32_t* din,
                               uint32_t* classes);
int gat_b200_read_graph(const char* path, uint64_t n, uint64_t e, uint32_t din, uint64_t* row,
                        uint32_t* col, float* x);
int gat_b200_write_graph(const char* path, uint64_t n, uint64_t e, uint32_t din, uint32_t classes,
                         const uint64_t* row, const uint32_t* col, const float* x);

/* GATWGT1 checkpoints for the 3-layer model din -> 8x32 -> 8x32 -> 1xclasses.
 * Replaces gat::load_model / save_model (baseline/src/common.cpp:63-79).
 * w[l], al[l], ar[l] are caller buffers of in_l*width_l, width_l, width_l. */
int gat_b200_read_weights(const char* path, int din, int classes, float* const* w,
                          float* const* al, float* const* ar);
int gat_b200_write_weights(const char* path, int din, int classes, const float* const* w,
                           const float* const* al, const float* const* ar);

/* Seeded untrained model with the reference's generator: mt19937(seed+11*l),
 * W ~ N(0,1)/sqrt(in), a ~ N(0,1)/sqrt(dim). Replaces gat::random_model
 * (baseline/src/common.cpp:50-62); bit-identical with the same C++ library. */
int gat_b200_random_model(int din, int classes, int seed, float* const* w, float* const* al,
                          float* const* ar);

/* Seeded synthetic inputs (no reference counterpart: the reference reads
 * prepared OGB files, implementation/tools/prepare_arxiv.py:28-52).
 *  - uniform: every row has `sources` distinct uniform sources != self, plus
 *    the self loop; e = n*(sources+1).
 *  - powerlaw: row degrees follow a power law of exponent gamma with the given
 *    maximum and exactly e edges (self loops included); sources are drawn by
 *    the same popularity law.
 *  - normal / uniform: count floats ~ N(0,scale^2) / U(lo,hi) from (seed,stream). */
int gat_b200_synth_uniform_graph(uint64_t n, uint32_t sources, uint64_t seed, uint64_t* row,
                                 uint32_t* col);
int gat_b200_synth_powerlaw_graph(uint64_t n, uint64_t e, uint64_t max_degree, double gamma,
                                  uint64_t seed, uint64_t* row, uint32_t* col);
int gat_b200_synth_normal(uint64_t count, double scale, uint64_t seed, uint64_t stream, float* out);
/* Rank-local pieces of the same inputs, for multi-GPU runs where no process
 * builds the whole graph: elements [offset, offset+count) of synth_normal, and
 * all n+1 row pointers of synth_powerlaw_graph with the sources of rows
 * [r_lo, r_hi) only (col holds row[r_hi]-row[r_lo] entries; NULL = row
 * pointers only). Identical values to the whole-graph calls. */
int gat_b200_synth_normal_range(uint64_t offset, uint64_t count, double scale, uint64_t seed,
                                uint64_t stream, float* out);
int gat_b200_synth_powerlaw_rows(uint64_t n, uint64_t e, uint64_t max_degree, double gamma,
                                 uint64_t seed, uint64_t r_lo, uint64_t r_hi, uint64_t* row,
                                 uint32_t* col);
int gat_b200_synth_uniform(uint64_t count, double lo, double hi, uint64_t seed, uint64_t stream,
                           float* out);
/* RMAT stress graph (configuration c5), generated on the current CUDA device:
 * 2^log2_nodes nodes, `edges` draws with quadrant probabilities (a, b, c,
 * 1-a-b-c) per level (source bit first), one self loop per node, duplicate
 * (destination, source) pairs kept once, destination-row CSR with sources
 * ascending. Writes all 2^log2_nodes + 1 row pointers to row (host) and the
 * sources of rows [r_lo, r_hi) to col (host, may be NULL), and the edge count
 * to *e_total (may be NULL). Identical on every device (counter-based draws).
 * edges + 2^log2_nodes < 2^31. */
int gat_b200_synth_rmat(int log2_nodes, uint64_t edges, double a, double b, double c, uint64_t seed,
                        uint64_t r_lo, uint64_t r_hi, uint64_t* row, uint32_t* col, uint64_t* e_total);

/* GATFIX1 fixed-p fixture of one layer: the graph's CSR, the layer's W/aL/aR,
 * its input [n][in] and the attention weights p [e][heads] with their sums
 * den [n][heads]. Replaces gat::save_fixture / gat::load_fixture
 * (baseline/src/common.cpp:171-194); read_fixture rejects a file whose shape,
 * CSR or checkpoint differ from the given ones, non-finite values, p outside
 * [0,1] and den that is not the sum of its row's p (the reference's checks and
 * messages). */
int gat_b200_write_fixture(const char* path, uint64_t n, uint64_t e, int in, int heads, int dim,
                           const uint64_t* row, const uint32_t* col, const float* w, const float* al,
                           const float* ar, const float* input, const float* p, const float* den);
int gat_b200_read_fixture(const char* path, uint64_t n, uint64_t e, int in, int heads, int dim,
                          const uint64_t* row, const uint32_t* col, const float* w, const float* al,
                          const float* ar, float* input, float* p, float* den);

/* ======================================================================== *
 *  Device: graph and degree schedule                                       *
 * ======================================================================== */

typedef struct gat_b200_graph gat_b200_graph;

/* Uploads a destination-row CSR (host arrays) to the current device, checks it
 * on the device (the CSR checks of Graph::validate, baseline/src/common.cpp:24-28)
 * and builds the degree schedule (replaces gat::degree_schedule,
 * baseline/src/common.cpp:120-125): the stable (degree, row id) ascending
 * permutation and neighbor_steps, computed on the device by a stable radix sort.
 * The kernels walk that permutation from the largest degree down and give rows
 * above a degree threshold a whole CTA. */
int gat_b200_graph_create(uint64_t n, uint64_t e, const uint64_t* row, const uint32_t* col,
                          void* stream, gat_b200_graph** out);
/* A slice of a partitioned graph: n destination rows whose source ids index a
 * feature table of n_src rows (the all-gathered projected features of every
 * rank in the multi-GPU forward). No reference counterpart (the reference runs
 * on one CPU); validation and schedule as gat_b200_graph_create, with the
 * source bound n_src instead of n. */
int gat_b200_graph_create_part(uint64_t n, uint64_t n_src, uint64_t e, const uint64_t* row,
                               const uint32_t* col, void* stream, gat_b200_graph** out);
int gat_b200_graph_destroy(gat_b200_graph* g);
/* Copies the schedule back: perm[n] (may be NULL) and neighbor_steps (may be NULL). */
int gat_b200_graph_schedule(const gat_b200_graph* g, uint32_t* perm, uint64_t* neighbor_steps);
/* Device pointers of the uploaded CSR (row[n+1] u64, col[e] u32). */
int gat_b200_graph_device_csr(const gat_b200_graph* g, const uint64_t** row, const uint32_t** col);
/* Schedule statistics: rows, edges, largest degree, number of rows split into
 * segments of at most seg_edges edges (n_hub), and those segments (n_seg). */
int gat_b200_graph_info(const gat_b200_graph* g, uint64_t* n, uint64_t* e, uint32_t* max_degree,
                        uint32_t* n_hub, uint32_t* n_seg, uint32_t* seg_edges);

/* ======================================================================== *
 *  Device: prepared layer parameters                                       *
 * ======================================================================== */

typedef struct gat_b200_layer gat_b200_layer;

/* Replaces gat::prepare (baseline/src/common.cpp:97-119) and Param::validate
 * (common.cpp:45-49): heads in [1,8], dim in [1,64]. Uploads BF16 RNE(W) in the
 * tensor-core layout, FP32 W, aL, aR and blr = W.a ([in][2*heads],
 * common.cpp:100-108). Host input arrays. */
int gat_b200_layer_create(int in, int heads, int dim, const float* w, const float* al,
                          const float* ar, gat_b200_layer** out);
int gat_b200_layer_destroy(gat_b200_layer* p);

/* ======================================================================== *
 *  Device: stage kernels (device pointers, caller-owned buffers)           *
 * ======================================================================== */

/* FP32 [n][width] (row stride ld_in) -> BF16 RNE [n][ld_out], padding zeroed.
 * Replaces gat::convert (baseline/src/common.cpp:85-93). */
int gat_b200_convert(uint64_t n, int width, const float* in, int ld_in, uint16_t* out, int ld_out,
                     void* stream);

/* Projection with fused attention dots. Replaces gat::projection followed by
 * gat::lr_from_z (baseline/src/baseline_standard.cpp:3-20):
 *   Z = X W (FP32 accumulate), left[i][h] = Z_ih . aL_h, right[i][h] = Z_ih . aR_h.
 * precision BF16: x must be BF16 [n][ldx] and the product runs on tcgen05
 *   tensor cores (BF16 RNE(W)); FP32: x FP32 [n][ldx], FP32 CUDA-core GEMM.
 * Outputs (each may be NULL): h = Z in h_dtype [n][ldh] (BF16 RNE or FP32),
 * left/right FP32 [n][heads]. */
int gat_b200_projection(const gat_b200_layer* p, uint64_t n, const void* x, int ldx, int precision,
                        void* h, int h_dtype, int ldh, float* left, float* right, void* stream);

/* m[i][h] = leaky(L_ih + max_{j in N(i)} R_jh), 0 for empty rows.
 * Replaces gat::max_prescan (baseline/src/baseline_standard.cpp:44-51). */
int gat_b200_max_prescan(const gat_b200_graph* g, int heads, const float* left, const float* right,
                         float* max, void* stream);

/* Edge softmax + weighted aggregation writing the UNNORMALIZED out[n][heads*dim]
 * (FP32, stride ldo) and den[n][heads] (and max[n][heads] if not NULL).
 * Replaces gat::standard_aggregate (baseline/src/baseline_standard.cpp:52-84).
 * With fixed_p ([e][heads]) the weights come from it and den from fixed_den,
 * as the reference's fixed-p mode (baseline/bench/main.cpp:132). */
int gat_b200_standard_aggregate(const gat_b200_graph* g, int heads, int dim, const void* h,
                                int h_dtype, int ldh, const float* left, const float* right,
                                const float* fixed_p, const float* fixed_den, float* out, int ldo,
                                float* den, float* max, void* stream);

/* R0's edge softmax trace (baseline/src/ref_fp32.cpp:7-14): per row i and
 * head h, score[e][h] = leaky(L_ih + R_jh) over the row's edges, the row
 * maximum m (max[i][h], 0 for an empty row), p[e][h] = exp(score - m),
 * den[i][h] = the sum of the row's p in edge order, alpha[e][h] = p / den.
 * One thread per (row, head), so that the FP32 sums run in the reference's
 * order; exp is the device's expf (within 2 ulp of the host's). The weights of
 * the reference's fixed-p fixtures (GATFIX1) are p and den. score, max and
 * alpha may be NULL; left [n][heads], right [sources][heads] (device). */
int gat_b200_edge_softmax(const gat_b200_graph* g, int heads, const float* left, const float* right,
                          float* score, float* max, float* p, float* den, float* alpha, void* stream);

/* out *= (den>0 ? 1/den : 0), then ELU if hidden. Replaces gat::finish
 * (baseline/src/baseline_standard.cpp:85-97). FP32 out [n][ldo]. */
int gat_b200_finish(uint64_t n, int heads, int dim, const float* den, int hidden, float* out,
                    int ldo, void* stream);

/* The fused hot kernel: edge softmax with an online (running max/sum) update,
 * weighted aggregation, normalisation, ELU when hidden, and the store in
 * out_dtype (BF16 RNE = the next layer's input, which equals the reference's
 * convert() of its FP32 output). Replaces the sequence max_prescan +
 * standard_aggregate + finish (+ convert of the next layer) of gat::standard_layer
 * (baseline/src/baseline_standard.cpp:98-108). */
int gat_b200_aggregate_fused(const gat_b200_graph* g, int heads, int dim, const void* h,
                             int h_dtype, int ldh, const float* left, const float* right,
                             int hidden, void* out, int out_dtype, int ldo, void* stream);

/* No counterpart in the reference. The fused aggregation above for callers
 * that cannot allocate device memory themselves: a plugin inside another
 * framework whose allocator owns the GPU's memory, or a serving loop where
 * cudaMalloc would synchronize the device and stall other streams. It takes
 * the destination-row CSR as device pointers (no gat_b200_graph handle, no
 * degree schedule: rows are split into equal edge ranges instead) and keeps
 * its scratch in a 32 MiB array compiled into the library, which every GPU
 * that loads the library's module keeps until the process exits. Limits:
 * at most 7936 * 65536 = 520,093,696 edges (larger graphs get
 * GAT_B200_EUNSUPPORTED), heads <= 8, dim <= 64. Every call looks up the
 * array's device address in the current device's context
 * (cudaGetSymbolAddress); the first call on a device also loads the module
 * there, so make that first call before any stream capture. All calls share the
 * array: calls whose kernels can overlap on the GPU (other streams, other host
 * threads) race on it and must be serialized by the caller. The CSR is read as
 * given: it must be a valid destination-row CSR (row[0] = 0, row[n] = e,
 * non-decreasing, every source id < n), which gat_b200_validate_csr checks on a
 * host copy; gat_b200_graph_create validates on the device. Arguments and
 * output as in gat_b200_aggregate_fused; out_dtype must be GAT_B200_BF16 or
 * GAT_B200_F32, and padding columns [heads*dim, ldo) are written as zeros. */
int gat_b200_aggregate_fused_noalloc(uint64_t n, uint64_t e, const uint64_t* row,
                                     const uint32_t* col, int heads, int dim, const void* h,
                                     int h_dtype, int ldh, const float* left, const float* right,
                                     int hidden, void* out, int out_dtype, int ldo, void* stream);

/* One full layer on device buffers. Replaces gat::standard_layer
 * (baseline/src/baseline_standard.cpp:98-108) for path STANDARD_BF16 (x BF16)
 * or STANDARD_FP32 (x FP32). Scratch: h [n][ldh] (BF16 for STANDARD_BF16, FP32
 * otherwise, ldh = gat_b200_padded_ld(heads*dim, that dtype)), left/right
 * [n][heads]. Output as in gat_b200_aggregate_fused. */
int gat_b200_standard_layer(const gat_b200_graph* g, const gat_b200_layer* p, const void* x,
                            int ldx, int path, int hidden, void* h, float* left, float* right,
                            void* out, int out_dtype, int ldo, void* stream);

/* ---- TFS path (aggregate the layer input first, then project) ---------- */

/* [L|R] = X . blr with blr[k][h] = sum_d W[k][h*dim+d] aL[h*dim+d] (and aR),
 * computed once at layer_create (prepare, baseline/src/common.cpp:100-106).
 * Replaces gat::lr_reordered (baseline/src/baseline_standard.cpp:29-43) for
 * policy GAT_B200_LR_BF16 ("bf16") or GAT_B200_LR_FP32 ("fp32"); x is FP32 or
 * BF16 [n][ldx]. If x_bf16 is not NULL the BF16 RNE copy of x (the TFS
 * gather table, convert() of common.cpp:85-93) is written there with row
 * stride ld_bf16 (padding columns zeroed). left/right: FP32 [n][heads]. */
int gat_b200_lr_reordered(const gat_b200_layer* p, uint64_t n, const void* x, int x_dtype, int ldx,
                          int policy, void* x_bf16, int ld_bf16, float* left, float* right,
                          void* stream);

/* TFS aggregation writing the UNNORMALIZED out[n][heads*dim] (FP32, stride
 * ldo) and den[n][heads] (and the final row maximum into max_out if not NULL).
 * x: BF16 layer input [n][ldx] (the gathered table). Replaces
 *   rounding EDGE,  max given, block 0: gat::tfs_aggregate (B1,
 *       baseline/src/baseline_tfs.cpp:16-110; fixed_p/fixed_den as its
 *       fixed-p mode, baseline/bench/main.cpp:133);
 *   rounding EDGE,  max NULL, block B: gat::icpp_online::aggregate
 *       (baseline/tfs_online/icpp_online.hpp:37-39, running max per block);
 *   rounding BLOCK, max NULL, block B: gat::icpp_block::aggregate
 *       (baseline/tfs_online/icpp_block.hpp:33-35);
 *   rounding SPLIT, max NULL, block B, threshold T:
 *       gat::icpp_heads_hybrid::aggregate (icpp_heads_hybrid.hpp:18-20).
 * With max given the prescan maximum is used for every block (the online
 * variants end at that same maximum; only their rescale roundings differ).
 * block 0 = one block per row, except that with BLOCK/SPLIT rounding a row
 * longer than the graph's segment length (seg_edges of gat_b200_graph_info)
 * takes one block per segment. SPLIT with block 0, threshold 1 and max given
 * runs on the tcgen05 kernel when the layer fits it (in <= 120,
 * heads*dim <= 256); everything else on the CUDA-core kernel. */
int gat_b200_tfs_aggregate(const gat_b200_graph* g, const gat_b200_layer* p, const void* x, int ldx,
                           const float* left, const float* right, const float* max,
                           const float* fixed_p, const float* fixed_den, int rounding, int block,
                           int threshold, float* out, int ldo, float* den, float* max_out,
                           void* stream);

/* One TFS layer: lr_reordered (writing the BF16 copy of x into x_bf16, stride
 * gat_b200_padded_ld(in, BF16)), max_prescan, TFS aggregation, finish (and
 * ELU when hidden), output in out_dtype with stride ldo. Replaces
 * gat::tfs_layer (baseline/src/baseline_tfs.cpp:111-117; rounding EDGE,
 * block 0) and the layer() functions of icpp_online / icpp_block /
 * icpp_heads_hybrid (other rounding/block/threshold). Scratch: x_bf16,
 * left/right/max/den [n][heads]. */
int gat_b200_tfs_layer(const gat_b200_graph* g, const gat_b200_layer* p, const void* x, int x_dtype,
                       int ldx, int hidden, int policy, int rounding, int block, int threshold,
                       void* x_bf16, float* left, float* right, float* max, float* den, void* out,
                       int out_dtype, int ldo, void* stream);

/* Device memory for callers that hold no CUDA runtime of their own (the C++
 * mirror of the reference API, include/gat_b200.hpp): a zero-filled
 * allocation on the current device, its release, and synchronous copies
 * between host and device memory. */
int gat_b200_device_alloc(uint64_t bytes, void** ptr);
/* Device selection for the same callers (one process or thread per GPU):
 * the number of visible devices, and the device the calling thread's later
 * calls use (cudaSetDevice). */
int gat_b200_device_count(int* count);
int gat_b200_set_device(int device);
int gat_b200_device_free(void* ptr);
int gat_b200_copy_to_device(void* dst, const void* src, uint64_t bytes);
int gat_b200_copy_to_host(void* dst, const void* src, uint64_t bytes);

/* icpp_online's exact counters (baseline/tfs_online/icpp_online.hpp:18-22) for
 * the online TFS variant with neighbour blocks of `block`, from the layer's
 * left/right ([n][heads], device): per (row, head) the blocks taken, the max
 * updates and the rescales (row_* device [n][heads] uint64, each may be NULL),
 * and totals (host, 5 values) = {blocks, max_updates, rescales,
 * rescale_events, neighbor_steps}, rows batched 16 at a time in the degree
 * order as the reference does. The reference's other counters follow:
 * amx_calls = neighbor_steps * padded_in/32 * ceil(dim/16), executed_fma =
 * neighbor_steps * 16 * padded_in * ceil(dim/16) * 16, rescaled feature
 * elements = rescales * dim, spill/reload bytes = rescale_events *
 * ceil(dim/16) * 1024. Synchronizes with `stream`. */
int gat_b200_tfs_online_counters(const gat_b200_graph* g, int heads, const float* left, const float* right,
                                 int block, uint64_t* row_blocks, uint64_t* row_updates, uint64_t* row_rescales,
                                 uint64_t* totals, void* stream);

/* Reports (and clears) a device-side failure recorded by an earlier kernel:
 * GAT_B200_ETIMEOUT if a bounded wait inside a kernel gave up. Synchronizes
 * with the device. */
int gat_b200_check_device(void);

/* ======================================================================== *
 *  Device: three-layer model (the benchmarked forward)                     *
 * ======================================================================== */

typedef struct gat_b200_model gat_b200_model;

/* Binds a graph and the three prepared layers, allocating every device buffer
 * the forward needs up front (the reference allocates all workspaces before
 * timing, baseline/bench/main.cpp:156). The layers must chain:
 * in(l+1) == heads(l)*dim(l). */
int gat_b200_model_create(const gat_b200_graph* g, const gat_b200_layer* const* layers, int path,
                          gat_b200_model** out);
int gat_b200_model_destroy(gat_b200_model* m);
/* Three-layer forward: layers 1-2 hidden (ELU), layer 3 logits, as the
 * reference's model loop (baseline/bench/main.cpp:171-172). x: FP32 [n][din]
 * (dense rows) in host memory (x_on_host=1) or device memory; logits: FP32
 * [n][classes] (dense rows) in host or device memory. Host buffers should be
 * pinned for asynchronous copies. Work is enqueued on `stream`; when logits
 * are in host memory the call returns after the copy completed. */
int gat_b200_model_forward(gat_b200_model* m, const float* x, int x_on_host, float* logits,
                           int logits_on_host, void* stream);
/* Per-stage timing, the device counterpart of the reference's Times and its
 * per-layer JSON fields (baseline/include/gat.hpp:68-76, common.cpp:155-170).
 * enable_timing(m, k) records CUDA events around every stage of the next
 * forwards into a ring of k sets (0 disables). stage_times waits for them and
 * writes ms[set*9 + stage] for stages {h2d, convert, projection L1, aggregation
 * L1, projection L2, aggregation L2, projection L3, aggregation L3, d2h};
 * returns the number of sets written (or a negative status on error). */
int gat_b200_model_enable_timing(gat_b200_model* m, int steps);
int gat_b200_model_stage_times(gat_b200_model* m, float* ms);
/* Number of kernels the last forward launched. */
int gat_b200_model_launches(const gat_b200_model* m);

/* No counterpart in the reference (its forward runs on host memory in place).
 * A stream of host-to-host forwards, for a serving loop: uploads x (pinned
 * FP32 [n][din]), runs the forward on `stream` and downloads the logits into
 * `logits` (pinned FP32 [n][classes]), returning at once. Two device slots and
 * the model's own upload / download streams let request k's download and
 * request k+1's upload overlap compute. The host buffers of a call must stay
 * untouched until a later gat_b200_model_join has been waited on.
 * gat_b200_model_join makes `stream` wait (on the device, without blocking the
 * host) until every submitted forward has finished its download. */
int gat_b200_model_forward_async(gat_b200_model* m, const float* x, float* logits, void* stream);
int gat_b200_model_join(gat_b200_model* m, void* stream);

/* ======================================================================== *
 *  Multi-GPU exchange (one process per GPU on one NVLink/NVSwitch node)    *
 * ======================================================================== *
 * No counterpart in the reference, whose forward runs in one CPU process
 * (baseline/bench/main.cpp:171-172). With destination rows partitioned over
 * ranks, every layer's projected features H and right scores R of a rank's
 * rows must reach every rank's feature table before that layer's aggregation.
 * These calls do it without a separate collective: the projection kernel
 * stores its output tiles into the other ranks' tables over NVLink. */

#define GAT_B200_PEER_HANDLE_BYTES 64

/* Device allocation (zero-filled) that other processes of the node can map:
 * *ptr receives the local pointer, handle (GAT_B200_PEER_HANDLE_BYTES bytes)
 * the token to pass to gat_b200_peer_open in the other processes. */
int gat_b200_peer_alloc(uint64_t bytes, void** ptr, void* handle);
/* Maps another process's gat_b200_peer_alloc allocation into this one. */
int gat_b200_peer_open(const void* handle, void** ptr);
/* Unmaps what gat_b200_peer_open mapped / frees what gat_b200_peer_alloc
 * allocated. NULL is a no-op. */
int gat_b200_peer_close(void* ptr);
int gat_b200_peer_free(void* ptr);

/* gat_b200_projection (precision BF16, BF16 H on the tensor-core kernel) that
 * also stores every H row into h_peer[i] and every R row into r_peer[i],
 * i < npeer (<= 7): the other ranks' tables, mapped with gat_b200_peer_open,
 * each pointer already offset to this call's first row. h/h_peer rows have
 * stride ldh; right/r_peer rows hold `heads` floats. Pointers 16-byte aligned. */
int gat_b200_projection_scatter(const gat_b200_layer* p, uint64_t n, const void* x, int ldx, void* h,
                                int ldh, float* left, float* right, int npeer, void* const* h_peer,
                                float* const* r_peer, void* stream);

/* Copy-engine push of one block to up to 7 peers: dst[j] <- src (`bytes`
 * bytes) as one cudaMemcpyAsync on streams[j] each, so the copies use no SMs
 * and run beside kernels on other streams. */
int gat_b200_copy_to_peers(const void* src, void* const* dst, int ndst, uint64_t bytes, void* const* streams);

/* Cross-GPU barrier on `stream`: flags[j] is rank j's flag array (a
 * gat_b200_peer_alloc allocation of at least world*4 bytes, mapped in this
 * process; flags[rank] the own one). Every rank calls it with the same epoch,
 * which must grow by at least one per call. Stores enqueued on `stream` before
 * the barrier, to local or peer memory, are visible to work enqueued after it
 * on every rank. A peer that does not arrive within about a second makes the
 * next gat_b200_check_device return GAT_B200_ETIMEOUT. world <= 8. */
int gat_b200_peer_barrier(void* const* flags, int world, int rank, uint32_t epoch, void* stream);

/* ======================================================================== *
 *  Multi-GPU forward behind the C ABI                                      *
 * ======================================================================== *
 * No counterpart in the reference (one CPU process). One process per GPU of
 * one NVLink/NVSwitch node runs the reference's model loop
 * (baseline/bench/main.cpp:171-172) on its share of destination rows; the
 * calls below are everything such a process needs, with no framework around
 * it. */

/* ---- communicator ------------------------------------------------------ */
typedef struct gat_b200_comm gat_b200_comm;
#define GAT_B200_COMM_ID_BYTES 128

/* A fresh NCCL unique id (rank 0), to hand to the other ranks out of band. */
int gat_b200_comm_id(void* id);
/* Joins the node's communicator as `rank` of `world` (<= 8) on the current
 * device; every rank passes rank 0's id. Blocks until all ranks joined. NCCL
 * (libnccl.so.2) is loaded at run time; NCCL_NVLS_ENABLE defaults to 0. */
int gat_b200_comm_create(const void* id, int world, int rank, gat_b200_comm** out);
/* The same, with the id passed through a file: rank 0 writes a fresh id to
 * `path` (atomically, by rename), the other ranks wait up to timeout_ms for it
 * (GAT_B200_ETIMEOUT after that). Use a path no earlier run has written. */
int gat_b200_comm_create_file(const char* path, int world, int rank, int timeout_ms, gat_b200_comm** out);
int gat_b200_comm_info(const gat_b200_comm* c, int* world, int* rank);
/* Host-memory all-gather of `bytes` per rank into recv[world * bytes]
 * (rank order), and a host barrier. Both block until done. */
int gat_b200_comm_all_gather(gat_b200_comm* c, const void* send, void* recv, uint64_t bytes);
int gat_b200_comm_barrier(gat_b200_comm* c);
int gat_b200_comm_destroy(gat_b200_comm* c);

/* ---- row partition (host) ---------------------------------------------- */
/* The layout of the partitioned forward for a destination-row CSR of n rows
 * (row pointers only): rank k owns rows [cuts[k], cuts[k+1]), cuts[k] the
 * first row whose CSR offset reaches k*e/world; each rank's rows are cut again
 * into `chunks` row chunks balanced by edges (chunk_cuts[k*(chunks+1) + c],
 * global rows). Every layer's feature table holds chunks*world blocks of
 * *block_rows rows (the largest chunk, rounded up to 4): chunk c of rank k at
 * table row (c*world + k) * block_rows; *table_rows = chunks*world*block_rows.
 * Any output may be NULL. */
int gat_b200_partition(uint64_t n, const uint64_t* row, int world, int chunks, uint64_t* cuts,
                       uint64_t* chunk_cuts, uint64_t* block_rows, uint64_t* table_rows);
/* Table rows of `count` global source ids under that layout. */
int gat_b200_partition_slots(uint64_t n, const uint64_t* row, int world, int chunks, uint64_t count,
                             const uint32_t* src, uint32_t* slots);

/* ---- partitioned three-layer model ------------------------------------- */
typedef struct gat_b200_part_model gat_b200_part_model;
/* Exchange of each layer's projected features between the ranks:
 *  P2P  (default): peer memory over NVLink (CUDA IPC). Layer 1's BF16 input
 *        rows are stored into every rank's input table by the conversion
 *        kernel itself and every rank projects the whole table; layer 2's
 *        input rows likewise by the layer-1 aggregation's epilogue (see
 *        gat_b200_part_model_set_layer2_exchange); for layer 3 the
 *        projection kernel stores each H/R tile into every rank's table; a
 *        bounded cross-GPU flag barrier closes each exchange.
 *  NCCL: each rank projects its own rows and NCCL all-gathers H and R. */
#define GAT_B200_EXCHANGE_P2P 0
#define GAT_B200_EXCHANGE_NCCL 1

/* Collective: every rank calls it with the same n, row (all n+1 row
 * pointers), chunks, exchange and layer shapes. col_rows holds the sources of
 * this rank's rows (col[row[cuts[rank]] .. row[cuts[rank+1]]) of the whole
 * CSR; gat_b200_part_model_rows gives that range). Source ids are remapped to
 * table rows once, and each chunk's slice is validated and scheduled as
 * gat_b200_graph_create does. Layers as gat_b200_model_create. */
int gat_b200_part_model_create(gat_b200_comm* comm, uint64_t n, const uint64_t* row, const uint32_t* col_rows,
                               const gat_b200_layer* const* layers, int exchange, int chunks, void* stream,
                               gat_b200_part_model** out);
/* This rank's destination rows [*lo, *hi) and its edge count. */
int gat_b200_part_model_rows(const gat_b200_part_model* m, uint64_t* lo, uint64_t* hi, uint64_t* edges);
/* The forward of this rank's rows: x FP32 [hi-lo][din] (host or device),
 * logits FP32 [hi-lo][classes] (host or device). Every rank calls it the same
 * number of times (the exchange pairs the ranks' calls). With host logits the
 * call returns after the copy. */
int gat_b200_part_model_forward(gat_b200_part_model* m, const float* x, int x_on_host, float* logits,
                                int logits_on_host, void* stream);
/* Pipelined host-to-host requests, as gat_b200_model_forward_async / join. */
int gat_b200_part_model_forward_async(gat_b200_part_model* m, const float* x, float* logits, void* stream);
int gat_b200_part_model_join(gat_b200_part_model* m, void* stream);
/* Per-stage CUDA-event times of the last forward (enable first):
 * ms[0..11] = {h2d, input exchange, barrier 1, projection L1, aggregation L1,
 * projection+exchange L2, barrier 2, aggregation L2, projection+exchange L3,
 * barrier 3, aggregation L3, d2h}. With chunks > 1 a layer's aggregation time
 * also holds the projections of its earlier chunks. */
#define GAT_B200_PART_STAGES 12
int gat_b200_part_model_enable_timing(gat_b200_part_model* m, int on);
int gat_b200_part_model_stage_times(gat_b200_part_model* m, float* ms);
int gat_b200_part_model_launches(const gat_b200_part_model* m);
/* Overlap of the layer-2/3 exchange with the aggregation (P2P exchange,
 * chunks > 1): chunk c's projection, which stores into the peers' tables,
 * runs on its own stream on `reserved_sms` SMs while chunk c+1 aggregates on
 * the others (one aggregation block per SM). Default 16 when chunks > 1;
 * 0 runs projection and aggregation one after the other. */
int gat_b200_part_model_set_overlap(gat_b200_part_model* m, int reserved_sms);
/* How layer 2's features reach the ranks under the P2P exchange. 1 (the
 * default with more than one rank): the layer-1 aggregation stores every
 * output row (layer 2's BF16 input) into every rank's layer-2 input table as
 * it writes it, so the exchange runs inside the aggregation; after the
 * barrier every rank projects the whole table (stage 5 of
 * gat_b200_part_model_stage_times is that projection, stage 6 the barrier
 * before it). 0: each rank projects its own rows and the projection stores
 * H and R into every rank's table, as for layer 3. */
int gat_b200_part_model_set_layer2_exchange(gat_b200_part_model* m, int inputs);
/* Collective: frees the model after a host barrier (peers may still be
 * storing into this rank's tables until every rank finished its forward). */
int gat_b200_part_model_destroy(gat_b200_part_model* m);

#ifdef __cplusplus
}
#endif
#endif
