/*
 * gat_oracle.h -- CPU restatement of the reference GAT forward, used ONLY as a
 * test/benchmark checker.
 *
 * TEST INFRASTRUCTURE. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load this library, and only to check
 * or time against it. The product path (libgat_b200.so) never calls it.
 *
 * Every function cites the reference file:line it restates (paths relative to
 * the huamiao123/GAT-TFS project root). Parity of this restatement with the
 * reference itself is pinned by tests/test_oracle_golden.py against vectors
 * that the reference's own code produced (tests/golden/make_golden.py).
 *
 * Layouts follow the reference: destination-row CSR (row[n+1] u64, col[e] u32),
 * row-major features x[n][in], W[in][heads*dim] (head-major columns),
 * aL/aR[heads*dim], per-row/head arrays [n][heads], per-edge arrays [e][heads].
 */
#ifndef GAT_ORACLE_H
#define GAT_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* baseline/src/common.cpp:80-83 (rne) and :84 (expand). */
uint16_t oracle_rne(float x);
float oracle_expand(uint16_t b);
void oracle_quantize(const float* in, float* out, uint64_t count);

/* baseline/src/common.cpp:120-125 (degree_schedule): rows sorted by
 * (degree ascending, row id ascending); neighbor_steps = sum over consecutive
 * 16-row tiles of the degree of the tile's last row. Returns neighbor_steps. */
uint64_t oracle_degree_schedule(uint64_t n, const uint64_t* row, uint32_t* perm);

/* baseline/src/ref_fp32.cpp:3-26 (ref_layer, "R0"): FP32 projection, scalar
 * L/R (baseline_standard.cpp:7-20 with scalar=true), explicit score/max/p/den/
 * alpha, aggregation, ELU when hidden. Empty rows: max=0, den=0, out=0.
 * Any of z/left/right/max/den/p_edge may be NULL (p_edge is [e][heads]). */
void oracle_ref_layer(uint64_t n, const uint64_t* row, const uint32_t* col,
                      int in, int heads, int dim, const float* x, const float* w,
                      const float* al, const float* ar, int hidden,
                      float* z, float* left, float* right, float* max, float* den,
                      float* p_edge, float* out);

/* baseline/tests/boundaries.cpp:15-21: independent FP64 oracle (no ELU). */
void oracle_fp64_layer(uint64_t n, const uint64_t* row, const uint32_t* col,
                       int in, int heads, int dim, const float* x, const float* w,
                       const float* al, const float* ar, float* out);

/* baseline/src/baseline_standard.cpp:98-108 (standard_layer, "B0") restated
 * for the BF16 (bf16=1) and FP32 (bf16=0) variants: convert (common.cpp:85-93),
 * projection (3-6), lr_from_z (7-20), max_prescan (44-51), standard_aggregate
 * (52-84), finish (85-97). round_z=1 additionally rounds Z to BF16 before the
 * aggregation (the B200 build stores the projected features H in BF16); it
 * leaves L/R computed from the FP32 Z, as the B200 projection epilogue does. */
void oracle_b0_layer(uint64_t n, const uint64_t* row, const uint32_t* col,
                     int in, int heads, int dim, const float* x, const float* w,
                     const float* al, const float* ar, int hidden, int bf16, int round_z,
                     float* z, float* left, float* right, float* max, float* den,
                     float* out);

/* icpp_online's exact counters (baseline/tfs_online/icpp_online.cpp:50-116,
 * 146-164, 229-233, 330-346). Rows go in batches of 16 consecutive entries of
 * the degree order (perm), per head; a batch walks neighbour blocks of `block`
 * up to its largest degree. For each row with degree above the block start:
 * one block; the block maximum of leaky(L_i + R_j) raising the running maximum
 * (strictly) is a max update; an update after the row's first block (den > 0)
 * is a rescale. A batch block with any rescale is one rescale event; each
 * neighbour step of a batch (its largest degree) is one neighbor step.
 * row_blocks / row_updates / row_rescales ([n][heads]) may be NULL;
 * totals = {blocks, max_updates, rescales, rescale_events, neighbor_steps}. */
void oracle_online_counters(uint64_t n, const uint64_t* row, const uint32_t* col, const uint32_t* perm,
                            int heads, const float* left, const float* right, int block,
                            uint64_t* row_blocks, uint64_t* row_updates, uint64_t* row_rescales,
                            uint64_t* totals);

/* baseline/src/baseline_standard.cpp:44-51 (max_prescan). */
void oracle_max_prescan(uint64_t n, const uint64_t* row, const uint32_t* col, int heads,
                        const float* left, const float* right, float* max);

/* baseline/src/baseline_standard.cpp:52-84 (standard_aggregate): writes the
 * UNNORMALIZED out[n][heads*dim] and den[n][heads]. With fixed_p (per edge,
 * [e][heads]) the weights are taken from it and den from fixed_den. */
void oracle_standard_aggregate(uint64_t n, const uint64_t* row, const uint32_t* col,
                               int heads, int dim, const float* z, const float* left,
                               const float* right, const float* max,
                               const float* fixed_p, const float* fixed_den,
                               float* out, float* den);

/* TFS ("transform from sum") aggregation family, restated per destination
 * row (the reference's 16-row batching does not change a row's arithmetic).
 * xq: BF16-valued features [n][in]; wq: BF16-valued W [in][heads*dim].
 * Every variant writes the UNNORMALIZED V[n][heads*dim], den[n][heads] and,
 * if max_out is set, the final row maximum.
 *
 *  rounding 0, max given, block 0   baseline/src/baseline_tfs.cpp:16-110
 *      (tfs_aggregate, B1): p from the prescan max, every product rounded,
 *      V += RNE(p*x) . W in neighbour order. fixed_p/fixed_den as B0.
 *  rounding 0, max NULL, block B    baseline/tfs_online/icpp_online.cpp:40-215
 *      (icpp_online): running max per block of B neighbours, V and den
 *      rescaled by exp(old-new) when it grows, products rounded as B1.
 *  rounding 1, max NULL, block B    baseline/tfs_online/icpp_block.cpp:36-210
 *      (icpp_block): U_B = sum_{j in block} p_j x_j (FP32 FMA chain),
 *      V += RNE(U_B) . W.
 *  rounding 2, max NULL, block B    baseline/tfs_online/icpp_heads_hybrid.cpp:44-290
 *      (icpp_heads_hybrid): as rounding 1 for rows with fewer than `threshold`
 *      neighbours in the block; otherwise U_B = sum p_hi x + sum p_lo x with
 *      p = p_hi + p_lo split into two BF16 values (the AMX high/low path).
 *  max given with rounding 1 or 2 uses that maximum for every block (no
 *  rescale): the B200 tensor-core kernel's semantics. block 0 = whole row.
 * All V accumulation is sequential FP32 in (neighbour, feature) order, the
 * order of AMX tdpbf16ps over the reference's K blocks. */
void oracle_tfs_aggregate(uint64_t n, const uint64_t* row, const uint32_t* col, int in, int heads, int dim,
                          const float* xq, const float* wq, const float* left, const float* right,
                          const float* max_in, const float* fixed_p, const float* fixed_den, int rounding,
                          int block, int threshold, float* out, float* den, float* max_out);

/* baseline/src/common.cpp:100-106 (prepare, attention=true): blr[k][h] =
 * sum_d W[k][h*dim+d] * aL[h*dim+d] (and aR at [k][heads+h]), one FMA chain
 * per entry (the reference is compiled with FMA contraction). */
void oracle_prepare_blr(int in, int heads, int dim, const float* w, const float* al, const float* ar,
                        float* blr);

/* baseline/src/baseline_standard.cpp:29-43 (lr_reordered): [L|R] = X . blr.
 * policy 0 "bf16": BF16 X (xq) times RNE(blr); 1 "fp32": FP32 X times blr.
 * Each dot is a sequential FMA chain over the input features. */
void oracle_lr_reordered(uint64_t n, int in, int heads, const float* x, const float* xq, const float* blr,
                         int policy, float* left, float* right);

/* baseline/src/baseline_standard.cpp:85-97 (finish): out *= 1/den (0 if den<=0),
 * then ELU (gat.hpp:53) when hidden. */
void oracle_finish(uint64_t n, int heads, int dim, const float* den, int hidden, float* out);

#ifdef __cplusplus
}
#endif
#endif
