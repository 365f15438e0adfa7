// C++ mirror of the reference's online TFS experiments
// (baseline/tfs_online/icpp_online.hpp, icpp_block.hpp, icpp_heads.hpp,
// icpp_heads_hybrid.hpp) over the C ABI of libgat_b200.so, on top of the
// gat.hpp mirror (gat_b200.hpp). A caller of those headers switches with
//
//   #include "gat_b200_online.hpp"
//   namespace gat = gat_b200;
//
// and keeps gat::icpp_online, gat::icpp_block and gat::icpp_heads_hybrid.
// Header-only; link with -lgat_b200.
#pragma once
#include <algorithm>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "gat_b200.hpp"

namespace gat_b200 {

// ---- Online TFS variants (baseline/tfs_online/icpp_*.hpp) --------------------
// The entry points, workspaces and statistics of the reference's online TFS
// experiments, on gat_b200_tfs_aggregate with the running row maximum:
//   icpp_online        rounding EDGE,  neighbour blocks of `block`
//   icpp_block         rounding BLOCK, neighbour blocks of `block`
//   icpp_heads_hybrid  rounding SPLIT (high/low p for blocks of at least
//                      `threshold` neighbours) for heads 8, dim 32, in <= 256;
//                      other shapes run icpp_block, as the reference falls back.
// `panel` and `profile_period` partition and sample the reference's CPU
// workers: they are validated as there and change nothing on the device, where
// one grid covers every row. The per-worker scratch of the reference (ubuf,
// bbuf, vbuf) has no device counterpart and stays empty. Timing holds host
// times of stages that each end in a device synchronization; the BF16 copy of
// the input is written by the lr_reordered call, so convert is 0.
// With counters=true the exact counts are filled: the Online units (blocks, max
// updates, rescales, rescale events and the per-row arrays) from
// gat_b200_tfs_online_counters, and the counts of the reference's fixed CPU
// schedule (neighbour steps, AMX calls and FMAs, conversions, spills, and
// heads_hybrid's PH work by its AVX/AMX split per block) from the CSR and the
// degree order in batches of 16 rows. The sampled seconds stay 0.
namespace icpp_online {
struct Timing {
    double convert = 0, lr = 0, kernel = 0, normalize = 0, activation = 0, total = 0;
};
// Counters of the reference's CPU schedule. blocks, max_updates, rescales,
// rescale_events and neighbor_steps are the device's exact counts
// (gat_b200_tfs_online_counters). The AMX call, FMA, tile, spill/reload and
// rescaled-element counts are MODELLED from those counts with the reference's
// CPU work identities (AMX tiles of 16 rows, 32-wide K blocks, register
// spills per rescale event); the GPU kernels do not execute that schedule, so
// they are not device measurements. The drivers print them with
// cpu_schedule_counters=modelled_not_measured_on_gpu.
struct Stats {
    double score_generation = 0, block_max = 0, exp_den = 0;
    double rescale_store = 0, rescale_vector = 0, rescale_reload = 0;
    double source_gather = 0, weighted_convert = 0, tile_load = 0, amx_compute = 0;
    double final_store = 0, output_write = 0, scheduling = 0, tile_config = 0;
    uint64_t blocks = 0, max_updates = 0, rescales = 0;
    uint64_t rescaled_feature_elements = 0, rescaled_padded_feature_elements = 0;
    uint64_t spill_bytes = 0, reload_bytes = 0, rescale_events = 0;
    uint64_t amx_calls = 0, neighbor_steps = 0, executed_fma = 0;
    uint64_t sampled_tiles = 0, total_tiles = 0;
};
struct Workspace {
    gat_b200::Workspace base;
    std::vector<uint64_t> row_blocks, row_max_updates, row_rescales;
    uint64_t allocated_n = 0;
    int allocated_in = 0, allocated_heads = 0, allocated_dim = 0, thread_capacity = 1;
    std::shared_ptr<gat_b200::detail::DeviceBuffer> d_counts = std::make_shared<gat_b200::detail::DeviceBuffer>();
    // icpp_online.cpp:293-306
    void allocate(const Graph& g, const Param& p, bool counters = false) {
        p.validate();
        if (!g.n || g.row.size() != g.n + 1 || g.col.size() != g.e)
            throw std::runtime_error("ICPP Online requires a validated destination CSR");
        base = gat_b200::Workspace{};
        base.allocate(g, p, "tfs_bf16");
        allocated_n = g.n;
        allocated_in = p.in;
        allocated_heads = p.heads;
        allocated_dim = p.dim;
        const size_t nk = checked(g.n, uint64_t(p.heads));
        if (counters) {
            row_blocks.assign(nk, 0);
            row_max_updates.assign(nk, 0);
            row_rescales.assign(nk, 0);
        } else {
            row_blocks.clear();
            row_max_updates.clear();
            row_rescales.clear();
        }
    }
    size_t bytes() const {
        return base.bytes() + (row_blocks.size() + row_max_updates.size() + row_rescales.size()) * sizeof(uint64_t);
    }
};
}  // namespace icpp_online

namespace icpp_block {
using Timing = icpp_online::Timing;
struct Workspace {
    icpp_online::Workspace original;
    std::vector<float> ubuf;
    std::vector<BF16> bbuf;
    void allocate(const Graph& g, const Param& p, bool counters = false) { original.allocate(g, p, counters); }
    size_t bytes() const { return original.bytes() + ubuf.size() * sizeof(float) + bbuf.size() * sizeof(BF16); }
};
struct Stats {
    icpp_online::Stats baseline;
    uint64_t actual_input_feature_FMA = 0;
    uint64_t padded_input_feature_FMA = 0;
    uint64_t useful_projection_FMA = 0;
    uint64_t logical_H_bytes = 0;
    uint64_t block_projection_calls = 0;
    uint64_t conversion_elements = 0;
    uint64_t source_neighbor_steps = 0;
};
}  // namespace icpp_block

namespace icpp_heads {
using Timing = icpp_online::Timing;
struct Workspace {
    icpp_block::Workspace fallback;
    std::vector<float> ubuf, vbuf;
    std::vector<BF16> bbuf;
    void allocate(const Graph& g, const Param& p, bool counters = false) { fallback.allocate(g, p, counters); }
    size_t bytes() const {
        return fallback.bytes() + (ubuf.size() + vbuf.size()) * sizeof(float) + bbuf.size() * sizeof(BF16);
    }
};
struct Stats {
    icpp_online::Stats baseline;
    bool optimized = false;
    uint64_t ph_calls = 0, ph_physical_fma = 0, ph_useful_fma = 0;
    uint64_t raw_H_bytes = 0, packed_H_bytes = 0, projection_calls = 0;
    uint64_t head_switch_store_bytes = 0, head_switch_reload_bytes = 0, ub_scatter_bytes = 0;
    double source_index = 0, H_pack = 0, P_pack = 0, PH_load = 0, PH_compute = 0;
    double PH_store_scatter = 0, UB_convert = 0, UW_load = 0, UW_compute = 0;
    double V_store = 0, V_reload = 0, row_rescale = 0, transition = 0;
};
}  // namespace icpp_heads

namespace detail {
// The reference's tiles: 16 consecutive rows of the degree order per head (its
// panels are multiples of 16, so the batching does not depend on them). Per
// head: the batches, those with an edge, the sum of the batches' maximum
// degrees and of their neighbour blocks ceil(max / block).
struct BatchSteps {
    uint64_t batches = 0, active = 0, steps = 0, blocks = 0;
};
inline BatchSteps batch_steps(const Graph& g, const Schedule& s, int block) {
    BatchSteps r;
    for (uint64_t first = 0; first < g.n; first += 16) {
        uint64_t m = 0;
        for (uint64_t i = first; i < std::min<uint64_t>(g.n, first + 16); ++i) {
            const uint32_t v = s.perm[i];
            if (v >= g.n) throw std::runtime_error("schedule is not a permutation of the rows");
            m = std::max<uint64_t>(m, g.row[v + 1] - g.row[v]);
        }
        ++r.batches;
        r.active += m > 0;
        r.steps += m;
        r.blocks += (m + uint64_t(block) - 1) / uint64_t(block);
    }
    return r;
}
// Tile counts of a call (icpp_online.cpp:330-338): every tile of every head
// when counting or sampling, every profile_period-th of them sampled.
inline void tiles(const Graph& g, int heads, int profile_period, bool counters, icpp_online::Stats& s) {
    const uint64_t t = uint64_t(heads) * ((g.n + 15) / 16);
    if (counters || profile_period > 0) s.total_tiles = t;
    if (profile_period > 0) s.sampled_tiles = (t + uint64_t(profile_period) - 1) / uint64_t(profile_period);
}
// The checks of validate_call (icpp_online.cpp:265-290, icpp_block.cpp:244-270)
// that apply on the device, with the reference's messages under `who`.
inline void online_check(const Graph& g, const Param& p, const Prepared& q, const Schedule& sched,
                         const icpp_online::Workspace& w, int block, int panel, int profile_period, bool counters,
                         const std::string& who, bool block_range = true) {
    if (block_range && (block < 1 || block > 64))
        throw std::runtime_error(who == "ICPP Online" ? "ICPP Online block must be in [1,64]"
                                                      : "ICPP block size must be in [1,64]");
    if (panel < 16 || panel % 16) throw std::runtime_error(who + " panel must be a multiple of 16");
    if (profile_period < 0) throw std::runtime_error(who + " profile period must be nonnegative");
    if (!g.n || p.in <= 0 || p.heads < 1 || p.heads > 8 || p.dim < 1 || p.dim > 64 || w.allocated_n != g.n ||
        w.allocated_in != p.in || w.allocated_heads != p.heads || w.allocated_dim != p.dim)
        throw std::runtime_error(who + " workspace or parameter shape mismatch");
    const size_t nk = checked(g.n, uint64_t(p.heads)), nw = checked(g.n, uint64_t(p.width()));
    const auto& b = w.base;
    if (g.row.size() != g.n + 1 || g.col.size() != g.e || sched.perm.size() != g.n || !q.layer ||
        q.padded_in != (p.in + 31) / 32 * 32 || q.output_blocks != (p.dim + 15) / 16 ||
        b.xbf.size() != checked(g.n, uint64_t(p.in)) || b.left.size() != nk || b.right.size() != nk ||
        b.max.size() != nk || b.den.size() != nk || b.out.size() != nw)
        throw std::runtime_error(who + " CSR, packed weights, or buffer size mismatch");
    if (counters && (w.row_blocks.size() != nk || w.row_max_updates.size() != nk || w.row_rescales.size() != nk))
        throw std::runtime_error(who + " counter arrays not allocated");
}
// The attention-policy check of the layer() functions.
inline int online_policy(const std::string& policy, const std::string& who) {
    if (policy != "fp32" && policy != "bf16" && policy != "avx")
        throw std::runtime_error(who + " attention policy or prepared buffer mismatch");
    return lr_policy(policy);
}
// The online aggregation of x (BF16 [n][ldb], device) with the attention terms
// l, r (device): unnormalized out, den and the final row maxima into w.base;
// with counters the per-row Online units into w's arrays and their totals
// {blocks, max_updates, rescales, rescale_events, neighbor_steps} into tot.
inline void online_run(const Graph& g, const Param& p, const Prepared& q, icpp_online::Workspace& w, const void* x,
                       int ldb, const float* l, const float* r, int rounding, int block, int threshold,
                       bool counters, uint64_t tot[5]) {
    gat_b200::Workspace& b = w.base;
    float* o = static_cast<float*>(b.d_out->get(b.out.size() * 4));
    float* dn = static_cast<float*>(b.d_den->get(b.den.size() * 4));
    float* mx = static_cast<float*>(b.d_max->get(b.max.size() * 4));
    check(gat_b200_tfs_aggregate(b.graph->of(g), q.layer->p, x, ldb, l, r, nullptr, nullptr, nullptr, rounding, block,
                                 threshold, o, p.width(), dn, mx, nullptr));
    check(gat_b200_check_device());
    b.d_out->download(b.out);
    b.d_den->download(b.den);
    b.d_max->download(b.max);
    if (!counters) return;
    const size_t nk = checked(g.n, uint64_t(p.heads));
    uint64_t* rows = static_cast<uint64_t*>(w.d_counts->get(3 * nk * sizeof(uint64_t)));
    check(gat_b200_tfs_online_counters(b.graph->of(g), p.heads, l, r, block, rows, rows + nk, rows + 2 * nk, tot,
                                       nullptr));
    check(gat_b200_copy_to_host(w.row_blocks.data(), rows, nk * sizeof(uint64_t)));
    check(gat_b200_copy_to_host(w.row_max_updates.data(), rows + nk, nk * sizeof(uint64_t)));
    check(gat_b200_copy_to_host(w.row_rescales.data(), rows + 2 * nk, nk * sizeof(uint64_t)));
}
// online_run from the host copies in w.base (xbf, left, right): the
// aggregate() entry points.
inline void online_from_host(const Graph& g, const Param& p, const Prepared& q, icpp_online::Workspace& w,
                             int rounding, int block, int threshold, bool counters, uint64_t tot[5]) {
    gat_b200::Workspace& b = w.base;
    const int ldb = padded(p.in, GAT_B200_BF16);
    std::vector<BF16> xp(size_t(g.n) * ldb, 0);
    for (uint64_t i = 0; i < g.n; ++i)
        std::copy(b.xbf.begin() + i * p.in, b.xbf.begin() + (i + 1) * p.in, xp.begin() + i * ldb);
    const void* x = b.d_xb->upload(xp);
    const float* l = b.d_left->upload(b.left);
    const float* r = b.d_right->upload(b.right);
    online_run(g, p, q, w, x, ldb, l, r, rounding, block, threshold, counters, tot);
}
// A whole layer on the device (icpp_online.cpp:360-382): lr_reordered writing
// the BF16 copy of the input, the online aggregation, finish; the host copies
// of xbf, left, right, max, den and the finished out are left in w.base.
inline void online_layer(const Graph& g, const Param& p, const Prepared& q, const std::vector<float>& input,
                         icpp_online::Workspace& w, bool hidden, int policy, int rounding, int block,
                         int threshold, bool counters, icpp_online::Timing& t, uint64_t tot[5]) {
    gat_b200::Workspace& b = w.base;
    t = icpp_online::Timing{};
    const auto begin = Clock::now();
    auto a = begin;
    const float* x = b.d_x->upload(input);
    const int ldb = padded(p.in, GAT_B200_BF16);
    void* xb = b.d_xb->get(size_t(g.n) * ldb * 2);
    float* l = static_cast<float*>(b.d_left->get(b.left.size() * 4));
    float* r = static_cast<float*>(b.d_right->get(b.right.size() * 4));
    check(gat_b200_lr_reordered(q.layer->p, g.n, x, GAT_B200_F32, p.in, policy, xb, ldb, l, r, nullptr));
    check(gat_b200_check_device());
    t.lr = seconds(a, Clock::now());
    a = Clock::now();
    online_run(g, p, q, w, xb, ldb, l, r, rounding, block, threshold, counters, tot);
    t.kernel = seconds(a, Clock::now());
    a = Clock::now();
    check(gat_b200_finish(g.n, p.heads, p.dim, static_cast<const float*>(b.d_den->p), hidden,
                          static_cast<float*>(b.d_out->p), p.width(), nullptr));
    check(gat_b200_check_device());
    b.d_out->download(b.out);
    t.normalize = seconds(a, Clock::now());
    b.d_left->download(b.left);
    b.d_right->download(b.right);
    std::vector<BF16> tmp(size_t(g.n) * ldb);
    check(gat_b200_copy_to_host(tmp.data(), xb, tmp.size() * 2));
    for (uint64_t i = 0; i < g.n; ++i)
        std::copy(tmp.begin() + i * ldb, tmp.begin() + i * ldb + p.in, b.xbf.begin() + i * p.in);
    t.total = seconds(begin, Clock::now());
}
// Online units shared by the three variants; `padded_dim` is the padded
// feature count a rescale touches in the reference's kernel.
inline void online_units(const uint64_t tot[5], uint64_t dim, uint64_t padded_dim, icpp_online::Stats& s) {
    s.blocks = tot[0];
    s.max_updates = tot[1];
    s.rescales = tot[2];
    s.rescale_events = tot[3];
    s.rescaled_feature_elements = tot[2] * dim;
    s.rescaled_padded_feature_elements = tot[2] * padded_dim;
}
// The counts of icpp_online (icpp_online.cpp:100-235): one AMX step per
// neighbour position of a batch.
inline void online_stats(const Param& p, const Prepared& q, const uint64_t tot[5], icpp_online::Stats& s) {
    const uint64_t dp = uint64_t(q.padded_in), obs = uint64_t(q.output_blocks);
    online_units(tot, uint64_t(p.dim), obs * 16, s);
    s.spill_bytes = s.reload_bytes = tot[3] * obs * 1024;
    s.neighbor_steps = tot[4];
    s.amx_calls = tot[4] * (dp / 32) * obs;
    s.executed_fma = tot[4] * 16 * dp * obs * 16;
}
// The counts of icpp_block (icpp_block.cpp:100-212): one AMX projection per
// neighbour block of a batch.
inline void block_stats(const Graph& g, const Param& p, const Prepared& q, const Schedule& sched, int block,
                        const uint64_t tot[5], icpp_block::Stats& st) {
    auto& s = st.baseline;
    const uint64_t dp = uint64_t(q.padded_in), obs = uint64_t(q.output_blocks), K = uint64_t(p.heads);
    const uint64_t in = uint64_t(p.in), calls = K * batch_steps(g, sched, block).blocks;
    online_units(tot, uint64_t(p.dim), obs * 16, s);
    s.spill_bytes = s.reload_bytes = tot[3] * obs * 1024;
    s.neighbor_steps = calls;
    s.amx_calls = calls * (dp / 32) * obs;
    s.executed_fma = calls * 16 * dp * obs * 16;
    st.block_projection_calls = calls;
    st.conversion_elements = calls * 16 * dp;
    st.source_neighbor_steps = tot[4];
    st.useful_projection_FMA = tot[0] * in * uint64_t(p.dim);
    st.actual_input_feature_FMA = K * g.e * in;
    st.padded_input_feature_FMA = K * g.e * ((in + 15) / 16 * 16);
    st.logical_H_bytes = K * g.e * in * sizeof(BF16);
}
}  // namespace detail

namespace icpp_online {
// icpp_online.hpp:37-39: unnormalized V of base.xbf, base.left, base.right
// into base.out, with base.den and base.max.
inline void aggregate(const Graph& g, const Param& p, const Prepared& q, const Schedule& sched, Workspace& w,
                      int block, int panel, Stats& stats, int profile_period = 0, bool counters = false) {
    detail::online_check(g, p, q, sched, w, block, panel, profile_period, counters, "ICPP Online");
    stats = Stats{};
    uint64_t tot[5] = {};
    detail::online_from_host(g, p, q, w, GAT_B200_TFS_EDGE, block, 1, counters, tot);
    if (counters) detail::online_stats(p, q, tot, stats);
    detail::tiles(g, p.heads, profile_period, counters, stats);
}
// icpp_online.hpp:40-43
inline void layer(const Graph& g, const Param& p, const Prepared& q, const Schedule& sched,
                  const std::vector<float>& input, Workspace& w, bool hidden, int block, int panel, Timing& t,
                  Stats& stats, int profile_period = 0, bool counters = false,
                  const std::string& lr_policy = "fp32") {
    detail::online_check(g, p, q, sched, w, block, panel, profile_period, counters, "ICPP Online");
    if (input.size() != checked(g.n, uint64_t(p.in))) throw std::runtime_error("ICPP Online input shape mismatch");
    const int policy = detail::online_policy(lr_policy, "ICPP Online");
    stats = Stats{};
    uint64_t tot[5] = {};
    detail::online_layer(g, p, q, input, w, hidden, policy, GAT_B200_TFS_EDGE, block, 1, counters, t, tot);
    if (counters) detail::online_stats(p, q, tot, stats);
    detail::tiles(g, p.heads, profile_period, counters, stats);
}
}  // namespace icpp_online

namespace icpp_block {
// icpp_block.hpp:33-35
inline void aggregate(const Graph& g, const Param& p, const Prepared& q, const Schedule& sched, Workspace& w,
                      int block, int panel, Stats& stats, int profile_period = 0, bool counters = false) {
    detail::online_check(g, p, q, sched, w.original, block, panel, profile_period, counters, "ICPP block");
    stats = Stats{};
    uint64_t tot[5] = {};
    detail::online_from_host(g, p, q, w.original, GAT_B200_TFS_BLOCK, block, 1, counters, tot);
    if (counters) detail::block_stats(g, p, q, sched, block, tot, stats);
    detail::tiles(g, p.heads, profile_period, counters, stats.baseline);
}
// icpp_block.hpp:36-39
inline void layer(const Graph& g, const Param& p, const Prepared& q, const Schedule& sched,
                  const std::vector<float>& input, Workspace& w, bool hidden, int block, int panel, Timing& t,
                  Stats& stats, int profile_period = 0, bool counters = false,
                  const std::string& lr_policy = "fp32") {
    detail::online_check(g, p, q, sched, w.original, block, panel, profile_period, counters, "ICPP block");
    if (input.size() != checked(g.n, uint64_t(p.in))) throw std::runtime_error("ICPP block input shape mismatch");
    const int policy = detail::online_policy(lr_policy, "ICPP block");
    stats = Stats{};
    uint64_t tot[5] = {};
    detail::online_layer(g, p, q, input, w.original, hidden, policy, GAT_B200_TFS_BLOCK, block, 1, counters, t, tot);
    if (counters) detail::block_stats(g, p, q, sched, block, tot, stats);
    detail::tiles(g, p.heads, profile_period, counters, stats.baseline);
}
}  // namespace icpp_block

namespace icpp_heads_hybrid {
using Timing = icpp_heads::Timing;
using Workspace = icpp_heads::Workspace;
using Stats = icpp_heads::Stats;
namespace detail {
// icpp_heads_hybrid.cpp:35-41
inline void check_threshold(int threshold) {
    if (threshold < 1 || threshold > 33) throw std::runtime_error("ICPP heads hybrid threshold must be in [1,33]");
}
inline bool optimized_shape(const Param& p) { return p.heads == 8 && p.dim == 32 && p.in > 0 && p.in <= 256; }
// validate() of icpp_heads_hybrid.cpp:296-316 (the device-side subset)
inline void validate(const Graph& g, const Param& p, const Prepared& q, const Schedule& sched, const Workspace& w,
                  int block, int panel, int profile_period, bool counters) {
    if (block != 16 && block != 32) throw std::runtime_error("optimized ICPP heads block must be 16 or 32");
    const auto& o = w.fallback.original;
    if (panel < 16 || panel % 16) throw std::runtime_error("ICPP heads panel must be a multiple of 16");
    if (profile_period < 0) throw std::runtime_error("ICPP heads profile period must be nonnegative");
    if (!g.n || o.allocated_n != g.n || o.allocated_in != p.in || o.allocated_heads != p.heads ||
        o.allocated_dim != p.dim)
        throw std::runtime_error("ICPP heads workspace shape/thread capacity mismatch");
    try {
        gat_b200::detail::online_check(g, p, q, sched, o, block, panel, profile_period, false, "ICPP heads", false);
    } catch (const std::runtime_error&) {
        throw std::runtime_error("ICPP heads CSR, prepared weights or local buffer shape mismatch");
    }
    const size_t nk = checked(g.n, uint64_t(p.heads));
    if (counters && (o.row_blocks.size() != nk || o.row_max_updates.size() != nk || o.row_rescales.size() != nk))
        throw std::runtime_error("ICPP heads counter arrays not allocated");
}
// The counts of the optimized kernel (icpp_heads_hybrid.cpp:100-265), as the
// reference's own work identities state them (tfs_online/adaptive_main.cpp:
// 44-60): one UW projection per head and neighbour block of a batch, V stored
// at every head switch and reloaded after the first block; per row and block of
// `len` neighbours, PH on AMX (high and low halves) when len >= threshold, else
// on AVX over the FP32 p.
inline void stats_of(const Graph& g, const Param& p, const Prepared& q, const Schedule& sched, int block,
                     int threshold, const uint64_t tot[5], Stats& st) {
    auto& s = st.baseline;
    const uint64_t dp = uint64_t(q.padded_in), K = uint64_t(p.heads), in = uint64_t(p.in);
    const uint64_t in16 = (in + 15) / 16 * 16;
    const auto b = gat_b200::detail::batch_steps(g, sched, block);
    const uint64_t calls = K * b.blocks;
    gat_b200::detail::online_units(tot, 32, 32, s);
    s.neighbor_steps = calls;
    s.amx_calls = calls * (dp / 32) * 2;
    s.executed_fma = calls * 16 * dp * 32;
    st.projection_calls = calls;
    st.head_switch_store_bytes = calls * 2048;
    st.head_switch_reload_bytes = (calls - K * b.active) * 2048;
    uint64_t amx = 0, avx = 0, avx_edges = 0;
    for (uint64_t i = 0; i < g.n; ++i) {
        const uint64_t deg = g.row[i + 1] - g.row[i];
        for (uint64_t at = 0; at < deg; at += uint64_t(block)) {
            const uint64_t len = std::min<uint64_t>(uint64_t(block), deg - at);
            if (len < uint64_t(threshold)) {
                ++avx;
                avx_edges += len;
            } else {
                ++amx;
            }
        }
    }
    st.ph_calls = amx * (dp / 16) * 2;
    st.ph_physical_fma = amx * K * 32 * dp * 2 + avx_edges * K * in16;
    st.ph_useful_fma = g.e * K * in;
    st.raw_H_bytes = g.e * in * sizeof(BF16);
    st.packed_H_bytes = amx * 32 * dp * sizeof(BF16);
    st.ub_scatter_bytes = amx * K * dp * sizeof(float) + avx * K * in16 * sizeof(float);
}
}  // namespace detail
// icpp_heads_hybrid.hpp:18-20
inline void aggregate(const Graph& g, const Param& p, const Prepared& q, const Schedule& sched, Workspace& w,
                      int block, int panel, Stats& stats, int profile_period = 0, bool counters = false,
                      int threshold = 16) {
    detail::check_threshold(threshold);
    stats = Stats{};
    if (!detail::optimized_shape(p)) {
        icpp_block::Stats fallback;
        icpp_block::aggregate(g, p, q, sched, w.fallback, block, panel, fallback, profile_period, counters);
        stats.baseline = fallback.baseline;
        stats.projection_calls = fallback.block_projection_calls;
        return;
    }
    detail::validate(g, p, q, sched, w, block, panel, profile_period, counters);
    stats.optimized = true;
    uint64_t tot[5] = {};
    gat_b200::detail::online_from_host(g, p, q, w.fallback.original, GAT_B200_TFS_SPLIT, block, threshold, counters,
                                       tot);
    if (counters) detail::stats_of(g, p, q, sched, block, threshold, tot, stats);
    gat_b200::detail::tiles(g, p.heads, profile_period, counters, stats.baseline);
}
// icpp_heads_hybrid.hpp:21-24
inline void layer(const Graph& g, const Param& p, const Prepared& q, const Schedule& sched,
                  const std::vector<float>& input, Workspace& w, bool hidden, int block, int panel, Timing& t,
                  Stats& stats, int profile_period = 0, bool counters = false,
                  const std::string& lr_policy = "fp32", int threshold = 16) {
    detail::check_threshold(threshold);
    if (!detail::optimized_shape(p)) {
        icpp_block::Stats fallback;
        icpp_block::layer(g, p, q, sched, input, w.fallback, hidden, block, panel, t, fallback, profile_period,
                          counters, lr_policy);
        stats = Stats{};
        stats.baseline = fallback.baseline;
        stats.projection_calls = fallback.block_projection_calls;
        return;
    }
    detail::validate(g, p, q, sched, w, block, panel, profile_period, counters);
    if (input.size() != checked(g.n, uint64_t(p.in)))
        throw std::runtime_error("ICPP heads hybrid input shape mismatch");
    const int policy = gat_b200::detail::online_policy(lr_policy, "ICPP heads hybrid");
    stats = Stats{};
    stats.optimized = true;
    uint64_t tot[5] = {};
    gat_b200::detail::online_layer(g, p, q, input, w.fallback.original, hidden, policy, GAT_B200_TFS_SPLIT, block,
                                   threshold, counters, t, tot);
    if (counters) detail::stats_of(g, p, q, sched, block, threshold, tot, stats);
    gat_b200::detail::tiles(g, p.heads, profile_period, counters, stats.baseline);
}
}  // namespace icpp_heads_hybrid

}  // namespace gat_b200
