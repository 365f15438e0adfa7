// Row-partitioned three-layer GAT forward behind the C ABI: one process per
// GPU of one NVLink/NVSwitch node, each running the reference's model loop
// (baseline/bench/main.cpp:171-172) on its share of destination rows.
//
// Destination rows are independent given the projected features of all their
// sources, so each layer is: projection of the rank's rows, one exchange that
// puts every rank's H and R into every rank's feature table, aggregation of
// the rank's rows from that table.
//
// Layout (gat_b200_partition): rank k owns rows [cuts[k], cuts[k+1]),
// balanced by edge count; its rows are cut again into `chunks` row chunks.
// Each layer's feature table is chunk-major with equal blocks (an all-gather
// moves equal blocks): chunk c of rank k sits at table row
// (c*world + k) * block_rows, and every chunk's CSR slice has its source ids
// remapped to table rows once, at create.
//
// Exchange P2P (default): the tables are CUDA IPC allocations every rank
// maps.
//  * Layer 1 moves its BF16 input rows (din padded to 16 bytes: 208 bytes on
//    c4), narrower than H (512 bytes): the conversion kernel stores each
//    converted row into every rank's input table, a bounded cross-GPU flag
//    barrier closes the exchange, and every rank projects the whole table
//    itself (the same kernel on the same bytes gives the same H everywhere).
//  * Layers 2 and 3: the projection kernel of the rank's rows stores each H/R
//    tile into every rank's table (gat_b200_projection_scatter), then the
//    barrier.
// A rank writes layer l's table of forward s+1 only after it passed the
// barrier of layer l+1 of forward s, which every rank reaches after its
// layer-l aggregation of forward s: no store lands on rows a peer may still
// read, and no end-of-forward barrier is needed.
//
// Exchange NCCL: each rank projects its own rows into a send block and NCCL
// all-gathers H and R into full tables (on the model's stream).
#include <algorithm>
#include <array>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "device.cuh"
#include "graph.cuh"

namespace gatb {
int aggregate_dispatch_reserved(const gat_b200_graph* g, int heads, int dim, const void* h, int h_dtype, int ldh,
                                const float* left, const float* right, const float* fixed_p, const float* fixed_den,
                                int unnorm, int hidden, void* out, int out_bf16, int ldo, float* den, float* max,
                                cudaStream_t st, int reserve_sms, int npeer, uint16_t* const* out_peer);
int convert_launch(uint64_t n, int width, const float* in, int ld_in, uint16_t* out, int ld_out, cudaStream_t st);
int convert_scatter_launch(uint64_t n, int width, const float* in, int ld_in, int ndst, uint16_t* const* dst,
                           int ld_out, cudaStream_t st);
int projection_tc_launch(const gat_b200_layer* p, uint64_t n, const uint16_t* x, int ldx, uint16_t* h, int ldh,
                         float* z, int ldz, float* left, float* right, cudaStream_t st, int npeer,
                         uint16_t* const* h_peer, float* const* r_peer, int max_ctas);
int peer_barrier_launch(void* const* flags, int world, int rank, uint32_t epoch, cudaStream_t st);
int graph_create_part_basis(uint64_t n, uint64_t n_src, uint64_t e, const uint64_t* row, const uint32_t* col,
                            void* stream, uint64_t basis_e, gat_b200_graph** out);
int device_check_errors();

namespace {

constexpr int kMaxWorld = 8;
constexpr int kMaxChunks = 64;
constexpr int kEvents = GAT_B200_PART_STAGES + 1;
// SMs left to the projection-and-exchange kernel while an aggregation runs
// beside it (P2P exchange with several row chunks).
constexpr int kDefaultReserve = 16;
// P2P tables per rank: H of layers 1-3, R of layers 1-3, layer-1 BF16 input,
// barrier flags, layer-2 BF16 input
constexpr int kTables = 9;

struct Layout {
    int world = 1, chunks = 1;
    std::vector<uint64_t> cuts;    // [world + 1]
    std::vector<uint64_t> ccuts;   // [world * (chunks + 1)], global rows
    std::vector<uint64_t> starts;  // [world * chunks] first row of (rank, chunk), ascending
    uint64_t block_rows = 0, table_rows = 0;
};

// First index i in [lo, hi] with row[i] >= x.
uint64_t first_reaching(const uint64_t* row, uint64_t lo, uint64_t hi, uint64_t x) {
    return uint64_t(std::lower_bound(row + lo, row + hi + 1, x) - row);
}

int layout_build(uint64_t n, const uint64_t* row, int world, int chunks, Layout& L) {
    if (!row || n == 0) return fail("partition: empty graph");
    if (world < 1 || world > kMaxWorld) return fail("partition: world size must be 1..8");
    if (chunks < 1 || chunks > kMaxChunks) return fail("partition: chunks must be 1..64");
    if (row[0] != 0) return fail("nonmonotone CSR");
    for (uint64_t i = 0; i < n; ++i)
        if (row[i + 1] < row[i]) return fail("nonmonotone CSR");
    const uint64_t e = row[n];
    L.world = world;
    L.chunks = chunks;
    L.cuts.assign(world + 1, 0);
    L.cuts[world] = n;
    for (int k = 1; k < world; ++k) {
        const uint64_t t = uint64_t((unsigned __int128)e * unsigned(k) / unsigned(world));
        L.cuts[k] = std::max(L.cuts[k - 1], std::min(first_reaching(row, 0, n, t), n));
    }
    L.ccuts.assign(size_t(world) * (chunks + 1), 0);
    uint64_t biggest = 0;
    for (int r = 0; r < world; ++r) {
        const uint64_t lo = L.cuts[r], hi = L.cuts[r + 1];
        uint64_t* cc = &L.ccuts[size_t(r) * (chunks + 1)];
        cc[0] = lo;
        cc[chunks] = hi;
        const uint64_t e0 = row[lo], e1 = row[hi];
        for (int k = 1; k < chunks; ++k) {
            const uint64_t t = e0 + uint64_t((unsigned __int128)(e1 - e0) * unsigned(k) / unsigned(chunks));
            cc[k] = std::max(cc[k - 1], std::min(std::max(first_reaching(row, lo, hi, t), lo), hi));
        }
        for (int k = 0; k < chunks; ++k) biggest = std::max(biggest, cc[k + 1] - cc[k]);
    }
    L.block_rows = (std::max<uint64_t>(1, biggest) + 3) / 4 * 4;
    L.table_rows = uint64_t(chunks) * world * L.block_rows;
    if (L.table_rows > uint64_t(INT32_MAX)) return fail_code(GAT_B200_EUNSUPPORTED, "partition: table too large");
    L.starts.resize(size_t(world) * chunks);
    for (int r = 0; r < world; ++r)
        for (int c = 0; c < chunks; ++c) L.starts[size_t(r) * chunks + c] = L.ccuts[size_t(r) * (chunks + 1) + c];
    return 0;
}

// Table row of global source id src (chunks of zero rows are skipped).
uint32_t layout_slot(const Layout& L, uint64_t src) {
    const size_t k = size_t(std::upper_bound(L.starts.begin(), L.starts.end(), src) - L.starts.begin()) - 1;
    const uint64_t r = k / L.chunks, c = k % L.chunks;
    return uint32_t((c * L.world + r) * L.block_rows + (src - L.starts[k]));
}

int dalloc(void** p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e == cudaSuccess) e = cudaMemset(*p, 0, bytes ? bytes : 16);
    return e == cudaSuccess ? 0 : cuda_fail(e, "part_model: device allocation");
}

}  // namespace
}  // namespace gatb

using namespace gatb;

struct gat_b200_part_model {
    struct Chunk {
        uint64_t a = 0, b = 0;   // local rows [a, b)
        uint64_t row0 = 0;       // table row of this chunk's block
        gat_b200_graph* g = nullptr;
    };
    gat_b200_comm* comm = nullptr;
    int world = 1, rank = 0, exchange = GAT_B200_EXCHANGE_P2P;
    Layout L;
    uint64_t lo = 0, hi = 0, n_loc = 0, e_loc = 0;
    const gat_b200_layer* layers[3] = {};
    int din = 0, classes = 0, ld0 = 0, ldx = 0, ldh[3] = {}, heads[3] = {};
    std::vector<Chunk> chunks;
    // P2P: tables t = 0..2 H of layer t+1, 3..5 R of layer t-2, 6 the layer-1
    // BF16 input, 7 the barrier flags; tab[j][t] = rank j's table t as mapped here.
    std::vector<std::array<void*, kTables>> tab;
    // P2P: layer 2's input rows reach every rank through the layer-1
    // aggregation's epilogue (table 8) and every rank projects the whole table
    bool x2x = false;
    bool x2_last = false;  // the last forward ran the layer-2 input exchange
    std::vector<void*> owned, mapped;
    uint32_t epoch = 0;
    // Overlap (P2P, chunks > 1): the projection and exchange of chunk c run on
    // xst, on reserve_sms SMs the aggregation of chunk c+1 leaves free.
    int reserve_sms = 0;
    cudaStream_t xst = nullptr;
    std::vector<cudaEvent_t> ev_agg;
    cudaEvent_t ev_xdone = nullptr;
    // NCCL: full tables and per-chunk send blocks (plain device memory).
    void* h_full[3] = {};
    float* r_full[3] = {};
    void* h_send = nullptr;
    float* r_send = nullptr;
    uint16_t* x0 = nullptr;  // NCCL: this rank's BF16 input rows
    // working buffers of this rank's rows
    float* x_f32 = nullptr;
    float* left0 = nullptr;     // P2P: L of every table row for layer 1
    float* left[2] = {};        // L of this rank's rows, layers 1 (NCCL) / 2 / 3
    void* xs[2] = {};           // BF16 hidden outputs (inputs of layers 2 and 3)
    float* logits = nullptr;
    // timing
    bool timing = false;
    cudaEvent_t ev[kEvents] = {};
    int launches_last = 0;
    uint64_t forwards = 0;
    // pipelined requests
    float* ax[2] = {};
    float* alog[2] = {};
    cudaEvent_t ev_up[2] = {}, ev_done[2] = {}, ev_down[2] = {};
    cudaStream_t up = nullptr, down = nullptr;
    uint64_t submitted = 0;

    uint16_t* H(int j, int l) const { return static_cast<uint16_t*>(tab[j][l]); }
    float* R(int j, int l) const { return static_cast<float*>(tab[j][3 + l]); }
};

namespace {

void mark(gat_b200_part_model* m, int k, cudaStream_t st) {
    if (m->timing) cudaEventRecord(m->ev[k], st);
}

// Layers 2 and 3 (l = 1, 2): projection of chunk c's rows of the previous
// layer's output and its exchange.
int project_chunk(gat_b200_part_model* m, int l, const gat_b200_part_model::Chunk& ch, cudaStream_t st, int& launches,
                  int max_ctas) {
    const gat_b200_layer* p = m->layers[l];
    const int K = p->heads, ldh = m->ldh[l];
    const uint64_t nr = ch.b - ch.a;
    if (!nr) return 0;
    const uint16_t* x = static_cast<const uint16_t*>(m->xs[(l - 1) & 1]) + ch.a * uint64_t(m->ldx);
    float* left = m->left[l & 1] + ch.a * K;
    int rc;
    if (m->exchange == GAT_B200_EXCHANGE_P2P) {
        uint16_t* hp[7];
        float* rp[7];
        int np = 0;
        for (int j = 0; j < m->world; ++j) {
            if (j == m->rank) continue;
            hp[np] = m->H(j, l) + ch.row0 * ldh;
            rp[np] = m->R(j, l) + ch.row0 * K;
            ++np;
        }
        rc = projection_tc_launch(p, nr, x, m->ldx, m->H(m->rank, l) + ch.row0 * ldh, ldh, nullptr, 0, left,
                                  m->R(m->rank, l) + ch.row0 * K, st, np, hp, rp, max_ctas);
        if (rc == GAT_B200_EUNSUPPORTED)
            return fail_code(rc, "part_model: layer outside the tensor-core projection (input or width > 256)");
        ++launches;
        return rc;
    }
    // NCCL: own rows into the send block, then the all-gather of chunk c
    const size_t hb = size_t(m->L.block_rows) * ldh * 2, rb = size_t(m->L.block_rows) * K * 4;
    rc = projection_tc_launch(p, nr, x, m->ldx, static_cast<uint16_t*>(m->h_send), ldh, nullptr, 0, left,
                              m->r_send, st, 0, nullptr, nullptr, 0);
    if (rc == GAT_B200_EUNSUPPORTED)
        return fail_code(rc, "part_model: layer outside the tensor-core projection (input or width > 256)");
    if (rc) return rc;
    ++launches;
    const size_t c = size_t(&ch - m->chunks.data());
    char* hf = static_cast<char*>(m->h_full[l]) + c * m->world * hb;
    char* rf = reinterpret_cast<char*>(m->r_full[l]) + c * m->world * rb;
    if ((rc = comm_all_gather_device(m->comm, m->h_send, hf, hb, st))) return rc;
    return comm_all_gather_device(m->comm, m->r_send, rf, rb, st);
}

int barrier(gat_b200_part_model* m, cudaStream_t st, int& launches) {
    if (m->exchange != GAT_B200_EXCHANGE_P2P || m->world == 1) return 0;
    void* flags[kMaxWorld];
    for (int j = 0; j < m->world; ++j) flags[j] = m->tab[j][7];
    ++launches;
    return peer_barrier_launch(flags, m->world, m->rank, ++m->epoch, st);
}

}  // namespace

extern "C" {

int gat_b200_partition(uint64_t n, const uint64_t* row, int world, int chunks, uint64_t* cuts, uint64_t* chunk_cuts,
                       uint64_t* block_rows, uint64_t* table_rows) {
    clear_error();
    Layout L;
    int rc = layout_build(n, row, world, chunks, L);
    if (rc) return rc;
    if (cuts) std::copy(L.cuts.begin(), L.cuts.end(), cuts);
    if (chunk_cuts) std::copy(L.ccuts.begin(), L.ccuts.end(), chunk_cuts);
    if (block_rows) *block_rows = L.block_rows;
    if (table_rows) *table_rows = L.table_rows;
    return 0;
}

int gat_b200_partition_slots(uint64_t n, const uint64_t* row, int world, int chunks, uint64_t count,
                             const uint32_t* src, uint32_t* slots) {
    clear_error();
    if (count && (!src || !slots)) return fail("partition_slots: null buffer");
    Layout L;
    int rc = layout_build(n, row, world, chunks, L);
    if (rc) return rc;
    for (uint64_t i = 0; i < count; ++i) {
        if (src[i] >= n) return fail("source index out of bounds");
        slots[i] = layout_slot(L, src[i]);
    }
    return 0;
}

int gat_b200_part_model_destroy(gat_b200_part_model* m);

int gat_b200_part_model_create(gat_b200_comm* comm, uint64_t n, const uint64_t* row, const uint32_t* col_rows,
                               const gat_b200_layer* const* layers, int exchange, int chunks, void* stream,
                               gat_b200_part_model** out) {
    clear_error();
    if (!out) return fail("part_model_create: null output handle");
    *out = nullptr;
    if (!comm || !row || !layers || !layers[0] || !layers[1] || !layers[2]) return fail("part_model_create: null argument");
    if (exchange != GAT_B200_EXCHANGE_P2P && exchange != GAT_B200_EXCHANGE_NCCL)
        return fail("part_model_create: bad exchange");
    for (int l = 0; l < 2; ++l)
        if (layers[l + 1]->in != layers[l]->width) return fail("part_model_create: layer widths do not chain");
    cudaStream_t st = as_stream(stream);
    gat_b200_part_model* m = new (std::nothrow) gat_b200_part_model();
    if (!m) return fail("part_model_create: out of host memory");
    m->comm = comm;
    m->world = comm_world(comm);
    m->rank = comm_rank(comm);
    m->exchange = exchange;
    int rc = layout_build(n, row, m->world, chunks, m->L);
    if (rc) {
        delete m;
        return rc;
    }
    const Layout& L = m->L;
    m->lo = L.cuts[m->rank];
    m->hi = L.cuts[m->rank + 1];
    m->n_loc = m->hi - m->lo;
    m->e_loc = row[m->hi] - row[m->lo];
    if (m->e_loc && !col_rows) {
        delete m;
        return fail("part_model_create: null col_rows");
    }
    for (int l = 0; l < 3; ++l) {
        m->layers[l] = layers[l];
        m->heads[l] = layers[l]->heads;
        m->ldh[l] = gat_b200_padded_ld(layers[l]->width, GAT_B200_BF16);
    }
    m->din = layers[0]->in;
    m->classes = layers[2]->width;
    m->ld0 = gat_b200_padded_ld(m->din, GAT_B200_BF16);
    m->ldx = gat_b200_padded_ld(std::max(layers[0]->width, layers[1]->width), GAT_B200_BF16);
    const uint64_t nt = L.table_rows, nl = m->n_loc;
    do {
        // chunk slices with sources remapped to table rows
        const uint64_t base = row[m->lo];
        std::vector<uint64_t> rl;
        std::vector<uint32_t> cl;
        m->chunks.resize(chunks);
        for (int c = 0; c < chunks; ++c) {
            auto& ch = m->chunks[c];
            const uint64_t A = L.ccuts[size_t(m->rank) * (chunks + 1) + c];
            const uint64_t B = L.ccuts[size_t(m->rank) * (chunks + 1) + c + 1];
            ch.a = A - m->lo;
            ch.b = B - m->lo;
            ch.row0 = (uint64_t(c) * m->world + m->rank) * L.block_rows;
            if (B <= A) continue;
            rl.resize(B - A + 1);
            for (uint64_t i = A; i <= B; ++i) rl[i - A] = row[i] - row[A];
            cl.resize(row[B] - row[A]);
            for (uint64_t k = 0; k < cl.size(); ++k) {
                const uint32_t s = col_rows[row[A] - base + k];
                if (s >= n) {
                    rc = fail("source index out of bounds");
                    break;
                }
                cl[k] = layout_slot(L, s);
            }
            if (rc) break;
            // hub rows cut where the one-GPU graph cuts them (segment length
            // from the whole graph's edge count): the same sums, in the same
            // order, on any number of GPUs
            if ((rc = graph_create_part_basis(B - A, nt, cl.size(), rl.data(), cl.data(), stream, row[n], &ch.g)))
                break;
        }
        if (rc) break;
        const int K0 = m->heads[0];
        if ((rc = dalloc((void**)&m->x_f32, nl * size_t(m->din) * 4))) break;
        for (int b = 0; b < 2; ++b) {
            if ((rc = dalloc((void**)&m->left[b], std::max<uint64_t>(nl, 1) * 8 * 4))) break;
            if ((rc = dalloc(&m->xs[b], nl * size_t(m->ldx) * 2))) break;
        }
        if (rc) break;
        if ((rc = dalloc((void**)&m->logits, nl * size_t(m->classes) * 4))) break;
        if (exchange == GAT_B200_EXCHANGE_P2P) {
            if ((rc = dalloc((void**)&m->left0, nt * K0 * 4))) break;
            // this rank's tables, their IPC handles to every rank, the peers' mapped
            const uint64_t bytes[kTables] = {nt * m->ldh[0] * 2, nt * m->ldh[1] * 2, nt * m->ldh[2] * 2,
                                             nt * m->heads[0] * 4, nt * m->heads[1] * 4, nt * m->heads[2] * 4,
                                             nt * m->ld0 * 2, 64, nt * m->ldx * 2};
            std::vector<unsigned char> handles(kTables * GAT_B200_PEER_HANDLE_BYTES);
            std::array<void*, kTables> own{};
            for (int t = 0; t < kTables && !rc; ++t) {
                rc = gat_b200_peer_alloc(bytes[t], &own[t], &handles[t * GAT_B200_PEER_HANDLE_BYTES]);
                if (!rc) m->owned.push_back(own[t]);
            }
            if (rc) break;
            std::vector<unsigned char> all(handles.size() * m->world);
            if ((rc = gat_b200_comm_all_gather(comm, handles.data(), all.data(), handles.size()))) break;
            m->tab.assign(m->world, std::array<void*, kTables>{});
            for (int j = 0; j < m->world && !rc; ++j) {
                if (j == m->rank) {
                    m->tab[j] = own;
                    continue;
                }
                for (int t = 0; t < kTables && !rc; ++t) {
                    rc = gat_b200_peer_open(&all[(size_t(j) * kTables + t) * GAT_B200_PEER_HANDLE_BYTES],
                                            &m->tab[j][t]);
                    if (!rc) m->mapped.push_back(m->tab[j][t]);
                }
            }
            if (rc) break;
            // every rank's tables exist and are zeroed before any rank stores into them
            if ((rc = gat_b200_comm_barrier(comm))) break;
            m->x2x = m->world > 1 && m->heads[1] <= m->heads[0];
        } else {
            if ((rc = dalloc((void**)&m->x0, nl * size_t(m->ld0) * 2))) break;
            int ldm = std::max(m->ldh[0], std::max(m->ldh[1], m->ldh[2]));
            if ((rc = dalloc(&m->h_send, L.block_rows * size_t(ldm) * 2))) break;
            if ((rc = dalloc((void**)&m->r_send, L.block_rows * 8 * 4))) break;
            for (int l = 0; l < 3 && !rc; ++l) {
                if ((rc = dalloc(&m->h_full[l], nt * size_t(m->ldh[l]) * 2))) break;
                rc = dalloc((void**)&m->r_full[l], nt * size_t(m->heads[l]) * 4);
            }
            if (rc) break;
        }
        for (int k = 0; k < kEvents && !rc; ++k)
            if (cudaEventCreate(&m->ev[k]) != cudaSuccess) rc = fail("part_model_create: event");
        if (rc) break;
        // the exchange stream (highest priority) and its events
        {
            int least = 0, greatest = 0;
            cudaError_t e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
            if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&m->xst, cudaStreamNonBlocking, greatest);
            m->ev_agg.assign(chunks, nullptr);
            for (int c = 0; c < chunks && e == cudaSuccess; ++c)
                e = cudaEventCreateWithFlags(&m->ev_agg[c], cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&m->ev_xdone, cudaEventDisableTiming);
            if (e != cudaSuccess) {
                rc = cuda_fail(e, "part_model_create: exchange stream");
                break;
            }
        }
        m->reserve_sms = (exchange == GAT_B200_EXCHANGE_P2P && chunks > 1) ? kDefaultReserve : 0;
        cudaError_t e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) rc = cuda_fail(e, "part_model_create");
    } while (0);
    if (rc) {
        // release what exists without the collective teardown
        m->comm = nullptr;
        gat_b200_part_model_destroy(m);
        return rc;
    }
    *out = m;
    return 0;
}

int gat_b200_part_model_rows(const gat_b200_part_model* m, uint64_t* lo, uint64_t* hi, uint64_t* edges) {
    clear_error();
    if (!m) return fail("part_model_rows: null handle");
    if (lo) *lo = m->lo;
    if (hi) *hi = m->hi;
    if (edges) *edges = m->e_loc;
    return 0;
}

int gat_b200_part_model_forward(gat_b200_part_model* m, const float* x, int x_on_host, float* logits,
                                int logits_on_host, void* stream) {
    clear_error();
    if (!m || (m->n_loc && (!x || !logits))) return fail("part_model_forward: null argument");
    cudaStream_t st = as_stream(stream);
    const uint64_t nl = m->n_loc;
    int launches = 0, rc = 0;
    mark(m, 0, st);
    const float* xin = x;
    if (x_on_host && nl) {
        GATB_CUDA(cudaMemcpyAsync(m->x_f32, x, nl * size_t(m->din) * 4, cudaMemcpyHostToDevice, st));
        xin = m->x_f32;
    }
    mark(m, 1, st);
    const bool p2p = m->exchange == GAT_B200_EXCHANGE_P2P;
    const gat_b200_layer* p0 = m->layers[0];
    if (p2p) {
        // layer-1 input rows into every rank's input table
        for (const auto& ch : m->chunks) {
            if (ch.b <= ch.a) continue;
            uint16_t* dst[kMaxWorld];
            for (int j = 0; j < m->world; ++j) dst[j] = static_cast<uint16_t*>(m->tab[j][6]) + ch.row0 * m->ld0;
            if ((rc = convert_scatter_launch(ch.b - ch.a, m->din, xin + ch.a * m->din, m->din, m->world, dst, m->ld0,
                                             st)))
                return rc;
            ++launches;
        }
        mark(m, 2, st);
        if ((rc = barrier(m, st, launches))) return rc;
        mark(m, 3, st);
        // every rank projects the whole input table: H, L and R of every row
        rc = projection_tc_launch(p0, m->L.table_rows, static_cast<const uint16_t*>(m->tab[m->rank][6]), m->ld0,
                                  m->H(m->rank, 0), m->ldh[0], nullptr, 0, m->left0, m->R(m->rank, 0), st, 0,
                                  nullptr, nullptr, 0);
        if (rc == GAT_B200_EUNSUPPORTED)
            return fail_code(rc, "part_model: layer outside the tensor-core projection (input or width > 256)");
        if (rc) return rc;
        ++launches;
    } else {
        if (nl) {
            if ((rc = convert_launch(nl, m->din, xin, m->din, m->x0, m->ld0, st))) return rc;
            ++launches;
        }
        mark(m, 2, st);
        mark(m, 3, st);
        const size_t hb = size_t(m->L.block_rows) * m->ldh[0] * 2, rb = size_t(m->L.block_rows) * m->heads[0] * 4;
        for (size_t c = 0; c < m->chunks.size(); ++c) {
            const auto& ch = m->chunks[c];
            if (ch.b > ch.a) {
                rc = projection_tc_launch(p0, ch.b - ch.a, m->x0 + ch.a * m->ld0, m->ld0,
                                          static_cast<uint16_t*>(m->h_send), m->ldh[0], nullptr, 0,
                                          m->left[0] + ch.a * m->heads[0], m->r_send, st, 0, nullptr, nullptr, 0);
                if (rc == GAT_B200_EUNSUPPORTED)
                    return fail_code(rc, "part_model: layer outside the tensor-core projection");
                if (rc) return rc;
                ++launches;
            }
            if ((rc = comm_all_gather_device(m->comm, m->h_send, static_cast<char*>(m->h_full[0]) + c * m->world * hb,
                                             hb, st)))
                return rc;
            if ((rc = comm_all_gather_device(m->comm, m->r_send,
                                             reinterpret_cast<char*>(m->r_full[0]) + c * m->world * rb, rb, st)))
                return rc;
        }
    }
    mark(m, 4, st);
    float* dst_logits = logits_on_host ? m->logits : logits;
    for (int l = 0; l < 3; ++l) {
        const gat_b200_layer* p = m->layers[l];
        const int K = p->heads, ldh = m->ldh[l];
        const bool last = l == 2;
        const void* htab = p2p ? static_cast<const void*>(m->H(m->rank, l)) : m->h_full[l];
        const float* rtab = p2p ? m->R(m->rank, l) : m->r_full[l];
        // overlap: chunk c's projection and exchange (stream xst, reserve_sms
        // SMs) run while chunk c+1 aggregates on the other SMs; the last
        // chunk's projection runs alone on every SM
        // x2 exchange: layer 1's aggregation stores each output row into every
        // rank's layer-2 input table; layer 2 then projects the whole table
        const bool x2 = p2p && m->x2x && l == 0;
        const bool overlap = !last && !x2 && p2p && m->reserve_sms > 0 && m->chunks.size() > 1;
        const size_t nch = m->chunks.size();
        for (size_t c = 0; c < nch; ++c) {
            const auto& ch = m->chunks[c];
            if (ch.g) {
                const bool table_left = p2p && (l == 0 || (l == 1 && m->x2x));
                const float* left = table_left ? m->left0 + ch.row0 * K : m->left[l & 1] + ch.a * K;
                void* o = last ? static_cast<void*>(dst_logits + ch.a * m->classes)
                               : x2 ? static_cast<void*>(static_cast<uint16_t*>(m->tab[m->rank][8]) + ch.row0 * m->ldx)
                                    : static_cast<void*>(static_cast<uint16_t*>(m->xs[l & 1]) + ch.a * m->ldx);
                uint16_t* peers[7];
                int np = 0;
                if (x2)
                    for (int j = 0; j < m->world; ++j)
                        if (j != m->rank) peers[np++] = static_cast<uint16_t*>(m->tab[j][8]) + ch.row0 * m->ldx;
                if ((rc = aggregate_dispatch_reserved(ch.g, K, p->dim, htab, GAT_B200_BF16, ldh, left, rtab, nullptr,
                                                      nullptr, 0, last ? 0 : 1, o, last ? 0 : 1,
                                                      last ? m->classes : m->ldx, nullptr, nullptr, st,
                                                      overlap ? m->reserve_sms : 0, np, peers)))
                    return rc;
                launches += 1 + (ch.g->n_hub ? 1 : 0);
            }
            if (c + 1 == nch) mark(m, 5 + 3 * l, st);
            if (last || x2) continue;
            if (overlap) {
                GATB_CUDA(cudaEventRecord(m->ev_agg[c], st));
                GATB_CUDA(cudaStreamWaitEvent(m->xst, m->ev_agg[c], 0));
                if ((rc = project_chunk(m, l + 1, ch, m->xst, launches, c + 1 == nch ? 0 : m->reserve_sms))) return rc;
            } else if ((rc = project_chunk(m, l + 1, ch, st, launches, 0))) {
                return rc;
            }
        }
        if (overlap) {
            GATB_CUDA(cudaEventRecord(m->ev_xdone, m->xst));
            GATB_CUDA(cudaStreamWaitEvent(st, m->ev_xdone, 0));
        }
        if (x2) {
            // every rank's layer-2 input rows have landed: project the whole table
            if ((rc = barrier(m, st, launches))) return rc;
            mark(m, 6, st);
            const gat_b200_layer* p1 = m->layers[1];
            rc = projection_tc_launch(p1, m->L.table_rows, static_cast<const uint16_t*>(m->tab[m->rank][8]), m->ldx,
                                      m->H(m->rank, 1), m->ldh[1], nullptr, 0, m->left0, m->R(m->rank, 1), st, 0,
                                      nullptr, nullptr, 0);
            if (rc == GAT_B200_EUNSUPPORTED)
                return fail_code(rc, "part_model: layer outside the tensor-core projection (input or width > 256)");
            if (rc) return rc;
            ++launches;
            mark(m, 7, st);
        } else if (!last) {
            mark(m, 6 + 3 * l, st);
            if ((rc = barrier(m, st, launches))) return rc;
            mark(m, 7 + 3 * l, st);
        }
    }
    if (logits_on_host && nl)
        GATB_CUDA(cudaMemcpyAsync(logits, m->logits, nl * size_t(m->classes) * 4, cudaMemcpyDeviceToHost, st));
    mark(m, 12, st);
    m->x2_last = p2p && m->x2x;
    m->launches_last = launches;
    ++m->forwards;
    if (logits_on_host) {
        GATB_CUDA(cudaStreamSynchronize(st));
        return device_check_errors();
    }
    return 0;
}

int gat_b200_part_model_forward_async(gat_b200_part_model* m, const float* x, float* logits, void* stream) {
    clear_error();
    if (!m || (m->n_loc && (!x || !logits))) return fail("part_model_forward_async: null argument");
    cudaStream_t st = as_stream(stream);
    const size_t xb = m->n_loc * size_t(m->din) * 4, lb = m->n_loc * size_t(m->classes) * 4;
    if (!m->up) {
        for (int b = 0; b < 2; ++b) {
            int rc;
            if ((rc = dalloc((void**)&m->ax[b], xb)) || (rc = dalloc((void**)&m->alog[b], lb))) return rc;
            GATB_CUDA(cudaEventCreateWithFlags(&m->ev_up[b], cudaEventDisableTiming));
            GATB_CUDA(cudaEventCreateWithFlags(&m->ev_done[b], cudaEventDisableTiming));
            GATB_CUDA(cudaEventCreateWithFlags(&m->ev_down[b], cudaEventDisableTiming));
        }
        GATB_CUDA(cudaStreamCreateWithFlags(&m->up, cudaStreamNonBlocking));
        GATB_CUDA(cudaStreamCreateWithFlags(&m->down, cudaStreamNonBlocking));
    }
    const int b = int(m->submitted & 1);
    if (m->submitted >= 2) GATB_CUDA(cudaStreamWaitEvent(m->up, m->ev_done[b], 0));
    if (xb) GATB_CUDA(cudaMemcpyAsync(m->ax[b], x, xb, cudaMemcpyHostToDevice, m->up));
    GATB_CUDA(cudaEventRecord(m->ev_up[b], m->up));
    GATB_CUDA(cudaStreamWaitEvent(st, m->ev_up[b], 0));
    if (m->submitted >= 2) GATB_CUDA(cudaStreamWaitEvent(st, m->ev_down[b], 0));
    int rc = gat_b200_part_model_forward(m, m->ax[b], 0, m->alog[b], 0, stream);
    if (rc) return rc;
    GATB_CUDA(cudaEventRecord(m->ev_done[b], st));
    GATB_CUDA(cudaStreamWaitEvent(m->down, m->ev_done[b], 0));
    if (lb) GATB_CUDA(cudaMemcpyAsync(logits, m->alog[b], lb, cudaMemcpyDeviceToHost, m->down));
    GATB_CUDA(cudaEventRecord(m->ev_down[b], m->down));
    ++m->submitted;
    return 0;
}

int gat_b200_part_model_join(gat_b200_part_model* m, void* stream) {
    clear_error();
    if (!m) return fail("part_model_join: null argument");
    if (!m->submitted) return 0;
    const int b = int((m->submitted - 1) & 1);
    GATB_CUDA(cudaStreamWaitEvent(as_stream(stream), m->ev_down[b], 0));
    return 0;
}

int gat_b200_part_model_enable_timing(gat_b200_part_model* m, int on) {
    clear_error();
    if (!m) return fail("part_model_enable_timing: null handle");
    m->timing = on != 0;
    m->forwards = 0;
    return 0;
}

int gat_b200_part_model_stage_times(gat_b200_part_model* m, float* ms) {
    clear_error();
    if (!m || !ms) return fail("part_model_stage_times: bad argument");
    if (!m->timing || !m->forwards) return fail("part_model_stage_times: no timed forward");
    GATB_CUDA(cudaEventSynchronize(m->ev[kEvents - 1]));
    for (int k = 0; k < GAT_B200_PART_STAGES; ++k) {
        float t = 0;
        GATB_CUDA(cudaEventElapsedTime(&t, m->ev[k], m->ev[k + 1]));
        ms[k] = t;
    }
    // With the layer-2 input exchange the barrier (events 5-6) precedes the
    // whole-table projection (events 6-7): report each under its own name.
    if (m->x2_last) std::swap(ms[5], ms[6]);
    return 0;
}

int gat_b200_part_model_launches(const gat_b200_part_model* m) { return m ? m->launches_last : 0; }

int gat_b200_part_model_set_layer2_exchange(gat_b200_part_model* m, int inputs) {
    clear_error();
    if (!m) return fail("part_model_set_layer2_exchange: null handle");
    if (inputs && (m->exchange != GAT_B200_EXCHANGE_P2P || m->heads[1] > m->heads[0]))
        return fail("part_model_set_layer2_exchange: needs the P2P exchange and layer 2 heads <= layer 1 heads");
    m->x2x = inputs != 0 && m->world > 1;
    return 0;
}

int gat_b200_part_model_set_overlap(gat_b200_part_model* m, int reserved_sms) {
    clear_error();
    if (!m) return fail("part_model_set_overlap: null handle");
    int dev = 0, sms = 0;
    GATB_CUDA(cudaGetDevice(&dev));
    GATB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if (reserved_sms < 0 || reserved_sms >= sms) return fail("part_model_set_overlap: reserved SMs out of range");
    m->reserve_sms = reserved_sms;
    return 0;
}

int gat_b200_part_model_destroy(gat_b200_part_model* m) {
    clear_error();
    if (!m) return 0;
    int rc = 0;
    cudaDeviceSynchronize();
    if (m->comm && !m->owned.empty()) rc = gat_b200_comm_barrier(m->comm);
    for (void* p : m->mapped) gat_b200_peer_close(p);
    for (void* p : m->owned) gat_b200_peer_free(p);
    for (auto& ch : m->chunks)
        if (ch.g) gat_b200_graph_destroy(ch.g);
    void* bufs[] = {m->x_f32, m->left0, m->left[0], m->left[1], m->xs[0], m->xs[1], m->logits, m->x0, m->h_send,
                    m->r_send, m->h_full[0], m->h_full[1], m->h_full[2], m->r_full[0], m->r_full[1], m->r_full[2],
                    m->ax[0], m->ax[1], m->alog[0], m->alog[1]};
    for (void* p : bufs)
        if (p) cudaFree(p);
    for (auto e : m->ev)
        if (e) cudaEventDestroy(e);
    for (auto e : m->ev_agg)
        if (e) cudaEventDestroy(e);
    if (m->ev_xdone) cudaEventDestroy(m->ev_xdone);
    if (m->xst) cudaStreamDestroy(m->xst);
    for (int b = 0; b < 2; ++b) {
        if (m->ev_up[b]) cudaEventDestroy(m->ev_up[b]);
        if (m->ev_done[b]) cudaEventDestroy(m->ev_done[b]);
        if (m->ev_down[b]) cudaEventDestroy(m->ev_down[b]);
    }
    if (m->up) cudaStreamDestroy(m->up);
    if (m->down) cudaStreamDestroy(m->down);
    delete m;
    return rc;
}

}  // extern "C"
