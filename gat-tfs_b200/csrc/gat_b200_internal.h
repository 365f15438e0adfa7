// Internal declarations shared by the host (.cpp) and device (.cu) sources of
// libgat_b200.so. Not part of the C-ABI (that is include/gat_b200.h).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>

#include "../../include/gat_b200.h"

namespace gatb {

// Thread-local last error (gat_b200_last_error). fail() records the message and
// returns GAT_B200_EINVAL; fail_code() lets the caller choose the status.
int fail(const std::string& msg);
int fail_code(int code, const std::string& msg);
void clear_error();

// Row stride (in elements) used for every device feature buffer of `width`
// columns: rows start on 16-byte boundaries (TMA and 128-bit gathers need it)
// and the padding columns are kept at zero.
inline int padded_ld(int width, int elem_bytes) {
    int per16 = 16 / elem_bytes;
    return (width + per16 - 1) / per16 * per16;
}

// Synthetic inputs (synth.cpp).
int synth_uniform_graph(uint64_t n, uint32_t sources, uint64_t seed, uint64_t* row, uint32_t* col);
int synth_powerlaw_graph(uint64_t n, uint64_t e_target, uint64_t max_degree, double gamma,
                         uint64_t seed, uint64_t* row, uint32_t* col);
int synth_powerlaw_rows(uint64_t n, uint64_t e_target, uint64_t max_degree, double gamma, uint64_t seed,
                        uint64_t r_lo, uint64_t r_hi, uint64_t* row, uint32_t* col);
int synth_normal(uint64_t count, double scale, uint64_t seed, uint64_t stream, float* out, uint64_t offset);
int synth_uniform(uint64_t count, double lo, double hi, uint64_t seed, uint64_t stream, float* out);

// Communicator of the multi-GPU forward (comm.cpp). comm_all_gather_device:
// every rank's `bytes` device bytes, rank-ordered, into recv (device) on
// `stream`; the NCCL all-gather for world > 1.
int comm_all_gather_device(gat_b200_comm* c, const void* send, void* recv, size_t bytes, void* stream);
int comm_world(const gat_b200_comm* c);
int comm_rank(const gat_b200_comm* c);
int comm_device(const gat_b200_comm* c);

}  // namespace gatb
