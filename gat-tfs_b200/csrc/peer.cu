// Peer memory and the cross-GPU barrier of the row-partitioned multi-GPU
// forward (one process per GPU on one NVLink/NVSwitch node).
//
// Every rank allocates its feature tables and one flag array with
// gat_b200_peer_alloc and hands the IPC handles to the other ranks, which map
// them with gat_b200_peer_open. The projection kernel then stores each tile of
// H and R into every rank's table (gat_b200_projection_scatter), and
// gat_b200_peer_barrier orders those stores before any rank's aggregation reads
// its table:
//
//   rank k, epoch e:  fence.sys; for every peer j: st.release.sys flags_j[k] = e
//                     for every peer j: wait until ld.acquire.sys flags_k[j] >= e
//
// The barrier kernel runs after the projection kernel on the same stream, so
// the projection's stores (to local and peer memory) precede the release; the
// aggregation kernel runs after the barrier, so it sees every peer's stores
// once the acquires returned. Waits are bounded (~1 s of clock64 cycles): a
// peer that never arrives sets g_peer_error (GAT_B200_ETIMEOUT on the next
// check) and the kernel returns.
#include <cstring>

#include "device.cuh"

namespace gatb {

__device__ unsigned g_peer_error = 0;

namespace {

constexpr int kMaxRanks = 8;

struct FlagSet {
    uint32_t* f[kMaxRanks];  // f[j] = rank j's flag array (mapped); f[rank] own
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void peer_barrier_kernel(FlagSet fs, int world, int rank, uint32_t epoch) {
    const int j = threadIdx.x;
    const bool peer = j < world && j != rank;
    if (peer) {
        __threadfence_system();
        st_release_sys(fs.f[j] + rank, epoch);
    }
    if (!peer) return;
    const uint32_t* mine = fs.f[rank] + j;
    const long long start = clock64();
    for (uint32_t it = 0;; ++it) {
        if (int(ld_acquire_sys(mine) - epoch) >= 0) break;
        if ((it & 15) == 15) {
            __nanosleep(128);
            if (clock64() - start > (1ll << 31)) {
                atomicOr(&g_peer_error, 1u);
                break;
            }
        }
    }
}

}  // namespace

int peer_barrier_launch(void* const* flags, int world, int rank, uint32_t epoch, cudaStream_t st) {
    if (!flags) return fail("peer_barrier: null flag table");
    if (world < 1 || world > kMaxRanks) return fail("peer_barrier: world size must be 1..8");
    if (rank < 0 || rank >= world) return fail("peer_barrier: rank outside the world");
    if (world == 1) return 0;
    FlagSet fs{};
    for (int j = 0; j < world; ++j) {
        if (!flags[j]) return fail("peer_barrier: null flag array");
        fs.f[j] = static_cast<uint32_t*>(flags[j]);
    }
    peer_barrier_kernel<<<1, 32, 0, st>>>(fs, world, rank, epoch);
    GATB_LAUNCH("peer barrier kernel");
    return 0;
}

int peer_check_error() {
    unsigned e = 0;
    GATB_CUDA(cudaMemcpyFromSymbol(&e, g_peer_error, sizeof(e)));
    if (e) {
        unsigned z = 0;
        cudaMemcpyToSymbol(g_peer_error, &z, sizeof(z));
        return fail_code(GAT_B200_ETIMEOUT, "peer barrier: a peer did not arrive within the bounded wait");
    }
    return 0;
}

}  // namespace gatb

extern "C" {

int gat_b200_peer_alloc(uint64_t bytes, void** ptr, void* handle) {
    gatb::clear_error();
    if (!ptr || !handle) return gatb::fail("peer_alloc: null output");
    *ptr = nullptr;
    void* p = nullptr;
    GATB_CUDA(cudaMalloc(&p, bytes ? bytes : 16));
    cudaError_t e = cudaMemset(p, 0, bytes ? bytes : 16);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return gatb::cuda_fail(e, "peer_alloc");
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == GAT_B200_PEER_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return 0;
}

int gat_b200_peer_open(const void* handle, void** ptr) {
    gatb::clear_error();
    if (!ptr || !handle) return gatb::fail("peer_open: null argument");
    *ptr = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    GATB_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return 0;
}

int gat_b200_peer_close(void* ptr) {
    gatb::clear_error();
    if (!ptr) return 0;
    GATB_CUDA(cudaIpcCloseMemHandle(ptr));
    return 0;
}

int gat_b200_peer_free(void* ptr) {
    gatb::clear_error();
    if (!ptr) return 0;
    GATB_CUDA(cudaFree(ptr));
    return 0;
}

int gat_b200_copy_to_peers(const void* src, void* const* dst, int ndst, uint64_t bytes, void* const* streams) {
    gatb::clear_error();
    if (ndst < 0 || ndst > 7) return gatb::fail("copy_to_peers: ndst must be 0..7");
    if (ndst && (!src || !dst || !streams)) return gatb::fail("copy_to_peers: null argument");
    for (int j = 0; j < ndst; ++j) {
        if (!dst[j]) return gatb::fail("copy_to_peers: null destination");
        GATB_CUDA(cudaMemcpyAsync(dst[j], src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(streams[j])));
    }
    return 0;
}

int gat_b200_peer_barrier(void* const* flags, int world, int rank, uint32_t epoch, void* stream) {
    gatb::clear_error();
    return gatb::peer_barrier_launch(flags, world, rank, epoch, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
