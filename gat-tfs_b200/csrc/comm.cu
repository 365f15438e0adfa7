// Communicator of the row-partitioned multi-GPU forward (one process per GPU
// on one NVLink/NVSwitch node): an NCCL communicator over the node's ranks.
//
// It serves three purposes: exchanging the CUDA IPC handles of the feature
// tables once at set-up (an all-gather), host-side barriers (set-up and
// teardown), and the NCCL exchange mode of the partitioned model (one
// all-gather of H and R per layer). The default exchange does not use it in
// the forward: the projection kernel stores into the peers' tables directly.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2 on first use), so the
// library carries no link-time NCCL dependency and shares the NCCL already
// loaded into the process when there is one (PyTorch's). The unique id comes
// from rank 0 (gat_b200_comm_id) and reaches the other ranks out of band (the
// caller's own channel, or a file: gat_b200_comm_create_file).
#include <dlfcn.h>
#include <nccl.h>
#include <unistd.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include <cuda_runtime.h>

#include "device.cuh"

namespace gatb {
namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
    std::string why;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char* e = dlerror();
            api.why = std::string("libnccl.so.2 could not be loaded: ") + (e ? e : "unknown");
            return;
        }
        auto sym = [&](const char* name) { return dlsym(h, name); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
        api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
        api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather && api.all_reduce &&
                 api.group_start && api.group_end && api.error_string;
        if (!api.ok) api.why = "libnccl.so.2 lacks an entry point this library needs";
    });
    return api;
}

int nccl_fail(ncclResult_t r, const char* what) {
    const char* s = nccl().error_string ? nccl().error_string(r) : "?";
    return fail_code(GAT_B200_ECUDA, std::string(what) + ": NCCL error " + std::to_string(int(r)) + " (" + s + ")");
}

}  // namespace
}  // namespace gatb

struct gat_b200_comm {
    int world = 1, rank = 0, device = 0;
    ncclComm_t nccl = nullptr;
    cudaStream_t st = nullptr;
    void* dbuf = nullptr;  // device scratch of the host-side collectives
    size_t dbuf_bytes = 0;
};

namespace gatb {

int comm_ensure_scratch(gat_b200_comm* c, size_t bytes) {
    if (c->dbuf_bytes >= bytes) return 0;
    if (c->dbuf) cudaFree(c->dbuf);
    c->dbuf = nullptr;
    c->dbuf_bytes = 0;
    GATB_CUDA(cudaMalloc(&c->dbuf, bytes));
    c->dbuf_bytes = bytes;
    return 0;
}

int comm_all_gather_device(gat_b200_comm* c, const void* send, void* recv, size_t bytes, void* stream) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (c->world == 1) {
        if (send != recv) GATB_CUDA(cudaMemcpyAsync(recv, send, bytes, cudaMemcpyDeviceToDevice, st));
        return 0;
    }
    ncclResult_t r = nccl().all_gather(send, recv, bytes, ncclUint8, c->nccl, st);
    if (r != ncclSuccess) return nccl_fail(r, "all_gather");
    return 0;
}

int comm_world(const gat_b200_comm* c) { return c->world; }
int comm_rank(const gat_b200_comm* c) { return c->rank; }
int comm_device(const gat_b200_comm* c) { return c->device; }

}  // namespace gatb

using namespace gatb;

extern "C" {

int gat_b200_comm_id(void* id) {
    clear_error();
    if (!id) return fail("comm_id: null output");
    NcclApi& api = nccl();
    if (!api.ok) return fail_code(GAT_B200_EUNSUPPORTED, "comm_id: " + api.why);
    ncclUniqueId u;
    ncclResult_t r = api.get_unique_id(&u);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    static_assert(sizeof(u) == GAT_B200_COMM_ID_BYTES, "NCCL unique id size");
    std::memcpy(id, &u, sizeof(u));
    return 0;
}

int gat_b200_comm_create(const void* id, int world, int rank, gat_b200_comm** out) {
    clear_error();
    if (!out) return fail("comm_create: null output");
    *out = nullptr;
    if (world < 1 || world > 8) return fail("comm_create: world size must be 1..8 (one NVLink node)");
    if (rank < 0 || rank >= world) return fail("comm_create: rank outside the world");
    if (world > 1 && !id) return fail("comm_create: null unique id");
    gat_b200_comm* c = new gat_b200_comm();
    c->world = world;
    c->rank = rank;
    cudaError_t e = cudaGetDevice(&c->device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e, "comm_create");
    }
    if (world > 1) {
        NcclApi& api = nccl();
        if (!api.ok) {
            cudaStreamDestroy(c->st);
            delete c;
            return fail_code(GAT_B200_EUNSUPPORTED, "comm_create: " + api.why);
        }
        // NVLink SHARP (NVLS) stays off unless the caller asked for it: the
        // default exchange does not use NCCL collectives in the forward.
        setenv("NCCL_NVLS_ENABLE", "0", 0);
        ncclUniqueId u;
        std::memcpy(&u, id, sizeof(u));
        ncclResult_t r = api.comm_init_rank(&c->nccl, world, u, rank);
        if (r != ncclSuccess) {
            cudaStreamDestroy(c->st);
            delete c;
            return nccl_fail(r, "ncclCommInitRank");
        }
    }
    *out = c;
    return 0;
}

int gat_b200_comm_create_file(const char* path, int world, int rank, int timeout_ms, gat_b200_comm** out) {
    clear_error();
    if (!out) return fail("comm_create_file: null output");
    *out = nullptr;
    if (!path || !*path) return fail("comm_create_file: null path");
    unsigned char id[GAT_B200_COMM_ID_BYTES] = {};
    if (world > 1) {
        if (rank == 0) {
            int rc = gat_b200_comm_id(id);
            if (rc) return rc;
            const std::string tmp = std::string(path) + ".tmp" + std::to_string(getpid());
            FILE* f = std::fopen(tmp.c_str(), "wb");
            if (!f) return fail_code(GAT_B200_EIO, std::string("comm_create_file: cannot write ") + tmp);
            const bool ok = std::fwrite(id, 1, sizeof(id), f) == sizeof(id);
            std::fclose(f);
            if (!ok || std::rename(tmp.c_str(), path) != 0)
                return fail_code(GAT_B200_EIO, std::string("comm_create_file: cannot publish ") + path);
        } else {
            const auto t0 = std::chrono::steady_clock::now();
            for (;;) {
                FILE* f = std::fopen(path, "rb");
                if (f) {
                    const size_t got = std::fread(id, 1, sizeof(id), f);
                    std::fclose(f);
                    if (got == sizeof(id)) break;
                }
                const auto waited =
                    std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
                if (waited.count() > timeout_ms)
                    return fail_code(GAT_B200_ETIMEOUT, std::string("comm_create_file: no unique id in ") + path +
                                                            " within " + std::to_string(timeout_ms) + " ms");
                std::this_thread::sleep_for(std::chrono::milliseconds(5));
            }
        }
    }
    return gat_b200_comm_create(id, world, rank, out);
}

int gat_b200_comm_info(const gat_b200_comm* c, int* world, int* rank) {
    clear_error();
    if (!c) return fail("comm_info: null handle");
    if (world) *world = c->world;
    if (rank) *rank = c->rank;
    return 0;
}

int gat_b200_comm_all_gather(gat_b200_comm* c, const void* send, void* recv, uint64_t bytes) {
    clear_error();
    if (!c || (bytes && (!send || !recv))) return fail("comm_all_gather: null argument");
    if (!bytes) return 0;
    int rc = comm_ensure_scratch(c, size_t(bytes) * (c->world + 1));
    if (rc) return rc;
    char* d = static_cast<char*>(c->dbuf);
    GATB_CUDA(cudaMemcpyAsync(d, send, bytes, cudaMemcpyHostToDevice, c->st));
    if ((rc = comm_all_gather_device(c, d, d + bytes, bytes, c->st))) return rc;
    GATB_CUDA(cudaMemcpyAsync(recv, d + bytes, size_t(bytes) * c->world, cudaMemcpyDeviceToHost, c->st));
    GATB_CUDA(cudaStreamSynchronize(c->st));
    return 0;
}

int gat_b200_comm_barrier(gat_b200_comm* c) {
    clear_error();
    if (!c) return fail("comm_barrier: null handle");
    if (c->world == 1) return 0;
    int rc = comm_ensure_scratch(c, 64);
    if (rc) return rc;
    ncclResult_t r = nccl().all_reduce(c->dbuf, c->dbuf, 1, ncclInt32, ncclSum, c->nccl, c->st);
    if (r != ncclSuccess) return nccl_fail(r, "comm_barrier");
    GATB_CUDA(cudaStreamSynchronize(c->st));
    return 0;
}

int gat_b200_comm_destroy(gat_b200_comm* c) {
    clear_error();
    if (!c) return 0;
    if (c->nccl) nccl().comm_destroy(c->nccl);
    if (c->dbuf) cudaFree(c->dbuf);
    if (c->st) cudaStreamDestroy(c->st);
    delete c;
    return 0;
}

}  // extern "C"
