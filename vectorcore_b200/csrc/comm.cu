// comm.cu -- cross-GPU exchange of shard partials over NCCL (NVLink 5 /
// NVSwitch on a B200 box).
//
// Tensors shard along the leading axis, one process per GPU. Elementwise work
// needs no communication; a reduction over the sharded axis computes a
// per-rank partial (vc_cuda_reduce_axis_partial and friends), all-gathers the
// partials -- at most a few hundred KB, so the exchange is latency-bound -- and
// every rank combines them in rank order 0..R-1 (vc_cuda_combine_partials),
// so the result does not depend on NCCL's ring or tree order. An all-reduce is
// deliberately not used: its summation order is NCCL's choice.
//
// NCCL is loaded at run time (dlopen "libnccl.so.2"): in a process where
// torch already loaded its NCCL, the same library is reused. The communicator
// is created non-blocking (ncclConfig_t.blocking = 0) and every wait on it has
// a deadline; on timeout the communicator is aborted (ncclCommAbort also
// stops NCCL kernels still waiting for a peer) and the call fails with
// VC_ERR_TIMEOUT, so a rank that died cannot hang the others forever.
#include "vc_internal.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

namespace vc {
namespace {

struct NcclApi {
    void* handle{nullptr};
    ncclResult_t (*GetUniqueId)(ncclUniqueId*){nullptr};
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*){nullptr};
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*){nullptr};
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t){nullptr};
    ncclResult_t (*GroupStart)(){nullptr};
    ncclResult_t (*GroupEnd)(){nullptr};
    ncclResult_t (*CommAbort)(ncclComm_t){nullptr};
    ncclResult_t (*CommDestroy)(ncclComm_t){nullptr};
    const char* (*GetErrorString)(ncclResult_t){nullptr};
    ncclResult_t (*GetVersion)(int*){nullptr};
};

std::mutex g_comm_mutex;
NcclApi g_nccl;
ncclComm_t g_comm = nullptr;
int g_ranks = 0, g_rank = -1;
int g_timeout_ms = 60000;

template <typename F>
void bind(F& fn, const char* name) {
    fn = reinterpret_cast<F>(dlsym(g_nccl.handle, name));
    if (!fn) fail(VC_ERR_RUNTIME, std::string("NCCL symbol missing: ") + name);
}

void load_nccl() {
    if (g_nccl.handle) return;
    const char* override_path = std::getenv("VC_CUDA_NCCL_LIBRARY");
    void* h = dlopen(override_path ? override_path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) fail(VC_ERR_RUNTIME, std::string("cannot load NCCL (libnccl.so.2): ") + dlerror());
    g_nccl.handle = h;
    bind(g_nccl.GetUniqueId, "ncclGetUniqueId");
    bind(g_nccl.CommInitRankConfig, "ncclCommInitRankConfig");
    bind(g_nccl.CommGetAsyncError, "ncclCommGetAsyncError");
    bind(g_nccl.AllGather, "ncclAllGather");
    bind(g_nccl.GroupStart, "ncclGroupStart");
    bind(g_nccl.GroupEnd, "ncclGroupEnd");
    bind(g_nccl.CommAbort, "ncclCommAbort");
    bind(g_nccl.CommDestroy, "ncclCommDestroy");
    bind(g_nccl.GetErrorString, "ncclGetErrorString");
    bind(g_nccl.GetVersion, "ncclGetVersion");
}

std::string nccl_error(ncclResult_t r) { return g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "NCCL error"; }

void abort_comm_locked() {
    if (g_comm) g_nccl.CommAbort(g_comm);
    g_comm = nullptr;
    g_ranks = 0;
    g_rank = -1;
}

// Wait until the communicator leaves ncclInProgress; abort it on error or at
// the deadline. An enqueue normally completes within microseconds: the first
// polls only yield the thread, later ones sleep 50 us.
void wait_comm_ready_locked(const char* what) {
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(g_timeout_ms);
    for (int polls = 0;; ++polls) {
        ncclResult_t state = ncclSuccess;
        const ncclResult_t r = g_nccl.CommGetAsyncError(g_comm, &state);
        if (r != ncclSuccess) state = r;
        if (state == ncclSuccess) return;
        if (state != ncclInProgress) {
            abort_comm_locked();
            fail(VC_ERR_RUNTIME, std::string(what) + ": " + nccl_error(state));
        }
        if (std::chrono::steady_clock::now() > deadline) {
            abort_comm_locked();
            fail(VC_ERR_TIMEOUT, std::string(what) + " did not finish within " + std::to_string(g_timeout_ms) +
                                     " ms; the communicator was aborted");
        }
        if (polls < 4096)
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // namespace
}  // namespace vc

using namespace vc;

extern "C" {

vc_status vc_cuda_comm_unique_id(void* id, size_t bytes) {
    VC_API_BEGIN
    if (!id || bytes < sizeof(ncclUniqueId)) fail(VC_ERR_INVALID, "comm_unique_id: buffer smaller than 128 bytes");
    std::lock_guard<std::mutex> lock(g_comm_mutex);
    load_nccl();
    ncclUniqueId uid;
    const ncclResult_t r = g_nccl.GetUniqueId(&uid);
    if (r != ncclSuccess) fail(VC_ERR_RUNTIME, "ncclGetUniqueId: " + nccl_error(r));
    std::memcpy(id, &uid, sizeof uid);
    VC_API_END
}

vc_status vc_cuda_comm_init(int nranks, int rank, const void* id, size_t bytes, int timeout_ms) {
    VC_API_BEGIN
    ensure_init();
    if (nranks < 1 || rank < 0 || rank >= nranks) fail(VC_ERR_OUT_OF_RANGE, "comm_init: bad rank / world size");
    if (!id || bytes < sizeof(ncclUniqueId)) fail(VC_ERR_INVALID, "comm_init: unique id must be 128 bytes");
    std::lock_guard<std::mutex> lock(g_comm_mutex);
    load_nccl();
    if (g_comm) fail(VC_ERR_INVALID, "comm_init: a communicator is already open (vc_cuda_comm_destroy first)");
    if (timeout_ms > 0) g_timeout_ms = timeout_ms;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof uid);
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    const ncclResult_t r = g_nccl.CommInitRankConfig(&g_comm, nranks, uid, rank, &config);
    if (r != ncclSuccess && r != ncclInProgress) {
        if (g_comm) g_nccl.CommAbort(g_comm);
        g_comm = nullptr;
        fail(VC_ERR_RUNTIME, "ncclCommInitRankConfig: " + nccl_error(r));
    }
    g_ranks = nranks;
    g_rank = rank;
    wait_comm_ready_locked("NCCL communicator initialisation");
    VC_API_END
}

vc_status vc_cuda_comm_allgather(const void* send, void* recv, size_t bytes_per_rank) {
    VC_API_BEGIN
    ensure_init();
    std::lock_guard<std::mutex> lock(g_comm_mutex);
    if (!g_comm) fail(VC_ERR_INVALID, "comm_allgather: no communicator (vc_cuda_comm_init first)");
    if (!bytes_per_rank) return VC_OK;
    if (!send || !recv) fail(VC_ERR_INVALID, "comm_allgather: null buffer");
    const ncclResult_t r = g_nccl.AllGather(send, recv, bytes_per_rank, ncclInt8, g_comm, stream());
    if (r != ncclSuccess && r != ncclInProgress) {
        abort_comm_locked();
        fail(VC_ERR_RUNTIME, "ncclAllGather: " + nccl_error(r));
    }
    wait_comm_ready_locked("enqueueing ncclAllGather");
    VC_API_END
}

vc_status vc_cuda_comm_allgather_group(const void* const* sends, void* const* recvs, const size_t* bytes_per_rank,
                                       int count) {
    VC_API_BEGIN
    ensure_init();
    std::lock_guard<std::mutex> lock(g_comm_mutex);
    if (!g_comm) fail(VC_ERR_INVALID, "comm_allgather_group: no communicator (vc_cuda_comm_init first)");
    if (count < 0 || (count > 0 && (!sends || !recvs || !bytes_per_rank)))
        fail(VC_ERR_INVALID, "comm_allgather_group: bad arguments");
    for (int i = 0; i < count; ++i)
        if (bytes_per_rank[i] && (!sends[i] || !recvs[i])) fail(VC_ERR_INVALID, "comm_allgather_group: null buffer");
    ncclResult_t r = g_nccl.GroupStart();
    for (int i = 0; i < count && (r == ncclSuccess || r == ncclInProgress); ++i)
        if (bytes_per_rank[i]) r = g_nccl.AllGather(sends[i], recvs[i], bytes_per_rank[i], ncclInt8, g_comm, stream());
    const ncclResult_t e = g_nccl.GroupEnd();  // always closes the group
    if (r == ncclSuccess || r == ncclInProgress) r = e;
    if (r != ncclSuccess && r != ncclInProgress) {
        abort_comm_locked();
        fail(VC_ERR_RUNTIME, "grouped ncclAllGather: " + nccl_error(r));
    }
    wait_comm_ready_locked("enqueueing the grouped ncclAllGather");
    VC_API_END
}

vc_status vc_cuda_comm_synchronize(int timeout_ms) {
    VC_API_BEGIN
    ensure_init();
    const int limit = timeout_ms > 0 ? timeout_ms : g_timeout_ms;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(limit);
    for (;;) {
        const cudaError_t q = cudaStreamQuery(stream());
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) VC_CUDA(q);
        {
            std::lock_guard<std::mutex> lock(g_comm_mutex);
            if (g_comm) {
                ncclResult_t state = ncclSuccess;
                g_nccl.CommGetAsyncError(g_comm, &state);
                if (state != ncclSuccess && state != ncclInProgress) {
                    abort_comm_locked();
                    fail(VC_ERR_RUNTIME, "NCCL reported: " + nccl_error(state));
                }
            }
        }
        if (std::chrono::steady_clock::now() > deadline) {
            std::lock_guard<std::mutex> lock(g_comm_mutex);
            abort_comm_locked();
            fail(VC_ERR_TIMEOUT, "device work did not finish within " + std::to_string(limit) +
                                     " ms (a peer may have left); the communicator was aborted");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    VC_API_END
}

vc_status vc_cuda_comm_destroy(void) {
    VC_API_BEGIN
    std::lock_guard<std::mutex> lock(g_comm_mutex);
    if (!g_comm) return VC_OK;
    const ncclResult_t r = g_nccl.CommDestroy(g_comm);
    g_comm = nullptr;
    g_ranks = 0;
    g_rank = -1;
    if (r != ncclSuccess && r != ncclInProgress) fail(VC_ERR_RUNTIME, "ncclCommDestroy: " + nccl_error(r));
    VC_API_END
}

int vc_cuda_comm_size(void) { return g_ranks; }
int vc_cuda_comm_rank(void) { return g_rank; }

}  // extern "C"
