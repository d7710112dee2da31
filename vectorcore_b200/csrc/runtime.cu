// runtime.cu -- device selection, the enqueue stream, the stream-ordered
// size-class buffer pool, error reporting and the memory entry points.
//
// Design (B200-first, mirroring what the Metal host does in
// src/metal/metal_backend.mm):
//  * one process drives one GPU; all work goes to one CUDA stream, so work
//    executes in submission order (Metal: one serial command queue, :517-560);
//  * buffers come from a size-class pool (256 B minimum, powers of two up to
//    4 MiB, then 1 MiB steps -- the same classes as bucket_bytes, :487-499).
//    A freed block is reusable immediately: its next user is enqueued after
//    every earlier user on the same stream, which is the ordering Metal needs a
//    completion handler for (:184-191, :531-554);
//  * the pool keeps at most VC_CUDA_POOL_LIMIT bytes cached (default 96 GiB,
//    sized for 180 GB of HBM3e); on cudaMalloc failure it returns every cached
//    block to the driver and retries once;
//  * kernels that detect a problem set bits in a device error word; blocking
//    calls read and clear it and report the failure (Metal: async_error_,
//    :428-443).
#include "vc_internal.cuh"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <condition_variable>
#include <map>
#include <mutex>
#include <thread>
#include <unordered_map>
#include <vector>

namespace vc {

namespace {

thread_local std::string t_last_error;

// A captured CUDA graph and the pool blocks it owns. Every block allocated
// while the graph is being captured belongs to it: freed during the capture,
// a block may serve a later allocation of the same capture (stream order);
// freed after it, the block stays reserved -- the graph's replays still use
// it -- until the graph is destroyed.
struct GraphRecord {
    cudaGraph_t graph{nullptr};
    cudaGraphExec_t exec{nullptr};
    std::map<std::size_t, std::vector<void*>> capture_free;  // reusable during capture
    std::vector<std::pair<void*, std::size_t>> reserved;      // (block, bucket) freed after capture
    std::size_t kernels{0};
};

struct Pool {
    std::mutex mutex;
    GraphRecord* capturing{nullptr};
    std::unordered_map<void*, GraphRecord*> owner;           // block -> graph that owns it
    std::map<std::size_t, std::vector<void*>> free_blocks;  // bucket bytes -> blocks
    std::unordered_map<void*, std::size_t> live;             // block -> bucket bytes
    std::size_t cached_bytes{0};
    std::size_t in_use_bytes{0};
    std::size_t hits{0};
    std::size_t misses{0};
    std::size_t limit{96ull << 30};
};

// Asynchronous host transfers: one copy stream per direction, completion
// tickets backed by a ring of events, and the device ranges of transfers that
// may still be in flight (so a freed pool block is not reused under them).
constexpr unsigned kTicketRing = 1024;

struct Transfers {
    std::mutex mutex;
    cudaStream_t h2d{nullptr}, d2h{nullptr};
    cudaEvent_t order[2]{};                 // compute -> copy ordering, per direction
    cudaEvent_t ring[kTicketRing]{};        // completion of ticket t in ring[t % kTicketRing]
    unsigned long long next{1};             // the next ticket
    struct Pending {
        const char* lo;
        const char* hi;
        unsigned long long ticket;
    };
    std::vector<Pending> pending;
};

// Pageable host transfers through page-locked staging. The driver's own path
// for pageable memory runs far below the link (10-17 GB/s against 52-56 GB/s
// page-locked on the B200 hosts measured), so large copies go in kStageChunk
// pieces through two page-locked buffers: host threads copy piece k+1 while
// the DMA of piece k runs.
constexpr std::size_t kStageChunk = 32u << 20;
constexpr std::size_t kStageMin = 8u << 20;  // smaller copies take the driver's path

// memcpy split over a few persistent host threads and the caller.
class CopyWorkers {
public:
    explicit CopyWorkers(unsigned n) {
        for (unsigned i = 0; i < n; ++i) {
            std::thread t([this, i] { loop(i); });
            t.detach();  // parked on the condition variable for the process lifetime
            ++workers_;
        }
    }
    void copy(void* dst, const void* src, std::size_t len) {
        {
            std::lock_guard<std::mutex> lock(m_);
            dst_ = static_cast<char*>(dst);
            src_ = static_cast<const char*>(src);
            len_ = len;
            piece_ = (len / (workers_ + 1) + 4095) & ~static_cast<std::size_t>(4095);
            pending_ = workers_;
            ++generation_;
        }
        work_.notify_all();
        part(workers_);
        std::unique_lock<std::mutex> lock(m_);
        done_.wait(lock, [&] { return pending_ == 0; });
    }

private:
    void part(unsigned i) {
        const std::size_t lo = std::min(len_, i * piece_);
        const std::size_t hi = i == workers_ ? len_ : std::min(len_, (i + 1) * piece_);
        if (hi > lo) std::memcpy(dst_ + lo, src_ + lo, hi - lo);
    }
    void loop(unsigned i) {
        unsigned long long seen = 0;
        std::unique_lock<std::mutex> lock(m_);
        for (;;) {
            work_.wait(lock, [&] { return generation_ != seen; });
            seen = generation_;
            lock.unlock();
            part(i);
            lock.lock();
            if (--pending_ == 0) done_.notify_one();
        }
    }
    unsigned workers_{0};
    std::mutex m_;
    std::condition_variable work_, done_;
    char* dst_{nullptr};
    const char* src_{nullptr};
    std::size_t len_{0}, piece_{0}, pending_{0};
    unsigned long long generation_{0};
};

struct Staging {
    std::mutex mutex;
    void* buf[2]{};
    cudaEvent_t done[2]{};  // the last DMA that used each buffer
    CopyWorkers* workers{nullptr};
};

struct State {
    std::mutex init_mutex;
    bool ready{false};
    int device{-1};
    int sms{148};
    cudaStream_t own_stream{nullptr};
    cudaStream_t stream{nullptr};
    cudaStream_t side{nullptr};  // second compute stream (SideStream), created on first use
    unsigned* counters{nullptr};
    unsigned* error_word{nullptr};
    char name[256]{};
    Pool pool;
    Transfers xfer;
    Staging staging;
};

State& state() {
    static State* s = new State();  // never destroyed: tensors may outlive static teardown
    return *s;
}

std::size_t bucket_bytes(std::size_t bytes) {
    constexpr std::size_t kMin = 256, kPow2Limit = 4u << 20, kStep = 1u << 20;
    if (bytes <= kMin) return kMin;
    if (bytes <= kPow2Limit) {
        std::size_t b = kMin;
        while (b < bytes) b <<= 1;
        return b;
    }
    return (bytes + kStep - 1) / kStep * kStep;
}

void release_cached_locked(Pool& pool) {
    for (auto& entry : pool.free_blocks)
        for (void* p : entry.second) cudaFree(p);
    pool.free_blocks.clear();
    pool.cached_bytes = 0;
}

// A ticket whose ring slot was recorded again is known complete: the slot's
// earlier event is waited for before it is reused.
bool ticket_retired(const Transfers& x, unsigned long long t) { return t + kTicketRing < x.next; }

void prune_transfers_locked(Transfers& x) {
    std::size_t k = 0;
    for (const auto& p : x.pending) {
        const bool done = ticket_retired(x, p.ticket) || cudaEventQuery(x.ring[p.ticket % kTicketRing]) == cudaSuccess;
        if (!done) x.pending[k++] = p;
    }
    cudaGetLastError();  // cudaErrorNotReady from the queries
    x.pending.resize(k);
}

}  // namespace

void set_last_error(const std::string& message) { t_last_error = message; }

void fail(vc_status status, const std::string& message) { throw Error(status, message); }

void check_cuda(cudaError_t err, const char* what) {
    if (err == cudaSuccess) return;
    const vc_status st = err == cudaErrorMemoryAllocation ? VC_ERR_OOM : VC_ERR_RUNTIME;
    throw Error(st, std::string("CUDA error in ") + what + ": " + cudaGetErrorString(err));
}

void check_launch(const char* what) {
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess)
        throw Error(VC_ERR_RUNTIME, std::string("kernel launch failed (") + what + "): " +
                                        cudaGetErrorString(err));
}

static void init_device(int device) {
    State& s = state();
    std::lock_guard<std::mutex> lock(s.init_mutex);
    if (s.ready) {
        if (device == s.device) return;
        fail(VC_ERR_INVALID, "the VectorCore CUDA device is already bound to GPU " +
                                 std::to_string(s.device) + " in this process");
    }
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        cudaGetLastError();
        fail(VC_ERR_RUNTIME, "no CUDA device is available");
    }
    if (device < 0 || device >= count) fail(VC_ERR_OUT_OF_RANGE, "CUDA device index out of range");
    cudaDeviceProp prop{};
    VC_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        fail(VC_ERR_RUNTIME, std::string("the VectorCore CUDA device is built for sm_100a (B200); "
                                         "found ") + prop.name);
    VC_CUDA(cudaSetDevice(device));
    VC_CUDA(cudaStreamCreateWithFlags(&s.own_stream, cudaStreamNonBlocking));
    s.stream = s.own_stream;
    s.sms = prop.multiProcessorCount;
    std::snprintf(s.name, sizeof s.name, "%s", prop.name);
    VC_CUDA(cudaMalloc(&s.counters, kCounterSlots * sizeof(unsigned)));
    VC_CUDA(cudaMemset(s.counters, 0, kCounterSlots * sizeof(unsigned)));
    VC_CUDA(cudaMalloc(&s.error_word, sizeof(unsigned)));
    VC_CUDA(cudaMemset(s.error_word, 0, sizeof(unsigned)));
    if (const char* lim = std::getenv("VC_CUDA_POOL_LIMIT")) s.pool.limit = std::strtoull(lim, nullptr, 10);
    s.device = device;
    s.ready = true;
}

void ensure_init() {
    if (!state().ready) init_device(0);
    // Work may be issued from any host thread: make sure it targets our GPU.
    int current = -1;
    if (cudaGetDevice(&current) == cudaSuccess && current != state().device) VC_CUDA(cudaSetDevice(state().device));
}

bool initialized() { return state().ready; }
int bound_device() { return state().ready ? state().device : -1; }

namespace {
// Work issued by this host thread inside a SideStream goes to the side
// stream, and the scratch it frees waits for the join.
thread_local cudaStream_t t_stream_override = nullptr;
thread_local std::vector<void*>* t_deferred_frees = nullptr;
}  // namespace

cudaStream_t stream() { return t_stream_override ? t_stream_override : state().stream; }
int sm_count() { return state().sms; }
unsigned* counters() { return state().counters; }

unsigned* stream_tickets() {
    static std::mutex m;
    static std::unordered_map<cudaStream_t, unsigned> slots;
    const cudaStream_t st = stream();
    std::lock_guard<std::mutex> lock(m);
    auto it = slots.find(st);
    if (it == slots.end()) {
        const std::size_t next = slots.size();
        if ((next + 1) * kPerStreamTickets > kCounterSlots)
            fail(VC_ERR_RUNTIME, "too many distinct streams for the per-stream ticket counters");
        it = slots.emplace(st, static_cast<unsigned>(next)).first;
    }
    return state().counters + static_cast<std::size_t>(it->second) * kPerStreamTickets;
}
unsigned* device_error_word() { return state().error_word; }

static void* pool_alloc(std::size_t bytes) {
    ensure_init();
    State& s = state();
    Pool& pool = s.pool;
    const std::size_t b = bucket_bytes(bytes ? bytes : 1);
    GraphRecord* graph = nullptr;
    {
        std::lock_guard<std::mutex> lock(pool.mutex);
        graph = pool.capturing;
        if (graph) {
            auto ct = graph->capture_free.find(b);
            if (ct != graph->capture_free.end() && !ct->second.empty()) {
                void* p = ct->second.back();
                ct->second.pop_back();
                pool.in_use_bytes += b;
                pool.live[p] = b;
                ++pool.hits;
                return p;
            }
        }
        auto it = pool.free_blocks.find(b);
        if (it != pool.free_blocks.end() && !it->second.empty()) {
            void* p = it->second.back();
            it->second.pop_back();
            pool.cached_bytes -= b;
            pool.in_use_bytes += b;
            pool.live[p] = b;
            if (graph) pool.owner[p] = graph;
            ++pool.hits;
            return p;
        }
        ++pool.misses;
    }
    if (std::getenv("VC_CUDA_FAKE_OOM")) fail(VC_ERR_OOM, "device allocation failed (VC_CUDA_FAKE_OOM)");
    void* p = nullptr;
    cudaError_t err = cudaMalloc(&p, b);
    if (err == cudaErrorMemoryAllocation && !graph) {
        cudaGetLastError();
        // Cached blocks may still be referenced by enqueued work: finish it,
        // hand the cache back to the driver and retry once.
        VC_CUDA(cudaStreamSynchronize(s.stream));
        {
            std::lock_guard<std::mutex> lock(pool.mutex);
            release_cached_locked(pool);
        }
        err = cudaMalloc(&p, b);
    }
    if (err != cudaSuccess) {
        cudaGetLastError();
        fail(VC_ERR_OOM, "device allocation of " + std::to_string(b) + " bytes failed: " +
                             cudaGetErrorString(err));
    }
    std::lock_guard<std::mutex> lock(pool.mutex);
    pool.in_use_bytes += b;
    pool.live[p] = b;
    if (graph) pool.owner[p] = graph;
    return p;
}

static void pool_free(void* p) {
    if (!p) return;
    State& s = state();
    Pool& pool = s.pool;
    std::lock_guard<std::mutex> lock(pool.mutex);
    auto it = pool.live.find(p);
    if (it == pool.live.end()) fail(VC_ERR_INVALID, "vc_cuda_free: pointer was not allocated by the pool");
    const std::size_t b = it->second;
    pool.live.erase(it);
    pool.in_use_bytes -= b;
    {
        // The next user of the block is ordered on the compute stream: make
        // that stream wait for transfers still reading or writing it.
        Transfers& x = s.xfer;
        std::lock_guard<std::mutex> xlock(x.mutex);
        if (!x.pending.empty()) {
            prune_transfers_locked(x);
            const char* lo = static_cast<const char*>(p);
            const char* hi = lo + b;
            for (const auto& q : x.pending)
                if (q.lo < hi && lo < q.hi) VC_CUDA(cudaStreamWaitEvent(s.stream, x.ring[q.ticket % kTicketRing], 0));
        }
    }
    auto own = pool.owner.find(p);
    if (own != pool.owner.end()) {
        GraphRecord* g = own->second;
        if (g == pool.capturing) g->capture_free[b].push_back(p);
        else g->reserved.emplace_back(p, b);
        return;
    }
    if (pool.cached_bytes + b > pool.limit) {
        // Over the cache limit: let the driver have it (cudaFree waits for
        // the device, so enqueued users finish first).
        cudaFree(p);
        return;
    }
    pool.free_blocks[b].push_back(p);
    pool.cached_bytes += b;
}

Scratch::Scratch(std::size_t bytes) : ptr_(pool_alloc(bytes)) {}
Scratch::~Scratch() {
    try {
        if (t_deferred_frees && ptr_) t_deferred_frees->push_back(ptr_);
        else pool_free(ptr_);
    } catch (...) {
    }
}

SideStream::SideStream() {
    State& s = state();
    {
        std::lock_guard<std::mutex> lock(s.init_mutex);
        if (!s.side) VC_CUDA(cudaStreamCreateWithFlags(&s.side, cudaStreamNonBlocking));
    }
    static thread_local cudaEvent_t events[2] = {nullptr, nullptr};
    for (auto& e : events)
        if (!e) VC_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    fork_ = events[0];
    join_ = events[1];
    main_ = s.stream;
    side_ = s.side;
    VC_CUDA(cudaEventRecord(fork_, main_));
    VC_CUDA(cudaStreamWaitEvent(side_, fork_, 0));
    t_stream_override = side_;
    t_deferred_frees = &deferred_;
    active_ = true;
}

void SideStream::leave() {
    if (!active_) return;
    t_stream_override = nullptr;
    t_deferred_frees = nullptr;
    active_ = false;
}

void SideStream::join() {
    leave();
    if (joined_) return;
    joined_ = true;
    VC_CUDA(cudaEventRecord(join_, side_));
    VC_CUDA(cudaStreamWaitEvent(main_, join_, 0));
    // the main stream now runs after the side work: its scratch may be reused
    for (void* p : deferred_) pool_free(p);
    deferred_.clear();
}

SideStream::~SideStream() {
    try {
        join();
    } catch (...) {
    }
}

std::size_t checked_numel(const size_t* shape, int rank) {
    std::size_t total = 1;
    for (int i = 0; i < rank; ++i) {
        const std::size_t d = shape[i];
        if (d != 0 && total > SIZE_MAX / d) fail(VC_ERR_OVERFLOW, "tensor element count overflows size_t");
        total *= d;
    }
    return total;
}

void validate_rank(int rank, const char* what) {
    if (rank < 0 || rank > kMaxRank)
        fail(VC_ERR_INVALID, std::string(what) + ": the CUDA device supports tensors of rank 0.." +
                                 std::to_string(kMaxRank));
}

// One thread waits on an mbarrier whose phase nothing completes, with the
// bounded wait of the pipelined kernels limited to `polls` polls: it gives
// up, sets kErrWaitTimeout and returns (the failure path, without a fault).
__global__ void selftest_wait_timeout_kernel(long long polls, unsigned* err) {
    __shared__ unsigned long long bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    mbar_fence_init();
    mbar_wait_bounded(&bar, 0, err, polls);
}

static void surface_device_errors() {
    State& s = state();
    unsigned word = 0;
    VC_CUDA(cudaMemcpy(&word, s.error_word, sizeof word, cudaMemcpyDeviceToHost));
    if (!word) return;
    VC_CUDA(cudaMemset(s.error_word, 0, sizeof(unsigned)));
    std::string what;
    if (word & kErrBadTarget) what += "cross_entropy target class out of range; ";
    if (word & kErrBadIndex) what += "scatter index out of range; ";
    if (word & kErrWaitTimeout) what += "a bounded device-side wait timed out; ";
    fail(word & kErrWaitTimeout ? VC_ERR_TIMEOUT : VC_ERR_OUT_OF_RANGE,
         "CUDA device reported: " + what.substr(0, what.size() - 2));
}

}  // namespace vc

using namespace vc;

extern "C" {

int vc_cuda_available(void) {
    try {
        ensure_init();
        return 1;
    } catch (const Error& e) {
        set_last_error(e.what());
        return 0;
    }
}

vc_status vc_cuda_init(int device) {
    VC_API_BEGIN
    init_device(device);
    VC_API_END
}

const char* vc_cuda_last_error(void) { return t_last_error.c_str(); }

vc_status vc_cuda_device_name(char* buffer, size_t length) {
    VC_API_BEGIN
    ensure_init();
    if (!buffer || !length) fail(VC_ERR_INVALID, "vc_cuda_device_name: empty buffer");
    std::snprintf(buffer, length, "%s", state().name);
    VC_API_END
}

vc_status vc_cuda_synchronize(void) {
    VC_API_BEGIN
    ensure_init();
    {
        Transfers& x = state().xfer;
        std::lock_guard<std::mutex> lock(x.mutex);
        if (x.h2d) {
            VC_CUDA(cudaStreamSynchronize(x.h2d));
            VC_CUDA(cudaStreamSynchronize(x.d2h));
            x.pending.clear();
        }
    }
    VC_CUDA(cudaStreamSynchronize(state().stream));
    surface_device_errors();
    VC_API_END
}

void* vc_cuda_stream(void) {
    try {
        ensure_init();
        return state().stream;
    } catch (const Error& e) {
        set_last_error(e.what());
        return nullptr;
    }
}

vc_status vc_cuda_set_stream(void* s) {
    VC_API_BEGIN
    ensure_init();
    State& st = state();
    cudaStream_t next = s ? static_cast<cudaStream_t>(s) : st.own_stream;
    if (next == st.stream) return VC_OK;
    // Pooled blocks were last used on the old stream: drain it so their
    // reuse on the new one is ordered.
    VC_CUDA(cudaStreamSynchronize(st.stream));
    st.stream = next;
    VC_API_END
}

int vc_cuda_sm_count(void) {
    try {
        ensure_init();
        return state().sms;
    } catch (const Error& e) {
        set_last_error(e.what());
        return 0;
    }
}

vc_status vc_cuda_alloc(size_t bytes, void** pointer) {
    VC_API_BEGIN
    if (!pointer) fail(VC_ERR_INVALID, "vc_cuda_alloc: null output pointer");
    *pointer = pool_alloc(bytes);
    VC_API_END
}

vc_status vc_cuda_free(void* pointer) {
    VC_API_BEGIN
    if (!state().ready) return VC_OK;
    pool_free(pointer);
    VC_API_END
}

vc_status vc_cuda_selftest_wait_timeout(long long polls) {
    VC_API_BEGIN
    ensure_init();
    if (polls < 1 || polls > kWaitPolls) fail(VC_ERR_OUT_OF_RANGE, "selftest_wait_timeout: polls must be in [1, 2^21]");
    selftest_wait_timeout_kernel<<<1, 32, 0, stream()>>>(polls, device_error_word());
    check_launch("selftest_wait_timeout_kernel");
    VC_API_END
}

vc_status vc_cuda_pool_stats(size_t* cached_bytes, size_t* in_use_bytes, size_t* hits,
                             size_t* misses) {
    VC_API_BEGIN
    Pool& pool = state().pool;
    std::lock_guard<std::mutex> lock(pool.mutex);
    if (cached_bytes) *cached_bytes = pool.cached_bytes;
    if (in_use_bytes) *in_use_bytes = pool.in_use_bytes;
    if (hits) *hits = pool.hits;
    if (misses) *misses = pool.misses;
    VC_API_END
}

vc_status vc_cuda_graph_begin(void) {
    VC_API_BEGIN
    ensure_init();
    State& s = state();
    {
        std::lock_guard<std::mutex> lock(s.pool.mutex);
        if (s.pool.capturing) fail(VC_ERR_INVALID, "vc_cuda_graph_begin: a capture is already in progress");
        s.pool.capturing = new GraphRecord();
    }
    const cudaError_t err = cudaStreamBeginCapture(s.stream, cudaStreamCaptureModeRelaxed);
    if (err != cudaSuccess) {
        std::lock_guard<std::mutex> lock(s.pool.mutex);
        delete s.pool.capturing;
        s.pool.capturing = nullptr;
        check_cuda(err, "cudaStreamBeginCapture");
    }
    VC_API_END
}

vc_status vc_cuda_graph_end(void** graph) {
    VC_API_BEGIN
    ensure_init();
    State& s = state();
    GraphRecord* g = nullptr;
    {
        std::lock_guard<std::mutex> lock(s.pool.mutex);
        g = s.pool.capturing;
        if (!g) fail(VC_ERR_INVALID, "vc_cuda_graph_end: no capture in progress");
        s.pool.capturing = nullptr;
        // blocks freed during the capture stay with the graph
        for (auto& entry : g->capture_free)
            for (void* p : entry.second) g->reserved.emplace_back(p, entry.first);
        g->capture_free.clear();
    }
    cudaError_t err = cudaStreamEndCapture(s.stream, &g->graph);
    if (err == cudaSuccess) err = cudaGraphInstantiate(&g->exec, g->graph, 0);
    if (err == cudaSuccess) {
        std::size_t nodes = 0;
        if (cudaGraphGetNodes(g->graph, nullptr, &nodes) == cudaSuccess) g->kernels = nodes;
    }
    if (err != cudaSuccess) {
        cudaGetLastError();
        vc_cuda_graph_destroy(g);
        check_cuda(err, "graph capture (an operation in the captured region synchronised or failed)");
    }
    if (!graph) {
        vc_cuda_graph_destroy(g);
        fail(VC_ERR_INVALID, "vc_cuda_graph_end: null output");
    }
    *graph = g;
    VC_API_END
}

vc_status vc_cuda_graph_launch(void* graph) {
    VC_API_BEGIN
    ensure_init();
    auto* g = static_cast<GraphRecord*>(graph);
    if (!g || !g->exec) fail(VC_ERR_INVALID, "vc_cuda_graph_launch: not a captured graph");
    VC_CUDA(cudaGraphLaunch(g->exec, state().stream));
    VC_API_END
}

vc_status vc_cuda_graph_nodes(void* graph, size_t* nodes) {
    VC_API_BEGIN
    auto* g = static_cast<GraphRecord*>(graph);
    if (!g || !nodes) fail(VC_ERR_INVALID, "vc_cuda_graph_nodes: null argument");
    *nodes = g->kernels;
    VC_API_END
}

vc_status vc_cuda_graph_destroy(void* graph) {
    VC_API_BEGIN
    auto* g = static_cast<GraphRecord*>(graph);
    if (!g) return VC_OK;
    State& s = state();
    // replays already enqueued run before any later user of the blocks
    // (one stream); the reserved blocks go back to the pool
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    {
        // blocks still held by tensors lose the graph tag (freed normally
        // later); the reserved ones return to the cache
        std::lock_guard<std::mutex> lock(s.pool.mutex);
        for (auto it = s.pool.owner.begin(); it != s.pool.owner.end();) {
            if (it->second == g) it = s.pool.owner.erase(it);
            else ++it;
        }
        for (const auto& entry : g->reserved) {
            s.pool.free_blocks[entry.second].push_back(entry.first);
            s.pool.cached_bytes += entry.second;
        }
    }
    delete g;
    VC_API_END
}

vc_status vc_cuda_pool_trim(void) {
    VC_API_BEGIN
    ensure_init();
    VC_CUDA(cudaStreamSynchronize(state().stream));
    Pool& pool = state().pool;
    std::lock_guard<std::mutex> lock(pool.mutex);
    release_cached_locked(pool);
    VC_API_END
}

vc_status vc_cuda_host_alloc(size_t bytes, void** pointer) {
    VC_API_BEGIN
    ensure_init();
    if (!pointer) fail(VC_ERR_INVALID, "vc_cuda_host_alloc: null output pointer");
    VC_CUDA(cudaHostAlloc(pointer, bytes ? bytes : 1, cudaHostAllocPortable));
    VC_API_END
}

vc_status vc_cuda_host_free(void* pointer) {
    VC_API_BEGIN
    if (pointer) VC_CUDA(cudaFreeHost(pointer));
    VC_API_END
}

}  // extern "C"

namespace vc {
namespace {

Staging& staging() {
    Staging& st = state().staging;
    if (!st.workers) {
        for (int b = 0; b < 2; ++b) {
            VC_CUDA(cudaHostAlloc(&st.buf[b], kStageChunk, cudaHostAllocPortable));
            VC_CUDA(cudaEventCreateWithFlags(&st.done[b], cudaEventDisableTiming));
        }
        unsigned n = std::thread::hardware_concurrency();
        n = n > 1 ? std::min(n - 1, 7u) : 0u;
        if (const char* env = std::getenv("VC_CUDA_COPY_THREADS")) n = static_cast<unsigned>(std::strtoul(env, nullptr, 10));
        st.workers = new CopyWorkers(n);  // lives as long as the process
    }
    return st;
}

// Host -> device from pageable memory: returns once src may be reused (the
// last pieces' DMAs may still run from the staging buffers; the next staged
// copy waits for them before refilling a buffer).
void staged_upload(void* dst, const void* src, std::size_t bytes) {
    State& s = state();
    std::lock_guard<std::mutex> lock(s.staging.mutex);
    Staging& st = staging();
    const char* in = static_cast<const char*>(src);
    char* out = static_cast<char*>(dst);
    for (std::size_t off = 0, k = 0; off < bytes; off += kStageChunk, ++k) {
        const std::size_t len = std::min(kStageChunk, bytes - off);
        const unsigned b = k & 1u;
        VC_CUDA(cudaEventSynchronize(st.done[b]));
        st.workers->copy(st.buf[b], in + off, len);
        VC_CUDA(cudaMemcpyAsync(out + off, st.buf[b], len, cudaMemcpyHostToDevice, s.stream));
        VC_CUDA(cudaEventRecord(st.done[b], s.stream));
    }
}

// Device -> pageable host memory: the DMA of piece k+1 runs while the host
// threads copy piece k out of the other staging buffer.
void staged_download(void* dst, const void* src, std::size_t bytes) {
    State& s = state();
    std::lock_guard<std::mutex> lock(s.staging.mutex);
    Staging& st = staging();
    const char* in = static_cast<const char*>(src);
    char* out = static_cast<char*>(dst);
    const std::size_t pieces = (bytes + kStageChunk - 1) / kStageChunk;
    auto issue = [&](std::size_t k) {
        const std::size_t off = k * kStageChunk, len = std::min(kStageChunk, bytes - off);
        VC_CUDA(cudaMemcpyAsync(st.buf[k & 1u], in + off, len, cudaMemcpyDeviceToHost, s.stream));
        VC_CUDA(cudaEventRecord(st.done[k & 1u], s.stream));
    };
    issue(0);
    if (pieces > 1) issue(1);
    for (std::size_t k = 0; k < pieces; ++k) {
        const std::size_t off = k * kStageChunk, len = std::min(kStageChunk, bytes - off);
        VC_CUDA(cudaEventSynchronize(st.done[k & 1u]));
        st.workers->copy(out + off, st.buf[k & 1u], len);
        if (k + 2 < pieces) issue(k + 2);
    }
}

bool capturing() {
    Pool& pool = state().pool;
    std::lock_guard<std::mutex> lock(pool.mutex);
    return pool.capturing != nullptr;
}

bool is_pinned(const void* host) {
    cudaPointerAttributes attr{};
    const bool pinned = cudaPointerGetAttributes(&attr, host) == cudaSuccess && attr.type == cudaMemoryTypeHost;
    cudaGetLastError();
    return pinned;
}

}  // namespace
}  // namespace vc

extern "C" {

vc_status vc_cuda_upload(void* dst, const void* src, size_t bytes) {
    VC_API_BEGIN
    ensure_init();
    if (!bytes) return VC_OK;
    if (!dst || !src) fail(VC_ERR_INVALID, "vc_cuda_upload: null pointer");
    const bool pinned = is_pinned(src);
    if (!pinned && bytes >= kStageMin && !capturing()) {
        staged_upload(dst, src, bytes);
        return VC_OK;
    }
    VC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, state().stream));
    // Pageable sources are staged by the driver before cudaMemcpyAsync
    // returns; a pinned source is read later, so wait for this copy to keep
    // the "src may be reused on return" contract.
    if (pinned) VC_CUDA(cudaStreamSynchronize(state().stream));
    VC_API_END
}

vc_status vc_cuda_download(void* dst, const void* src, size_t bytes) {
    VC_API_BEGIN
    ensure_init();
    if (!bytes) return VC_OK;
    if (!dst || !src) fail(VC_ERR_INVALID, "vc_cuda_download: null pointer");
    if (bytes >= kStageMin && !is_pinned(dst) && !capturing()) {
        staged_download(dst, src, bytes);
    } else {
        VC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, state().stream));
    }
    VC_CUDA(cudaStreamSynchronize(state().stream));
    surface_device_errors();
    VC_API_END
}

}  // extern "C"

namespace vc {
namespace {

// Enqueue one asynchronous copy: after the compute work enqueued so far, on
// the direction's copy stream; returns its ticket.
unsigned long long enqueue_transfer(bool upload, void* dst, const void* src, std::size_t bytes) {
    State& s = state();
    {
        std::lock_guard<std::mutex> lock(s.pool.mutex);
        if (s.pool.capturing) fail(VC_ERR_INVALID, "asynchronous transfers cannot be captured in a CUDA graph");
    }
    const void* host = upload ? src : dst;
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, host) != cudaSuccess || attr.type != cudaMemoryTypeHost) {
        cudaGetLastError();
        fail(VC_ERR_INVALID, "asynchronous transfers need page-locked host memory (vc_cuda_host_alloc)");
    }
    Transfers& x = s.xfer;
    std::lock_guard<std::mutex> lock(x.mutex);
    if (!x.h2d) {
        VC_CUDA(cudaStreamCreateWithFlags(&x.h2d, cudaStreamNonBlocking));
        VC_CUDA(cudaStreamCreateWithFlags(&x.d2h, cudaStreamNonBlocking));
        for (auto& e : x.order) VC_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        for (auto& e : x.ring) VC_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
    prune_transfers_locked(x);
    cudaStream_t cs = upload ? x.h2d : x.d2h;
    cudaEvent_t order = x.order[upload ? 0 : 1];
    VC_CUDA(cudaEventRecord(order, s.stream));
    VC_CUDA(cudaStreamWaitEvent(cs, order, 0));
    VC_CUDA(cudaMemcpyAsync(dst, src, bytes, upload ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost, cs));
    const unsigned long long t = x.next;
    cudaEvent_t done = x.ring[t % kTicketRing];
    VC_CUDA(cudaEventSynchronize(done));  // the slot's previous ticket has completed
    VC_CUDA(cudaEventRecord(done, cs));
    ++x.next;
    const char* dev = static_cast<const char*>(upload ? dst : src);
    x.pending.push_back({dev, dev + bytes, t});
    return t;
}

cudaEvent_t ticket_event(unsigned long long ticket, const char* what) {
    Transfers& x = state().xfer;
    if (ticket == 0 || ticket >= x.next) fail(VC_ERR_INVALID, std::string(what) + ": unknown transfer ticket");
    if (ticket_retired(x, ticket)) return nullptr;
    return x.ring[ticket % kTicketRing];
}

}  // namespace
}  // namespace vc

extern "C" {

vc_status vc_cuda_upload_async(void* dst, const void* src, size_t bytes, uint64_t* ticket) {
    VC_API_BEGIN
    ensure_init();
    if (!ticket) fail(VC_ERR_INVALID, "vc_cuda_upload_async: null ticket");
    if (!dst || !src) fail(VC_ERR_INVALID, "vc_cuda_upload_async: null pointer");
    *ticket = enqueue_transfer(true, dst, src, bytes);
    VC_API_END
}

vc_status vc_cuda_download_async(void* dst, const void* src, size_t bytes, uint64_t* ticket) {
    VC_API_BEGIN
    ensure_init();
    if (!ticket) fail(VC_ERR_INVALID, "vc_cuda_download_async: null ticket");
    if (!dst || !src) fail(VC_ERR_INVALID, "vc_cuda_download_async: null pointer");
    *ticket = enqueue_transfer(false, dst, const_cast<void*>(src), bytes);
    VC_API_END
}

vc_status vc_cuda_transfer_wait(uint64_t ticket) {
    VC_API_BEGIN
    ensure_init();
    Transfers& x = state().xfer;
    std::lock_guard<std::mutex> lock(x.mutex);
    if (cudaEvent_t e = ticket_event(ticket, "vc_cuda_transfer_wait")) VC_CUDA(cudaStreamWaitEvent(state().stream, e, 0));
    VC_API_END
}

vc_status vc_cuda_transfer_sync(uint64_t ticket) {
    VC_API_BEGIN
    ensure_init();
    cudaEvent_t e = nullptr;
    {
        Transfers& x = state().xfer;
        std::lock_guard<std::mutex> lock(x.mutex);
        e = ticket_event(ticket, "vc_cuda_transfer_sync");
    }
    if (e) VC_CUDA(cudaEventSynchronize(e));
    VC_API_END
}

vc_status vc_cuda_copy(void* dst, const void* src, size_t bytes) {
    VC_API_BEGIN
    ensure_init();
    if (!bytes) return VC_OK;
    VC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, state().stream));
    VC_API_END
}

}  // extern "C"
