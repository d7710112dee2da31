// vc_internal.cuh -- shared host/device plumbing of the VectorCore CUDA device.
#pragma once

#include "vc_cuda.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace vc {

// ---------------------------------------------------------------------------
// Host-side error model. Internal code throws vc::Error; every extern "C"
// entry point catches it (VC_API_BEGIN/END), records the message in a
// thread-local string and returns the status.
// ---------------------------------------------------------------------------
struct Error : std::runtime_error {
    vc_status status;
    Error(vc_status s, const std::string& message) : std::runtime_error(message), status(s) {}
};

[[noreturn]] void fail(vc_status status, const std::string& message);
void set_last_error(const std::string& message);
void check_cuda(cudaError_t err, const char* what);

#define VC_CUDA(expr) ::vc::check_cuda((expr), #expr)

#define VC_API_BEGIN try {
#define VC_API_END                                                   \
    return VC_OK;                                                    \
    }                                                                \
    catch (const ::vc::Error& e) {                                   \
        ::vc::set_last_error(e.what());                              \
        return e.status;                                             \
    }                                                                \
    catch (const std::exception& e) {                                \
        ::vc::set_last_error(e.what());                              \
        return VC_ERR_RUNTIME;                                       \
    }                                                                \
    catch (...) {                                                    \
        ::vc::set_last_error("unknown error in the VectorCore CUDA device"); \
        return VC_ERR_RUNTIME;                                       \
    }

// ---------------------------------------------------------------------------
// Runtime state (runtime.cu).
// ---------------------------------------------------------------------------
void ensure_init();              // init device 0 if nothing was selected yet
bool initialized();              // vc_cuda_init (or a first call) has bound a GPU
int bound_device();              // that GPU's index (-1 before initialisation)
cudaStream_t stream();           // the enqueue stream
int sm_count();
unsigned* counters();            // zeroed ticket counters (kCounterSlots)
// kPerStreamTickets zeroed counters owned by the current enqueue stream:
// kernels that reset their ticket in-kernel use these, so calls in flight on
// different streams never share a counter (calls on one stream are ordered).
unsigned* stream_tickets();
constexpr unsigned kPerStreamTickets = 4;
unsigned* device_error_word();   // sticky device error bits
void check_launch(const char* what);

constexpr std::size_t kCounterSlots = 1u << 16;

// Device error bits (set with atomicOr by kernels, read at sync points).
constexpr unsigned kErrWaitTimeout = 1u << 0;   // a bounded wait gave up
constexpr unsigned kErrBadTarget = 1u << 1;     // class target out of range
constexpr unsigned kErrBadIndex = 1u << 2;      // scatter index out of range

// Stream-ordered scratch from the pool; returned to the pool on scope exit
// (after the kernels that use it were enqueued, which stream order makes safe).
class Scratch {
public:
    explicit Scratch(std::size_t bytes);
    ~Scratch();
    Scratch(const Scratch&) = delete;
    Scratch& operator=(const Scratch&) = delete;
    template <typename T> T* as() const { return static_cast<T*>(ptr_); }
private:
    void* ptr_{nullptr};
};

// Fork / join of a second compute stream for two independent halves of one
// call (e.g. the two gradients of a broadcast binary op): the constructor
// makes the side stream wait for the work enqueued so far and routes this
// host thread's launches to it; leave() routes them back to the main stream;
// join() (also on destruction) makes the main stream wait for the side work.
// Scratch the side work frees is returned to the pool only after the join,
// so nothing on the main stream can be handed a block still in use there.
// Enqueue the side half first: its allocations then precede the main half's
// frees, so it cannot be handed a block the main half still uses.
class SideStream {
public:
    SideStream();
    ~SideStream();
    SideStream(const SideStream&) = delete;
    SideStream& operator=(const SideStream&) = delete;
    void leave();
    void join();
private:
    cudaStream_t main_{nullptr}, side_{nullptr};
    cudaEvent_t fork_{nullptr}, join_{nullptr};
    std::vector<void*> deferred_;
    bool active_{false}, joined_{false};
};

inline bool aligned16(const void* p) { return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0; }

// Streaming layout of the flat elementwise kernels (same-shape, scalar and
// their backward rules): CTA b owns the kChunk4 float4 groups
// [kChunk4 * b, kChunk4 * (b + 1)) -- 16 KiB of each operand, one group per
// thread in each of four rounds, every load issued before the first store --
// and the grid has one CTA per chunk. Many short-lived CTAs each on one
// contiguous piece keep HBM busier than a grid-stride loop: a 1 GiB 1:1 float4
// stream measured 6.88 TB/s this way against 5.9-6.3 TB/s grid-stride
// (2:1 streams 7.06 TB/s, 3:2 streams 7.01 TB/s; the copy peak is 6.55).
constexpr unsigned kStreamThreads = 256;
constexpr unsigned kStreamRounds = 4;
constexpr unsigned long long kChunk4 = kStreamThreads * kStreamRounds;
inline unsigned stream_grid(std::size_t n) {
    const unsigned long long chunks = std::max<unsigned long long>(1, ((n >> 2) + kChunk4 - 1) / kChunk4);
    if (chunks > 0x7fffffffull) throw std::runtime_error("tensor too large for one launch");
    return static_cast<unsigned>(chunks);
}

inline unsigned grid_for(std::size_t work_items, unsigned threads, unsigned max_ctas_per_sm = 8) {
    const std::size_t ctas = (work_items + threads - 1) / threads;
    const std::size_t cap = static_cast<std::size_t>(sm_count()) * max_ctas_per_sm;
    std::size_t g = ctas < cap ? ctas : cap;
    return static_cast<unsigned>(g ? g : 1);
}

// ---------------------------------------------------------------------------
// Device helpers.
// ---------------------------------------------------------------------------

// 32-bit division by a runtime-invariant divisor d >= 1 (Granlund-Montgomery,
// round-up multiplier): with l = ceil(log2 d) and
// mul = floor(2^32 * (2^l - d) / d) + 1, q = (umulhi(n, mul) + n) >> l for
// every 32-bit n (the sum is formed in 64 bits).
struct FastDiv {
    unsigned divisor{1};
    unsigned mul{1};
    unsigned shift{0};
    FastDiv() = default;
    explicit FastDiv(unsigned d) : divisor(d) {
        unsigned l = 0;
        while ((1ull << l) < d) ++l;
        mul = static_cast<unsigned>(((1ull << 32) * ((1ull << l) - d)) / d + 1);
        shift = l;
    }
    __device__ __forceinline__ unsigned div(unsigned n) const {
        const unsigned hi = __umulhi(n, mul);
        return static_cast<unsigned>((static_cast<unsigned long long>(hi) + n) >> shift);
    }
    __device__ __forceinline__ void divmod(unsigned n, unsigned& q, unsigned& r) const {
        q = div(n);
        r = n - q * divisor;
    }
};

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

// Streaming (evict-first, ld/st.global.cs) variants for data touched once.
// Intrinsics rather than volatile asm so the compiler may hoist the loads of
// later iterations above earlier stores.
__device__ __forceinline__ float4 ld4_stream(const float* p) { return __ldcs(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ void st4_stream(float* p, float4 v) { __stcs(reinterpret_cast<float4*>(p), v); }

// ---------------------------------------------------------------------------
// mbarrier helpers for bulk copies (TMA). Every wait is bounded: after
// kWaitPolls polls it sets kErrWaitTimeout in the device error word and gives
// up, so a lost completion surfaces as an error at the next sync instead of a
// hung kernel.
// ---------------------------------------------------------------------------

// Programmatic dependent launch. A kernel launched by launch_pdl may begin
// while the kernel before it on the stream is still finishing (its launch and
// CTA set-up overlap that kernel's tail). pdl_wait() blocks until every
// earlier kernel has completed and its writes are visible -- call it before
// the first global read or write; for a normal launch it returns at once.
// pdl_trigger() lets the next programmatic launch start scheduling its CTAs.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, std::size_t smem, cudaStream_t s,
                       Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
    if (err != cudaSuccess) throw std::runtime_error(std::string("cudaLaunchKernelEx: ") + cudaGetErrorString(err));
}

__device__ __forceinline__ unsigned smem_addr(const void* p) {
    return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Order this CTA's earlier generic-proxy accesses of shared memory before
// later async-proxy (bulk copy) writes to it.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
// One poll. The thread may sleep in it for up to kWaitHintNs (or until the
// phase completes) instead of spinning, so a waiting warp issues few
// instructions.
constexpr unsigned kWaitHintNs = 2000;
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(kWaitHintNs)
        : "memory");
    return ok != 0;
}
// Wait for phase `parity` with an iteration limit (at most `polls` polls of
// up to kWaitHintNs each; the kernels use kWaitPolls, a few seconds); false
// (and the device error bit) when it gave up.
constexpr long long kWaitPolls = 1ll << 21;
__device__ __forceinline__ bool mbar_wait_bounded(unsigned long long* bar, unsigned parity, unsigned* err,
                                                  long long polls = kWaitPolls) {
    for (long long i = 0; i < polls; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    atomicOr(err, kErrWaitTimeout);
    return false;
}

// Named barrier ID (1..15) of the CTA's first N threads (a multiple of 32)
// that also returns the OR of a predicate over them: a producer/consumer
// kernel's consumers meet here without the producer warp, and a wait that
// gave up in any consumer reaches all of them at the same barrier.
template <unsigned ID, unsigned N>
__device__ __forceinline__ bool named_barrier_or(bool x) {
    static_assert(ID >= 1 && ID < 16 && N % 32 == 0, "named barrier");
    unsigned r;
    asm volatile(
        "{\n .reg .pred pin, pout;\n setp.ne.u32 pin, %1, 0;\n bar.red.or.pred pout, %2, %3, pin;\n selp.u32 %0, 1, "
        "0, pout;\n}\n"
        : "=r"(r)
        : "r"(static_cast<unsigned>(x)), "n"(ID), "n"(N)
        : "memory");
    return r != 0;
}

// Max/argmax candidate under the reference's scan semantics: a larger value
// wins; equal values (==, so -0 == +0) keep the smaller index; NaN is never
// a candidate (the caller applies the "NaN at index 0 wins" rule).
struct MaxCand {
    float v;
    long long i;  // -1: no candidate
};

__device__ __forceinline__ MaxCand max_combine(MaxCand a, MaxCand b) {
    if (a.i < 0) return b;
    if (b.i < 0) return a;
    if (b.v > a.v) return b;
    if (a.v > b.v) return a;
    return b.i < a.i ? b : a;
}

__device__ __forceinline__ MaxCand max_take(MaxCand c, float v, long long i) {
    // Elements of one thread arrive in increasing index order.
    if (v != v) return c;  // NaN
    if (c.i < 0 || v > c.v) return MaxCand{v, i};
    return c;
}

__device__ __forceinline__ MaxCand shfl_xor_cand(MaxCand c, int mask) {
    MaxCand o;
    o.v = __shfl_xor_sync(0xffffffffu, c.v, mask);
    o.i = __shfl_xor_sync(0xffffffffu, c.i, mask);
    return o;
}

// Fixed-shape warp and block trees (the combine order depends only on the
// thread index, so results do not depend on scheduling).
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

__device__ __forceinline__ MaxCand warp_max(MaxCand c) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) c = max_combine(c, shfl_xor_cand(c, m));
    return c;
}

// Block reductions over blockDim.x threads (multiple of 32, <= 1024). The
// result is returned to every thread. `scratch` needs 32 entries.
__device__ __forceinline__ double block_sum(double v, double* scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    double t = lane < nw ? scratch[lane] : 0.0;
    t = warp_sum(t);
    return t;
}

__device__ __forceinline__ MaxCand block_max(MaxCand c, float* sv, long long* si) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    c = warp_max(c);
    __syncthreads();
    if (lane == 0) { sv[warp] = c.v; si[warp] = c.i; }
    __syncthreads();
    MaxCand t = lane < nw ? MaxCand{sv[lane], si[lane]} : MaxCand{0.0f, -1};
    return warp_max(t);
}

// ---------------------------------------------------------------------------
// Shapes.
// ---------------------------------------------------------------------------
constexpr int kMaxRank = 8;

struct ShapeView {
    int rank{0};
    std::size_t dims[kMaxRank]{};
};

std::size_t checked_numel(const size_t* shape, int rank);
void validate_rank(int rank, const char* what);

// out (out_shape) = src broadcast from src_shape, bit for bit (elementwise.cu).
void broadcast_copy(const float* src, const size_t* src_shape, int src_rank, float* out,
                    const size_t* out_shape, int out_rank);

}  // namespace vc
