// noalloc.cu -- an allocation-free full sum.
//
// vc_cuda_reduce_all(VC_REDUCE_SUM, ...) keeps its per-segment partials in
// scratch taken from the device pool, which may call cudaMalloc (and the
// pool's recovery path calls cudaFree, which waits for the whole device).
// Some callers cannot allow either: a host that reserved all device memory up
// front under a hard budget, or a latency-critical loop that must not stall on
// an allocation. vc_cuda_reduce_sum_noalloc computes the same sum with its
// scratch in a fixed array compiled into this library instead: 4096 doubles
// (32 KiB), one per 65536-element chunk, which bounds the input at 2^28
// elements. Every GPU that loads the library holds the array until the process
// exits.
#include "vc_internal.cuh"

#include <algorithm>
#include <mutex>

namespace vc {
namespace {

constexpr unsigned long long kChunk = 1ull << 16;                 // elements per partial
constexpr unsigned kMaxPartials = 4096;                           // slots in the array
constexpr unsigned long long kMaxCount = kChunk * kMaxPartials;   // 2^28 elements
constexpr unsigned kThreads = 256;
constexpr int kMaxDevices = 64;

// The scratch. Kernels receive its device address (cudaGetSymbolAddress);
// in host code the name only stands for a host-side shadow.
static __device__ __align__(256) double g_partials[kMaxPartials];

// One CTA per 65536-element chunk: double accumulation, fixed block tree.
// Every chunk writes its slot, so nothing has to be zeroed between calls.
__global__ void __launch_bounds__(kThreads)
noalloc_chunk_sums(const float* __restrict__ in, unsigned long long n, double* __restrict__ partials) {
    __shared__ double s_red[32];
    const unsigned long long chunks = (n + kChunk - 1) / kChunk;
    const bool vec = (reinterpret_cast<std::uintptr_t>(in) & 15u) == 0;
    for (unsigned long long c = blockIdx.x; c < chunks; c += gridDim.x) {
        const unsigned long long begin = c * kChunk;
        const unsigned long long end = min(n, begin + kChunk);
        double acc0 = 0.0, acc1 = 0.0;
        // chunks start at multiples of 65536 elements, so an aligned input
        // keeps every chunk aligned; the last chunk may end with a scalar tail
        const unsigned long long body_end = vec ? begin + ((end - begin) & ~3ull) : begin;
        for (unsigned long long e = begin + threadIdx.x * 4ull; e < body_end; e += kThreads * 4ull) {
            const float4 v = ldg4(in + e);
            acc0 += static_cast<double>(v.x) + static_cast<double>(v.y);
            acc1 += static_cast<double>(v.z) + static_cast<double>(v.w);
        }
        for (unsigned long long k = body_end + threadIdx.x; k < end; k += kThreads)
            acc0 += static_cast<double>(__ldg(in + k));
        const double total = block_sum(acc0 + acc1, s_red);
        if (threadIdx.x == 0) partials[c] = total;
        __syncthreads();
    }
}

// Sum the chunk partials in a fixed order and round once.
__global__ void __launch_bounds__(1024)
noalloc_finish(const double* __restrict__ partials, unsigned chunks, float* __restrict__ out) {
    __shared__ double s_red[32];
    double acc = 0.0;
    for (unsigned c = threadIdx.x; c < chunks; c += blockDim.x) acc += partials[c];
    acc = block_sum(acc, s_red);
    if (threadIdx.x == 0) out[0] = static_cast<float>(acc);
}

std::mutex g_mutex;
double* g_address[kMaxDevices] = {};

// Device address of the array on `device`, looked up once per device and
// cached. The caller has made `device` current on this thread.
double* partials_address(int device) {
    if (device < 0 || device >= kMaxDevices) fail(VC_ERR_RUNTIME, "device index out of range for the allocation-free sum");
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_address[device]) {
        void* p = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&p, g_partials);
        if (err != cudaSuccess) {
            cudaGetLastError();
            fail(VC_ERR_RUNTIME, std::string("cudaGetSymbolAddress for the allocation-free sum failed: ") +
                                     cudaGetErrorString(err));
        }
        g_address[device] = static_cast<double*>(p);
    }
    return g_address[device];
}

}  // namespace
}  // namespace vc

using namespace vc;

extern "C" {

vc_status vc_cuda_reduce_sum_noalloc(const float* in, size_t count, float* out) {
    VC_API_BEGIN
    if (!initialized())
        fail(VC_ERR_RUNTIME, "vc_cuda_reduce_sum_noalloc: call vc_cuda_init first (this entry point allocates "
                             "nothing, not even the device's stream)");
    // The calling host thread may never have called into the library, or may
    // have another GPU current: bind it to the library's GPU, whose stream
    // the kernels go to and whose copy of the array they must use.
    ensure_init();
    const int device = bound_device();
    if (!out) fail(VC_ERR_INVALID, "vc_cuda_reduce_sum_noalloc: null output");
    if (count > kMaxCount)
        fail(VC_ERR_OVERFLOW, "vc_cuda_reduce_sum_noalloc: " + std::to_string(count) +
                                  " elements exceed its maximum of 268435456 (2^28: 4096 partials of 65536)");
    double* partials = partials_address(device);
    if (count == 0) {
        VC_CUDA(cudaMemsetAsync(out, 0, sizeof(float), stream()));
        return VC_OK;
    }
    if (!in) fail(VC_ERR_INVALID, "vc_cuda_reduce_sum_noalloc: null input");
    const unsigned chunks = static_cast<unsigned>((count + kChunk - 1) / kChunk);
    const unsigned grid = std::min<unsigned>(chunks, static_cast<unsigned>(sm_count()) * 8);
    noalloc_chunk_sums<<<grid, kThreads, 0, stream()>>>(in, count, partials);
    check_launch("noalloc_chunk_sums");
    noalloc_finish<<<1, 1024, 0, stream()>>>(partials, chunks, out);
    check_launch("noalloc_finish");
    VC_API_END
}

}  // extern "C"
