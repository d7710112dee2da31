// matmul.cu -- batched matmul and last-two-axes transpose.
//
// Both are "existing ops" for this device (the hot path is bandwidth-bound;
// tensor cores are not used here): correct float32 kernels so models built on
// VectorCore (Linear, the examples) run on the cuda device, not tuned ones.
// Semantics follow MetalBackend::matmul / transpose_last2
// (include/vectorcore/metal_backend.hpp:33-39): output batch z is
// op(A)[a_offsets[z] ...] @ op(B)[b_offsets[z] ...], each (m x k) @ (k x n);
// with trans_a A is stored (k x m), with trans_b B is stored (n x k).
#include "vc_internal.cuh"

#include <algorithm>
#include <vector>

namespace vc {
namespace {

constexpr int TM = 64, TN = 64, TK = 16;  // CTA tile; 16x16 threads, 4x4 outputs each

template <bool TA, bool TB>
__global__ void __launch_bounds__(256)
sgemm_kernel(const float* __restrict__ A, const float* __restrict__ Bm, float* __restrict__ C, int m, int k, int n,
             const unsigned long long* __restrict__ a_off, const unsigned long long* __restrict__ b_off) {
    __shared__ float sa[TK][TM + 4];
    __shared__ float sb[TK][TN + 4];
    const int z = blockIdx.z;
    const float* a = A + a_off[z];
    const float* b = Bm + b_off[z];
    float* c = C + static_cast<unsigned long long>(z) * m * n;
    const int row0 = blockIdx.y * TM, col0 = blockIdx.x * TN;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < k; k0 += TK) {
        for (int e = threadIdx.x; e < TM * TK; e += 256) {
            const int r = e / TK, kk = e % TK;  // element (row0 + r, k0 + kk) of op(A)
            const int gr = row0 + r, gk = k0 + kk;
            float v = 0.0f;
            if (gr < m && gk < k) v = TA ? a[static_cast<long long>(gk) * m + gr] : a[static_cast<long long>(gr) * k + gk];
            sa[kk][r] = v;
        }
        for (int e = threadIdx.x; e < TN * TK; e += 256) {
            const int kk = e / TN, cc = e % TN;  // element (k0 + kk, col0 + cc) of op(B)
            const int gk = k0 + kk, gc = col0 + cc;
            float v = 0.0f;
            if (gk < k && gc < n) v = TB ? b[static_cast<long long>(gc) * k + gk] : b[static_cast<long long>(gk) * n + gc];
            sb[kk][cc] = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < TK; ++kk) {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = sa[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = sb[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += av[i] * bv[j];
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = row0 + ty * 4 + i;
        if (r >= m) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int cc = col0 + tx * 4 + j;
            if (cc < n) c[static_cast<long long>(r) * n + cc] = acc[i][j];
        }
    }
}

__global__ void __launch_bounds__(256)
transpose_kernel(const float* __restrict__ in, float* __restrict__ out, unsigned long long rows,
                 unsigned long long cols) {
    __shared__ float tile[32][33];
    const unsigned long long z = blockIdx.z;
    const float* src = in + z * rows * cols;
    float* dst = out + z * rows * cols;
    const unsigned long long r0 = static_cast<unsigned long long>(blockIdx.y) * 32, c0 = static_cast<unsigned long long>(blockIdx.x) * 32;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const unsigned long long r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[i][threadIdx.x] = src[r * cols + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
        const unsigned long long c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) dst[c * rows + r] = tile[threadIdx.x][i];
    }
}

}  // namespace
}  // namespace vc

using namespace vc;

extern "C" {

vc_status vc_cuda_matmul(const float* a, const float* b, float* out, size_t m, size_t k, size_t n,
                         const size_t* a_offsets, const size_t* b_offsets, size_t batch, int trans_a,
                         int trans_b) {
    VC_API_BEGIN
    ensure_init();
    if (batch == 0 || m == 0 || n == 0) return VC_OK;
    if (!out) fail(VC_ERR_INVALID, "matmul: null output");
    if (k == 0) {
        VC_CUDA(cudaMemsetAsync(out, 0, batch * m * n * sizeof(float), stream()));
        return VC_OK;
    }
    if (!a || !b || !a_offsets || !b_offsets) fail(VC_ERR_INVALID, "matmul: null pointer");
    if (m > (1u << 30) || n > (1u << 30) || k > (1u << 30)) fail(VC_ERR_OVERFLOW, "matmul dimension too large");
    if (batch > 65535) fail(VC_ERR_OVERFLOW, "matmul: more than 65535 batches");
    std::vector<unsigned long long> offs(2 * batch);
    for (size_t z = 0; z < batch; ++z) {
        offs[z] = a_offsets[z];
        offs[batch + z] = b_offsets[z];
    }
    Scratch d_off(offs.size() * sizeof(unsigned long long));
    VC_CUDA(cudaMemcpyAsync(d_off.as<unsigned long long>(), offs.data(), offs.size() * sizeof(unsigned long long),
                            cudaMemcpyHostToDevice, stream()));
    // the host vector must outlive the copy: wait for it
    VC_CUDA(cudaStreamSynchronize(stream()));
    dim3 grid(static_cast<unsigned>((n + TN - 1) / TN), static_cast<unsigned>((m + TM - 1) / TM),
              static_cast<unsigned>(batch));
    const unsigned long long* ao = d_off.as<unsigned long long>();
    const unsigned long long* bo = ao + batch;
    const int mi = static_cast<int>(m), ki = static_cast<int>(k), ni = static_cast<int>(n);
    if (!trans_a && !trans_b) sgemm_kernel<false, false><<<grid, 256, 0, stream()>>>(a, b, out, mi, ki, ni, ao, bo);
    else if (trans_a && !trans_b) sgemm_kernel<true, false><<<grid, 256, 0, stream()>>>(a, b, out, mi, ki, ni, ao, bo);
    else if (!trans_a && trans_b) sgemm_kernel<false, true><<<grid, 256, 0, stream()>>>(a, b, out, mi, ki, ni, ao, bo);
    else sgemm_kernel<true, true><<<grid, 256, 0, stream()>>>(a, b, out, mi, ki, ni, ao, bo);
    check_launch("matmul");
    VC_API_END
}

vc_status vc_cuda_transpose_last2(const float* in, float* out, size_t batch, size_t rows, size_t cols) {
    VC_API_BEGIN
    ensure_init();
    if (!batch || !rows || !cols) return VC_OK;
    if (!in || !out) fail(VC_ERR_INVALID, "transpose: null pointer");
    if (batch > 65535 || (rows + 31) / 32 > 65535) fail(VC_ERR_OVERFLOW, "transpose: too many tiles");
    dim3 grid(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((rows + 31) / 32),
              static_cast<unsigned>(batch));
    transpose_kernel<<<grid, dim3(32, 8), 0, stream()>>>(in, out, rows, cols);
    check_launch("transpose");
    VC_API_END
}

}  // extern "C"
