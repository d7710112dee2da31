// fused.cu -- fused forward chains for sm_100a: relu(x + b).sum() for a
// row-broadcast bias b, forward and backward, each ONE launch.
//
// The reference runs the chain as separate ops with a full-size temporary per
// step (src/ops.cpp:27-52 add, :395-403 relu, :288-302 sum) and its backward
// as broadcast_to + relu backward + sum_to_shape (src/autograd.cpp:50-91):
// five to seven passes. Here the forward reads x and b once; the backward
// recomputes h = x + b (the same float add, so the same bits) instead of
// reading a saved h, writes dx once and reduces db in the same pass.
//
// Arithmetic, as the reference:
//   h = x + b;  y = h > 0 ? h : 0;  loss = float(sum of y)
//   g = u + 0 (broadcast_to of the upstream scalar);  dx = g * (h > 0 ? 1 : 0)
//   db[j] = float(sum over rows of dx[i, j])
// dx and db are bit-exact (db from exact integer counts, see db_from_count).
// The loss sum is double (groups of four terms in float, then double) over
// shape-derived splits finished by the last CTA to arrive (a ticket counter)
// in a fixed order, so it does not depend on timing.
#include "vc_internal.cuh"

#include <algorithm>

namespace vc {

namespace {

constexpr unsigned kThreads = 256;
constexpr unsigned kTicketForward = 0;        // slots among the stream's ticket counters
constexpr unsigned kTicketBackward = 1;
constexpr unsigned kFwdPerThread = 4;         // forward: float4 groups per thread (in flight together)
// backward CTA: 64 float4 columns (256 floats) x 4 row groups x 4 rows
constexpr unsigned kBwdLanes = 64;
constexpr unsigned kBwdGroups = kThreads / kBwdLanes;
constexpr unsigned kBwdRowsPerThread = 4;
constexpr unsigned kBwdSegRows = kBwdGroups * kBwdRowsPerThread;
constexpr unsigned kBwdColBlock = kBwdLanes * 4;
// forward, flat: 512 threads x 8 float4 groups in flight = 4096 groups per CTA
constexpr unsigned kFwdThreads = 512;
constexpr unsigned kFwdGroups = 8;
constexpr unsigned long long kFwdPerCta = kFwdThreads * kFwdGroups;
// backward, column strips: a CTA owns 16 floats of every row (four float4
// lanes x 128 row slots, six rows in flight per thread)
constexpr unsigned kStripThreads = 512;
constexpr unsigned kStripLanes = 4;
constexpr unsigned kStripSlots = kStripThreads / kStripLanes;
constexpr unsigned kStripRowsInFlight = 6;
constexpr unsigned kStripCols = kStripLanes * 4;
constexpr unsigned long long kStripMaxRows = 4096;

__device__ __forceinline__ float relu_of(float h) { return h > 0.0f ? h : 0.0f; }

// Last CTA to arrive (ticket == expected - 1) sees every CTA's partial.
__device__ __forceinline__ bool arrive_last(unsigned* ticket, unsigned expected, bool* s_last) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        *s_last = atomicAdd(ticket, 1u) == expected - 1;
    }
    __syncthreads();
    if (*s_last) __threadfence();
    return *s_last;
}

// Forward over x viewed as float4 groups (x rows a multiple of 4 floats,
// 16-byte aligned). CTA k owns groups [4096 k, 4096 (k + 1)); thread t loads
// groups t + 512 j (j < 8) together, so the whole tensor is requested in one
// wave, and adds them in j order. The last CTA to arrive adds the per-CTA
// partials in CTA order, each thread loading its partials before adding
// (independent loads, one L2 round trip), then a fixed block tree.
// Two CTAs per SM (at most 64 registers), so the 256 CTAs of a
// 1024 x 4096 problem run in one wave on 148 SMs.
__global__ void __launch_bounds__(kFwdThreads, 2)
bias_relu_sum_fwd_wide(const float* __restrict__ x, const float* __restrict__ b, unsigned long long units,
                       FastDiv cols_fd, double* __restrict__ partial, unsigned* __restrict__ ticket,
                       float* __restrict__ loss, double* __restrict__ loss_d) {
    __shared__ double s_red[32];
    __shared__ bool s_last;
    pdl_wait();
    pdl_trigger();
    const unsigned long long base = static_cast<unsigned long long>(blockIdx.x) * kFwdPerCta;
    float4 xv[kFwdGroups];
#pragma unroll
    for (unsigned k = 0; k < kFwdGroups; ++k) {
        const unsigned long long e = base + k * kFwdThreads + threadIdx.x;
        if (e < units) xv[k] = ldg4(x + 4 * e);
    }
    // the bias groups (L1 hits: b is one row) are loaded as they are used,
    // so the x groups alone hold registers while in flight
    double acc = 0.0;
#pragma unroll
    for (unsigned k = 0; k < kFwdGroups; ++k) {
        const unsigned long long e = base + k * kFwdThreads + threadIdx.x;
        if (e >= units) continue;
        unsigned q, r;
        cols_fd.divmod(static_cast<unsigned>(e), q, r);
        const float4 bv = ldg4(b + 4ull * r);
        const float y0 = relu_of(xv[k].x + bv.x), y1 = relu_of(xv[k].y + bv.y);
        const float y2 = relu_of(xv[k].z + bv.z), y3 = relu_of(xv[k].w + bv.w);
        acc += static_cast<double>((y0 + y1) + (y2 + y3));
    }
    acc = block_sum(acc, s_red);
    if (threadIdx.x == 0) partial[blockIdx.x] = acc;
    if (!arrive_last(ticket, gridDim.x, &s_last)) return;
    double t = 0.0;
    for (unsigned s0 = 0; s0 < gridDim.x; s0 += 4 * kFwdThreads) {
        double p[4];
#pragma unroll
        for (unsigned j = 0; j < 4; ++j) {
            const unsigned s = s0 + j * kFwdThreads + threadIdx.x;
            p[j] = s < gridDim.x ? __ldcg(partial + s) : 0.0;
        }
#pragma unroll
        for (unsigned j = 0; j < 4; ++j) t += p[j];
    }
    t = block_sum(t, s_red);
    if (threadIdx.x == 0) {
        if (loss) *loss = static_cast<float>(t);
        if (loss_d) *loss_d = t;
        *ticket = 0;  // ready for the next launch (stream order)
    }
}

// Forward over x viewed flat: CTA k owns the 1024 float4 groups (or
// elements) [k * 1024, ...); thread t adds groups t, t + 256, t + 512,
// t + 768 of them (four loads in flight), each group's bias from its column.
// The last CTA adds the per-CTA partials in order.
template <bool VEC>
__global__ void __launch_bounds__(kThreads)
bias_relu_sum_fwd(const float* __restrict__ x, const float* __restrict__ b, unsigned long long units,
                  unsigned long long cols_units, FastDiv cols_fd, bool cols_small, double* __restrict__ partial,
                  unsigned* __restrict__ ticket, float* __restrict__ loss, double* __restrict__ loss_d) {
    __shared__ double s_red[32];
    __shared__ bool s_last;
    const unsigned long long base = static_cast<unsigned long long>(blockIdx.x) * kThreads * kFwdPerThread;
    auto col_of = [&](unsigned long long e) -> unsigned long long {
        if (cols_small) {  // e < 2^32: FastDiv
            unsigned q, r;
            cols_fd.divmod(static_cast<unsigned>(e), q, r);
            return r;
        }
        return e % cols_units;
    };
    double acc = 0.0;
    if constexpr (VEC) {
        float4 xv[kFwdPerThread], bv[kFwdPerThread];
        bool ok[kFwdPerThread];
#pragma unroll
        for (unsigned k = 0; k < kFwdPerThread; ++k) {
            const unsigned long long e = base + k * kThreads + threadIdx.x;
            ok[k] = e < units;
            if (ok[k]) {
                xv[k] = ldg4(x + 4 * e);
                bv[k] = ldg4(b + 4 * col_of(e));
            }
        }
#pragma unroll
        for (unsigned k = 0; k < kFwdPerThread; ++k) {
            if (!ok[k]) continue;
            const float y0 = relu_of(xv[k].x + bv[k].x), y1 = relu_of(xv[k].y + bv[k].y);
            const float y2 = relu_of(xv[k].z + bv[k].z), y3 = relu_of(xv[k].w + bv[k].w);
            acc += static_cast<double>((y0 + y1) + (y2 + y3));
        }
    } else {
#pragma unroll
        for (unsigned k = 0; k < kFwdPerThread; ++k) {
            const unsigned long long e = base + k * kThreads + threadIdx.x;
            if (e < units) acc += static_cast<double>(relu_of(__ldg(x + e) + __ldg(b + col_of(e))));
        }
    }
    acc = block_sum(acc, s_red);
    if (threadIdx.x == 0) partial[blockIdx.x] = acc;
    if (!arrive_last(ticket, gridDim.x, &s_last)) return;
    double t = 0.0;
    for (unsigned s = threadIdx.x; s < gridDim.x; s += kThreads) t += __ldcg(partial + s);
    t = block_sum(t, s_red);
    if (threadIdx.x == 0) {
        if (loss) *loss = static_cast<float>(t);
        if (loss_d) *loss_d = t;
        *ticket = 0;  // ready for the next launch (stream order)
    }
}

// db[j] from the count of rows with x + b > 0. Every dx[i, j] is g * 1 = g or
// g * 0 = +-0, so the reference's double sum over rows is g * count exactly
// (no rounding while count < 2^29: 24 + 29 bits), +0 for a zero count (the
// sum starts at +0), NaN for a NaN g, and for an infinite g +-inf only when
// every row contributes g (inf * 0 is NaN).
__device__ __forceinline__ double db_from_count(float g, unsigned long long count, unsigned long long rows) {
    if (g != g) return static_cast<double>(g);
    if (isinf(g)) return count == rows ? static_cast<double>(g) : static_cast<double>(__int_as_float(0x7fc00000));
    if (count == 0) return 0.0;
    return static_cast<double>(g) * static_cast<double>(count);
}

// Backward. grid = (column blocks of 256, row segments of 16). Thread
// (lane, group) owns columns c0 + 4*lane .. +3 (or c0 + lane + 64k without
// float4) over rows r0 + 4*group .. +3: loads them together, writes dx and
// counts its rows with h > 0. The four groups' counts meet in shared memory
// and go to `counts` with one integer atomic per column and CTA (exact in any
// order); the last CTA converts them to db and clears them.
template <bool VEC>
__global__ void __launch_bounds__(kThreads)
bias_relu_sum_bwd(const float* __restrict__ x, const float* __restrict__ b, const float* __restrict__ upstream,
                  unsigned long long rows, unsigned long long cols, float* __restrict__ dx, float* __restrict__ db,
                  double* __restrict__ db_d, unsigned* __restrict__ counts, unsigned* __restrict__ ticket) {
    __shared__ bool s_last;
    __shared__ unsigned s_cnt[kBwdGroups][kBwdColBlock];
    const float g = __ldg(upstream) + 0.0f;  // broadcast_to(u): u + 0
    const unsigned lane = threadIdx.x % kBwdLanes, grp = threadIdx.x / kBwdLanes;
    const unsigned long long r0 = static_cast<unsigned long long>(blockIdx.y) * kBwdSegRows + grp * kBwdRowsPerThread;
    const unsigned long long c0 = static_cast<unsigned long long>(blockIdx.x) * kBwdColBlock;
    unsigned n[4] = {0, 0, 0, 0};
    if constexpr (VEC) {
        const unsigned long long c = c0 + 4ull * lane;
        if (c < cols) {
            const float4 bv = ldg4(b + c);
            float4 xs[kBwdRowsPerThread];
#pragma unroll
            for (unsigned k = 0; k < kBwdRowsPerThread; ++k)
                if (r0 + k < rows) xs[k] = ldg4(x + (r0 + k) * cols + c);
#pragma unroll
            for (unsigned k = 0; k < kBwdRowsPerThread; ++k) {
                if (r0 + k >= rows) break;
                const float4 xv = xs[k];
                const bool p0 = (xv.x + bv.x) > 0.0f, p1 = (xv.y + bv.y) > 0.0f;
                const bool p2 = (xv.z + bv.z) > 0.0f, p3 = (xv.w + bv.w) > 0.0f;
                st4_stream(dx + (r0 + k) * cols + c, make_float4(g * (p0 ? 1.0f : 0.0f), g * (p1 ? 1.0f : 0.0f),
                                                                 g * (p2 ? 1.0f : 0.0f), g * (p3 ? 1.0f : 0.0f)));
                n[0] += p0;
                n[1] += p1;
                n[2] += p2;
                n[3] += p3;
            }
        }
#pragma unroll
        for (unsigned j = 0; j < 4; ++j) s_cnt[grp][4 * lane + j] = n[j];
    } else {
#pragma unroll
        for (unsigned j = 0; j < 4; ++j) {
            const unsigned long long c = c0 + lane + kBwdLanes * j;
            if (c < cols) {
                const float bv = __ldg(b + c);
                for (unsigned k = 0; k < kBwdRowsPerThread && r0 + k < rows; ++k) {
                    const bool p = (__ldg(x + (r0 + k) * cols + c) + bv) > 0.0f;
                    dx[(r0 + k) * cols + c] = g * (p ? 1.0f : 0.0f);
                    n[j] += p;
                }
            }
            s_cnt[grp][lane + kBwdLanes * j] = n[j];
        }
    }
    __syncthreads();
    for (unsigned col = threadIdx.x; col < kBwdColBlock; col += kThreads) {
        const unsigned long long c = c0 + col;
        unsigned t = 0;
#pragma unroll
        for (unsigned q = 0; q < kBwdGroups; ++q) t += s_cnt[q][col];
        if (t && c < cols) atomicAdd(counts + c, t);
    }
    if (!arrive_last(ticket, gridDim.x * gridDim.y, &s_last)) return;
    for (unsigned long long c = threadIdx.x; c < cols; c += kThreads) {
        const unsigned count = __ldcg(counts + c);
        counts[c] = 0;
        const double v = db_from_count(g, count, rows);
        if (db_d) db_d[c] = v;
        else db[c] = static_cast<float>(v);
    }
    if (threadIdx.x == 0) *ticket = 0;
}

// Backward for up to 4096 rows whose length is a multiple of 16 floats:
// CTA k owns columns [16 k, 16 k + 16) of every row, so db needs no
// cross-CTA step (no counter buffer, atomics or ticket). Thread (slot, lane)
// = (tid / 4, tid % 4) owns the float4 column 16 k + 4 lane over rows
// slot + 128 i: it loads six rows together, writes dx and counts the rows
// with h > 0. A warp's eight slots meet by shuffles (lanes of one column are
// 4 apart), the 16 warps through shared memory; integer counts are exact in
// any order.
__global__ void __launch_bounds__(kStripThreads, 2)  // two CTAs per SM: 256 strips in one wave
bias_relu_sum_bwd_strip(const float* __restrict__ x, const float* __restrict__ b, const float* __restrict__ upstream,
                        unsigned rows, unsigned long long cols, float* __restrict__ dx, float* __restrict__ db,
                        double* __restrict__ db_d) {
    __shared__ unsigned s_cnt[kStripThreads / 32][kStripCols];
    pdl_wait();
    pdl_trigger();
    const float g = __ldg(upstream) + 0.0f;  // broadcast_to(u): u + 0
    const unsigned lane = threadIdx.x % kStripLanes, slot = threadIdx.x / kStripLanes;
    const unsigned long long c = static_cast<unsigned long long>(blockIdx.x) * kStripCols + 4ull * lane;
    const float4 bv = ldg4(b + c);
    unsigned n0 = 0, n1 = 0, n2 = 0, n3 = 0;
    for (unsigned r0 = slot; r0 < rows; r0 += kStripSlots * kStripRowsInFlight) {
        float4 xs[kStripRowsInFlight];
#pragma unroll
        for (unsigned k = 0; k < kStripRowsInFlight; ++k) {
            const unsigned r = r0 + k * kStripSlots;
            if (r < rows) xs[k] = ldg4(x + r * cols + c);
        }
#pragma unroll
        for (unsigned k = 0; k < kStripRowsInFlight; ++k) {
            const unsigned r = r0 + k * kStripSlots;
            if (r >= rows) break;
            const bool p0 = (xs[k].x + bv.x) > 0.0f, p1 = (xs[k].y + bv.y) > 0.0f;
            const bool p2 = (xs[k].z + bv.z) > 0.0f, p3 = (xs[k].w + bv.w) > 0.0f;
            st4_stream(dx + r * cols + c, make_float4(g * (p0 ? 1.0f : 0.0f), g * (p1 ? 1.0f : 0.0f),
                                                      g * (p2 ? 1.0f : 0.0f), g * (p3 ? 1.0f : 0.0f)));
            n0 += p0;
            n1 += p1;
            n2 += p2;
            n3 += p3;
        }
    }
#pragma unroll
    for (unsigned off = kStripLanes; off < 32; off <<= 1) {
        n0 += __shfl_xor_sync(0xffffffffu, n0, off);
        n1 += __shfl_xor_sync(0xffffffffu, n1, off);
        n2 += __shfl_xor_sync(0xffffffffu, n2, off);
        n3 += __shfl_xor_sync(0xffffffffu, n3, off);
    }
    const unsigned warp = threadIdx.x / 32;
    if (threadIdx.x % 32 < kStripLanes) {
        s_cnt[warp][4 * lane + 0] = n0;
        s_cnt[warp][4 * lane + 1] = n1;
        s_cnt[warp][4 * lane + 2] = n2;
        s_cnt[warp][4 * lane + 3] = n3;
    }
    __syncthreads();
    if (threadIdx.x < kStripCols) {
        unsigned t = 0;
#pragma unroll
        for (unsigned w = 0; w < kStripThreads / 32; ++w) t += s_cnt[w][threadIdx.x];
        const unsigned long long col = static_cast<unsigned long long>(blockIdx.x) * kStripCols + threadIdx.x;
        const double v = db_from_count(g, t, rows);
        if (db_d) db_d[col] = v;
        else db[col] = static_cast<float>(v);
    }
}

}  // namespace

}  // namespace vc

using namespace vc;

extern "C" {

vc_status vc_cuda_bias_relu_sum(const float* x, const float* b, size_t rows, size_t cols, float* loss,
                                double* loss_partial) {
    VC_API_BEGIN
    ensure_init();
    const size_t dims[2] = {rows, cols};
    checked_numel(dims, 2);
    if (!loss && !loss_partial) fail(VC_ERR_INVALID, "bias_relu_sum: null output");
    if (!rows || !cols) {
        if (loss) VC_CUDA(cudaMemsetAsync(loss, 0, sizeof(float), stream()));
        if (loss_partial) VC_CUDA(cudaMemsetAsync(loss_partial, 0, sizeof(double), stream()));
        return VC_OK;
    }
    if (!x || !b) fail(VC_ERR_INVALID, "bias_relu_sum: null input");
    const bool vec = cols % 4 == 0 && aligned16(x) && aligned16(b);
    const unsigned long long units = vec ? rows * cols / 4 : rows * cols;
    const unsigned long long cols_units = vec ? cols / 4 : cols;
    const unsigned long long ctas = (units + kThreads * kFwdPerThread - 1) / (kThreads * kFwdPerThread);
    if (ctas > 0x7fffffffull) fail(VC_ERR_OVERFLOW, "bias_relu_sum: tensor too large");
    const bool cols_small = units < (1ull << 32) && cols_units < (1ull << 32);
    const FastDiv cols_fd(cols_small ? static_cast<unsigned>(cols_units) : 1u);
    unsigned* ticket = stream_tickets() + kTicketForward;
    if (vec && cols_small) {
        const unsigned long long wide = (units + kFwdPerCta - 1) / kFwdPerCta;
        Scratch partial(wide * sizeof(double));
        // programmatic launch: this kernel's set-up overlaps the previous kernel's tail
        launch_pdl(bias_relu_sum_fwd_wide, dim3(static_cast<unsigned>(wide)), dim3(kFwdThreads), 0, stream(), x, b,
                   units, cols_fd, partial.as<double>(), ticket, loss, loss_partial);
        check_launch("bias_relu_sum");
        return VC_OK;
    }
    Scratch partial(ctas * sizeof(double));
    if (vec) bias_relu_sum_fwd<true><<<static_cast<unsigned>(ctas), kThreads, 0, stream()>>>(x, b, units, cols_units, cols_fd, cols_small, partial.as<double>(), ticket, loss, loss_partial);
    else bias_relu_sum_fwd<false><<<static_cast<unsigned>(ctas), kThreads, 0, stream()>>>(x, b, units, cols_units, cols_fd, cols_small, partial.as<double>(), ticket, loss, loss_partial);
    check_launch("bias_relu_sum");
    VC_API_END
}

vc_status vc_cuda_bias_relu_sum_backward(const float* x, const float* b, const float* upstream, size_t rows,
                                         size_t cols, float* dx, float* db, double* db_partial) {
    VC_API_BEGIN
    ensure_init();
    const size_t dims[2] = {rows, cols};
    checked_numel(dims, 2);
    if (!cols) return VC_OK;
    if (!db && !db_partial) fail(VC_ERR_INVALID, "bias_relu_sum_backward: null db");
    if (!rows) {
        if (db) VC_CUDA(cudaMemsetAsync(db, 0, cols * sizeof(float), stream()));
        if (db_partial) VC_CUDA(cudaMemsetAsync(db_partial, 0, cols * sizeof(double), stream()));
        return VC_OK;
    }
    if (!x || !b || !upstream || !dx) fail(VC_ERR_INVALID, "bias_relu_sum_backward: null pointer");
    const unsigned long long col_blocks = (cols + kBwdColBlock - 1) / kBwdColBlock;
    const unsigned long long segs = (rows + kBwdSegRows - 1) / kBwdSegRows;
    if (col_blocks > 0x7fffffffull || segs > 65535 || col_blocks * segs > 0xffffffffull)
        fail(VC_ERR_OVERFLOW, "bias_relu_sum_backward: tensor too large");
    if (rows >= (1ull << 32)) fail(VC_ERR_OVERFLOW, "bias_relu_sum_backward: too many rows for 32-bit counts");
    const bool vec = cols % 4 == 0 && aligned16(x) && aligned16(b) && aligned16(dx);
    if (vec && cols % kStripCols == 0 && rows <= kStripMaxRows && cols / kStripCols <= 0x7fffffffull) {
        launch_pdl(bias_relu_sum_bwd_strip, dim3(static_cast<unsigned>(cols / kStripCols)), dim3(kStripThreads), 0,
                   stream(), x, b, upstream, static_cast<unsigned>(rows), cols, dx, db, db_partial);
        check_launch("bias_relu_sum_backward");
        return VC_OK;
    }
    Scratch counts(cols * sizeof(unsigned));
    VC_CUDA(cudaMemsetAsync(counts.as<unsigned>(), 0, cols * sizeof(unsigned), stream()));
    const dim3 grid(static_cast<unsigned>(col_blocks), static_cast<unsigned>(segs));
    unsigned* ticket = stream_tickets() + kTicketBackward;
    if (vec) bias_relu_sum_bwd<true><<<grid, kThreads, 0, stream()>>>(x, b, upstream, rows, cols, dx, db, db_partial, counts.as<unsigned>(), ticket);
    else bias_relu_sum_bwd<false><<<grid, kThreads, 0, stream()>>>(x, b, upstream, rows, cols, dx, db, db_partial, counts.as<unsigned>(), ticket);
    check_launch("bias_relu_sum_backward");
    VC_API_END
}

}  // extern "C"
