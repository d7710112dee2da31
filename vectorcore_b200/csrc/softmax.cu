// softmax.cu -- fused softmax, log_softmax and softmax cross-entropy
// (forward and backward) for sm_100a.
//
// The reference composes these from primitive ops -- six launches and four
// full-size temporaries for log_softmax, plus a host-built one-hot mask for
// cross-entropy (src/ops.cpp:378-388, src/nn.cpp:31-53). Here each is ONE
// pass over HBM: read x (and g) once, write the result once.
//
// Rows (reduction over the last axis), by row length:
//  * aligned rows up to 32K floats: a group of warps per row reads the row
//    from HBM once into registers, combines its statistics in shared memory
//    and re-reads the row from L2 for the output (row_reread_kernel);
//    cross-entropy's forward writes nothing per element and streams each
//    row once, a warp per row (ce_rows_kernel);
//  * longer aligned rows: one thread-block cluster of C CTAs per row, C in
//    {1, 2, 4, 8}; each CTA stages its slice in shared memory with TMA bulk
//    copies (cp.async.bulk, completion on an mbarrier, the next row in
//    flight), and the partials are exchanged through distributed shared
//    memory and combined in rank order, so every CTA of the cluster derives
//    the same row statistics (row_pipe_kernel); unaligned rows take the
//    one-shot cluster kernel with plain loads (row_kernel).
// Other axes (and rows too long for a cluster) take a column kernel that
// walks the axis in global memory.
//
// The arithmetic is the reference's, operation by operation:
//   m  = max(x) with the scan semantics of cpu::reduce_axis,
//   s  = float(sum of exp(x - m)),  l = logf(s),
//   log_softmax = (x - m) - l,  softmax = expf(log_softmax),
// and the backward passes replay the reference autograd chain (engine order
// of src/tensor.cpp:266-300) from the saved m and s:
//   log_softmax: dx = g + ((float(sum(-g)) / s) + 0) * expf(x - m)
//   softmax:     gy = g * y;  dx = gy + ((float(sum(-gy)) / s) + 0) * expf(x - m)
//   cross-entropy (upstream u, batch B): dp = (-(u / B)) + 0,
//     dx = dp * onehot + ((dl / s) + 0) * expf(x - m) with dl = sum(-dp*onehot).
// The reference sums in double. Here the staged (TMA) paths add each group of
// four terms in float and the group sums in double, and the exp terms of s
// come from exp_sum_term / exp_term (ex2-based) rather than expf; the
// per-element outputs use expf, except the re-read kernel's softmax forward
// and softmax backward, which use exp_sfu (within 2e-6 relative of e^t for
// |t| <= 20). Results therefore differ from the CPU
// path only through exp/log ulps and the order and grouping of the additions,
// all far inside the 1e-5 sum tolerance.
#include "vc_internal.cuh"

#include <cooperative_groups.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <utility>

namespace cg = cooperative_groups;

namespace vc {

namespace {

constexpr unsigned kThreads = 256;
constexpr unsigned kSliceTarget = 8192;     // floats per CTA slice (32 KB)
constexpr unsigned kSliceMax = 24576;       // floats per CTA slice at cluster size 8 (96 KB)

enum Mode { LSM_FWD = 0, SM_FWD = 1, CE_FWD = 2, LSM_BWD = 3, SM_BWD = 4 };

// ---- bulk copy into this CTA's shared memory (mbarrier helpers: vc_internal.cuh)
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes, unsigned long long* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

struct RowArgs {
    const float* x;
    const float* g;
    float* y;
    float* row_max;    // in (bwd) or out (fwd), per row
    float* row_sum;
    const long long* targets;
    float* row_term;   // CE: per-row log_softmax at the target
    unsigned long long rows;
    unsigned long long L;
    unsigned seg;      // floats per CTA slice (multiple of 4)
    unsigned* err;
};

// ---- row-sum helpers ----------------------------------------------------------
// exp(x) for the terms of a row sum (x = logit - row max <= 0): 2^(x log2 e)
// on the SFU's ex2.approx. Rounding x * log2(e) to float perturbs a term by
// at most |x| * 2^-24 * log2(e) * ln 2 relative, so the terms near the max
// (which carry the sum) are within a few float ulps and the far ones, though
// less accurate, are exponentially small: the row sum stays within about
// 2e-7 of the reference's double sum of expf, far inside the 1e-5 tolerance.
// Per-element outputs keep expf. x is clamped (NaN-preserving) at -110,
// where 2^t is already 0 (and -inf logits give 0, not NaN).
constexpr float kL2e = 0x1.715476p+0f;  // log2(e) rounded to float
__device__ __forceinline__ float exp_sum_term(float x) {
    float xc;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(xc) : "f"(x), "f"(-110.0f));
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(xc * kL2e));
    return e;
}

// e^t for per-element outputs on the SFU: 2^(t * log2 e), the product
// rounded to float. The rounding perturbs the result by at most
// |t| * 2^-24 * log2(e) * ln 2 relative (1.2e-6 at |t| = 20, 4.8e-6 at 80,
// where e^t < 2e-35), plus ex2.approx's 2 ulp; results below 2^-126 flush
// to zero (an absolute error under 1.2e-38), e^-inf = 0, e^+inf = inf, NaN
// stays NaN. Two instructions per element where expf takes about ten: the
// softmax outputs and the softmax backward evaluate one to three of these
// per element and are issue-bound otherwise (keeping subnormal results costs
// softmax's forward 4 points of HBM bandwidth).
__device__ __forceinline__ float exp_sfu(float t) {
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(t * kL2e));
    return e;
}
// 2^(t log2 e) for row-sum terms, subnormal results flushed to zero.
__device__ __forceinline__ float exp_term(float t) {
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(t * kL2e));
    return e;
}

// Row sums accumulate per float4: the four terms in float ((x + y) + (z + w)),
// that partial in double -- one float->double conversion per four elements
// rather than per element (the conversion pipe runs at 16/clk/SM and the
// SFU's ex2 shares it). A float partial that is not finite (overflow of large
// upstream gradients) is replaced by the four terms added in double, so an
// infinity appears only where the double sum has one.
__device__ __forceinline__ double quad_sum(float4 v) {
    const float q = (v.x + v.y) + (v.z + v.w);
    if (isfinite(q)) return static_cast<double>(q);
    return ((static_cast<double>(v.x) + static_cast<double>(v.y)) + static_cast<double>(v.z)) + static_cast<double>(v.w);
}

// ---- block / cluster combines (fixed order: the same result in every CTA) ----
__device__ __forceinline__ float block_fmax(float v, float* scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = lane < nw ? scratch[lane] : -INFINITY;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, m));
    return t;
}

__device__ __forceinline__ unsigned long long block_umin(unsigned long long v, unsigned long long* scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, m));
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    unsigned long long t = lane < nw ? scratch[lane] : ~0ull;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) t = min(t, __shfl_xor_sync(0xffffffffu, t, m));
    return t;
}

__device__ __forceinline__ float cluster_fmax(cg::cluster_group& cluster, float mine, float* slot, unsigned C) {
    if (threadIdx.x == 0) *slot = mine;
    cluster.sync();
    float m = -INFINITY;
    for (unsigned r = 0; r < C; ++r) m = fmaxf(m, *cluster.map_shared_rank(slot, r));
    return m;
}

__device__ __forceinline__ unsigned long long cluster_umin(cg::cluster_group& cluster, unsigned long long mine,
                                                           unsigned long long* slot, unsigned C) {
    if (threadIdx.x == 0) *slot = mine;
    cluster.sync();
    unsigned long long m = ~0ull;
    for (unsigned r = 0; r < C; ++r) m = min(m, *cluster.map_shared_rank(slot, r));
    return m;
}

__device__ __forceinline__ double cluster_sum(cg::cluster_group& cluster, double mine, double* slot, unsigned C) {
    if (threadIdx.x == 0) *slot = mine;
    cluster.sync();
    double t = 0.0;
    for (unsigned r = 0; r < C; ++r) t += *cluster.map_shared_rank(slot, r);
    return t;
}

__device__ __forceinline__ float4 ld_smem4(const float* s, unsigned j) { return reinterpret_cast<const float4*>(s)[j]; }

// One cluster per row. Dynamic shared memory: [slice of x][slice of g].
// BULK: the slice was staged with a TMA bulk copy, and the row length, the
// slice start and the slice length are multiples of 4, so every pass is
// float4-wide (shared and global).
template <int MODE, bool BULK>
__global__ void __launch_bounds__(kThreads)
row_kernel(const RowArgs a, unsigned long long row0) {
    extern __shared__ __align__(128) float smem[];
    __shared__ unsigned long long bar;
    __shared__ double s_red[32];
    __shared__ float s_f[32];
    __shared__ unsigned long long s_u[32];
    __shared__ float x_max;               // cluster exchange slots, one per phase
    __shared__ unsigned long long x_idx;
    __shared__ double x_sum;

    cg::cluster_group cluster = cg::this_cluster();
    const unsigned C = cluster.num_blocks();
    const unsigned rank = cluster.block_rank();
    const unsigned long long row = row0 + blockIdx.x / C;
    if (row >= a.rows) return;  // whole cluster exits together (same row)

    constexpr bool FWD = MODE == LSM_FWD || MODE == SM_FWD || MODE == CE_FWD;
    constexpr bool STAGE_X = FWD || MODE == SM_BWD;
    constexpr bool STAGE_G = MODE == LSM_BWD || MODE == SM_BWD;
    const unsigned long long c0 = static_cast<unsigned long long>(rank) * a.seg;
    const unsigned n = c0 < a.L ? static_cast<unsigned>(min(static_cast<unsigned long long>(a.seg), a.L - c0)) : 0u;
    const unsigned n4 = n / 4;
    float* sx = smem;
    float* sg = smem + (STAGE_X ? a.seg : 0);
    const float* xrow = a.x + row * a.L + c0;
    const float* grow = STAGE_G ? a.g + row * a.L + c0 : nullptr;
    float* yrow = a.y ? a.y + row * a.L + c0 : nullptr;

    // ---- stage the slice(s) -----------------------------------------------------
    if constexpr (BULK) {
        const unsigned bytes = n * 4u * ((STAGE_X ? 1u : 0u) + (STAGE_G ? 1u : 0u));
        if (threadIdx.x == 0) {
            mbar_init(&bar, 1);
            mbar_fence_init();
        }
        __syncthreads();
        if (threadIdx.x == 0 && bytes) {
            mbar_expect_tx(&bar, bytes);
            if (STAGE_X) bulk_load(sx, xrow, n * 4u, &bar);
            if (STAGE_G) bulk_load(sg, grow, n * 4u, &bar);
        }
        if (bytes) mbar_wait_bounded(&bar, 0, a.err);
    } else {
        for (unsigned k = threadIdx.x; k < n; k += kThreads) {
            if (STAGE_X) sx[k] = __ldg(xrow + k);
            if (STAGE_G) sg[k] = __ldg(grow + k);
        }
        __syncthreads();
    }

    if constexpr (FWD) {
        // ---- row max m: fmaxf skips NaN; then the scan's exact rules ------------
        float mloc = -INFINITY;
        if constexpr (BULK) {
            for (unsigned j = threadIdx.x; j < n4; j += kThreads) {
                const float4 v = ld_smem4(sx, j);
                mloc = fmaxf(mloc, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
            }
        } else {
            for (unsigned k = threadIdx.x; k < n; k += kThreads) mloc = fmaxf(mloc, sx[k]);
        }
        float m = cluster_fmax(cluster, block_fmax(mloc, s_f), &x_max, C);
        const float first = __ldg(a.x + row * a.L);
        if (first != first) {
            m = first;  // the scan never leaves a NaN at index 0
        } else if (m == 0.0f) {
            // a zero maximum is the FIRST zero of the row (its sign matters);
            // the condition is the same in every CTA of the cluster
            unsigned long long idx = ~0ull;
            for (unsigned k = threadIdx.x; k < n; k += kThreads)
                if (sx[k] == 0.0f) { idx = c0 + k; break; }
            idx = cluster_umin(cluster, block_umin(idx, s_u), &x_idx, C);
            m = __ldg(a.x + row * a.L + idx);
        }
        // ---- s = float(double sum of expf(x - m)) ----
        double acc0 = 0.0, acc1 = 0.0;
        if constexpr (BULK) {
            for (unsigned j = threadIdx.x; j < n4; j += kThreads) {
                const float4 v = ld_smem4(sx, j);
                acc0 += quad_sum(make_float4(exp_sum_term(v.x - m), exp_sum_term(v.y - m), exp_sum_term(v.z - m),
                                             exp_sum_term(v.w - m)));
            }
        } else {
            for (unsigned k = threadIdx.x; k < n; k += kThreads) acc0 += static_cast<double>(expf(sx[k] - m));
        }
        const float s = static_cast<float>(cluster_sum(cluster, block_sum(acc0 + acc1, s_red), &x_sum, C));
        const float l = logf(s);
        if (rank == 0 && threadIdx.x == 0) {
            if (a.row_max) a.row_max[row] = m;
            if (a.row_sum) a.row_sum[row] = s;
        }
        if constexpr (MODE == CE_FWD) {
            const long long t = __ldg(a.targets + row);
            if (t < 0 || static_cast<unsigned long long>(t) >= a.L) {
                if (rank == 0 && threadIdx.x == 0) { atomicOr(a.err, kErrBadTarget); a.row_term[row] = 0.0f; }
            } else if (threadIdx.x == 0 && static_cast<unsigned long long>(t) >= c0 &&
                       static_cast<unsigned long long>(t) < c0 + n) {
                a.row_term[row] = (sx[t - c0] - m) - l;
            }
        } else {
            auto f = [&](float v) {
                const float ls = (v - m) - l;
                return MODE == SM_FWD ? expf(ls) : ls;
            };
            if constexpr (BULK) {
                for (unsigned j = threadIdx.x; j < n4; j += kThreads) {
                    const float4 v = ld_smem4(sx, j);
                    st4_stream(yrow + 4 * j, make_float4(f(v.x), f(v.y), f(v.z), f(v.w)));
                }
            } else {
                for (unsigned k = threadIdx.x; k < n; k += kThreads) yrow[k] = f(sx[k]);
            }
        }
    } else {
        const float m = __ldg(a.row_max + row);
        const float s = __ldg(a.row_sum + row);
        if constexpr (MODE == LSM_BWD) {
            // dx = g + ((float(sum(-g)) / s) + 0) * expf(x - m)
            double acc0 = 0.0, acc1 = 0.0;
            if constexpr (BULK) {
                for (unsigned j = threadIdx.x; j < n4; j += kThreads) {
                    const float4 g = ld_smem4(sg, j);
                    acc0 += quad_sum(make_float4(-g.x, -g.y, -g.z, -g.w));
                }
            } else {
                for (unsigned k = threadIdx.x; k < n; k += kThreads) acc0 += static_cast<double>(-sg[k]);
            }
            const float dl = static_cast<float>(cluster_sum(cluster, block_sum(acc0 + acc1, s_red), &x_sum, C));
            const float de = (dl / s) + 0.0f;
            if constexpr (BULK) {
                for (unsigned j = threadIdx.x; j < n4; j += kThreads) {
                    const float4 g = ld_smem4(sg, j);
                    const float4 x = ld4_stream(xrow + 4 * j);
                    st4_stream(yrow + 4 * j, make_float4(g.x + de * expf(x.x - m), g.y + de * expf(x.y - m),
                                                         g.z + de * expf(x.z - m), g.w + de * expf(x.w - m)));
                }
            } else {
                for (unsigned k = threadIdx.x; k < n; k += kThreads) yrow[k] = sg[k] + de * expf(__ldg(xrow + k) - m);
            }
        } else {  // SM_BWD: gy = g * y; dx = gy + ((float(sum(-gy)) / s) + 0) * expf(x - m)
            const float l = logf(s);
            double acc0 = 0.0, acc1 = 0.0;
            auto gy_of = [&](float x, float g) { return g * expf((x - m) - l); };
            if constexpr (BULK) {
                for (unsigned j = threadIdx.x; j < n4; j += kThreads) {
                    const float4 x = ld_smem4(sx, j), g = ld_smem4(sg, j);
                    const float4 gy = make_float4(gy_of(x.x, g.x), gy_of(x.y, g.y), gy_of(x.z, g.z), gy_of(x.w, g.w));
                    reinterpret_cast<float4*>(sg)[j] = gy;
                    acc0 += quad_sum(make_float4(-gy.x, -gy.y, -gy.z, -gy.w));
                }
            } else {
                for (unsigned k = threadIdx.x; k < n; k += kThreads) {
                    const float gy = gy_of(sx[k], sg[k]);
                    sg[k] = gy;
                    acc0 += static_cast<double>(-gy);
                }
            }
            const float dl = static_cast<float>(cluster_sum(cluster, block_sum(acc0 + acc1, s_red), &x_sum, C));
            const float de = (dl / s) + 0.0f;
            if constexpr (BULK) {
                for (unsigned j = threadIdx.x; j < n4; j += kThreads) {
                    const float4 x = ld_smem4(sx, j), gy = ld_smem4(sg, j);
                    st4_stream(yrow + 4 * j, make_float4(gy.x + de * expf(x.x - m), gy.y + de * expf(x.y - m),
                                                         gy.z + de * expf(x.z - m), gy.w + de * expf(x.w - m)));
                }
            } else {
                for (unsigned k = threadIdx.x; k < n; k += kThreads) yrow[k] = sg[k] + de * expf(sx[k] - m);
            }
        }
    }
    // Keep this CTA's shared memory alive until every rank has read it.
    cluster.sync();
}

// Column kernel: one thread per (o, i) position walks the axis in global
// memory. Handles any [outer, length, inner] (inner >= 1).
template <int MODE>
__global__ void __launch_bounds__(kThreads)
col_kernel(const RowArgs a, unsigned long long outer, unsigned long long inner) {
    const unsigned long long count = outer * inner;
    const unsigned long long stride = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
    const unsigned long long L = a.L;
    for (unsigned long long k = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x; k < count;
         k += stride) {
        const unsigned long long ob = k / inner, i = k - ob * inner;
        const unsigned long long base = ob * L * inner + i;
        const float* x = a.x + base;
        float m, s;
        if constexpr (MODE == LSM_FWD || MODE == SM_FWD || MODE == CE_FWD) {
            MaxCand c{0.0f, -1};
            for (unsigned long long j = 0; j < L; ++j) c = max_take(c, x[j * inner], static_cast<long long>(j));
            m = x[0] != x[0] ? x[0] : c.v;
            double acc = 0.0;
            for (unsigned long long j = 0; j < L; ++j) acc += static_cast<double>(expf(x[j * inner] - m));
            s = static_cast<float>(acc);
            const float l = logf(s);
            if (a.row_max) a.row_max[k] = m;
            if (a.row_sum) a.row_sum[k] = s;
            if constexpr (MODE == CE_FWD) {
                const long long t = a.targets[k];
                if (t < 0 || static_cast<unsigned long long>(t) >= L) {
                    atomicOr(a.err, kErrBadTarget);
                    a.row_term[k] = 0.0f;
                } else {
                    a.row_term[k] = (x[t * inner] - m) - l;
                }
            } else {
                for (unsigned long long j = 0; j < L; ++j) {
                    const float ls = (x[j * inner] - m) - l;
                    a.y[base + j * inner] = MODE == SM_FWD ? expf(ls) : ls;
                }
            }
        } else {
            m = a.row_max[k];
            s = a.row_sum[k];
            const float* g = a.g + base;
            if constexpr (MODE == LSM_BWD) {
                double acc = 0.0;
                for (unsigned long long j = 0; j < L; ++j) acc += static_cast<double>(-g[j * inner]);
                const float de = (static_cast<float>(acc) / s) + 0.0f;
                for (unsigned long long j = 0; j < L; ++j)
                    a.y[base + j * inner] = g[j * inner] + de * expf(x[j * inner] - m);
            } else {
                const float l = logf(s);
                double acc = 0.0;
                for (unsigned long long j = 0; j < L; ++j) {
                    const float y = expf((x[j * inner] - m) - l);
                    acc += static_cast<double>(-(g[j * inner] * y));
                }
                const float de = (static_cast<float>(acc) / s) + 0.0f;
                for (unsigned long long j = 0; j < L; ++j) {
                    const float y = expf((x[j * inner] - m) - l);
                    const float gy = g[j * inner] * y;
                    a.y[base + j * inner] = gy + de * expf(x[j * inner] - m);
                }
            }
        }
    }
}

// loss = (-(float)(sum of row terms, double)) / B; partial = the double sum.
__global__ void __launch_bounds__(1024)
ce_finish_kernel(const float* __restrict__ row_term, unsigned long long rows, float batch_total,
                 float* __restrict__ loss, double* __restrict__ partial) {
    __shared__ double s_red[32];
    double acc = 0.0;
    for (unsigned long long r = threadIdx.x; r < rows; r += blockDim.x) acc += static_cast<double>(row_term[r]);
    acc = block_sum(acc, s_red);
    if (threadIdx.x == 0) {
        const float t = static_cast<float>(acc);
        const float neg = -t;
        if (loss) *loss = neg / batch_total;
        if (partial) *partial = acc;
    }
}

// Cross-entropy backward: a streaming pass, no reduction needed.
template <bool VEC>
__global__ void __launch_bounds__(kThreads)
ce_backward_kernel(const float* __restrict__ x, const long long* __restrict__ targets,
                   const float* __restrict__ row_max, const float* __restrict__ row_sum,
                   const float* __restrict__ upstream, unsigned long long rows, unsigned long long classes,
                   float batch_total, float* __restrict__ dx) {
    const float u = __ldg(upstream);
    const float dn = u / batch_total;
    const float dt = -dn;
    const float dp = dt + 0.0f;
    // dl = float(sum over the row of -(dp * onehot)) accumulated from +0.0.
    float dl;
    if (dp == 0.0f) dl = 0.0f;
    else if (isinf(dp) && classes > 1) dl = __int_as_float(0x7fc00000);
    else dl = -dp;
    for (unsigned long long row = blockIdx.x; row < rows; row += gridDim.x) {
        const float m = __ldg(row_max + row);
        const float s = __ldg(row_sum + row);
        const long long t = __ldg(targets + row);
        const float de = (dl / s) + 0.0f;
        const float* xr = x + row * classes;
        float* dr = dx + row * classes;
        if constexpr (VEC) {
            for (unsigned long long c = threadIdx.x * 4ull; c < classes; c += kThreads * 4ull) {
                const float4 xv = ldg4(xr + c);
                float4 o;
                o.x = dp * (static_cast<long long>(c) == t ? 1.0f : 0.0f) + de * expf(xv.x - m);
                o.y = dp * (static_cast<long long>(c + 1) == t ? 1.0f : 0.0f) + de * expf(xv.y - m);
                o.z = dp * (static_cast<long long>(c + 2) == t ? 1.0f : 0.0f) + de * expf(xv.z - m);
                o.w = dp * (static_cast<long long>(c + 3) == t ? 1.0f : 0.0f) + de * expf(xv.w - m);
                st4_stream(dr + c, o);
            }
        } else {
            for (unsigned long long c = threadIdx.x; c < classes; c += kThreads)
                dr[c] = dp * (static_cast<long long>(c) == t ? 1.0f : 0.0f) + de * expf(__ldg(xr + c) - m);
        }
    }
}

// The same dlogits over the flat [rows, classes] array as a chunked stream
// (classes % 4 == 0, rows * classes / 4 < 2^32): CTA b owns float4 groups
// [kChunk4 * b, kChunk4 * (b + 1)), four per thread, all loads first; a
// group's row comes from a FastDiv by classes / 4, and the row's m, s, target
// and de = (dl / s) + 0 are reloaded only when the row changes (at most four
// times per thread for classes >= 1024). The exponential is
// exp_sfu (within 2e-6 relative of expf for |x - m| <= 20).
__global__ void __launch_bounds__(kThreads)
ce_backward_stream(const float* __restrict__ x, const long long* __restrict__ targets,
                   const float* __restrict__ row_max, const float* __restrict__ row_sum,
                   const float* __restrict__ upstream, unsigned long long n4, FastDiv classes4,
                   float batch_total, float* __restrict__ dx) {
    const float u = __ldg(upstream);
    const float dn = u / batch_total;
    const float dt = -dn;
    const float dp = dt + 0.0f;
    float dl;
    if (dp == 0.0f) dl = 0.0f;
    else if (isinf(dp) && classes4.divisor * 4ull > 1) dl = __int_as_float(0x7fc00000);
    else dl = -dp;
    const unsigned long long base = static_cast<unsigned long long>(blockIdx.x) * kChunk4 + threadIdx.x;
    float4 xv[kStreamRounds];
#pragma unroll
    for (unsigned k = 0; k < kStreamRounds; ++k) {
        const unsigned long long i = base + k * kStreamThreads;
        if (i < n4) xv[k] = ldg4(x + 4 * i);
    }
    unsigned cur = 0xffffffffu;
    float m = 0.0f, de = 0.0f;
    long long t = -1;
#pragma unroll
    for (unsigned k = 0; k < kStreamRounds; ++k) {
        const unsigned long long i = base + k * kStreamThreads;
        if (i >= n4) break;
        unsigned row, c4;
        classes4.divmod(static_cast<unsigned>(i), row, c4);
        if (row != cur) {
            cur = row;
            m = __ldg(row_max + row);
            de = (dl / __ldg(row_sum + row)) + 0.0f;
            t = __ldg(targets + row);
        }
        const long long c = 4ll * c4;
        float4 o;
        o.x = dp * (c == t ? 1.0f : 0.0f) + de * exp_sfu(xv[k].x - m);
        o.y = dp * (c + 1 == t ? 1.0f : 0.0f) + de * exp_sfu(xv[k].y - m);
        o.z = dp * (c + 2 == t ? 1.0f : 0.0f) + de * exp_sfu(xv[k].z - m);
        o.w = dp * (c + 3 == t ? 1.0f : 0.0f) + de * exp_sfu(xv[k].w - m);
        st4(dx + 4 * i, o);
    }
}

// ---------------------------------------------------------------------------
// Pipelined row kernel for 16-byte-aligned rows whose length is a multiple
// of 4: a persistent grid of clusters, cluster k handling rows k,
// k + clusters, ... Each CTA double-buffers its slice of the row in shared
// memory ([x slice][g slice] per stage; x in every mode, g in the backward
// ones): the bulk copy of the next row's slice is issued when the current
// row starts, so the copy engine streams HBM while the CTA computes.
//
// Waiting: only thread 0 polls an mbarrier (stage copies and exchanges);
// __syncthreads_and then releases the CTA and shares whether the wait
// succeeded, so no warp spins on shared memory.
//
// Cluster exchange without cluster barriers: every warp pushes its partial
// into slot [rank * kWarps + warp] of EVERY CTA of the cluster with st.async,
// whose completion is counted in bytes on the receiving CTA's mbarrier; each
// CTA then folds its C * kWarps slots lane-parallel with a fixed xor tree (the
// same result in every CTA). No release fence is involved (a cluster
// barrier's would wait for all of the thread's global stores in flight).
// Slots and mbarriers are double-buffered by row parity: a CTA can run at
// most one exchange ahead of a peer, since it needs that peer's contribution
// to finish the previous one.
// ---------------------------------------------------------------------------
constexpr unsigned kWarps = kThreads / 32;
constexpr unsigned kMaxCluster = 8;
constexpr unsigned kStageFloats = 8192;     // floats per stage (x and g together)
constexpr unsigned kStageFloatsMax = 24576; // ... at cluster size 8 (96 KB a stage, two stages)

template <int MODE> struct PipeTraits {
    static constexpr bool FWD = MODE == LSM_FWD || MODE == SM_FWD || MODE == CE_FWD;
    static constexpr bool STAGE_G = MODE == LSM_BWD || MODE == SM_BWD;
    static constexpr unsigned NBUF = STAGE_G ? 2u : 1u;
    // resident CTAs per SM the register budget is sized for (each holds
    // 64 KB of stages: three fit)
    static constexpr unsigned MIN_CTAS = 3u;
};

__device__ __forceinline__ float warp_fmax(float v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}
__device__ __forceinline__ unsigned long long warp_umin(unsigned long long v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}
__device__ __forceinline__ unsigned mapa_cluster(unsigned cta_addr, unsigned rank) {
    unsigned r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(cta_addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_async_b64(unsigned addr, unsigned long long v, unsigned bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b64 [%0], %1, [%2];" ::"r"(addr), "l"(v),
                 "r"(bar)
                 : "memory");
}
__device__ __forceinline__ unsigned long long bits64(double v) { return static_cast<unsigned long long>(__double_as_longlong(v)); }
__device__ __forceinline__ unsigned long long bits64(unsigned long long v) { return v; }

// Push this warp's value (lane 0's) to every CTA of the cluster, then wait
// (thread 0, bounded) for all C * kWarps values of this exchange to land in
// this CTA's `slots`. Returns the CTA-uniform success flag. When an earlier
// wait failed (ok false) the values are still sent, so no peer is left
// waiting, but nobody waits here.
template <class T>
__device__ __forceinline__ bool exchange(T v, T* slots, unsigned long long* bar, unsigned parity, unsigned C,
                                         unsigned rank, bool ok, unsigned* err) {
    if (threadIdx.x == 0) mbar_expect_tx(bar, C * kWarps * static_cast<unsigned>(sizeof(T)));
    if ((threadIdx.x & 31) == 0) {
        const unsigned slot = smem_addr(slots + rank * kWarps + (threadIdx.x >> 5));
        const unsigned b = smem_addr(bar);
        for (unsigned r = 0; r < C; ++r) st_async_b64(mapa_cluster(slot, r), bits64(v), mapa_cluster(b, r));
    }
    bool good = ok;
    if (threadIdx.x == 0 && ok) good = mbar_wait_bounded(bar, parity, err);
    return __syncthreads_and(good) != 0;
}

__device__ __forceinline__ unsigned long long fold_umin(const unsigned long long* slots, unsigned C) {
    unsigned long long t = ~0ull;
    for (unsigned i = threadIdx.x & 31; i < C * kWarps; i += 32) t = min(t, slots[i]);
    return warp_umin(t);
}
__device__ __forceinline__ double fold_sum(const double* slots, unsigned C) {
    double t = 0.0;
    for (unsigned i = threadIdx.x & 31; i < C * kWarps; i += 32) t += slots[i];
    return warp_sum(t);
}
__device__ __forceinline__ float4 neg4(float4 v) { return make_float4(-v.x, -v.y, -v.z, -v.w); }

// The per-warp (max, sum of exp(x - max)) pairs of a row: one exchange of
// 16-byte slots {double(m_w), s_w}.
__device__ __forceinline__ void st_async_v2_b64(unsigned addr, unsigned long long a, unsigned long long b,
                                                unsigned bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.b64 [%0], {%1, %2}, [%3];" ::"r"(addr),
                 "l"(a), "l"(b), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ bool exchange_pair(float m, double s, double2* slots, unsigned long long* bar,
                                              unsigned parity, unsigned C, unsigned rank, bool ok, unsigned* err) {
    if (threadIdx.x == 0) mbar_expect_tx(bar, C * kWarps * static_cast<unsigned>(sizeof(double2)));
    if ((threadIdx.x & 31) == 0) {
        const unsigned slot = smem_addr(slots + rank * kWarps + (threadIdx.x >> 5));
        const unsigned b = smem_addr(bar);
        for (unsigned r = 0; r < C; ++r)
            st_async_v2_b64(mapa_cluster(slot, r), bits64(static_cast<double>(m)), bits64(s), mapa_cluster(b, r));
    }
    bool good = ok;
    if (threadIdx.x == 0 && ok) good = mbar_wait_bounded(bar, parity, err);
    return __syncthreads_and(good) != 0;
}
// Row max m = max of the m_w (fmaxf skips NaN) and s = sum of s_w * exp(m_w - m)
// in double, lane-parallel then a fixed xor tree. A slot with m_w = -inf
// carries s_w = 0 (or NaN): its weight exp(-inf - m) is 0 and NaN survives.
__device__ __forceinline__ void fold_pairs(const double2* slots, unsigned C, float& m, double& s) {
    float mm = -INFINITY;
    for (unsigned i = threadIdx.x & 31; i < C * kWarps; i += 32) mm = fmaxf(mm, static_cast<float>(slots[i].x));
    mm = warp_fmax(mm);
    double t = 0.0;
    for (unsigned i = threadIdx.x & 31; i < C * kWarps; i += 32)
        t += slots[i].y * static_cast<double>(expf(static_cast<float>(slots[i].x) - mm));
    m = mm;
    s = warp_sum(t);
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, PipeTraits<MODE>::MIN_CTAS)
row_pipe_kernel(const RowArgs a) {
    using T = PipeTraits<MODE>;
    extern __shared__ __align__(128) float smem[];
    __shared__ unsigned long long bar[2];        // stage copies
    __shared__ unsigned long long xbar[3][2];    // exchanges: max, first-zero index, sum
    __shared__ double2 xs_ms[2][kMaxCluster * kWarps];
    __shared__ unsigned long long xs_idx[2][kMaxCluster * kWarps];
    __shared__ double xs_sum[2][kMaxCluster * kWarps];

    cg::cluster_group cluster = cg::this_cluster();
    const unsigned C = cluster.num_blocks();
    const unsigned rank = cluster.block_rank();
    const unsigned long long nclusters = gridDim.x / C;
    const unsigned long long cid = blockIdx.x / C;
    const unsigned long long c0 = static_cast<unsigned long long>(rank) * a.seg;
    const unsigned n = c0 < a.L ? static_cast<unsigned>(min(static_cast<unsigned long long>(a.seg), a.L - c0)) : 0u;
    const unsigned n4 = n / 4;
    const unsigned stage_floats = a.seg * T::NBUF;
    const unsigned bytes = n * 4u * T::NBUF;

    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        for (int k = 0; k < 3; ++k) {
            mbar_init(&xbar[k][0], 1);
            mbar_init(&xbar[k][1], 1);
        }
        mbar_fence_init();
    }
    // every CTA's mbarriers are initialised before any peer signals them
    cluster.sync();
    unsigned loads[2] = {0, 0}, seen[2] = {0, 0};  // thread 0: copies issued / completed per stage
    auto issue = [&](unsigned st, unsigned long long row) {
        float* base = smem + st * stage_floats;
        mbar_expect_tx(&bar[st], bytes);
        bulk_load(base, a.x + row * a.L + c0, n * 4u, &bar[st]);
        if (T::STAGE_G) bulk_load(base + a.seg, a.g + row * a.L + c0, n * 4u, &bar[st]);
        ++loads[st];
    };
    if (threadIdx.x == 0 && bytes && cid < a.rows) issue(0, cid);

    bool ok = true;                   // CTA-uniform: every wait so far completed
    unsigned it = 0, nz = 0;          // rows done; first-zero exchanges done
    for (unsigned long long row = cid; row < a.rows; row += nclusters, ++it) {
        const unsigned st = it & 1u, par = (it >> 1) & 1u;
        float m_saved = 0.0f, s_saved = 0.0f;
        if constexpr (!T::FWD) {
            m_saved = __ldg(a.row_max + row);
            s_saved = __ldg(a.row_sum + row);
        }
        bool good = ok;
        if (threadIdx.x == 0 && ok && bytes) {
            good = mbar_wait_bounded(&bar[st], par, a.err);
            if (good) ++seen[st];
        }
        // publishes the stage; every thread is also done with the other stage
        // (the previous row), which is refilled with the next row right away
        ok = __syncthreads_and(good) != 0;
        if (threadIdx.x == 0 && ok && bytes && row + nclusters < a.rows) {
            fence_proxy_async_smem();
            issue(st ^ 1u, row + nclusters);
        }
        float* sx = smem + st * stage_floats;
        float* sg = sx + a.seg;
        float* yrow = a.y ? a.y + row * a.L + c0 : nullptr;

        if constexpr (T::FWD) {
            const float first = __ldg(a.x + row * a.L);
            // ---- per warp: its max m_w (fmaxf skips NaN) and s_w = sum of
            // exp(x - m_w); ONE cluster exchange of the (m_w, s_w) pairs gives
            // the row max m and s = sum of s_w * exp(m_w - m) ----
            float mloc = -INFINITY;
            for (unsigned j = threadIdx.x; j < n4; j += kThreads) {
                const float4 v = ld_smem4(sx, j);
                mloc = fmaxf(mloc, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
            }
            const float mw = warp_fmax(mloc);
            double part = 0.0;
            for (unsigned j = threadIdx.x; j < n4; j += kThreads) {
                const float4 v = ld_smem4(sx, j);
                part += quad_sum(make_float4(exp_sum_term(v.x - mw), exp_sum_term(v.y - mw), exp_sum_term(v.z - mw),
                                             exp_sum_term(v.w - mw)));
            }
            double sw = warp_sum(part);
            if (mw == -INFINITY) {
                // no finite value among this warp's elements: they add 0 to
                // the row sum, or NaN when one of them is NaN
                bool nan = false;
                for (unsigned j = threadIdx.x; j < n4; j += kThreads) {
                    const float4 v = ld_smem4(sx, j);
                    nan = nan || v.x != v.x || v.y != v.y || v.z != v.z || v.w != v.w;
                }
                sw = __any_sync(0xffffffffu, nan) ? static_cast<double>(__int_as_float(0x7fc00000)) : 0.0;
            }
            ok = exchange_pair(mw, sw, xs_ms[st], &xbar[0][st], par, C, rank, ok, a.err);
            float m;
            double s_row;
            fold_pairs(xs_ms[st], C, m, s_row);
            // a row of -inf only: the reference's x - m is NaN everywhere
            if (m == -INFINITY) s_row = static_cast<double>(__int_as_float(0x7fc00000));
            if (first != first) {
                m = first;  // the scan never leaves a NaN at index 0
            } else if (m == 0.0f) {
                // a zero maximum is the FIRST zero of the row (its sign
                // matters); the condition is the same in every CTA
                unsigned long long idx = ~0ull;
                for (unsigned k = threadIdx.x; k < n; k += kThreads)
                    if (sx[k] == 0.0f) { idx = c0 + k; break; }
                const unsigned zb = nz & 1u;
                ok = exchange(warp_umin(idx), xs_idx[zb], &xbar[1][zb], (nz >> 1) & 1u, C, rank, ok, a.err);
                idx = fold_umin(xs_idx[zb], C);
                ++nz;
                if (idx < a.L) m = __ldg(a.x + row * a.L + idx);
            }
            const float s = static_cast<float>(s_row);
            const float l = logf(s);
            if (rank == 0 && threadIdx.x == 0) {
                if (a.row_max) a.row_max[row] = m;
                if (a.row_sum) a.row_sum[row] = s;
            }
            if constexpr (MODE == CE_FWD) {
                const long long t = __ldg(a.targets + row);
                if (t < 0 || static_cast<unsigned long long>(t) >= a.L) {
                    if (rank == 0 && threadIdx.x == 0) { atomicOr(a.err, kErrBadTarget); a.row_term[row] = 0.0f; }
                } else if (threadIdx.x == 0 && static_cast<unsigned long long>(t) >= c0 &&
                           static_cast<unsigned long long>(t) < c0 + n) {
                    a.row_term[row] = (sx[t - c0] - m) - l;
                }
            } else {
                auto f = [&](float v) {
                    const float ls = (v - m) - l;
                    return MODE == SM_FWD ? expf(ls) : ls;
                };
                for (unsigned j = threadIdx.x; j < n4; j += kThreads) {
                    const float4 v = ld_smem4(sx, j);
                    st4_stream(yrow + 4 * j, make_float4(f(v.x), f(v.y), f(v.z), f(v.w)));
                }
            }
        } else if constexpr (MODE == LSM_BWD) {
            // dx = g + ((float(sum(-g)) / s) + 0) * expf(x - m)
            const float m = m_saved, s = s_saved;
            double part = 0.0;
            for (unsigned j = threadIdx.x; j < n4; j += kThreads) part += quad_sum(neg4(ld_smem4(sg, j)));
            ok = exchange(warp_sum(part), xs_sum[st], &xbar[2][st], par, C, rank, ok, a.err);
            const float dl = static_cast<float>(fold_sum(xs_sum[st], C));
            const float de = (dl / s) + 0.0f;
            for (unsigned j = threadIdx.x; j < n4; j += kThreads) {
                const float4 g = ld_smem4(sg, j), x = ld_smem4(sx, j);
                st4_stream(yrow + 4 * j, make_float4(g.x + de * expf(x.x - m), g.y + de * expf(x.y - m),
                                                     g.z + de * expf(x.z - m), g.w + de * expf(x.w - m)));
            }
        } else {  // SM_BWD: gy = g * y; dx = gy + ((float(sum(-gy)) / s) + 0) * expf(x - m)
            const float m = m_saved, s = s_saved;
            const float l = logf(s);
            auto gy_of = [&](float x, float g) { return g * expf((x - m) - l); };
            double part = 0.0;
            for (unsigned j = threadIdx.x; j < n4; j += kThreads) {
                const float4 x = ld_smem4(sx, j), g = ld_smem4(sg, j);
                const float4 gy = make_float4(gy_of(x.x, g.x), gy_of(x.y, g.y), gy_of(x.z, g.z), gy_of(x.w, g.w));
                reinterpret_cast<float4*>(sg)[j] = gy;
                part += quad_sum(neg4(gy));
            }
            ok = exchange(warp_sum(part), xs_sum[st], &xbar[2][st], par, C, rank, ok, a.err);
            const float dl = static_cast<float>(fold_sum(xs_sum[st], C));
            const float de = (dl / s) + 0.0f;
            for (unsigned j = threadIdx.x; j < n4; j += kThreads) {
                const float4 x = ld_smem4(sx, j), gy = ld_smem4(sg, j);
                st4_stream(yrow + 4 * j, make_float4(gy.x + de * expf(x.x - m), gy.y + de * expf(x.y - m),
                                                     gy.z + de * expf(x.z - m), gy.w + de * expf(x.w - m)));
            }
        }
    }
    // Only a wait that gave up can leave a copy in flight: wait (bounded)
    // for every copy issued but not seen complete before the memory goes.
    if (!ok && threadIdx.x == 0)
        for (unsigned s2 = 0; s2 < 2; ++s2)
            for (unsigned k = seen[s2]; k < loads[s2]; ++k) mbar_wait_bounded(&bar[s2], k & 1u, a.err);
    // No CTA leaves while a peer may still signal or write its shared memory.
    cluster.sync();
}

// ---------------------------------------------------------------------------
// Cross-entropy forward, aligned rows: one warp per row streams it ONCE from
// HBM (float4, four loads per lane in flight) with an online max / sum --
// no staging, no cluster exchange: CE writes nothing per element, so only the
// row statistics and x[target] are needed. Per 16-value group: if the
// group's max exceeds the lane's running max m, s *= exp(m - max) and m =
// max; then the group's exp(x - m) terms are added (quads in float, then
// double). Lanes fold as sum of s_l * exp(m_l - m) in a fixed xor tree.
// NaN anywhere makes s NaN; a row without a finite value makes s NaN (the
// reference's x - m is NaN); m follows the scan's rules (NaN at index 0, the
// first zero for a zero maximum), found with warp ballots.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fmax4(float4 v) { return fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)); }
__device__ __forceinline__ bool has_nan4(float4 v) { return v.x != v.x || v.y != v.y || v.z != v.z || v.w != v.w; }

// float4 loads per lane in flight: eight (four CTAs of 8 warps per SM at 56
// registers) keep more of the row in flight than four (six CTAs at 40).
constexpr int kCeDepth = 8;

__global__ void __launch_bounds__(kThreads)
ce_rows_kernel(const RowArgs a) {
    const unsigned lane = threadIdx.x & 31;
    const unsigned long long nwarps = (static_cast<unsigned long long>(gridDim.x) * blockDim.x) >> 5;
    const unsigned long long L4 = a.L / 4;
    for (unsigned long long row = (static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
         row < a.rows; row += nwarps) {
        const float4* xr = reinterpret_cast<const float4*>(a.x + row * a.L);
        float m = -INFINITY;
        double s = 0.0;
        bool nan_seen = false;
        auto take = [&](const float4* v, int count) {
            float mx = -INFINITY;
            for (int k = 0; k < count; ++k) mx = fmaxf(mx, fmax4(v[k]));
            if (mx > m) {  // NaN never compares greater
                if (m != -INFINITY) s *= static_cast<double>(expf(m - mx));
                m = mx;
            }
            if (m == -INFINITY) {
                for (int k = 0; k < count; ++k) nan_seen = nan_seen || has_nan4(v[k]);
            } else {
                for (int k = 0; k < count; ++k)
                    s += quad_sum(make_float4(exp_sum_term(v[k].x - m), exp_sum_term(v[k].y - m),
                                              exp_sum_term(v[k].z - m), exp_sum_term(v[k].w - m)));
            }
        };
        unsigned long long j = lane;
        for (; j + 32 * (kCeDepth - 1) < L4; j += 32 * kCeDepth) {
            float4 v[kCeDepth];
#pragma unroll
            for (int k = 0; k < kCeDepth; ++k) v[k] = __ldcs(xr + j + 32 * k);
            take(v, kCeDepth);
        }
        for (; j < L4; j += 32) {
            const float4 v = __ldcs(xr + j);
            take(&v, 1);
        }
        // fold the lanes: m = max of m_l; s = sum of s_l * exp(m_l - m)
        const float mrow = warp_fmax(m);
        double t = m == -INFINITY ? (nan_seen ? static_cast<double>(__int_as_float(0x7fc00000)) : 0.0)
                                  : s * static_cast<double>(expf(m - mrow));
        t = warp_sum(t);
        if (mrow == -INFINITY || __any_sync(0xffffffffu, nan_seen)) t = static_cast<double>(__int_as_float(0x7fc00000));
        float mm = mrow;
        const float first = __ldg(a.x + row * a.L);
        if (first != first) {
            mm = first;
        } else if (mm == 0.0f) {
            // the first zero of the row decides the sign of a zero maximum
            for (unsigned long long q0 = 0; q0 < L4; q0 += 32) {  // warp-uniform trip count
                const unsigned long long q = q0 + lane;
                int pos = -1;
                if (q < L4) {
                    const float4 v = __ldg(xr + q);
                    pos = v.x == 0.0f ? 0 : (v.y == 0.0f ? 1 : (v.z == 0.0f ? 2 : (v.w == 0.0f ? 3 : -1)));
                }
                const unsigned hit = __ballot_sync(0xffffffffu, pos >= 0);
                if (hit) {
                    const int src = __ffs(hit) - 1;
                    const int p = __shfl_sync(0xffffffffu, pos, src);
                    const unsigned long long qq = q0 + src;
                    mm = __ldg(a.x + row * a.L + qq * 4 + p);
                    break;
                }
            }
        }
        const float sf = static_cast<float>(t);
        const float l = logf(sf);
        if (lane == 0) {
            if (a.row_max) a.row_max[row] = mm;
            if (a.row_sum) a.row_sum[row] = sf;
            const long long tg = __ldg(a.targets + row);
            if (tg < 0 || static_cast<unsigned long long>(tg) >= a.L) {
                atomicOr(a.err, kErrBadTarget);
                a.row_term[row] = 0.0f;
            } else {
                a.row_term[row] = (__ldg(a.x + row * a.L + tg) - mm) - l;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Softmax family on aligned rows of up to kRereadMaxL floats, re-read
// design: a group of W warps (W a power of two, 1..16) owns a row.
//   pass 1 streams the row from HBM (four float4 loads per thread in flight)
//          with an L2 evict_last policy and reduces it: forward, an online
//          (max, sum of exp) per lane, rescaled when the lane's max grows;
//          backward, the double sum the chain needs;
//   the warps of the group combine their results through shared memory
//          (one CTA barrier per row, slots double-buffered by iteration);
//   pass 2 re-reads the row, now an L2 hit, with an evict_first policy and
//          writes the output once.
// No cluster lockstep and no shared-memory staging: the loads in flight are
// bounded by registers, not by stage buffers. A CTA holds at most one row per
// group, so the rows in flight (two 16-warp CTAs per SM) take a fraction of
// the 126 MB L2 and HBM sees each input byte once. The per-element arithmetic
// is the pipelined kernel's.
// ---------------------------------------------------------------------------
constexpr unsigned kRThreads = 512;
constexpr unsigned kRWarps = kRThreads / 32;
constexpr unsigned long long kRereadMaxL = 32768;

__device__ __forceinline__ unsigned long long policy_evict_last() {
    unsigned long long p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ unsigned long long policy_evict_first() {
    unsigned long long p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// Read-only float4 load with an L2 cache policy; not allocated in L1.
__device__ __forceinline__ float4 ld4_hint(const float4* p, unsigned long long policy) {
    float4 v;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
        : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
        : "l"(p), "l"(policy));
    return v;
}

// The first zero of a row (whose maximum is zero) decides the maximum's
// sign: one warp scans the row with ballots (warp-uniform trip count).
__device__ __forceinline__ float first_zero(const float* row, unsigned long long L4, unsigned lane) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    for (unsigned long long q0 = 0; q0 < L4; q0 += 32) {
        const unsigned long long q = q0 + lane;
        int pos = -1;
        if (q < L4) {
            const float4 v = __ldg(r4 + q);
            pos = v.x == 0.0f ? 0 : (v.y == 0.0f ? 1 : (v.z == 0.0f ? 2 : (v.w == 0.0f ? 3 : -1)));
        }
        const unsigned hit = __ballot_sync(0xffffffffu, pos >= 0);
        if (hit) {
            const int src = __ffs(hit) - 1;
            const int p = __shfl_sync(0xffffffffu, pos, src);
            return __ldg(row + (q0 + src) * 4 + p);
        }
    }
    return 0.0f;  // not reached: the caller saw a zero maximum
}

// Depth of a pass: float4 loads per thread per array in flight (one array
// forward, x and g together backward).
template <int MODE> __host__ __device__ constexpr unsigned reread_depth() {
    return (MODE == LSM_FWD || MODE == SM_FWD) ? 8u : 4u;
}

template <int MODE>
__global__ void __launch_bounds__(kRThreads, 2)
row_reread_kernel(const RowArgs a, unsigned wlog2) {
    constexpr bool FWD = MODE == LSM_FWD || MODE == SM_FWD;
    constexpr unsigned D = reread_depth<MODE>();
    __shared__ double2 slots[2][kRWarps];
    const unsigned warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned W = 1u << wlog2;
    const unsigned G = kRWarps >> wlog2;  // rows per CTA iteration
    const unsigned grp = warp >> wlog2;
    const unsigned gt = ((warp & (W - 1)) << 5) | lane, GT = W << 5;
    const unsigned L4 = static_cast<unsigned>(a.L / 4);  // at most kRereadMaxL / 4
    // softmax backward: g * y of the first H float4 of each row of the
    // group, kept in shared memory from pass 1 to pass 2 (dynamic, G * H).
    // (The same for the forward's x measured slower: 0.93 -> 0.86.)
    extern __shared__ float4 rr_dyn[];
    const unsigned H = MODE == SM_BWD ? L4 / 2 : 0;
    float4* sgy = rr_dyn + static_cast<std::size_t>(grp) * H;
    const unsigned long long keep = policy_evict_last(), drop = policy_evict_first();
    const double qnan = static_cast<double>(__int_as_float(0x7fc00000));

    // Every pass walks the row in rounds of D float4 per thread, all D loads
    // of a round issued before any is used; in the last round the loads past
    // the row's end re-read its last float4 and their values go unused.
    unsigned it = 0;
    for (unsigned long long base = static_cast<unsigned long long>(blockIdx.x) * G; base < a.rows;
         base += static_cast<unsigned long long>(gridDim.x) * G, ++it) {
        const unsigned long long row = base + grp;
        const bool active = row < a.rows;
        const float4* xr = reinterpret_cast<const float4*>(a.x + row * a.L);
        const float4* gr = reinterpret_cast<const float4*>(a.g + row * a.L);
        float4* yr = reinterpret_cast<float4*>(a.y + row * a.L);
        double2* sl = slots[it & 1u];

        // ---------------- pass 1 ----------------
        if constexpr (FWD) {
            // Online (max, sum of e^(x - max)) per thread, one round of D
            // float4 at a time: the round's maximum first (NaN never wins,
            // the positions past the row end count as -inf), one rescale of
            // the running sum when it grows, then the round's 4D terms
            // e^(x - m) added in float by float4 and across the round, the
            // round's total in double.
            float m = -INFINITY;
            double s = 0.0;
            bool nan_seen = false;
            if (active) {
                for (unsigned j = gt; j < L4; j += D * GT) {
                    float4 v[D];
#pragma unroll
                    for (unsigned k = 0; k < D; ++k) v[k] = ld4_hint(xr + min(j + k * GT, L4 - 1), keep);
#pragma unroll
                    for (unsigned k = 0; k < D; ++k)
                        if (j + k * GT >= L4) v[k] = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
                    float bm = -INFINITY;
#pragma unroll
                    for (unsigned k = 0; k < D; ++k)
                        bm = fmaxf(bm, fmaxf(fmaxf(v[k].x, v[k].y), fmaxf(v[k].z, v[k].w)));
                    if (bm > m) {  // NaN never compares greater
                        if (m != -INFINITY) s *= static_cast<double>(expf(m - bm));
                        m = bm;
                    }
                    if (m == -INFINITY) {  // nothing but -inf (and NaN) so far: no terms yet
#pragma unroll
                        for (unsigned k = 0; k < D; ++k)
                            nan_seen = nan_seen || v[k].x != v[k].x || v[k].y != v[k].y || v[k].z != v[k].z ||
                                       v[k].w != v[k].w;
                    } else {
                        float r = 0.0f;
#pragma unroll
                        for (unsigned k = 0; k < D; ++k)
                            r += (exp_term(v[k].x - m) + exp_term(v[k].y - m)) + (exp_term(v[k].z - m) + exp_term(v[k].w - m));
                        s += static_cast<double>(r);
                    }
                }
            }
            const float mw = warp_fmax(m);
            double t = m == -INFINITY ? (nan_seen ? qnan : 0.0) : s * static_cast<double>(expf(m - mw));
            t = warp_sum(t);
            if (__any_sync(0xffffffffu, nan_seen)) t = qnan;
            if (lane == 0) sl[warp] = make_double2(static_cast<double>(mw), t);
        } else {
            double part = 0.0;
            if (active) {
                const float m = MODE == SM_BWD ? __ldg(a.row_max + row) : 0.0f;
                const float l = MODE == SM_BWD ? logf(__ldg(a.row_sum + row)) : 0.0f;
                for (unsigned j = gt; j < L4; j += D * GT) {
                    float4 g[D], x[D];
#pragma unroll
                    for (unsigned k = 0; k < D; ++k) {
                        const unsigned jk = min(j + k * GT, L4 - 1);
                        // softmax: the first half's g is not read again (its
                        // g * y waits in shared memory), so L2 need not keep it
                        g[k] = ld4_hint(gr + jk, MODE == SM_BWD && jk < H ? drop : keep);
                        if constexpr (MODE == SM_BWD) x[k] = ld4_hint(xr + jk, keep);
                    }
#pragma unroll
                    for (unsigned k = 0; k < D; ++k)
                        if (j + k * GT < L4) {
                            if constexpr (MODE == LSM_BWD) {
                                part += quad_sum(neg4(g[k]));
                            } else {
                                const float4 gv = g[k], xv = x[k];
                                const float4 gy = make_float4(gv.x * exp_sfu((xv.x - m) - l), gv.y * exp_sfu((xv.y - m) - l),
                                                              gv.z * exp_sfu((xv.z - m) - l), gv.w * exp_sfu((xv.w - m) - l));
                                part += quad_sum(neg4(gy));
                                if (j + k * GT < H) sgy[j + k * GT] = gy;
                            }
                        }
                }
            }
            part = warp_sum(part);
            if (lane == 0) sl[warp] = make_double2(part, 0.0);
        }
        __syncthreads();
        if (!active) continue;  // the barrier above is the only one of an iteration

        // ---------------- combine the group's warps (same order in each) ----------------
        const double2* gs = sl + (grp << wlog2);
        if constexpr (FWD) {
            float mm = lane < W ? static_cast<float>(gs[lane].x) : -INFINITY;
            mm = warp_fmax(mm);
            double t = lane < W ? gs[lane].y * static_cast<double>(expf(static_cast<float>(gs[lane].x) - mm)) : 0.0;
            double s_row = warp_sum(t);
            // a row of -inf only: the reference's x - m is NaN everywhere
            if (mm == -INFINITY) s_row = qnan;
            float m = mm;
            const float first = __ldg(a.x + row * a.L);
            if (first != first) m = first;  // the scan never leaves a NaN at index 0
            else if (m == 0.0f) m = first_zero(a.x + row * a.L, L4, lane);
            const float s = static_cast<float>(s_row);
            const float l = logf(s);
            if (gt == 0) {
                if (a.row_max) a.row_max[row] = m;
                if (a.row_sum) a.row_sum[row] = s;
            }
            auto f = [&](float v) {
                const float ls = (v - m) - l;
                return MODE == SM_FWD ? exp_sfu(ls) : ls;
            };
            // ---------------- pass 2 ----------------
            for (unsigned j = gt; j < L4; j += D * GT) {
                float4 v[D];
#pragma unroll
                for (unsigned k = 0; k < D; ++k) v[k] = ld4_hint(xr + min(j + k * GT, L4 - 1), drop);
#pragma unroll
                for (unsigned k = 0; k < D; ++k)
                    if (j + k * GT < L4)
                        st4_stream(reinterpret_cast<float*>(yr + j + k * GT),
                                   make_float4(f(v[k].x), f(v[k].y), f(v[k].z), f(v[k].w)));
            }
        } else {
            const float m = __ldg(a.row_max + row), s = __ldg(a.row_sum + row);
            const float l = MODE == SM_BWD ? logf(s) : 0.0f;
            const float dl = static_cast<float>(warp_sum(lane < W ? gs[lane].x : 0.0));
            const float de = (dl / s) + 0.0f;
            // LSM_BWD: dx = g + de * expf(x - m)
            // SM_BWD:  dx = gy + de * expf(x - m), gy = g * expf((x - m) - l)
            // softmax: three exponentials per element on the SFU; log_softmax
            // (one, and at the HBM roofline) keeps expf
            auto f_gy = [&](float gy, float x) {
                return gy + de * (MODE == SM_BWD ? exp_sfu(x - m) : expf(x - m));
            };
            auto f = [&](float g, float x) { return f_gy(MODE == SM_BWD ? g * exp_sfu((x - m) - l) : g, x); };
            // ---------------- pass 2 ----------------
            for (unsigned j = gt; j < L4; j += D * GT) {
                float4 g[D], x[D];
                bool have_gy[D];
#pragma unroll
                for (unsigned k = 0; k < D; ++k) {
                    const unsigned jk = min(j + k * GT, L4 - 1);
                    // softmax, first half: g * y as pass 1 computed it (this
                    // thread's own shared-memory slots), the same bits
                    have_gy[k] = MODE == SM_BWD && jk < H;
                    g[k] = have_gy[k] ? sgy[jk] : ld4_hint(gr + jk, drop);
                    x[k] = MODE == SM_BWD ? ld4_hint(xr + jk, drop) : ld4_stream(reinterpret_cast<const float*>(xr + jk));
                }
#pragma unroll
                for (unsigned k = 0; k < D; ++k)
                    if (j + k * GT < L4) {
                        const float4 o = have_gy[k] ? make_float4(f_gy(g[k].x, x[k].x), f_gy(g[k].y, x[k].y),
                                                                  f_gy(g[k].z, x[k].z), f_gy(g[k].w, x[k].w))
                                                    : make_float4(f(g[k].x, x[k].x), f(g[k].y, x[k].y),
                                                                  f(g[k].z, x[k].z), f(g[k].w, x[k].w));
                        st4_stream(reinterpret_cast<float*>(yr + j + k * GT), o);
                    }
            }
        }
    }
}

template <int MODE>
static void launch_rows_reread(const RowArgs& a) {
    const unsigned long long L4 = a.L / 4;
    unsigned wlog2 = 0;
    while (wlog2 < 4 && L4 > (32ull << wlog2) * 16) ++wlog2;  // at most 16 float4 per thread
    const unsigned long long rows_per_cta = kRWarps >> wlog2;
    // one CTA per row group (no persistent loop over rows): short-lived CTAs
    // keep HBM busier (softmax backward 78% -> 97% against two resident CTAs
    // per SM walking the rows)
    const unsigned long long ctas = std::min<unsigned long long>((a.rows + rows_per_cta - 1) / rows_per_cta,
                                                                 0x7fffffffull);
    // softmax backward keeps g * y of each row's first half in shared memory
    // (at most 64 KB per CTA: two CTAs per SM still fit)
    constexpr bool HALF = MODE == SM_BWD;
    const std::size_t smem = HALF ? rows_per_cta * (L4 / 2) * sizeof(float4) : 0;
    static bool configured = false;
    if (HALF && !configured) {
        VC_CUDA(cudaFuncSetAttribute(row_reread_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kRereadMaxL / 8 * sizeof(float4))));
        configured = true;
    }
    row_reread_kernel<MODE><<<static_cast<unsigned>(ctas), kRThreads, smem, stream()>>>(a, wlog2);
    check_launch("softmax_rows_reread");
}

// ---------------------------------------------------------------------------
// Softmax / log_softmax forward on aligned rows of kRingMinL..kRingMaxL
// floats, ring design: one CTA per SM walks the rows blockIdx.x,
// blockIdx.x + gridDim.x, ... One lane of warp 16 (the producer) bulk-copies
// each row TWICE, in chunks of kRingChunk floats, into a ring of kRingSlots
// shared-memory slots: first for pass 1 (from HBM, L2 evict_last), then
// straight away for pass 2 (an L2 hit by then, evict_first). Each slot has a
// "full" mbarrier (completed by the copy's byte count) and an "empty" one
// (one arrival per consumer warp); the consumers release a chunk as soon as
// they have used it, so the producer streams without pause and the
// consumers issue no loads at all. (The re-read kernel issues its loads
// from the consumer threads, so HBM idles while its CTAs reduce and write.
// Measured on the way here: the whole row kept in the ring until pass 2,
// which left too few slots for the next row, 0.80 of the copy peak; pass 1
// from the ring and pass 2 as consumer loads from L2, 0.64; 8 KB chunks, one
// float4 per thread each, 0.59 -- 43 instructions per element, the slot
// bookkeeping of every wait.)
// 16 consumer warps; thread t handles float4 t + 512 k (k < 4) of every
// chunk; both sides walk the ring with running (slot, phase) counters:
//   pass 1: per chunk, its maximum first (NaN never wins, positions past
//           the row's end count as -inf), the running sum rescaled at most
//           once per chunk, the chunk's terms added in float and its total
//           in double (the re-read kernel's arithmetic);
//   combine: per-warp (max, sum) through shared memory (double-buffered by
//           row parity) at a barrier of the consumer warps that also ORs
//           their wait give-ups, so all leave at the same row;
//   pass 2: the row's second copy, outputs written once (streaming stores).
// Every wait is bounded; a give-up skips the rest of the row's waits and
// stores and reaches every consumer at the next barrier. The producer stops
// issuing when its wait gives up and, before it returns, waits (bounded) for
// the copies it issued.
// ---------------------------------------------------------------------------
constexpr unsigned kRingChunk = 8192;                     // floats per slot (32 KB)
constexpr unsigned kRingChunk4 = kRingChunk / 4;
constexpr unsigned kRingSlots = 7;
constexpr unsigned kRingConsumerWarps = 16;
constexpr unsigned kRingConsumers = kRingConsumerWarps * 32;
constexpr unsigned kRingPer = kRingChunk4 / kRingConsumers;  // float4 of a chunk per thread
constexpr unsigned kRingThreads = kRingConsumers + 32;
constexpr unsigned long long kRingMinL = 8192;
constexpr unsigned long long kRingMaxL = 40960;

constexpr std::size_t ring_smem() {
    return 128 + static_cast<std::size_t>(kRingSlots) * kRingChunk * sizeof(float) +
           2 * kRingConsumerWarps * sizeof(double2) + 2 * kRingSlots * sizeof(unsigned long long);
}

__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src, unsigned bytes, unsigned long long* bar,
                                               unsigned long long policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

template <int MODE>
__global__ void __launch_bounds__(kRingThreads, 1)
row_ring_kernel(const RowArgs a) {
    extern __shared__ unsigned char ring_raw[];
    unsigned char* base = ring_raw + ((128 - (smem_addr(ring_raw) & 127)) & 127);
    float4* ring = reinterpret_cast<float4*>(base);  // [slots][kRingChunk4]
    double2* wslots = reinterpret_cast<double2*>(ring + kRingSlots * kRingChunk4);  // [2][16]
    unsigned long long* full = reinterpret_cast<unsigned long long*>(wslots + 2 * kRingConsumerWarps);
    unsigned long long* empty = full + kRingSlots;

    const unsigned t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const unsigned long long L = a.L;
    const unsigned L4 = static_cast<unsigned>(L / 4);
    const unsigned R = static_cast<unsigned>((L + kRingChunk - 1) / kRingChunk);  // chunks per row
    if (t == 0) {
        for (unsigned s = 0; s < kRingSlots; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, kRingConsumerWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kRingConsumerWarps) {  // producer
        if (lane == 0) {
            const unsigned long long keep = policy_evict_last(), drop = policy_evict_first();
            unsigned slot = 0, phase = 0, issued = 0;
            bool stop = false;
            for (unsigned long long row = blockIdx.x; row < a.rows && !stop; row += gridDim.x) {
                const float* xr = a.x + row * L;
                for (unsigned cc = 0; cc < 2 * R; ++cc) {  // pass 1's copy, then pass 2's
                    const unsigned c = cc < R ? cc : cc - R;
                    // the slot's previous chunk (one lap earlier) has been released
                    if (issued >= kRingSlots && !mbar_wait_bounded(empty + slot, phase ^ 1u, a.err)) {
                        stop = true;
                        break;
                    }
                    const unsigned long long rest = L - static_cast<unsigned long long>(c) * kRingChunk;
                    const unsigned bytes = static_cast<unsigned>(rest < kRingChunk ? rest : kRingChunk) * 4u;
                    mbar_expect_tx(full + slot, bytes);
                    bulk_load_hint(ring + slot * kRingChunk4, xr + static_cast<unsigned long long>(c) * kRingChunk,
                                   bytes, full + slot, cc < R ? keep : drop);
                    ++issued;
                    if (++slot == kRingSlots) {
                        slot = 0;
                        phase ^= 1u;
                    }
                }
            }
            // the last copies issued land before the CTA may finish
            for (unsigned k = issued > kRingSlots ? issued - kRingSlots : 0; k < issued; ++k)
                mbar_wait_bounded(full + k % kRingSlots, (k / kRingSlots) & 1u, a.err, kWaitPolls / 16);
        }
        return;
    }

    // consumers
    const double qnan = static_cast<double>(__int_as_float(0x7fc00000));
    unsigned slot = 0, phase = 0;
    auto next_slot = [&]() {
        if (++slot == kRingSlots) {
            slot = 0;
            phase ^= 1u;
        }
    };
    auto release = [&]() {  // this warp is done with the chunk in `slot`
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + slot);
        next_slot();
    };
    unsigned it = 0;
    bool ok = true;  // no wait has given up (a pass-2 give-up reaches the next row's barrier)
    for (unsigned long long row = blockIdx.x; row < a.rows; row += gridDim.x, ++it) {
        // ---------------- pass 1 ----------------
        float m = -INFINITY;
        double s = 0.0;
        bool nan_seen = false;
        for (unsigned c = 0; c < R; ++c) {
            if (ok) ok = mbar_wait_bounded(full + slot, phase, a.err);  // one give-up ends the waits
            float4 v[kRingPer];
            const float4* ch = ring + slot * kRingChunk4;
#pragma unroll
            for (unsigned k = 0; k < kRingPer; ++k) {
                const unsigned q = c * kRingChunk4 + k * kRingConsumers + t;
                v[k] = ok && q < L4 ? ch[k * kRingConsumers + t] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            }
            float bm = -INFINITY;
#pragma unroll
            for (unsigned k = 0; k < kRingPer; ++k) bm = fmaxf(bm, fmaxf(fmaxf(v[k].x, v[k].y), fmaxf(v[k].z, v[k].w)));
            release();  // the chunk's values are in registers
            if (bm > m) {  // NaN never compares greater
                if (m != -INFINITY) s *= static_cast<double>(expf(m - bm));
                m = bm;
            }
            if (m == -INFINITY) {  // nothing but -inf (and NaN) so far: no terms yet
#pragma unroll
                for (unsigned k = 0; k < kRingPer; ++k)
                    nan_seen = nan_seen || v[k].x != v[k].x || v[k].y != v[k].y || v[k].z != v[k].z ||
                               v[k].w != v[k].w;
            } else {
                float r = 0.0f;
#pragma unroll
                for (unsigned k = 0; k < kRingPer; ++k)
                    r += (exp_term(v[k].x - m) + exp_term(v[k].y - m)) + (exp_term(v[k].z - m) + exp_term(v[k].w - m));
                s += static_cast<double>(r);
            }
        }
        const float mw = warp_fmax(m);
        double tw = m == -INFINITY ? (nan_seen ? qnan : 0.0) : s * static_cast<double>(expf(m - mw));
        tw = warp_sum(tw);
        if (__any_sync(0xffffffffu, nan_seen)) tw = qnan;
        double2* sl = wslots + (it & 1u) * kRingConsumerWarps;
        if (lane == 0) sl[warp] = make_double2(static_cast<double>(mw), tw);
        if (named_barrier_or<1, kRingConsumers>(!ok)) return;  // a wait gave up: this row is not written

        // ---------------- combine the 16 warps (the same order in each) ----------------
        float mm = lane < kRingConsumerWarps ? static_cast<float>(sl[lane].x) : -INFINITY;
        mm = warp_fmax(mm);
        const double tq =
            lane < kRingConsumerWarps ? sl[lane].y * static_cast<double>(expf(static_cast<float>(sl[lane].x) - mm)) : 0.0;
        double s_row = warp_sum(tq);
        if (mm == -INFINITY) s_row = qnan;  // a row of -inf only: the reference's x - m is NaN everywhere
        float mrow = mm;
        const float* xr = a.x + row * L;
        const float first = __ldg(xr);
        if (first != first) mrow = first;  // the scan never leaves a NaN at index 0
        else if (mrow == 0.0f) mrow = first_zero(xr, L4, lane);
        const float srow = static_cast<float>(s_row);
        const float l = logf(srow);
        if (t == 0) {
            if (a.row_max) a.row_max[row] = mrow;
            if (a.row_sum) a.row_sum[row] = srow;
        }
        auto f = [&](float v) {
            const float ls = (v - mrow) - l;
            return MODE == SM_FWD ? exp_sfu(ls) : ls;
        };
        // ---------------- pass 2 ----------------
        float4* yr = reinterpret_cast<float4*>(a.y + row * L);
        for (unsigned c = 0; c < R; ++c) {
            if (ok) ok = mbar_wait_bounded(full + slot, phase, a.err);
            const float4* ch = ring + slot * kRingChunk4;
            float4 v[kRingPer];
#pragma unroll
            for (unsigned k = 0; k < kRingPer; ++k) v[k] = ch[k * kRingConsumers + t];
#pragma unroll
            for (unsigned k = 0; k < kRingPer; ++k) {
                const unsigned q = c * kRingChunk4 + k * kRingConsumers + t;
                if (ok && q < L4)
                    st4_stream(reinterpret_cast<float*>(yr + q), make_float4(f(v[k].x), f(v[k].y), f(v[k].z), f(v[k].w)));
            }
            release();
        }
    }
}

template <int MODE>
static void launch_rows_ring(const RowArgs& a) {
    static bool configured = false;
    if (!configured) {
        VC_CUDA(cudaFuncSetAttribute(row_ring_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(ring_smem())));
        configured = true;
    }
    const unsigned long long ctas = std::min<unsigned long long>(a.rows, static_cast<unsigned long long>(sm_count()));
    row_ring_kernel<MODE><<<static_cast<unsigned>(ctas), kRingThreads, ring_smem(), stream()>>>(a);
    check_launch("softmax_rows_ring");
}

template <int MODE, bool BULK>
static void launch_rows_mode(const RowArgs& a, unsigned C, std::size_t smem) {
    static bool configured = false;
    if (!configured) {
        VC_CUDA(cudaFuncSetAttribute(row_kernel<MODE, BULK>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        VC_CUDA(cudaFuncSetAttribute(row_kernel<MODE, BULK>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        configured = true;
    }
    const unsigned long long max_rows_per_launch = (1ull << 31) / 8 / C;
    for (unsigned long long row0 = 0; row0 < a.rows; row0 += max_rows_per_launch) {
        const unsigned long long rows = std::min<unsigned long long>(a.rows - row0, max_rows_per_launch);
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(static_cast<unsigned>(rows * C), 1, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream();
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = C;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        VC_CUDA(cudaLaunchKernelEx(&cfg, row_kernel<MODE, BULK>, a, row0));
    }
    check_launch("softmax_rows");
}

static cudaLaunchConfig_t cluster_config(unsigned long long ctas, unsigned C, std::size_t smem,
                                         cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(ctas), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream();
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

// Persistent grid size: the clusters of (C, smem) the device holds at once,
// queried once per configuration.
template <int MODE>
static unsigned long long resident_clusters(unsigned C, std::size_t smem) {
    static std::mutex mu;
    static std::map<std::pair<unsigned, std::size_t>, int> cache;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find({C, smem});
    if (it != cache.end()) return static_cast<unsigned long long>(it->second);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cluster_config(static_cast<unsigned long long>(C) * sm_count(), C, smem, attr);
    int n = 0;
    VC_CUDA(cudaOccupancyMaxActiveClusters(&n, row_pipe_kernel<MODE>, &cfg));
    if (n < 1) fail(VC_ERR_RUNTIME, "softmax: no cluster of this shape fits on the device");
    cache[{C, smem}] = n;
    return static_cast<unsigned long long>(n);
}

template <int MODE>
static void launch_rows_pipelined(const RowArgs& a, unsigned C, std::size_t smem) {
    static bool configured = false;
    if (!configured) {
        VC_CUDA(cudaFuncSetAttribute(row_pipe_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        VC_CUDA(cudaFuncSetAttribute(row_pipe_kernel<MODE>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        configured = true;
    }
    const unsigned long long clusters = std::min<unsigned long long>(a.rows, resident_clusters<MODE>(C, smem));
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cluster_config(clusters * C, C, smem, attr);
    VC_CUDA(cudaLaunchKernelEx(&cfg, row_pipe_kernel<MODE>, a));
    check_launch("softmax_rows_pipelined");
}

template <int MODE>
static void launch_family(RowArgs a, std::size_t outer, std::size_t length, std::size_t inner) {
    constexpr bool STAGE_X = MODE == LSM_FWD || MODE == SM_FWD || MODE == CE_FWD || MODE == SM_BWD;
    constexpr bool STAGE_G = MODE == LSM_BWD || MODE == SM_BWD;
    a.err = device_error_word();
    a.L = length;
    if (inner == 1) {
        a.rows = outer;
        const bool aligned = length % 4 == 0 && aligned16(a.x) && (!STAGE_G || aligned16(a.g)) &&
                             (!a.y || aligned16(a.y));
        if (MODE == CE_FWD && length % 4 == 0 && aligned16(a.x)) {
            const unsigned long long warps_per_cta = kThreads / 32;
            const unsigned long long ctas = std::min<unsigned long long>((outer + warps_per_cta - 1) / warps_per_cta,
                                                                         0x7fffffffull);
            ce_rows_kernel<<<static_cast<unsigned>(ctas), kThreads, 0, stream()>>>(a);
            check_launch("cross_entropy_rows");
            return;
        }
        if constexpr (MODE == LSM_FWD || MODE == SM_FWD) {
            if (aligned && length >= kRingMinL && length <= kRingMaxL) {
                launch_rows_ring<MODE>(a);
                return;
            }
        }
        if constexpr (MODE != CE_FWD) {
            if (aligned && length <= kRereadMaxL) {
                launch_rows_reread<MODE>(a);
                return;
            }
        }
        if (aligned) {
            constexpr unsigned NB = PipeTraits<MODE>::NBUF;
            unsigned C = 1;
            while (C < 8 && (length + C - 1) / C > kStageFloats / NB) C <<= 1;
            const unsigned long long seg = ((length + C - 1) / C + 3) / 4 * 4;
            if (seg * NB <= kStageFloatsMax) {
                a.seg = static_cast<unsigned>(seg);
                launch_rows_pipelined<MODE>(a, C, 2 * seg * NB * sizeof(float));
                return;
            }
        }
        if (length <= 8ull * kSliceMax) {
            unsigned C = 1;
            while (C < 8 && (length + C - 1) / C > kSliceTarget) C <<= 1;
            unsigned long long seg = (length + C - 1) / C;
            seg = (seg + 3) / 4 * 4;
            a.seg = static_cast<unsigned>(seg);
            const std::size_t smem = seg * sizeof(float) * ((STAGE_X ? 1 : 0) + (STAGE_G ? 1 : 0));
            const bool bulk = length % 4 == 0 && (!STAGE_X || aligned16(a.x)) && (!STAGE_G || aligned16(a.g));
            if (bulk) launch_rows_mode<MODE, true>(a, C, smem);
            else launch_rows_mode<MODE, false>(a, C, smem);
            return;
        }
    }
    a.rows = outer * inner;
    col_kernel<MODE><<<grid_for(outer * inner, kThreads), kThreads, 0, stream()>>>(a, outer, inner);
    check_launch("softmax_cols");
}

}  // namespace

}  // namespace vc

using namespace vc;

extern "C" {

static void check_dims(size_t outer, size_t length, size_t inner) {
    const size_t dims[3] = {outer, length, inner};
    checked_numel(dims, 3);
}

vc_status vc_cuda_log_softmax(const float* x, float* y, float* row_max, float* row_sum, size_t outer,
                              size_t length, size_t inner) {
    VC_API_BEGIN
    ensure_init();
    check_dims(outer, length, inner);
    if (!outer || !length || !inner) return VC_OK;
    if (!x || !y) fail(VC_ERR_INVALID, "log_softmax: null pointer");
    RowArgs a{};
    a.x = x; a.y = y; a.row_max = row_max; a.row_sum = row_sum;
    launch_family<LSM_FWD>(a, outer, length, inner);
    VC_API_END
}

vc_status vc_cuda_softmax(const float* x, float* y, float* row_max, float* row_sum, size_t outer,
                          size_t length, size_t inner) {
    VC_API_BEGIN
    ensure_init();
    check_dims(outer, length, inner);
    if (!outer || !length || !inner) return VC_OK;
    if (!x || !y) fail(VC_ERR_INVALID, "softmax: null pointer");
    RowArgs a{};
    a.x = x; a.y = y; a.row_max = row_max; a.row_sum = row_sum;
    launch_family<SM_FWD>(a, outer, length, inner);
    VC_API_END
}

vc_status vc_cuda_log_softmax_backward(const float* x, const float* row_max, const float* row_sum,
                                       const float* g, float* dx, size_t outer, size_t length, size_t inner) {
    VC_API_BEGIN
    ensure_init();
    check_dims(outer, length, inner);
    if (!outer || !length || !inner) return VC_OK;
    if (!x || !row_max || !row_sum || !g || !dx) fail(VC_ERR_INVALID, "log_softmax_backward: null pointer");
    RowArgs a{};
    a.x = x; a.g = g; a.y = dx;
    a.row_max = const_cast<float*>(row_max); a.row_sum = const_cast<float*>(row_sum);
    launch_family<LSM_BWD>(a, outer, length, inner);
    VC_API_END
}

vc_status vc_cuda_softmax_backward(const float* x, const float* row_max, const float* row_sum,
                                   const float* g, float* dx, size_t outer, size_t length, size_t inner) {
    VC_API_BEGIN
    ensure_init();
    check_dims(outer, length, inner);
    if (!outer || !length || !inner) return VC_OK;
    if (!x || !row_max || !row_sum || !g || !dx) fail(VC_ERR_INVALID, "softmax_backward: null pointer");
    RowArgs a{};
    a.x = x; a.g = g; a.y = dx;
    a.row_max = const_cast<float*>(row_max); a.row_sum = const_cast<float*>(row_sum);
    launch_family<SM_BWD>(a, outer, length, inner);
    VC_API_END
}

vc_status vc_cuda_cross_entropy(const float* logits, const int64_t* targets, size_t batch, size_t classes,
                                size_t batch_total, float* loss, float* row_max, float* row_sum,
                                double* partial) {
    VC_API_BEGIN
    ensure_init();
    check_dims(batch, classes, 1);
    if (batch_total == 0) batch_total = batch;
    if (batch_total == 0) fail(VC_ERR_INVALID, "cross_entropy of an empty batch is undefined");
    if (classes == 0) fail(VC_ERR_INVALID, "cross_entropy needs at least one class");
    if (batch && (!logits || !targets)) fail(VC_ERR_INVALID, "cross_entropy: null pointer");
    Scratch terms(batch * sizeof(float) + 16);
    if (batch) {
        RowArgs a{};
        a.x = logits;
        a.targets = reinterpret_cast<const long long*>(targets);
        a.row_max = row_max;
        a.row_sum = row_sum;
        a.row_term = terms.as<float>();
        launch_family<CE_FWD>(a, batch, classes, 1);
    }
    ce_finish_kernel<<<1, 1024, 0, stream()>>>(terms.as<float>(), batch, static_cast<float>(batch_total), loss,
                                                partial);
    check_launch("cross_entropy_finish");
    VC_API_END
}

vc_status vc_cuda_cross_entropy_backward(const float* logits, const int64_t* targets, const float* row_max,
                                         const float* row_sum, const float* upstream, size_t batch,
                                         size_t classes, size_t batch_total, float* dlogits) {
    VC_API_BEGIN
    ensure_init();
    check_dims(batch, classes, 1);
    if (batch_total == 0) batch_total = batch;
    if (!batch || !classes) return VC_OK;
    if (!logits || !targets || !row_max || !row_sum || !upstream || !dlogits)
        fail(VC_ERR_INVALID, "cross_entropy_backward: null pointer");
    const bool vec = classes % 4 == 0 && aligned16(logits) && aligned16(dlogits);
    const auto* t = reinterpret_cast<const long long*>(targets);
    const unsigned long long n4 = static_cast<unsigned long long>(batch) * classes / 4;
    if (vec && classes >= 1024 && n4 < (1ull << 32)) {
        static_assert(kThreads == kStreamThreads, "ce_backward_stream launches stream_grid CTAs");
        ce_backward_stream<<<stream_grid(4 * n4), kThreads, 0, stream()>>>(
            logits, t, row_max, row_sum, upstream, n4, FastDiv(static_cast<unsigned>(classes / 4)),
            static_cast<float>(batch_total), dlogits);
        check_launch("cross_entropy_backward");
        return VC_OK;
    }
    const unsigned grid = static_cast<unsigned>(std::min<std::size_t>(batch, static_cast<std::size_t>(sm_count()) * 16));
    if (vec) ce_backward_kernel<true><<<grid, kThreads, 0, stream()>>>(logits, t, row_max, row_sum, upstream, batch, classes, static_cast<float>(batch_total), dlogits);
    else ce_backward_kernel<false><<<grid, kThreads, 0, stream()>>>(logits, t, row_max, row_sum, upstream, batch, classes, static_cast<float>(batch_total), dlogits);
    check_launch("cross_entropy_backward");
    VC_API_END
}

}  // extern "C"
