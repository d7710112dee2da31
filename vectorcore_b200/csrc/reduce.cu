// reduce.cu -- deterministic reductions for sm_100a:
//   * the fused broadcast-gradient reduction (sum_to_shape) and the fused
//     backward rules of the binary ops, which compute g*b, g/b, -(g*a)/(b*b)
//     per element and reduce over every broadcast axis in ONE pass (the
//     reference runs one full pass per axis plus a temporary per product,
//     src/autograd.cpp:50-72, src/ops.cpp:98-156);
//   * full and per-axis sum / mean (cpu::sum, cpu::reduce_axis);
//   * per-axis and full max / argmax with the reference's strict '>' scan
//     semantics, and their fused backward (scatter) passes.
//
// Every kernel streams its input once from HBM. Sums accumulate in double and
// round to float once (the reference accumulates in double, cpu_backend.cpp
// :392-418, :434-441). The work split -- segments of the reduced index space,
// each producing a partial in stream-ordered scratch, combined in segment
// order by a second kernel -- is derived from the shapes only (never from the
// SM count), so results do not depend on the launch configuration.
#include "vc_internal.cuh"

#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

namespace vc {

namespace {

constexpr unsigned kThreads = 256;
// Aim for about this many threads of work before splitting a reduction into
// segments (a constant, so the split depends on the problem size alone).
constexpr unsigned long long kTargetThreads = 1ull << 17;  // 2^19 split axis-0 reductions 4x finer: partials and finishes cost 2.5 points
constexpr unsigned long long kMinSegment = 16;         // reduced positions per segment (column)
// Column sums take at most this many segments, so the partials stay small
// next to the input when the outputs are few (the compact reductions of a
// broadcast gradient: 1024 columns of 32768 rows).
constexpr unsigned long long kMaxSumSegments = 512;
constexpr unsigned kSliceThreads = 1024;               // sliced kernels: 32 outputs x 32 slices
constexpr unsigned kSlices = kSliceThreads / 32;
constexpr unsigned long long kSlicedMaxRows = 1024;    // single-launch column sums up to this many rows
constexpr unsigned long long kSlicedMaxOutputs = 32768;
constexpr unsigned long long kSlicedMaxElements = 1ull << 20;  // larger sums stream on float4 columns
constexpr unsigned long long kReplicateMax = 1ull << 20;  // replicas written by the reduction itself, floats
constexpr unsigned long long kRowTargetCtas = 4096;    // aim for this many (row, segment) CTAs
constexpr unsigned long long kRowMinSegment = 4096;    // elements per row segment, at least

// Segments per row for a ROW-layout reduction of K rows of W elements: enough
// (row, segment) CTAs to fill the machine, each at least kRowMinSegment long.
// A function of the shape only.
// Few outputs (a full sum or max): aim for 16384 segments of at least 16384
// elements -- 64 KiB pieces, the read-only stream's sweet spot (1 GiB:
// 7.1 TB/s in 64 KiB pieces, 6.9 in 256 KiB ones) -- and finish the
// partials with 1024 threads per output.
constexpr unsigned long long kRowFewOutputs = 64;
constexpr unsigned long long kRowFewTargetCtas = 16384;
constexpr unsigned long long kRowFewMinSegment = 16384;
constexpr unsigned kFinishWideThreads = 1024;
inline unsigned long long row_segments(unsigned long long K, unsigned long long W) {
    const bool few = K < kRowFewOutputs;
    unsigned long long S = ((few ? kRowFewTargetCtas : kRowTargetCtas) + K - 1) / K;
    const unsigned long long min_seg = few ? kRowFewMinSegment : kRowMinSegment;
    S = std::min<unsigned long long>(S, (W + min_seg - 1) / min_seg);
    return std::max<unsigned long long>(1, std::min<unsigned long long>(S, 65535));
}
// Threads per CTA of the row finishes: 1024 for few outputs with many
// segments (a shape-only choice: it fixes the order of the additions).
inline unsigned row_finish_threads(unsigned long long K, unsigned long long S) {
    return K < kRowFewOutputs && S >= 1024 ? kFinishWideThreads : 256;
}

// Element functions of the backward rules, arithmetic exactly as written in
// src/ops.cpp: p, q are the other operands broadcast to the output shape.
enum Vjp { V_G = 0, V_NEG = 1, V_MUL = 2, V_DIV_A = 3, V_DIV_B = 4 };

template <int F>
__device__ __forceinline__ float vjp(float g, float p, float q) {
    if constexpr (F == V_G) return g;
    else if constexpr (F == V_NEG) return -g;
    else if constexpr (F == V_MUL) return g * p;
    else if constexpr (F == V_DIV_A) return g / p;
    else {  // -(gradient * a) / (b * b)
        const float ga = g * p;
        const float neg = -ga;
        const float bb = q * q;
        return neg / bb;
    }
}

template <int F> __host__ __device__ constexpr int operands() { return F == V_G || F == V_NEG ? 1 : (F == V_DIV_B ? 3 : 2); }

// Canonical reduction layout. Dimensions of the source (forward output)
// shape are classified kept / reduced and merged; operand 0 is g, 1 is p,
// 2 is q. COLUMN layout: the innermost dim is kept (a run of `inner`
// outputs). ROW layout: the innermost dim is reduced (a run of `inner`
// reduced elements).
struct RedDesc {
    int nk;
    unsigned long long kdims[kMaxRank];
    long long ks[3][kMaxRank];
    int nr;
    unsigned long long rdims[kMaxRank];
    long long rs[3][kMaxRank];
    unsigned long long inner;
    long long is[3];
    unsigned long long K;   // kept-outer positions
    unsigned long long R;   // reduced-outer positions (COLUMN: all reduced positions)
    unsigned long long seg; // COLUMN: reduced positions per segment; ROW: elements per segment
    unsigned S;             // segments
    float divisor;          // mean: divide the rounded sum by this (0 = none)
    double* out_d;          // when set: write the unrounded double sums here
                            // (a shard's partial for a cross-GPU combine)
};

__device__ __forceinline__ void decode(unsigned long long idx, int n, const unsigned long long* dims,
                                       const long long (*st)[kMaxRank], long long off[3],
                                       unsigned long long* coord) {
    off[0] = off[1] = off[2] = 0;
    for (int k = n - 1; k >= 0; --k) {
        const unsigned long long c = idx % dims[k];
        idx /= dims[k];
        if (coord) coord[k] = c;
        off[0] += static_cast<long long>(c) * st[0][k];
        off[1] += static_cast<long long>(c) * st[1][k];
        off[2] += static_cast<long long>(c) * st[2][k];
    }
}

__device__ __forceinline__ float4 load4(const float* base, long long off, long long inner_stride,
                                        unsigned long long i) {
    if (inner_stride == 0) {
        const float v = __ldg(base + off);
        return make_float4(v, v, v, v);
    }
    return ldg4(base + off + static_cast<long long>(i));
}

__device__ __forceinline__ float round_out(double acc, float divisor) {
    const float s = static_cast<float>(acc);
    return divisor != 0.0f ? s / divisor : s;
}

// ---------------------------------------------------------------------------
// COLUMN layout. grid = (ceil(inner / (256*V)), min(K, 65535), S).
// ---------------------------------------------------------------------------
template <int F, bool VEC>
__global__ void __launch_bounds__(kThreads)
reduce_col_kernel(const float* __restrict__ g, const float* __restrict__ p, const float* __restrict__ q,
                  const RedDesc d, float* __restrict__ out, double* __restrict__ partial) {
    constexpr int V = VEC ? 4 : 1;
    constexpr int NOPS = operands<F>();
    const unsigned long long i0 = (static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x) * V;
    if (i0 >= d.inner) return;
    const unsigned s = blockIdx.z;
    const unsigned long long r0 = s * d.seg;
    const unsigned long long r1 = min(d.R, r0 + d.seg);
    for (unsigned long long ko = blockIdx.y; ko < d.K; ko += gridDim.y) {
        long long base[3];
        decode(ko, d.nk, d.kdims, d.ks, base, nullptr);
        long long off[3];
        unsigned long long coord[kMaxRank];
        decode(r0, d.nr, d.rdims, d.rs, off, coord);
        double acc[V];
#pragma unroll
        for (int v = 0; v < V; ++v) acc[v] = 0.0;
        // advance the reduced coordinate by one position (row-major carry)
        auto advance = [&]() {
            for (int k = d.nr - 1; k >= 0; --k) {
                off[0] += d.rs[0][k];
                off[1] += d.rs[1][k];
                off[2] += d.rs[2][k];
                if (++coord[k] < d.rdims[k]) break;
                coord[k] = 0;
                off[0] -= d.rs[0][k] * static_cast<long long>(d.rdims[k]);
                off[1] -= d.rs[1][k] * static_cast<long long>(d.rdims[k]);
                off[2] -= d.rs[2][k] * static_cast<long long>(d.rdims[k]);
            }
        };
        auto fetch = [&](const long long o[3]) -> float4 {
            if constexpr (VEC) {
                const float4 gv = load4(g, base[0] + o[0], d.is[0], i0);
                const float4 pv = NOPS > 1 ? load4(p, base[1] + o[1], d.is[1], i0) : gv;
                const float4 qv = NOPS > 2 ? load4(q, base[2] + o[2], d.is[2], i0) : gv;
                return make_float4(vjp<F>(gv.x, pv.x, qv.x), vjp<F>(gv.y, pv.y, qv.y), vjp<F>(gv.z, pv.z, qv.z),
                                   vjp<F>(gv.w, pv.w, qv.w));
            } else {
                const long long ii = static_cast<long long>(i0);
                const float gv = __ldg(g + base[0] + o[0] + ii * d.is[0]);
                const float pv = NOPS > 1 ? __ldg(p + base[1] + o[1] + ii * d.is[1]) : gv;
                const float qv = NOPS > 2 ? __ldg(q + base[2] + o[2] + ii * d.is[2]) : gv;
                return make_float4(vjp<F>(gv, pv, qv), 0.f, 0.f, 0.f);
            }
        };
        auto accumulate = [&](float4 v) {
            acc[0] += static_cast<double>(v.x);
            if constexpr (VEC) {
                acc[1] += static_cast<double>(v.y);
                acc[2] += static_cast<double>(v.z);
                acc[3] += static_cast<double>(v.w);
            }
        };
        unsigned long long r = r0;
        // eight reduced positions in flight, accumulated in order
        for (; r + 7 < r1; r += 8) {
            long long o[8][3];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                o[k][0] = off[0];
                o[k][1] = off[1];
                o[k][2] = off[2];
                advance();
            }
            float4 v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = fetch(o[k]);
#pragma unroll
            for (int k = 0; k < 8; ++k) accumulate(v[k]);
        }
        for (; r < r1; ++r) {
            accumulate(fetch(off));
            advance();
        }
        const unsigned long long o = ko * d.inner + i0;
        if (d.S == 1 && d.out_d) {
#pragma unroll
            for (int v = 0; v < V; ++v) d.out_d[o + v] = acc[v];
        } else if (d.S == 1) {
            if constexpr (VEC)
                st4(out + o, make_float4(round_out(acc[0], d.divisor), round_out(acc[1], d.divisor),
                                         round_out(acc[2], d.divisor), round_out(acc[3], d.divisor)));
            else out[o] = round_out(acc[0], d.divisor);
        } else {
            double* dst = partial + static_cast<unsigned long long>(s) * d.K * d.inner + o;
#pragma unroll
            for (int v = 0; v < V; ++v) dst[v] = acc[v];
        }
    }
}

// COLUMN layout with one reduced dim and no kept outer dims (K = 1): the
// axis-0 sum of a matrix, the gradient of a row bias, a merged run of
// reduced dims. A thread owns a float4 column and steps row pointers down its
// segment with D loads per operand in flight; without the general kernel's
// per-row coordinate carry and offset arrays it needs fewer registers, so
// more CTAs stay resident. Same order of double additions as
// reduce_col_kernel: the results are identical. G_CONST: operand 0 is one
// value for the whole reduction (the 0-d upstream gradient of a sum); it is
// loaded once, and the loads in flight go to the other operands.
template <int F, bool G_CONST = false>
__global__ void __launch_bounds__(kThreads, operands<F>() == 1 ? 5 : 4)
reduce_col_simple(const float* __restrict__ g, const float* __restrict__ p, const float* __restrict__ q,
                  const RedDesc d, float* __restrict__ out, double* __restrict__ partial) {
    constexpr int NOPS = operands<F>();
    constexpr int LOADED = NOPS - (G_CONST ? 1 : 0);
    constexpr int D = LOADED <= 1 ? 8 : (LOADED == 2 ? 4 : 2);
    const unsigned long long i0 = (static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i0 >= d.inner) return;
    const unsigned s = blockIdx.z;
    const unsigned long long r0 = s * d.seg;
    const unsigned long long r1 = min(d.R, r0 + d.seg);
    const float* ptr[3] = {g, p, q};
    const float* base[3];
    long long step[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        step[k] = d.rs[k][0];
        base[k] = ptr[k] + static_cast<long long>(r0) * step[k] + (d.is[k] ? static_cast<long long>(i0) : 0);
    }
    const float gc = G_CONST ? __ldg(g) : 0.0f;
    auto fetch = [&](int k, long long row) -> float4 {
        if (G_CONST && k == 0) return make_float4(gc, gc, gc, gc);
        const float* a = base[k] + row * step[k];
        if (d.is[k] == 0) {
            const float v = __ldg(a);
            return make_float4(v, v, v, v);
        }
        return ldg4(a);
    };
    double acc0 = 0.0, acc1 = 0.0, acc2 = 0.0, acc3 = 0.0;
    auto accumulate = [&](float4 gv, float4 pv, float4 qv) {
        acc0 += static_cast<double>(vjp<F>(gv.x, pv.x, qv.x));
        acc1 += static_cast<double>(vjp<F>(gv.y, pv.y, qv.y));
        acc2 += static_cast<double>(vjp<F>(gv.z, pv.z, qv.z));
        acc3 += static_cast<double>(vjp<F>(gv.w, pv.w, qv.w));
    };
    const long long n = static_cast<long long>(r1 - r0);
    long long r = 0;
    for (; r + D <= n; r += D) {
        float4 v[NOPS][D];
#pragma unroll
        for (int j = 0; j < D; ++j)
#pragma unroll
            for (int k = 0; k < NOPS; ++k) v[k][j] = fetch(k, r + j);
#pragma unroll
        for (int j = 0; j < D; ++j)
            accumulate(v[0][j], NOPS > 1 ? v[NOPS > 1 ? 1 : 0][j] : v[0][j], NOPS > 2 ? v[NOPS > 2 ? 2 : 0][j] : v[0][j]);
    }
    for (; r < n; ++r) {
        const float4 gv = fetch(0, r);
        const float4 pv = NOPS > 1 ? fetch(1, r) : gv;
        const float4 qv = NOPS > 2 ? fetch(2, r) : gv;
        accumulate(gv, pv, qv);
    }
    if (d.S == 1 && d.out_d) {
        d.out_d[i0] = acc0;
        d.out_d[i0 + 1] = acc1;
        d.out_d[i0 + 2] = acc2;
        d.out_d[i0 + 3] = acc3;
    } else if (d.S == 1) {
        st4(out + i0, make_float4(round_out(acc0, d.divisor), round_out(acc1, d.divisor), round_out(acc2, d.divisor),
                                  round_out(acc3, d.divisor)));
    } else {
        double* dst = partial + static_cast<unsigned long long>(s) * d.inner + i0;
        dst[0] = acc0;
        dst[1] = acc1;
        dst[2] = acc2;
        dst[3] = acc3;
    }
}

// Combine COLUMN partials [S][K*inner] in segment order.
__global__ void __launch_bounds__(kThreads)
reduce_col_finish(const double* __restrict__ partial, unsigned S, unsigned long long count,
                  float divisor, float* __restrict__ out, double* __restrict__ out_d) {
    pdl_wait();  // a programmatic launch: the partials' kernel has finished and its writes are visible
    const unsigned long long stride = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
    for (unsigned long long o = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x; o < count;
         o += stride) {
        // eight segment partials in flight, added in segment order
        double acc = 0.0;
        unsigned s = 0;
        for (; s + 8 <= S; s += 8) {
            double v[8];
#pragma unroll
            for (unsigned k = 0; k < 8; ++k) v[k] = __ldg(partial + static_cast<unsigned long long>(s + k) * count + o);
#pragma unroll
            for (unsigned k = 0; k < 8; ++k) acc += v[k];
        }
        for (; s < S; ++s) acc += __ldg(partial + static_cast<unsigned long long>(s) * count + o);
        if (out_d) out_d[o] = acc;
        else out[o] = round_out(acc, divisor);
    }
}

// Write the 32 results of a sliced CTA (s_res) to `rep` consecutive copies
// of the output block: the compact result of a broadcast gradient, replicated
// along the leading dims every operand is constant on.
__device__ __forceinline__ void write_replicas(const float* s_res, float* __restrict__ out, unsigned long long count,
                                               unsigned long long rep) {
    const unsigned lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const unsigned long long o = static_cast<unsigned long long>(blockIdx.x) * 32 + lane;
    if (o >= count) return;
    const float v = s_res[lane];
    for (unsigned long long k = w; k < rep; k += kSlices) out[k * count + o] = v;
}

// Combine COLUMN partials [S][count] when the outputs are few and the
// segments many (a plain thread per output would walk thousands of partials
// one L2 round trip per eight). A CTA owns 32 outputs; warp w adds the
// partials of segments [w * per, (w + 1) * per) in segment order, eight in
// flight, and the 32 slice sums of an output are added in slice order. The
// order depends on S alone. Float results go to `rep` copies (write_replicas).
__global__ void __launch_bounds__(kSliceThreads)
reduce_col_finish_sliced(const double* __restrict__ partial, unsigned S, unsigned long long count,
                         float divisor, float* __restrict__ out, double* __restrict__ out_d,
                         unsigned long long rep) {
    pdl_wait();  // a programmatic launch: the partials' kernel has finished and its writes are visible
    __shared__ double s_slice[kSlices][32];
    __shared__ float s_res[32];
    const unsigned lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const unsigned long long o = static_cast<unsigned long long>(blockIdx.x) * 32 + lane;
    const unsigned per = (S + kSlices - 1) / kSlices;
    const unsigned s0 = min(S, w * per), s1 = min(S, s0 + per);
    double acc = 0.0;
    if (o < count) {
        unsigned s = s0;
        for (; s + 8 <= s1; s += 8) {
            double v[8];
#pragma unroll
            for (unsigned k = 0; k < 8; ++k) v[k] = __ldg(partial + static_cast<unsigned long long>(s + k) * count + o);
#pragma unroll
            for (unsigned k = 0; k < 8; ++k) acc += v[k];
        }
        for (; s < s1; ++s) acc += __ldg(partial + static_cast<unsigned long long>(s) * count + o);
    }
    s_slice[w][lane] = acc;
    __syncthreads();
    if (w == 0) {
        double t = 0.0;
#pragma unroll
        for (unsigned j = 0; j < kSlices; ++j) t += s_slice[j][lane];
        if (out_d) {
            if (o < count) out_d[o] = t;
        } else {
            s_res[lane] = round_out(t, divisor);
        }
    }
    if (out_d) return;
    __syncthreads();
    write_replicas(s_res, out, count, rep);
}

// out[k * n + j] = out[j] for k in [1, rep): copies of the block just
// written at the front of the same buffer (the compact result of a broadcast
// gradient), as a chunked store stream (stream_grid: one CTA per 1024 float4
// groups of the copies, four per thread); the source group comes from L1/L2
// (the block is small and every copy reads it). n % 4 == 0 and `out` 16-byte
// aligned; (rep - 1) * n / 4 < 2^32 (FastDiv).
__global__ void __launch_bounds__(kThreads)
replicate_front_block(float* __restrict__ out, unsigned long long n4, FastDiv n4_fd, unsigned long long total4) {
    const float4* src = reinterpret_cast<const float4*>(out);
    float4* dst = reinterpret_cast<float4*>(out) + n4;
    const unsigned long long base = static_cast<unsigned long long>(blockIdx.x) * kChunk4 + threadIdx.x;
    float4 v[kStreamRounds];
#pragma unroll
    for (unsigned u = 0; u < kStreamRounds; ++u) {
        const unsigned long long i = base + u * kStreamThreads;
        if (i < total4) {
            unsigned q, r;
            n4_fd.divmod(static_cast<unsigned>(i), q, r);
            v[u] = __ldg(src + r);
        }
    }
#pragma unroll
    for (unsigned u = 0; u < kStreamRounds; ++u) {
        const unsigned long long i = base + u * kStreamThreads;
        if (i < total4) dst[i] = v[u];
    }
}

// Column sums over a single reduced dim of at most kSlicedMaxRows rows, few
// outputs and at most 2^20 terms (small, launch-bound sums), in ONE launch (no partials, no finish): a CTA owns 32
// consecutive outputs, one per lane; warp w adds rows [w * per, (w + 1) * per)
// of its lane's column in row order, eight rows in flight, and the 32 slice
// sums of an output are added in slice order (an order fixed by R alone).
// Float results go to `rep` copies (write_replicas).
template <int F>
__global__ void __launch_bounds__(kSliceThreads)
reduce_col_sliced(const float* __restrict__ g, const float* __restrict__ p, const float* __restrict__ q,
                  const RedDesc d, float* __restrict__ out, unsigned long long rep) {
    constexpr int NOPS = operands<F>();
    __shared__ double s_slice[kSlices][32];
    __shared__ float s_res[32];
    const unsigned lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const unsigned long long l = static_cast<unsigned long long>(blockIdx.x) * 32 + lane;
    const unsigned long long per = (d.R + kSlices - 1) / kSlices;
    const unsigned long long r0 = min(d.R, w * per), r1 = min(d.R, r0 + per);
    double acc = 0.0;
    if (l < d.inner) {
        const float* ptr[3] = {g, p, q};
        const float* base[3];
        long long step[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            step[k] = d.rs[k][0];
            base[k] = ptr[k] + static_cast<long long>(r0) * step[k] + static_cast<long long>(l) * d.is[k];
        }
        const long long n = static_cast<long long>(r1 - r0);
        long long r = 0;
        for (; r + 8 <= n; r += 8) {
            float v[3][8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
#pragma unroll
                for (int k = 0; k < NOPS; ++k) v[k][j] = __ldg(base[k] + (r + j) * step[k]);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                acc += static_cast<double>(vjp<F>(v[0][j], NOPS > 1 ? v[1][j] : 0.0f, NOPS > 2 ? v[2][j] : 0.0f));
        }
        for (; r < n; ++r) {
            const float gv = __ldg(base[0] + r * step[0]);
            const float pv = NOPS > 1 ? __ldg(base[1] + r * step[1]) : 0.0f;
            const float qv = NOPS > 2 ? __ldg(base[2] + r * step[2]) : 0.0f;
            acc += static_cast<double>(vjp<F>(gv, pv, qv));
        }
    }
    s_slice[w][lane] = acc;
    __syncthreads();
    if (w == 0) {
        double t = 0.0;
#pragma unroll
        for (unsigned j = 0; j < kSlices; ++j) t += s_slice[j][lane];
        if (d.out_d) {
            if (l < d.inner) d.out_d[l] = t;
        } else {
            s_res[lane] = round_out(t, d.divisor);
        }
    }
    if (d.out_d) return;
    __syncthreads();
    write_replicas(s_res, out, d.inner, rep);
}

// ---------------------------------------------------------------------------
// ROW layout. Each output k reduces W = R * inner elements (e = r*inner + l).
// grid = (min(K, 65535) rows, S segments of d.seg elements).
// ---------------------------------------------------------------------------
// The VJP values of the element group at reduced position e (4 lanes when
// VEC, else lane x only).
template <int F, bool VEC, bool HAS_R>
__device__ __forceinline__ float4 row_fetch(const float* __restrict__ g, const float* __restrict__ p,
                                            const float* __restrict__ q, const RedDesc& d, const long long base[3],
                                            unsigned long long e) {
    constexpr int NOPS = operands<F>();
    long long off[3] = {0, 0, 0};
    unsigned long long l = e;
    if constexpr (HAS_R) {
        const unsigned long long r = e / d.inner;
        l = e - r * d.inner;
        decode(r, d.nr, d.rdims, d.rs, off, nullptr);
    }
    if constexpr (VEC) {
        const float4 gv = load4(g, base[0] + off[0], d.is[0], l);
        const float4 pv = NOPS > 1 ? load4(p, base[1] + off[1], d.is[1], l) : gv;
        const float4 qv = NOPS > 2 ? load4(q, base[2] + off[2], d.is[2], l) : gv;
        return make_float4(vjp<F>(gv.x, pv.x, qv.x), vjp<F>(gv.y, pv.y, qv.y), vjp<F>(gv.z, pv.z, qv.z),
                           vjp<F>(gv.w, pv.w, qv.w));
    } else {
        const long long li = static_cast<long long>(l);
        const float gv = __ldg(g + base[0] + off[0] + li * d.is[0]);
        const float pv = NOPS > 1 ? __ldg(p + base[1] + off[1] + li * d.is[1]) : gv;
        const float qv = NOPS > 2 ? __ldg(q + base[2] + off[2] + li * d.is[2]) : gv;
        return make_float4(vjp<F>(gv, pv, qv), 0.f, 0.f, 0.f);
    }
}

template <bool VEC>
__device__ __forceinline__ void row_accumulate(double& acc0, double& acc1, float4 v) {
    if constexpr (VEC) {
        acc0 += static_cast<double>(v.x) + static_cast<double>(v.y);
        acc1 += static_cast<double>(v.z) + static_cast<double>(v.w);
    } else {
        acc0 += static_cast<double>(v.x);
    }
}

template <int F, bool VEC, bool HAS_R>
__global__ void __launch_bounds__(kThreads)
reduce_row_kernel(const float* __restrict__ g, const float* __restrict__ p, const float* __restrict__ q,
                  const RedDesc d, float* __restrict__ out, double* __restrict__ partial) {
    constexpr int V = VEC ? 4 : 1;
    constexpr unsigned long long STEP = static_cast<unsigned long long>(kThreads) * V;
    __shared__ double s_red[32];
    const unsigned long long W = d.R * d.inner;
    const unsigned s = blockIdx.y;
    const unsigned long long e0 = s * d.seg;
    const unsigned long long e1 = min(W, e0 + d.seg);
    for (unsigned long long k = blockIdx.x; k < d.K; k += gridDim.x) {
        long long base[3];
        decode(k, d.nk, d.kdims, d.ks, base, nullptr);
        double acc0 = 0.0, acc1 = 0.0;
        unsigned long long e = e0 + threadIdx.x * V;
        // eight independent groups in flight per thread (the bytes in flight,
        // not the arithmetic, set the pace of a streaming reduction)
        for (; e + 7 * STEP < e1; e += 8 * STEP) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = row_fetch<F, VEC, HAS_R>(g, p, q, d, base, e + u * STEP);
#pragma unroll
            for (int u = 0; u < 8; ++u) row_accumulate<VEC>(acc0, acc1, v[u]);
        }
        for (; e < e1; e += STEP) row_accumulate<VEC>(acc0, acc1, row_fetch<F, VEC, HAS_R>(g, p, q, d, base, e));
        const double total = block_sum(acc0 + acc1, s_red);
        if (threadIdx.x == 0) {
            if (d.S == 1 && d.out_d) d.out_d[k] = total;
            else if (d.S == 1) out[k] = round_out(total, d.divisor);
            else partial[k * d.S + s] = total;
        }
        __syncthreads();
    }
}

// Combine ROW partials [K][S]: one CTA per output, thread t adds partials
// t, t+256, ... and a fixed block tree combines the threads (an order that
// depends only on S), so few outputs with many segments (a full sum) finish in
// parallel rather than in one thread.
__global__ void __launch_bounds__(kFinishWideThreads)
reduce_row_finish(const double* __restrict__ partial, unsigned S, unsigned long long K, float divisor,
                  float* __restrict__ out, double* __restrict__ out_d) {
    pdl_wait();  // a programmatic launch: the partials' kernel has finished and its writes are visible
    __shared__ double s_red[32];
    for (unsigned long long k = blockIdx.x; k < K; k += gridDim.x) {
        double acc = 0.0;
        // partials t, t + B, t + 2B, ... in order, eight loads in flight
        for (unsigned s0 = threadIdx.x; s0 < S; s0 += 8 * blockDim.x) {
            double v[8];
#pragma unroll
            for (unsigned j = 0; j < 8; ++j) {
                const unsigned s = s0 + j * blockDim.x;
                v[j] = s < S ? partial[k * S + s] : 0.0;
            }
#pragma unroll
            for (unsigned j = 0; j < 8; ++j)
                if (s0 + j * blockDim.x < S) acc += v[j];
        }
        acc = block_sum(acc, s_red);
        if (threadIdx.x == 0) {
            if (out_d) out_d[k] = acc;
            else out[k] = round_out(acc, divisor);
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// Host: build the canonical layout and launch.
// ---------------------------------------------------------------------------
struct Src {
    const float* ptr{nullptr};
    long long st[kMaxRank]{};  // aligned to the source dims
};

// Strides of a contiguous operand of `shape` aligned to the source shape.
static Src align(const float* ptr, const size_t* shape, int rank, const size_t* src_shape, int src_rank,
                 const char* what) {
    Src s;
    s.ptr = ptr;
    if (rank > src_rank) fail(VC_ERR_INVALID, std::string(what) + ": operand rank exceeds the output rank");
    long long contiguous = 1;
    for (int i = rank - 1; i >= 0; --i) {
        const int o = i + (src_rank - rank);
        if (shape[i] != src_shape[o] && shape[i] != 1)
            fail(VC_ERR_INVALID, std::string(what) + ": operand does not broadcast to the output shape");
        s.st[o] = shape[i] == 1 ? 0 : contiguous;
        contiguous *= static_cast<long long>(shape[i]);
    }
    return s;
}

// Returns whether the float output was written `rep` times (consecutive
// copies of the target block); otherwise only the first copy is written.
template <int F>
static bool launch_vjp_reduce(const Src ops[3], const size_t* src_shape, int src_rank, const size_t* t_shape,
                              int t_rank, float* out, float divisor, double* out_d = nullptr,
                              unsigned long long rep = 1) {
    // 1. classify source dims: 0 drop (size 1), 1 kept, 2 reduced.
    if (t_rank > src_rank) fail(VC_ERR_INVALID, "sum_to_shape: cannot reduce to a larger rank");
    const int lead = src_rank - t_rank;
    int cls[kMaxRank];
    std::size_t outsz = 1;
    for (int i = 0; i < src_rank; ++i) {
        const std::size_t td = i < lead ? 1 : t_shape[i - lead];
        const std::size_t sd = src_shape[i];
        if (td != sd && td != 1) fail(VC_ERR_INVALID, "sum_to_shape: cannot reduce the gradient to the target shape");
        cls[i] = sd == 1 ? 0 : (td == 1 ? 2 : 1);
        if (cls[i] == 1) outsz *= sd;
    }
    // 1b. A kept dim along which every operand is constant (stride 0) gives
    // the same result at every index: reduce on the compact shape without it
    // and broadcast the result (e.g. the gradient of a * b for the scalar
    // upstream of sum(): 2^32 products collapse to 2^17). Same values,
    // bit for bit: each output sums the same products in the same order.
    if (outsz > 0 && !out_d) {
        bool any = false;
        size_t c_src[kMaxRank], c_tgt[kMaxRank], full_tgt[kMaxRank];
        for (int i = 0; i < src_rank; ++i) {
            bool inv = cls[i] == 1;
            for (int k = 0; k < operands<F>(); ++k) inv = inv && ops[k].st[i] == 0;
            any = any || inv;
            full_tgt[i] = i < lead ? 1 : t_shape[i - lead];
            c_src[i] = inv ? 1 : src_shape[i];
            c_tgt[i] = inv ? 1 : full_tgt[i];
        }
        if (any) {
            std::size_t csz = 1;
            for (int i = 0; i < src_rank; ++i) csz *= c_tgt[i];
            // When every such dim lies outside the others (a leading
            // replication: the target is rep consecutive copies of the
            // compact block), reduce straight into the first copy and let a
            // small reduction write the copies itself; else broadcast.
            bool leading = true, seen_other = false;
            for (int i = 0; i < src_rank; ++i) {
                if (full_tgt[i] == 1) continue;
                if (c_tgt[i] == 1) leading = leading && !seen_other;
                else seen_other = true;
            }
            const unsigned long long rep = outsz / csz;
            if (leading) {
                const unsigned long long ask = rep * csz <= kReplicateMax ? rep : 1;
                const bool all = launch_vjp_reduce<F>(ops, c_src, src_rank, c_tgt, src_rank, out, divisor, nullptr, ask) &&
                                 ask == rep;
                if (!all) {
                    const unsigned long long total4 = (rep - 1) * csz / 4;
                    if (csz % 4 == 0 && aligned16(out) && total4 < (1ull << 32)) {
                        replicate_front_block<<<stream_grid(4 * total4), kThreads, 0, stream()>>>(
                            out, csz / 4, FastDiv(static_cast<unsigned>(csz / 4)), total4);
                        check_launch("replicate");
                    } else {
                        const size_t one_shape[2] = {1, csz}, rest_shape[2] = {static_cast<size_t>(rep - 1), csz};
                        broadcast_copy(out, one_shape, 2, out + csz, rest_shape, 2);
                    }
                }
                return true;
            }
            Scratch compact(csz * sizeof(float));
            launch_vjp_reduce<F>(ops, c_src, src_rank, c_tgt, src_rank, compact.as<float>(), divisor);
            broadcast_copy(compact.as<float>(), c_tgt, src_rank, out, full_tgt, src_rank);
            return true;
        }
    }
    // 2. merge neighbours of the same class that are contiguous for every operand.
    struct Dim { int cls; unsigned long long size; long long st[3]; };
    Dim dims[kMaxRank];
    int nd = 0;
    for (int i = 0; i < src_rank; ++i) {
        if (cls[i] == 0) continue;
        Dim cur{cls[i], src_shape[i], {ops[0].st[i], ops[1].st[i], ops[2].st[i]}};
        if (nd > 0 && dims[nd - 1].cls == cur.cls) {
            Dim& prev = dims[nd - 1];
            bool ok = true;
            for (int k = 0; k < 3; ++k)
                ok = ok && prev.st[k] == cur.st[k] * static_cast<long long>(cur.size);
            if (ok) {
                prev.size *= cur.size;
                for (int k = 0; k < 3; ++k) prev.st[k] = cur.st[k];
                continue;
            }
        }
        dims[nd++] = cur;
    }
    if (outsz == 0) return true;
    RedDesc d{};
    d.divisor = divisor;
    d.out_d = out_d;
    if (nd == 0 || dims[nd - 1].cls == 1) {
        // COLUMN (also covers "nothing to reduce").
        const unsigned long long inner = nd ? dims[nd - 1].size : 1;
        d.inner = inner;
        for (int k = 0; k < 3; ++k) d.is[k] = nd ? dims[nd - 1].st[k] : 0;
        d.K = 1;
        d.R = 1;
        for (int i = 0; i + 1 < nd; ++i) {
            if (dims[i].cls == 1) {
                d.kdims[d.nk] = dims[i].size;
                for (int k = 0; k < 3; ++k) d.ks[k][d.nk] = dims[i].st[k];
                ++d.nk;
                d.K *= dims[i].size;
            } else {
                d.rdims[d.nr] = dims[i].size;
                for (int k = 0; k < 3; ++k) d.rs[k][d.nr] = dims[i].st[k];
                ++d.nr;
                d.R *= dims[i].size;
            }
        }
        bool vec = inner % 4 == 0 && aligned16(out);
        for (int k = 0; k < operands<F>(); ++k) {
            if (d.is[k] == 0) continue;
            if (d.is[k] != 1 || !aligned16(ops[k].ptr)) { vec = false; break; }
            for (int i = 0; i < d.nk; ++i) vec = vec && d.ks[k][i] % 4 == 0;
            for (int i = 0; i < d.nr; ++i) vec = vec && d.rs[k][i] % 4 == 0;
        }
        if (d.nk == 0 && d.nr == 1 && d.R <= kSlicedMaxRows && inner <= kSlicedMaxOutputs &&
            d.R * inner <= kSlicedMaxElements && (!out_d || rep == 1)) {
            reduce_col_sliced<F><<<static_cast<unsigned>((inner + 31) / 32), kSliceThreads, 0, stream()>>>(
                ops[0].ptr, ops[1].ptr, ops[2].ptr, d, out, rep);
            check_launch("reduce_col_sliced");
            return true;
        }
        const unsigned V = vec ? 4 : 1;
        const unsigned long long lanes = (inner + V - 1) / V;
        const unsigned long long threads_now = lanes * d.K;
        unsigned long long S = (kTargetThreads + threads_now - 1) / threads_now;
        S = std::min<unsigned long long>(S, (d.R + kMinSegment - 1) / kMinSegment);
        S = std::max<unsigned long long>(S, 1);
        S = std::min<unsigned long long>(S, kMaxSumSegments);
        d.seg = (d.R + S - 1) / S;
        d.S = static_cast<unsigned>((d.R + d.seg - 1) / d.seg);
        dim3 grid(static_cast<unsigned>((lanes + kThreads - 1) / kThreads),
                  static_cast<unsigned>(std::min<unsigned long long>(d.K, 65535)), d.S);
        if (grid.x > 0x7fffffffu) fail(VC_ERR_OVERFLOW, "reduction inner run too long");
        Scratch partial(d.S > 1 ? static_cast<std::size_t>(d.S) * d.K * d.inner * sizeof(double) : 8);
        const bool g_const = d.is[0] == 0 && d.rs[0][0] == 0;  // operand 0 is one value (a 0-d gradient)
        if (vec && d.nk == 0 && d.nr == 1 && g_const && operands<F>() > 1)
            reduce_col_simple<F, true><<<grid, kThreads, 0, stream()>>>(ops[0].ptr, ops[1].ptr, ops[2].ptr, d, out, partial.as<double>());
        else if (vec && d.nk == 0 && d.nr == 1)
            reduce_col_simple<F><<<grid, kThreads, 0, stream()>>>(ops[0].ptr, ops[1].ptr, ops[2].ptr, d, out, partial.as<double>());
        else if (vec) reduce_col_kernel<F, true><<<grid, kThreads, 0, stream()>>>(ops[0].ptr, ops[1].ptr, ops[2].ptr, d, out, partial.as<double>());
        else reduce_col_kernel<F, false><<<grid, kThreads, 0, stream()>>>(ops[0].ptr, ops[1].ptr, ops[2].ptr, d, out, partial.as<double>());
        check_launch("reduce_col");
        if (d.S > 1) {
            const unsigned long long count = d.K * d.inner;
            // shape-only choice: the order of the additions is part of the result
            if (d.S >= 2 * kSlices && count <= kSlicedMaxOutputs) {
                launch_pdl(reduce_col_finish_sliced, dim3(static_cast<unsigned>((count + 31) / 32)), dim3(kSliceThreads), 0,
                           stream(), partial.as<double>(), d.S, count, divisor, out, out_d,
                           out_d ? 1ull : static_cast<unsigned long long>(rep));
                check_launch("reduce_col_finish");
                return true;
            }
            launch_pdl(reduce_col_finish, dim3(grid_for(count, kThreads)), dim3(kThreads), 0, stream(), partial.as<double>(),
                       d.S, count, divisor, out, out_d);
            check_launch("reduce_col_finish");
        }
        return rep == 1;
    }
    // ROW: innermost reduced run.
    const unsigned long long inner = dims[nd - 1].size;
    d.inner = inner;
    for (int k = 0; k < 3; ++k) d.is[k] = dims[nd - 1].st[k];
    d.K = 1;
    d.R = 1;
    for (int i = 0; i + 1 < nd; ++i) {
        if (dims[i].cls == 1) {
            d.kdims[d.nk] = dims[i].size;
            for (int k = 0; k < 3; ++k) d.ks[k][d.nk] = dims[i].st[k];
            ++d.nk;
            d.K *= dims[i].size;
        } else {
            d.rdims[d.nr] = dims[i].size;
            for (int k = 0; k < 3; ++k) d.rs[k][d.nr] = dims[i].st[k];
            ++d.nr;
            d.R *= dims[i].size;
        }
    }
    bool vec = inner % 4 == 0;
    for (int k = 0; k < operands<F>(); ++k) {
        if (d.is[k] == 0) continue;
        if (d.is[k] != 1 || !aligned16(ops[k].ptr)) { vec = false; break; }
        for (int i = 0; i < d.nk; ++i) vec = vec && d.ks[k][i] % 4 == 0;
        for (int i = 0; i < d.nr; ++i) vec = vec && d.rs[k][i] % 4 == 0;
    }
    const unsigned long long W = d.R * d.inner;
    unsigned long long S = row_segments(d.K, W);
    unsigned long long seg = (W + S - 1) / S;
    seg = (seg + 3) / 4 * 4;  // keep float4 groups inside one segment
    d.seg = seg;
    d.S = static_cast<unsigned>((W + seg - 1) / seg);
    dim3 grid(static_cast<unsigned>(std::min<unsigned long long>(d.K, 1u << 20)), d.S);
    Scratch partial(d.S > 1 ? static_cast<std::size_t>(d.S) * d.K * sizeof(double) : 8);
    const bool has_r = d.nr > 0;
#define VC_ROW(V, H) reduce_row_kernel<F, V, H><<<grid, kThreads, 0, stream()>>>(ops[0].ptr, ops[1].ptr, ops[2].ptr, d, out, partial.as<double>())
    if (vec) { if (has_r) VC_ROW(true, true); else VC_ROW(true, false); }
    else { if (has_r) VC_ROW(false, true); else VC_ROW(false, false); }
#undef VC_ROW
    check_launch("reduce_row");
    if (d.S > 1) {
        launch_pdl(reduce_row_finish,
                   dim3(static_cast<unsigned>(std::min<unsigned long long>(d.K, static_cast<unsigned long long>(sm_count()) * 8))),
                   dim3(row_finish_threads(d.K, d.S)), 0, stream(), partial.as<double>(), d.S, d.K, divisor, out, out_d);
        check_launch("reduce_row_finish");
    }
    return rep == 1;
}

static void vjp_reduce(int f, const Src ops[3], const size_t* src_shape, int src_rank, const size_t* t_shape,
                       int t_rank, float* out, float divisor = 0.0f, double* out_d = nullptr) {
    switch (f) {
        case V_G: launch_vjp_reduce<V_G>(ops, src_shape, src_rank, t_shape, t_rank, out, divisor, out_d); return;
        case V_NEG: launch_vjp_reduce<V_NEG>(ops, src_shape, src_rank, t_shape, t_rank, out, divisor, out_d); return;
        case V_MUL: launch_vjp_reduce<V_MUL>(ops, src_shape, src_rank, t_shape, t_rank, out, divisor, out_d); return;
        case V_DIV_A: launch_vjp_reduce<V_DIV_A>(ops, src_shape, src_rank, t_shape, t_rank, out, divisor, out_d); return;
        default: launch_vjp_reduce<V_DIV_B>(ops, src_shape, src_rank, t_shape, t_rank, out, divisor, out_d); return;
    }
}

// ---------------------------------------------------------------------------
// Same-shape binary backward: both gradients in one pass (20 B/elem for mul
// and div: read g, a, b; write da, db).
// ---------------------------------------------------------------------------
template <int OP>
__device__ __forceinline__ void bb_one(float av, float bv, float gv, float& ga, float& gb) {
    if constexpr (OP == VC_ADD) { ga = gv; gb = gv; }
    else if constexpr (OP == VC_SUB) { ga = gv; gb = -gv; }
    else if constexpr (OP == VC_MUL) { ga = vjp<V_MUL>(gv, bv, 0.f); gb = vjp<V_MUL>(gv, av, 0.f); }
    else { ga = vjp<V_DIV_A>(gv, bv, 0.f); gb = vjp<V_DIV_B>(gv, av, bv); }
}

template <int OP>
__device__ __forceinline__ void bb_four(const float4& av, const float4& bv, const float4& gv, float4& ga, float4& gb) {
    bb_one<OP>(av.x, bv.x, gv.x, ga.x, gb.x);
    bb_one<OP>(av.y, bv.y, gv.y, ga.y, gb.y);
    bb_one<OP>(av.z, bv.z, gv.z, ga.z, gb.z);
    bb_one<OP>(av.w, bv.w, gv.w, ga.w, gb.w);
}

// Chunked stream (stream_grid): CTA b owns float4 groups
// [kChunk4 * b, kChunk4 * (b + 1)), four per thread, all loads first.
template <int OP, bool VEC>
__global__ void __launch_bounds__(kThreads)
binary_backward_flat(const float* __restrict__ a, const float* __restrict__ b, const float* __restrict__ g,
                     float* __restrict__ da, float* __restrict__ db, std::size_t n) {
    constexpr bool NEED_AB = OP == VC_MUL || OP == VC_DIV;
    if constexpr (VEC) {
        const std::size_t n4 = n >> 2;
        const std::size_t base = static_cast<std::size_t>(blockIdx.x) * kChunk4 + threadIdx.x;
        float4 gv[kStreamRounds], av[kStreamRounds], bv[kStreamRounds];
#pragma unroll
        for (unsigned u = 0; u < kStreamRounds; ++u) {
            const std::size_t k = base + u * kStreamThreads;
            if (k < n4) {
                gv[u] = ldg4(g + 4 * k);
                av[u] = NEED_AB ? ldg4(a + 4 * k) : gv[u];
                bv[u] = NEED_AB ? ldg4(b + 4 * k) : gv[u];
            }
        }
#pragma unroll
        for (unsigned u = 0; u < kStreamRounds; ++u) {
            const std::size_t k = base + u * kStreamThreads;
            if (k < n4) {
                float4 ga, gb;
                bb_four<OP>(av[u], bv[u], gv[u], ga, gb);
                st4(da + 4 * k, ga);
                st4(db + 4 * k, gb);
            }
        }
        if (blockIdx.x == gridDim.x - 1)
            for (std::size_t k = n4 * 4 + threadIdx.x; k < n; k += kStreamThreads)
                bb_one<OP>(NEED_AB ? a[k] : 0.f, NEED_AB ? b[k] : 0.f, g[k], da[k], db[k]);
    } else {
        const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
        const std::size_t tid = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
        for (std::size_t k = tid; k < n; k += stride)
            bb_one<OP>(NEED_AB ? a[k] : 0.f, NEED_AB ? b[k] : 0.f, g[k], da[k], db[k]);
    }
}

// ---------------------------------------------------------------------------
// Two-sided broadcast backward from ONE read of a dense upstream g.
//
// When a and b are both broadcast (out = a * b with a [P,1,R,L] and
// b [1,Q,1,L], say), each needs its own reduction of g: da over the dims
// where a has extent 1, db over the dims where b has. The reference runs one
// full pass per reduced axis for each (src/autograd.cpp:50-72 after
// src/ops.cpp:124-156). Canonical layout after dropping unit dims and merging
// neighbours of one class:
//   L -- the innermost run, kept by both gradients (float4 columns);
//   U -- the dims only a spans (da keeps them, db reduces them), at most two;
//   V -- the dims only b spans (db keeps them, da reduces them), V <= 128;
//   K -- outer dims both span (independent problems, grid.z), at most two.
// A CTA owns 32 floats of L (8 float4 columns), all V and a segment of U.
// Its 512 threads are 64 row slots x 8 columns; row slot rs = (us, vs) with
// VS v-slots (a power of two, 4..64) and US = 64 / VS u-slots: a step covers
// US consecutive u, and the thread owns v = vs + VS*i (i < NV <= 2) at its
// column for every step, so b sits in registers. Loads are plain 128-bit
// loads of g, UNR = 8 / NV steps per group, so every thread keeps eight in
// flight (two 512-thread CTAs per SM keep HBM busy on these 128-byte pieces
// of 2 MB-strided rows); the group's a rows arrive in shared memory by
// cp.async one group ahead. Per step
//   * da: the thread folds its NV terms in float (i order), the 4 v-slots of
//     a warp (one u) fold in float across lanes (xor 8, then 16), and the
//     VS / 4 warp partials of a u are combined in double, in a fixed tree,
//     through an XOR-swizzled shared buffer (conflict-free both ways); da is
//     written rounded once;
//   * db: the terms add into a per-(v, column) float block that is flushed
//     every 8 steps into double accumulators in shared memory; at the end
//     the US u-slots are combined in order into db (or into this U segment's
//     partial, summed in segment order by reduce_col_finish).
// Every combine order depends on the shape only. The float blocks (at most 8
// terms) add a relative error of a few float ulps of the block; the
// reference's sums round once per axis, so both sit well inside the sum
// tolerance.
// ---------------------------------------------------------------------------
constexpr unsigned kFThreads = 512;
constexpr unsigned kFCols = 8;                  // float4 columns per CTA
constexpr unsigned kFChunk = kFCols * 4;        // floats of L per CTA
constexpr unsigned kFRowSlots = kFThreads / kFCols;
constexpr unsigned kFWarps = kFThreads / 32;
constexpr unsigned kFMaxV = 128;
constexpr unsigned kFFlush = 8;                 // steps per float block of db
// CTAs to aim for: 8 waves of 148 SMs x 2 resident CTAs (a constant: the
// split, and so the result, depends on the shape alone).
constexpr unsigned long long kFTargetCtas = 148ull * 2 * 8;
constexpr unsigned long long kFMinUSeg = 128;
constexpr std::size_t kFMaxSmem = 112 * 1024;

struct FusedDesc {
    int nk;
    unsigned U0, U1;
    FastDiv u1fd;
    long long ua0, ua1;          // da (= a layout) strides of the U dims
    long long gu0, gu1;          // g strides of the U dims
    unsigned long long kdims[2]; // K dims, outer first
    long long ka[2], kb[2], kg[2];  // da / db / g strides of the K dims
    int nv;
    unsigned vdims[2];           // V dims, outer first
    long long vb[2], vg[2];      // db (= b layout) / g strides of the V dims
    unsigned U, V;
    unsigned long long L;        // innermost run, a multiple of 4
    unsigned useg, S;            // u positions per segment, segments
    unsigned VS, US;             // v-slots, u-slots per step
    unsigned vs_log2;
    unsigned long long db_count; // elements of db (the partial stride)
    double* da_d;                // unrounded outputs (shard partials) when set
    double* db_d;
};

__device__ __forceinline__ long long decode_v(const FusedDesc& d, unsigned v, const long long* st) {
    long long o = 0;
    for (int i = d.nv - 1; i >= 0; --i) {
        const unsigned c = v % d.vdims[i];
        v /= d.vdims[i];
        o += static_cast<long long>(c) * st[i];
    }
    return o;
}

__device__ __forceinline__ float4 add4(float4 x, float4 y) { return make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w); }
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <unsigned NV> __host__ __device__ constexpr unsigned fused_unroll() { return 8u / NV; }

// Shared memory of one CTA: [2][UNR][kFWarps][32] float da partials,
// [NV][2][kFThreads] double2 db accumulators, [2][UNR][US][kFCols] float4 a rows.
template <unsigned NV>
static std::size_t fused_smem(unsigned US) {
    constexpr unsigned UNR = fused_unroll<NV>();
    return 2ull * UNR * kFWarps * 32 * sizeof(float) + NV * 2ull * kFThreads * sizeof(double2) +
           2ull * UNR * US * kFCols * sizeof(float4);
}

// The four row slots of a warp (lanes c, c+8, c+16, c+24: the four v-slots
// of one u at column c) fold their float4 into one float per lane: a
// reduce-scatter in the fixed tree ((r0 + r1) + (r2 + r3)) per component,
// three shuffles instead of eight. Lane row slot k ends with component
// (k & 1) * 2 + (k >> 1) of the column.
// Read-only float4 load that asks L2 to fetch the whole 256-byte block around
// it: the fused backward reads g in 128-byte pieces (32 floats of a row per
// CTA) and the CTA on the neighbouring 32 floats runs at the same time, so
// each DRAM access serves both (dense-g backward of configuration 5: about
// one point of HBM bandwidth, 84-85% -> 86%).
__device__ __forceinline__ float4 ld4_l2_256(const float* p) {
    float4 v;
    asm("ld.global.nc.L2::256B.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ float fold4_scatter(float4 v, unsigned k) {
    const bool odd = k & 1u, high = k & 2u;
    float keep0 = odd ? v.z : v.x, keep1 = odd ? v.w : v.y;
    const float send0 = odd ? v.x : v.z, send1 = odd ? v.y : v.w;
    keep0 += __shfl_xor_sync(0xffffffffu, send0, 8);
    keep1 += __shfl_xor_sync(0xffffffffu, send1, 8);
    const float keep = high ? keep1 : keep0, send = high ? keep0 : keep1;
    return keep + __shfl_xor_sync(0xffffffffu, send, 16);
}

// FULL: every v of the thread exists (V = NV * VS) and every column is
// inside L (L a multiple of 32), so the per-row and per-column checks go.
template <int OP, unsigned NV, bool FULL>
__global__ void __launch_bounds__(kFThreads, 2)
bcast_backward_fused(const float* __restrict__ g, const float* __restrict__ a, const float* __restrict__ b,
                     const FusedDesc d, float* __restrict__ da, float* __restrict__ db,
                     double* __restrict__ partial) {
    constexpr unsigned UNR = fused_unroll<NV>();
    constexpr bool NEED_AB = OP == VC_MUL || OP == VC_DIV;
    extern __shared__ __align__(16) unsigned char fsm[];
    float* part = reinterpret_cast<float*>(fsm);
    double2* dacc = reinterpret_cast<double2*>(part + 2 * UNR * kFWarps * 32);
    float4* arow = reinterpret_cast<float4*>(dacc + NV * 2 * kFThreads);

    const unsigned t = threadIdx.x, c = t & (kFCols - 1), rs = t / kFCols, w = t >> 5, lane = t & 31;
    const unsigned rk = lane >> 3;  // row slot within the warp
    const unsigned vs = rs & (d.VS - 1), us = rs >> d.vs_log2;
    const unsigned long long l0 = static_cast<unsigned long long>(blockIdx.x) * kFChunk;
    const bool col_ok = FULL || l0 + 4 * c < d.L;
    const unsigned seg = blockIdx.y;
    const unsigned u0 = seg * d.useg;
    const unsigned u1 = min(d.U, u0 + d.useg);
    const unsigned nsteps = (u1 - u0 + d.US - 1) / d.US;
    const unsigned ngroups = (nsteps + UNR - 1) / UNR;

    // K position of this CTA: da / db / g offsets
    long long ka = 0, kb = 0, kg = 0;
    {
        unsigned long long r = blockIdx.z;
        for (int i = d.nk - 1; i >= 0; --i) {
            const unsigned long long q = r % d.kdims[i];
            r /= d.kdims[i];
            ka += static_cast<long long>(q) * d.ka[i];
            kb += static_cast<long long>(q) * d.kb[i];
            kg += static_cast<long long>(q) * d.kg[i];
        }
    }
    const float* ak = a + ka + static_cast<long long>(l0);

    float4 breg[NV], facc[NV];
    const float* gp[NV];  // this thread's rows of g at u = 0
    bool vok[NV];
#pragma unroll
    for (unsigned i = 0; i < NV; ++i) {
        const unsigned v = vs + d.VS * i;
        vok[i] = FULL || (v < d.V && col_ok);
        gp[i] = g + kg + (vok[i] ? decode_v(d, v, d.vg) : 0) + static_cast<long long>(l0 + 4 * c);
        breg[i] = NEED_AB && vok[i] ? ldg4(b + kb + decode_v(d, v, d.vb) + static_cast<long long>(l0 + 4 * c))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
        facc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        dacc[(i * 2 + 0) * kFThreads + t] = make_double2(0.0, 0.0);
        dacc[(i * 2 + 1) * kFThreads + t] = make_double2(0.0, 0.0);
    }
    // a rows of group n (UNR steps x US u x kFCols columns) into arow[n & 1]
    auto fetch_a = [&](unsigned n) {
        float4* dst = arow + (n & 1u) * UNR * d.US * kFCols;
        const unsigned count = UNR * d.US * kFCols;
        for (unsigned e = t; e < count; e += kFThreads) {
            const unsigned cc = e % kFCols, q = e / kFCols;  // q = k * US + u-slot
            const unsigned u = u0 + n * UNR * d.US + q;
            if (u < u1 && (FULL || l0 + 4 * cc < d.L)) {
                unsigned c0, c1;
                d.u1fd.divmod(u, c0, c1);
                cp_async16(dst + e, ak + static_cast<long long>(c0) * d.ua0 + static_cast<long long>(c1) * d.ua1 + 4 * cc);
            }
        }
    };
    if (NEED_AB) {
        fetch_a(0);
        cp_async_wait_all();
    }
    __syncthreads();

    // One group of UNR steps; CHECK: some step of it lies past the segment.
    auto group = [&](unsigned n, auto check) {
        constexpr bool CHECK = decltype(check)::value;
        const unsigned s0 = n * UNR;
        float4 gv[UNR][NV];
        bool sok[UNR];
#pragma unroll
        for (unsigned k = 0; k < UNR; ++k) {
            const unsigned u = u0 + (s0 + k) * d.US + us;
            sok[k] = !CHECK || u < u1;
            unsigned c0 = 0, c1 = 0;
            if (sok[k]) d.u1fd.divmod(u, c0, c1);
            const long long go = static_cast<long long>(c0) * d.gu0 + static_cast<long long>(c1) * d.gu1;
#pragma unroll
            for (unsigned i = 0; i < NV; ++i)
                gv[k][i] = sok[k] && vok[i] ? ld4_l2_256(gp[i] + go) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float* pb = part + (n & 1u) * UNR * kFWarps * 32;
        const float4* ab = arow + (n & 1u) * UNR * d.US * kFCols;
#pragma unroll
        for (unsigned k = 0; k < UNR; ++k) {
            float4 dap = make_float4(0.f, 0.f, 0.f, 0.f);
            if (sok[k]) {
                const float4 av = NEED_AB ? ab[(k * d.US + us) * kFCols + c] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (unsigned i = 0; i < NV; ++i) {
                    if (!vok[i]) continue;
                    float4 ga, gb;
                    bb_four<OP>(av, breg[i], gv[k][i], ga, gb);
                    dap = i == 0 ? ga : add4(dap, ga);
                    facc[i] = add4(facc[i], gb);
                }
            }
            pb[(k * kFWarps + w) * 32 + c * 4 + (rk & 1u) * 2 + (rk >> 1)] = fold4_scatter(dap, rk);
            if ((s0 + k + 1) % kFFlush == 0) {
#pragma unroll
                for (unsigned i = 0; i < NV; ++i) {
                    double2& lo = dacc[(i * 2 + 0) * kFThreads + t];
                    double2& hi = dacc[(i * 2 + 1) * kFThreads + t];
                    lo.x += static_cast<double>(facc[i].x);
                    lo.y += static_cast<double>(facc[i].y);
                    hi.x += static_cast<double>(facc[i].z);
                    hi.y += static_cast<double>(facc[i].w);
                    facc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        }
    };

    const unsigned gw = d.VS >> 2;  // warps per u
    for (unsigned n = 0; n < ngroups; ++n) {
        if (NEED_AB && n + 1 < ngroups) fetch_a(n + 1);
        if (u0 + ((n + 1) * UNR) * d.US <= u1) group(n, std::false_type{});
        else group(n, std::true_type{});
        if (NEED_AB) cp_async_wait_all();  // the next group's a rows
        __syncthreads();
        // da: one output float per item, the gw warp partials of its u
        // added in warp order (double)
        const unsigned s0 = n * UNR;
        const float* pb = part + (n & 1u) * UNR * kFWarps * 32;
        for (unsigned item = t; item < UNR * d.US * 32; item += kFThreads) {
            const unsigned f = item & 31, q = item >> 5;  // q = k * US + u-slot
            const unsigned k = q / d.US, uslot = q - k * d.US;
            const unsigned u = u0 + (s0 + k) * d.US + uslot;
            if (u >= u1 || (!FULL && l0 + f >= d.L)) continue;
            const float* src = pb + (k * kFWarps + uslot * gw) * 32 + f;
            double s = 0.0;
            for (unsigned j = 0; j < gw; ++j) s += static_cast<double>(src[j * 32]);
            unsigned c0, c1;
            d.u1fd.divmod(u, c0, c1);
            const long long off = ka + static_cast<long long>(c0) * d.ua0 + static_cast<long long>(c1) * d.ua1 +
                                  static_cast<long long>(l0 + f);
            if (d.da_d) d.da_d[off] = s;
            else da[off] = static_cast<float>(s);
        }
    }
    // db: the last float block, then the US u-slots in order
#pragma unroll
    for (unsigned i = 0; i < NV; ++i) {
        double2& lo = dacc[(i * 2 + 0) * kFThreads + t];
        double2& hi = dacc[(i * 2 + 1) * kFThreads + t];
        lo.x += static_cast<double>(facc[i].x);
        lo.y += static_cast<double>(facc[i].y);
        hi.x += static_cast<double>(facc[i].z);
        hi.y += static_cast<double>(facc[i].w);
    }
    __syncthreads();
    for (unsigned o = t; o < d.V * kFCols * 2; o += kFThreads) {
        const unsigned h = o & 1u, cc = (o >> 1) & (kFCols - 1), v = o / (2 * kFCols);
        if (!FULL && l0 + 4 * cc >= d.L) continue;
        const unsigned vsl = v & (d.VS - 1), i = v >> d.vs_log2;
        double2 s = make_double2(0.0, 0.0);
        for (unsigned x = 0; x < d.US; ++x) {
            const double2 q = dacc[(i * 2 + h) * kFThreads + ((x << d.vs_log2) + vsl) * kFCols + cc];
            s.x += q.x;
            s.y += q.y;
        }
        const long long off = kb + decode_v(d, v, d.vb) + static_cast<long long>(l0 + 4 * cc + 2 * h);
        if (d.S > 1) {
            double* p = partial + static_cast<unsigned long long>(seg) * d.db_count + off;
            p[0] = s.x;
            p[1] = s.y;
        } else if (d.db_d) {
            d.db_d[off] = s.x;
            d.db_d[off + 1] = s.y;
        } else {
            db[off] = static_cast<float>(s.x);
            db[off + 1] = static_cast<float>(s.y);
        }
    }
}

template <int OP, unsigned NV, bool FULL>
static void launch_fused(const float* g, const float* a, const float* b, const FusedDesc& d, dim3 grid,
                         float* da, float* db, double* partial) {
    static bool configured = false;
    if (!configured) {
        VC_CUDA(cudaFuncSetAttribute(bcast_backward_fused<OP, NV, FULL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kFMaxSmem)));
        configured = true;
    }
    bcast_backward_fused<OP, NV, FULL><<<grid, kFThreads, fused_smem<NV>(d.US), stream()>>>(g, a, b, d, da, db,
                                                                                            partial);
}

template <int OP>
static void launch_fused_nv(unsigned nv, bool full, const float* g, const float* a, const float* b,
                            const FusedDesc& d, dim3 grid, float* da, float* db, double* partial) {
    if (nv == 1) {
        if (full) launch_fused<OP, 1, true>(g, a, b, d, grid, da, db, partial);
        else launch_fused<OP, 1, false>(g, a, b, d, grid, da, db, partial);
    } else {
        if (full) launch_fused<OP, 2, true>(g, a, b, d, grid, da, db, partial);
        else launch_fused<OP, 2, false>(g, a, b, d, grid, da, db, partial);
    }
}

// ---------------------------------------------------------------------------
// The same two-sided broadcast backward, fed by the tensor memory accelerator
// (TMA), for the shapes where the V rows of g at one u form one tensor-map
// box: one V dim of 16 * NVT rows (NVT = 1, 2, 4 or 8), no K dims, L a
// multiple of 64, g dense, a / b strides in whole 16-byte units. g is viewed
// as the 4-D tensor (l, u1, v, u0) -- innermost first -- whatever the order
// of its strides.
//
// A CTA owns 64 floats of L and a segment of U. One lane of warp 8 (the
// producer) streams, per u, the [V x 64] tile of g (one 4-D tensor copy) and
// a's 64 floats (one bulk copy) into a ring of shared-memory stages, each
// with a "full" mbarrier (completed by the copies' byte count) and an
// "empty" one (one arrival per consumer warp). The copies of the next stages
// stay in flight while the 8 consumer warps reduce the current stage, so the
// kernel does not wait on memory latency at its per-step barrier.
//
// Consumer thread (float4 column c = lane & 15, v-group q = 2 * warp +
// lane / 16) owns the rows v = 16 j + q, j < NVT (its b values stay in
// registers), per step:
//   * da[u, 4c .. 4c+3]: its NVT terms folded in float (j order), the two
//     half-warps added (one shuffle; a + b == b + a), and the 8 warp
//     partials added in double in warp order by the CTA's first 64 threads,
//     after a barrier of the consumer warps; da is rounded once;
//   * db[v, 4c ..]: float blocks of 8 steps flushed into double registers;
//     at the end each thread writes its own NVT x 4 outputs (or this U
//     segment's partial, summed in segment order by reduce_col_finish).
// The combine orders depend on the shape only.
//
// Every wait is bounded. A consumer whose wait gives up (error word set)
// skips the stage; the consumer barrier is a reduction (bar.red.or), so all
// consumers see the give-up at the same step and leave together, writing
// nothing. The producer stops issuing when its own wait gives up, and before
// it returns waits (bounded) for every copy it issued, so no copy lands in a
// finished CTA's shared memory.
// ---------------------------------------------------------------------------
constexpr unsigned kTCols = 64;                  // floats of L per CTA
constexpr unsigned kTConsumerWarps = 8;
constexpr unsigned kTConsumers = kTConsumerWarps * 32;
constexpr unsigned kTThreads = kTConsumers + 32;  // + the producer warp
constexpr std::size_t kTSmemMax = 227 * 1024;   // opt-in shared memory per CTA
constexpr unsigned kTMaxStages = 16;
constexpr unsigned kTFlush = 8;                  // steps per float block of db
// CTAs to aim for: 4 waves of 148 SMs x 1 resident CTA (a constant: the split,
// and so the result, depends on the shape alone).
constexpr unsigned long long kTTargetCtas = 148ull * 4;

struct TmaDesc {
    unsigned U, U1;
    FastDiv u1fd;
    long long ua0, ua1;           // a (= da) strides of the U dims
    long long vb;                 // b (= db) stride of the V dim
    unsigned useg, S, stages;
    unsigned long long db_count;  // elements of db (the partial stride)
    double* da_d;                 // unrounded outputs (shard partials) when set
    double* db_d;
};

// Shared memory of one CTA: alignment slack, [stages][16 NVT][64] g tiles,
// [stages][64] a rows, [2][8][64] float da partials, [4 NVT][256] double db
// accumulators (thread-minor), 2 x stages mbarriers.
template <unsigned NVT>
static std::size_t tma_smem_fixed() {
    return 128 + 2 * kTConsumerWarps * kTCols * sizeof(float) + 4ull * NVT * kTConsumers * sizeof(double);
}
template <unsigned NVT>
static std::size_t tma_stage_bytes() {
    return (16ull * NVT * kTCols + kTCols) * sizeof(float) + 2 * 8;
}
template <unsigned NVT>
static unsigned tma_stages() {
    return static_cast<unsigned>(std::min<std::size_t>(kTMaxStages, (kTSmemMax - tma_smem_fixed<NVT>()) /
                                                                         tma_stage_bytes<NVT>()));
}
template <unsigned NVT>
static std::size_t tma_smem(unsigned stages) {
    return tma_smem_fixed<NVT>() + stages * tma_stage_bytes<NVT>();
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, unsigned long long* bar, int x,
                                            int y, int z, int w) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<unsigned long long>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void bulk_load_smem(void* dst, const void* src, unsigned bytes, unsigned long long* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

template <int OP, unsigned NVT>
__global__ void __launch_bounds__(kTThreads, 1)
bcast_backward_tma(const __grid_constant__ CUtensorMap gmap, const float* __restrict__ a,
                   const float* __restrict__ b, const TmaDesc d, float* __restrict__ da, float* __restrict__ db,
                   double* __restrict__ partial, unsigned* __restrict__ err) {
    constexpr bool NEED_AB = OP == VC_MUL || OP == VC_DIV;
    constexpr unsigned kTile = 16 * NVT * kTCols;  // floats of g per stage
    extern __shared__ unsigned char tsm_raw[];
    // stage tiles 128-byte aligned (tensor copy destination)
    unsigned char* tsm = tsm_raw + ((128 - (smem_addr(tsm_raw) & 127)) & 127);
    float* gst = reinterpret_cast<float*>(tsm);     // [stages][16 NVT][64]
    float* ast = gst + d.stages * kTile;            // [stages][64]
    float* part = ast + d.stages * kTCols;          // [2][8 warps][64]
    double* dsm = reinterpret_cast<double*>(part + 2 * kTConsumerWarps * kTCols);  // [4 NVT][256]
    unsigned long long* full = reinterpret_cast<unsigned long long*>(dsm + 4 * NVT * kTConsumers);
    unsigned long long* empty = full + d.stages;

    const unsigned t = threadIdx.x, w = t >> 5, lane = t & 31;
    const unsigned l0 = blockIdx.x * kTCols;
    const unsigned seg = blockIdx.y;
    const unsigned u0 = seg * d.useg;
    const unsigned nsteps = min(d.U, u0 + d.useg) - u0;
    if (t == 0) {
        for (unsigned s = 0; s < d.stages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, kTConsumerWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (w == kTConsumerWarps) {  // producer
        if (lane == 0) {
            constexpr unsigned kTx = (kTile + (NEED_AB ? kTCols : 0)) * sizeof(float);
            unsigned issued = 0;
            for (unsigned s = 0; s < nsteps; ++s) {
                const unsigned slot = s % d.stages;
                if (s >= d.stages && !mbar_wait_bounded(empty + slot, ((s / d.stages) - 1) & 1u, err)) break;
                unsigned c0, c1;
                d.u1fd.divmod(u0 + s, c0, c1);
                mbar_expect_tx(full + slot, kTx);
                tma_load_4d(gst + slot * kTile, &gmap, full + slot, static_cast<int>(l0), static_cast<int>(c1), 0,
                            static_cast<int>(c0));
                if (NEED_AB)
                    bulk_load_smem(ast + slot * kTCols,
                                   a + static_cast<long long>(c0) * d.ua0 + static_cast<long long>(c1) * d.ua1 + l0,
                                   kTCols * sizeof(float), full + slot);
                ++issued;
            }
            // the last `stages` copies issued land before the CTA may finish
            for (unsigned s = issued > d.stages ? issued - d.stages : 0; s < issued; ++s)
                mbar_wait_bounded(full + s % d.stages, (s / d.stages) & 1u, err, kWaitPolls / 16);
        }
        return;
    }

    // consumers
    const unsigned c = lane & 15, q = 2 * w + (lane >> 4);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 breg[NVT], facc[NVT];
    double* dacc = dsm + t;  // element k of this thread: dacc[k * 256]
#pragma unroll
    for (unsigned j = 0; j < NVT; ++j) {
        breg[j] = NEED_AB ? ldg4(b + static_cast<long long>(16 * j + q) * d.vb + l0 + 4 * c) : zero;
        facc[j] = zero;
#pragma unroll
        for (unsigned k = 0; k < 4; ++k) dacc[(4 * j + k) * kTConsumers] = 0.0;
    }
    auto flush = [&]() {
#pragma unroll
        for (unsigned j = 0; j < NVT; ++j) {
            dacc[(4 * j + 0) * kTConsumers] += static_cast<double>(facc[j].x);
            dacc[(4 * j + 1) * kTConsumers] += static_cast<double>(facc[j].y);
            dacc[(4 * j + 2) * kTConsumers] += static_cast<double>(facc[j].z);
            dacc[(4 * j + 3) * kTConsumers] += static_cast<double>(facc[j].w);
            facc[j] = zero;
        }
    };
    bool gave_up = false;
    for (unsigned s = 0; s < nsteps; ++s) {
        const unsigned slot = s % d.stages;
        const bool ok = mbar_wait_bounded(full + slot, (s / d.stages) & 1u, err);
        float4 dap = zero;
        if (ok) {
            const float4* tile = reinterpret_cast<const float4*>(gst + slot * kTile);
            const float4 av = NEED_AB ? reinterpret_cast<const float4*>(ast + slot * kTCols)[c] : zero;
#pragma unroll
            for (unsigned j = 0; j < NVT; ++j) {
                float4 ga, gb;
                bb_four<OP>(av, breg[j], tile[(16 * j + q) * (kTCols / 4) + c], ga, gb);
                dap = j == 0 ? ga : add4(dap, ga);
                facc[j] = add4(facc[j], gb);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + slot);
        dap.x += __shfl_xor_sync(0xffffffffu, dap.x, 16);
        dap.y += __shfl_xor_sync(0xffffffffu, dap.y, 16);
        dap.z += __shfl_xor_sync(0xffffffffu, dap.z, 16);
        dap.w += __shfl_xor_sync(0xffffffffu, dap.w, 16);
        float* pb = part + (s & 1u) * kTConsumerWarps * kTCols;
        if (lane < 16) reinterpret_cast<float4*>(pb + w * kTCols)[c] = dap;
        if (named_barrier_or<1, kTConsumers>(!ok)) {
            gave_up = true;
            break;
        }
        if (t < kTCols) {
            double sum = 0.0;
#pragma unroll
            for (unsigned k = 0; k < kTConsumerWarps; ++k) sum += static_cast<double>(pb[k * kTCols + t]);
            unsigned c0, c1;
            d.u1fd.divmod(u0 + s, c0, c1);
            const long long off = static_cast<long long>(c0) * d.ua0 + static_cast<long long>(c1) * d.ua1 + l0 + t;
            if (d.da_d) d.da_d[off] = sum;
            else da[off] = static_cast<float>(sum);
        }
        if ((s + 1) % kTFlush == 0) flush();
    }
    if (gave_up) return;
    flush();
#pragma unroll
    for (unsigned j = 0; j < NVT; ++j) {
        const long long off = static_cast<long long>(16 * j + q) * d.vb + l0 + 4 * c;
        const double r0 = dacc[(4 * j + 0) * kTConsumers], r1 = dacc[(4 * j + 1) * kTConsumers],
                     r2 = dacc[(4 * j + 2) * kTConsumers], r3 = dacc[(4 * j + 3) * kTConsumers];
        if (d.S > 1) {
            double* p = partial + static_cast<unsigned long long>(seg) * d.db_count + off;
            p[0] = r0;
            p[1] = r1;
            p[2] = r2;
            p[3] = r3;
        } else if (d.db_d) {
            d.db_d[off] = r0;
            d.db_d[off + 1] = r1;
            d.db_d[off + 2] = r2;
            d.db_d[off + 3] = r3;
        } else {
            st4(db + off, make_float4(static_cast<float>(r0), static_cast<float>(r1), static_cast<float>(r2),
                                      static_cast<float>(r3)));
        }
    }
}

template <int OP, unsigned NVT>
static void launch_tma(const CUtensorMap& map, const float* a, const float* b, const TmaDesc& d, dim3 grid, float* da,
                       float* db, double* partial) {
    static bool configured = false;
    const std::size_t smem = tma_smem<NVT>(d.stages);
    if (!configured) {
        VC_CUDA(cudaFuncSetAttribute(bcast_backward_tma<OP, NVT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(tma_smem<NVT>(tma_stages<NVT>()))));
        configured = true;
    }
    bcast_backward_tma<OP, NVT><<<grid, kTThreads, smem, stream()>>>(map, a, b, d, da, db, partial,
                                                                      device_error_word());
}

template <int OP>
static void launch_tma_nvt(unsigned nvt, const CUtensorMap& map, const float* a, const float* b, const TmaDesc& d,
                           dim3 grid, float* da, float* db, double* partial) {
    switch (nvt) {
        case 1: launch_tma<OP, 1>(map, a, b, d, grid, da, db, partial); break;
        case 2: launch_tma<OP, 2>(map, a, b, d, grid, da, db, partial); break;
        case 4: launch_tma<OP, 4>(map, a, b, d, grid, da, db, partial); break;
        default: launch_tma<OP, 8>(map, a, b, d, grid, da, db, partial); break;
    }
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime
// (the library does not link libcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return static_cast<EncodeTiledFn>(nullptr);
        }
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// Launch bcast_backward_tma for a classified shape (FusedDesc filled by the
// caller) when it qualifies; false, having launched nothing, otherwise.
static bool try_tma_bcast_backward(int op, const float* a, const float* b, const float* g, const FusedDesc& fd,
                                   float* da, float* db, double* da_d, double* db_d, std::size_t b_numel) {
    if (fd.nk != 0 || fd.nv != 1 || fd.L % kTCols != 0 || fd.L > 0x7fffffffull) return false;
    const unsigned V = fd.V;
    if (V != 16 && V != 32 && V != 64 && V != 128) return false;
    const bool need_ab = op == VC_MUL || op == VC_DIV;
    if (fd.vb[0] % 4 != 0 || (need_ab && (fd.ua0 % 4 != 0 || fd.ua1 % 4 != 0))) return false;
    if (fd.gu0 % 4 != 0 || fd.gu1 % 4 != 0 || fd.vg[0] % 4 != 0) return false;
    if (fd.U0 > 0x7fffffffu || fd.U1 > 0x7fffffffu) return false;
    EncodeTiledFn encode = encode_tiled();
    if (!encode) return false;
    // g as (l, u1, v, u0); a size-1 dim gets a harmless valid stride
    const auto stride_of = [&](unsigned size, long long st) -> cuuint64_t {
        return static_cast<cuuint64_t>(size > 1 ? st : static_cast<long long>(fd.L)) * sizeof(float);
    };
    const cuuint64_t dims[4] = {fd.L, fd.U1, V, fd.U0};
    const cuuint64_t strides[3] = {stride_of(fd.U1, fd.gu1), stride_of(V, fd.vg[0]), stride_of(fd.U0, fd.gu0)};
    for (cuuint64_t s : strides)
        if (s % 16 != 0 || s >= (1ull << 40)) return false;
    const cuuint32_t box[4] = {kTCols, 1, V, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUtensorMap map;
    if (encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(g), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;

    TmaDesc d{};
    d.U = fd.U;
    d.U1 = fd.U1;
    d.u1fd = fd.u1fd;
    d.ua0 = fd.ua0;
    d.ua1 = fd.ua1;
    d.vb = fd.vb[0];
    const unsigned long long chunks = fd.L / kTCols;
    unsigned long long S = (kTTargetCtas + chunks - 1) / chunks;
    S = std::max<unsigned long long>(1, std::min<unsigned long long>({S, (fd.U + kFMinUSeg - 1) / kFMinUSeg, 65535}));
    const unsigned long long useg = (fd.U + S - 1) / S;
    d.useg = static_cast<unsigned>(useg);
    d.S = static_cast<unsigned>((fd.U + useg - 1) / useg);
    d.stages = V == 16 ? tma_stages<1>() : V == 32 ? tma_stages<2>() : V == 64 ? tma_stages<4>() : tma_stages<8>();
    d.db_count = b_numel;
    d.da_d = da_d;
    d.db_d = db_d;
    if (chunks > 0x7fffffffull) return false;

    Scratch partial(d.S > 1 ? static_cast<std::size_t>(d.S) * b_numel * sizeof(double) : 8);
    const dim3 grid(static_cast<unsigned>(chunks), d.S, 1);
    const unsigned nvt = V / 16;
    switch (op) {
        case VC_ADD: launch_tma_nvt<VC_ADD>(nvt, map, a, b, d, grid, da, db, partial.as<double>()); break;
        case VC_SUB: launch_tma_nvt<VC_SUB>(nvt, map, a, b, d, grid, da, db, partial.as<double>()); break;
        case VC_MUL: launch_tma_nvt<VC_MUL>(nvt, map, a, b, d, grid, da, db, partial.as<double>()); break;
        default: launch_tma_nvt<VC_DIV>(nvt, map, a, b, d, grid, da, db, partial.as<double>()); break;
    }
    check_launch("bcast_backward_tma");
    if (d.S > 1) {
        reduce_col_finish<<<grid_for(b_numel, kThreads), kThreads, 0, stream()>>>(partial.as<double>(), d.S, b_numel,
                                                                                   0.0f, db, db_d);
        check_launch("bcast_backward_finish");
    }
    return true;
}

// Classify the output dims of a two-sided broadcast backward and launch
// bcast_backward_fused when the shape fits it (see above; also g dense over
// the output and every pointer 16-byte aligned). Returns false, having
// launched nothing, otherwise.
static bool try_fused_bcast_backward(int op, const float* a, const Src& sa, const float* b, const Src& sb,
                                     const float* g, const Src& sg, const size_t* src, int rank, float* da,
                                     float* db, double* da_d, double* db_d, std::size_t b_numel) {
    if (!(da || da_d) || !(db || db_d)) return false;
    long long contiguous = 1;
    for (int i = rank - 1; i >= 0; --i) {
        if (src[i] != 1 && sg.st[i] != contiguous) return false;
        contiguous *= static_cast<long long>(src[i]);
    }
    // classes: 1 = both span (kept by both), 2 = only a spans (U), 3 = only b spans (V)
    struct Dim { int cls; unsigned long long size; long long st[3]; };  // g, a, b strides
    Dim dims[kMaxRank];
    int nd = 0;
    for (int i = 0; i < rank; ++i) {
        if (src[i] == 1) continue;
        const bool in_a = sa.st[i] != 0, in_b = sb.st[i] != 0;
        if (!in_a && !in_b) return false;
        Dim cur{in_a && in_b ? 1 : (in_a ? 2 : 3), src[i], {sg.st[i], sa.st[i], sb.st[i]}};
        if (nd > 0 && dims[nd - 1].cls == cur.cls) {
            Dim& prev = dims[nd - 1];
            bool ok = true;
            for (int k = 0; k < 3; ++k) ok = ok && prev.st[k] == cur.st[k] * static_cast<long long>(cur.size);
            if (ok) {
                prev.size *= cur.size;
                for (int k = 0; k < 3; ++k) prev.st[k] = cur.st[k];
                continue;
            }
        }
        dims[nd++] = cur;
    }
    if (nd < 3 || dims[nd - 1].cls != 1) return false;
    FusedDesc d{};
    d.L = dims[nd - 1].size;
    if (d.L % 4 != 0 || d.L > 0x7fffffffull) return false;
    const void* ptrs[5] = {a, b, g, da ? static_cast<const void*>(da) : da_d, db ? static_cast<const void*>(db) : db_d};
    for (int k = 0; k < 5; ++k)
        if (!aligned16(ptrs[k])) return false;
    Dim ud[2], vd[2], kd[2];  // outer first
    int nu = 0, nv = 0, nk = 0;
    for (int i = 0; i + 1 < nd; ++i) {
        const Dim& x = dims[i];
        if (x.size > 0x7fffffffull) return false;
        if (x.cls == 2) { if (nu == 2) return false; ud[nu++] = x; }
        else if (x.cls == 3) { if (nv == 2) return false; vd[nv++] = x; }
        else { if (nk == 2) return false; kd[nk++] = x; }
    }
    if (nu == 0 || nv == 0) return false;
    unsigned long long U = 1, V = 1, K = 1;
    for (int i = 0; i < nu; ++i) U *= ud[i].size;
    for (int i = 0; i < nv; ++i) V *= vd[i].size;
    for (int i = 0; i < nk; ++i) K *= kd[i].size;
    if (V < 2 || V > kFMaxV || U < 2 || U > 0x7fffffffull || K > 65535) return false;
    d.U = static_cast<unsigned>(U);
    d.V = static_cast<unsigned>(V);
    d.nv = nv;
    for (int i = 0; i < nv; ++i) {
        d.vdims[i] = static_cast<unsigned>(vd[i].size);
        d.vb[i] = vd[i].st[2];
        d.vg[i] = vd[i].st[0];
    }
    d.nk = nk;
    for (int i = 0; i < nk; ++i) {
        d.kdims[i] = kd[i].size;
        d.ka[i] = kd[i].st[1];
        d.kb[i] = kd[i].st[2];
        d.kg[i] = kd[i].st[0];
    }
    // U as (U0 outer, U1 inner); one U dim is (1, U)
    const Dim uinner = ud[nu - 1];
    const Dim uouter = nu == 2 ? ud[0] : Dim{2, 1, {uinner.st[0] * static_cast<long long>(uinner.size),
                                                    uinner.st[1] * static_cast<long long>(uinner.size), 0}};
    d.U1 = static_cast<unsigned>(uinner.size);
    d.U0 = static_cast<unsigned>(uouter.size);
    d.u1fd = FastDiv(d.U1);
    d.ua1 = uinner.st[1];
    d.ua0 = uouter.st[1];
    d.gu1 = uinner.st[0];
    d.gu0 = uouter.st[0];
    if (try_tma_bcast_backward(op, a, b, g, d, da, db, da_d, db_d, b_numel)) return true;
    unsigned vs = 4;
    while (vs < V && vs < kFRowSlots) vs *= 2;
    d.VS = vs;
    d.US = kFRowSlots / vs;
    const unsigned nvper = static_cast<unsigned>((V + vs - 1) / vs);
    d.vs_log2 = 0;
    while ((1u << d.vs_log2) < vs) ++d.vs_log2;
    const unsigned long long chunks = (d.L + kFChunk - 1) / kFChunk;
    unsigned long long S = (kFTargetCtas + chunks * K - 1) / (chunks * K);
    S = std::min<unsigned long long>(S, (U + kFMinUSeg - 1) / kFMinUSeg);
    S = std::max<unsigned long long>(1, std::min<unsigned long long>(S, 65535));
    unsigned long long useg = (U + S - 1) / S;
    useg = (useg + d.US - 1) / d.US * d.US;
    d.useg = static_cast<unsigned>(useg);
    d.S = static_cast<unsigned>((U + useg - 1) / useg);
    d.db_count = b_numel;
    d.da_d = da_d;
    d.db_d = db_d;
    if ((nvper == 1 ? fused_smem<1>(d.US) : fused_smem<2>(d.US)) > kFMaxSmem) return false;
    Scratch partial(d.S > 1 ? static_cast<std::size_t>(d.S) * b_numel * sizeof(double) : 8);
    const dim3 grid(static_cast<unsigned>(chunks), d.S, static_cast<unsigned>(K));
    const bool full = V == static_cast<unsigned long long>(nvper) * vs && d.L % kFChunk == 0;
    switch (op) {
        case VC_ADD: launch_fused_nv<VC_ADD>(nvper, full, g, a, b, d, grid, da, db, partial.as<double>()); break;
        case VC_SUB: launch_fused_nv<VC_SUB>(nvper, full, g, a, b, d, grid, da, db, partial.as<double>()); break;
        case VC_MUL: launch_fused_nv<VC_MUL>(nvper, full, g, a, b, d, grid, da, db, partial.as<double>()); break;
        default: launch_fused_nv<VC_DIV>(nvper, full, g, a, b, d, grid, da, db, partial.as<double>()); break;
    }
    check_launch("bcast_backward_fused");
    if (d.S > 1) {
        reduce_col_finish<<<grid_for(b_numel, kThreads), kThreads, 0, stream()>>>(partial.as<double>(), d.S, b_numel,
                                                                                   0.0f, db, db_d);
        check_launch("bcast_backward_finish");
    }
    return true;
}

// ---------------------------------------------------------------------------
// Max / argmax over [outer, length, inner] with the reference's scan
// semantics (cpu_backend.cpp:443-453): a strictly larger value replaces the
// best, so the first maximal index wins; NaN never replaces, so a NaN wins
// only at index 0. Candidates exclude NaN; the finish step applies the
// index-0 rule (unless `continuation`, used by later shards of a sharded
// axis, which report -1 when they have no candidate).
// ---------------------------------------------------------------------------
struct MaxOut {
    float* values;        // max value, or argmax as float (reference convention)
    long long* index;     // int64 argmax (optional)
    int argmax_as_value;  // write the index (as float) into values
    int continuation;
    long long index_base; // added to indices (shard offset)
};

__device__ __forceinline__ void max_finish_write(MaxCand c, float first, const MaxOut& o, unsigned long long k) {
    if (!o.continuation && first != first) c = MaxCand{first, 0};  // NaN at index 0 wins
    const long long idx = c.i < 0 ? -1 : c.i + o.index_base;
    if (o.values) o.values[k] = o.argmax_as_value ? static_cast<float>(idx) : c.v;
    if (o.index) o.index[k] = idx;
}

// ROW (inner == 1): grid = (rows, segments).
template <bool VEC>
__global__ void __launch_bounds__(kThreads)
max_row_kernel(const float* __restrict__ in, unsigned long long outer, unsigned long long length,
               unsigned long long seg, unsigned S, MaxOut o, float* __restrict__ pv, long long* __restrict__ pi) {
    __shared__ float s_v[32];
    __shared__ long long s_i[32];
    const unsigned s = blockIdx.y;
    const unsigned long long e0 = s * seg, e1 = min(length, e0 + seg);
    for (unsigned long long row = blockIdx.x; row < outer; row += gridDim.x) {
        const float* x = in + row * length;
        MaxCand c{0.0f, -1};
        if constexpr (VEC) {
            constexpr unsigned long long STEP = kThreads * 4ull;
            auto take4 = [&](const float4& v, unsigned long long e) {
                c = max_take(c, v.x, static_cast<long long>(e));
                c = max_take(c, v.y, static_cast<long long>(e + 1));
                c = max_take(c, v.z, static_cast<long long>(e + 2));
                c = max_take(c, v.w, static_cast<long long>(e + 3));
            };
            unsigned long long e = e0 + threadIdx.x * 4;
            for (; e + STEP < e1; e += 2 * STEP) {  // two loads in flight, taken in index order
                const float4 v0 = ldg4(x + e), v1 = ldg4(x + e + STEP);
                take4(v0, e);
                take4(v1, e + STEP);
            }
            for (; e < e1; e += STEP) take4(ldg4(x + e), e);
        } else {
            for (unsigned long long e = e0 + threadIdx.x; e < e1; e += kThreads)
                c = max_take(c, __ldg(x + e), static_cast<long long>(e));
        }
        c = block_max(c, s_v, s_i);
        if (threadIdx.x == 0) {
            if (S == 1) max_finish_write(c, __ldg(x), o, row);
            else { pv[row * S + s] = c.v; pi[row * S + s] = c.i; }
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kFinishWideThreads)
max_row_finish(const float* __restrict__ in, unsigned long long outer, unsigned long long length, unsigned S,
               const float* __restrict__ pv, const long long* __restrict__ pi, MaxOut o) {
    pdl_wait();  // a programmatic launch: the partials' kernel has finished and its writes are visible
    // One CTA per row. max_combine (larger value, then smaller index) is
    // associative and commutative, so the tree order cannot change the result.
    __shared__ float s_v[32];
    __shared__ long long s_i[32];
    for (unsigned long long row = blockIdx.x; row < outer; row += gridDim.x) {
        MaxCand c{0.0f, -1};
        for (unsigned s0 = threadIdx.x; s0 < S; s0 += 4 * blockDim.x) {
            MaxCand v[4];
#pragma unroll
            for (unsigned j = 0; j < 4; ++j) {
                const unsigned s = s0 + j * blockDim.x;
                v[j] = s < S ? MaxCand{pv[row * S + s], pi[row * S + s]} : MaxCand{0.0f, -1};
            }
#pragma unroll
            for (unsigned j = 0; j < 4; ++j) c = max_combine(c, v[j]);
        }
        c = block_max(c, s_v, s_i);
        if (threadIdx.x == 0) max_finish_write(c, in[row * length], o, row);
        __syncthreads();
    }
}

// COLUMN (inner > 1): grid = (ceil(inner/(256*V)), min(outer, 65535), segments).
// VEC: each thread owns 4 adjacent columns (float4 loads); four positions of
// the reduced axis in flight, taken in index order.
template <bool VEC>
__global__ void __launch_bounds__(kThreads)
max_col_kernel(const float* __restrict__ in, unsigned long long outer, unsigned long long length,
               unsigned long long inner, unsigned long long seg, unsigned S, MaxOut o,
               float* __restrict__ pv, long long* __restrict__ pi) {
    constexpr int V = VEC ? 4 : 1;
    const unsigned long long i = (static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x) * V;
    if (i >= inner) return;
    const unsigned s = blockIdx.z;
    const unsigned long long a0 = s * seg, a1 = min(length, a0 + seg);
    for (unsigned long long ob = blockIdx.y; ob < outer; ob += gridDim.y) {
        const float* x = in + ob * length * inner + i;
        MaxCand c[V];
#pragma unroll
        for (int v = 0; v < V; ++v) c[v] = MaxCand{0.0f, -1};
        auto take = [&](const float4& v, unsigned long long a) {
            const long long ai = static_cast<long long>(a);
            c[0] = max_take(c[0], v.x, ai);
            if constexpr (VEC) {
                c[1] = max_take(c[1], v.y, ai);
                c[2] = max_take(c[2], v.z, ai);
                c[3] = max_take(c[3], v.w, ai);
            }
        };
        auto load = [&](unsigned long long a) -> float4 {
            if constexpr (VEC) return ldg4(x + a * inner);
            else return make_float4(__ldg(x + a * inner), 0.f, 0.f, 0.f);
        };
        unsigned long long a = a0;
        for (; a + 7 < a1; a += 8) {
            float4 v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = load(a + k);
#pragma unroll
            for (int k = 0; k < 8; ++k) take(v[k], a + k);
        }
        for (; a < a1; ++a) take(load(a), a);
#pragma unroll
        for (int v = 0; v < V; ++v) {
            const unsigned long long k = ob * inner + i + v;
            if (S == 1) max_finish_write(c[v], __ldg(x + v), o, k);
            else { pv[s * outer * inner + k] = c[v].v; pi[s * outer * inner + k] = c[v].i; }
        }
    }
}

__global__ void __launch_bounds__(kThreads)
max_col_finish(const float* __restrict__ in, unsigned long long outer, unsigned long long length,
               unsigned long long inner, unsigned S, const float* __restrict__ pv,
               const long long* __restrict__ pi, MaxOut o) {
    pdl_wait();  // a programmatic launch: the partials' kernel has finished and its writes are visible
    const unsigned long long count = outer * inner;
    const unsigned long long stride = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
    for (unsigned long long k = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x; k < count;
         k += stride) {
        // eight segment candidates in flight, combined in segment order
        MaxCand c{0.0f, -1};
        unsigned s = 0;
        for (; s + 8 <= S; s += 8) {
            MaxCand v[8];
#pragma unroll
            for (unsigned q = 0; q < 8; ++q)
                v[q] = MaxCand{__ldg(pv + (s + q) * count + k), __ldg(pi + (s + q) * count + k)};
#pragma unroll
            for (unsigned q = 0; q < 8; ++q) c = max_combine(c, v[q]);
        }
        for (; s < S; ++s) c = max_combine(c, MaxCand{pv[s * count + k], pi[s * count + k]});
        const unsigned long long ob = k / inner, i = k - ob * inner;
        max_finish_write(c, in[ob * length * inner + i], o, k);
    }
}

static void launch_max(const float* in, std::size_t outer, std::size_t length, std::size_t inner, MaxOut o) {
    if (outer * inner == 0) return;
    if (length == 0) fail(VC_ERR_INVALID, "max/argmax over an empty axis is undefined");
    cudaStream_t st = stream();
    if (inner == 1) {
        const unsigned long long S = row_segments(outer, length);
        unsigned long long seg = ((length + S - 1) / S + 3) / 4 * 4;
        const unsigned Sn = static_cast<unsigned>((length + seg - 1) / seg);
        const bool vec = aligned16(in) && length % 4 == 0;
        Scratch pv(Sn > 1 ? outer * Sn * sizeof(float) : 8), pi(Sn > 1 ? outer * Sn * sizeof(long long) : 8);
        dim3 grid(static_cast<unsigned>(std::min<std::size_t>(outer, 1u << 20)), Sn);
        if (vec) max_row_kernel<true><<<grid, kThreads, 0, st>>>(in, outer, length, seg, Sn, o, pv.as<float>(), pi.as<long long>());
        else max_row_kernel<false><<<grid, kThreads, 0, st>>>(in, outer, length, seg, Sn, o, pv.as<float>(), pi.as<long long>());
        check_launch("max_row");
        if (Sn > 1) {
            launch_pdl(max_row_finish,
                       dim3(static_cast<unsigned>(std::min<std::size_t>(outer, static_cast<std::size_t>(sm_count()) * 8))),
                       dim3(row_finish_threads(outer, Sn)), 0, st, in, static_cast<unsigned long long>(outer),
                       static_cast<unsigned long long>(length), Sn, pv.as<float>(), pi.as<long long>(), o);
            check_launch("max_row_finish");
        }
        return;
    }
    const bool vec = inner % 4 == 0 && aligned16(in);
    const unsigned long long lanes = vec ? inner / 4 : inner;
    const unsigned long long threads_now = lanes * outer;
    unsigned long long S = (kTargetThreads + threads_now - 1) / threads_now;
    S = std::min<unsigned long long>(S, (length + kMinSegment - 1) / kMinSegment);
    S = std::max<unsigned long long>(1, std::min<unsigned long long>(S, 4096));
    const unsigned long long seg = (length + S - 1) / S;
    const unsigned Sn = static_cast<unsigned>((length + seg - 1) / seg);
    Scratch pv(Sn > 1 ? outer * inner * Sn * sizeof(float) : 8), pi(Sn > 1 ? outer * inner * Sn * sizeof(long long) : 8);
    dim3 grid(static_cast<unsigned>((lanes + kThreads - 1) / kThreads),
              static_cast<unsigned>(std::min<std::size_t>(outer, 65535)), Sn);
    if (vec) max_col_kernel<true><<<grid, kThreads, 0, st>>>(in, outer, length, inner, seg, Sn, o, pv.as<float>(), pi.as<long long>());
    else max_col_kernel<false><<<grid, kThreads, 0, st>>>(in, outer, length, inner, seg, Sn, o, pv.as<float>(), pi.as<long long>());
    check_launch("max_col");
    if (Sn > 1) {
        launch_pdl(max_col_finish, dim3(grid_for(outer * inner, kThreads)), dim3(kThreads), 0, st, in,
                   static_cast<unsigned long long>(outer), static_cast<unsigned long long>(length),
                   static_cast<unsigned long long>(inner), Sn, pv.as<float>(), pi.as<long long>(), o);
        check_launch("max_col_finish");
    }
}

// ---------------------------------------------------------------------------
// Backward of axis reductions, one write pass over [outer, length, inner]:
// MODE 0 sum  (g + 0), 1 mean ((g / length) + 0), 2 max (g at the argmax
// index, +0 elsewhere -- cpu::scatter_axis, cpu_backend.cpp:462-471).
// The output is walked as rows: with inner == 1 a row is one outer slice of
// `length` values sharing g[o]; with inner > 1 a row is (o, a) and holds
// `inner` values copied from g[o, :]. One division per row, 128-bit stores.
// ---------------------------------------------------------------------------
template <int MODE>
__device__ __forceinline__ float expand_value(float gv, long long w, unsigned long long a, float len) {
    if constexpr (MODE == 0) return gv + 0.0f;
    else if constexpr (MODE == 1) return (gv / len) + 0.0f;
    else return static_cast<unsigned long long>(w) == a ? gv : 0.0f;
}

template <int MODE, bool VEC>
__global__ void __launch_bounds__(kThreads)
expand_rows_kernel(const float* __restrict__ g, const long long* __restrict__ idx, const float* __restrict__ idxf,
                   float* __restrict__ out, unsigned long long outer, unsigned long long length,
                   unsigned* __restrict__ err) {
    const float len = static_cast<float>(length);
    for (unsigned long long o = blockIdx.x; o < outer; o += gridDim.x) {
        const float gv = __ldg(g + o);
        long long w = -1;
        if constexpr (MODE == 2) {
            w = idx ? __ldg(idx + o) : static_cast<long long>(__ldg(idxf + o));
            if (threadIdx.x == 0 && (w < 0 || static_cast<unsigned long long>(w) >= length)) atomicOr(err, kErrBadIndex);
        }
        float* row = out + o * length;
        if constexpr (VEC) {
            for (unsigned long long a = threadIdx.x * 4ull; a < length; a += kThreads * 4ull)
                st4_stream(row + a, make_float4(expand_value<MODE>(gv, w, a, len), expand_value<MODE>(gv, w, a + 1, len),
                                                expand_value<MODE>(gv, w, a + 2, len), expand_value<MODE>(gv, w, a + 3, len)));
        } else {
            for (unsigned long long a = threadIdx.x; a < length; a += kThreads) row[a] = expand_value<MODE>(gv, w, a, len);
        }
    }
}

template <int MODE, bool VEC>
__global__ void __launch_bounds__(kThreads)
expand_cols_kernel(const float* __restrict__ g, const long long* __restrict__ idx, const float* __restrict__ idxf,
                   float* __restrict__ out, unsigned long long outer, unsigned long long length,
                   unsigned long long inner, unsigned* __restrict__ err) {
    const float len = static_cast<float>(length);
    const unsigned long long rows = outer * length;
    for (unsigned long long t = blockIdx.x; t < rows; t += gridDim.x) {
        const unsigned long long o = t / length, a = t - o * length;
        const float* grow = g + o * inner;
        float* orow = out + t * inner;
        if constexpr (VEC) {
            for (unsigned long long i = threadIdx.x * 4ull; i < inner; i += kThreads * 4ull) {
                const float4 gv = ldg4(grow + i);
                long long w[4] = {-1, -1, -1, -1};
                if constexpr (MODE == 2) {
                    for (int u = 0; u < 4; ++u) {
                        const unsigned long long k = o * inner + i + u;
                        w[u] = idx ? __ldg(idx + k) : static_cast<long long>(__ldg(idxf + k));
                        if (a == 0 && (w[u] < 0 || static_cast<unsigned long long>(w[u]) >= length)) atomicOr(err, kErrBadIndex);
                    }
                }
                st4_stream(orow + i, make_float4(expand_value<MODE>(gv.x, w[0], a, len), expand_value<MODE>(gv.y, w[1], a, len),
                                                 expand_value<MODE>(gv.z, w[2], a, len), expand_value<MODE>(gv.w, w[3], a, len)));
            }
        } else {
            for (unsigned long long i = threadIdx.x; i < inner; i += kThreads) {
                const unsigned long long k = o * inner + i;
                long long w = -1;
                if constexpr (MODE == 2) {
                    w = idx ? __ldg(idx + k) : static_cast<long long>(__ldg(idxf + k));
                    if (a == 0 && (w < 0 || static_cast<unsigned long long>(w) >= length)) atomicOr(err, kErrBadIndex);
                }
                orow[i] = expand_value<MODE>(__ldg(grow + i), w, a, len);
            }
        }
    }
}

template <int MODE>
static void launch_expand_mode(const float* g, const long long* idx, const float* idxf, float* out,
                               std::size_t outer, std::size_t length, std::size_t inner) {
    cudaStream_t st = stream();
    unsigned* err = device_error_word();
    if (inner == 1) {
        const bool vec = length % 4 == 0 && aligned16(out);
        const unsigned grid = static_cast<unsigned>(std::min<std::size_t>(outer, 0x7fffffffull));  // a CTA per row
        if (vec) expand_rows_kernel<MODE, true><<<grid, kThreads, 0, st>>>(g, idx, idxf, out, outer, length, err);
        else expand_rows_kernel<MODE, false><<<grid, kThreads, 0, st>>>(g, idx, idxf, out, outer, length, err);
    } else {
        const bool vec = inner % 4 == 0 && aligned16(out) && aligned16(g);
        const unsigned grid = static_cast<unsigned>(std::min<std::size_t>(outer * length, static_cast<std::size_t>(sm_count()) * 16));
        if (vec) expand_cols_kernel<MODE, true><<<grid, kThreads, 0, st>>>(g, idx, idxf, out, outer, length, inner, err);
        else expand_cols_kernel<MODE, false><<<grid, kThreads, 0, st>>>(g, idx, idxf, out, outer, length, inner, err);
    }
    check_launch("axis_expand");
}

static void launch_axis_expand(int mode, const float* g, const long long* idx, const float* idxf, float* out,
                               std::size_t outer, std::size_t length, std::size_t inner) {
    if (!outer || !length || !inner) return;
    if (!g || !out) fail(VC_ERR_INVALID, "axis backward: null pointer");
    if (mode == 0) launch_expand_mode<0>(g, idx, idxf, out, outer, length, inner);
    else if (mode == 1) launch_expand_mode<1>(g, idx, idxf, out, outer, length, inner);
    else launch_expand_mode<2>(g, idx, idxf, out, outer, length, inner);
}

// ---------------------------------------------------------------------------
// Cross-GPU combine of shard partials laid out [nranks][count] (the order of
// an all-gather), always in rank order 0..R-1 -- independent of the order in
// which the collective moved the bytes.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads)
combine_sum_kernel(const double* __restrict__ parts, int nranks, unsigned long long count, float divisor, int negate,
                   float* __restrict__ out) {
    const unsigned long long stride = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
    for (unsigned long long k = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x; k < count;
         k += stride) {
        double acc = 0.0;
        for (int r = 0; r < nranks; ++r) acc += parts[static_cast<unsigned long long>(r) * count + k];
        float s = static_cast<float>(acc);
        if (negate) s = -s;
        out[k] = divisor != 0.0f ? s / divisor : s;
    }
}

// Rank 0's partial already carries the "NaN at index 0" rule; later shards
// report -1 when they have no candidate. max_combine keeps the smaller
// (global) index on ties, i.e. the lower rank.
__global__ void __launch_bounds__(kThreads)
combine_max_kernel(const float* __restrict__ vals, const long long* __restrict__ idx, int nranks,
                   unsigned long long count, int argmax_as_value, float* __restrict__ out_value,
                   long long* __restrict__ out_index) {
    const unsigned long long stride = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
    for (unsigned long long k = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x; k < count;
         k += stride) {
        MaxCand c{0.0f, -1};
        for (int r = 0; r < nranks; ++r) {
            const unsigned long long o = static_cast<unsigned long long>(r) * count + k;
            c = max_combine(c, MaxCand{vals[o], idx[o]});
        }
        if (out_value) out_value[k] = argmax_as_value ? static_cast<float>(c.i) : c.v;
        if (out_index) out_index[k] = c.i;
    }
}

}  // namespace

}  // namespace vc

using namespace vc;

extern "C" {

vc_status vc_cuda_sum_to_shape(const float* g, const size_t* g_shape, int g_rank, float* out,
                               const size_t* t_shape, int t_rank) {
    VC_API_BEGIN
    ensure_init();
    validate_rank(g_rank, "sum_to_shape");
    validate_rank(t_rank, "sum_to_shape");
    if (checked_numel(t_shape, t_rank) == 0) return VC_OK;
    if (!g || !out) fail(VC_ERR_INVALID, "sum_to_shape: null pointer");
    Src ops[3];
    ops[0] = align(g, g_shape, g_rank, g_shape, g_rank, "sum_to_shape");
    if (checked_numel(g_shape, g_rank) == 0) {
        VC_CUDA(cudaMemsetAsync(out, 0, checked_numel(t_shape, t_rank) * sizeof(float), stream()));
        return VC_OK;
    }
    vjp_reduce(V_G, ops, g_shape, g_rank, t_shape, t_rank, out);
    VC_API_END
}

vc_status vc_cuda_binary_backward(int op, const float* a, const size_t* a_shape, int a_rank,
                                  const float* b, const size_t* b_shape, int b_rank,
                                  const float* g, const size_t* g_shape, int g_rank,
                                  float* da, float* db) {
    VC_API_BEGIN
    ensure_init();
    validate_rank(a_rank, "binary_backward");
    validate_rank(b_rank, "binary_backward");
    validate_rank(g_rank, "binary_backward");
    if (op < VC_ADD || op > VC_DIV) fail(VC_ERR_INVALID, "unknown binary operation");
    // Output (source) shape = broadcast(a, b).
    const int rank = std::max(a_rank, b_rank);
    size_t src[kMaxRank];
    for (int i = 0; i < rank; ++i) {
        const size_t ad = i < rank - a_rank ? 1 : a_shape[i - (rank - a_rank)];
        const size_t bd = i < rank - b_rank ? 1 : b_shape[i - (rank - b_rank)];
        if (ad != bd && ad != 1 && bd != 1) fail(VC_ERR_INVALID, "binary_backward: operand shapes do not broadcast");
        src[i] = std::max(ad, bd);
    }
    const std::size_t n = checked_numel(src, rank);
    if (!g) fail(VC_ERR_INVALID, "binary_backward: null gradient");
    if (n == 0) {
        if (da) VC_CUDA(cudaMemsetAsync(da, 0, checked_numel(a_shape, a_rank) * sizeof(float), stream()));
        if (db) VC_CUDA(cudaMemsetAsync(db, 0, checked_numel(b_shape, b_rank) * sizeof(float), stream()));
        return VC_OK;
    }
    const Src sg = align(g, g_shape, g_rank, src, rank, "binary_backward");
    const Src sa = align(a, a_shape, a_rank, src, rank, "binary_backward");
    const Src sb = align(b, b_shape, b_rank, src, rank, "binary_backward");
    auto same = [&](const size_t* s, int r) {
        if (r != rank) return false;
        for (int i = 0; i < r; ++i) if (s[i] != src[i]) return false;
        return true;
    };
    if (da && db && same(a_shape, a_rank) && same(b_shape, b_rank) && same(g_shape, g_rank)) {
        const bool vec = aligned16(a) && aligned16(b) && aligned16(g) && aligned16(da) && aligned16(db);
        static_assert(kThreads == kStreamThreads, "binary_backward_flat launches stream_grid CTAs");
        const unsigned grid = vec ? stream_grid(n) : grid_for(n, kThreads);
#define VC_BB(OP) do { if (vec) binary_backward_flat<OP, true><<<grid, kThreads, 0, stream()>>>(a, b, g, da, db, n); \
                       else binary_backward_flat<OP, false><<<grid, kThreads, 0, stream()>>>(a, b, g, da, db, n); } while (0)
        switch (op) {
            case VC_ADD: VC_BB(VC_ADD); break;
            case VC_SUB: VC_BB(VC_SUB); break;
            case VC_MUL: VC_BB(VC_MUL); break;
            default: VC_BB(VC_DIV); break;
        }
#undef VC_BB
        check_launch("binary_backward_flat");
        return VC_OK;
    }
    if (da && db && try_fused_bcast_backward(op, a, sa, b, sb, g, sg, src, rank, da, db, nullptr, nullptr,
                                             checked_numel(b_shape, b_rank)))
        return VC_OK;
    // The two gradients are independent reductions: with both wanted, db's
    // runs on the side stream while da's runs on the main one, so their
    // small latency-bound launches (compact sums, finishes) hide under each
    // other's streams -- e.g. sum()'s scalar upstream on a [P,1,R,L] x
    // [1,Q,1,L] product writes da and reads a at the same time.
    const int fa = (op == VC_ADD || op == VC_SUB) ? V_G : (op == VC_MUL ? V_MUL : V_DIV_A);
    const int fb = op == VC_ADD ? V_G : (op == VC_SUB ? V_NEG : (op == VC_MUL ? V_MUL : V_DIV_B));
    Src ops_a[3] = {sg, sb, sb};
    Src ops_b[3] = {sg, sa, sb};
    if (da && db) {
        SideStream side;
        vjp_reduce(fb, ops_b, src, rank, b_shape, b_rank, db);
        side.leave();
        vjp_reduce(fa, ops_a, src, rank, a_shape, a_rank, da);
        side.join();
        return VC_OK;
    }
    if (da) vjp_reduce(fa, ops_a, src, rank, a_shape, a_rank, da);
    if (db) vjp_reduce(fb, ops_b, src, rank, b_shape, b_rank, db);
    VC_API_END
}

vc_status vc_cuda_reduce_all(int op, const float* in, size_t count, float* out_value, int64_t* out_index) {
    VC_API_BEGIN
    ensure_init();
    if (!in && count) fail(VC_ERR_INVALID, "reduce_all: null input");
    if (op == VC_REDUCE_SUM || op == VC_REDUCE_MEAN) {
        if (!out_value) fail(VC_ERR_INVALID, "reduce_all: null output");
        if (count == 0) {
            if (op == VC_REDUCE_MEAN) fail(VC_ERR_INVALID, "mean of an empty tensor is undefined");
            VC_CUDA(cudaMemsetAsync(out_value, 0, sizeof(float), stream()));
            return VC_OK;
        }
        Src ops[3];
        const size_t shape[1] = {count};
        ops[0] = align(in, shape, 1, shape, 1, "reduce_all");
        vjp_reduce(V_G, ops, shape, 1, nullptr, 0, out_value,
                   op == VC_REDUCE_MEAN ? static_cast<float>(count) : 0.0f);
        return VC_OK;
    }
    if (op != VC_REDUCE_MAX && op != VC_REDUCE_ARGMAX) fail(VC_ERR_INVALID, "unknown reduction");
    if (count == 0) fail(VC_ERR_INVALID, "max of an empty tensor is undefined");
    MaxOut o{out_value, reinterpret_cast<long long*>(out_index), op == VC_REDUCE_ARGMAX, 0, 0};
    launch_max(in, 1, count, 1, o);
    VC_API_END
}

vc_status vc_cuda_reduce_axis(int op, const float* in, size_t outer, size_t length, size_t inner,
                              float* out_value, int64_t* out_index) {
    VC_API_BEGIN
    ensure_init();
    const size_t dims[3] = {outer, length, inner};
    checked_numel(dims, 3);
    if (op == VC_REDUCE_SUM || op == VC_REDUCE_MEAN) {
        if (op == VC_REDUCE_MEAN && length == 0) fail(VC_ERR_INVALID, "mean over an empty axis is undefined");
        if (outer * inner == 0) return VC_OK;
        if (!out_value) fail(VC_ERR_INVALID, "reduce_axis: null output");
        if (length == 0) {
            VC_CUDA(cudaMemsetAsync(out_value, 0, outer * inner * sizeof(float), stream()));
            return VC_OK;
        }
        Src ops[3];
        const size_t target[3] = {outer, 1, inner};
        ops[0] = align(in, dims, 3, dims, 3, "reduce_axis");
        vjp_reduce(V_G, ops, dims, 3, target, 3, out_value,
                   op == VC_REDUCE_MEAN ? static_cast<float>(length) : 0.0f);
        return VC_OK;
    }
    if (op != VC_REDUCE_MAX && op != VC_REDUCE_ARGMAX) fail(VC_ERR_INVALID, "unknown reduction");
    if (length == 0) fail(VC_ERR_INVALID, "max/argmax over an empty axis is undefined");
    MaxOut o{out_value, reinterpret_cast<long long*>(out_index), op == VC_REDUCE_ARGMAX, 0, 0};
    launch_max(in, outer, length, inner, o);
    VC_API_END
}

vc_status vc_cuda_scatter_axis(const float* values, const float* indices_f32, const int64_t* indices_i64,
                               float* out, size_t outer, size_t length, size_t inner) {
    VC_API_BEGIN
    ensure_init();
    if ((indices_f32 == nullptr) == (indices_i64 == nullptr))
        fail(VC_ERR_INVALID, "scatter_axis: pass exactly one of the float or int64 indices");
    launch_axis_expand(2, values, reinterpret_cast<const long long*>(indices_i64), indices_f32, out, outer, length, inner);
    VC_API_END
}

vc_status vc_cuda_reduce_axis_backward(int op, const float* g, const int64_t* indices, float* out,
                                       size_t outer, size_t length, size_t inner) {
    VC_API_BEGIN
    ensure_init();
    int mode;
    switch (op) {
        case VC_REDUCE_SUM: mode = 0; break;
        case VC_REDUCE_MEAN: mode = 1; break;
        case VC_REDUCE_MAX:
            if (!indices) fail(VC_ERR_INVALID, "reduce_axis_backward: max needs the argmax indices");
            mode = 2;
            break;
        default: fail(VC_ERR_INVALID, "reduce_axis_backward: operation has no backward rule");
    }
    launch_axis_expand(mode, g, reinterpret_cast<const long long*>(indices), nullptr, out, outer, length, inner);
    VC_API_END
}

}  // extern "C"

// ---- multi-GPU: shard partials and their rank-order combine ------------------

extern "C" {

vc_status vc_cuda_reduce_axis_partial(int op, const float* in, size_t outer, size_t length, size_t inner,
                                      int64_t index_base, int continuation, double* partial_sum,
                                      float* partial_value, int64_t* partial_index) {
    VC_API_BEGIN
    ensure_init();
    const size_t dims[3] = {outer, length, inner};
    checked_numel(dims, 3);
    const std::size_t count = outer * inner;
    if (!count) return VC_OK;
    if (op == VC_REDUCE_SUM || op == VC_REDUCE_MEAN) {
        if (!partial_sum) fail(VC_ERR_INVALID, "reduce_axis_partial: null partial_sum");
        if (length == 0) {
            VC_CUDA(cudaMemsetAsync(partial_sum, 0, count * sizeof(double), stream()));
            return VC_OK;
        }
        Src ops[3];
        const size_t target[3] = {outer, 1, inner};
        ops[0] = align(in, dims, 3, dims, 3, "reduce_axis_partial");
        vjp_reduce(V_G, ops, dims, 3, target, 3, nullptr, 0.0f, partial_sum);
        return VC_OK;
    }
    if (op != VC_REDUCE_MAX && op != VC_REDUCE_ARGMAX) fail(VC_ERR_INVALID, "unknown reduction");
    if (!partial_value || !partial_index) fail(VC_ERR_INVALID, "reduce_axis_partial: null partial_value/index");
    if (length == 0) {
        if (!continuation) fail(VC_ERR_INVALID, "max/argmax over an empty axis is undefined");
        // an empty later shard has no candidate: value 0, index -1
        VC_CUDA(cudaMemsetAsync(partial_value, 0, count * sizeof(float), stream()));
        VC_CUDA(cudaMemsetAsync(partial_index, 0xff, count * sizeof(int64_t), stream()));
        return VC_OK;
    }
    MaxOut o{partial_value, reinterpret_cast<long long*>(partial_index), 0, continuation ? 1 : 0,
             static_cast<long long>(index_base)};
    launch_max(in, outer, length, inner, o);
    VC_API_END
}

vc_status vc_cuda_binary_backward_partial(int op, const float* a, const size_t* a_shape, int a_rank,
                                          const float* b, const size_t* b_shape, int b_rank,
                                          const float* g, const size_t* g_shape, int g_rank,
                                          double* da_partial, double* db_partial) {
    VC_API_BEGIN
    ensure_init();
    validate_rank(a_rank, "binary_backward_partial");
    validate_rank(b_rank, "binary_backward_partial");
    validate_rank(g_rank, "binary_backward_partial");
    if (op < VC_ADD || op > VC_DIV) fail(VC_ERR_INVALID, "unknown binary operation");
    const int rank = std::max(a_rank, b_rank);
    size_t src[kMaxRank];
    for (int i = 0; i < rank; ++i) {
        const size_t ad = i < rank - a_rank ? 1 : a_shape[i - (rank - a_rank)];
        const size_t bd = i < rank - b_rank ? 1 : b_shape[i - (rank - b_rank)];
        if (ad != bd && ad != 1 && bd != 1) fail(VC_ERR_INVALID, "binary_backward_partial: shapes do not broadcast");
        src[i] = std::max(ad, bd);
    }
    if (!g) fail(VC_ERR_INVALID, "binary_backward_partial: null gradient");
    if (checked_numel(src, rank) == 0) {
        if (da_partial) VC_CUDA(cudaMemsetAsync(da_partial, 0, checked_numel(a_shape, a_rank) * sizeof(double), stream()));
        if (db_partial) VC_CUDA(cudaMemsetAsync(db_partial, 0, checked_numel(b_shape, b_rank) * sizeof(double), stream()));
        return VC_OK;
    }
    const Src sg = align(g, g_shape, g_rank, src, rank, "binary_backward_partial");
    const Src sa = align(a, a_shape, a_rank, src, rank, "binary_backward_partial");
    const Src sb = align(b, b_shape, b_rank, src, rank, "binary_backward_partial");
    if (da_partial && db_partial &&
        try_fused_bcast_backward(op, a, sa, b, sb, g, sg, src, rank, nullptr, nullptr, da_partial, db_partial,
                                 checked_numel(b_shape, b_rank)))
        return VC_OK;
    if (da_partial) {
        Src ops[3] = {sg, sb, sb};
        const int f = (op == VC_ADD || op == VC_SUB) ? V_G : (op == VC_MUL ? V_MUL : V_DIV_A);
        vjp_reduce(f, ops, src, rank, a_shape, a_rank, nullptr, 0.0f, da_partial);
    }
    if (db_partial) {
        Src ops[3] = {sg, sa, sb};
        const int f = op == VC_ADD ? V_G : (op == VC_SUB ? V_NEG : (op == VC_MUL ? V_MUL : V_DIV_B));
        vjp_reduce(f, ops, src, rank, b_shape, b_rank, nullptr, 0.0f, db_partial);
    }
    VC_API_END
}

vc_status vc_cuda_combine_partials(int op, const double* partial_sum, const float* partial_value,
                                   const int64_t* partial_index, int nranks, size_t count, float divisor,
                                   int negate, float* out_value, int64_t* out_index) {
    VC_API_BEGIN
    ensure_init();
    if (nranks <= 0) fail(VC_ERR_INVALID, "combine_partials: nranks must be positive");
    if (!count) return VC_OK;
    const unsigned grid = grid_for(count, kThreads);
    if (op == VC_REDUCE_SUM || op == VC_REDUCE_MEAN) {
        if (!partial_sum || !out_value) fail(VC_ERR_INVALID, "combine_partials: null pointer");
        combine_sum_kernel<<<grid, kThreads, 0, stream()>>>(partial_sum, nranks, count, divisor, negate, out_value);
    } else if (op == VC_REDUCE_MAX || op == VC_REDUCE_ARGMAX) {
        if (!partial_value || !partial_index) fail(VC_ERR_INVALID, "combine_partials: null pointer");
        combine_max_kernel<<<grid, kThreads, 0, stream()>>>(partial_value, reinterpret_cast<const long long*>(partial_index),
                                                           nranks, count, op == VC_REDUCE_ARGMAX, out_value,
                                                           reinterpret_cast<long long*>(out_index));
    } else {
        fail(VC_ERR_INVALID, "unknown reduction");
    }
    check_launch("combine_partials");
    VC_API_END
}

}  // extern "C"
