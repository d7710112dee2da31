// elementwise.cu -- broadcast binary ops, unary ops, their fused backward
// rules, broadcast_to, fill and axpy for sm_100a.
//
// Every kernel here is HBM-bandwidth-bound (<= 1 flop per 4 bytes moved), so
// the design is about bytes in flight and instruction count per byte:
//  * flat paths (same shape, scalar operand) and their backward rules:
//    chunked streams -- one short-lived CTA per 16 KiB of each operand, four
//    float4 per thread, every load issued before the first store (the
//    stream_grid layout in vc_internal.cuh);
//  * every other broadcast layout: dimensions are collapsed on the host and
//    the innermost run of L elements is a "row" (what the reference's CPU
//    kernel resolves per row, src/cpu/cpu_backend.cpp:59-105). Long float4
//    rows (L >= 128) take one warp per row, offsets decoded with FastDiv in
//    registers; other layouts resolve the operand offsets of a tile of rows
//    once into shared memory and then stream the tile. Offsets are 64-bit:
//    config 5 has 2^32 outputs.
// Arithmetic is the reference's (src/cpu/cpu_backend.cpp:24-27, 291-316),
// compiled with -fmad=false and IEEE division so add/sub/mul/div/neg/relu
// are bit-identical to the CPU path; exp and sigmoid's exponential use
// exp_acc (a table-driven float exponential, ~0.52 ulp, below) and log uses
// CUDA's logf, all within 2 ulp of glibc's expf / logf.
#include "vc_internal.cuh"

#include <algorithm>
#include <vector>

namespace vc {

// ---------------------------------------------------------------------------
// Scalar arithmetic, exactly as the reference writes it.
// ---------------------------------------------------------------------------
template <int OP>
__device__ __forceinline__ float bop(float x, float y) {
    if constexpr (OP == VC_ADD) return x + y;
    else if constexpr (OP == VC_SUB) return x - y;
    else if constexpr (OP == VC_MUL) return x * y;
    else return x / y;
}

// exp rounded once from double precision: CUDA's double exp is within 1 ulp
// of a double, so the rounding to float is correct except within about 2^-29
// of a rounding boundary. Only for the inputs exp_acc leaves aside; kept out
// of line so the unrolled stream loops carry one call, not sixteen copies.
__device__ __noinline__ float exp_rn(float x) { return static_cast<float>(exp(static_cast<double>(x))); }

// Why exp_acc: glibc's float exp (the reference's std::exp on float) is
// within 0.502 ulp of the true value and CUDA's expf within 2 ulp, so the two
// can land 3 floats apart; a 16 M-sample sweep found sigmoid inputs 3 ulp from
// the reference, outside the 2-ulp class. Double exp closes the gap but costs
// 25-40% of the stream's speed; exp_acc stays within ~0.52 ulp of the true
// value (at most one float from glibc's) at close to expf's cost. log keeps
// CUDA's logf: the same sweep found it within 1 ulp of glibc's logf.

// Rounding to an integer by adding 1.5 * 2^23 (exact for |v| < 2^22): the
// float and integer forms of rint(v) come from FMA-pipe adds and an integer
// subtract instead of conversion instructions, which issue at a quarter of
// the rate on the SM.
constexpr float kRoundMagic = 0x1.8p+23f;
constexpr int kRoundMagicBits = 0x4b400000;

// e^x, Tang's table-driven method (ACM TOMS 15(2), 1989) with a 32-entry
// table. n = 32 m + j = rint(x * 32 / ln 2), r = x - n * ln2/32 from a
// two-part ln2/32 (the first product exact inside an FMA), |r| <= ln2/64;
// e^x = 2^m * 2^(j/32) * e^r with 2^(j/32) = T_hi + T_lo (float pair) and
// e^r - 1 = r + r^2 (1/2 + r/6 + r^2/24) (truncation 2^-39). Every term but
// T_hi is below 0.022 in magnitude, so their rounding errors stay near 0.01
// ulp of the result and the last addition T_hi + s rounds once: ~0.52 ulp.
// |x| > 86 (results near or below FLT_MIN, overflow), infinities and NaN
// take exp_rn. Table: 2^(j/32) rounded to float and the remainder, computed
// to 60 digits; constants 32 / ln 2, ln2/32 rounded to float and its
// remainder.
__device__ const float2 kExp2Frac[32] = {
    {0x1p+0f, 0x0p+0f},                       {0x1.059b0ep+0f, -0x1.9d4f52p-25f},
    {0x1.0b5586p+0f, 0x1.9f3122p-25f},        {0x1.11301ep+0f, -0x1.fdb496p-25f},
    {0x1.172b84p+0f, -0x1.c15742p-27f},       {0x1.1d4874p+0f, -0x1.d2e8cap-25f},
    {0x1.2387a6p+0f, 0x1.ceac48p-25f},        {0x1.29e9e0p+0f, -0x1.5c0424p-25f},
    {0x1.306fe0p+0f, 0x1.4636e2p-25f},        {0x1.371a74p+0f, -0x1.18aac6p-25f},
    {0x1.3dea64p+0f, 0x1.824684p-25f},        {0x1.44e086p+0f, 0x1.8624b4p-30f},
    {0x1.4bfdaep+0f, -0x1.593abcp-25f},       {0x1.5342b6p+0f, -0x1.2c5610p-25f},
    {0x1.5ab07ep+0f, -0x1.5bd5ecp-27f},       {0x1.6247ecp+0f, -0x1.f8b550p-25f},
    {0x1.6a09e6p+0f, 0x1.9fcef4p-26f},        {0x1.71f75ep+0f, 0x1.1d8beep-25f},
    {0x1.7a1148p+0f, -0x1.829fd0p-25f},       {0x1.82589ap+0f, -0x1.accc7cp-26f},
    {0x1.8ace54p+0f, 0x1.15506ep-27f},        {0x1.93737cp+0f, -0x1.e64744p-25f},
    {0x1.9c4918p+0f, 0x1.51f848p-27f},        {0x1.a5503cp+0f, -0x1.b83b54p-25f},
    {0x1.ae89fap+0f, -0x1.a94b14p-26f},       {0x1.b7f770p+0f, -0x1.a09438p-25f},
    {0x1.c199bep+0f, -0x1.3d56b2p-27f},       {0x1.cb720ep+0f, -0x1.8837ccp-27f},
    {0x1.d5818ep+0f, -0x1.822dbcp-27f},       {0x1.dfc974p+0f, -0x1.908c94p-25f},
    {0x1.ea4afap+0f, 0x1.52486cp-27f},        {0x1.f50766p+0f, -0x1.246eb0p-26f},
};
constexpr float kInvLn2x32 = 0x1.715476p+5f;
constexpr float kLn2d32Hi = 0x1.62e430p-6f;
constexpr float kLn2d32Lo = -0x1.05c610p-34f;

__device__ __forceinline__ float exp_acc(float x) {
    if (!(fabsf(x) <= 86.0f)) return exp_rn(x);
    const float tm = fmaf(x, kInvLn2x32, kRoundMagic);  // |x * 32 / ln 2| < 2^12
    const int n = __float_as_int(tm) - kRoundMagicBits;
    const float nf = tm - kRoundMagic;
    const float r1 = fmaf(-nf, kLn2d32Hi, x);
    const float r2 = -nf * kLn2d32Lo;
    const float poly = fmaf(r1, fmaf(r1, 1.0f / 24.0f, 1.0f / 6.0f), 0.5f);
    const float q = fmaf(r1 * r1, poly, r2);
    const float2 t = __ldg(&kExp2Frac[n & 31]);
    float s = fmaf(t.x, q, t.y);
    s = fmaf(t.x, r1, s);
    const float y = t.x + s;
    return __int_as_float(__float_as_int(y) + ((n >> 5) << 23));
}

// num / d for 1 <= d <= 2 and 0 <= num <= 1 (no overflow; only num may be
// subnormal): Markstein's division -- an approximate reciprocal refined by one
// Newton-Raphson step, the quotient corrected once with its exact FMA
// remainder (P. W. Markstein, "Computation of elementary functions on the IBM
// RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990). A few FMAs where
// the general IEEE division also handles the ranges this operand pair never
// reaches; the sweeps check the sigmoid stays within 2 ulp of the reference's.
__device__ __forceinline__ float div_unit_interval(float num, float d) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d));
    y = fmaf(fmaf(-d, y, 1.0f), y, y);
    const float q = num * y;
    return fmaf(fmaf(-d, q, num), y, q);
}

template <int OP>
__device__ __forceinline__ float uop(float x) {
    if constexpr (OP == VC_NEG) return -x;
    else if constexpr (OP == VC_RELU) return x > 0.0f ? x : 0.0f;
    else if constexpr (OP == VC_RELU_GRAD) return x > 0.0f ? 1.0f : 0.0f;
    else if constexpr (OP == VC_SIGMOID) {
        // cpu_backend.cpp:302-307 computes 1/(1+exp(-x)) for x >= 0 and
        // e/(1+e) with e = exp(x) otherwise. Both branches evaluate
        // exp(-|x|), so selecting the numerator gives the same value with one
        // exponential and one division and no warp divergence (NaN takes the
        // second form, as in the reference). 1 + e lies in [1, 2].
        const float e = exp_acc(-fabsf(x));
        const float num = x >= 0.0f ? 1.0f : e;
        return div_unit_interval(num, 1.0f + e);
    } else if constexpr (OP == VC_EXP) return exp_acc(x);
    else return logf(x);
}

// Backward rules of src/ops.cpp (negate :158-164, exp :360-367, log
// :369-376, relu :395-403, sigmoid :405-413), each one fused pass.
template <int OP>
__device__ __forceinline__ float ubwd(float x, float y, float g) {
    if constexpr (OP == VC_NEG) return -g;
    else if constexpr (OP == VC_EXP) return g * y;
    else if constexpr (OP == VC_LOG) return g / x;
    else if constexpr (OP == VC_RELU) return g * (x > 0.0f ? 1.0f : 0.0f);
    else {  // VC_SIGMOID: gradient * y * (1.0F - y), left to right
        const float gy = g * y;
        const float one_minus = 1.0f - y;
        return gy * one_minus;
    }
}

template <int OP>
__device__ __forceinline__ float4 bop4(float4 x, float4 y) {
    return make_float4(bop<OP>(x.x, y.x), bop<OP>(x.y, y.y), bop<OP>(x.z, y.z), bop<OP>(x.w, y.w));
}

constexpr unsigned kThreads = 256;
static_assert(kThreads == kStreamThreads, "the flat kernels launch stream_grid CTAs of kStreamThreads");

// ---------------------------------------------------------------------------
// Flat binary: MODE 0 same shape, 1 scalar rhs, 2 scalar lhs. The scalar is
// *sp when sp is not null (a one-element device tensor) else sv.
// VEC: all pointers 16-byte aligned.
// ---------------------------------------------------------------------------
template <int OP, int MODE, bool VEC>
__global__ void __launch_bounds__(kThreads)
binary_flat_kernel(const float* __restrict__ a, const float* __restrict__ b,
                   float* __restrict__ out, std::size_t n, const float* __restrict__ sp, float sv) {
    const float s = sp ? __ldg(sp) : sv;
    if constexpr (VEC) {  // chunked stream (stream_grid)
        const std::size_t n4 = n >> 2;
        const float4 s4 = make_float4(s, s, s, s);
        const std::size_t base = static_cast<std::size_t>(blockIdx.x) * kChunk4 + threadIdx.x;
        float4 x[kStreamRounds], y[kStreamRounds];
#pragma unroll
        for (unsigned u = 0; u < kStreamRounds; ++u) {
            const std::size_t k = base + u * kStreamThreads;
            if (k < n4) {
                x[u] = MODE == 2 ? s4 : ldg4(a + 4 * k);
                y[u] = MODE == 1 ? s4 : ldg4(b + 4 * k);
            }
        }
#pragma unroll
        for (unsigned u = 0; u < kStreamRounds; ++u) {
            const std::size_t k = base + u * kStreamThreads;
            if (k < n4) st4(out + 4 * k, bop4<OP>(x[u], y[u]));
        }
        if (blockIdx.x == gridDim.x - 1)
            for (std::size_t k = n4 * 4 + threadIdx.x; k < n; k += kStreamThreads)
                out[k] = bop<OP>(MODE == 2 ? s : a[k], MODE == 1 ? s : b[k]);
    } else {
        const std::size_t tid = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
        const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
        for (std::size_t k = tid; k < n; k += stride)
            out[k] = bop<OP>(MODE == 2 ? s : a[k], MODE == 1 ? s : b[k]);
    }
}

// ---------------------------------------------------------------------------
// Tiled strided broadcast. The collapsed output is [rows, L]; operand X's
// element (row, col) is X[off_X(row) + col * inner_X] where off_X(row)
// decodes `row` over the leading collapsed dims. A CTA handles TR rows per
// tile: thread t < TR resolves row t's offsets into shared memory, then the
// CTA streams the TR*L tile elements.
// ---------------------------------------------------------------------------
constexpr int kTileRowsMax = 256;
constexpr unsigned kTileElems = 4096;   // output elements per tile

// Tile t covers rows [rt * tile_rows, +tile_rows) and, when a row is longer
// than a tile, the column chunk [cc * chunk, +chunk) of a single row
// (t = rt * col_chunks + cc), so long rows spread over many CTAs.
struct BcastDesc {
    int lead_rank;                      // collapsed leading dims (row decode)
    std::size_t lead_dims[kMaxRank];
    long long a_lead[kMaxRank];         // per-dim element strides
    long long b_lead[kMaxRank];
    long long a_inner, b_inner;         // stride along the row (0 or any)
    std::size_t rows, L;
    unsigned tile_rows;                 // > 1 only when L < kTileElems (then col_chunks == 1)
    std::size_t chunk, col_chunks;
    FastDiv div_L;
};

template <int OP, bool VEC>
__global__ void __launch_bounds__(kThreads)
binary_tiled_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ out,
                    const BcastDesc d, float av, float bv) {
    __shared__ long long s_aoff[kTileRowsMax];
    __shared__ long long s_boff[kTileRowsMax];
    // A by-value operand is encoded as a null pointer with all strides 0.
    const std::size_t row_tiles = (d.rows + d.tile_rows - 1) / d.tile_rows;
    const std::size_t tiles = row_tiles * d.col_chunks;
    for (std::size_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const std::size_t rt = tile / d.col_chunks, cc = tile - rt * d.col_chunks;
        const std::size_t row0 = rt * d.tile_rows;
        const std::size_t c0 = cc * d.chunk;
        const unsigned nrows = static_cast<unsigned>(min(static_cast<std::size_t>(d.tile_rows), d.rows - row0));
        const unsigned clen = static_cast<unsigned>(min(d.chunk, d.L - c0));
        if (threadIdx.x < nrows) {
            std::size_t r = row0 + threadIdx.x;
            long long ao = 0, bo = 0;
            for (int k = d.lead_rank - 1; k >= 0; --k) {
                const std::size_t dim = d.lead_dims[k];
                const std::size_t c = r % dim;
                r /= dim;
                ao += static_cast<long long>(c) * d.a_lead[k];
                bo += static_cast<long long>(c) * d.b_lead[k];
            }
            s_aoff[threadIdx.x] = ao + static_cast<long long>(c0) * d.a_inner;
            s_boff[threadIdx.x] = bo + static_cast<long long>(c0) * d.b_inner;
        }
        __syncthreads();
        const unsigned tile_elems = nrows * clen;
        float* tile_out = out + row0 * d.L + c0;
        if constexpr (VEC) {
            for (unsigned e = threadIdx.x * 4; e < tile_elems; e += kThreads * 4) {
                unsigned row = 0, col = e;
                if (nrows > 1) d.div_L.divmod(e, row, col);
                float4 x, y;
                if (!a) x = make_float4(av, av, av, av);
                else if (d.a_inner == 0) { const float v = __ldg(a + s_aoff[row]); x = make_float4(v, v, v, v); }
                else x = ldg4(a + s_aoff[row] + col);
                if (!b) y = make_float4(bv, bv, bv, bv);
                else if (d.b_inner == 0) { const float v = __ldg(b + s_boff[row]); y = make_float4(v, v, v, v); }
                else y = ldg4(b + s_boff[row] + col);
                st4_stream(tile_out + static_cast<std::size_t>(row) * d.L + col, bop4<OP>(x, y));
            }
        } else {
            for (unsigned e = threadIdx.x; e < tile_elems; e += kThreads) {
                unsigned row = 0, col = e;
                if (nrows > 1) d.div_L.divmod(e, row, col);
                const float x = a ? __ldg(a + s_aoff[row] + static_cast<long long>(col) * d.a_inner) : av;
                const float y = b ? __ldg(b + s_boff[row] + static_cast<long long>(col) * d.b_inner) : bv;
                tile_out[static_cast<std::size_t>(row) * d.L + col] = bop<OP>(x, y);
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// Row-broadcast path for long rows (L >= 128, float4-aligned): one warp per
// output row, no shared memory and no block barrier. Each lane decodes the
// row's operand offsets with FastDiv (the same value in every lane, so no
// shuffle is needed) and streams float4 groups with four loads in flight; an
// operand constant along the row (inner stride 0) is read once per row.
// ---------------------------------------------------------------------------
struct RowsDesc {
    int lead_rank;
    FastDiv lead[kMaxRank];             // leading (row) dims, outer first
    long long a_lead[kMaxRank], b_lead[kMaxRank];
    long long a_inner, b_inner;         // 0 or 1
    unsigned rows;                      // < 2^31
    unsigned L4;                        // row length / 4
};

__device__ __forceinline__ float4 rows_fetch(const float* p, float v, long long inner, float per_row, unsigned j) {
    if (!p) return make_float4(v, v, v, v);
    if (inner == 0) return make_float4(per_row, per_row, per_row, per_row);
    return ldg4(p + 4ull * j);
}

template <int OP>
__global__ void __launch_bounds__(kThreads)
binary_rows_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ out,
                   const RowsDesc d, float av, float bv) {
    const unsigned lane = threadIdx.x & 31;
    const unsigned warps = (gridDim.x * blockDim.x) >> 5;
    for (unsigned row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < d.rows; row += warps) {
        unsigned r = row;
        long long ao = 0, bo = 0;
        for (int k = d.lead_rank - 1; k >= 0; --k) {
            unsigned q, c;
            d.lead[k].divmod(r, q, c);
            r = q;
            ao += static_cast<long long>(c) * d.a_lead[k];
            bo += static_cast<long long>(c) * d.b_lead[k];
        }
        const float* ar = a ? a + ao : nullptr;
        const float* br = b ? b + bo : nullptr;
        const float ar0 = ar && d.a_inner == 0 ? __ldg(ar) : 0.0f;
        const float br0 = br && d.b_inner == 0 ? __ldg(br) : 0.0f;
        float* orow = out + static_cast<std::size_t>(row) * d.L4 * 4;
        unsigned j = lane;
        for (; j + 96 < d.L4; j += 128) {
            float4 x[4], y[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                x[u] = rows_fetch(ar, av, d.a_inner, ar0, j + 32 * u);
                y[u] = rows_fetch(br, bv, d.b_inner, br0, j + 32 * u);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) st4_stream(orow + 4ull * (j + 32 * u), bop4<OP>(x[u], y[u]));
        }
        for (; j < d.L4; j += 32)
            st4_stream(orow + 4ull * j, bop4<OP>(rows_fetch(ar, av, d.a_inner, ar0, j),
                                                rows_fetch(br, bv, d.b_inner, br0, j)));
    }
}

// ---------------------------------------------------------------------------
// Row-broadcast path with operand reuse. When one operand X is constant along
// a leading dim k* that the other operand Y spans (a [P,1,R,L] * b [1,Q,1,L]:
// a is constant along Q), a warp keeps a chunk of X's row in registers and
// walks a run of k* positions, loading only Y's row for each output row: one
// load per output float4 instead of two, and X's rows -- the larger operand,
// which the plain row path re-reads from L2 for every output row -- are read
// once per run. Task = (run of k*, column chunk, outer row), outer row
// fastest so neighbouring warps write neighbouring rows. Two rows' loads are
// in flight per iteration and the stores are plain write-back stores (with
// evict-first stores, or one row in flight, the kernel ran 8% slower on
// cfg5's 17 GB output). Same element values as every other path.
// ---------------------------------------------------------------------------
constexpr unsigned kReuseKeep = 4;  // float4 per lane per chunk (512 floats)
constexpr unsigned kReuseRun = 16;  // shortest run of k* positions per task

struct ReuseDesc {
    int outer_rank;                      // leading dims other than k*, outer first
    FastDiv outer[kMaxRank];
    long long x_outer[kMaxRank], y_outer[kMaxRank], o_outer[kMaxRank];
    long long y_step, o_step;            // strides of k* in Y and in the output
    unsigned nq;                         // extent of k*
    unsigned run;                        // k* positions per task
    unsigned runs, chunks;
    unsigned outer_rows;                 // product of the outer dims (< 2^31)
    unsigned long long tasks;
    unsigned L4;
    long long x_inner, y_inner;          // 0 or 1
};

template <int OP, bool X_IS_A>
__global__ void __launch_bounds__(kThreads)
binary_reuse_kernel(const float* __restrict__ xp, const float* __restrict__ yp, float* __restrict__ out,
                    const ReuseDesc d) {
    const unsigned lane = threadIdx.x & 31;
    const unsigned long long warps = (static_cast<unsigned long long>(gridDim.x) * blockDim.x) >> 5;
    for (unsigned long long task = (static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
         task < d.tasks; task += warps) {
        // chunk fastest, then the outer row: a CTA's eight warps cover whole
        // neighbouring rows, so each q step writes one contiguous piece
        const unsigned chunk = static_cast<unsigned>(task % d.chunks);
        const unsigned long long rest = task / d.chunks;
        const unsigned orow = static_cast<unsigned>(rest % d.outer_rows);
        const unsigned run = static_cast<unsigned>(rest / d.outer_rows);
        long long xo = 0, yo = 0, oo = 0;
        unsigned r = orow;
        for (int k = d.outer_rank - 1; k >= 0; --k) {
            unsigned q, c;
            d.outer[k].divmod(r, q, c);
            r = q;
            xo += static_cast<long long>(c) * d.x_outer[k];
            yo += static_cast<long long>(c) * d.y_outer[k];
            oo += static_cast<long long>(c) * d.o_outer[k];
        }
        const unsigned j0 = chunk * 32 * kReuseKeep + lane;
        float4 xv[kReuseKeep];
        const float xs = d.x_inner == 0 ? __ldg(xp + xo) : 0.0f;
#pragma unroll
        for (unsigned u = 0; u < kReuseKeep; ++u) {
            const unsigned j = j0 + 32 * u;
            xv[u] = d.x_inner == 0 ? make_float4(xs, xs, xs, xs)
                                   : (j < d.L4 ? ldg4(xp + xo + 4ll * j) : make_float4(0.f, 0.f, 0.f, 0.f));
        }
        const unsigned q0 = run * d.run, q1 = min(d.nq, q0 + d.run);
        unsigned q = q0;
        for (; q + 1 < q1; q += 2) {
            float4 yv[2][kReuseKeep];
#pragma unroll
            for (unsigned h = 0; h < 2; ++h) {
                const float* yr = yp + yo + static_cast<long long>(q + h) * d.y_step;
                const float ys = d.y_inner == 0 ? __ldg(yr) : 0.0f;
#pragma unroll
                for (unsigned u = 0; u < kReuseKeep; ++u) {
                    const unsigned j = j0 + 32 * u;
                    yv[h][u] = d.y_inner == 0 ? make_float4(ys, ys, ys, ys)
                                           : (j < d.L4 ? ldg4(yr + 4ll * j) : make_float4(0.f, 0.f, 0.f, 0.f));
                }
            }
#pragma unroll
            for (unsigned h = 0; h < 2; ++h) {
                float* orow_p = out + oo + static_cast<long long>(q + h) * d.o_step;
#pragma unroll
                for (unsigned u = 0; u < kReuseKeep; ++u) {
                    const unsigned j = j0 + 32 * u;
                    if (j < d.L4) st4(orow_p + 4ll * j, X_IS_A ? bop4<OP>(xv[u], yv[h][u]) : bop4<OP>(yv[h][u], xv[u]));
                }
            }
        }
        for (; q < q1; ++q) {
            const float* yr = yp + yo + static_cast<long long>(q) * d.y_step;
            float* orow_p = out + oo + static_cast<long long>(q) * d.o_step;
            const float ys = d.y_inner == 0 ? __ldg(yr) : 0.0f;
            float4 yv[kReuseKeep];
#pragma unroll
            for (unsigned u = 0; u < kReuseKeep; ++u) {
                const unsigned j = j0 + 32 * u;
                yv[u] = d.y_inner == 0 ? make_float4(ys, ys, ys, ys)
                                       : (j < d.L4 ? ldg4(yr + 4ll * j) : make_float4(0.f, 0.f, 0.f, 0.f));
            }
#pragma unroll
            for (unsigned u = 0; u < kReuseKeep; ++u) {
                const unsigned j = j0 + 32 * u;
                if (j < d.L4) st4(orow_p + 4ll * j, X_IS_A ? bop4<OP>(xv[u], yv[u]) : bop4<OP>(yv[u], xv[u]));
            }
        }
    }
}

// Both operands constant over the whole output (e.g. the 0-d gradient of a
// sum broadcast back): every element is op(a0, b0).
template <int OP>
__global__ void __launch_bounds__(kThreads)
binary_splat_kernel(const float* __restrict__ ap, float av, const float* __restrict__ bp, float bv,
                    float* __restrict__ out, std::size_t n, bool vec) {
    const float v = bop<OP>(ap ? __ldg(ap) : av, bp ? __ldg(bp) : bv);
    if (vec) {  // chunked stream (stream_grid): a write-only stream, 7.3 TB/s chunked vs 6.2 grid-stride
        const std::size_t n4 = n >> 2;
        const float4 v4 = make_float4(v, v, v, v);
        const std::size_t base = static_cast<std::size_t>(blockIdx.x) * kChunk4 + threadIdx.x;
#pragma unroll
        for (unsigned u = 0; u < kStreamRounds; ++u) {
            const std::size_t k = base + u * kStreamThreads;
            if (k < n4) st4(out + 4 * k, v4);
        }
        if (blockIdx.x == gridDim.x - 1)
            for (std::size_t k = n4 * 4 + threadIdx.x; k < n; k += kStreamThreads) out[k] = v;
        return;
    }
    const std::size_t tid = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
    for (std::size_t k = tid; k < n; k += stride) out[k] = v;
}

// ---------------------------------------------------------------------------
// Unary and unary-backward flat kernels.
// ---------------------------------------------------------------------------
template <int OP, bool VEC>
__global__ void __launch_bounds__(kThreads)
unary_kernel(const float* __restrict__ in, float* __restrict__ out, std::size_t n) {
    if constexpr (VEC) {  // chunked stream (stream_grid)
        const std::size_t n4 = n >> 2;
        const std::size_t base = static_cast<std::size_t>(blockIdx.x) * kChunk4 + threadIdx.x;
        float4 x[kStreamRounds];
#pragma unroll
        for (unsigned u = 0; u < kStreamRounds; ++u) {
            const std::size_t k = base + u * kStreamThreads;
            if (k < n4) x[u] = ldg4(in + 4 * k);
        }
#pragma unroll
        for (unsigned u = 0; u < kStreamRounds; ++u) {
            const std::size_t k = base + u * kStreamThreads;
            if (k < n4) st4(out + 4 * k, make_float4(uop<OP>(x[u].x), uop<OP>(x[u].y), uop<OP>(x[u].z), uop<OP>(x[u].w)));
        }
        if (blockIdx.x == gridDim.x - 1)
            for (std::size_t k = n4 * 4 + threadIdx.x; k < n; k += kStreamThreads) out[k] = uop<OP>(in[k]);
    } else {
        const std::size_t tid = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
        const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
        for (std::size_t k = tid; k < n; k += stride) out[k] = uop<OP>(in[k]);
    }
}

// Reads only the operands the rule needs (NEED_X / NEED_Y).
template <int OP, bool VEC>
__global__ void __launch_bounds__(kThreads)
unary_backward_kernel(const float* __restrict__ x, const float* __restrict__ y,
                      const float* __restrict__ g, float* __restrict__ dx, std::size_t n) {
    constexpr bool NEED_X = OP == VC_LOG || OP == VC_RELU;
    constexpr bool NEED_Y = OP == VC_EXP || OP == VC_SIGMOID;
    if constexpr (VEC) {  // chunked stream (stream_grid)
        const std::size_t n4 = n >> 2;
        const std::size_t base = static_cast<std::size_t>(blockIdx.x) * kChunk4 + threadIdx.x;
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        float4 gx[kStreamRounds], xx[kStreamRounds], yy[kStreamRounds];
#pragma unroll
        for (unsigned u = 0; u < kStreamRounds; ++u) {
            const std::size_t k = base + u * kStreamThreads;
            if (k < n4) {
                gx[u] = ldg4(g + 4 * k);
                xx[u] = NEED_X ? ldg4(x + 4 * k) : z;
                yy[u] = NEED_Y ? ldg4(y + 4 * k) : z;
            }
        }
#pragma unroll
        for (unsigned u = 0; u < kStreamRounds; ++u) {
            const std::size_t k = base + u * kStreamThreads;
            if (k < n4)
                st4(dx + 4 * k, make_float4(ubwd<OP>(xx[u].x, yy[u].x, gx[u].x), ubwd<OP>(xx[u].y, yy[u].y, gx[u].y),
                                            ubwd<OP>(xx[u].z, yy[u].z, gx[u].z), ubwd<OP>(xx[u].w, yy[u].w, gx[u].w)));
        }
        if (blockIdx.x == gridDim.x - 1)
            for (std::size_t k = n4 * 4 + threadIdx.x; k < n; k += kStreamThreads)
                dx[k] = ubwd<OP>(NEED_X ? x[k] : 0.f, NEED_Y ? y[k] : 0.f, g[k]);
    } else {
        const std::size_t tid = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
        const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
        for (std::size_t k = tid; k < n; k += stride)
            dx[k] = ubwd<OP>(NEED_X ? x[k] : 0.f, NEED_Y ? y[k] : 0.f, g[k]);
    }
}

__global__ void __launch_bounds__(kThreads)
fill_kernel(float* __restrict__ out, std::size_t n, float value) {
    const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
    for (std::size_t k = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n; k += stride)
        out[k] = value;
}

__global__ void __launch_bounds__(kThreads)
axpy_kernel(float* __restrict__ t, const float* __restrict__ s, std::size_t n, float alpha) {
    const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
    for (std::size_t k = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n; k += stride)
        t[k] = t[k] + alpha * s[k];
}

// ---------------------------------------------------------------------------
// Host side: canonicalise a broadcast and pick a path.
// ---------------------------------------------------------------------------
struct Operand {
    const float* ptr{nullptr};  // null: by-value constant
    float value{0.0f};
    long long strides[kMaxRank]{};  // aligned to the output dims; 0 = broadcast
};

// Align an operand of `shape` (contiguous, or with `strides`) to the output.
static Operand align_operand(const float* ptr, const size_t* shape, const size_t* strides, int rank,
                             const size_t* out_shape, int out_rank, const char* what) {
    Operand op;
    op.ptr = ptr;
    if (rank > out_rank) fail(VC_ERR_INVALID, std::string(what) + ": operand rank exceeds the output rank");
    std::size_t contiguous = 1;
    for (int i = rank - 1; i >= 0; --i) {
        const int o = i + (out_rank - rank);
        const std::size_t dim = shape[i];
        if (dim != out_shape[o] && dim != 1)
            fail(VC_ERR_INVALID, std::string(what) + ": cannot broadcast operand to the output shape");
        const std::size_t st = strides ? strides[i] : contiguous;
        op.strides[o] = dim == 1 ? 0 : static_cast<long long>(st);
        contiguous *= dim;
    }
    return op;
}

struct Canon {
    int rank{0};
    std::size_t dims[kMaxRank]{};
    long long sa[kMaxRank]{};
    long long sb[kMaxRank]{};
};

// Drop size-1 output dims and merge neighbours that are contiguous for both
// operands (or broadcast in both).
static Canon canonicalise(const size_t* out_shape, int out_rank, const Operand& a, const Operand& b) {
    Canon c;
    for (int i = 0; i < out_rank; ++i) {
        if (out_shape[i] == 1) continue;
        c.dims[c.rank] = out_shape[i];
        c.sa[c.rank] = a.strides[i];
        c.sb[c.rank] = b.strides[i];
        ++c.rank;
    }
    Canon m;
    for (int i = 0; i < c.rank; ++i) {
        if (m.rank > 0) {
            const int j = m.rank - 1;
            const long long d = static_cast<long long>(c.dims[i]);
            if (m.sa[j] == c.sa[i] * d && m.sb[j] == c.sb[i] * d) {
                m.dims[j] *= c.dims[i];
                m.sa[j] = c.sa[i];
                m.sb[j] = c.sb[i];
                continue;
            }
        }
        m.dims[m.rank] = c.dims[i];
        m.sa[m.rank] = c.sa[i];
        m.sb[m.rank] = c.sb[i];
        ++m.rank;
    }
    return m;
}

// Pick the leading dim k* for binary_reuse_kernel: one operand constant
// along it (stride 0), the other spanning it, at least kReuseRun long; among
// those, keep the operand with the larger footprint in registers. Returns
// false (nothing launched) when no dim qualifies.
template <int OP>
static bool try_launch_reuse(const float* a, const float* b, float* out, const BcastDesc& d) {
    const int R = d.lead_rank;
    if (R < 1 || d.L / 4 > 0xffffffffull) return false;
    std::size_t foot_a = d.a_inner ? d.L : 1, foot_b = d.b_inner ? d.L : 1;
    for (int i = 0; i < R; ++i) {
        if (d.a_lead[i]) foot_a *= d.lead_dims[i];
        if (d.b_lead[i]) foot_b *= d.lead_dims[i];
    }
    int best = -1;
    bool best_x_is_a = false;
    std::size_t best_foot = 0, best_size = 0;
    for (int i = 0; i < R; ++i) {
        const std::size_t size = d.lead_dims[i];
        if (size < kReuseRun) continue;
        const bool a_const = d.a_lead[i] == 0 && d.b_lead[i] != 0;
        const bool b_const = d.b_lead[i] == 0 && d.a_lead[i] != 0;
        if (!a_const && !b_const) continue;
        const std::size_t foot = a_const ? foot_a : foot_b;
        if (foot > best_foot || (foot == best_foot && size > best_size)) {
            best = i;
            best_x_is_a = a_const;
            best_foot = foot;
            best_size = size;
        }
    }
    if (best < 0) return false;
    ReuseDesc rd{};
    std::size_t o_stride[kMaxRank];
    std::size_t acc = d.L;
    for (int i = R - 1; i >= 0; --i) {
        o_stride[i] = acc;
        acc *= d.lead_dims[i];
    }
    unsigned long long outer_rows = 1;
    for (int i = 0; i < R; ++i) {
        if (i == best) continue;
        const int k = rd.outer_rank++;
        rd.outer[k] = FastDiv(static_cast<unsigned>(d.lead_dims[i]));
        rd.x_outer[k] = best_x_is_a ? d.a_lead[i] : d.b_lead[i];
        rd.y_outer[k] = best_x_is_a ? d.b_lead[i] : d.a_lead[i];
        rd.o_outer[k] = static_cast<long long>(o_stride[i]);
        outer_rows *= d.lead_dims[i];
    }
    if (outer_rows >= (1ull << 31)) return false;
    rd.outer_rows = static_cast<unsigned>(outer_rows);
    rd.nq = static_cast<unsigned>(d.lead_dims[best]);
    rd.y_step = best_x_is_a ? d.b_lead[best] : d.a_lead[best];
    rd.o_step = static_cast<long long>(o_stride[best]);
    rd.L4 = static_cast<unsigned>(d.L / 4);
    rd.chunks = (rd.L4 + 32 * kReuseKeep - 1) / (32 * kReuseKeep);
    // The longest run that still leaves four waves of warps: X's row chunk is
    // then read once for the whole run instead of once per 16 positions (the
    // other runs of a row come round long after it left L2: configuration 5
    // read a eight times from HBM with runs of 16). Every output element is
    // computed alone, so the split does not change a single value.
    const unsigned long long want = 4ull * static_cast<unsigned long long>(sm_count()) * (2048 / 32);
    const unsigned long long per_run = static_cast<unsigned long long>(rd.outer_rows) * rd.chunks;
    rd.run = rd.nq;
    while (rd.run > kReuseRun && per_run * ((rd.nq + rd.run - 1) / rd.run) < want) rd.run = (rd.run + 1) / 2;
    if (rd.run < kReuseRun) rd.run = std::min<unsigned>(kReuseRun, rd.nq);
    rd.runs = (rd.nq + rd.run - 1) / rd.run;
    rd.tasks = per_run * rd.runs;
    rd.x_inner = best_x_is_a ? d.a_inner : d.b_inner;
    rd.y_inner = best_x_is_a ? d.b_inner : d.a_inner;
    const std::size_t warps_per_cta = kThreads / 32;
    // one task per warp (no persistent loop): short-lived CTAs on contiguous
    // output pieces stream better (cfg5 forward 92% -> 96%)
    const unsigned grid = static_cast<unsigned>(std::min<std::size_t>((rd.tasks + warps_per_cta - 1) / warps_per_cta,
                                                                      0x7fffffffull));
    if (best_x_is_a) binary_reuse_kernel<OP, true><<<grid, kThreads, 0, stream()>>>(a, b, out, rd);
    else binary_reuse_kernel<OP, false><<<grid, kThreads, 0, stream()>>>(b, a, out, rd);
    check_launch("binary_reuse");
    return true;
}

template <int OP>
static void launch_binary_op(const Operand& a, const Operand& b, float* out, const Canon& c, std::size_t n) {
    cudaStream_t s = stream();
    const bool a_flat = c.rank <= 1 && (c.rank == 0 || c.sa[0] == 1);
    const bool b_flat = c.rank <= 1 && (c.rank == 0 || c.sb[0] == 1);
    const bool a_scalar = c.rank == 0 || (c.rank == 1 && c.sa[0] == 0);
    const bool b_scalar = c.rank == 0 || (c.rank == 1 && c.sb[0] == 0);
    int mode = -1;
    if (a.ptr && b.ptr && a_flat && b_flat) mode = 0;
    else if (a.ptr && a_flat && b_scalar) mode = 1;
    else if (b.ptr && b_flat && a_scalar) mode = 2;
    if (mode >= 0) {
        const bool vec = aligned16(out) && (mode == 2 || aligned16(a.ptr)) && (mode == 1 || aligned16(b.ptr));
        const unsigned grid = vec ? stream_grid(n) : grid_for(n, kThreads);
        const float* sp = mode == 1 ? b.ptr : (mode == 2 ? a.ptr : nullptr);
        const float sv = mode == 1 ? b.value : a.value;
#define VC_FLAT(M, V) binary_flat_kernel<OP, M, V><<<grid, kThreads, 0, s>>>(a.ptr, b.ptr, out, n, sp, sv)
        if (mode == 0) { if (vec) VC_FLAT(0, true); else VC_FLAT(0, false); }
        else if (mode == 1) { if (vec) VC_FLAT(1, true); else VC_FLAT(1, false); }
        else { if (vec) VC_FLAT(2, true); else VC_FLAT(2, false); }
#undef VC_FLAT
        check_launch("binary_flat");
        return;
    }
    // Both operands constant everywhere: splat.
    bool all_zero = true;
    for (int i = 0; i < c.rank; ++i) all_zero = all_zero && c.sa[i] == 0 && c.sb[i] == 0;
    if (all_zero) {
        const bool vec = aligned16(out);
        binary_splat_kernel<OP><<<vec ? stream_grid(n) : grid_for(n, kThreads), kThreads, 0, s>>>(
            a.ptr, a.value, b.ptr, b.value, out, n, vec);
        check_launch("binary_splat");
        return;
    }
    // Tiled strided path.
    BcastDesc d{};
    const int r = c.rank;  // >= 1 here
    d.L = c.dims[r - 1];
    d.a_inner = c.sa[r - 1];
    d.b_inner = c.sb[r - 1];
    d.lead_rank = r - 1;
    d.rows = 1;
    for (int i = 0; i < r - 1; ++i) {
        d.lead_dims[i] = c.dims[i];
        d.a_lead[i] = c.sa[i];
        d.b_lead[i] = c.sb[i];
        d.rows *= c.dims[i];
    }
    if (d.L >= kTileElems) {
        d.tile_rows = 1;
        d.chunk = kTileElems;
        d.col_chunks = (d.L + kTileElems - 1) / kTileElems;
    } else {
        d.tile_rows = static_cast<unsigned>(std::min<std::size_t>({kTileElems / d.L,
                                                                   static_cast<std::size_t>(kTileRowsMax), d.rows}));
        d.chunk = d.L;
        d.col_chunks = 1;
        d.div_L = FastDiv(static_cast<unsigned>(d.L));
    }
    auto lead_ok = [&](const long long* lead, long long inner, const float* p) {
        if (!p || inner == 0) return true;
        if (inner != 1 || !aligned16(p)) return false;
        for (int i = 0; i < d.lead_rank; ++i)
            if (lead[i] % 4) return false;
        return true;
    };
    const bool vec = d.L % 4 == 0 && aligned16(out) && lead_ok(d.a_lead, d.a_inner, a.ptr) &&
                     lead_ok(d.b_lead, d.b_inner, b.ptr);
    bool rows_ok = vec && d.L >= 128 && d.rows < (1ull << 31) && d.L / 4 < (1ull << 31) &&
                   d.rows * (d.L / 4) < (1ull << 62);
    for (int i = 0; i < d.lead_rank; ++i) rows_ok = rows_ok && d.lead_dims[i] < (1ull << 31);
    if (rows_ok && a.ptr && b.ptr && try_launch_reuse<OP>(a.ptr, b.ptr, out, d)) return;
    if (rows_ok) {
        RowsDesc rd{};
        rd.lead_rank = d.lead_rank;
        for (int i = 0; i < d.lead_rank; ++i) {
            rd.lead[i] = FastDiv(static_cast<unsigned>(d.lead_dims[i]));
            rd.a_lead[i] = d.a_lead[i];
            rd.b_lead[i] = d.b_lead[i];
        }
        rd.a_inner = a.ptr ? d.a_inner : 0;
        rd.b_inner = b.ptr ? d.b_inner : 0;
        rd.rows = static_cast<unsigned>(d.rows);
        rd.L4 = static_cast<unsigned>(d.L / 4);
        const std::size_t warps_per_cta = kThreads / 32;
        const std::size_t ctas = (d.rows + warps_per_cta - 1) / warps_per_cta;
        // one CTA per 8 rows, no persistent loop (short-lived CTAs stream better)
        const unsigned grid = static_cast<unsigned>(std::min<std::size_t>(ctas, 0x7fffffffull));
        binary_rows_kernel<OP><<<grid, kThreads, 0, s>>>(a.ptr, b.ptr, out, rd, a.value, b.value);
        check_launch("binary_rows");
        return;
    }
    const std::size_t tiles = (d.rows + d.tile_rows - 1) / d.tile_rows * d.col_chunks;
    const unsigned grid = static_cast<unsigned>(std::min<std::size_t>(tiles, 0x7fffffffull));  // a CTA per tile
    if (vec) binary_tiled_kernel<OP, true><<<grid, kThreads, 0, s>>>(a.ptr, b.ptr, out, d, a.value, b.value);
    else binary_tiled_kernel<OP, false><<<grid, kThreads, 0, s>>>(a.ptr, b.ptr, out, d, a.value, b.value);
    check_launch("binary_tiled");
}

static void launch_binary(int op, const Operand& a, const Operand& b, float* out,
                          const size_t* out_shape, int out_rank) {
    const std::size_t n = checked_numel(out_shape, out_rank);
    if (n == 0) return;
    if (!out) fail(VC_ERR_INVALID, "binary: null output");
    const Canon c = canonicalise(out_shape, out_rank, a, b);
    switch (op) {
        case VC_ADD: return launch_binary_op<VC_ADD>(a, b, out, c, n);
        case VC_SUB: return launch_binary_op<VC_SUB>(a, b, out, c, n);
        case VC_MUL: return launch_binary_op<VC_MUL>(a, b, out, c, n);
        case VC_DIV: return launch_binary_op<VC_DIV>(a, b, out, c, n);
        default: fail(VC_ERR_INVALID, "unknown binary operation");
    }
}

// x + (-0.0f) == x for every float (including -0, +0 and NaN payload class),
// so this is an exact broadcast copy built on the tiled path.
void broadcast_copy(const float* src, const size_t* src_shape, int src_rank, float* out,
                    const size_t* out_shape, int out_rank) {
    const Operand s = align_operand(src, src_shape, nullptr, src_rank, out_shape, out_rank, "broadcast");
    Operand minus_zero;
    minus_zero.value = -0.0f;
    launch_binary(VC_ADD, s, minus_zero, out, out_shape, out_rank);
}

template <int OP>
static void launch_unary_op(const float* in, float* out, std::size_t n) {
    const bool vec = aligned16(in) && aligned16(out);
    const unsigned grid = vec ? stream_grid(n) : grid_for(n, kThreads);
    if (vec) unary_kernel<OP, true><<<grid, kThreads, 0, stream()>>>(in, out, n);
    else unary_kernel<OP, false><<<grid, kThreads, 0, stream()>>>(in, out, n);
    check_launch("unary");
}

template <int OP>
static void launch_unary_backward_op(const float* x, const float* y, const float* g, float* dx, std::size_t n) {
    constexpr bool NEED_X = OP == VC_LOG || OP == VC_RELU;
    constexpr bool NEED_Y = OP == VC_EXP || OP == VC_SIGMOID;
    if ((NEED_X && !x) || (NEED_Y && !y)) fail(VC_ERR_INVALID, "unary_backward: the saved tensor this rule needs is null");
    const bool vec = aligned16(g) && aligned16(dx) && (!NEED_X || aligned16(x)) && (!NEED_Y || aligned16(y));
    const unsigned grid = vec ? stream_grid(n) : grid_for(n, kThreads);
    if (vec) unary_backward_kernel<OP, true><<<grid, kThreads, 0, stream()>>>(x, y, g, dx, n);
    else unary_backward_kernel<OP, false><<<grid, kThreads, 0, stream()>>>(x, y, g, dx, n);
    check_launch("unary_backward");
}

}  // namespace vc

using namespace vc;

extern "C" {

vc_status vc_cuda_binary(int op, const float* a, const size_t* a_shape, const size_t* a_strides, int a_rank,
                         const float* b, const size_t* b_shape, const size_t* b_strides, int b_rank,
                         float* out, const size_t* out_shape, int out_rank) {
    VC_API_BEGIN
    ensure_init();
    validate_rank(a_rank, "binary");
    validate_rank(b_rank, "binary");
    validate_rank(out_rank, "binary");
    if (op < VC_ADD || op > VC_DIV) fail(VC_ERR_INVALID, "unknown binary operation");
    if (checked_numel(out_shape, out_rank) == 0) return VC_OK;
    if (!a || !b) fail(VC_ERR_INVALID, "binary: null operand");
    const Operand oa = align_operand(a, a_shape, a_strides, a_rank, out_shape, out_rank, "binary");
    const Operand ob = align_operand(b, b_shape, b_strides, b_rank, out_shape, out_rank, "binary");
    launch_binary(op, oa, ob, out, out_shape, out_rank);
    VC_API_END
}

vc_status vc_cuda_binary_scalar(int op, const float* a, float scalar, int scalar_first, float* out,
                                size_t count) {
    VC_API_BEGIN
    ensure_init();
    if (op < VC_ADD || op > VC_DIV) fail(VC_ERR_INVALID, "unknown binary operation");
    if (!count) return VC_OK;
    if (!a || !out) fail(VC_ERR_INVALID, "binary_scalar: null pointer");
    Operand t, s;
    t.ptr = a;
    t.strides[0] = 1;
    s.ptr = nullptr;
    s.value = scalar;
    const size_t shape[1] = {count};
    if (scalar_first) launch_binary(op, s, t, out, shape, 1);
    else launch_binary(op, t, s, out, shape, 1);
    VC_API_END
}

vc_status vc_cuda_unary(int op, const float* in, float* out, size_t count) {
    VC_API_BEGIN
    ensure_init();
    if (!count) return VC_OK;
    if (!in || !out) fail(VC_ERR_INVALID, "unary: null pointer");
    switch (op) {
        case VC_NEG: launch_unary_op<VC_NEG>(in, out, count); break;
        case VC_RELU: launch_unary_op<VC_RELU>(in, out, count); break;
        case VC_SIGMOID: launch_unary_op<VC_SIGMOID>(in, out, count); break;
        case VC_RELU_GRAD: launch_unary_op<VC_RELU_GRAD>(in, out, count); break;
        case VC_EXP: launch_unary_op<VC_EXP>(in, out, count); break;
        case VC_LOG: launch_unary_op<VC_LOG>(in, out, count); break;
        default: fail(VC_ERR_INVALID, "unknown unary operation");
    }
    VC_API_END
}

vc_status vc_cuda_unary_backward(int op, const float* x, const float* y, const float* g, float* dx,
                                 size_t count) {
    VC_API_BEGIN
    ensure_init();
    if (!count) return VC_OK;
    if (!g || !dx) fail(VC_ERR_INVALID, "unary_backward: null pointer");
    switch (op) {
        case VC_NEG: launch_unary_backward_op<VC_NEG>(x, y, g, dx, count); break;
        case VC_RELU: launch_unary_backward_op<VC_RELU>(x, y, g, dx, count); break;
        case VC_SIGMOID: launch_unary_backward_op<VC_SIGMOID>(x, y, g, dx, count); break;
        case VC_EXP: launch_unary_backward_op<VC_EXP>(x, y, g, dx, count); break;
        case VC_LOG: launch_unary_backward_op<VC_LOG>(x, y, g, dx, count); break;
        default: fail(VC_ERR_INVALID, "unary_backward: operation has no backward rule");
    }
    VC_API_END
}

vc_status vc_cuda_broadcast_to(const float* value, const size_t* v_shape, int v_rank, float* out,
                               const size_t* t_shape, int t_rank) {
    VC_API_BEGIN
    ensure_init();
    validate_rank(v_rank, "broadcast_to");
    validate_rank(t_rank, "broadcast_to");
    if (checked_numel(t_shape, t_rank) == 0) return VC_OK;
    if (!value) fail(VC_ERR_INVALID, "broadcast_to: null value");
    const Operand ov = align_operand(value, v_shape, nullptr, v_rank, t_shape, t_rank, "broadcast_to");
    Operand zero;  // by-value 0.0f: value + 0 turns -0 into +0 like the reference
    launch_binary(VC_ADD, ov, zero, out, t_shape, t_rank);
    VC_API_END
}

vc_status vc_cuda_fill(float* out, size_t count, float value) {
    VC_API_BEGIN
    ensure_init();
    if (!count) return VC_OK;
    fill_kernel<<<grid_for(count, kThreads), kThreads, 0, stream()>>>(out, count, value);
    check_launch("fill");
    VC_API_END
}

vc_status vc_cuda_axpy(float* target, const float* source, size_t count, float alpha) {
    VC_API_BEGIN
    ensure_init();
    if (!count) return VC_OK;
    if (!target || !source) fail(VC_ERR_INVALID, "axpy: null pointer");
    axpy_kernel<<<grid_for(count, kThreads), kThreads, 0, stream()>>>(target, source, count, alpha);
    check_launch("axpy");
    VC_API_END
}

}  // extern "C"
