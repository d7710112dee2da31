/*
 * vc_oracle.c -- CPU restatement of VectorCore's float32 hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see vc_oracle.h): the checker for the CUDA
 * device, never linked into the product. Parity of this restatement with the
 * reference is pinned by tests/test_oracle.py against the reference's own
 * code built from its sources (oracle/_ref) and against tests/golden/.
 *
 * Build: gcc -O2 -ffp-contract=off (no fused multiply-add, like the
 * reference's x86-64 build), linked against glibc's libm for expf/logf.
 */
#include "vc_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static char g_error[256];

const char* vco_last_error(void) { return g_error; }

static int fail(const char* message) {
    snprintf(g_error, sizeof g_error, "%s", message);
    return -1;
}

static size_t numel(const size_t* shape, int rank) {
    size_t total = 1;
    for (int i = 0; i < rank; ++i) total *= shape[i];
    return total;
}

/* src/shape.cpp:34-47 */
int vco_broadcast_shape(const size_t* a, int a_rank, const size_t* b, int b_rank,
                        size_t* out, int* out_rank) {
    const int rank = a_rank > b_rank ? a_rank : b_rank;
    for (int i = 0; i < rank; ++i) {
        const size_t ai = i < rank - a_rank ? 1 : a[i - (rank - a_rank)];
        const size_t bi = i < rank - b_rank ? 1 : b[i - (rank - b_rank)];
        if (ai != bi && ai != 1 && bi != 1) return fail("cannot broadcast shapes");
        out[i] = ai > bi ? ai : bi;
    }
    *out_rank = rank;
    return 0;
}

static float apply_binary(int op, float x, float y) {
    switch (op) {
        case VCO_ADD: return x + y;   /* cpu_backend.cpp:24 */
        case VCO_SUB: return x - y;   /* :25 */
        case VCO_MUL: return x * y;   /* :26 */
        default: return x / y;        /* :27 */
    }
}

/* Offset of the element of a right-aligned, broadcast operand that feeds the
 * output element with multi-index `coord` (cpu_backend.cpp:76-87). */
static size_t broadcast_offset(const size_t* coord, int out_rank,
                               const size_t* shape, int rank) {
    size_t offset = 0, stride = 1;
    for (int axis = rank - 1; axis >= 0; --axis) {
        const int oaxis = axis + (out_rank - rank);
        if (shape[axis] != 1) offset += coord[oaxis] * stride;
        stride *= shape[axis];
    }
    return offset;
}

/* src/cpu/cpu_backend.cpp:29-106. Every fast path there computes
 * out[i] = Op(a[off_a(i)], b[off_b(i)]); this restates that per element. */
int vco_binary(int op, const float* a, const size_t* a_shape, int a_rank,
               const float* b, const size_t* b_shape, int b_rank,
               float* out, const size_t* out_shape, int out_rank) {
    size_t coord[16];
    if (out_rank > 16) return fail("rank too large for the oracle");
    const size_t count = numel(out_shape, out_rank);
    for (size_t i = 0; i < count; ++i) {
        size_t rem = i;
        for (int axis = out_rank - 1; axis >= 0; --axis) {
            coord[axis] = rem % out_shape[axis];
            rem /= out_shape[axis];
        }
        const size_t oa = broadcast_offset(coord, out_rank, a_shape, a_rank);
        const size_t ob = broadcast_offset(coord, out_rank, b_shape, b_rank);
        out[i] = apply_binary(op, a[oa], b[ob]);
    }
    return 0;
}

/* src/cpu/cpu_backend.cpp:291-316 */
static float apply_unary(int op, float x) {
    switch (op) {
        case VCO_NEG: return -x;
        case VCO_RELU: return x > 0.0f ? x : 0.0f;
        case VCO_RELU_GRAD: return x > 0.0f ? 1.0f : 0.0f;
        case VCO_SIGMOID:
            if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
            {
                const float e = expf(x);
                return e / (1.0f + e);
            }
        case VCO_EXP: return expf(x);
        default: return logf(x);
    }
}

void vco_unary(int op, const float* in, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = apply_unary(op, in[i]);
}

/* src/cpu/cpu_backend.cpp:392-418 */
float vco_sum(const float* in, size_t n) {
    const size_t chunk = (size_t)1 << 16;
    double total = 0.0;
    for (size_t begin = 0; begin < n; begin += chunk) {
        const size_t end = begin + chunk < n ? begin + chunk : n;
        double acc[4] = {0.0, 0.0, 0.0, 0.0};
        size_t i = begin;
        for (; i + 4 <= end; i += 4) {
            acc[0] += in[i];
            acc[1] += in[i + 1];
            acc[2] += in[i + 2];
            acc[3] += in[i + 3];
        }
        double part = acc[0] + acc[1] + acc[2] + acc[3];
        for (; i < end; ++i) part += in[i];
        total += part;
    }
    return (float)total;
}

/* src/cpu/cpu_backend.cpp:420-460 */
int vco_reduce_axis(int op, const float* in, float* out, int64_t* idx64,
                    size_t outer, size_t length, size_t inner) {
    if (length == 0 && op != VCO_SUM) return fail("max/argmax over an empty axis is undefined");
    for (size_t o = 0; o < outer; ++o) {
        const float* base = in + o * length * inner;
        for (size_t i = 0; i < inner; ++i) {
            if (op == VCO_SUM) {
                double total = 0.0;
                for (size_t a = 0; a < length; ++a) total += base[a * inner + i];
                out[o * inner + i] = (float)total;
                continue;
            }
            float best = base[i];
            size_t best_index = 0;
            for (size_t a = 1; a < length; ++a) {
                const float v = base[a * inner + i];
                if (v > best) {
                    best = v;
                    best_index = a;
                }
            }
            out[o * inner + i] = op == VCO_MAX ? best : (float)best_index;
            if (idx64) idx64[o * inner + i] = (int64_t)best_index;
        }
    }
    return 0;
}

/* src/cpu/cpu_backend.cpp:462-471 */
void vco_scatter_axis(const float* values, const float* indices, float* out,
                      size_t outer, size_t length, size_t inner) {
    memset(out, 0, outer * length * inner * sizeof(float));
    for (size_t o = 0; o < outer; ++o) {
        for (size_t i = 0; i < inner; ++i) {
            const size_t a = (size_t)indices[o * inner + i];
            out[(o * length + a) * inner + i] = values[o * inner + i];
        }
    }
}

/* src/autograd.cpp:50-72 */
int vco_sum_to_shape(const float* g, const size_t* g_shape, int g_rank,
                     float* out, const size_t* t_shape, int t_rank) {
    if (t_rank > g_rank) return fail("cannot reduce to larger rank");
    const int lead = g_rank - t_rank;
    size_t cur_shape[16];
    if (g_rank > 16) return fail("rank too large for the oracle");
    memcpy(cur_shape, g_shape, sizeof(size_t) * (size_t)g_rank);
    const size_t total = numel(g_shape, g_rank);
    float* current = (float*)malloc((total ? total : 1) * sizeof(float));
    float* next = (float*)malloc((total ? total : 1) * sizeof(float));
    memcpy(current, g, total * sizeof(float));
    for (int axis = 0; axis < g_rank; ++axis) {
        const size_t target_dim = axis < lead ? 1 : t_shape[axis - lead];
        if (target_dim == g_shape[axis]) continue;
        if (target_dim != 1) {
            free(current);
            free(next);
            return fail("cannot reduce gradient to target shape");
        }
        size_t outer = 1, inner = 1;
        for (int k = 0; k < axis; ++k) outer *= cur_shape[k];
        for (int k = axis + 1; k < g_rank; ++k) inner *= cur_shape[k];
        vco_reduce_axis(VCO_SUM, current, next, NULL, outer, cur_shape[axis], inner);
        cur_shape[axis] = 1;
        float* swap = current;
        current = next;
        next = swap;
    }
    memcpy(out, current, numel(t_shape, t_rank) * sizeof(float));
    free(current);
    free(next);
    return 0;
}

/* src/autograd.cpp:74-91 */
int vco_broadcast_to(const float* v, const size_t* v_shape, int v_rank,
                     float* out, const size_t* t_shape, int t_rank) {
    const float zero = 0.0f;
    return vco_binary(VCO_ADD, v, v_shape, v_rank, &zero, NULL, 0, out, t_shape, t_rank);
}

/* src/ops.cpp:98-156: the gradient of each operand is the upstream combined
 * with the other operand (broadcast to the output shape), then reduced with
 * sum_to_shape. */
int vco_binary_backward(int op, const float* a, const size_t* a_shape, int a_rank,
                        const float* b, const size_t* b_shape, int b_rank,
                        const float* g, float* da, float* db) {
    size_t o_shape[16];
    int o_rank = 0;
    if (vco_broadcast_shape(a_shape, a_rank, b_shape, b_rank, o_shape, &o_rank)) return -1;
    const size_t n = numel(o_shape, o_rank);
    float* t = (float*)malloc((n ? n : 1) * sizeof(float));
    float* u = (float*)malloc((n ? n : 1) * sizeof(float));
    int rc = 0;
    if (da) {
        switch (op) {
            case VCO_ADD:
            case VCO_SUB: memcpy(t, g, n * sizeof(float)); break;
            case VCO_MUL: vco_binary(VCO_MUL, g, o_shape, o_rank, b, b_shape, b_rank, t, o_shape, o_rank); break;
            default: vco_binary(VCO_DIV, g, o_shape, o_rank, b, b_shape, b_rank, t, o_shape, o_rank); break;
        }
        rc |= vco_sum_to_shape(t, o_shape, o_rank, da, a_shape, a_rank);
    }
    if (db) {
        switch (op) {
            case VCO_ADD: memcpy(t, g, n * sizeof(float)); break;
            case VCO_SUB: vco_unary(VCO_NEG, g, t, n); break;
            case VCO_MUL: vco_binary(VCO_MUL, g, o_shape, o_rank, a, a_shape, a_rank, t, o_shape, o_rank); break;
            default: {
                /* -(g * a) / (b * b) */
                const size_t nb = numel(b_shape, b_rank);
                float* bb = (float*)malloc((nb ? nb : 1) * sizeof(float));
                vco_binary(VCO_MUL, b, b_shape, b_rank, b, b_shape, b_rank, bb, b_shape, b_rank);
                vco_binary(VCO_MUL, g, o_shape, o_rank, a, a_shape, a_rank, u, o_shape, o_rank);
                vco_unary(VCO_NEG, u, u, n);
                vco_binary(VCO_DIV, u, o_shape, o_rank, bb, b_shape, b_rank, t, o_shape, o_rank);
                free(bb);
                break;
            }
        }
        rc |= vco_sum_to_shape(t, o_shape, o_rank, db, b_shape, b_rank);
    }
    free(t);
    free(u);
    return rc ? -1 : 0;
}

/* src/ops.cpp:158-164 (negate), :360-367 (exp: g*y), :369-376 (log: g/x),
 * :395-403 (relu: g*relugrad(x)), :405-413 (sigmoid: (g*y)*(1-y)). */
void vco_unary_backward(int op, const float* x, const float* y, const float* g,
                        float* dx, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        switch (op) {
            case VCO_NEG: dx[i] = -g[i]; break;
            case VCO_EXP: dx[i] = g[i] * y[i]; break;
            case VCO_LOG: dx[i] = g[i] / x[i]; break;
            case VCO_RELU: dx[i] = g[i] * (x[i] > 0.0f ? 1.0f : 0.0f); break;
            case VCO_SIGMOID: {
                const float gy = g[i] * y[i];
                const float one_minus = 1.0f - y[i];
                dx[i] = gy * one_minus;
                break;
            }
            default: dx[i] = g[i]; break;
        }
    }
}

/* src/ops.cpp:378-384: shifted = x - max(x.detach()); out = shifted -
 * log(sum(exp(shifted))) with the sum double-accumulated along the axis. */
void vco_log_softmax(const float* x, float* out, float* row_max, float* row_sum,
                     size_t outer, size_t length, size_t inner) {
    for (size_t o = 0; o < outer; ++o) {
        for (size_t i = 0; i < inner; ++i) {
            const float* base = x + o * length * inner + i;
            float m = base[0];
            for (size_t a = 1; a < length; ++a)
                if (base[a * inner] > m) m = base[a * inner];
            double total = 0.0;
            for (size_t a = 0; a < length; ++a) total += expf(base[a * inner] - m);
            const float s = (float)total;
            const float l = logf(s);
            for (size_t a = 0; a < length; ++a)
                out[o * length * inner + a * inner + i] = (base[a * inner] - m) - l;
            if (row_max) row_max[o * inner + i] = m;
            if (row_sum) row_sum[o * inner + i] = s;
        }
    }
}

/* src/ops.cpp:386-388: softmax = exp(log_softmax). */
void vco_softmax(const float* x, float* out, size_t outer, size_t length, size_t inner) {
    vco_log_softmax(x, out, NULL, NULL, outer, length, inner);
    vco_unary(VCO_EXP, out, out, outer * length * inner);
}

/* Backward of the log_softmax chain with upstream G, in the engine's
 * order (src/tensor.cpp:266-300): shifted first receives G (from
 * `shifted - l`), then G + (de * e) where dl = sum(-G), ds = dl / s and
 * de = broadcast_to(ds) = ds + 0. `gls` is the upstream of log_softmax. */
static void log_softmax_chain_backward(const float* x, const float* gls, float* dx,
                                       size_t outer, size_t length, size_t inner) {
    for (size_t o = 0; o < outer; ++o) {
        for (size_t i = 0; i < inner; ++i) {
            const float* base = x + o * length * inner + i;
            const float* gb = gls + o * length * inner + i;
            float m = base[0];
            for (size_t a = 1; a < length; ++a)
                if (base[a * inner] > m) m = base[a * inner];
            double total = 0.0;
            for (size_t a = 0; a < length; ++a) total += expf(base[a * inner] - m);
            const float s = (float)total;
            double neg = 0.0;
            for (size_t a = 0; a < length; ++a) neg += -gb[a * inner];
            const float dl = (float)neg;
            const float ds = dl / s;
            const float de = ds + 0.0f;
            for (size_t a = 0; a < length; ++a) {
                const float e = expf(base[a * inner] - m);
                dx[o * length * inner + a * inner + i] = gb[a * inner] + de * e;
            }
        }
    }
}

void vco_log_softmax_backward(const float* x, const float* g, float* dx,
                              size_t outer, size_t length, size_t inner) {
    log_softmax_chain_backward(x, g, dx, outer, length, inner);
}

/* softmax = exp(ls): the upstream of ls is G * y (y = saved softmax). */
void vco_softmax_backward(const float* x, const float* g, float* dx,
                          size_t outer, size_t length, size_t inner) {
    const size_t n = outer * length * inner;
    float* y = (float*)malloc((n ? n : 1) * sizeof(float));
    float* gy = (float*)malloc((n ? n : 1) * sizeof(float));
    vco_softmax(x, y, outer, length, inner);
    for (size_t k = 0; k < n; ++k) gy[k] = g[k] * y[k];
    log_softmax_chain_backward(x, gy, dx, outer, length, inner);
    free(y);
    free(gy);
}

/* src/nn.cpp:31-53: loss = -(log_softmax(x, 1) * one_hot).sum() / B.
 * Backward with upstream u: dn = u / B, dt = -dn, dp = broadcast(dt) =
 * dt + 0, dls = dp * mask, then the log_softmax chain with upstream dls. */
int vco_cross_entropy(const float* logits, size_t batch, size_t classes,
                      const int64_t* targets, float upstream, float* loss, float* dx) {
    if (batch == 0) return fail("cross_entropy of an empty batch is undefined");
    for (size_t r = 0; r < batch; ++r)
        if (targets[r] < 0 || (size_t)targets[r] >= classes) return fail("target class out of range");
    const size_t n = batch * classes;
    float* ls = (float*)malloc((n ? n : 1) * sizeof(float));
    float* p = (float*)malloc((n ? n : 1) * sizeof(float));
    vco_log_softmax(logits, ls, NULL, NULL, batch, classes, 1);
    for (size_t r = 0; r < batch; ++r)
        for (size_t c = 0; c < classes; ++c)
            p[r * classes + c] = ls[r * classes + c] * ((size_t)targets[r] == c ? 1.0f : 0.0f);
    const float t = vco_sum(p, n);
    const float neg = -t;
    *loss = neg / (float)batch;
    if (dx) {
        const float dn = upstream / (float)batch;
        const float dt = -dn;
        const float dp = dt + 0.0f;
        for (size_t r = 0; r < batch; ++r)
            for (size_t c = 0; c < classes; ++c)
                p[r * classes + c] = dp * ((size_t)targets[r] == c ? 1.0f : 0.0f);
        log_softmax_chain_backward(logits, p, dx, batch, classes, 1);
    }
    free(ls);
    free(p);
    return 0;
}

int vco_reduce_op(int kind, const float* x, const size_t* shape, int rank, int full,
                  long axis, float* out, const float* g, float* dx) {
    const size_t n = numel(shape, rank);
    size_t outer = 1, length = n, inner = 1;
    if (!full) {
        if (rank == 0) return fail("cannot reduce a scalar along an axis");
        if (axis < -rank || axis >= rank) return fail("axis out of range");
        const int ax = (int)(axis < 0 ? axis + rank : axis);
        outer = 1;
        inner = 1;
        for (int k = 0; k < ax; ++k) outer *= shape[k];
        for (int k = ax + 1; k < rank; ++k) inner *= shape[k];
        length = shape[ax];
    }
    const size_t m = outer * inner;
    if (kind == 0 || kind == 1) {
        /* full: cpu::sum (ops.cpp:288-302); axis: reduce_axis (ops.cpp:304-315) */
        if (kind == 1 && length == 0) return fail("mean over an empty axis is undefined");
        if (full) out[0] = vco_sum(x, n);
        else vco_reduce_axis(VCO_SUM, x, out, NULL, outer, length, inner);
        if (kind == 1) for (size_t k = 0; k < m; ++k) out[k] = out[k] / (float)length;
        if (dx) {
            /* mean: divide backward g / len, then broadcast_to (+ 0) */
            for (size_t o = 0; o < outer; ++o)
                for (size_t a = 0; a < length; ++a)
                    for (size_t i = 0; i < inner; ++i) {
                        float gv = g[o * inner + i];
                        if (kind == 1) gv = gv / (float)length;
                        dx[(o * length + a) * inner + i] = gv + 0.0f;
                    }
        }
        return 0;
    }
    /* max (ops.cpp:323-352): max value, then argmax + scatter for backward */
    if (length == 0) return fail("max of an empty axis is undefined");
    vco_reduce_axis(VCO_MAX, x, out, NULL, outer, length, inner);
    if (dx) {
        float* idx = (float*)malloc((m ? m : 1) * sizeof(float));
        vco_reduce_axis(VCO_ARGMAX, x, idx, NULL, outer, length, inner);
        vco_scatter_axis(g, idx, dx, outer, length, inner);
        free(idx);
    }
    return 0;
}
