// ref_shim.cpp -- C entry points into the reference's own CPU code.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles this file together with
// the reference's unmodified sources (src/*.cpp, src/cpu/*.cpp and the Metal
// stub, read in place from the reference checkout) into oracle/_ref/libvcref.so.
// Tests use it to pin the C restatement (vc_oracle.c) and the CUDA device
// against the real reference; bench.py's reference leg times it. The shim
// itself only marshals raw buffers into the reference's public C++ API
// (include/vectorcore/*.hpp) -- all arithmetic is the reference's.
#include "vectorcore/vectorcore.hpp"
#include "vectorcore/cpu_backend.hpp"
#include "vectorcore/detail/tensor_impl.hpp"
#include "parallel.hpp"

#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

using namespace vectorcore;

namespace {

std::string g_error;

Shape to_shape(const size_t* shape, int rank) { return Shape(shape, shape + rank); }

std::vector<float> to_values(const float* data, const Shape& shape) {
    const auto n = numel(shape);
    return std::vector<float>(data, data + n);
}

void copy_out(const Tensor& t, float* out) {
    const auto v = t.to_vector();
    if (!v.empty()) std::memcpy(out, v.data(), v.size() * sizeof(float));
}

template <typename F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return -1;
    }
}

Tensor apply_binary(int op, const Tensor& a, const Tensor& b) {
    switch (op) {
        case 0: return a + b;
        case 1: return a - b;
        case 2: return a * b;
        default: return a / b;
    }
}

Tensor apply_unary(int op, const Tensor& x) {
    switch (op) {
        case 0: return -x;
        case 1: return x.relu();
        case 2: return x.sigmoid();
        case 4: return x.exp();
        default: return x.log();
    }
}

} // namespace

extern "C" {

const char* vcref_last_error(void) { return g_error.c_str(); }

size_t vcref_threads(void) { return cpu::parallel_threads(); }

// cpu::binary (src/cpu/cpu_backend.cpp:275-289) on contiguous operands.
int vcref_binary(int op, const float* a, const size_t* a_shape, int a_rank,
                 const float* b, const size_t* b_shape, int b_rank,
                 float* out, const size_t* out_shape, int out_rank) {
    return guarded([&] {
        const auto as = to_shape(a_shape, a_rank), bs = to_shape(b_shape, b_rank);
        cpu::binary(a, as, contiguous_strides(as), b, bs, contiguous_strides(bs), out,
                    to_shape(out_shape, out_rank), static_cast<cpu::BinaryOp>(op));
    });
}

int vcref_unary(int op, const float* in, float* out, size_t n) {
    return guarded([&] { cpu::unary(in, out, n, static_cast<cpu::UnaryOp>(op)); });
}

float vcref_sum(const float* in, size_t n) { return cpu::sum(in, n); }

int vcref_reduce_axis(int op, const float* in, float* out, size_t outer, size_t length,
                      size_t inner) {
    return guarded([&] {
        cpu::reduce_axis(in, out, outer, length, inner, static_cast<cpu::ReduceOp>(op));
    });
}

void vcref_scatter_axis(const float* values, const float* indices, float* out, size_t outer,
                        size_t length, size_t inner) {
    cpu::scatter_axis(values, indices, out, outer, length, inner);
}

// detail::sum_to_shape (src/autograd.cpp:50-72).
int vcref_sum_to_shape(const float* g, const size_t* g_shape, int g_rank, float* out,
                       const size_t* t_shape, int t_rank) {
    return guarded([&] {
        const auto gs = to_shape(g_shape, g_rank);
        Tensor gt(to_values(g, gs), gs);
        copy_out(detail::sum_to_shape(gt, to_shape(t_shape, t_rank)), out);
    });
}

// Forward + backward of a binary op through the reference's autograd.
int vcref_binary_backward(int op, const float* a, const size_t* a_shape, int a_rank,
                          const float* b, const size_t* b_shape, int b_rank, const float* g,
                          float* out, float* da, float* db) {
    return guarded([&] {
        const auto as = to_shape(a_shape, a_rank), bs = to_shape(b_shape, b_rank);
        Tensor ta(to_values(a, as), as, da != nullptr);
        Tensor tb(to_values(b, bs), bs, db != nullptr);
        auto y = apply_binary(op, ta, tb);
        if (out) copy_out(y, out);
        if (!da && !db) return;
        y.backward(Tensor(to_values(g, y.shape()), y.shape()));
        if (da) copy_out(ta.grad(), da);
        if (db) copy_out(tb.grad(), db);
    });
}

int vcref_unary_backward(int op, const float* x, size_t n, const float* g, float* y,
                         float* dx) {
    return guarded([&] {
        Tensor tx(std::vector<float>(x, x + n), {n}, true);
        auto out = apply_unary(op, tx);
        if (y) copy_out(out, y);
        out.backward(Tensor(std::vector<float>(g, g + n), {n}));
        copy_out(tx.grad(), dx);
    });
}

// kind: 0 sum, 1 mean, 2 max, 3 argmax; full != 0 reduces every element.
int vcref_reduce_op(int kind, const float* x, const size_t* shape, int rank, int full,
                    long axis, float* out, const float* g, float* dx) {
    return guarded([&] {
        const auto s = to_shape(shape, rank);
        Tensor t(to_values(x, s), s, dx != nullptr && kind != 3);
        Tensor y;
        switch (kind) {
            case 0: y = full ? t.sum() : t.sum(axis, false); break;
            case 1: y = full ? t.mean() : t.mean(axis, false); break;
            case 2: y = full ? t.max() : t.max(axis, false); break;
            default: y = full ? t.flatten().argmax(0, false) : t.argmax(axis, false); break;
        }
        copy_out(y, out);
        if (dx && kind != 3) {
            y.backward(Tensor(to_values(g, y.shape()), y.shape()));
            copy_out(t.grad(), dx);
        }
    });
}

// kind 0: log_softmax, 1: softmax, along `axis`; g/dx optional.
int vcref_softmax_op(int kind, const float* x, const size_t* shape, int rank, long axis,
                     float* out, const float* g, float* dx) {
    return guarded([&] {
        const auto s = to_shape(shape, rank);
        Tensor t(to_values(x, s), s, dx != nullptr);
        auto y = kind == 0 ? t.log_softmax(axis) : t.softmax(axis);
        copy_out(y, out);
        if (dx) {
            y.backward(Tensor(to_values(g, s), s));
            copy_out(t.grad(), dx);
        }
    });
}

// nn::cross_entropy (src/nn.cpp:31-53), forward and optional backward.
int vcref_cross_entropy(const float* logits, size_t batch, size_t classes,
                        const int64_t* targets, float upstream, float* loss, float* dx) {
    return guarded([&] {
        Tensor t(std::vector<float>(logits, logits + batch * classes), {batch, classes},
                 dx != nullptr);
        std::vector<std::size_t> tg(batch);
        for (size_t r = 0; r < batch; ++r) tg[r] = static_cast<std::size_t>(targets[r]);
        auto y = nn::cross_entropy(t, tg);
        *loss = y.item();
        if (dx) {
            y.backward(Tensor({upstream}, {}));
            copy_out(t.grad(), dx);
        }
    });
}

} // extern "C"
