// cuda_backend.cpp -- CudaBackend / CudaStorage over the vc_cuda_* C ABI.
#include "cuda_backend.hpp"

#include "vc_cuda.h"

#include <stdexcept>
#include <string>

// The Device value CUDA storages report: Device::cuda() on a host whose
// device.hpp has the CUDA enumerator; the plugin-slot build (metal_slot.cpp)
// serves the reference's existing non-CPU device value instead.
#ifndef VECTORCORE_CUDA_DEVICE
#ifdef VECTORCORE_HAS_CUDA_DEVICE
#define VECTORCORE_CUDA_DEVICE ::vectorcore::Device::cuda()
#else
#define VECTORCORE_CUDA_DEVICE ::vectorcore::Device::metal()
#endif
#endif

namespace vectorcore {

namespace {

// vc_status -> the exception the reference throws for the same condition.
void check(vc_status status, const char* what) {
    if (status == VC_OK) return;
    std::string message = vc_cuda_last_error();
    if (message.empty()) message = what;
    switch (status) {
        case VC_ERR_INVALID: throw std::invalid_argument(message);
        case VC_ERR_OUT_OF_RANGE: throw std::out_of_range(message);
        case VC_ERR_OVERFLOW: throw std::overflow_error(message);
        default: throw std::runtime_error("CUDA device: " + message);
    }
}

const CudaStorage& as_cuda(const Storage& s) {
    const auto* c = dynamic_cast<const CudaStorage*>(&s);
    if (!c) throw std::invalid_argument("storage does not belong to the CUDA device");
    return *c;
}

float* ptr(const Storage& s) { return as_cuda(s).device_data(); }

std::size_t count_of(const Shape& shape) { return numel(shape); }

std::shared_ptr<CudaStorage> make(std::size_t elements, Device device, std::size_t element_bytes = sizeof(float)) {
    return std::make_shared<CudaStorage>(elements, device, element_bytes);
}

}  // namespace

CudaStorage::CudaStorage(std::size_t elements, Device device, std::size_t element_bytes)
    : size_(elements), device_(device) {
    check(vc_cuda_alloc((elements ? elements : 1) * element_bytes, &ptr_), "allocation failed");
}

CudaStorage::~CudaStorage() {
    if (ptr_) vc_cuda_free(ptr_);  // stream-ordered: queued users finish first
}

CudaBackend& CudaBackend::instance() {
    static CudaBackend backend(VECTORCORE_CUDA_DEVICE);
    return backend;
}

CudaBackend::CudaBackend(Device device) : device_(device) {}

bool CudaBackend::available() const noexcept { return vc_cuda_available() != 0; }

std::string CudaBackend::device_name() const {
    char name[256];
    if (vc_cuda_device_name(name, sizeof name) != VC_OK) return "unavailable";
    return name;
}

std::string CudaBackend::last_error() const { return vc_cuda_last_error(); }

std::string CudaBackend::gemm_kernel() const { return available() ? "cuda-tiled-sgemm" : "unavailable"; }

std::shared_ptr<Storage> CudaBackend::allocate(std::size_t elements) { return make(elements, device_); }

std::shared_ptr<Storage> CudaBackend::upload(const float* data, std::size_t elements) {
    auto s = make(elements, device_);
    if (elements) check(vc_cuda_upload(s->raw(), data, elements * sizeof(float)), "upload failed");
    return s;
}

void CudaBackend::download(const Storage& source, float* destination, std::size_t elements) {
    if (elements > source.size()) throw std::out_of_range("CUDA download exceeds storage");
    check(vc_cuda_download(destination, as_cuda(source).raw(), elements * sizeof(float)), "download failed");
}

std::shared_ptr<Storage> CudaBackend::binary(const Storage& a, const Shape& a_shape, const Strides& a_strides,
                                             const Storage& b, const Shape& b_shape, const Strides& b_strides,
                                             const Shape& out_shape, cpu::BinaryOp operation) {
    auto out = make(count_of(out_shape), device_);
    check(vc_cuda_binary(static_cast<int>(operation), ptr(a), a_shape.data(),
                         a_strides.empty() ? nullptr : a_strides.data(), static_cast<int>(a_shape.size()), ptr(b),
                         b_shape.data(), b_strides.empty() ? nullptr : b_strides.data(),
                         static_cast<int>(b_shape.size()), out->device_data(), out_shape.data(),
                         static_cast<int>(out_shape.size())),
          "binary failed");
    return out;
}

std::shared_ptr<Storage> CudaBackend::unary(const Storage& input, std::size_t count, cpu::UnaryOp operation) {
    auto out = make(count, device_);
    check(vc_cuda_unary(static_cast<int>(operation), ptr(input), out->device_data(), count), "unary failed");
    return out;
}

std::shared_ptr<Storage> CudaBackend::matmul(const Storage& a, const Storage& b, std::size_t m, std::size_t k,
                                             std::size_t n, const std::vector<std::size_t>& a_offsets,
                                             const std::vector<std::size_t>& b_offsets, bool trans_a, bool trans_b) {
    if (a_offsets.size() != b_offsets.size() || a_offsets.empty())
        throw std::invalid_argument("CUDA matmul needs one A and B offset per batch");
    auto out = make(a_offsets.size() * m * n, device_);
    check(vc_cuda_matmul(ptr(a), ptr(b), out->device_data(), m, k, n, a_offsets.data(), b_offsets.data(),
                         a_offsets.size(), trans_a, trans_b),
          "matmul failed");
    return out;
}

std::shared_ptr<Storage> CudaBackend::transpose_last2(const Storage& input, std::size_t batch, std::size_t rows,
                                                      std::size_t cols) {
    auto out = make(batch * rows * cols, device_);
    check(vc_cuda_transpose_last2(ptr(input), out->device_data(), batch, rows, cols), "transpose failed");
    return out;
}

std::shared_ptr<Storage> CudaBackend::reduce_sum(const Storage& input, std::size_t count) {
    auto out = make(1, device_);
    check(vc_cuda_reduce_all(VC_REDUCE_SUM, ptr(input), count, out->device_data(), nullptr), "reduce_sum failed");
    return out;
}

std::shared_ptr<Storage> CudaBackend::reduce_axis(const Storage& input, std::size_t outer, std::size_t length,
                                                  std::size_t inner, cpu::ReduceOp operation) {
    auto out = make(outer * inner, device_);
    check(vc_cuda_reduce_axis(static_cast<int>(operation), ptr(input), outer, length, inner, out->device_data(),
                              nullptr),
          "reduce_axis failed");
    return out;
}

std::shared_ptr<Storage> CudaBackend::scatter_axis(const Storage& values, const Storage& indices, std::size_t outer,
                                                   std::size_t length, std::size_t inner) {
    auto out = make(outer * length * inner, device_);
    check(vc_cuda_scatter_axis(ptr(values), ptr(indices), nullptr, out->device_data(), outer, length, inner),
          "scatter_axis failed");
    return out;
}

void CudaBackend::axpy_inplace(Storage& target, const Storage& source, std::size_t count, float alpha) {
    if (count > target.size() || count > source.size()) throw std::out_of_range("CUDA axpy exceeds storage");
    check(vc_cuda_axpy(ptr(target), ptr(source), count, alpha), "axpy failed");
}

void CudaBackend::synchronize() { check(vc_cuda_synchronize(), "synchronize failed"); }

std::shared_ptr<Storage> CudaBackend::broadcast_to(const Storage& value, const Shape& value_shape,
                                                   const Shape& target_shape) {
    auto out = make(count_of(target_shape), device_);
    check(vc_cuda_broadcast_to(ptr(value), value_shape.data(), static_cast<int>(value_shape.size()),
                               out->device_data(), target_shape.data(), static_cast<int>(target_shape.size())),
          "broadcast_to failed");
    return out;
}

CudaBackend::MaxResult CudaBackend::max_with_index(const Storage& input, std::size_t outer, std::size_t length,
                                                   std::size_t inner) {
    MaxResult r{make(outer * inner, device_), make(outer * inner, device_, sizeof(std::int64_t))};
    check(vc_cuda_reduce_axis(VC_REDUCE_MAX, ptr(input), outer, length, inner, ptr(*r.values),
                              static_cast<int64_t*>(as_cuda(*r.indices).raw())),
          "max failed");
    return r;
}

std::shared_ptr<Storage> CudaBackend::max_backward(const Storage& gradient, const Storage& indices, std::size_t outer,
                                                   std::size_t length, std::size_t inner) {
    auto out = make(outer * length * inner, device_);
    check(vc_cuda_reduce_axis_backward(VC_REDUCE_MAX, ptr(gradient),
                                       static_cast<const int64_t*>(as_cuda(indices).raw()), out->device_data(), outer,
                                       length, inner),
          "max backward failed");
    return out;
}

std::shared_ptr<Storage> CudaBackend::sum_to_shape(const Storage& gradient, const Shape& g_shape,
                                                   const Shape& target_shape) {
    auto out = make(count_of(target_shape), device_);
    check(vc_cuda_sum_to_shape(ptr(gradient), g_shape.data(), static_cast<int>(g_shape.size()), out->device_data(),
                               target_shape.data(), static_cast<int>(target_shape.size())),
          "sum_to_shape failed");
    return out;
}

void CudaBackend::binary_backward(cpu::BinaryOp operation, const Storage& a, const Shape& a_shape, const Storage& b,
                                  const Shape& b_shape, const Storage& gradient, const Shape& g_shape,
                                  std::shared_ptr<Storage>* da, std::shared_ptr<Storage>* db) {
    std::shared_ptr<CudaStorage> ga = da ? make(count_of(a_shape), device_) : nullptr;
    std::shared_ptr<CudaStorage> gb = db ? make(count_of(b_shape), device_) : nullptr;
    check(vc_cuda_binary_backward(static_cast<int>(operation), ptr(a), a_shape.data(), static_cast<int>(a_shape.size()),
                                  ptr(b), b_shape.data(), static_cast<int>(b_shape.size()), ptr(gradient),
                                  g_shape.data(), static_cast<int>(g_shape.size()), ga ? ga->device_data() : nullptr,
                                  gb ? gb->device_data() : nullptr),
          "binary_backward failed");
    if (da) *da = ga;
    if (db) *db = gb;
}

std::shared_ptr<Storage> CudaBackend::unary_backward(cpu::UnaryOp operation, const Storage* x, const Storage* y,
                                                     const Storage& gradient, std::size_t count) {
    auto out = make(count, device_);
    check(vc_cuda_unary_backward(static_cast<int>(operation), x ? ptr(*x) : nullptr, y ? ptr(*y) : nullptr,
                                 ptr(gradient), out->device_data(), count),
          "unary_backward failed");
    return out;
}

CudaBackend::SoftmaxResult CudaBackend::softmax(const Storage& x, std::size_t outer, std::size_t length,
                                                std::size_t inner, bool log) {
    SoftmaxResult r{make(outer * length * inner, device_), make(outer * inner, device_), make(outer * inner, device_)};
    auto fn = log ? vc_cuda_log_softmax : vc_cuda_softmax;
    check(fn(ptr(x), ptr(*r.values), ptr(*r.row_max), ptr(*r.row_sum), outer, length, inner), "softmax failed");
    return r;
}

std::shared_ptr<Storage> CudaBackend::softmax_backward(const Storage& x, const Storage& row_max, const Storage& row_sum,
                                                       const Storage& gradient, std::size_t outer, std::size_t length,
                                                       std::size_t inner, bool log) {
    auto out = make(outer * length * inner, device_);
    auto fn = log ? vc_cuda_log_softmax_backward : vc_cuda_softmax_backward;
    check(fn(ptr(x), ptr(row_max), ptr(row_sum), ptr(gradient), out->device_data(), outer, length, inner),
          "softmax_backward failed");
    return out;
}

CudaBackend::CrossEntropyResult CudaBackend::cross_entropy(const Storage& logits, const std::vector<std::size_t>& targets,
                                                           std::size_t batch, std::size_t classes) {
    if (targets.size() != batch)
        throw std::invalid_argument("cross_entropy received " + std::to_string(targets.size()) +
                                    " targets for a batch of " + std::to_string(batch));
    if (batch == 0) throw std::invalid_argument("cross_entropy of an empty batch is undefined");
    std::vector<std::int64_t> t(batch);
    for (std::size_t r = 0; r < batch; ++r) {
        if (targets[r] >= classes)
            throw std::out_of_range("target class " + std::to_string(targets[r]) + " is out of range for " +
                                    std::to_string(classes) + " classes");
        t[r] = static_cast<std::int64_t>(targets[r]);
    }
    CrossEntropyResult r{make(1, device_), make(batch, device_), make(batch, device_),
                         make(batch, device_, sizeof(std::int64_t))};
    check(vc_cuda_upload(as_cuda(*r.targets).raw(), t.data(), batch * sizeof(std::int64_t)), "upload failed");
    check(vc_cuda_cross_entropy(ptr(logits), static_cast<const int64_t*>(as_cuda(*r.targets).raw()), batch, classes,
                                batch, ptr(*r.loss), ptr(*r.row_max), ptr(*r.row_sum), nullptr),
          "cross_entropy failed");
    return r;
}

std::shared_ptr<Storage> CudaBackend::cross_entropy_backward(const Storage& logits, const CrossEntropyResult& forward,
                                                             const Storage& upstream, std::size_t batch,
                                                             std::size_t classes) {
    auto out = make(batch * classes, device_);
    check(vc_cuda_cross_entropy_backward(ptr(logits), static_cast<const int64_t*>(as_cuda(*forward.targets).raw()),
                                         ptr(*forward.row_max), ptr(*forward.row_sum), ptr(upstream), batch, classes,
                                         batch, out->device_data()),
          "cross_entropy_backward failed");
    return out;
}

bool cuda_available() { return CudaBackend::instance().available(); }

std::string cuda_device_name() { return CudaBackend::instance().device_name(); }

void cuda_synchronize() {
    if (CudaBackend::instance().available()) CudaBackend::instance().synchronize();
}

}  // namespace vectorcore
