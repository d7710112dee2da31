// cuda_backend.hpp -- VectorCore's CUDA device for the C++20 host.
//
// The reference's host dispatches every non-CPU op to a device object with
// the method set of MetalBackend (include/vectorcore/metal_backend.hpp:13-56).
// CudaBackend has that method set, with the same argument meaning, on top of
// the C ABI in include/vc_cuda.h, plus the fused entry points of the CUDA
// device. It compiles against the reference's own headers (Storage, Shape,
// cpu::BinaryOp/UnaryOp/ReduceOp): the host gains a DeviceType::CUDA and
// routes it to CudaBackend::instance() at its dispatch sites
// (src/ops.cpp:31-39 and the others), as reference_cuda_device.patch in this
// directory does. Storages report Device::cuda() when the host's device.hpp
// defines VECTORCORE_HAS_CUDA_DEVICE, else the host's non-CPU device value
// (the plugin-slot build, metal_slot.cpp).
//
// Errors: every failing vc_cuda_* call becomes the reference's exception type
// for the status -- std::invalid_argument, std::out_of_range,
// std::overflow_error or std::runtime_error -- carrying vc_cuda_last_error().
// Execution is asynchronous; download() and synchronize() block.
#pragma once

#include "vectorcore/cpu_backend.hpp"
#include "vectorcore/device.hpp"
#include "vectorcore/shape.hpp"
#include "vectorcore/storage.hpp"

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

namespace vectorcore {

// Device buffer from the CUDA device's stream-ordered pool; the base class
// carries the version counter shared by every view (storage.hpp:22-23).
// Not host-addressable: data()/mutable_data() throw like other device storage.
class CudaStorage final : public Storage {
public:
    CudaStorage(std::size_t elements, Device device, std::size_t element_bytes = sizeof(float));
    ~CudaStorage() override;
    CudaStorage(const CudaStorage&) = delete;
    CudaStorage& operator=(const CudaStorage&) = delete;

    [[nodiscard]] Device device() const noexcept override { return device_; }
    [[nodiscard]] std::size_t size() const noexcept override { return size_; }
    [[nodiscard]] float* device_data() const noexcept { return static_cast<float*>(ptr_); }
    [[nodiscard]] void* raw() const noexcept { return ptr_; }

private:
    void* ptr_{nullptr};
    std::size_t size_{0};
    Device device_;
};

class CudaBackend {
public:
    // `device` is the Device value the storages report (Device(DeviceType::CUDA)
    // once the host has that enumerator).
    static CudaBackend& instance();
    explicit CudaBackend(Device device);

    [[nodiscard]] bool available() const noexcept;
    [[nodiscard]] std::string device_name() const;
    [[nodiscard]] std::string last_error() const;
    [[nodiscard]] std::string gemm_kernel() const;

    // ---- MetalBackend's method set ----------------------------------------
    [[nodiscard]] std::shared_ptr<Storage> allocate(std::size_t elements);
    [[nodiscard]] std::shared_ptr<Storage> upload(const float* data, std::size_t elements);
    void download(const Storage& source, float* destination, std::size_t elements);
    [[nodiscard]] std::shared_ptr<Storage> binary(const Storage& a, const Shape& a_shape, const Strides& a_strides,
                                                  const Storage& b, const Shape& b_shape, const Strides& b_strides,
                                                  const Shape& out_shape, cpu::BinaryOp operation);
    [[nodiscard]] std::shared_ptr<Storage> unary(const Storage& input, std::size_t count, cpu::UnaryOp operation);
    [[nodiscard]] std::shared_ptr<Storage> matmul(const Storage& a, const Storage& b, std::size_t m, std::size_t k,
                                                  std::size_t n, const std::vector<std::size_t>& a_offsets,
                                                  const std::vector<std::size_t>& b_offsets, bool trans_a = false,
                                                  bool trans_b = false);
    [[nodiscard]] std::shared_ptr<Storage> transpose_last2(const Storage& input, std::size_t batch, std::size_t rows,
                                                           std::size_t cols);
    [[nodiscard]] std::shared_ptr<Storage> reduce_sum(const Storage& input, std::size_t count);
    [[nodiscard]] std::shared_ptr<Storage> reduce_axis(const Storage& input, std::size_t outer, std::size_t length,
                                                       std::size_t inner, cpu::ReduceOp operation);
    [[nodiscard]] std::shared_ptr<Storage> scatter_axis(const Storage& values, const Storage& indices,
                                                        std::size_t outer, std::size_t length, std::size_t inner);
    void axpy_inplace(Storage& target, const Storage& source, std::size_t count, float alpha);
    void synchronize();

    // ---- fused entry points of the CUDA device ------------------------------
    // detail::broadcast_to (src/autograd.cpp:74-91): value + 0 into target_shape,
    // without the one-float upload of the scalar zero the reference adds.
    [[nodiscard]] std::shared_ptr<Storage> broadcast_to(const Storage& value, const Shape& value_shape,
                                                        const Shape& target_shape);
    // max along the middle axis together with its first-maximum index (int64),
    // one pass; the reference runs a second argmax pass when grad is needed
    // (src/ops.cpp:323-331).
    struct MaxResult {
        std::shared_ptr<Storage> values, indices;
    };
    [[nodiscard]] MaxResult max_with_index(const Storage& input, std::size_t outer, std::size_t length,
                                           std::size_t inner);
    // The max backward: the upstream gradient scattered at the int64 indices
    // (cpu::scatter_axis, src/cpu/cpu_backend.cpp:462-471).
    [[nodiscard]] std::shared_ptr<Storage> max_backward(const Storage& gradient, const Storage& indices,
                                                        std::size_t outer, std::size_t length, std::size_t inner);
    // detail::sum_to_shape (src/autograd.cpp:50-72) in one strided reduce.
    [[nodiscard]] std::shared_ptr<Storage> sum_to_shape(const Storage& gradient, const Shape& g_shape,
                                                        const Shape& target_shape);
    // Both gradients of a (op) b, each reduced to its operand's shape.
    void binary_backward(cpu::BinaryOp operation, const Storage& a, const Shape& a_shape, const Storage& b,
                         const Shape& b_shape, const Storage& gradient, const Shape& g_shape,
                         std::shared_ptr<Storage>* da, std::shared_ptr<Storage>* db);
    // VJP of a unary op from the forward input x and/or output y.
    [[nodiscard]] std::shared_ptr<Storage> unary_backward(cpu::UnaryOp operation, const Storage* x, const Storage* y,
                                                          const Storage& gradient, std::size_t count);
    struct SoftmaxResult {
        std::shared_ptr<Storage> values, row_max, row_sum;
    };
    [[nodiscard]] SoftmaxResult softmax(const Storage& x, std::size_t outer, std::size_t length, std::size_t inner,
                                        bool log);
    [[nodiscard]] std::shared_ptr<Storage> softmax_backward(const Storage& x, const Storage& row_max,
                                                            const Storage& row_sum, const Storage& gradient,
                                                            std::size_t outer, std::size_t length, std::size_t inner,
                                                            bool log);
    struct CrossEntropyResult {
        std::shared_ptr<Storage> loss, row_max, row_sum, targets;
    };
    // Targets are validated on the host (std::out_of_range, as nn.cpp:39-42)
    // and uploaded as int64.
    [[nodiscard]] CrossEntropyResult cross_entropy(const Storage& logits, const std::vector<std::size_t>& targets,
                                                   std::size_t batch, std::size_t classes);
    [[nodiscard]] std::shared_ptr<Storage> cross_entropy_backward(const Storage& logits,
                                                                  const CrossEntropyResult& forward,
                                                                  const Storage& upstream, std::size_t batch,
                                                                  std::size_t classes);

private:
    Device device_;
};

// Free functions next to metal_available() / metal_device_name() /
// synchronize() (include/vectorcore/metal_backend.hpp:58-63).
[[nodiscard]] bool cuda_available();
[[nodiscard]] std::string cuda_device_name();
// Block until the CUDA device's queued work finished and surface its
// asynchronous errors; a no-op when no CUDA device is usable.
void cuda_synchronize();

}  // namespace vectorcore
