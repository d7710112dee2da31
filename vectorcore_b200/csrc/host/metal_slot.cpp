// metal_slot.cpp -- the CUDA device in the reference's existing device slot.
//
// The reference compiles exactly one implementation of the MetalBackend
// interface: src/metal/metal_backend.mm on Apple, src/metal/
// metal_backend_stub.cpp elsewhere (include/vectorcore/metal_backend.hpp:13-63).
// Its dispatch sites send every non-CPU tensor to MetalBackend::instance()
// (src/ops.cpp:31-39, src/autograd.cpp:81-89, src/tensor.cpp:57-64, ...). This file
// is a third implementation of that interface which forwards to CudaBackend:
// linked with the reference's UNMODIFIED sources in place of the stub, the
// reference's own Tensor / autograd / nn / pybind11 surface runs on the B200,
// with the non-CPU device value (spelled "metal" by the reference's
// Device::str()) meaning the CUDA device. It demonstrates the drop-in
// boundary without editing a reference file; the integration proper adds
// DeviceType::CUDA next to CPU and Metal and calls CudaBackend directly
// (reference_cuda_device.patch in this directory).
#include "cuda_backend.hpp"

#include "vectorcore/metal_backend.hpp"

namespace vectorcore {
namespace {

class CudaInMetalSlot final : public MetalBackend {
public:
    bool available() const noexcept override { return cuda().available(); }
    std::string device_name() const override { return cuda().device_name(); }
    std::string last_error() const override { return cuda().last_error(); }
    std::string gemm_kernel() const override { return cuda().gemm_kernel(); }
    std::shared_ptr<Storage> allocate(std::size_t elements) override { return cuda().allocate(elements); }
    std::shared_ptr<Storage> upload(const float* data, std::size_t elements) override {
        return cuda().upload(data, elements);
    }
    void download(const Storage& source, float* destination, std::size_t elements) override {
        cuda().download(source, destination, elements);
    }
    std::shared_ptr<Storage> binary(const Storage& a, const Shape& a_shape, const Strides& a_strides, const Storage& b,
                                    const Shape& b_shape, const Strides& b_strides, const Shape& out_shape,
                                    cpu::BinaryOp operation) override {
        return cuda().binary(a, a_shape, a_strides, b, b_shape, b_strides, out_shape, operation);
    }
    std::shared_ptr<Storage> unary(const Storage& input, std::size_t count, cpu::UnaryOp operation) override {
        return cuda().unary(input, count, operation);
    }
    std::shared_ptr<Storage> matmul(const Storage& a, const Storage& b, std::size_t m, std::size_t k, std::size_t n,
                                    const std::vector<std::size_t>& a_offsets,
                                    const std::vector<std::size_t>& b_offsets, bool trans_a,
                                    bool trans_b) override {
        return cuda().matmul(a, b, m, k, n, a_offsets, b_offsets, trans_a, trans_b);
    }
    std::shared_ptr<Storage> transpose_last2(const Storage& input, std::size_t batch, std::size_t rows,
                                             std::size_t cols) override {
        return cuda().transpose_last2(input, batch, rows, cols);
    }
    std::shared_ptr<Storage> reduce_sum(const Storage& input, std::size_t count) override {
        return cuda().reduce_sum(input, count);
    }
    std::shared_ptr<Storage> reduce_axis(const Storage& input, std::size_t outer, std::size_t length,
                                         std::size_t inner, cpu::ReduceOp operation) override {
        return cuda().reduce_axis(input, outer, length, inner, operation);
    }
    std::shared_ptr<Storage> scatter_axis(const Storage& values, const Storage& indices, std::size_t outer,
                                          std::size_t length, std::size_t inner) override {
        return cuda().scatter_axis(values, indices, outer, length, inner);
    }
    void axpy_inplace(Storage& target, const Storage& source, std::size_t count, float alpha) override {
        cuda().axpy_inplace(target, source, count, alpha);
    }
    void synchronize() override { cuda().synchronize(); }

private:
    static CudaBackend& cuda() { return CudaBackend::instance(); }
};

}  // namespace

MetalBackend& MetalBackend::instance() {
    static CudaInMetalSlot backend;
    return backend;
}

bool metal_available() { return MetalBackend::instance().available(); }
std::string metal_device_name() { return MetalBackend::instance().device_name(); }
void synchronize() {
    if (MetalBackend::instance().available()) MetalBackend::instance().synchronize();
}

}  // namespace vectorcore
