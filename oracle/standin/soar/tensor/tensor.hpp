// TEST INFRASTRUCTURE ONLY (oracle). Never linked into the product library.
//
// Minimal stand-in for the reference's include/soar/tensor/tensor.hpp so that
// the reference's unmodified src/optim/adamw.cpp compiles on its own (the real
// header pulls in Vulkan and palloc, whose submodules are empty). It provides
// exactly the surface adamw.cpp touches:
//   numel(), data(), grad(), set_grad(), is_cuda(), is_on_device(),
//   sync_to_host(), sync_to_device(), sync_to_cuda(), zero_grad()
// (reference tensor.hpp:47,51,79,95,97,69,75,76,84,98), over caller-owned host
// memory so the oracle updates numpy buffers in place. All tensors are
// host-resident, so every sync_* is a no-op, as it is for a host tensor in the
// reference (tensor.cpp:131-165 only act when a device copy exists).
#pragma once

#include <cstddef>
#include <cstring>
#include <memory>
#include <vector>

namespace soar {

class Tensor;
using TensorPtr = std::shared_ptr<Tensor>;

class Tensor {
public:
    Tensor(float* data, size_t numel) : data_(data), numel_(numel) {}
    explicit Tensor(size_t numel) : own_(numel, 0.0f), data_(own_.data()), numel_(numel) {}

    static TensorPtr create(size_t shape, bool /*requires_grad*/) {
        return std::make_shared<Tensor>(shape);
    }
    [[nodiscard]] size_t shape() const noexcept { return numel_; }

    [[nodiscard]] size_t numel() const noexcept { return numel_; }
    [[nodiscard]] float* data() noexcept { return data_; }
    [[nodiscard]] const float* data() const noexcept { return data_; }

    [[nodiscard]] TensorPtr grad() const noexcept { return grad_; }
    void set_grad(TensorPtr g) noexcept { grad_ = std::move(g); }

    [[nodiscard]] bool is_cuda() const noexcept { return false; }
    [[nodiscard]] bool is_on_device() const noexcept { return false; }
    void sync_to_host() {}
    void sync_to_device() {}
    void sync_to_cuda(void* = nullptr) {}

    // reference tensor.cpp:167-171 -> zero_() (tensor.cpp:99-107): host fill.
    void zero_grad() {
        if (grad_ && grad_->data_ && grad_->numel_) {
            std::memset(grad_->data_, 0, grad_->numel_ * sizeof(float));
        }
    }

private:
    std::vector<float> own_;
    float* data_;
    size_t numel_;
    TensorPtr grad_;
};

}  // namespace soar
