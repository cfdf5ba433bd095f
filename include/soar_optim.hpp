// soar_optim.hpp -- C++ API of the B200 optimizer step, source-compatible with
// the reference's soar::optim::AdamW / AdamWOptions / CosineAnnealingLR
// (include/soar/optim/adamw.hpp:10-57). Header-only over the C-ABI in
// soar_optim.h; link libsoar_optim.so.
//
// The constructor takes the reference's own parameter list type: any
// std::vector<P> whose elements behave like the reference's TensorPtr
// (p->numel(), p->cuda_data(), p->grad() returning a pointer-like with
// cuda_data(); include/soar/tensor/tensor.hpp:47,80,95). Params must be on the
// GPU (the reference keeps a host copy and a CUDA copy; this step reads and
// writes only the CUDA copy). As in the reference, params without a gradient
// are skipped and the optimizer owns m and v (adamw.hpp:33-39).
//
// Differences, all additive: step()/zero_grad() take an optional stream; the
// optimizer is move-only (the reference's Trainer holds it by value,
// trainer.hpp:100, and moves it in); errors throw std::runtime_error carrying
// soar_last_error() where the reference would throw DeviceError.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "soar_optim.h"

namespace soar::optim {

struct AdamWOptions {  // adamw.hpp:10-16, same fields and defaults
    float lr{1e-3f};
    float beta1{0.9f};
    float beta2{0.999f};
    float eps{1e-8f};
    float weight_decay{1e-2f};
};

// Extensions with no reference counterpart (mixed precision, fused clip,
// loss scaler). Defaults reproduce the reference's fp32 behaviour.
struct AdamWExtOptions {
    int layout{SOAR_LAYOUT_FP32};
    float max_grad_norm{0.0f};
    bool use_loss_scaler{false};
    float init_scale{65536.0f};
    float growth_factor{2.0f};
    float backoff_factor{0.5f};
    int growth_interval{200};
    int device{0};
};

namespace detail {
inline void check(int rc, const char* what) {
    if (rc != SOAR_OK) throw std::runtime_error(std::string(what) + ": " + soar_last_error());
}
}  // namespace detail

class AdamW {
public:
    // AdamW(std::vector<TensorPtr> params, AdamWOptions options = {}) (adamw.hpp:23)
    template <class P>
    explicit AdamW(const std::vector<P>& params, AdamWOptions options = {},
                   AdamWExtOptions ext = {}) {
        std::vector<soar_tensor_desc> d;
        d.reserve(params.size());
        for (const auto& p : params) {
            soar_tensor_desc t{};
            if (p) {
                t.param = p->cuda_data();
                auto g = p->grad();
                t.grad = g ? g->cuda_data() : nullptr;
                t.numel = static_cast<uint64_t>(p->numel());
            }
            t.weight_decay = options.weight_decay;
            d.push_back(t);
        }
        create(d, options, ext);
    }

    // Raw descriptors (per-tensor weight decay = parameter groups).
    AdamW(const std::vector<soar_tensor_desc>& tensors, AdamWOptions options,
          AdamWExtOptions ext) {
        create(tensors, options, ext);
    }

    AdamW(AdamW&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
    AdamW& operator=(AdamW&& o) noexcept {
        if (this != &o) {
            reset();
            h_ = std::exchange(o.h_, nullptr);
        }
        return *this;
    }
    AdamW(const AdamW&) = delete;
    AdamW& operator=(const AdamW&) = delete;
    ~AdamW() { reset(); }

    void step(void* stream = nullptr) { detail::check(soar_optim_step(h_, stream), "step"); }
    void zero_grad(void* stream = nullptr) {
        detail::check(soar_optim_zero_grad(h_, stream), "zero_grad");
    }
    float clip_grad_norm(float max_norm, void* stream = nullptr) {
        float n = 0.0f;
        detail::check(soar_optim_clip_grad_norm(h_, max_norm, &n, stream), "clip_grad_norm");
        return n;
    }
    // The same clip without the host round trip, for a caller that ignores the
    // returned norm (the reference's Trainer, trainer.cpp:157): the next step()
    // clips by max_norm; the norm is that step's info().grad_norm.
    void clip_grad_norm_async(float max_norm, void* stream = nullptr) {
        detail::check(soar_optim_clip_grad_norm_async(h_, max_norm, stream),
                      "clip_grad_norm_async");
    }
    void set_lr(float lr) noexcept { soar_optim_set_lr(h_, lr); }
    [[nodiscard]] float get_lr() const noexcept {
        float lr = 0.0f;
        soar_optim_get_lr(h_, &lr);
        return lr;
    }

    [[nodiscard]] soar_step_info info(void* stream = nullptr) const {
        soar_step_info i{};
        detail::check(soar_optim_get_info(h_, &i, stream), "get_info");
        return i;
    }
    // Enqueues the same readback on `stream` into caller-owned (pinned) host
    // memory; *out is valid once an event recorded after this call completes.
    void info_async(soar_step_info* out, void* stream = nullptr) const {
        detail::check(soar_optim_get_info_async(h_, out, stream), "get_info_async");
    }
    [[nodiscard]] void* handle() const noexcept { return h_; }

private:
    void create(const std::vector<soar_tensor_desc>& d, const AdamWOptions& o,
                const AdamWExtOptions& ext) {
        soar_adamw_opts c;
        soar_adamw_default_opts(&c);
        c.lr = o.lr;
        c.beta1 = o.beta1;
        c.beta2 = o.beta2;
        c.eps = o.eps;
        c.weight_decay = o.weight_decay;
        c.layout = ext.layout;
        c.max_grad_norm = ext.max_grad_norm;
        c.use_loss_scaler = ext.use_loss_scaler ? 1 : 0;
        c.init_scale = ext.init_scale;
        c.growth_factor = ext.growth_factor;
        c.backoff_factor = ext.backoff_factor;
        c.growth_interval = ext.growth_interval;
        c.device = ext.device;
        detail::check(soar_optim_create(d.data(), static_cast<int>(d.size()), &c, &h_), "create");
    }
    void reset() noexcept {
        if (h_) soar_optim_destroy(h_);
        h_ = nullptr;
    }
    void* h_{nullptr};
};

struct SGDOptions {  // include/soar/optim/sgd.hpp:9-15, same fields and defaults
    float lr{1e-2f};
    float momentum{0.0f};
    float dampening{0.0f};
    float weight_decay{0.0f};
    bool nesterov{false};
};

// soar::optim::SGD (sgd.hpp:21-38) on the same device step. Same methods as
// the reference's (step, zero_grad, clip_grad_norm, set_lr, get_lr).
class SGD {
public:
    template <class P>
    explicit SGD(const std::vector<P>& params, SGDOptions options = {},
                 AdamWExtOptions ext = {}) {
        std::vector<soar_tensor_desc> d;
        d.reserve(params.size());
        for (const auto& p : params) {
            soar_tensor_desc t{};
            if (p) {
                t.param = p->cuda_data();
                auto g = p->grad();
                t.grad = g ? g->cuda_data() : nullptr;
                t.numel = static_cast<uint64_t>(p->numel());
            }
            t.weight_decay = options.weight_decay;
            d.push_back(t);
        }
        soar_sgd_opts c;
        soar_sgd_default_opts(&c);
        c.lr = options.lr;
        c.momentum = options.momentum;
        c.dampening = options.dampening;
        c.weight_decay = options.weight_decay;
        c.nesterov = options.nesterov ? 1 : 0;
        c.layout = ext.layout;
        c.max_grad_norm = ext.max_grad_norm;
        c.use_loss_scaler = ext.use_loss_scaler ? 1 : 0;
        c.init_scale = ext.init_scale;
        c.growth_factor = ext.growth_factor;
        c.backoff_factor = ext.backoff_factor;
        c.growth_interval = ext.growth_interval;
        c.device = ext.device;
        detail::check(soar_sgd_create(d.data(), static_cast<int>(d.size()), &c, &h_),
                      "sgd_create");
    }
    SGD(SGD&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
    SGD& operator=(SGD&& o) noexcept {
        if (this != &o) {
            if (h_) soar_optim_destroy(h_);
            h_ = std::exchange(o.h_, nullptr);
        }
        return *this;
    }
    SGD(const SGD&) = delete;
    SGD& operator=(const SGD&) = delete;
    ~SGD() {
        if (h_) soar_optim_destroy(h_);
    }

    void step(void* stream = nullptr) { detail::check(soar_optim_step(h_, stream), "step"); }
    void zero_grad(void* stream = nullptr) {
        detail::check(soar_optim_zero_grad(h_, stream), "zero_grad");
    }
    float clip_grad_norm(float max_norm, void* stream = nullptr) {
        float n = 0.0f;
        detail::check(soar_optim_clip_grad_norm(h_, max_norm, &n, stream), "clip_grad_norm");
        return n;
    }
    void clip_grad_norm_async(float max_norm, void* stream = nullptr) {
        detail::check(soar_optim_clip_grad_norm_async(h_, max_norm, stream),
                      "clip_grad_norm_async");
    }
    void set_lr(float lr) noexcept { soar_optim_set_lr(h_, lr); }
    [[nodiscard]] float get_lr() const noexcept {
        float lr = 0.0f;
        soar_optim_get_lr(h_, &lr);
        return lr;
    }
    [[nodiscard]] void* handle() const noexcept { return h_; }

private:
    void* h_{nullptr};
};

// CosineAnnealingLR(AdamW&, total_steps, eta_min = 1e-6f, warmup_steps = 0)
// (adamw.hpp:45-57). Bound to the optimizer's handle, so it follows the
// optimizer across moves (the reference binds a reference to the object).
class CosineAnnealingLR {
public:
    CosineAnnealingLR(AdamW& optimizer, size_t total_steps, float eta_min = 1e-6f,
                      size_t warmup_steps = 0) {
        detail::check(soar_cosine_create(optimizer.handle(), total_steps, eta_min, warmup_steps,
                                         &h_),
                      "cosine_create");
    }
    CosineAnnealingLR(CosineAnnealingLR&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
    CosineAnnealingLR(const CosineAnnealingLR&) = delete;
    CosineAnnealingLR& operator=(const CosineAnnealingLR&) = delete;
    ~CosineAnnealingLR() {
        if (h_) soar_cosine_destroy(h_);
    }
    void step() { detail::check(soar_cosine_step(h_), "cosine_step"); }

private:
    void* h_{nullptr};
};

// ---- data parallel (no reference counterpart) ------------------------------

// NCCL communicator of one process (one GPU) of a data-parallel job
// (soar_dp_init). Rank 0 creates the unique id (unique_id()) and hands the
// bytes to the other ranks over any host channel.
class Communicator {
public:
    static std::vector<unsigned char> unique_id() {
        std::vector<unsigned char> id(SOAR_DP_UNIQUE_ID_BYTES);
        detail::check(soar_dp_unique_id(id.data()), "dp_unique_id");
        return id;
    }
    Communicator(int rank, int world, const std::vector<unsigned char>& id, int device)
        : device_(device) {
        if (id.size() != SOAR_DP_UNIQUE_ID_BYTES) throw std::runtime_error("bad unique id size");
        detail::check(soar_dp_init(rank, world, id.data(), device, &h_), "dp_init");
    }
    Communicator(Communicator&& o) noexcept
        : h_(std::exchange(o.h_, nullptr)), device_(o.device_) {}
    Communicator(const Communicator&) = delete;
    Communicator& operator=(const Communicator&) = delete;
    ~Communicator() {
        if (h_) soar_dp_destroy(h_);
    }
    void barrier(void* stream = nullptr) { detail::check(soar_dp_barrier(h_, stream), "barrier"); }
    [[nodiscard]] void* handle() const noexcept { return h_; }
    [[nodiscard]] int device() const noexcept { return device_; }

private:
    void* h_{nullptr};
    int device_;
};

// Fused ZeRO-1 AdamW over a Communicator (soar_dp_zero1_create): the flat bf16
// parameter and gradient buffers of n_params elements are the library's;
// fill grads() with this rank's gradient, call step() on every rank, and
// params() holds the updated model on every rank. Collective to construct and
// to destroy. The communicator must outlive it.
class ZeroOneAdamW {
public:
    ZeroOneAdamW(Communicator& comm, uint64_t n_params, uint64_t bucket,
                 AdamWOptions options = {}, AdamWExtOptions ext = {},
                 const void* init_params = nullptr, int sync_mode = SOAR_DP_SYNC_DEVICE) {
        soar_adamw_opts c;
        soar_adamw_default_opts(&c);
        c.lr = options.lr;
        c.beta1 = options.beta1;
        c.beta2 = options.beta2;
        c.eps = options.eps;
        c.weight_decay = options.weight_decay;
        c.layout = SOAR_LAYOUT_BF16_MIXED;
        c.max_grad_norm = ext.max_grad_norm;
        c.use_loss_scaler = ext.use_loss_scaler ? 1 : 0;
        c.init_scale = ext.init_scale;
        c.growth_factor = ext.growth_factor;
        c.backoff_factor = ext.backoff_factor;
        c.growth_interval = ext.growth_interval;
        c.device = comm.device();
        detail::check(soar_dp_zero1_create(comm.handle(), n_params, bucket, &c, init_params,
                                           sync_mode, &h_),
                      "dp_zero1_create");
        detail::check(soar_dp_zero1_get_info(h_, &info_), "dp_zero1_get_info");
    }
    ZeroOneAdamW(ZeroOneAdamW&& o) noexcept : h_(std::exchange(o.h_, nullptr)), info_(o.info_) {}
    ZeroOneAdamW(const ZeroOneAdamW&) = delete;
    ZeroOneAdamW& operator=(const ZeroOneAdamW&) = delete;
    ~ZeroOneAdamW() {
        if (h_) soar_dp_zero1_destroy(h_);
    }
    void step(void* stream = nullptr) { detail::check(soar_dp_zero1_step(h_, stream), "dp_step"); }
    // A further gradient buffer (collective); returns its index (the first is 0).
    int add_grads() {
        int k = -1;
        detail::check(soar_dp_zero1_add_grads(h_, &k), "dp_zero1_add_grads");
        return k;
    }
    // The buffer the next steps reduce (every rank the same index).
    void use_grads(int index) {
        detail::check(soar_dp_zero1_use_grads(h_, index), "dp_zero1_use_grads");
        detail::check(soar_dp_zero1_get_info(h_, &info_), "dp_zero1_get_info");
    }
    [[nodiscard]] void* grads(int index) const {
        void* p = nullptr;
        detail::check(soar_dp_zero1_grads(h_, index, &p), "dp_zero1_grads");
        return p;
    }
    [[nodiscard]] void* params() const noexcept { return info_.params; }
    [[nodiscard]] void* grads() const noexcept { return info_.grads; }
    [[nodiscard]] uint64_t shard_params() const noexcept { return info_.shard_params; }
    [[nodiscard]] soar_step_info info(void* stream = nullptr) const {
        soar_step_info i{};
        detail::check(soar_optim_get_info(info_.optimizer, &i, stream), "get_info");
        return i;
    }
    [[nodiscard]] int error() const {
        int e = 0;
        detail::check(soar_zero1_error(info_.zero1, &e), "zero1_error");
        return e;
    }
    void set_lr(float lr) noexcept { soar_optim_set_lr(info_.optimizer, lr); }

private:
    void* h_{nullptr};
    soar_dp_zero1_info info_{};
};

}  // namespace soar::optim
