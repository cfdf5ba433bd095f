// A Trainer-shaped driver of the fused optimizer step, as the reference's
// engine would hold it after the drop-in:
//   - the Trainer owns the optimizer by value (include/soar/engine/trainer.hpp:100)
//     and a scheduler, with grad_clip_ defaulting to 2.0f (trainer.hpp:103);
//   - the caller builds the optimizer, binds the scheduler to it and then
//     moves both into the Trainer (src/main.cpp:712-716);
//   - train_step runs clip_grad_norm(grad_clip_) -> step() -> zero_grad()
//     (src/engine/trainer.cpp:157-159) on device tensors, here with the
//     asynchronous clip, so a step never waits on the host.
// Checked: after 20 steps the parameters equal, bit for bit, those of a
// second optimizer driven in the reference's synchronous sequence
// (clip_grad_norm returning the norm, then step, zero_grad) with the same
// gradients and schedule; the scheduler reached the moved optimizer; and
// the host enqueued all 20 steps before the GPU finished them (no host
// synchronisation inside a step). Exit code 0 = pass.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <vector>

#include <cuda_runtime.h>

#include "soar_optim.hpp"

namespace {

int g_failures = 0;
#define CHECK(cond, ...)                                      \
    do {                                                      \
        if (!(cond)) {                                        \
            std::printf("FAIL %s:%d: ", __FILE__, __LINE__);  \
            std::printf(__VA_ARGS__);                         \
            std::printf("\n");                                \
            ++g_failures;                                     \
        }                                                     \
    } while (0)

// Device tensor with the reference Tensor's optimizer-facing surface
// (numel, cuda_data, grad: include/soar/tensor/tensor.hpp:47,80,95).
class DevTensor;
using TensorPtr = std::shared_ptr<DevTensor>;
class DevTensor {
public:
    explicit DevTensor(const std::vector<float>& v) : n_(v.size()) {
        cudaMalloc(&d_, n_ * sizeof(float));
        cudaMemcpy(d_, v.data(), n_ * sizeof(float), cudaMemcpyHostToDevice);
    }
    ~DevTensor() { cudaFree(d_); }
    size_t numel() const noexcept { return n_; }
    float* cuda_data() noexcept { return d_; }
    TensorPtr grad() const noexcept { return grad_; }
    void set_grad(TensorPtr g) { grad_ = std::move(g); }
    std::vector<float> host() const {
        std::vector<float> v(n_);
        cudaMemcpy(v.data(), d_, n_ * sizeof(float), cudaMemcpyDeviceToHost);
        return v;
    }

private:
    float* d_{nullptr};
    size_t n_;
    TensorPtr grad_;
};

// Seeded normal values: SplitMix64 then Box-Muller in double.
std::vector<float> normals(uint64_t seed, size_t n, double std_dev) {
    std::vector<float> out(n);
    uint64_t s = seed;
    auto next = [&s]() {
        uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    for (size_t i = 0; i < n; i += 2) {
        const double u1 = (static_cast<double>(next() >> 11) + 1.0) * 0x1.0p-53;
        const double u2 = static_cast<double>(next() >> 11) * 0x1.0p-53;
        const double r = std::sqrt(-2.0 * std::log(u1)) * std_dev;
        out[i] = static_cast<float>(r * std::cos(2.0 * M_PI * u2));
        if (i + 1 < n) out[i + 1] = static_cast<float>(r * std::sin(2.0 * M_PI * u2));
    }
    return out;
}

// The reference Trainer's optimizer-facing part.
class Trainer {
public:
    Trainer(std::vector<TensorPtr> params, soar::optim::AdamW optimizer,
            std::unique_ptr<soar::optim::CosineAnnealingLR> scheduler, float grad_clip = 2.0f)
        : params_(std::move(params)), optimizer_(std::move(optimizer)),
          scheduler_(std::move(scheduler)), grad_clip_(grad_clip) {}

    // One step on `stream`. The backward pass is stood in for by copying this
    // step's gradients into the gradient tensors from pinned host memory.
    void train_step(const std::vector<const float*>& host_grads, cudaStream_t stream) {
        for (size_t i = 0; i < params_.size(); ++i)
            cudaMemcpyAsync(params_[i]->grad()->cuda_data(), host_grads[i],
                            params_[i]->numel() * sizeof(float), cudaMemcpyHostToDevice, stream);
        optimizer_.clip_grad_norm_async(grad_clip_, stream);  // trainer.cpp:157
        optimizer_.step(stream);                              // trainer.cpp:158
        optimizer_.zero_grad(stream);                         // trainer.cpp:159
    }
    void step_scheduler() { scheduler_->step(); }
    soar::optim::AdamW& optimizer() { return optimizer_; }

private:
    std::vector<TensorPtr> params_;
    soar::optim::AdamW optimizer_;
    std::unique_ptr<soar::optim::CosineAnnealingLR> scheduler_;
    float grad_clip_{2.0f};
};

constexpr int kSteps = 20;
const size_t kSizes[3] = {6000000, 1000003, 4099};

std::vector<TensorPtr> make_params(uint64_t seed) {
    std::vector<TensorPtr> ps;
    for (int i = 0; i < 3; ++i) {
        auto p = std::make_shared<DevTensor>(normals(seed + i, kSizes[i], 0.02));
        p->set_grad(std::make_shared<DevTensor>(std::vector<float>(kSizes[i], 0.0f)));
        ps.push_back(p);
    }
    return ps;
}

}  // namespace

int main() {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        std::printf("no CUDA device\n");
        return 77;
    }
    // the gradients of every step, in pinned host memory (three sets cycled;
    // std 0.05 over ~7M elements gives norms of ~130, so every step clips)
    std::vector<float*> pinned[3];
    for (int k = 0; k < 3; ++k)
        for (int i = 0; i < 3; ++i) {
            float* h = nullptr;
            cudaMallocHost(&h, kSizes[i] * sizeof(float));
            const std::vector<float> g = normals(1000 + 10 * k + i, kSizes[i], 0.05);
            std::memcpy(h, g.data(), g.size() * sizeof(float));
            pinned[k].push_back(h);
        }
    auto grads_of = [&](int t) {
        return std::vector<const float*>(pinned[t % 3].begin(), pinned[t % 3].end());
    };
    cudaStream_t stream;
    cudaStreamCreate(&stream);
    soar::optim::AdamWOptions opts;
    opts.lr = 1e-3f;

    // --- the Trainer: optimizer built, scheduler bound, both moved in ------
    auto params = make_params(7);
    soar::optim::AdamW optimizer(params, opts);
    auto scheduler = std::make_unique<soar::optim::CosineAnnealingLR>(optimizer, kSteps, 1e-6f, 2);
    Trainer trainer(params, std::move(optimizer), std::move(scheduler));
    cudaStreamSynchronize(stream);
    for (int t = 0; t < kSteps; ++t) {
        trainer.train_step(grads_of(t), stream);
        trainer.step_scheduler();
    }
    cudaEvent_t done;
    cudaEventCreate(&done);
    cudaEventRecord(done, stream);
    const cudaError_t q = cudaEventQuery(done);
    CHECK(q == cudaErrorNotReady,
          "the host waited for the GPU inside the steps (event already complete: %d)", int(q));
    cudaStreamSynchronize(stream);
    const soar_step_info ti = trainer.optimizer().info(stream);

    // --- the reference's synchronous sequence on a second optimizer --------
    auto ref_params = make_params(7);
    soar::optim::AdamW ref(ref_params, opts);
    soar::optim::CosineAnnealingLR ref_sched(ref, kSteps, 1e-6f, 2);
    std::vector<float> norms;
    for (int t = 0; t < kSteps; ++t) {
        const auto g = grads_of(t);
        for (int i = 0; i < 3; ++i)
            cudaMemcpyAsync(ref_params[i]->grad()->cuda_data(), g[i], kSizes[i] * sizeof(float),
                            cudaMemcpyHostToDevice, stream);
        norms.push_back(ref.clip_grad_norm(2.0f, stream));
        ref.step(stream);
        ref.zero_grad(stream);
        ref_sched.step();
    }
    cudaStreamSynchronize(stream);
    const soar_step_info ri = ref.info(stream);

    CHECK(ti.step == kSteps && ri.step == kSteps, "steps %llu / %llu",
          (unsigned long long)ti.step, (unsigned long long)ri.step);
    CHECK(ti.grad_norm == norms.back(), "last pre-clip norm %.9g vs %.9g", ti.grad_norm,
          norms.back());
    CHECK(norms.back() > 2.0f && ti.clip_coef < 1.0f, "the steps clipped (norm %.9g)", norms.back());
    CHECK(trainer.optimizer().get_lr() == ref.get_lr() && ref.get_lr() < opts.lr,
          "the scheduler drives the moved optimizer (lr %.9g vs %.9g)",
          trainer.optimizer().get_lr(), ref.get_lr());
    size_t diff = 0;
    for (int i = 0; i < 3; ++i) {
        const auto a = params[i]->host(), b = ref_params[i]->host();
        diff += std::memcmp(a.data(), b.data(), a.size() * sizeof(float)) != 0;
        const auto ga = params[i]->grad()->host();
        bool zero = true;
        for (float x : ga) zero = zero && x == 0.0f;
        CHECK(zero, "zero_grad left tensor %d's gradient non-zero", i);
    }
    CHECK(diff == 0, "%zu tensors differ from the synchronous sequence", diff);
    cudaEventDestroy(done);
    cudaStreamDestroy(stream);
    for (auto& set : pinned)
        for (float* h : set) cudaFreeHost(h);
    if (g_failures) {
        std::printf("%d FAILURE(S)\n", g_failures);
        return 1;
    }
    std::printf("TRAINER DRIVER TEST PASSED (%d steps, last norm %.6g, lr %.6g)\n", kSteps,
                ti.grad_norm, trainer.optimizer().get_lr());
    return 0;
}
