// TEST INFRASTRUCTURE ONLY (oracle). Never linked into the product library.
//
// extern "C" shim over the reference's own, unmodified optimizer code
// (src/optim/adamw.cpp, compiled from where it lies in the reference tree by
// oracle/Makefile into oracle/_ref/libsoar_ref_adamw.so). Lets Python tests
// drive soar::optim::AdamW / CosineAnnealingLR exactly as the reference's
// tests/test_optimizers.cpp does, on numpy buffers that the stand-in Tensor
// views in place.
//
// AdamW keeps m_, v_ and step_count_ private (reference adamw.hpp:32-39). The
// parity tests must read and seed them, so this translation unit widens access
// for the reference header only; the class layout is unchanged and the
// reference's adamw.cpp itself is compiled without this.
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <memory>
#include <vector>

#include <soar/tensor/tensor.hpp>  // the stand-in (oracle/standin)

#define private public
#include <soar/optim/adamw.hpp>  // the reference header, unmodified
#undef private
#include <soar/optim/sgd.hpp>    // the reference header, unmodified
#include <soar/nn/module.hpp>    // the stand-in (oracle/standin)
#include <soar/utils/ema.hpp>    // the reference header, unmodified

namespace {

struct RefOptim {
    std::vector<soar::TensorPtr> params;
    std::unique_ptr<soar::optim::AdamW> opt;
};

struct RefSgd {
    std::vector<soar::TensorPtr> params;
    std::unique_ptr<soar::optim::SGD> opt;
};

struct RefEma {
    std::shared_ptr<soar::nn::Module> model;
    std::unique_ptr<soar::utils::ModelEMA> ema;
};

struct RefSched {
    std::unique_ptr<soar::optim::CosineAnnealingLR> sched;
};

}  // namespace

extern "C" {

// params[i]/grads[i]: host fp32 buffers of numel[i] elements. grads[i] may be
// NULL: the reference then skips that param (adamw.cpp:30-31,74-75).
void* soar_ref_adamw_create(float** params, float** grads, const uint64_t* numel, int n,
                            float lr, float beta1, float beta2, float eps, float wd) {
    auto* h = new RefOptim();
    for (int i = 0; i < n; ++i) {
        auto p = std::make_shared<soar::Tensor>(params[i], static_cast<size_t>(numel[i]));
        if (grads && grads[i]) {
            p->set_grad(std::make_shared<soar::Tensor>(grads[i], static_cast<size_t>(numel[i])));
        }
        h->params.push_back(p);
    }
    soar::optim::AdamWOptions o;
    o.lr = lr;
    o.beta1 = beta1;
    o.beta2 = beta2;
    o.eps = eps;
    o.weight_decay = wd;
    h->opt = std::make_unique<soar::optim::AdamW>(h->params, o);
    return h;
}

void soar_ref_adamw_destroy(void* h) { delete static_cast<RefOptim*>(h); }

void soar_ref_adamw_step(void* h) { static_cast<RefOptim*>(h)->opt->step(); }

float soar_ref_adamw_clip_grad_norm(void* h, float max_norm) {
    return static_cast<RefOptim*>(h)->opt->clip_grad_norm(max_norm);
}

void soar_ref_adamw_zero_grad(void* h) { static_cast<RefOptim*>(h)->opt->zero_grad(); }

void soar_ref_adamw_set_lr(void* h, float lr) { static_cast<RefOptim*>(h)->opt->set_lr(lr); }

float soar_ref_adamw_get_lr(void* h) { return static_cast<RefOptim*>(h)->opt->get_lr(); }

uint64_t soar_ref_adamw_get_step(void* h) { return static_cast<RefOptim*>(h)->opt->step_count_; }

void soar_ref_adamw_set_step(void* h, uint64_t t) { static_cast<RefOptim*>(h)->opt->step_count_ = t; }

// which: 0 = m, 1 = v. Copies numel floats of param idx's moment out / in.
int soar_ref_adamw_get_moment(void* h, int idx, int which, float* out) {
    auto* r = static_cast<RefOptim*>(h);
    auto& vec = which == 0 ? r->opt->m_ : r->opt->v_;
    if (idx < 0 || static_cast<size_t>(idx) >= vec.size()) return -1;
    std::memcpy(out, vec[idx].data(), vec[idx].size() * sizeof(float));
    return 0;
}

int soar_ref_adamw_set_moment(void* h, int idx, int which, const float* in) {
    auto* r = static_cast<RefOptim*>(h);
    auto& vec = which == 0 ? r->opt->m_ : r->opt->v_;
    if (idx < 0 || static_cast<size_t>(idx) >= vec.size()) return -1;
    std::memcpy(vec[idx].data(), in, vec[idx].size() * sizeof(float));
    return 0;
}

void* soar_ref_cosine_create(void* h, uint64_t total_steps, float eta_min, uint64_t warmup_steps) {
    auto* s = new RefSched();
    s->sched = std::make_unique<soar::optim::CosineAnnealingLR>(
        *static_cast<RefOptim*>(h)->opt, static_cast<size_t>(total_steps), eta_min,
        static_cast<size_t>(warmup_steps));
    return s;
}

void soar_ref_cosine_step(void* s) { static_cast<RefSched*>(s)->sched->step(); }

void soar_ref_cosine_destroy(void* s) { delete static_cast<RefSched*>(s); }

// The reference's SGD (src/optim/sgd.cpp) over numpy fp32 buffers.
void* soar_ref_sgd_create(float** params, float** grads, const uint64_t* numel, int n, float lr,
                          float momentum, float dampening, float wd, int nesterov) {
    auto* h = new RefSgd();
    for (int i = 0; i < n; ++i) {
        auto p = std::make_shared<soar::Tensor>(params[i], static_cast<size_t>(numel[i]));
        if (grads && grads[i])
            p->set_grad(std::make_shared<soar::Tensor>(grads[i], static_cast<size_t>(numel[i])));
        h->params.push_back(p);
    }
    soar::optim::SGDOptions o;
    o.lr = lr;
    o.momentum = momentum;
    o.dampening = dampening;
    o.weight_decay = wd;
    o.nesterov = nesterov != 0;
    h->opt = std::make_unique<soar::optim::SGD>(h->params, o);
    return h;
}
void soar_ref_sgd_step(void* h) { static_cast<RefSgd*>(h)->opt->step(); }
float soar_ref_sgd_clip_grad_norm(void* h, float max_norm) {
    return static_cast<RefSgd*>(h)->opt->clip_grad_norm(max_norm);
}
void soar_ref_sgd_set_lr(void* h, float lr) { static_cast<RefSgd*>(h)->opt->set_lr(lr); }
void soar_ref_sgd_destroy(void* h) { delete static_cast<RefSgd*>(h); }

// The reference's ModelEMA over numpy weight buffers (viewed in place).
void* soar_ref_ema_create(float** params, const uint64_t* numel, int n, float decay) {
    std::vector<soar::TensorPtr> ps;
    for (int i = 0; i < n; ++i)
        ps.push_back(std::make_shared<soar::Tensor>(params[i], static_cast<size_t>(numel[i])));
    auto* h = new RefEma();
    h->model = std::make_shared<soar::nn::Module>(ps);
    h->ema = std::make_unique<soar::utils::ModelEMA>(h->model, decay);
    return h;
}
void soar_ref_ema_update(void* h) {
    auto* r = static_cast<RefEma*>(h);
    r->ema->update(r->model);
}
void soar_ref_ema_apply_to(void* h) {
    auto* r = static_cast<RefEma*>(h);
    r->ema->apply_to(r->model);
}
int soar_ref_ema_shadow(void* h, int idx, float* out) {
    auto* r = static_cast<RefEma*>(h);
    const auto& sh = r->ema->shadow_params();
    if (idx < 0 || static_cast<size_t>(idx) >= sh.size()) return -1;
    std::memcpy(out, sh[idx]->data(), sh[idx]->numel() * sizeof(float));
    return 0;
}
void soar_ref_ema_destroy(void* h) { delete static_cast<RefEma*>(h); }

}  // extern "C"
