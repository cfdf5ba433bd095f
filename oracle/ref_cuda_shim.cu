// TEST INFRASTRUCTURE ONLY (secondary GPU baseline). Never linked into the
// product library.
//
// extern "C" entry points over the reference's own CUDA AdamW kernels
// (src/cuda/ops/optimizer_kernels.cu: k_adamw_multi_tensor :44 and
// k_adamw_step :117, host launchers :154-240), which the reference builds for
// sm_60-sm_89 and never calls. oracle/Makefile compiles them unmodified, from
// where they lie, for sm_100a into oracle/_ref/libsoar_ref_cuda.so so the
// tests can run them beside this repository's kernels.
#include <cstdint>

#include <soar/cuda/cuda_kernels.hpp>

extern "C" {

// Arrays are host arrays of device pointers (the reference's launcher builds
// its per-launch metadata on the host).
void soar_refcuda_adamw_multi_tensor(float** params, const float** grads, float** m, float** v,
                                     const int64_t* numel, int n_tensors, float lr, float beta1,
                                     float beta2, float eps, float wd, float step_size,
                                     float sqrt_bc2, void* stream) {
    soar::cuda::kernels::adamw_step_multi_tensor(params, grads, m, v, numel, n_tensors, lr,
                                                 beta1, beta2, eps, wd, step_size, sqrt_bc2,
                                                 stream);
}

void soar_refcuda_adamw_step(float* theta, const float* g, float* m, float* v, float lr,
                             float beta1, float beta2, float eps, float wd, float step_size,
                             float sqrt_bc2, uint64_t n, void* stream) {
    soar::cuda::kernels::adamw_step(theta, g, m, v, lr, beta1, beta2, eps, wd, step_size,
                                    sqrt_bc2, static_cast<size_t>(n), stream);
}

}  // extern "C"
