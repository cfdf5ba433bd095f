// Device-side data structures shared by the optimizer-step kernels and the
// host code that builds them.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace soarb {

// Elements per chunk-table entry. A multiple of 4 (the vector width), large
// enough that the per-chunk descriptor read (64 B) is noise next to the
// 28 B/element the update streams (458 KB per full chunk).
constexpr uint32_t kChunkElems = 16384;

// Chunk flag: every pointer of the chunk is vector aligned at its first
// element (16 B for fp32 streams, 8 B for 4 x bf16), so the body runs on
// 128-bit (fp32) / 64-bit (4 x bf16) loads and stores.
constexpr uint32_t kChunkVec = 1u;

// One contiguous run of at most kChunkElems elements of one tensor, with all
// pointers already offset to the run's first element. The update of one
// element touches exactly: param, grad, master (== param in the fp32 layout),
// m and v at the same index.
struct __align__(16) Chunk {
    void* param;        // fp32* or bf16* (bf16 as uint16_t bits)
    const void* grad;   // fp32* or bf16*
    float* master;      // fp32 master weights (== param for the fp32 layout)
    float* m;
    float* v;
    uint32_t n;         // elements in this chunk
    float wd;           // the tensor's decoupled weight decay
    uint32_t flags;     // kChunkVec
    uint32_t tensor;    // tensor index (diagnostics)
};
static_assert(sizeof(Chunk) == 64, "Chunk descriptor must stay one 64-byte line");

// Device-resident step control block. Persistent fields carry the optimizer's
// counters across steps with no host round trip; the tickets implement the
// single-pass grid reductions (last CTA finalises, then resets its ticket).
struct __align__(64) Ctl {
    float scale;            // live loss scale (1 without a scaler)
    int32_t tracker;        // clean steps since the last scale change
    uint64_t t;             // AdamW step count (skipped steps excluded)
    uint64_t skipped;       // skipped steps
    float last_norm;        // pre-clip global norm of the last step
    int32_t last_found_inf;
    float last_clip_coef;
    float last_lr;
    double sumsq;           // single-GPU K1 output: sum of squared unscaled grads
    uint32_t ticket_sumsq;  // grid-reduction ticket of the sum-of-squares kernel
    uint32_t ticket_apply;  // completion ticket of the update kernel
};

// Per-launch arguments of the update kernel.
struct ApplyArgs {
    float lr, beta1, beta2, eps;
    float max_norm;       // > 0: clip by the global norm
    float pending_coef;   // coefficient from a standalone clip_grad_norm (1: none)
    float growth, backoff;
    int32_t interval;
    int32_t use_scaler;
    int32_t n_parts;      // number of fp64 partial sums in `parts` (0: no norm info)
    const double* parts;  // device, n_parts partial sums (rank order)
    const float2* bc;     // device table, bc[t] = (1 - beta1^t, sqrt(1 - beta2^t)), t >= 1
    uint32_t bc_len;      // entries in bc; t >= bc_len uses bc[bc_len - 1]
};

// Launchers (optim_kernels.cu). Each returns the launch status.
cudaError_t launch_grad_sumsq(bool bf16, const Chunk* chunks, int n_chunks, Ctl* ctl,
                              double* partials, int grid, int use_scaler, double* out,
                              cudaStream_t stream);
cudaError_t launch_apply(bool mixed, const Chunk* chunks, int n_chunks, Ctl* ctl,
                         const ApplyArgs& args, int grid, cudaStream_t stream);
cudaError_t launch_scale_grads_f32(const Chunk* chunks, int n_chunks, float coef, int grid,
                                   cudaStream_t stream);
cudaError_t launch_bf16_to_f32(const uint16_t* src, float* dst, uint64_t n,
                               cudaStream_t stream);
cudaError_t launch_set_counters(Ctl* ctl, uint64_t t, uint64_t skipped, float scale,
                                int32_t tracker, cudaStream_t stream);

// Resident CTAs per SM of each kernel at its launch configuration.
int occupancy_grad_sumsq(bool bf16);
int occupancy_apply(bool mixed);

constexpr int kThreads = 256;

}  // namespace soarb
