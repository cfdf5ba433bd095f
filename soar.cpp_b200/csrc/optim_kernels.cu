// Optimizer-step kernels for B200 (sm_100a).
//
// The step is HBM-bound streaming work (~15 flop per 28 bytes), so it runs on
// the SIMT pipes with vector loads, not on tensor cores. Two kernels over one
// tensor-list chunk table (Chunk, optim_kernels.cuh):
//
//   k_grad_sumsq  reads every gradient once (2 B bf16 / 4 B fp32 per element),
//                 unscales it by the live loss scale and accumulates the fp64
//                 sum of squares: per thread, warp shuffle, block, then a
//                 single-pass grid reduction (each CTA writes its partial, the
//                 last CTA to take a ticket folds them in fixed order).
//                 Non-finite gradients make the sum non-finite, so the same
//                 number carries the inf/NaN verdict.
//   k_apply       derives skip / clip coefficient / bias corrections from the
//                 partial sums, then streams the update: unscale, clip,
//                 decoupled weight decay, AdamW moments, fp32 master update,
//                 bf16 write-back. It walks the chunks in the reverse order of
//                 k_grad_sumsq so the gradients read last there are still in
//                 L2 when it starts. The last CTA to finish commits the step
//                 counters and the loss-scaler update.
//
// Numerics follow the reference's AdamW::step / clip_grad_norm
// (src/optim/adamw.cpp:87-176) operation for operation with explicitly
// rounded intrinsics (no contraction, IEEE sqrt and division), so the fp32
// update reproduces the reference's bits.
#include "optim_kernels.cuh"

#include <cuda_bf16.h>

namespace soarb {
namespace {

// ------------------------------------------------------------ bf16 helpers --

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

// Two fp32 -> packed bf16x2, round to nearest even (lo in the low half).
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

__device__ __forceinline__ uint16_t f32_to_bf16_rn(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// -------------------------------------------------------------- reductions --

__device__ __forceinline__ double warp_sum(double x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// Deterministic block sum (fixed shuffle pattern, fixed warp order).
__device__ __forceinline__ double block_sum(double x, double* smem /* >= 32 */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    x = warp_sum(x);
    if (lane == 0) smem[warp] = x;
    __syncthreads();
    double r = 0.0;
    if (warp == 0) {
        r = lane < (kThreads / 32) ? smem[lane] : 0.0;
        r = warp_sum(r);
    }
    __syncthreads();
    return r;  // valid in thread 0
}

// ------------------------------------------------------------------ K1 -------

// Sum of (double(g * inv))^2. The square of a float is exact in double, so an
// fma here equals the reference's separate multiply and add
// (adamw.cpp:96-97) term by term; only the summation order differs.
__device__ __forceinline__ double sq_acc(double acc, float g) {
    const double d = static_cast<double>(g);
    return fma(d, d, acc);
}

template <bool kBf16>
__global__ void __launch_bounds__(kThreads)
k_grad_sumsq(const Chunk* __restrict__ chunks, int n_chunks, Ctl* __restrict__ ctl,
             double* __restrict__ partials, int use_scaler, double* __restrict__ out) {
    __shared__ double s_red[32];
    __shared__ int s_last;
    const float inv = use_scaler ? __fdiv_rn(1.0f, ctl->scale) : 1.0f;
    double acc = 0.0;
    for (int c = blockIdx.x; c < n_chunks; c += gridDim.x) {
        const Chunk* ch = chunks + c;
        const uint32_t n = ch->n;
        const void* gp = ch->grad;
        uint32_t scalar_from = 0;
        if (ch->flags & kChunkVec) {
            const uint32_t nv = n >> 2;
            scalar_from = nv << 2;
            if constexpr (kBf16) {
                const uint2* g4 = static_cast<const uint2*>(gp);
                uint32_t i = threadIdx.x;
                for (; i + 3 * kThreads < nv; i += 4 * kThreads) {
                    uint2 q[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) q[u] = __ldg(g4 + i + u * kThreads);
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        acc = sq_acc(acc, __fmul_rn(bf16_lo(q[u].x), inv));
                        acc = sq_acc(acc, __fmul_rn(bf16_hi(q[u].x), inv));
                        acc = sq_acc(acc, __fmul_rn(bf16_lo(q[u].y), inv));
                        acc = sq_acc(acc, __fmul_rn(bf16_hi(q[u].y), inv));
                    }
                }
                for (; i < nv; i += kThreads) {
                    const uint2 q = __ldg(g4 + i);
                    acc = sq_acc(acc, __fmul_rn(bf16_lo(q.x), inv));
                    acc = sq_acc(acc, __fmul_rn(bf16_hi(q.x), inv));
                    acc = sq_acc(acc, __fmul_rn(bf16_lo(q.y), inv));
                    acc = sq_acc(acc, __fmul_rn(bf16_hi(q.y), inv));
                }
            } else {
                const float4* g4 = static_cast<const float4*>(gp);
                uint32_t i = threadIdx.x;
                for (; i + 3 * kThreads < nv; i += 4 * kThreads) {
                    float4 q[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) q[u] = __ldg(g4 + i + u * kThreads);
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        acc = sq_acc(acc, __fmul_rn(q[u].x, inv));
                        acc = sq_acc(acc, __fmul_rn(q[u].y, inv));
                        acc = sq_acc(acc, __fmul_rn(q[u].z, inv));
                        acc = sq_acc(acc, __fmul_rn(q[u].w, inv));
                    }
                }
                for (; i < nv; i += kThreads) {
                    const float4 q = __ldg(g4 + i);
                    acc = sq_acc(acc, __fmul_rn(q.x, inv));
                    acc = sq_acc(acc, __fmul_rn(q.y, inv));
                    acc = sq_acc(acc, __fmul_rn(q.z, inv));
                    acc = sq_acc(acc, __fmul_rn(q.w, inv));
                }
            }
        }
        for (uint32_t i = scalar_from + threadIdx.x; i < n; i += kThreads) {
            const float g = kBf16 ? bf16_bits_to_f32(static_cast<const uint16_t*>(gp)[i])
                                  : static_cast<const float*>(gp)[i];
            acc = sq_acc(acc, __fmul_rn(g, inv));
        }
    }

    const double block_total = block_sum(acc, s_red);
    if (threadIdx.x == 0) {
        partials[blockIdx.x] = block_total;
        __threadfence();
        const unsigned prev = atomicAdd(&ctl->ticket_sumsq, 1u);
        s_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    // Last CTA: fold the per-CTA partials in a fixed order (deterministic).
    __threadfence();
    double s = 0.0;
    for (int i = threadIdx.x; i < static_cast<int>(gridDim.x); i += kThreads) s += __ldcg(partials + i);
    const double total = block_sum(s, s_red);
    if (threadIdx.x == 0) {
        *out = total;
        ctl->ticket_sumsq = 0u;
    }
}

// ------------------------------------------------------------------ K2 -------

struct Coeffs {
    float inv;        // 1 / loss scale
    float coef;       // clip coefficient (1: no clip)
    float beta1, omb1, beta2, omb2, eps;
    float step_size;  // lr / bias_correction1
    float sqrt_bc2;
    float lr;
};

// One element of AdamW::step (adamw.cpp:151-166) on an unscaled, clipped grad.
__device__ __forceinline__ void adamw_elem(float& th, float& m, float& v, float g,
                                           const Coeffs& k, float lr_wd, bool has_wd) {
    if (has_wd) th = __fsub_rn(th, __fmul_rn(lr_wd, th));
    m = __fadd_rn(__fmul_rn(k.beta1, m), __fmul_rn(k.omb1, g));
    v = __fadd_rn(__fmul_rn(k.beta2, v), __fmul_rn(__fmul_rn(k.omb2, g), g));
    const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), k.sqrt_bc2), k.eps);
    th = __fsub_rn(th, __fmul_rn(k.step_size, __fdiv_rn(m, denom)));
}

// Unscale (exact for power-of-two scales) then clip (adamw.cpp:108-110).
__device__ __forceinline__ float prep_grad(float graw, const Coeffs& k) {
    return __fmul_rn(__fmul_rn(graw, k.inv), k.coef);
}

constexpr int kApplyUnroll = 2;

template <bool kMixed>
__device__ __forceinline__ void apply_chunk(const Chunk& ch, const Coeffs& k) {
    const uint32_t n = ch.n;
    const float lr_wd = __fmul_rn(k.lr, ch.wd);
    const bool has_wd = ch.wd != 0.0f;
    uint32_t scalar_from = 0;
    if (ch.flags & kChunkVec) {
        const uint32_t nv = n >> 2;
        scalar_from = nv << 2;
        float4* ms4 = reinterpret_cast<float4*>(ch.master);
        float4* m4 = reinterpret_cast<float4*>(ch.m);
        float4* v4 = reinterpret_cast<float4*>(ch.v);
        for (uint32_t base = threadIdx.x; base < nv; base += kApplyUnroll * kThreads) {
            float4 th[kApplyUnroll], mm[kApplyUnroll], vv[kApplyUnroll], gg[kApplyUnroll];
#pragma unroll
            for (int u = 0; u < kApplyUnroll; ++u) {
                const uint32_t i = base + u * kThreads;
                if (i < nv) {
                    if constexpr (kMixed) {
                        const uint2 q = __ldcs(static_cast<const uint2*>(ch.grad) + i);
                        gg[u] = make_float4(bf16_lo(q.x), bf16_hi(q.x), bf16_lo(q.y), bf16_hi(q.y));
                    } else {
                        gg[u] = __ldcs(static_cast<const float4*>(ch.grad) + i);
                    }
                    th[u] = __ldcs(ms4 + i);
                    mm[u] = __ldcs(m4 + i);
                    vv[u] = __ldcs(v4 + i);
                }
            }
#pragma unroll
            for (int u = 0; u < kApplyUnroll; ++u) {
                const uint32_t i = base + u * kThreads;
                if (i < nv) {
                    adamw_elem(th[u].x, mm[u].x, vv[u].x, prep_grad(gg[u].x, k), k, lr_wd, has_wd);
                    adamw_elem(th[u].y, mm[u].y, vv[u].y, prep_grad(gg[u].y, k), k, lr_wd, has_wd);
                    adamw_elem(th[u].z, mm[u].z, vv[u].z, prep_grad(gg[u].z, k), k, lr_wd, has_wd);
                    adamw_elem(th[u].w, mm[u].w, vv[u].w, prep_grad(gg[u].w, k), k, lr_wd, has_wd);
                    __stcs(ms4 + i, th[u]);
                    __stcs(m4 + i, mm[u]);
                    __stcs(v4 + i, vv[u]);
                    if constexpr (kMixed) {
                        uint2 p;
                        p.x = pack_bf16x2_rn(th[u].x, th[u].y);
                        p.y = pack_bf16x2_rn(th[u].z, th[u].w);
                        reinterpret_cast<uint2*>(ch.param)[i] = p;
                    }
                }
            }
        }
    }
    for (uint32_t i = scalar_from + threadIdx.x; i < n; i += kThreads) {
        const float graw = kMixed ? bf16_bits_to_f32(static_cast<const uint16_t*>(ch.grad)[i])
                                  : static_cast<const float*>(ch.grad)[i];
        float th = ch.master[i], m = ch.m[i], v = ch.v[i];
        adamw_elem(th, m, v, prep_grad(graw, k), k, lr_wd, has_wd);
        ch.master[i] = th;
        ch.m[i] = m;
        ch.v[i] = v;
        if constexpr (kMixed) static_cast<uint16_t*>(ch.param)[i] = f32_to_bf16_rn(th);
    }
}

template <bool kMixed>
__global__ void __launch_bounds__(kThreads)
k_apply(const Chunk* __restrict__ chunks, int n_chunks, Ctl* __restrict__ ctl, ApplyArgs a) {
    __shared__ Coeffs s_k;
    __shared__ int s_skip;
    __shared__ uint64_t s_t;
    __shared__ float s_norm;
    __shared__ int s_found;
    if (threadIdx.x == 0) {
        // Every CTA derives the same decision from the same bits; counters are
        // only read here and only written by the last CTA below.
        int skip = 0, found = 0;
        float norm = 0.0f, coef = a.pending_coef;
        if (a.n_parts > 0) {
            double s = 0.0;
            for (int p = 0; p < a.n_parts; ++p) s += a.parts[p];
            found = !isfinite(s);
            norm = __double2float_rn(__dsqrt_rn(s));  // adamw.cpp:101
            if (a.use_scaler && found) skip = 1;
            // adamw.cpp:102-103: no eps, no min(1, .)
            if (a.max_norm > 0.0f && norm > a.max_norm && norm > 1e-6f)
                coef = __fdiv_rn(a.max_norm, norm);
        }
        const uint64_t t = ctl->t + (skip ? 0u : 1u);
        const uint64_t ti = t < a.bc_len ? t : static_cast<uint64_t>(a.bc_len - 1);
        const float2 bc = a.bc[ti];
        Coeffs k;
        k.inv = a.use_scaler ? __fdiv_rn(1.0f, ctl->scale) : 1.0f;
        k.coef = coef;
        k.beta1 = a.beta1;
        k.omb1 = __fsub_rn(1.0f, a.beta1);
        k.beta2 = a.beta2;
        k.omb2 = __fsub_rn(1.0f, a.beta2);
        k.eps = a.eps;
        k.step_size = __fdiv_rn(a.lr, bc.x);  // adamw.cpp:130
        k.sqrt_bc2 = bc.y;
        k.lr = a.lr;
        s_k = k;
        s_skip = skip;
        s_t = t;
        s_norm = norm;
        s_found = found;
    }
    __syncthreads();
    const Coeffs k = s_k;
    if (!s_skip) {
        for (int c = n_chunks - 1 - static_cast<int>(blockIdx.x); c >= 0; c -= gridDim.x) {
            apply_chunk<kMixed>(chunks[c], k);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(&ctl->ticket_apply, 1u);
        if (prev == gridDim.x - 1) {
            // Last CTA: every CTA has read the counters; commit the step.
            ctl->t = s_t;
            ctl->last_norm = s_norm;
            ctl->last_found_inf = s_found;
            ctl->last_clip_coef = s_skip ? 1.0f : k.coef;
            ctl->last_lr = a.lr;
            if (s_skip) ctl->skipped += 1u;
            if (a.use_scaler) {
                if (s_skip) {
                    ctl->scale = __fmul_rn(ctl->scale, a.backoff);
                    ctl->tracker = 0;
                } else {
                    const int32_t tr = ctl->tracker + 1;
                    if (tr == a.interval) {
                        ctl->scale = __fmul_rn(ctl->scale, a.growth);
                        ctl->tracker = 0;
                    } else {
                        ctl->tracker = tr;
                    }
                }
            }
            ctl->ticket_apply = 0u;
        }
    }
}

// ------------------------------------------------------------ small kernels --

// In-place fp32 clip of the gradients (adamw.cpp:104-110).
__global__ void __launch_bounds__(kThreads)
k_scale_grads_f32(const Chunk* __restrict__ chunks, int n_chunks, float coef) {
    for (int c = blockIdx.x; c < n_chunks; c += gridDim.x) {
        float* g = static_cast<float*>(const_cast<void*>(chunks[c].grad));
        const uint32_t n = chunks[c].n;
        for (uint32_t i = threadIdx.x; i < n; i += kThreads) g[i] = __fmul_rn(g[i], coef);
    }
}

__global__ void k_bf16_to_f32(const uint16_t* __restrict__ src, float* __restrict__ dst,
                              uint64_t n) {
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        dst[i] = bf16_bits_to_f32(src[i]);
}

__global__ void k_set_counters(Ctl* ctl, uint64_t t, uint64_t skipped, float scale,
                               int32_t tracker) {
    ctl->t = t;
    ctl->skipped = skipped;
    ctl->scale = scale;
    ctl->tracker = tracker;
}

}  // namespace

// --------------------------------------------------------------- launchers --

cudaError_t launch_grad_sumsq(bool bf16, const Chunk* chunks, int n_chunks, Ctl* ctl,
                              double* partials, int grid, int use_scaler, double* out,
                              cudaStream_t stream) {
    if (bf16)
        k_grad_sumsq<true><<<grid, kThreads, 0, stream>>>(chunks, n_chunks, ctl, partials,
                                                          use_scaler, out);
    else
        k_grad_sumsq<false><<<grid, kThreads, 0, stream>>>(chunks, n_chunks, ctl, partials,
                                                           use_scaler, out);
    return cudaGetLastError();
}

cudaError_t launch_apply(bool mixed, const Chunk* chunks, int n_chunks, Ctl* ctl,
                         const ApplyArgs& args, int grid, cudaStream_t stream) {
    if (mixed)
        k_apply<true><<<grid, kThreads, 0, stream>>>(chunks, n_chunks, ctl, args);
    else
        k_apply<false><<<grid, kThreads, 0, stream>>>(chunks, n_chunks, ctl, args);
    return cudaGetLastError();
}

cudaError_t launch_scale_grads_f32(const Chunk* chunks, int n_chunks, float coef, int grid,
                                   cudaStream_t stream) {
    k_scale_grads_f32<<<grid, kThreads, 0, stream>>>(chunks, n_chunks, coef);
    return cudaGetLastError();
}

cudaError_t launch_bf16_to_f32(const uint16_t* src, float* dst, uint64_t n,
                               cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    uint64_t blocks = (n + kThreads - 1) / kThreads;
    if (blocks > 4096) blocks = 4096;
    k_bf16_to_f32<<<static_cast<unsigned>(blocks), kThreads, 0, stream>>>(src, dst, n);
    return cudaGetLastError();
}

cudaError_t launch_set_counters(Ctl* ctl, uint64_t t, uint64_t skipped, float scale,
                                int32_t tracker, cudaStream_t stream) {
    k_set_counters<<<1, 1, 0, stream>>>(ctl, t, skipped, scale, tracker);
    return cudaGetLastError();
}

int occupancy_grad_sumsq(bool bf16) {
    int n = 0;
    if (bf16)
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_grad_sumsq<true>, kThreads, 0);
    else
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_grad_sumsq<false>, kThreads, 0);
    return n > 0 ? n : 1;
}

int occupancy_apply(bool mixed) {
    int n = 0;
    if (mixed)
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_apply<true>, kThreads, 0);
    else
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_apply<false>, kThreads, 0);
    return n > 0 ? n : 1;
}

}  // namespace soarb
