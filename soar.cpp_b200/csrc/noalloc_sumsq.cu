// Gradient sum of squares without any device allocation.
//
// Some callers cannot call cudaMalloc: a host runtime that reserves all of a
// GPU's memory up front in its own pool (an extra cudaMalloc either fails for
// lack of memory or escapes the pool's accounting), and latency-sensitive
// loops where cudaMalloc's implicit device-wide synchronisation would stall
// the work already in flight. soar_grad_sumsq_noalloc serves them: it is the
// global sum-of-squares reduction of k_grad_sumsq (optim_kernels.cu), but its
// scratch -- the per-CTA fp64 partials and the last-CTA ticket -- lives in a
// file-scope __device__ array instead of an optimizer's slab. Each GPU that
// loads this library holds that array (about 8 KB) until the process exits.
//
// The array is shared by every call on a device and keeps the contents of the
// last call: the ticket is cleared on the stream before each launch, and the
// partials are fully rewritten by each launch. Calls whose kernels overlap on
// the GPU (different streams without ordering between them) race on the
// array and produce wrong sums; serialise them.
#include <cstdint>
#include <mutex>
#include <string>

#include <cuda_runtime.h>

#include "../../include/soar_optim.h"

namespace soarb {
void record_error(const std::string& msg);  // optim_capi.cu
}

namespace {

constexpr int kMaxTensors = SOAR_NOALLOC_MAX_TENSORS;
constexpr int kMaxCtas = 1024;  // partials slots: 1024 x 8 B
constexpr int kThreads = 256;
constexpr int kMaxDevices = 64;

struct Scratch {
    double partials[kMaxCtas];
    unsigned int ticket;
};

// The only device memory this entry point uses.
static __device__ __align__(256) Scratch g_noalloc_scratch;

struct TensorList {
    const void* ptr[kMaxTensors];
    uint64_t numel[kMaxTensors];
    int n;
    int bf16;
    float inv_scale;
};

__device__ __forceinline__ double sq(double acc, float g) {
    const double d = static_cast<double>(g);
    return fma(d, d, acc);  // the square of a float is exact in fp64
}

__device__ __forceinline__ double block_sum(double x, double* smem) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) smem[warp] = x;
    __syncthreads();
    double r = 0.0;
    if (warp == 0) {
        r = lane < (kThreads / 32) ? smem[lane] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    }
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(kThreads)
k_grad_sumsq_noalloc(TensorList tl, Scratch* __restrict__ scratch, double* __restrict__ out) {
    __shared__ double s_red[32];
    __shared__ int s_last;
    const float inv = tl.inv_scale;
    const uint64_t tid = blockIdx.x * static_cast<uint64_t>(kThreads) + threadIdx.x;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kThreads;
    double acc = 0.0;
    for (int k = 0; k < tl.n; ++k) {
        const uint64_t n = tl.numel[k];
        const uintptr_t a = reinterpret_cast<uintptr_t>(tl.ptr[k]);
        uint64_t scalar_from = 0;
        if (tl.bf16) {
            const uint16_t* g = static_cast<const uint16_t*>(tl.ptr[k]);
            if (a % 8 == 0) {
                const uint64_t nv = n / 4;
                scalar_from = nv * 4;
                const uint2* g4 = reinterpret_cast<const uint2*>(g);
                for (uint64_t i = tid; i < nv; i += stride) {
                    const uint2 q = __ldg(g4 + i);
                    acc = sq(acc, __fmul_rn(__uint_as_float(q.x << 16), inv));
                    acc = sq(acc, __fmul_rn(__uint_as_float(q.x & 0xFFFF0000u), inv));
                    acc = sq(acc, __fmul_rn(__uint_as_float(q.y << 16), inv));
                    acc = sq(acc, __fmul_rn(__uint_as_float(q.y & 0xFFFF0000u), inv));
                }
            }
            for (uint64_t i = scalar_from + tid; i < n; i += stride)
                acc = sq(acc, __fmul_rn(__uint_as_float(static_cast<uint32_t>(g[i]) << 16), inv));
        } else {
            const float* g = static_cast<const float*>(tl.ptr[k]);
            if (a % 16 == 0) {
                const uint64_t nv = n / 4;
                scalar_from = nv * 4;
                const float4* g4 = reinterpret_cast<const float4*>(g);
                for (uint64_t i = tid; i < nv; i += stride) {
                    const float4 q = __ldg(g4 + i);
                    acc = sq(acc, __fmul_rn(q.x, inv));
                    acc = sq(acc, __fmul_rn(q.y, inv));
                    acc = sq(acc, __fmul_rn(q.z, inv));
                    acc = sq(acc, __fmul_rn(q.w, inv));
                }
            }
            for (uint64_t i = scalar_from + tid; i < n; i += stride) acc = sq(acc, __fmul_rn(g[i], inv));
        }
    }
    const double total = block_sum(acc, s_red);
    if (threadIdx.x == 0) {
        scratch->partials[blockIdx.x] = total;
        __threadfence();
        s_last = (atomicAdd(&scratch->ticket, 1u) == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    double s = 0.0;
    for (int i = threadIdx.x; i < static_cast<int>(gridDim.x); i += kThreads)
        s += __ldcg(scratch->partials + i);
    const double sum = block_sum(s, s_red);
    if (threadIdx.x == 0) {
        *out = sum;
        scratch->ticket = 0u;
    }
}

// Per-device set-up, done once by the first call on each device: the device
// address of g_noalloc_scratch (in host code the symbol's name only stands in
// for it) and the launch width. The address is cached for the life of the
// process, so it assumes the device's primary context lives as long: after a
// cudaDeviceReset the cached address no longer belongs to the new context, and
// this entry point must not be called again in that process.
struct DeviceSetup {
    Scratch* scratch = nullptr;
    int grid = 0;
};
std::mutex g_setup_mu;
DeviceSetup g_setup[kMaxDevices];

int fail(const std::string& m) {
    soarb::record_error(m);  // reported by soar_last_error()
    return SOAR_ERROR;
}

int setup_device(int dev, DeviceSetup* out) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    DeviceSetup& s = g_setup[dev];
    if (!s.scratch) {
        Scratch* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_noalloc_scratch);
        if (e != cudaSuccess)
            return fail(std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
        int sms = 0, occ = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return fail(std::string("SM count: ") + cudaGetErrorString(e));
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_grad_sumsq_noalloc, kThreads, 0);
        if (e != cudaSuccess) return fail(std::string("occupancy: ") + cudaGetErrorString(e));
        const int grid = sms * (occ > 0 ? occ : 1);
        s.grid = grid < kMaxCtas ? grid : kMaxCtas;
        s.scratch = p;
    }
    *out = s;
    return SOAR_OK;
}

}  // namespace

extern "C" SOAR_API int soar_grad_sumsq_noalloc(const void* const* grads, const uint64_t* numel,
                                                int n_tensors, int layout, float inv_scale,
                                                double* d_sumsq, void* stream) {
    if (!d_sumsq || n_tensors < 0 || (n_tensors > 0 && (!grads || !numel)))
        return fail("null argument");
    if (n_tensors > kMaxTensors)
        return fail("soar_grad_sumsq_noalloc: " + std::to_string(n_tensors) +
                    " tensors given, at most " + std::to_string(kMaxTensors) + " per call");
    if (layout != SOAR_LAYOUT_FP32 && layout != SOAR_LAYOUT_BF16_MIXED)
        return fail("unknown layout");
    TensorList tl{};
    tl.n = n_tensors;
    tl.bf16 = layout == SOAR_LAYOUT_BF16_MIXED;
    tl.inv_scale = inv_scale;
    const size_t eb = tl.bf16 ? 2 : 4;
    for (int i = 0; i < n_tensors; ++i) {
        if (numel[i] && !grads[i]) return fail("tensor " + std::to_string(i) + ": null grad");
        if (reinterpret_cast<uintptr_t>(grads[i]) % eb)
            return fail("tensor " + std::to_string(i) + ": pointer not aligned to its element size");
        tl.ptr[i] = grads[i];
        tl.numel[i] = numel[i];
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail("device ordinal out of range");
    DeviceSetup s;
    if (setup_device(dev, &s) != SOAR_OK) return SOAR_ERROR;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the ticket must start at zero; the partials are rewritten by every launch
    e = cudaMemsetAsync(&s.scratch->ticket, 0, sizeof(unsigned int), st);
    if (e != cudaSuccess) return fail(std::string("ticket clear: ") + cudaGetErrorString(e));
    k_grad_sumsq_noalloc<<<s.grid, kThreads, 0, st>>>(tl, s.scratch, d_sumsq);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail(std::string("launch: ") + cudaGetErrorString(e));
    return SOAR_OK;
}
