// Fused ZeRO-1 data-parallel step over peer memory (one process per GPU).
//
// Every rank allocates its flat bf16 parameter and gradient buffers with
// soar_ipc_alloc and opens the peers' buffers with soar_ipc_open (CUDA IPC over
// NVLink / NVSwitch), so all R buffers are addressable from every GPU at the
// same element offsets. Rank r owns the slice [own_start, own_start + n) of
// every bucket. A step is:
//
//   k_rs_sumsq   the reduce-scatter fused with the norm pass: for every tile of
//                the owned slices, one producer thread bulk-loads (1D
//                cp.async.bulk, no multicast) the tile from all R gradient
//                buffers -- R-1 of them across NVLink -- into a shared-memory
//                ring; consumer warps add them in fp32 in rank order, multiply
//                by 1/R once and round to bf16 once (deterministic, identical
//                to the oracle's reduce), write the result back into the local
//                buffer in place (bulk store) and accumulate the fp64 sum of
//                squares of the unscaled result. Each remote tile crosses
//                NVLink once.
//   (1-element all-gather of the R partial sums)
//   k_apply<ag>  the fused update of the owned slices (optim_kernels.cu), whose
//                bulk stores also write each updated bf16 param tile into every
//                peer's parameter buffer: the all-gather.
//
// Ordering across GPUs takes three synchronisation points: before k_rs_sumsq
// (every rank's gradients are complete), after it (every rank is done reading
// peer gradients; the partial sums are exchanged) and after the update (every
// peer's parameter writes landed). Two ways to provide them:
//   * caller-synchronised (soar_zero1_reduce_sumsq / soar_zero1_apply_allgather):
//     small collectives issued by the caller between the launches; no kernel
//     waits on another GPU.
//   * device-synchronised (soar_zero1_set_signals + soar_zero1_step): epoch
//     flags in a per-rank signal block of symmetric memory. Every CTA of
//     k_rs_sumsq publishes ready[rank] = epoch into every peer's block
//     (system-scope release stores) and waits for all ready flags in its own
//     block; its last CTA writes the rank's partial into every peer's
//     parts[rank], then part_flag[rank], waits for all part flags and leaves
//     the R partials, in rank order, where k_apply reads them. After k_apply
//     (whose peer stores are complete and fenced when it exits) a one-thread
//     kernel publishes done[rank] and waits for all done flags. Every wait
//     polls local memory, is bounded (1 s, then the handle's error flag is set
//     and the update skips the step) and waits only on flags that are
//     published before the publisher itself waits, so no wait depends on
//     co-residency and none can form a cycle.
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/soar_optim.h"
#include "optim_kernels.cuh"
#include "pipeline.cuh"

namespace soarb {
void record_error(const std::string& msg);  // optim_capi.cu
int optim_apply_allgather(void* optim, const double* parts, int n_parts, cudaStream_t stream,
                          const AgArgs& ag, const int* skip_if);
bool optim_tensor_info(void* optim, int index, void** param, void** grad, uint64_t* numel,
                       bool* mixed, Ctl** ctl, int* device);
}  // namespace soarb

namespace soarb {
namespace {

int fail(const std::string& m) {
    record_error(m);
    return SOAR_ERROR;
}

#define Z1_CUDA_TRY(expr)                                                                     \
    do {                                                                                      \
        cudaError_t e_ = (expr);                                                              \
        if (e_ != cudaSuccess) return fail(std::string(#expr) + ": " + cudaGetErrorString(e_)); \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        ok = (prev == dev) || (cudaSetDevice(dev) == cudaSuccess);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

#ifndef SOAR_RS_TILE
#define SOAR_RS_TILE 2048
#endif
#ifndef SOAR_RS_SMEM_KB
#define SOAR_RS_SMEM_KB 96
#endif
constexpr int kRsTile = SOAR_RS_TILE;   // bf16 elements per tile (4 KB per rank)
constexpr int kRsConsumerWarps = 8;     // 256 consumer threads, 8 elements each per tile
constexpr int kRsThreads = (kRsConsumerWarps + 1) * 32;
constexpr size_t kRsSmemBudget = SOAR_RS_SMEM_KB * 1024;  // ring of stages, per CTA
static_assert(kRsTile % 8 == 0 && kRsSmemBudget <= 200 * 1024, "reduce-scatter ring shape");

// One contiguous run of an owned slice: element offset in the flat buffers.
struct __align__(16) RsChunk {
    uint64_t off;
    uint32_t n;
    uint32_t vec;   // 1: every source and the destination are 16-byte aligned
};

struct RsArgs {
    Signals* sig[kMaxRanks];         // device-synchronised step (nullptr: caller-synchronised)
    uint64_t epoch;
    double* parts_out;               // (device sync) the R partials in rank order, for k_apply
    int* abort_out;                  // (device sync) 1: the step must be skipped
    const uint16_t* src[kMaxRanks];  // every rank's flat gradient buffer
    uint16_t* dst;                   // this rank's flat gradient buffer (reduced in place)
    int world;
    int rank;
    float inv_world;                 // 1.0f / world, rounded as the oracle's
    int use_scaler;
    int stages;
    uint32_t stage_bytes;            // world * kRsTile * 2
};

__device__ __forceinline__ double sq_acc_f(double acc, float g) {
    const double d = static_cast<double>(g);
    return fma(d, d, acc);
}

__device__ __forceinline__ double block_sum_rs(double x, double* smem) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) smem[warp] = x;
    __syncthreads();
    double r = 0.0;
    if (warp == 0) {
        r = lane < (kRsThreads / 32) ? smem[lane] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    }
    __syncthreads();
    return r;
}

// Reduced value of one element: fp32 sum in rank order, one multiply, one rounding.
__device__ __forceinline__ uint16_t reduce_scalar(const RsArgs& a, uint64_t e) {
    float s = 0.0f;
    for (int q = 0; q < a.world; ++q) s = __fadd_rn(s, bf16_bits_to_f32(a.src[q][e]));
    return f32_to_bf16_rn(__fmul_rn(s, a.inv_world));
}

__global__ void __launch_bounds__(kRsThreads, 1)
k_rs_sumsq(const RsChunk* __restrict__ chunks, int n_chunks, int n_vec, RsArgs a,
           const Ctl* __restrict__ ctl, double* __restrict__ partials,
           uint32_t* __restrict__ ticket, int* __restrict__ err, double* __restrict__ out) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int kMaxStages = 8;
    __shared__ __align__(8) uint64_t full_bar[kMaxStages], empty_bar[kMaxStages];
    __shared__ double s_red[32];
    __shared__ int s_err, s_drain_err, s_last, s_abort;
    __shared__ int s_cfail[2];
    __shared__ uint32_t s_issued;
    constexpr int kConsumers = kRsConsumerWarps * 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = a.stages;
    pdl_wait();
    pdl_trigger();
    const float inv = a.use_scaler ? __fdiv_rn(1.0f, ctl->scale) : 1.0f;
    if (threadIdx.x == 0) {
        s_err = s_drain_err = 0;
        s_cfail[0] = s_cfail[1] = 0;
        s_issued = 0;
        s_abort = 0;
        if (a.sig[0]) {
            // this rank's gradients are complete (stream order): tell every
            // peer, then wait for every peer's
            asm volatile("fence.acq_rel.sys;" ::: "memory");
            for (int q = 0; q < a.world; ++q) st_release_sys(&a.sig[q]->ready[a.rank], a.epoch);
            if (!wait_flags(a.sig[a.rank]->ready, a.world, a.epoch, err)) s_abort = 1;
        }
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    double acc = 0.0;
    // tile sequence: vector chunks from the end, grid-strided, kRsTile pieces
    auto for_each_tile = [&](auto&& f) {
        uint32_t q = 0;
        for (int c = n_vec - 1 - static_cast<int>(blockIdx.x); c >= 0; c -= gridDim.x) {
            const RsChunk ch = chunks[c];
            for (uint32_t t0 = 0; t0 < ch.n; t0 += kRsTile, ++q)
                if (!f(ch, t0, min(static_cast<uint32_t>(kRsTile), ch.n - t0), q)) return;
        }
    };

    if (s_abort) {
        // a peer never arrived: read no peer memory (nothing is reduced)
    } else if (warp == kRsConsumerWarps) {
        if (lane == 0) {
            for_each_tile([&](const RsChunk& ch, uint32_t t0, uint32_t len, uint32_t q) {
                const uint32_t s = q % S;
                if (q >= static_cast<uint32_t>(S) &&
                    !mbar_wait(smem_u32(&empty_bar[s]), ((q / S) + 1) & 1, &s_err))
                    return false;
                const uint32_t lv = len & ~7u;
                const uint32_t fb = smem_u32(&full_bar[s]);
                mbar_expect_tx(fb, 2u * lv * a.world);
                if (lv) {
                    const uint32_t base = smem_u32(smem + s * a.stage_bytes);
                    for (int r = 0; r < a.world; ++r)
                        bulk_load(base + r * (2u * kRsTile), a.src[r] + ch.off + t0, 2u * lv, fb);
                }
                s_issued = q + 1;
                return true;
            });
        }
    } else {
        const uint32_t tid = threadIdx.x;
        for_each_tile([&](const RsChunk& ch, uint32_t t0, uint32_t len, uint32_t q) {
            const uint32_t s = q % S;
            const bool ok = mbar_wait(smem_u32(&full_bar[s]), (q / S) & 1, &s_err);
            if (!ok) s_cfail[q & 1] = 1;
            const uint32_t lv = len & ~7u;
            unsigned char* st = smem + s * a.stage_bytes;
            if (ok) {
                const uint32_t nv = lv >> 3;  // 8 bf16 per 16-byte vector
                for (uint32_t i = tid; i < nv; i += kConsumers) {
                    float sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                    for (int r = 0; r < a.world; ++r) {
                        const uint4 w = reinterpret_cast<const uint4*>(st + r * (2u * kRsTile))[i];
                        sum[0] = __fadd_rn(sum[0], bf16_lo(w.x));
                        sum[1] = __fadd_rn(sum[1], bf16_hi(w.x));
                        sum[2] = __fadd_rn(sum[2], bf16_lo(w.y));
                        sum[3] = __fadd_rn(sum[3], bf16_hi(w.y));
                        sum[4] = __fadd_rn(sum[4], bf16_lo(w.z));
                        sum[5] = __fadd_rn(sum[5], bf16_hi(w.z));
                        sum[6] = __fadd_rn(sum[6], bf16_lo(w.w));
                        sum[7] = __fadd_rn(sum[7], bf16_hi(w.w));
                    }
                    uint4 o;
                    o.x = pack_bf16x2_rn(__fmul_rn(sum[0], a.inv_world), __fmul_rn(sum[1], a.inv_world));
                    o.y = pack_bf16x2_rn(__fmul_rn(sum[2], a.inv_world), __fmul_rn(sum[3], a.inv_world));
                    o.z = pack_bf16x2_rn(__fmul_rn(sum[4], a.inv_world), __fmul_rn(sum[5], a.inv_world));
                    o.w = pack_bf16x2_rn(__fmul_rn(sum[6], a.inv_world), __fmul_rn(sum[7], a.inv_world));
                    acc = sq_acc_f(acc, __fmul_rn(bf16_lo(o.x), inv));
                    acc = sq_acc_f(acc, __fmul_rn(bf16_hi(o.x), inv));
                    acc = sq_acc_f(acc, __fmul_rn(bf16_lo(o.y), inv));
                    acc = sq_acc_f(acc, __fmul_rn(bf16_hi(o.y), inv));
                    acc = sq_acc_f(acc, __fmul_rn(bf16_lo(o.z), inv));
                    acc = sq_acc_f(acc, __fmul_rn(bf16_hi(o.z), inv));
                    acc = sq_acc_f(acc, __fmul_rn(bf16_lo(o.w), inv));
                    acc = sq_acc_f(acc, __fmul_rn(bf16_hi(o.w), inv));
                    // the result takes this rank's slot of the stage
                    reinterpret_cast<uint4*>(st + a.rank * (2u * kRsTile))[i] = o;
                }
                // the < 16-byte tail of the tile: plain loads (peer memory included)
                for (uint32_t e = lv + tid; e < len; e += kConsumers) {
                    const uint64_t idx = ch.off + t0 + e;
                    const uint16_t r = reduce_scalar(a, idx);
                    a.dst[idx] = r;
                    acc = sq_acc_f(acc, __fmul_rn(bf16_bits_to_f32(r), inv));
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            consumers_sync<kConsumers>();
            if (s_cfail[q & 1]) return false;
            if (tid == 0) {
                if (lv) {
                    bulk_store(a.dst + ch.off + t0,
                               smem_u32(st + a.rank * (2u * kRsTile)), 2u * lv);
                    bulk_commit();
                    bulk_wait_read_all();
                }
                mbar_arrive(smem_u32(&empty_bar[s]));
            }
            return true;
        });
        if (tid == 0) bulk_wait_all();
        // scalar runs (heads before 16-byte alignment)
        if (!s_err) {
            for (int c = n_vec + static_cast<int>(blockIdx.x); c < n_chunks; c += gridDim.x) {
                const RsChunk ch = chunks[c];
                for (uint32_t e = tid; e < ch.n; e += kConsumers) {
                    const uint64_t idx = ch.off + e;
                    const uint16_t r = reduce_scalar(a, idx);
                    a.dst[idx] = r;
                    acc = sq_acc_f(acc, __fmul_rn(bf16_bits_to_f32(r), inv));
                }
            }
        }
    }
    __syncthreads();
    if (s_err && threadIdx.x == kRsConsumerWarps * 32) {
        const uint32_t qi = s_issued;
        for (uint32_t j = qi > static_cast<uint32_t>(S) ? qi - S : 0; j < qi; ++j)
            mbar_wait(smem_u32(&full_bar[j % S]), (j / S) & 1, &s_drain_err);
        atomicOr(err, 1);
    }
    // grid reduction of the sum of squares (last CTA folds in fixed order)
    const double total = block_sum_rs(acc, s_red);
    if (threadIdx.x == 0) {
        partials[blockIdx.x] = total;
        __threadfence();
        s_last = (atomicAdd(ticket, 1u) == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    double sum = 0.0;
    for (int i = threadIdx.x; i < static_cast<int>(gridDim.x); i += kRsThreads)
        sum += __ldcg(partials + i);
    const double all = block_sum_rs(sum, s_red);
    if (threadIdx.x == 0) {
        *out = all;
        *ticket = 0u;
        if (a.sig[0]) {
            // Every CTA is done reading peer gradients: publish the partial
            // (withheld after a failed wait, so the peers time out and skip),
            // then collect every rank's.
            int ok = *static_cast<volatile int*>(err) == 0;
            if (ok) {
                for (int q = 0; q < a.world; ++q) st_relaxed_sys_f64(&a.sig[q]->parts[a.rank], all);
                for (int q = 0; q < a.world; ++q) st_release_sys(&a.sig[q]->part_flag[a.rank], a.epoch);
                ok = wait_flags(a.sig[a.rank]->part_flag, a.world, a.epoch, err);
            }
            if (ok)
                for (int q = 0; q < a.world; ++q)
                    a.parts_out[q] = ld_relaxed_sys_f64(&a.sig[a.rank]->parts[q]);
            *a.abort_out = ok ? 0 : 1;
        }
    }
}

struct Zero1 {
    void* optim = nullptr;
    int device = 0;
    int world = 1, rank = 0;
    RsArgs rs{};
    AgArgs ag{};
    RsChunk* d_chunks = nullptr;
    int n_chunks = 0, n_vec = 0;
    double* partials = nullptr;
    uint32_t* ticket = nullptr;
    int* err = nullptr;
    Ctl* ctl = nullptr;
    int grid = 1;
    size_t smem = 0;
    Signals* sig[kMaxRanks] = {};  // device-synchronised step (soar_zero1_set_signals)
    uint64_t epoch = 0;
};

}  // namespace
}  // namespace soarb

using soarb::fail;
using soarb::DeviceGuard;
using soarb::Zero1;
using soarb::kMaxRanks;
using soarb::kChunkElems;
using soarb::RsChunk;
using soarb::kRsTile;
using soarb::kRsThreads;
using soarb::kRsSmemBudget;
using soarb::k_rs_sumsq;
using soarb::optim_tensor_info;
using soarb::optim_apply_allgather;
using soarb::Signals;
using soarb::launch_step_done;

extern "C" {

SOAR_API int soar_ipc_alloc(size_t bytes, int device, void** out_ptr, void* out_handle) {
    if (!out_ptr || !out_handle || bytes == 0) return fail("bad argument");
    DeviceGuard g(device);
    if (!g.ok) return fail("cannot select device");
    void* p = nullptr;
    Z1_CUDA_TRY(cudaMalloc(&p, bytes));
    cudaError_t e = cudaMemset(p, 0, bytes);  // zero-filled (signal blocks rely on it)
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(std::string("soar_ipc_alloc: ") + cudaGetErrorString(e));
    }
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
    }
    static_assert(sizeof(h) <= SOAR_IPC_HANDLE_BYTES, "IPC handle size");
    std::memset(out_handle, 0, SOAR_IPC_HANDLE_BYTES);
    std::memcpy(out_handle, &h, sizeof h);
    *out_ptr = p;
    return SOAR_OK;
}

SOAR_API int soar_ipc_free(void* ptr, int device) {
    if (!ptr) return fail("null pointer");
    DeviceGuard g(device);
    Z1_CUDA_TRY(cudaDeviceSynchronize());
    Z1_CUDA_TRY(cudaFree(ptr));
    return SOAR_OK;
}

SOAR_API int soar_ipc_open(const void* handle, int device, void** out_peer_ptr) {
    if (!handle || !out_peer_ptr) return fail("null argument");
    DeviceGuard g(device);
    if (!g.ok) return fail("cannot select device");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof h);
    void* p = nullptr;
    Z1_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    *out_peer_ptr = p;
    return SOAR_OK;
}

SOAR_API int soar_ipc_close(void* peer_ptr, int device) {
    if (!peer_ptr) return fail("null pointer");
    DeviceGuard g(device);
    Z1_CUDA_TRY(cudaDeviceSynchronize());
    Z1_CUDA_TRY(cudaIpcCloseMemHandle(peer_ptr));
    return SOAR_OK;
}

SOAR_API int soar_zero1_create(void* optim_handle, int rank, int world,
                               void* const* grad_bases, void* const* param_bases,
                               const soar_zero1_shard* shards, int n_shards, void** out) {
    if (!optim_handle || !grad_bases || !param_bases || !out || (n_shards > 0 && !shards))
        return fail("null argument");
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
        return fail("world size must be 1.." + std::to_string(kMaxRanks));
    *out = nullptr;
    auto* z = new Zero1();
    z->optim = optim_handle;
    z->world = world;
    z->rank = rank;
    // every tensor of the optimizer is one owned slice, in shard order
    bool mixed = false;
    for (int i = 0; i < n_shards; ++i) {
        void *p = nullptr, *gr = nullptr;
        uint64_t numel = 0;
        if (!optim_tensor_info(optim_handle, shards[i].tensor, &p, &gr, &numel, &mixed, &z->ctl,
                               &z->device)) {
            delete z;
            return fail("shard " + std::to_string(i) + ": bad optimizer tensor index");
        }
        const char* want_p = static_cast<const char*>(param_bases[rank]) + 2 * shards[i].offset;
        const char* want_g = static_cast<const char*>(grad_bases[rank]) + 2 * shards[i].offset;
        if (!mixed || p != want_p || gr != want_g || numel != shards[i].count) {
            delete z;
            return fail("shard " + std::to_string(i) +
                        ": the optimizer tensor must be the bf16 slice of the local buffers "
                        "at the shard's offset");
        }
    }
    if (n_shards == 0 &&
        !optim_tensor_info(optim_handle, -1, nullptr, nullptr, nullptr, &mixed, &z->ctl,
                           &z->device)) {
        delete z;
        return fail("bad optimizer handle");
    }
    // symmetric buffers must share their alignment phase
    for (int q = 0; q < world; ++q) {
        if ((reinterpret_cast<uintptr_t>(grad_bases[q]) - reinterpret_cast<uintptr_t>(grad_bases[0])) % 16 ||
            (reinterpret_cast<uintptr_t>(param_bases[q]) - reinterpret_cast<uintptr_t>(param_bases[0])) % 16) {
            delete z;
            return fail("peer buffers differ in 16-byte alignment phase");
        }
    }
    for (int q = 0; q < world; ++q) {
        z->rs.src[q] = static_cast<const uint16_t*>(grad_bases[q]);
        z->ag.peer_param_base[q] = static_cast<char*>(param_bases[q]);
    }
    z->rs.dst = static_cast<uint16_t*>(grad_bases[rank]);
    z->rs.world = world;
    z->rs.rank = rank;
    z->rs.inv_world = 1.0f / static_cast<float>(world);
    z->ag.world = world;
    z->ag.rank = rank;
    z->ag.local_param_base = static_cast<const char*>(param_bases[rank]);

    // reduce-scatter plan: scalar head to the first 16-byte boundary, then
    // chunks cut at 2 KB-multiple grad addresses (as the optimizer's table)
    std::vector<RsChunk> vec, scal;
    const uintptr_t gbase = reinterpret_cast<uintptr_t>(grad_bases[rank]);
    for (int i = 0; i < n_shards; ++i) {
        const uint64_t off = shards[i].offset, n = shards[i].count;
        const uintptr_t ga = gbase + 2 * off;
        const uint64_t h16 = std::min<uint64_t>(((16 - ga % 16) % 16) / 2, n);
        const uint64_t ab = 2ull * kChunkElems;
        const uint64_t e0 = std::min<uint64_t>(std::max<uint64_t>(((ab - ga % ab) % ab) / 2, h16), n);
        auto run = [&](uint64_t from, uint64_t to, bool v) {
            for (uint64_t s = from; s < to; s += kChunkElems)
                (v ? vec : scal).push_back({off + s, static_cast<uint32_t>(std::min<uint64_t>(kChunkElems, to - s)), v ? 1u : 0u});
        };
        run(0, h16, false);
        run(h16, e0, true);
        run(e0, n, true);
    }
    for (const RsChunk& c : vec) {
        for (int q = 0; q < world; ++q)
            if ((reinterpret_cast<uintptr_t>(z->rs.src[q] + c.off)) % 16) {
                delete z;
                return fail("internal reduce-scatter plan check failed: unaligned vector run");
            }
    }
    z->n_vec = static_cast<int>(vec.size());
    vec.insert(vec.end(), scal.begin(), scal.end());
    z->n_chunks = static_cast<int>(vec.size());

    DeviceGuard g(z->device);
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, z->device);
    z->rs.stage_bytes = static_cast<uint32_t>(world) * kRsTile * 2u;
    z->rs.stages = static_cast<int>(std::min<size_t>(8, kRsSmemBudget / z->rs.stage_bytes));
    if (z->rs.stages < 2) z->rs.stages = 2;
    z->smem = static_cast<size_t>(z->rs.stages) * z->rs.stage_bytes;
    cudaError_t e = cudaFuncSetAttribute(k_rs_sumsq, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(z->smem));
    int occ = 0;
    if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_rs_sumsq, kRsThreads, z->smem);
    if (e != cudaSuccess) {
        delete z;
        return fail(std::string("reduce-scatter kernel set-up: ") + cudaGetErrorString(e));
    }
    z->grid = std::max(1, std::min(sms * std::max(occ, 1), std::max(1, z->n_chunks)));
    const size_t chunk_bytes = std::max<size_t>(1, vec.size()) * sizeof(RsChunk);
    e = cudaMalloc(&z->d_chunks, chunk_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&z->partials, z->grid * sizeof(double) + 256);
    if (e == cudaSuccess) e = cudaMalloc(&z->ticket, 256);
    if (e == cudaSuccess) {
        z->err = reinterpret_cast<int*>(reinterpret_cast<char*>(z->ticket) + 64);
        e = cudaMemset(z->ticket, 0, 256);
    }
    if (e == cudaSuccess && !vec.empty())
        e = cudaMemcpy(z->d_chunks, vec.data(), vec.size() * sizeof(RsChunk), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(z->d_chunks);
        cudaFree(z->partials);
        cudaFree(z->ticket);
        delete z;
        return fail(std::string("zero1 set-up: ") + cudaGetErrorString(e));
    }
    z->rs.use_scaler = 1;  // the sum of squares is of unscaled values; 1/scale is 1 without a scaler
    *out = z;
    return SOAR_OK;
}

SOAR_API int soar_zero1_reduce_sumsq(void* handle, double* d_partial, void* stream) {
    if (!handle || !d_partial) return fail("null argument");
    auto* z = static_cast<Zero1*>(handle);
    DeviceGuard g(z->device);
    Z1_CUDA_TRY(soarb::launch_pdl(k_rs_sumsq, dim3(z->grid), dim3(kRsThreads), z->smem,
                                  static_cast<cudaStream_t>(stream), z->d_chunks, z->n_chunks,
                                  z->n_vec, z->rs, z->ctl, z->partials, z->ticket, z->err,
                                  d_partial));
    Z1_CUDA_TRY(cudaGetLastError());
    return SOAR_OK;
}

SOAR_API int soar_zero1_apply_allgather(void* handle, const double* d_parts, int n_parts,
                                        void* stream) {
    if (!handle) return fail("null handle");
    auto* z = static_cast<Zero1*>(handle);
    DeviceGuard g(z->device);
    return optim_apply_allgather(z->optim, d_parts, n_parts, static_cast<cudaStream_t>(stream),
                                 z->ag, nullptr);
}

SOAR_API int soar_zero1_set_signals(void* handle, void* const* signal_bases) {
    if (!handle || !signal_bases) return fail("null argument");
    auto* z = static_cast<Zero1*>(handle);
    if (z->epoch != 0) return fail("signal blocks are set once, before the first device-synchronised step");
    for (int q = 0; q < z->world; ++q) {
        if (!signal_bases[q] || reinterpret_cast<uintptr_t>(signal_bases[q]) % alignof(Signals))
            return fail("signal block " + std::to_string(q) + " is null or not 256-byte aligned");
    }
    static_assert(sizeof(Signals) <= SOAR_ZERO1_SIGNAL_BYTES, "signal block size");
    for (int q = 0; q < z->world; ++q) z->sig[q] = static_cast<Signals*>(signal_bases[q]);
    return SOAR_OK;
}

SOAR_API int soar_zero1_step(void* handle, void* stream) {
    if (!handle) return fail("null handle");
    auto* z = static_cast<Zero1*>(handle);
    if (!z->sig[0]) return fail("soar_zero1_step needs soar_zero1_set_signals");
    DeviceGuard g(z->device);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint64_t epoch = z->epoch + 1;
    soarb::RsArgs rs = z->rs;
    for (int q = 0; q < z->world; ++q) rs.sig[q] = z->sig[q];
    rs.epoch = epoch;
    // the slack past the per-CTA partials: this rank's partial, the R
    // partials in rank order, the skip word
    double* part = z->partials + z->grid;
    rs.parts_out = part + 1;
    rs.abort_out = reinterpret_cast<int*>(part + 1 + kMaxRanks);
    Z1_CUDA_TRY(soarb::launch_pdl(k_rs_sumsq, dim3(z->grid), dim3(kRsThreads), z->smem, s,
                                  z->d_chunks, z->n_chunks, z->n_vec, rs, z->ctl, z->partials,
                                  z->ticket, z->err, part));
    Z1_CUDA_TRY(cudaGetLastError());
    const int rc = optim_apply_allgather(z->optim, rs.parts_out, z->world, s, z->ag, rs.abort_out);
    if (rc != SOAR_OK) return rc;
    Z1_CUDA_TRY(launch_step_done(z->sig, z->world, z->rank, epoch, z->err, s));
    z->epoch = epoch;
    return SOAR_OK;
}

SOAR_API int soar_zero1_error(void* handle, int* out_error) {
    if (!handle || !out_error) return fail("null argument");
    auto* z = static_cast<Zero1*>(handle);
    DeviceGuard g(z->device);
    Z1_CUDA_TRY(cudaDeviceSynchronize());
    Z1_CUDA_TRY(cudaMemcpy(out_error, z->err, sizeof(int), cudaMemcpyDeviceToHost));
    return SOAR_OK;
}

SOAR_API int soar_zero1_destroy(void* handle) {
    if (!handle) return fail("null handle");
    auto* z = static_cast<Zero1*>(handle);
    {
        DeviceGuard g(z->device);
        cudaDeviceSynchronize();
        cudaFree(z->d_chunks);
        cudaFree(z->partials);
        cudaFree(z->ticket);
    }
    delete z;
    return SOAR_OK;
}

}  // extern "C"
