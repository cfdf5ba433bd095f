// NVLink rate probe for the fused data-parallel step: the raw throughput of
// its two peer-memory access patterns, with no arithmetic, on symmetric
// buffers. It is the measured denominator of the fused kernels' NVLink
// roofline (the bench reports k_rs_sumsq against `pull` and the all-gather of
// k_apply against `push`).
//
//   pull  every rank bulk-loads (cp.async.bulk, no multicast) its own slice
//         [rank * B, (rank + 1) * B) of every peer's buffer into a shared-memory
//         ring, tile by tile across the grid -- k_rs_sumsq's read pattern.
//   push  every rank bulk-stores a zero tile into its slice of every peer's
//         buffer, tile by tile -- k_apply<all-gather>'s write pattern.
//
// All ranks run it at once, so each GPU's links carry both directions, as in
// the step. Every wait is bounded (1 s) and reported through `err`.
//
// A measurement tool, not part of the optimizer library: it builds into its
// own library (libsoar_probe.so), declared in bench_probe.h, which only the
// bench loads.
#include <cstdint>
#include <string>

#include <cuda_runtime.h>

#include "bench_probe.h"
#include "optim_kernels.cuh"
#include "pipeline.cuh"

namespace soarb {
namespace {

thread_local std::string g_probe_error;
void record_error(const std::string& msg) { g_probe_error = msg; }

constexpr int kProbeMaxStages = 8;
constexpr size_t kProbeMaxSmem = 200 * 1024;

struct ProbePeers {
    char* base[kMaxRanks];
};

__global__ void k_probe_pull(ProbePeers peers, int world, int rank, uint64_t bytes_per_peer,
                             uint32_t tile, int stages, int* err) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t full[kProbeMaxStages];
    __shared__ int s_err;
    if (threadIdx.x != 0) return;
    s_err = 0;
    for (int s = 0; s < stages; ++s) mbar_init(smem_u32(&full[s]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint64_t n_tiles = bytes_per_peer / tile;
    const uint32_t stage_bytes = tile * static_cast<uint32_t>(world - 1);
    uint32_t q = 0;
    for (uint64_t i = blockIdx.x; i < n_tiles; i += gridDim.x, ++q) {
        const uint32_t s = q % stages;
        if (q >= static_cast<uint32_t>(stages) &&
            !mbar_wait(smem_u32(&full[s]), ((q / stages) - 1) & 1, &s_err))
            break;
        mbar_expect_tx(smem_u32(&full[s]), stage_bytes);
        uint32_t k = 0;
        for (int r = 0; r < world; ++r) {
            if (r == rank) continue;
            bulk_load(smem_u32(smem + s * stage_bytes + k * tile),
                      peers.base[r] + rank * bytes_per_peer + i * tile, tile, smem_u32(&full[s]));
            ++k;
        }
    }
    // let every load in flight land before the CTA exits
    for (uint32_t j = q > static_cast<uint32_t>(stages) ? q - stages : 0; j < q; ++j)
        mbar_wait(smem_u32(&full[j % stages]), (j / stages) & 1, &s_err);
    if (s_err) atomicOr(err, 1);
}

__global__ void k_probe_push(ProbePeers peers, int world, int rank, uint64_t bytes_per_peer,
                             uint32_t tile) {
    extern __shared__ __align__(128) unsigned char smem[];
    for (uint32_t b = threadIdx.x * 16u; b < tile; b += blockDim.x * 16u)
        *reinterpret_cast<uint4*>(smem + b) = make_uint4(0u, 0u, 0u, 0u);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (threadIdx.x != 0) return;
    const uint64_t n_tiles = bytes_per_peer / tile;
    for (uint64_t i = blockIdx.x; i < n_tiles; i += gridDim.x) {
        for (int r = 0; r < world; ++r)
            if (r != rank) bulk_store(peers.base[r] + rank * bytes_per_peer + i * tile, smem_u32(smem), tile);
        bulk_commit();
        bulk_wait_read_all();  // as k_apply: the tile's source is released after each tile
    }
    bulk_wait_all();
}

}  // namespace
}  // namespace soarb

extern "C" SOAR_PROBE_API const char* soar_probe_last_error(void) {
    return soarb::g_probe_error.c_str();
}

extern "C" SOAR_PROBE_API int soar_nvlink_probe(void* const* bases, int world, int rank,
                                          uint64_t bytes_per_peer, int mode, uint32_t tile_bytes,
                                          int stages, int grid, int* d_err, void* stream) {
    using namespace soarb;
    if (!bases || !d_err || world < 2 || world > kMaxRanks || rank < 0 || rank >= world ||
        grid < 1 || (mode != 0 && mode != 1)) {
        record_error("soar_nvlink_probe: bad argument");
        return -1;
    }
    if (tile_bytes == 0 || tile_bytes % 16 || bytes_per_peer % tile_bytes) {
        record_error("soar_nvlink_probe: tile_bytes must be a nonzero multiple of 16 dividing "
                     "bytes_per_peer");
        return -1;
    }
    ProbePeers p{};
    for (int r = 0; r < world; ++r) {
        if (!bases[r] || reinterpret_cast<uintptr_t>(bases[r]) % 16) {
            record_error("soar_nvlink_probe: null or unaligned buffer");
            return -1;
        }
        p.base[r] = static_cast<char*>(bases[r]);
    }
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (mode == 0) {
        const size_t smem = static_cast<size_t>(stages) * tile_bytes * (world - 1);
        if (stages < 1 || stages > kProbeMaxStages || smem > kProbeMaxSmem) {
            record_error("soar_nvlink_probe: stages x tile x (world - 1) exceeds the ring");
            return -1;
        }
        e = cudaFuncSetAttribute(k_probe_pull, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        if (e == cudaSuccess) {
            k_probe_pull<<<grid, 32, smem, s>>>(p, world, rank, bytes_per_peer, tile_bytes, stages,
                                                d_err);
            e = cudaGetLastError();
        }
    } else {
        if (tile_bytes > kProbeMaxSmem) {
            record_error("soar_nvlink_probe: tile exceeds shared memory");
            return -1;
        }
        e = cudaFuncSetAttribute(k_probe_push, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(tile_bytes));
        if (e == cudaSuccess) {
            k_probe_push<<<grid, 128, tile_bytes, s>>>(p, world, rank, bytes_per_peer, tile_bytes);
            e = cudaGetLastError();
        }
    }
    if (e != cudaSuccess) {
        record_error(std::string("soar_nvlink_probe: ") + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}
