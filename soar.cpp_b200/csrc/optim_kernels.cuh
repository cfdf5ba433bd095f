// Device-side data structures shared by the optimizer-step kernels and the
// host code that builds them.
#pragma once

#include <cstdint>
#include <utility>

#include <cuda_runtime.h>

namespace soarb {

// Launches `kernel` with programmatic stream serialization: it may be
// scheduled while the previous kernel on the stream drains (hiding the launch
// gap between back-to-back kernels); the kernel itself waits for that
// predecessor with griddepcontrol.wait before touching global memory.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Elements per chunk-table entry. A multiple of the tile, large enough that
// the per-chunk descriptor read (64 B) is noise next to the 28 B/element the
// update streams (458 KB per full chunk).
constexpr uint32_t kChunkElems = 16384;

// Vector alignment of a "vector" chunk: every stream starts on a 16-byte
// boundary (8 bf16 or 4 fp32 elements), as bulk async copies require.
constexpr uint32_t kVecBytes = 16;

// Chunk flag: all pointers of the chunk are 16-byte aligned at its first
// element. The host puts these chunks first in the table; the rest (short
// heads of misaligned tensors, tensors whose param and grad have different
// alignment phases) run a scalar path.
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
    int32_t error;          // nonzero: a pipeline wait timed out (the step is incomplete)
    uint32_t grab;          // chunks handed out so far by the running update (0 between launches)
};

// Per-launch arguments of the update kernel.
struct ApplyArgs {
    float lr, beta1, beta2, eps;
    float omb1, omb2;     // 1 - beta1, 1 - beta2, rounded as the reference's float expressions
    float max_norm;       // > 0: clip by the global norm
    float pending_coef;   // coefficient from a standalone clip_grad_norm (1: none)
    float growth, backoff;
    int32_t interval;
    int32_t use_scaler;
    int32_t n_parts;      // number of fp64 partial sums in `parts` (0: no norm info)
    const double* parts;  // device, n_parts partial sums (rank order)
    const int* skip_if;   // device word or nullptr: nonzero skips the step (failed peer sync)
    const float2* bc;     // device table, bc[t] = (1 - beta1^t, sqrt(1 - beta2^t)), t >= 1
    uint32_t bc_len;      // entries in bc; t >= bc_len uses bc[bc_len - 1]
    // fused weight EMA (ModelEMA::update): shadow = decay*shadow + (1-decay)*weight
    float ema_decay, ema_omd; // decay and (1 - decay) rounded as the reference's float expression
    long long ema_delta;      // element offset from a chunk's m pointer to its shadow pointer
    // SGD (the chunk's m pointer is the momentum buffer; v is unused)
    float momentum;
    float omdamp;             // 1 - dampening, rounded as the reference's float expression
    int32_t nesterov;
};

// Data-parallel all-gather fused into the update: after a tile of the rank's
// shard is updated, its params (bf16 in the mixed layout, fp32 otherwise) are
// also stored into every peer's parameter buffer at the same offset. The
// buffers are symmetric: every rank's flat parameter buffer holds the whole
// model at identical offsets.
constexpr int kMaxRanks = 8;

// Per-rank signal block in symmetric (IPC) memory for device-side step
// synchronisation. Every field is written only by the rank it is indexed by
// (system-scope release stores into each peer's block) and polled in the
// local block (acquire loads); values are step epochs, so they only grow.
struct __align__(256) Signals {
    uint64_t ready[kMaxRanks];      // ready[q] >= e: rank q's step-e gradients are complete
    uint64_t part_flag[kMaxRanks];  // part_flag[q] >= e: parts[q] holds rank q's step-e partial
    double parts[kMaxRanks];        // rank q's sum of squares
    uint64_t done[kMaxRanks];       // done[q] >= e: rank q's step-e param writes here landed
};

struct AgArgs {
    int world;
    int rank;
    const char* local_param_base;        // this rank's flat parameter buffer
    char* peer_param_base[kMaxRanks];    // every rank's flat parameter buffer (peer pointers)
};

// Update-kernel pipeline shape (measured best on B200 for the mixed layout:
// 1024-element tiles, 6 stages, 12 consumer warps + 1 producer warp, 2 CTAs/SM).
constexpr int kTile = 1024;
constexpr int kMaxStages = 6;
constexpr int kConsumerWarps = 12;
constexpr int kApplyThreads = (kConsumerWarps + 1) * 32;
// Update kernel with the fused all-gather: tiles whose stores may still be
// reading their stage while the consumers move on (0: every tile waits for
// its own stores' reads before the next).
#ifndef SOAR_AG_STORE_LAG
#define SOAR_AG_STORE_LAG 2
#endif
constexpr int kAgStoreLag = SOAR_AG_STORE_LAG;
// bytes of one pipeline stage: grad tile + master, m, v (AdamW) or master,
// momentum (SGD) tiles, + the EMA shadow tile
__host__ __device__ constexpr size_t stage_bytes(bool mixed, bool ema = false, bool sgd = false) {
    return (mixed ? 2u : 4u) * kTile + (sgd ? 8u : 12u) * kTile + (ema ? 4u : 0u) * kTile;
}
// Update kernel with the fused all-gather, bf16 params: the updated params of
// this many consecutive tiles of one chunk leave in one push per peer (from a
// double-buffered push area in shared memory, beside the ring); 0: every tile
// pushes its own params from its stage.
#ifndef SOAR_AG_PUSH_TILES
#define SOAR_AG_PUSH_TILES 8
#endif
constexpr int kAgPushTiles = SOAR_AG_PUSH_TILES;
__host__ __device__ constexpr size_t push_bytes(bool mixed, bool ag) {
    return mixed && ag && kAgPushTiles > 0 ? 2u * kAgPushTiles * kTile * 2u : 0u;
}
// stages that keep two CTAs per SM (<= ~108 KB of ring and push area each)
__host__ __device__ constexpr int apply_stages(bool mixed, bool ema = false, bool sgd = false,
                                               bool ag = false) {
    return static_cast<int>((110592 - push_bytes(mixed, ag)) / stage_bytes(mixed, ema, sgd)) <
                   kMaxStages
               ? static_cast<int>((110592 - push_bytes(mixed, ag)) / stage_bytes(mixed, ema, sgd))
               : kMaxStages;
}
static_assert(kAgStoreLag >= 0 && kAgStoreLag + 2 <= kMaxStages,
              "the producer keeps at least two stages of loads ahead");
__host__ __device__ constexpr size_t apply_smem_bytes(bool mixed, bool ema = false,
                                                      bool sgd = false, bool ag = false) {
    return stage_bytes(mixed, ema, sgd) * apply_stages(mixed, ema, sgd, ag) +
           push_bytes(mixed, ag);
}

// Register-fed update for short lists (k_apply_direct): up to kDirectMaxRuns
// runs of 16-byte-aligned elements (the vector part of each tensor), passed by
// value in the kernel parameters, so a thread's addresses need no table read
// before its loads. Vector index space: run r holds vectors [start[r],
// start[r + 1]) of 4 elements each (the last one of a run may be partial).
constexpr int kDirectMaxRuns = 4;
#ifndef SOAR_DIRECT_THREADS
#define SOAR_DIRECT_THREADS 256
#endif
#ifndef SOAR_DIRECT_VECS
#define SOAR_DIRECT_VECS 2
#endif
#ifndef SOAR_DIRECT_MIN_BLOCKS
#define SOAR_DIRECT_MIN_BLOCKS 4
#endif
constexpr int kDirectThreads = SOAR_DIRECT_THREADS;
constexpr int kDirectVecs = SOAR_DIRECT_VECS;  // 4-element vectors per thread per pass
constexpr int kDirectMinBlocks = SOAR_DIRECT_MIN_BLOCKS;
struct DirectRun {
    void* param;        // fp32* or bf16*, at the run's first element
    const void* grad;
    float* master;      // == param in the fp32 layout
    float* m;
    float* v;
    uint64_t n;         // elements in the run
    float wd;
};
struct DirectRuns {
    DirectRun run[kDirectMaxRuns];
    uint64_t start[kDirectMaxRuns + 1];  // prefix sums of the runs' vector counts
    int n_runs;
};

// Launchers (optim_kernels.cu). Each returns the launch status.
cudaError_t launch_grad_sumsq(bool bf16, const Chunk* chunks, int n_chunks, Ctl* ctl,
                              double* partials, int grid, int use_scaler, double* out,
                              cudaStream_t stream);
// ag == nullptr: plain update; otherwise the update with the fused all-gather.
// ema: also update the weight EMA shadow (args.ema_*). sgd: the SGD update
// (args.momentum/omdamp/nesterov) instead of AdamW. dyn: hand the chunks out
// dynamically (Ctl::grab) instead of the static grid-strided walk.
cudaError_t launch_apply(bool mixed, const Chunk* chunks, int n_chunks, int n_vec, Ctl* ctl,
                         const ApplyArgs& args, int grid, cudaStream_t stream,
                         const AgArgs* ag = nullptr, bool ema = false, bool sgd = false,
                         bool dyn = false);
// The register-fed update over `runs` plus the scalar chunks of the table
// (chunks[n_vec, n_chunks)): the AdamW step of k_apply without EMA, SGD or
// the fused all-gather.
cudaError_t launch_apply_direct(bool mixed, const DirectRuns& runs, const Chunk* chunks,
                                int n_chunks, int n_vec, Ctl* ctl, const ApplyArgs& args,
                                int grid, cudaStream_t stream);
int occupancy_apply_direct(bool mixed);
cudaError_t launch_scale_grads_f32(const Chunk* chunks, int n_chunks, float coef, int grid,
                                   cudaStream_t stream);
cudaError_t launch_bf16_to_f32(const uint16_t* src, float* dst, uint64_t n,
                               cudaStream_t stream);
cudaError_t launch_f32_to_bf16(const float* src, uint16_t* dst, uint64_t n,
                               cudaStream_t stream);
cudaError_t launch_set_counters(Ctl* ctl, uint64_t t, uint64_t skipped, float scale,
                                int32_t tracker, cudaStream_t stream);

// Device-synchronised end of a data-parallel step: publishes done[rank] =
// epoch into every peer's signal block, then waits (bounded) for every rank's.
cudaError_t launch_step_done(Signals* const* sig, int world, int rank, uint64_t epoch, int* err,
                             cudaStream_t stream);
cudaError_t launch_wait_selftest(uint64_t limit_ns, int* out_error, unsigned long long* out_ns,
                                 cudaStream_t stream);

// Attributes of the loaded update kernel (binaryVersion: the SASS target it
// was loaded as, 100 for sm_100a).
cudaError_t apply_kernel_attributes(cudaFuncAttributes* out);

// One-time per-process kernel attribute set-up (dynamic shared memory size).
cudaError_t prepare_kernels();

// Resident CTAs per SM of each kernel at its launch configuration.
int occupancy_grad_sumsq(bool bf16);
int occupancy_apply(bool mixed, bool ema = false, bool sgd = false);

constexpr int kThreads = 256;

}  // namespace soarb
