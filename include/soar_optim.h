/*
 * soar_optim.h -- C-ABI of the B200 (sm_100a) optimizer-step hot path.
 *
 * Drop-in for the update step of pomagrenate/soar.cpp: the reference's
 * soar::optim::AdamW / CosineAnnealingLR (include/soar/optim/adamw.hpp:10-57,
 * src/optim/adamw.cpp:7-143), which the Trainer calls as
 * clip_grad_norm(grad_clip) -> step() -> zero_grad()
 * (src/engine/trainer.cpp:157-159, 223-225). The reference exposes its engine
 * through an opaque-handle C-ABI (include/soar/api/c_api.h) bound from Python
 * with ctypes (soar/__init__.py:48-95); these entry points follow the same
 * conventions and are additive to it:
 *   - SOAR_API = default visibility (c_api.h:10-14);
 *   - opaque void* handles; int status, 0 = success, -1 = any failure or NULL
 *     argument (src/api/c_api.cpp:51, 80, 99-100, 143, 149-150);
 *   - caller-owned out-pointers;
 *   - plus a `void* stream` (a cudaStream_t; NULL = legacy default stream), the
 *     convention of the reference's kernel API (include/soar/cuda/cuda_kernels.hpp:108-127).
 * soar_last_error() returns the message of the calling thread's last failure.
 *
 * Memory: parameters and gradients are caller-owned device buffers (the model
 * owns its params, as in the reference where AdamW copies the TensorPtr list,
 * adamw.hpp:33). The optimizer owns its state -- fp32 master weights (mixed
 * layout), first and second moments -- in one device slab it allocates at
 * create time, as the reference's AdamW owns m_/v_ (adamw.hpp:38-39).
 *
 * No entry point synchronises the host except those documented as
 * synchronous (clip_grad_norm returns a value, as in the reference, and the
 * state readers copy to host memory).
 */
#ifndef SOAR_OPTIM_H
#define SOAR_OPTIM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define SOAR_API __declspec(dllexport)
#else
#define SOAR_API __attribute__((visibility("default")))
#endif

#define SOAR_OK 0
#define SOAR_ERROR (-1)

/* Storage layouts. 28 algorithmic bytes per parameter per step in both. */
enum soar_layout {
    /* fp32 params (updated in place, they are the master), fp32 grads, fp32 m/v:
       the reference's only layout (adamw.cpp:84-88). */
    SOAR_LAYOUT_FP32 = 0,
    /* bf16 params and grads, fp32 master/m/v owned by the optimizer; params are
       rewritten as round-to-nearest-even bf16 of the master every step. */
    SOAR_LAYOUT_BF16_MIXED = 1
};

/* Which optimizer-owned state array of a tensor (soar_optim_state_ptr & co). */
enum soar_state_kind {
    SOAR_STATE_MASTER = 0,
    SOAR_STATE_M = 1,
    SOAR_STATE_V = 2,
    SOAR_STATE_EMA = 3  /* weight-EMA shadow, when enabled */
};

/* One parameter tensor (the reference's TensorPtr list entry). */
typedef struct soar_tensor_desc {
    void* param;        /* device; fp32 (FP32 layout) or bf16 (BF16_MIXED) */
    void* grad;         /* device, same dtype as param. NULL: the tensor is skipped by
                           step/clip, as a param without grad is (adamw.cpp:30-31,74-75) */
    uint64_t numel;
    float weight_decay; /* this tensor's decoupled weight decay (per-param-group mask) */
} soar_tensor_desc;

/* Optimizer options. The first five fields are the reference's AdamWOptions
   (adamw.hpp:10-16, same defaults); the rest are extensions with no reference
   counterpart. Fill with soar_adamw_default_opts() first. */
typedef struct soar_adamw_opts {
    float lr;               /* 1e-3 */
    float beta1;            /* 0.9 */
    float beta2;            /* 0.999 */
    float eps;              /* 1e-8 */
    float weight_decay;     /* 1e-2: used by soar_optim_create_uniform; create() takes
                               each tensor's own weight_decay */
    int32_t layout;         /* enum soar_layout, default FP32 */
    float max_grad_norm;    /* > 0: step() clips by global L2 norm first, exactly as
                               clip_grad_norm(max_grad_norm) before step(); default 0 */
    int32_t use_loss_scaler;/* 1: grads arrive multiplied by the loss scale; unscale,
                               skip on inf/NaN, dynamic scale update. default 0 */
    float init_scale;       /* 65536 */
    float growth_factor;    /* 2 */
    float backoff_factor;   /* 0.5 */
    int32_t growth_interval;/* 200 clean steps */
    int32_t device;         /* CUDA device ordinal of every buffer; default 0 */
} soar_adamw_opts;

/* Step bookkeeping, read back from the device (soar_optim_get_info). */
typedef struct soar_step_info {
    uint64_t step;          /* AdamW step count t (adamw.hpp:35); skipped steps excluded */
    uint64_t skipped;       /* steps skipped for inf/NaN */
    float grad_norm;        /* pre-clip global norm of the last step (clip_grad_norm's return) */
    int32_t found_inf;      /* last step saw a non-finite unscaled gradient */
    float clip_coef;        /* coefficient applied by the last step (1 = none) */
    float loss_scale;       /* live loss scale (for the next backward) */
    int32_t growth_tracker; /* clean steps since the last scale change */
    float lr;               /* learning rate used by the last step */
    int32_t error;          /* nonzero: a device-side pipeline wait timed out in some
                               step; that step is incomplete and the state must not be
                               trusted (cleared by soar_optim_set_counters) */
} soar_step_info;

/* Reference-default options (adamw.hpp:10-16) and the extension defaults. */
SOAR_API void soar_adamw_default_opts(soar_adamw_opts* out);

/* Replaces AdamW::AdamW(std::vector<TensorPtr>, AdamWOptions) (adamw.cpp:7-18):
   allocates the optimizer state (m = v = 0; master = float(param) in the mixed
   layout) and the tensor-list chunk table on opts->device. */
SOAR_API int soar_optim_create(const soar_tensor_desc* tensors, int n_tensors,
                               const soar_adamw_opts* opts, void** out_handle);

/* Same, with every tensor's weight decay taken from opts->weight_decay (the
   reference constructor's single weight_decay, adamw.hpp:15). */
SOAR_API int soar_optim_create_uniform(void* const* params, void* const* grads,
                                       const uint64_t* numel, int n_tensors,
                                       const soar_adamw_opts* opts, void** out_handle);

/* SGD on the same device step: replaces soar::optim::SGD
   (include/soar/optim/sgd.hpp:9-38, src/optim/sgd.cpp). The first five fields
   are the reference's SGDOptions (same defaults); the rest are the AdamW
   extensions. The handle works with every soar_optim_* call (step, zero_grad,
   clip_grad_norm, set/get_lr, info, state: MASTER and M = momentum buffer,
   checkpoint, EMA, destroy). */
typedef struct soar_sgd_opts {
    float lr;               /* 1e-2 */
    float momentum;         /* 0 */
    float dampening;        /* 0 */
    float weight_decay;     /* 0 (coupled: d_p += wd * theta, sgd.cpp:72-74) */
    int32_t nesterov;       /* 0 */
    int32_t layout;
    float max_grad_norm;
    int32_t use_loss_scaler;
    float init_scale;
    float growth_factor;
    float backoff_factor;
    int32_t growth_interval;
    int32_t device;
} soar_sgd_opts;

SOAR_API void soar_sgd_default_opts(soar_sgd_opts* out);
/* Replaces SGD::SGD(std::vector<TensorPtr>, SGDOptions) (sgd.cpp:7-16). Each
   tensor's weight_decay is its own (parameter groups). */
SOAR_API int soar_sgd_create(const soar_tensor_desc* tensors, int n_tensors,
                             const soar_sgd_opts* opts, void** out_handle);

SOAR_API int soar_optim_destroy(void* handle);

/* Replaces AdamW::step() (adamw.cpp:60-117) -- and, with max_grad_norm > 0,
   the clip_grad_norm() call before it (adamw.cpp:28-58) -- as one fused
   device step: unscale, inf/NaN detect, global norm, clip, AdamW with
   per-tensor wd on the fp32 master, bf16 write-back, loss-scale update.
   Enqueued on `stream`; never synchronises the host. It may be captured into
   a CUDA graph (stream capture on `stream`): the step count, loss scale and
   skip decision live on the device, so every replay is a correct next step;
   the lr (and a pending standalone clip coefficient) are taken at capture,
   so a changed lr needs a new capture. (With beta2 so close to 1 that
   1 - beta2^t stays below 1.0f for more than 61440 steps, the
   bias-correction table grows on the host at those steps; such a step is not
   capture-safe.) */
SOAR_API int soar_optim_step(void* handle, void* stream);

/* Replaces AdamW::clip_grad_norm(max_norm) (adamw.cpp:28-58): returns the
   pre-clip global L2 norm in *out_norm and, when norm > max_norm and
   norm > 1e-6, scales the fp32 grads in place by max_norm/norm. In the mixed
   layout the bf16 grads are left untouched and the coefficient is applied in
   fp32 inside the next step(). With the loss scaler on, the norm is that of
   the unscaled grads. Synchronous (it returns a value, as the reference does). */
SOAR_API int soar_optim_clip_grad_norm(void* handle, float max_norm, float* out_norm,
                                       void* stream);

/* clip_grad_norm(max_norm) without the host round trip, for callers that
   ignore its return value, as the reference's Trainer does
   (src/engine/trainer.cpp:157): enqueues the global-norm pass on `stream`;
   the next soar_optim_step on the handle (on the same stream) then clips by
   max_norm from that norm -- coefficient max_norm/norm when norm > max_norm
   and norm > 1e-6, exactly as clip_grad_norm -- applied in fp32 inside the
   update (the gradient buffers are left untouched), and reuses the pass
   instead of running its own (the loss scaler's skip decision comes from the
   same sum). The pre-clip norm is the step's grad_norm (soar_optim_get_info,
   _async). Gradients must not change between this call and the step. */
SOAR_API int soar_optim_clip_grad_norm_async(void* handle, float max_norm, void* stream);

/* Replaces AdamW::zero_grad() (adamw.cpp:20-26): zeroes every gradient. */
SOAR_API int soar_optim_zero_grad(void* handle, void* stream);

/* Replace AdamW::set_lr / get_lr (adamw.hpp:29-30). Host-side, no device work. */
SOAR_API int soar_optim_set_lr(void* handle, float lr);
SOAR_API int soar_optim_get_lr(void* handle, float* out_lr);

/* Step bookkeeping readback (synchronises `stream`). No reference counterpart
   beyond get_lr; the reference keeps step_count_ private (adamw.hpp:35). */
SOAR_API int soar_optim_get_info(void* handle, soar_step_info* out, void* stream);

/* The same bookkeeping without synchronising the host: enqueues on `stream`
   a copy of the values as they stand once the stream's earlier work (the
   step) has run; they are in *out when an event recorded on `stream` after
   this call has completed. `out` should be pinned host memory
   (cudaHostAlloc) for the copy to stay asynchronous. */
SOAR_API int soar_optim_get_info_async(void* handle, soar_step_info* out, void* stream);

/* Restores step count, skip count, loss scale and growth tracker (resume). */
SOAR_API int soar_optim_set_counters(void* handle, uint64_t step, uint64_t skipped,
                                     float loss_scale, int32_t growth_tracker, void* stream);

/* Device address of tensor `index`'s optimizer state array (`kind`:
   enum soar_state_kind; MASTER is the param itself in the FP32 layout). The
   reference holds these as m_[idx] / v_[idx] (adamw.hpp:38-39). */
SOAR_API int soar_optim_state_ptr(void* handle, int index, int kind, void** out_ptr);

/* Synchronous host copies of one tensor's state (checkpointing, tests). */
SOAR_API int soar_optim_read_state(void* handle, int index, int kind, float* host_dst);
SOAR_API int soar_optim_write_state(void* handle, int index, int kind, const float* host_src);

/* Optimizer-state checkpoint. No counterpart in the reference, whose
   checkpoints hold model weights only (src/nn/soar_model.cpp:427-523), so a
   resumed run restarts Adam's moments and bias correction. Writes/reads a
   SOAR file (magic 'SOAR', version 2) in the reference's weight-record layout:
   records "optim.master.<i>", "optim.m.<i>", "optim.v.<i>" (fp32, tensor i of
   the list; plus "optim.ema.<i>" when the weight EMA is on) and "optim.counters" (step count, skipped steps, loss scale,
   growth tracker, lr). The reference's weight loader skips these names. Load
   needs an optimizer created over the same tensor list; in the mixed layout
   it also rewrites the bf16 params from the restored master. Synchronous. */
SOAR_API int soar_optim_save_state(void* handle, const char* path);
SOAR_API int soar_optim_load_state(void* handle, const char* path, void* stream);

/* Weight EMA fused into the update: replaces soar::utils::ModelEMA
   (include/soar/utils/ema.hpp:10-66). enable allocates the shadow and copies
   the current fp32 weights into it (init_shadow, ema.hpp:49-57); from then on
   every applied step also computes shadow = decay*shadow + (1-decay)*weight
   (update, ema.hpp:18-28) inside the update kernel, on the fp32 master
   weights (the fp32 params in the FP32 layout), for +8 bytes per param.
   Skipped steps leave the shadow unchanged. Calling enable again resets the
   shadow to the current weights and sets a new decay. */
SOAR_API int soar_optim_enable_ema(void* handle, float decay, void* stream);
/* ModelEMA::apply_to (ema.hpp:31-38): the weights become the shadow (master
   and bf16 params in the mixed layout). */
SOAR_API int soar_optim_ema_apply_to(void* handle, void* stream);

/* Gradient buffers that change between steps. The reference reads each
   parameter's current grad() at every step (adamw.cpp:74-75, 80-85); this
   optimizer binds gradient buffers when it is created, and a caller whose
   gradients live in more than one buffer (double-buffered host uploads,
   gradient accumulation into alternating buffers) registers each further set
   once: soar_optim_add_grads takes one gradient pointer per tensor (NULL
   exactly where the creating list had NULL; each with the same address
   modulo 16 bytes as the first set's, which torch and cudaMalloc buffers of
   one layout have) and returns the set's index in *out_set (the creating
   list is set 0). soar_optim_use_grads makes a set the one that step,
   clip_grad_norm and zero_grad use from the next call on: host-side, no
   device work; kernels already enqueued keep the set they were launched
   with, and a step captured into a CUDA graph keeps the set it was captured
   with (capture one graph per set to alternate them). Each added set holds its own copy of the chunk tables on the device
   (64 bytes per chunk of up to 16384 elements), freed by soar_optim_destroy. */
SOAR_API int soar_optim_add_grads(void* handle, void* const* grads, int* out_set);
SOAR_API int soar_optim_use_grads(void* handle, int set);

/* Which update kernel this optimizer's steps launch (*out_path): 0 = the
   bulk-copy pipeline (k_apply), 1 = the register-fed single-pass kernel for
   short lists (k_apply_direct: at most 4 tensors with a vector part and at
   most 16M elements (16 x 2^20), no weight EMA, AdamW). Both compute the same bits. */
SOAR_API int soar_optim_kernel_path(void* handle, int* out_path);

/* Device address of the live loss scale (fp32), for scaling the loss on the
   device without a host round trip. */
SOAR_API int soar_optim_loss_scale_ptr(void* handle, float** out_ptr);

/* Data-parallel split of soar_optim_step (ZeRO-1, one process per GPU):
   (1) soar_optim_grad_sumsq writes this rank's sum of squared unscaled grads
       (fp64) to the device address d_sumsq;
   (2) the caller gathers the R partials of all ranks into one device array
       (e.g. an all-gather over NCCL);
   (3) soar_optim_apply sums the partials in rank order -- so every rank takes
       the same skip/clip decision from identical bits -- and runs the update.
   With n_parts = 0 (and d_parts NULL) apply runs without norm/inf
   information: no clip and no skip. */
SOAR_API int soar_optim_grad_sumsq(void* handle, double* d_sumsq, void* stream);
SOAR_API int soar_optim_apply(void* handle, const double* d_parts, int n_parts, void* stream);

/* ---- Fused data-parallel step (ZeRO-1 over peer memory) -------------------
   No counterpart in the reference, which has no distributed code. One process
   per GPU; every rank's flat bf16 parameter and gradient buffers are allocated
   with soar_ipc_alloc and opened by every other rank with soar_ipc_open (CUDA
   IPC: the 64-byte handles travel between processes by any host channel, e.g.
   torch.distributed), so all buffers are addressable from every GPU at
   identical element offsets. */
#define SOAR_IPC_HANDLE_BYTES 64

/* Allocations are zero-filled. */
SOAR_API int soar_ipc_alloc(size_t bytes, int device, void** out_ptr, void* out_handle);
SOAR_API int soar_ipc_free(void* ptr, int device);
SOAR_API int soar_ipc_open(const void* handle, int device, void** out_peer_ptr);
SOAR_API int soar_ipc_close(void* peer_ptr, int device);

/* One slice of the flat buffers owned by this rank: elements
   [offset, offset + count), held by optimizer tensor `tensor`, whose param and
   grad must be exactly that slice of this rank's buffers. */
typedef struct soar_zero1_shard {
    uint64_t offset;
    uint64_t count;
    int32_t tensor;
} soar_zero1_shard;

/* Binds a bf16-mixed optimizer over this rank's owned slices to the R
   symmetric buffers (grad_bases[q] / param_bases[q]: rank q's buffers as seen
   from this process; index `rank` is the local one). At most 8 ranks. */
SOAR_API int soar_zero1_create(void* optim_handle, int rank, int world,
                               void* const* grad_bases, void* const* param_bases,
                               const soar_zero1_shard* shards, int n_shards, void** out_handle);

/* Reduce-scatter fused with the norm pass: every owned element becomes the
   average of the R ranks' gradients (fp32 sum in rank order, one multiply by
   1/R, one bf16 rounding), written in place into the local gradient buffer;
   *d_partial receives this rank's sum of squares of the unscaled averages.
   Every rank's gradients must be complete before it runs (a barrier). */
SOAR_API int soar_zero1_reduce_sumsq(void* zero1_handle, double* d_partial, void* stream);

/* The update (as soar_optim_apply, with the R rank-ordered partials) fused
   with the all-gather: each updated bf16 param tile is also written into
   every peer's parameter buffer. Peers may read their parameters only after
   every rank's call has completed (a barrier). */
SOAR_API int soar_zero1_apply_allgather(void* zero1_handle, const double* d_parts, int n_parts,
                                        void* stream);

/* Device-synchronised step. signal_bases[q]: rank q's signal block (at least
   SOAR_ZERO1_SIGNAL_BYTES, 256-byte aligned, zero-filled: one soar_ipc_alloc
   per rank, opened by every other rank like the buffers; index `rank` is the
   local one). Set once per handle, before its first soar_zero1_step, and
   every rank's block must be allocated (zeroed) before any rank steps; a block
   serves one handle for its lifetime. */
#define SOAR_ZERO1_SIGNAL_BYTES 4096
SOAR_API int soar_zero1_set_signals(void* zero1_handle, void* const* signal_bases);

/* The whole data-parallel step with no host collective: the reduce-scatter
   with the norm pass, the exchange of the R partial sums, the update with the
   all-gather and the end-of-step wait, synchronised across GPUs by epoch flags
   in the signal blocks (system-scope release / acquire, every wait bounded to
   1 s). Stream-ordered like soar_optim_step: it starts after this rank's
   earlier work on `stream` (the gradients) and, when it completes, every
   rank's parameter writes into this rank's buffer have landed. Every rank
   calls it once per step. A timed-out wait skips the step's update (counted
   as a skipped step) and sets the error flag (soar_zero1_error); after that
   the ranks' optimizer states may differ and training resumes from a
   checkpoint. */
SOAR_API int soar_zero1_step(void* zero1_handle, void* stream);

/* Nonzero in *out_error if a device-side wait of the data-parallel step timed
   out (synchronises the device). */
SOAR_API int soar_zero1_error(void* zero1_handle, int* out_error);
SOAR_API int soar_zero1_destroy(void* zero1_handle);

/* ---- Data-parallel bootstrap in the library ---------------------------
   No counterpart in the reference, which has no distributed code. One process
   per GPU, any host language: the ranks share an NCCL communicator and build
   the fused ZeRO-1 step over it without Python or torch.

   Rank 0 calls soar_dp_unique_id and hands the 128 bytes to every other rank
   over any host channel (a file, MPI, a TCP store); every rank then calls
   soar_dp_init with its rank, the world size (1..8), the id and its CUDA
   device. NCCL (libnccl.so.2) is loaded when soar_dp_unique_id or
   soar_dp_init is first called; like ncclCommInitRank, soar_dp_init returns
   once every rank has joined. */
#define SOAR_DP_UNIQUE_ID_BYTES 128
SOAR_API int soar_dp_unique_id(void* out_id);
SOAR_API int soar_dp_init(int rank, int world, const void* unique_id, int device,
                          void** out_comm);
SOAR_API int soar_dp_destroy(void* comm);
/* Stream-ordered barrier over the communicator (a 1-element all-reduce): it
   completes on this GPU once every rank's earlier work on its stream has. */
SOAR_API int soar_dp_barrier(void* comm, void* stream);
/* All-gather of `count` fp64 values per rank (rank order), on `stream`. */
SOAR_API int soar_dp_allgather_f64(void* comm, const double* d_send, double* d_recv,
                                   uint64_t count, void* stream);

/* The fused ZeRO-1 optimizer over the communicator (collective: every rank
   calls it with the same n_params, bucket and options). Allocates this rank's
   flat bf16 parameter and gradient buffers of n_params elements (IPC
   symmetric: every rank opens every other rank's), copies init_params into
   the parameter buffer (n_params bf16 values, host or device; NULL leaves the
   zeros), gives rank r the r-th ceil(size / world) slice of every bucket of
   `bucket` elements, and creates the bf16-mixed AdamW of those slices with
   `opts` (layout SOAR_LAYOUT_BF16_MIXED, opts->device = the communicator's
   device; every slice takes opts->weight_decay; its fp32 master starts from
   the initial params). sync_mode SOAR_DP_SYNC_DEVICE synchronises the ranks
   inside the kernels through flags in a signal block (no host collective in a
   step); SOAR_DP_SYNC_NCCL issues small collectives between the launches.
   A failure on any rank is reported on every rank (the others do not hang). */
#define SOAR_DP_SYNC_DEVICE 0
#define SOAR_DP_SYNC_NCCL 1
SOAR_API int soar_dp_zero1_create(void* comm, uint64_t n_params, uint64_t bucket,
                                  const soar_adamw_opts* opts, const void* init_params,
                                  int sync_mode, void** out_handle);

typedef struct soar_dp_zero1_info {
    void* params;          /* this rank's flat bf16 parameter buffer (device), n_params */
    void* grads;           /* this rank's flat bf16 gradient buffer: fill before a step */
    void* optimizer;       /* the shard optimizer: a soar_optim_* handle (info, lr,
                              checkpoint; owned by this object) */
    void* zero1;           /* the soar_zero1_* handle (error flag; owned by this object) */
    uint64_t n_params;
    uint64_t shard_params; /* elements this rank owns */
    int32_t rank;
    int32_t world;
} soar_dp_zero1_info;
SOAR_API int soar_dp_zero1_get_info(void* handle, soar_dp_zero1_info* out);

/* One data-parallel step on `stream`: every rank's gradient (in its buffer,
   complete in stream order) is averaged over the ranks, the owned slices are
   updated (unscale, norm, clip, AdamW, bf16 write-back, loss scaler) and
   every rank's parameter buffer holds the whole updated model once the step
   completes. The rank's owned slice of its gradient buffer is overwritten
   with the average. Every rank calls it once per step. */
SOAR_API int soar_dp_zero1_step(void* handle, void* stream);
/* Further gradient buffers, so that the next step's gradient can be written
   (an upload from the host, an accumulation) while a step still reads the
   current one. soar_dp_zero1_add_grads (collective) allocates another
   symmetric gradient buffer of n_params bf16 elements on every rank, with its
   own signal block, and returns its index in *out_index (the buffer made by
   soar_dp_zero1_create is 0). soar_dp_zero1_use_grads makes buffer `index` the
   one the next soar_dp_zero1_step calls reduce (host-side; every rank must
   use the same index for a step); soar_dp_zero1_get_info then reports it as
   `grads` and `zero1`. soar_dp_zero1_grads gives this rank's buffer `index`.
   A buffer may be rewritten once a step that read it has completed on this
   rank's stream: by then every peer has finished reading it. */
SOAR_API int soar_dp_zero1_add_grads(void* handle, int* out_index);
SOAR_API int soar_dp_zero1_use_grads(void* handle, int index);
SOAR_API int soar_dp_zero1_grads(void* handle, int index, void** out_grads);
/* Collective: releases the buffers once no rank maps them any more. */
SOAR_API int soar_dp_zero1_destroy(void* handle);

/* Replaces CosineAnnealingLR (adamw.hpp:45-57, adamw.cpp:119-143): linear
   warmup, cosine decay to eta_min, eta_min past the end; each step() sets the
   bound optimizer's lr (host-side float math, the reference's expressions).
   The scheduler keeps the optimizer handle, so moving the optimizer between
   owners cannot leave it bound to a stale object. */
SOAR_API int soar_cosine_create(void* optim_handle, uint64_t total_steps, float eta_min,
                                uint64_t warmup_steps, void** out_handle);
SOAR_API int soar_cosine_step(void* sched_handle);
SOAR_API int soar_cosine_destroy(void* sched_handle);

/* Allocation-free gradient sum of squares. No counterpart in the reference.
   For callers that cannot call cudaMalloc: a host runtime that reserves all of
   a GPU's memory up front in its own pool (an extra cudaMalloc fails or escapes
   the pool's accounting), or a latency-sensitive loop where cudaMalloc's
   implicit device-wide synchronisation would stall work in flight. Computes
   the same quantity as soar_optim_grad_sumsq -- sum over the tensors of
   (double)(g * inv_scale)^2, fp32 (FP32 layout) or bf16 (BF16_MIXED) grads --
   into the caller's device fp64 *d_sumsq, without an optimizer handle and
   without allocating: its scratch (per-CTA partials and a ticket, ~8 KB) is a
   static device array that every GPU loading the library holds until exit.
   At most SOAR_NOALLOC_MAX_TENSORS tensors per call (more is rejected with an
   error); element counts are unlimited. Runs on the current device. The first
   call on a device also sets up that device (looks up the array's device
   address, cached for the life of the process: it assumes the device's
   primary context lives as long, so a process that calls cudaDeviceReset must
   not call this entry point afterwards); make that first call before any
   stream capture. All calls share
   the array: calls whose kernels overlap on the GPU race and give wrong sums,
   so order them on one stream. */
#define SOAR_NOALLOC_MAX_TENSORS 64
SOAR_API int soar_grad_sumsq_noalloc(const void* const* grads, const uint64_t* numel,
                                     int n_tensors, int layout, float inv_scale,
                                     double* d_sumsq, void* stream);

/* Failure-detection self-test (no reference counterpart): runs the bounded
   wait that every device pipeline uses on an mbarrier nothing arrives at,
   with the given limit, on `device`. *out_timed_out is 1 when the wait gave up
   and reported it (the expected result), *out_waited_ns how long it waited.
   No fault, trap or hang is involved; the context stays usable. */
SOAR_API int soar_selftest_bounded_wait(uint64_t limit_ns, int device, int* out_timed_out,
                                        uint64_t* out_waited_ns);

/* Build query, no reference counterpart. *out_compiled: the architecture the
   kernels were compiled for, as nvcc's __CUDA_ARCH_LIST__ writes it (1000 for
   sm_100a); needs no GPU. With device >= 0 also *out_loaded: the SASS version
   the update kernel was loaded as on that device (cudaFuncGetAttributes
   binaryVersion: 100 for sm_100a), which needs the GPU. */
SOAR_API int soar_kernel_arch(int device, int* out_compiled, int* out_loaded);

/* Message of the calling thread's last failed call ("" if none). */
SOAR_API const char* soar_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* SOAR_OPTIM_H */
