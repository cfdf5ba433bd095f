// Optimizer-step kernels for B200 (sm_100a).
//
// The step is HBM-bound streaming work (~15 flop per 28 bytes), so it runs on
// the SIMT pipes fed by the Tensor Memory Accelerator, not on tensor cores.
// Two kernels over one tensor-list chunk table (Chunk, optim_kernels.cuh):
//
//   k_grad_sumsq  reads every gradient once (2 B bf16 / 4 B fp32 per element,
//                 16-byte loads), unscales it by the live loss scale and
//                 accumulates the fp64 sum of squares: per thread, warp
//                 shuffle, block, then a single-pass grid reduction (each CTA
//                 writes its partial, the last CTA to take a ticket folds them
//                 in fixed order). Non-finite gradients make the sum
//                 non-finite, so the same number carries the inf/NaN flag.
//   k_apply       derives skip / clip coefficient / bias corrections from the
//                 partial sums, then streams the update through a shared-memory
//                 pipeline: one producer thread issues 1D bulk async copies
//                 (cp.async.bulk, completion on an mbarrier) of 1024-element
//                 tiles of grad/master/m/v into a 6-stage ring; 12 consumer
//                 warps unscale, clip, apply decoupled weight decay and the
//                 AdamW moments, write master/m/v and the bf16 params back into
//                 the stage, and one of them bulk-stores the stage to HBM. The
//                 loads never wait on registers, so many tiles are in flight
//                 per SM. Chunks are taken from the top of the table down --
//                 the reverse of k_grad_sumsq's order, so the gradients read
//                 last there are still in L2 -- either by a static
//                 grid-strided walk or handed out dynamically (one atomic per
//                 chunk; chosen per optimizer on the host). The last CTA to
//                 finish commits the step counters and the loss-scaler update.
//
// Numerics follow the reference's AdamW::step / clip_grad_norm
// (src/optim/adamw.cpp:28-117) operation for operation with explicitly
// rounded intrinsics (no contraction, IEEE sqrt and division), so the fp32
// update reproduces the reference's bits.
//
// Every wait on an mbarrier is bounded (1 s of %globaltimer); on timeout the
// kernel records Ctl::error, stops issuing, waits (bounded) for its own copies
// in flight and returns.
#include "optim_kernels.cuh"
#include "pipeline.cuh"

namespace soarb {
namespace {

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
// (adamw.cpp:37-38) term by term; only the summation order differs.
__device__ __forceinline__ double sq_acc(double acc, float g) {
    const double d = static_cast<double>(g);
    return fma(d, d, acc);
}

__device__ __forceinline__ double sq_acc_bf16x8(double acc, const uint4& q, float inv) {
    acc = sq_acc(acc, __fmul_rn(bf16_lo(q.x), inv));
    acc = sq_acc(acc, __fmul_rn(bf16_hi(q.x), inv));
    acc = sq_acc(acc, __fmul_rn(bf16_lo(q.y), inv));
    acc = sq_acc(acc, __fmul_rn(bf16_hi(q.y), inv));
    acc = sq_acc(acc, __fmul_rn(bf16_lo(q.z), inv));
    acc = sq_acc(acc, __fmul_rn(bf16_hi(q.z), inv));
    acc = sq_acc(acc, __fmul_rn(bf16_lo(q.w), inv));
    acc = sq_acc(acc, __fmul_rn(bf16_hi(q.w), inv));
    return acc;
}

__device__ __forceinline__ double sq_acc_f32x4(double acc, const float4& q, float inv) {
    acc = sq_acc(acc, __fmul_rn(q.x, inv));
    acc = sq_acc(acc, __fmul_rn(q.y, inv));
    acc = sq_acc(acc, __fmul_rn(q.z, inv));
    acc = sq_acc(acc, __fmul_rn(q.w, inv));
    return acc;
}

template <bool kBf16>
__global__ void __launch_bounds__(kThreads)
k_grad_sumsq(const Chunk* __restrict__ chunks, int n_chunks, Ctl* __restrict__ ctl,
             double* __restrict__ partials, int use_scaler, double* __restrict__ out) {
    __shared__ double s_red[32];
    __shared__ int s_last;
    pdl_wait();
    pdl_trigger();
    const float inv = use_scaler ? __fdiv_rn(1.0f, ctl->scale) : 1.0f;
    double acc = 0.0;
    for (int c = blockIdx.x; c < n_chunks; c += gridDim.x) {
        const Chunk* ch = chunks + c;
        const uint32_t n = ch->n;
        const void* gp = ch->grad;
        uint32_t scalar_from = 0;
        if (ch->flags & kChunkVec) {
            // 16-byte vectors: 8 bf16 or 4 fp32
            constexpr uint32_t kPer = kBf16 ? 8u : 4u;
            const uint32_t nv = n / kPer;
            scalar_from = nv * kPer;
            const uint4* g4 = static_cast<const uint4*>(gp);
            uint32_t i = threadIdx.x;
            for (; i + 3 * kThreads < nv; i += 4 * kThreads) {
                uint4 q[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) q[u] = __ldg(g4 + i + u * kThreads);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    if constexpr (kBf16) acc = sq_acc_bf16x8(acc, q[u], inv);
                    else acc = sq_acc_f32x4(acc, *reinterpret_cast<const float4*>(&q[u]), inv);
                }
            }
            for (; i < nv; i += kThreads) {
                const uint4 q = __ldg(g4 + i);
                if constexpr (kBf16) acc = sq_acc_bf16x8(acc, q, inv);
                else acc = sq_acc_f32x4(acc, *reinterpret_cast<const float4*>(&q), inv);
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

// Per-step values derived on the device from the control block. The
// host-known coefficients stay in the launch arguments (kernel parameter
// space), which keeps them out of the register file of the streaming loop.
struct StepCoeffs {
    float inv;        // 1 / loss scale
    float coef;       // clip coefficient (1: no clip)
    float step_size;  // lr / bias_correction1 (AdamW)
    float sqrt_bc2;   // (AdamW)
    int has_buf;      // SGD: momentum buffers hold a previous step (sgd.cpp:75-80)
};

// One element of SGD::step (reference src/optim/sgd.cpp:70-88): coupled weight
// decay, momentum with dampening, optional Nesterov, theta -= lr * d_p. `m`
// is the momentum buffer.
__device__ __forceinline__ void sgd_elem(float& th, float& m, float g, const ApplyArgs& a,
                                         const StepCoeffs& k, float wd) {
    float d = g;
    if (wd != 0.0f) d = __fadd_rn(d, __fmul_rn(wd, th));
    if (a.momentum != 0.0f) {
        m = k.has_buf ? __fadd_rn(__fmul_rn(a.momentum, m), __fmul_rn(a.omdamp, d)) : d;
        d = a.nesterov ? __fadd_rn(d, __fmul_rn(a.momentum, m)) : m;
    }
    th = __fsub_rn(th, __fmul_rn(a.lr, d));
}

// One element of AdamW::step (adamw.cpp:92-107) on an unscaled, clipped grad.
__device__ __forceinline__ void adamw_elem(float& th, float& m, float& v, float g,
                                           const ApplyArgs& a, const StepCoeffs& k, float lr_wd,
                                           bool has_wd) {
    if (has_wd) th = __fsub_rn(th, __fmul_rn(lr_wd, th));
    m = __fadd_rn(__fmul_rn(a.beta1, m), __fmul_rn(a.omb1, g));
    v = __fadd_rn(__fmul_rn(a.beta2, v), __fmul_rn(__fmul_rn(a.omb2, g), g));
    const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), k.sqrt_bc2), a.eps);
    th = __fsub_rn(th, __fmul_rn(k.step_size, __fdiv_rn(m, denom)));
}

// Unscale (exact for power-of-two scales) then clip (adamw.cpp:49-51).
__device__ __forceinline__ float prep_grad(float graw, const StepCoeffs& k) {
    return __fmul_rn(__fmul_rn(graw, k.inv), k.coef);
}

// ModelEMA::update (ema.hpp:25) for one weight: decay*shadow + (1-decay)*weight.
__device__ __forceinline__ float ema_elem(float sh, float w, const ApplyArgs& a) {
    return __fadd_rn(__fmul_rn(a.ema_decay, sh), __fmul_rn(a.ema_omd, w));
}

// The step's decision, taken by one thread of every CTA from the same bits:
// skip (a failed peer sync, or inf/NaN with the scaler on), the pre-clip norm
// from the rank-ordered fp64 partial sums, the clip coefficient and the bias
// corrections of the step count the step will have. Counters are only read
// here and only written by the last CTA (commit_step).
struct StepDecision {
    StepCoeffs k;
    uint64_t t;
    float norm;
    int skip;
    int found;
};

__device__ __forceinline__ StepDecision decide_step(const ApplyArgs& a, const Ctl* ctl) {
    StepDecision d;
    d.skip = 0;
    d.found = 0;
    d.norm = 0.0f;
    float coef = a.pending_coef;
    if (a.skip_if && *a.skip_if) {
        d.skip = 1;  // a peer failed to synchronise: no update (the error flag tells)
    } else if (a.n_parts > 0) {
        double s = 0.0;
        for (int p = 0; p < a.n_parts; ++p) s += a.parts[p];
        d.found = !isfinite(s);
        d.norm = __double2float_rn(__dsqrt_rn(s));  // adamw.cpp:42
        if (a.use_scaler && d.found) d.skip = 1;
        // adamw.cpp:43-44: no eps, no min(1, .)
        if (a.max_norm > 0.0f && d.norm > a.max_norm && d.norm > 1e-6f)
            coef = __fdiv_rn(a.max_norm, d.norm);
    }
    d.t = ctl->t + (d.skip ? 0u : 1u);
    const uint64_t ti = d.t < a.bc_len ? d.t : static_cast<uint64_t>(a.bc_len - 1);
    const float2 bc = a.bc[ti];
    d.k.inv = a.use_scaler ? __fdiv_rn(1.0f, ctl->scale) : 1.0f;
    d.k.coef = coef;
    d.k.step_size = __fdiv_rn(a.lr, bc.x);  // adamw.cpp:71
    d.k.sqrt_bc2 = bc.y;
    d.k.has_buf = ctl->t > 0;  // applied steps so far (skipped steps never fill buffers)
    return d;
}

// Called by thread 0 of every CTA once the CTA is done: the last CTA to
// arrive (every CTA has read the counters by then) commits the step count,
// the bookkeeping and the loss-scaler update, and resets the tickets.
__device__ __forceinline__ void commit_step(Ctl* ctl, const ApplyArgs& a, const StepDecision& d) {
    __threadfence();
    const unsigned prev = atomicAdd(&ctl->ticket_apply, 1u);
    if (prev != gridDim.x - 1) return;
    ctl->t = d.t;
    ctl->last_norm = d.norm;
    ctl->last_found_inf = d.found;
    ctl->last_clip_coef = d.skip ? 1.0f : d.k.coef;
    ctl->last_lr = a.lr;
    if (d.skip) ctl->skipped += 1u;
    if (a.use_scaler) {
        if (d.skip) {
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
    ctl->grab = 0u;  // every CTA has stopped grabbing
    ctl->ticket_apply = 0u;
}

// Elements [from, to) of a chunk, straight from global memory. With kAg the
// updated params are also written into every peer's parameter buffer.
template <bool kMixed, bool kAg, bool kEma, bool kSgd>
__device__ __forceinline__ void apply_scalar(const Chunk& ch, uint32_t from, uint32_t to,
                                             uint32_t tid, uint32_t nthreads, const ApplyArgs& a,
                                             const StepCoeffs& k, float lr_wd, bool has_wd,
                                             const AgArgs& ag) {
    for (uint32_t i = from + tid; i < to; i += nthreads) {
        const float graw = kMixed ? bf16_bits_to_f32(static_cast<const uint16_t*>(ch.grad)[i])
                                  : static_cast<const float*>(ch.grad)[i];
        float th = ch.master[i];
        if constexpr (kSgd) {
            float m = a.momentum != 0.0f ? ch.m[i] : 0.0f;
            sgd_elem(th, m, prep_grad(graw, k), a, k, ch.wd);
            ch.master[i] = th;
            if (a.momentum != 0.0f) ch.m[i] = m;
        } else {
            float m = ch.m[i], v = ch.v[i];
            adamw_elem(th, m, v, prep_grad(graw, k), a, k, lr_wd, has_wd);
            ch.master[i] = th;
            ch.m[i] = m;
            ch.v[i] = v;
        }
        if constexpr (kEma) {
            float* sh = ch.m + a.ema_delta;
            sh[i] = ema_elem(sh[i], th, a);
        }
        uint16_t pb = 0;
        if constexpr (kMixed) {
            pb = f32_to_bf16_rn(th);
            static_cast<uint16_t*>(ch.param)[i] = pb;
        }
        if constexpr (kAg) {
            const size_t off = static_cast<const char*>(ch.param) - ag.local_param_base;
            for (int q = 0; q < ag.world; ++q) {
                if (q == ag.rank) continue;
                if constexpr (kMixed)
                    reinterpret_cast<uint16_t*>(ag.peer_param_base[q] + off)[i] = pb;
                else
                    reinterpret_cast<float*>(ag.peer_param_base[q] + off)[i] = th;
            }
        }
    }
}

// Visits the pipelined tiles of this CTA in order: vector chunks from the end
// of the vector part of the table, grid-strided, each in kTile pieces. The
// producer and the consumers walk exactly this sequence (static hand-out).
template <typename F>
__device__ __forceinline__ void for_each_tile(const Chunk* chunks, int n_vec, F&& f) {
    uint32_t q = 0;
    for (int c = n_vec - 1 - static_cast<int>(blockIdx.x); c >= 0; c -= gridDim.x) {
        const Chunk ch = chunks[c];
        for (uint32_t t0 = 0; t0 < ch.n; t0 += kTile, ++q) {
            if (!f(ch, t0, min(static_cast<uint32_t>(kTile), ch.n - t0), q)) return;
        }
    }
}

template <bool kMixed, bool kAg, bool kEma, bool kSgd, bool kDyn>
__global__ void __launch_bounds__(kApplyThreads, 2)
k_apply(const Chunk* __restrict__ chunks, int n_chunks, int n_vec, Ctl* __restrict__ ctl,
        ApplyArgs a, AgArgs ag) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int kStages = apply_stages(kMixed, kEma, kSgd, kAg);
    static_assert(!kAg || kStages >= kAgStoreLag + 2, "stages held by store reads");
    // bf16 params of the all-gather leave through the push area (see kAgPushTiles)
    constexpr bool kPushBuf = kMixed && kAg && kAgPushTiles > 0;
    constexpr uint32_t kPushHalf = static_cast<uint32_t>(kAgPushTiles) * kTile * 2u;
    constexpr uint32_t kPusher = 32;  // the consumer thread that issues those pushes
    __shared__ __align__(8) uint64_t full_bar[kStages], empty_bar[kStages];
    __shared__ StepCoeffs s_k;
    __shared__ int s_skip, s_found, s_err, s_drain_err;
    // consumer-only failure flags, one per tile parity: written before the
    // per-tile consumer barrier, read after it, so all consumers agree
    __shared__ int s_cfail[2];
    __shared__ uint64_t s_t;
    __shared__ float s_norm;
    __shared__ uint32_t s_issued;
    // (dynamic hand-out) per stage: the tile's chunk descriptor and (chunk index, tile offset)
    __shared__ Chunk s_chunk[kDyn ? kStages : 1];
    __shared__ int2 s_tile[kDyn ? kStages : 1];

    constexpr uint32_t kGradBytes = kMixed ? 2u : 4u;
    constexpr uint32_t kVecElems = kVecBytes / kGradBytes;  // elements per 16 B of grad
    constexpr uint32_t kStage = static_cast<uint32_t>(stage_bytes(kMixed, kEma, kSgd));
    // stage layout: grad | master | m (AdamW m, or the SGD momentum buffer) | v (AdamW) | EMA
    constexpr uint32_t kOffMaster = kGradBytes * kTile, kOffM = kOffMaster + 4u * kTile,
                       kOffV = kOffM + 4u * kTile, kOffE = kOffV + (kSgd ? 0u : 4u) * kTile;
    // SGD without momentum never touches its buffer
    const bool use_m = !kSgd || a.momentum != 0.0f;
    const uint32_t stream_bytes =
        kGradBytes + 4u + (use_m ? 4u : 0u) + (kSgd ? 0u : 4u) + (kEma ? 4u : 0u);
    constexpr int kConsumers = kConsumerWarps * 32;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) {
        const StepDecision d = decide_step(a, ctl);
        s_k = d.k;
        s_skip = d.skip;
        s_t = d.t;
        s_norm = d.norm;
        s_found = d.found;
        s_err = 0;
        s_drain_err = 0;
        s_cfail[0] = s_cfail[1] = 0;
        s_issued = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const StepCoeffs k = s_k;

    if (!s_skip) {
        if (warp == kConsumerWarps) {
            // ---- producer: one thread keeps the ring full -------------------
            if (lane == 0) {
                uint32_t q = 0;
                // Issues tile t0 of chunk c (c < 0: the stop marker, kDyn only)
                // into the next stage, once the consumers have released it.
                auto produce = [&](int c, const Chunk& ch, uint32_t t0) -> bool {
                    const uint32_t s = q % kStages;
                    if (q >= kStages &&
                        !mbar_wait(smem_u32(&empty_bar[s]), ((q / kStages) + 1) & 1, &s_err))
                        return false;
                    if constexpr (kDyn) {
                        s_chunk[s] = ch;
                        s_tile[s] = make_int2(c, static_cast<int>(t0));
                    }
                    const uint32_t fb = smem_u32(&full_bar[s]);
                    if (c < 0) {
                        mbar_arrive(fb);
                    } else {
                        const uint32_t len = min(static_cast<uint32_t>(kTile), ch.n - t0);
                        const uint32_t lv = len & ~(kVecElems - 1);
                        mbar_expect_tx(fb, stream_bytes * lv);
                        if (lv) {
                            const uint32_t base = smem_u32(smem + s * kStage);
                            bulk_load(base, static_cast<const char*>(ch.grad) + kGradBytes * t0,
                                      kGradBytes * lv, fb);
                            bulk_load(base + kOffMaster, ch.master + t0, 4u * lv, fb);
                            if (use_m) bulk_load(base + kOffM, ch.m + t0, 4u * lv, fb);
                            if constexpr (!kSgd) bulk_load(base + kOffV, ch.v + t0, 4u * lv, fb);
                            if constexpr (kEma)
                                bulk_load(base + kOffE, ch.m + a.ema_delta + t0, 4u * lv, fb);
                        }
                    }
                    s_issued = ++q;
                    return true;
                };
                if constexpr (kDyn) {
                    // Chunks are handed out one atomic on Ctl::grab at a time,
                    // from the top of the table down (the reverse of
                    // k_grad_sumsq's order, so the gradients it read last are
                    // still in L2). The next index and its descriptor are
                    // fetched one chunk ahead. The table ends in short pieces,
                    // so CTAs that run slower simply take fewer of them. Each
                    // stage's chunk and tile offset reach the consumers in
                    // shared memory, published by the stage's own mbarrier
                    // arrive; chunk -1 tells them to stop.
                    bool ok = true;
                    int c = n_vec - 1 - static_cast<int>(atomicAdd(&ctl->grab, 1u));
                    Chunk ch = c >= 0 ? chunks[c] : Chunk{};
                    int c_next =
                        c >= 0 ? n_vec - 1 - static_cast<int>(atomicAdd(&ctl->grab, 1u)) : -1;
                    while (ok && c >= 0) {
                        const Chunk ch_next = c_next >= 0 ? chunks[c_next] : Chunk{};
                        const int c_after =
                            c_next >= 0 ? n_vec - 1 - static_cast<int>(atomicAdd(&ctl->grab, 1u))
                                        : -1;
                        for (uint32_t t0 = 0; ok && t0 < ch.n; t0 += kTile)
                            ok = produce(c, ch, t0);
                        c = c_next;
                        ch = ch_next;
                        c_next = c_after;
                    }
                    if (ok) produce(-1, Chunk{}, 0u);
                } else {
                    // static walk: grid-strided from the top of the table; the
                    // consumers walk the same sequence themselves
                    for_each_tile(chunks, n_vec, [&](const Chunk& ch, uint32_t t0, uint32_t,
                                                     uint32_t) { return produce(0, ch, t0); });
                }
            }
        } else {
            // ---- consumers ---------------------------------------------------
            const uint32_t tid = threadIdx.x;
            // (all-gather) thread 0's store groups still reading their stage:
            // the tiles q-ag_np+1 .. q, consecutive, since a tile without
            // stores releases them all
            int ag_np = 0;
            // (push area) every consumer follows the same tile sequence: the
            // open group's next slot and its half of the push area
            uint32_t pb_slot = 0, pb_half = 0;
            const uint32_t push_base = smem_u32(smem + kStages * kStage);
            // Tile q (stage data already waited for). ok: compute it; stop:
            // the sequence ends here (stop marker or a failed wait). Returns
            // false when the consumers must leave the loop.
            auto tile = [&](const Chunk& ch, uint32_t t0, uint32_t len, uint32_t q, bool ok,
                            bool stop) -> bool {
                const uint32_t s = q % kStages;
                const uint32_t lv = len & ~(kVecElems - 1);
                unsigned char* st = smem + s * kStage;
                // (push area) a group is up to kAgPushTiles consecutive tiles of
                // one chunk, all full but the last; it closes at the chunk's
                // last tile, at a partial tile, or when it is full
                const bool pb_close = ok && (lv < static_cast<uint32_t>(kTile) ||
                                             t0 + kTile >= ch.n ||
                                             pb_slot + 1 == static_cast<uint32_t>(kAgPushTiles));
                const bool pb_data = pb_slot > 0 || lv > 0;  // the closing group holds params
                uint2* pb_out = reinterpret_cast<uint2*>(
                    smem + kStages * kStage + pb_half * kPushHalf + pb_slot * (kTile * 2u));
                if (ok) {
                    const float lr_wd = __fmul_rn(a.lr, ch.wd);
                    const bool has_wd = ch.wd != 0.0f;
                    float4* sms = reinterpret_cast<float4*>(st + kOffMaster);
                    float4* sm = reinterpret_cast<float4*>(st + kOffM);
                    float4* sv = reinterpret_cast<float4*>(st + kOffV);
                    float4* se = reinterpret_cast<float4*>(st + kOffE);
                    const uint32_t nv = lv >> 2;
                    for (uint32_t i = tid; i < nv; i += kConsumers) {
                        float4 g;
                        if constexpr (kMixed) {
                            const uint2 q2 = reinterpret_cast<const uint2*>(st)[i];
                            g = make_float4(bf16_lo(q2.x), bf16_hi(q2.x), bf16_lo(q2.y),
                                            bf16_hi(q2.y));
                        } else {
                            g = reinterpret_cast<const float4*>(st)[i];
                        }
                        float4 th = sms[i];
                        if constexpr (kSgd) {
                            float4 mm = use_m ? sm[i] : make_float4(0.f, 0.f, 0.f, 0.f);
                            sgd_elem(th.x, mm.x, prep_grad(g.x, k), a, k, ch.wd);
                            sgd_elem(th.y, mm.y, prep_grad(g.y, k), a, k, ch.wd);
                            sgd_elem(th.z, mm.z, prep_grad(g.z, k), a, k, ch.wd);
                            sgd_elem(th.w, mm.w, prep_grad(g.w, k), a, k, ch.wd);
                            if (use_m) sm[i] = mm;
                        } else {
                            float4 mm = sm[i], vv = sv[i];
                            adamw_elem(th.x, mm.x, vv.x, prep_grad(g.x, k), a, k, lr_wd, has_wd);
                            adamw_elem(th.y, mm.y, vv.y, prep_grad(g.y, k), a, k, lr_wd, has_wd);
                            adamw_elem(th.z, mm.z, vv.z, prep_grad(g.z, k), a, k, lr_wd, has_wd);
                            adamw_elem(th.w, mm.w, vv.w, prep_grad(g.w, k), a, k, lr_wd, has_wd);
                            sm[i] = mm;
                            sv[i] = vv;
                        }
                        sms[i] = th;
                        if constexpr (kEma) {
                            float4 e = se[i];
                            e.x = ema_elem(e.x, th.x, a);
                            e.y = ema_elem(e.y, th.y, a);
                            e.z = ema_elem(e.z, th.z, a);
                            e.w = ema_elem(e.w, th.w, a);
                            se[i] = e;
                        }
                        if constexpr (kMixed) {
                            // the bf16 params take the grad's place in the stage,
                            // or their slot of the push area
                            uint2 p;
                            p.x = pack_bf16x2_rn(th.x, th.y);
                            p.y = pack_bf16x2_rn(th.z, th.w);
                            if constexpr (kPushBuf)
                                pb_out[i] = p;
                            else
                                reinterpret_cast<uint2*>(st)[i] = p;
                        }
                    }
                    // the < 16-byte tail of the tile, straight from global memory
                    apply_scalar<kMixed, kAg, kEma, kSgd>(ch, t0 + lv, t0 + len, tid,
                                                          kConsumers, a, k, lr_wd, has_wd, ag);
                }
                if constexpr (kPushBuf) {
                    // The next group writes the other half of the push area: the
                    // pushes of the group before this one must have read it. They
                    // left kAgPushTiles tiles ago, so this rarely waits.
                    if (tid == kPusher && pb_close && pb_data) bulk_wait_read_all();
                }
                // make the stage's generic-proxy writes visible to the bulk store;
                // after the barrier every consumer reads the same failure flag
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                consumers_sync<kConsumers>();
                if (s_cfail[q & 1] || stop) return false;
                if constexpr (kPushBuf) {
                    if (pb_close) {
                        if (tid == kPusher && pb_data) {
                            // the group's params: into the local buffer and every peer
                            const uint32_t first = t0 - pb_slot * kTile;
                            const uint32_t bytes = 2u * (pb_slot * kTile + lv);
                            const uint32_t src = push_base + pb_half * kPushHalf;
                            bulk_store(static_cast<uint16_t*>(ch.param) + first, src, bytes);
                            const size_t off = static_cast<const char*>(ch.param) -
                                               ag.local_param_base + 2u * static_cast<size_t>(first);
                            for (int qq = 0; qq < ag.world; ++qq)
                                if (qq != ag.rank) bulk_store(ag.peer_param_base[qq] + off, src, bytes);
                            bulk_commit();
                        }
                        if (pb_data) pb_half ^= 1u;
                        pb_slot = 0;
                    } else {
                        ++pb_slot;
                    }
                }
                if (tid == 0) {
                    if (lv) {
                        const uint32_t base = smem_u32(st);
                        if constexpr (kMixed && !kPushBuf)
                            bulk_store(static_cast<uint16_t*>(ch.param) + t0, base, 2u * lv);
                        bulk_store(ch.master + t0, base + kOffMaster, 4u * lv);
                        if (use_m) bulk_store(ch.m + t0, base + kOffM, 4u * lv);
                        if constexpr (!kSgd) bulk_store(ch.v + t0, base + kOffV, 4u * lv);
                        if constexpr (kEma) bulk_store(ch.m + a.ema_delta + t0, base + kOffE, 4u * lv);
                        if constexpr (kAg && !kPushBuf) {
                            // the fused all-gather: the same param tile into every peer
                            const size_t off = static_cast<const char*>(ch.param) -
                                               ag.local_param_base +
                                               static_cast<size_t>(kGradBytes) * t0;
                            const uint32_t src = kMixed ? base : base + kOffMaster;
                            for (int qq = 0; qq < ag.world; ++qq)
                                if (qq != ag.rank)
                                    bulk_store(ag.peer_param_base[qq] + off, src, kGradBytes * lv);
                        }
                        bulk_commit();
                        if constexpr (kAg && kAgStoreLag > 0) {
                            // Peer stores read their tile out of shared memory at
                            // the link's pace. The stage is released kAgStoreLag
                            // tiles later, so those reads overlap the math of the
                            // next tiles instead of holding thread 0 (and with it
                            // every consumer) at this tile.
                            bulk_wait_read<kAgStoreLag>();
                            if (ag_np == kAgStoreLag)
                                mbar_arrive(smem_u32(&empty_bar[(q - kAgStoreLag) % kStages]));
                            else
                                ++ag_np;
                            return true;
                        }
                        bulk_wait_read_all();  // the stage may be refilled after this
                    } else if constexpr (kAg && kAgStoreLag > 0) {
                        if (ag_np) {
                            bulk_wait_read_all();
                            for (int j = 1; j <= ag_np; ++j)
                                mbar_arrive(smem_u32(&empty_bar[(q - j) % kStages]));
                            ag_np = 0;
                        }
                    }
                    mbar_arrive(smem_u32(&empty_bar[s]));
                }
                return true;
            };
            if constexpr (kDyn) {
                for (uint32_t q = 0;; ++q) {
                    const uint32_t s = q % kStages;
                    const bool ok = mbar_wait(smem_u32(&full_bar[s]), (q / kStages) & 1, &s_err);
                    if (!ok) s_cfail[q & 1] = 1;
                    const int2 w = s_tile[s];
                    const bool stop = !ok || w.x < 0;  // the same for every consumer that waited
                    const Chunk ch = s_chunk[s];
                    const uint32_t t0 = static_cast<uint32_t>(w.y);
                    const uint32_t len = stop ? 0u : min(static_cast<uint32_t>(kTile), ch.n - t0);
                    if (!tile(ch, t0, len, q, !stop, stop)) break;
                }
            } else {
                for_each_tile(chunks, n_vec, [&](const Chunk& ch, uint32_t t0, uint32_t len,
                                                 uint32_t q) {
                    const bool ok = mbar_wait(smem_u32(&full_bar[q % kStages]),
                                              (q / kStages) & 1, &s_err);
                    if (!ok) s_cfail[q & 1] = 1;
                    return tile(ch, t0, len, q, ok, !ok);
                });
            }
            if (tid == 0 || (kPushBuf && tid == kPusher)) bulk_wait_all();
            // scalar chunks (misaligned heads, mixed-phase tensors)
            for (int c = s_err ? n_chunks : n_vec + static_cast<int>(blockIdx.x); c < n_chunks; c += gridDim.x) {
                const Chunk ch = chunks[c];
                apply_scalar<kMixed, kAg, kEma, kSgd>(ch, 0, ch.n, tid, kConsumers, a, k,
                                                      __fmul_rn(a.lr, ch.wd), ch.wd != 0.0f, ag);
            }
        }
    }
    if constexpr (kAg) {
        // peer writes (bulk stores, waited above, and scalar stores) are
        // complete and visible system-wide before this CTA retires
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __threadfence_system();
    }
    __syncthreads();
    if (s_err && threadIdx.x == kConsumerWarps * 32) {
        // a wait timed out: let this CTA's own loads in flight land before exit
        const uint32_t qi = s_issued;
        for (uint32_t j = qi > kStages ? qi - kStages : 0; j < qi; ++j)
            mbar_wait(smem_u32(&full_bar[j % kStages]), (j / kStages) & 1, &s_drain_err);
        atomicOr(&ctl->error, 1);
    }
    if (threadIdx.x == 0) {
        StepDecision d;
        d.k = k;
        d.t = s_t;
        d.norm = s_norm;
        d.skip = s_skip;
        d.found = s_found;
        commit_step(ctl, a, d);
    }
}

// ---------------------------------------------------------------- K2 direct --

// One 4-element vector of a run: element offset e, n_valid (1..4) elements.
// Full vectors are 16-byte loads of the fp32 streams (8 bytes of bf16);
// the partial last vector of a run is loaded lane by lane.
template <bool kMixed>
__device__ __forceinline__ void direct_load(const DirectRun& r, uint64_t e, uint32_t n_valid,
                                            float4& g, float4& th, float4& m, float4& v) {
    if (n_valid == 4) {
        if constexpr (kMixed) {
            const uint2 q = __ldg(reinterpret_cast<const uint2*>(
                static_cast<const uint16_t*>(r.grad) + e));
            g = make_float4(bf16_lo(q.x), bf16_hi(q.x), bf16_lo(q.y), bf16_hi(q.y));
        } else {
            g = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(r.grad) + e));
        }
        th = *reinterpret_cast<const float4*>(r.master + e);
        m = *reinterpret_cast<const float4*>(r.m + e);
        v = *reinterpret_cast<const float4*>(r.v + e);
        return;
    }
    float gg[4] = {0.f, 0.f, 0.f, 0.f}, tt[4] = {0.f, 0.f, 0.f, 0.f},
          mm[4] = {0.f, 0.f, 0.f, 0.f}, vv[4] = {0.f, 0.f, 0.f, 0.f};
    for (uint32_t j = 0; j < n_valid; ++j) {
        gg[j] = kMixed ? bf16_bits_to_f32(static_cast<const uint16_t*>(r.grad)[e + j])
                       : static_cast<const float*>(r.grad)[e + j];
        tt[j] = r.master[e + j];
        mm[j] = r.m[e + j];
        vv[j] = r.v[e + j];
    }
    g = make_float4(gg[0], gg[1], gg[2], gg[3]);
    th = make_float4(tt[0], tt[1], tt[2], tt[3]);
    m = make_float4(mm[0], mm[1], mm[2], mm[3]);
    v = make_float4(vv[0], vv[1], vv[2], vv[3]);
}

template <bool kMixed>
__device__ __forceinline__ void direct_store(const DirectRun& r, uint64_t e, uint32_t n_valid,
                                             const float4& th, const float4& m, const float4& v) {
    if (n_valid == 4) {
        *reinterpret_cast<float4*>(r.master + e) = th;
        *reinterpret_cast<float4*>(r.m + e) = m;
        *reinterpret_cast<float4*>(r.v + e) = v;
        if constexpr (kMixed) {
            uint2 p;
            p.x = pack_bf16x2_rn(th.x, th.y);
            p.y = pack_bf16x2_rn(th.z, th.w);
            *reinterpret_cast<uint2*>(static_cast<uint16_t*>(r.param) + e) = p;
        }
        return;
    }
    const float tt[4] = {th.x, th.y, th.z, th.w}, mm[4] = {m.x, m.y, m.z, m.w},
                vv[4] = {v.x, v.y, v.z, v.w};
    for (uint32_t j = 0; j < n_valid; ++j) {
        r.master[e + j] = tt[j];
        r.m[e + j] = mm[j];
        r.v[e + j] = vv[j];
        if constexpr (kMixed) static_cast<uint16_t*>(r.param)[e + j] = f32_to_bf16_rn(tt[j]);
    }
}

// Register-fed AdamW step for short tensor lists (config 1, small config-5
// sizes), where the bulk-copy pipeline's set-up (prologue, ring fill, drain)
// is a large share of a step of a few microseconds. One pass: every thread
// issues the loads of its kDirectVecs vectors (grad, master, m, v) before
// the step decision is read, so the prologue's dependent reads (control
// block, bias-correction table) overlap the data in flight; then the same
// per-element arithmetic as k_apply (adamw_elem, explicitly rounded, the
// reference's order) and plain 16-byte stores. With the grid sized to the
// vectors, a list of a few million elements is a single wave. The run
// pointers come from the kernel parameters: no descriptor read precedes the
// data loads. Scalar chunks of the table (misaligned heads, mixed-phase
// tensors) follow, as in k_apply.
template <bool kMixed>
__global__ void __launch_bounds__(kDirectThreads, kDirectMinBlocks)
k_apply_direct(DirectRuns runs, const Chunk* __restrict__ chunks, int n_chunks, int n_vec,
               Ctl* __restrict__ ctl, ApplyArgs a) {
    __shared__ StepDecision s_d;
    pdl_wait();
    pdl_trigger();
    const uint32_t tid = threadIdx.x;
    const uint64_t total = runs.start[runs.n_runs];
    // Vector j of a pass is this thread's slot in the j-th grid-wide stripe,
    // so every thread of the (fully resident) grid gets its share and
    // consecutive threads read consecutive vectors.
    const uint64_t stripe = static_cast<uint64_t>(gridDim.x) * kDirectThreads;
    const uint64_t per_pass = stripe * kDirectVecs;

    // Vector vi -> run, element offset, valid elements (runs in kernel params).
    auto locate = [&](uint64_t vi, int& r, uint64_t& e, uint32_t& nv) {
        r = 0;
        while (r + 1 < runs.n_runs && vi >= runs.start[r + 1]) ++r;
        e = (vi - runs.start[r]) * 4u;
        const uint64_t left = runs.run[r].n - e;
        nv = left < 4u ? static_cast<uint32_t>(left) : 4u;
    };

    float4 g[kDirectVecs], th[kDirectVecs], m[kDirectVecs], v[kDirectVecs];
    int rr[kDirectVecs];
    uint64_t ee[kDirectVecs];
    uint32_t nn[kDirectVecs];
    auto load_pass = [&](uint64_t base) {
#pragma unroll
        for (int j = 0; j < kDirectVecs; ++j) {
            const uint64_t vi = base + static_cast<uint64_t>(j) * stripe;
            nn[j] = 0;
            if (vi < total) {
                locate(vi, rr[j], ee[j], nn[j]);
                direct_load<kMixed>(runs.run[rr[j]], ee[j], nn[j], g[j], th[j], m[j], v[j]);
            }
        }
    };

    uint64_t base = static_cast<uint64_t>(blockIdx.x) * kDirectThreads + tid;
    load_pass(base);  // in flight while thread 0 reads the step decision
    if (tid == 0) s_d = decide_step(a, ctl);
    __syncthreads();
    const StepCoeffs k = s_d.k;
    if (!s_d.skip) {
        for (;;) {
#pragma unroll
            for (int j = 0; j < kDirectVecs; ++j) {
                if (!nn[j]) continue;
                const DirectRun& r = runs.run[rr[j]];
                const float lr_wd = __fmul_rn(a.lr, r.wd);
                const bool has_wd = r.wd != 0.0f;
                adamw_elem(th[j].x, m[j].x, v[j].x, prep_grad(g[j].x, k), a, k, lr_wd, has_wd);
                adamw_elem(th[j].y, m[j].y, v[j].y, prep_grad(g[j].y, k), a, k, lr_wd, has_wd);
                adamw_elem(th[j].z, m[j].z, v[j].z, prep_grad(g[j].z, k), a, k, lr_wd, has_wd);
                adamw_elem(th[j].w, m[j].w, v[j].w, prep_grad(g[j].w, k), a, k, lr_wd, has_wd);
                direct_store<kMixed>(r, ee[j], nn[j], th[j], m[j], v[j]);
            }
            base += per_pass;
            if (base - tid >= total) break;  // the CTA's lowest vector: all threads leave together
            load_pass(base);
        }
        // scalar chunks (misaligned heads, mixed-phase tensors)
        const AgArgs none{};
        for (int c = n_vec + static_cast<int>(blockIdx.x); c < n_chunks; c += gridDim.x) {
            const Chunk ch = chunks[c];
            apply_scalar<kMixed, false, false, false>(ch, 0, ch.n, tid, kDirectThreads, a, k,
                                                      __fmul_rn(a.lr, ch.wd), ch.wd != 0.0f,
                                                      none);
        }
    }
    __syncthreads();
    if (tid == 0) commit_step(ctl, a, s_d);
}

// ------------------------------------------------------------ small kernels --

// In-place fp32 clip of the gradients (adamw.cpp:45-51).
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

__global__ void k_f32_to_bf16(const float* __restrict__ src, uint16_t* __restrict__ dst,
                              uint64_t n) {
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        dst[i] = f32_to_bf16_rn(src[i]);
}

// Self-test of the bounded wait every pipeline uses: one thread waits on an
// mbarrier that nothing will ever arrive at, with a short limit, and reports
// whether it gave up and how long it waited. Nothing faults or hangs.
__global__ void k_wait_selftest(uint64_t limit_ns, int* out_error, unsigned long long* out_ns) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int s_err;
    if (threadIdx.x == 0) {
        s_err = 0;
        mbar_init(smem_u32(&bar), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        const uint64_t t0 = global_timer_ns();
        const bool ok = mbar_wait(smem_u32(&bar), 0, &s_err, limit_ns);  // phase 0 never completes
        *out_ns = global_timer_ns() - t0;
        *out_error = ok ? 0 : s_err;
        // retire the barrier's pending phase so the CTA exits with it consistent
        mbar_arrive(smem_u32(&bar));
    }
}

struct SignalPtrs {
    Signals* q[kMaxRanks];
};

__global__ void k_step_done(SignalPtrs sig, int world, int rank, uint64_t epoch, int* err) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x != 0) return;
    // this rank's peer parameter stores finished with the previous kernel
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int q = 0; q < world; ++q) st_release_sys(&sig.q[q]->done[rank], epoch);
    wait_flags(sig.q[rank]->done, world, epoch, err);
}

__global__ void k_set_counters(Ctl* ctl, uint64_t t, uint64_t skipped, float scale,
                               int32_t tracker) {
    ctl->t = t;
    ctl->skipped = skipped;
    ctl->scale = scale;
    ctl->tracker = tracker;
    ctl->error = 0;
}

}  // namespace

// --------------------------------------------------------------- launchers --

template <bool kMixed, bool kAg, bool kEma, bool kSgd, bool kDyn>
static cudaError_t set_smem_attr() {
    return cudaFuncSetAttribute(k_apply<kMixed, kAg, kEma, kSgd, kDyn>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(apply_smem_bytes(kMixed, kEma, kSgd, kAg)));
}

template <bool kMixed, bool kAg, bool kEma, bool kSgd, bool kDyn>
static void launch_apply_t(const Chunk* chunks, int n_chunks, int n_vec, Ctl* ctl,
                           const ApplyArgs& args, int grid, cudaStream_t stream, const AgArgs& ag) {
    launch_pdl(k_apply<kMixed, kAg, kEma, kSgd, kDyn>, dim3(grid), dim3(kApplyThreads),
               apply_smem_bytes(kMixed, kEma, kSgd, kAg), stream, chunks, n_chunks, n_vec, ctl,
               args, ag);
}

// The 32 instantiations, indexed by (mixed, ag, ema, sgd, dyn) bits.
using SetFn = cudaError_t (*)();
using LaunchFn = void (*)(const Chunk*, int, int, Ctl*, const ApplyArgs&, int, cudaStream_t,
                          const AgArgs&);
#define SOARB_VARIANT(b)                                                                    \
    {set_smem_attr<(b & 16) != 0, (b & 8) != 0, (b & 4) != 0, (b & 2) != 0, (b & 1) != 0>, \
     launch_apply_t<(b & 16) != 0, (b & 8) != 0, (b & 4) != 0, (b & 2) != 0, (b & 1) != 0>}
struct Variant {
    SetFn set;
    LaunchFn launch;
};
static const Variant kVariants[32] = {
    SOARB_VARIANT(0),  SOARB_VARIANT(1),  SOARB_VARIANT(2),  SOARB_VARIANT(3),
    SOARB_VARIANT(4),  SOARB_VARIANT(5),  SOARB_VARIANT(6),  SOARB_VARIANT(7),
    SOARB_VARIANT(8),  SOARB_VARIANT(9),  SOARB_VARIANT(10), SOARB_VARIANT(11),
    SOARB_VARIANT(12), SOARB_VARIANT(13), SOARB_VARIANT(14), SOARB_VARIANT(15),
    SOARB_VARIANT(16), SOARB_VARIANT(17), SOARB_VARIANT(18), SOARB_VARIANT(19),
    SOARB_VARIANT(20), SOARB_VARIANT(21), SOARB_VARIANT(22), SOARB_VARIANT(23),
    SOARB_VARIANT(24), SOARB_VARIANT(25), SOARB_VARIANT(26), SOARB_VARIANT(27),
    SOARB_VARIANT(28), SOARB_VARIANT(29), SOARB_VARIANT(30), SOARB_VARIANT(31)};
#undef SOARB_VARIANT

static int variant_index(bool mixed, bool ag, bool ema, bool sgd, bool dyn) {
    return (mixed ? 16 : 0) | (ag ? 8 : 0) | (ema ? 4 : 0) | (sgd ? 2 : 0) | (dyn ? 1 : 0);
}

cudaError_t prepare_kernels() {
    for (const Variant& v : kVariants) {
        const cudaError_t e = v.set();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_grad_sumsq(bool bf16, const Chunk* chunks, int n_chunks, Ctl* ctl,
                              double* partials, int grid, int use_scaler, double* out,
                              cudaStream_t stream) {
    const cudaError_t e =
        bf16 ? launch_pdl(k_grad_sumsq<true>, dim3(grid), dim3(kThreads), 0, stream, chunks,
                          n_chunks, ctl, partials, use_scaler, out)
             : launch_pdl(k_grad_sumsq<false>, dim3(grid), dim3(kThreads), 0, stream, chunks,
                          n_chunks, ctl, partials, use_scaler, out);
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_apply(bool mixed, const Chunk* chunks, int n_chunks, int n_vec, Ctl* ctl,
                         const ApplyArgs& args, int grid, cudaStream_t stream, const AgArgs* ag,
                         bool ema, bool sgd, bool dyn) {
    const AgArgs none{};
    kVariants[variant_index(mixed, ag != nullptr, ema, sgd, dyn)].launch(
        chunks, n_chunks, n_vec, ctl, args, grid, stream, ag ? *ag : none);
    return cudaGetLastError();
}

cudaError_t launch_apply_direct(bool mixed, const DirectRuns& runs, const Chunk* chunks,
                                int n_chunks, int n_vec, Ctl* ctl, const ApplyArgs& args,
                                int grid, cudaStream_t stream) {
    const cudaError_t e =
        mixed ? launch_pdl(k_apply_direct<true>, dim3(grid), dim3(kDirectThreads), 0, stream,
                           runs, chunks, n_chunks, n_vec, ctl, args)
              : launch_pdl(k_apply_direct<false>, dim3(grid), dim3(kDirectThreads), 0, stream,
                           runs, chunks, n_chunks, n_vec, ctl, args);
    return e != cudaSuccess ? e : cudaGetLastError();
}

int occupancy_apply_direct(bool mixed) {
    int n = 0;
    if (mixed)
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_apply_direct<true>, kDirectThreads, 0);
    else
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_apply_direct<false>, kDirectThreads, 0);
    return n > 0 ? n : 1;
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

cudaError_t launch_f32_to_bf16(const float* src, uint16_t* dst, uint64_t n,
                               cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    uint64_t blocks = (n + kThreads - 1) / kThreads;
    if (blocks > 4096) blocks = 4096;
    k_f32_to_bf16<<<static_cast<unsigned>(blocks), kThreads, 0, stream>>>(src, dst, n);
    return cudaGetLastError();
}

cudaError_t launch_set_counters(Ctl* ctl, uint64_t t, uint64_t skipped, float scale,
                                int32_t tracker, cudaStream_t stream) {
    k_set_counters<<<1, 1, 0, stream>>>(ctl, t, skipped, scale, tracker);
    return cudaGetLastError();
}

cudaError_t launch_step_done(Signals* const* sig, int world, int rank, uint64_t epoch, int* err,
                             cudaStream_t stream) {
    SignalPtrs p{};
    for (int q = 0; q < world && q < kMaxRanks; ++q) p.q[q] = sig[q];
    const cudaError_t e = launch_pdl(k_step_done, dim3(1), dim3(32), 0, stream, p, world, rank,
                                     epoch, err);
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_wait_selftest(uint64_t limit_ns, int* out_error, unsigned long long* out_ns,
                                 cudaStream_t stream) {
    k_wait_selftest<<<1, 32, 0, stream>>>(limit_ns, out_error, out_ns);
    return cudaGetLastError();
}

cudaError_t apply_kernel_attributes(cudaFuncAttributes* out) {
    return cudaFuncGetAttributes(out, k_apply<true, false, false, false, false>);
}

int occupancy_grad_sumsq(bool bf16) {
    int n = 0;
    if (bf16)
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_grad_sumsq<true>, kThreads, 0);
    else
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_grad_sumsq<false>, kThreads, 0);
    return n > 0 ? n : 1;
}

template <bool kMixed, bool kEma, bool kSgd>
static int occupancy_t() {
    int n = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_apply<kMixed, false, kEma, kSgd, false>,
                                                  kApplyThreads,
                                                  apply_smem_bytes(kMixed, kEma, kSgd));
    return n;
}

int occupancy_apply(bool mixed, bool ema, bool sgd) {
    int n;
    switch ((mixed ? 4 : 0) | (ema ? 2 : 0) | (sgd ? 1 : 0)) {
        case 0: n = occupancy_t<false, false, false>(); break;
        case 1: n = occupancy_t<false, false, true>(); break;
        case 2: n = occupancy_t<false, true, false>(); break;
        case 3: n = occupancy_t<false, true, true>(); break;
        case 4: n = occupancy_t<true, false, false>(); break;
        case 5: n = occupancy_t<true, false, true>(); break;
        case 6: n = occupancy_t<true, true, false>(); break;
        default: n = occupancy_t<true, true, true>(); break;
    }
    return n > 0 ? n : 1;
}

}  // namespace soarb
