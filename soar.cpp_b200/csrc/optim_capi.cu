// Host side of the optimizer-step C-ABI (include/soar_optim.h).
//
// Owns, per optimizer, one device slab carved DeviceSlab-style (aligned bump
// offsets over a single cudaMalloc; the reference's DeviceSlabSubAllocator,
// src/memory/device_slab.cpp:6-38) holding the fp32 master weights, m, v, the
// chunk table, the per-CTA reduction partials and the step control block.
// Builds the tensor-list chunk table once at create time, so a step is two
// kernel launches with no host work beyond filling the launch arguments.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <map>
#include <cstdint>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/soar_optim.h"
#include "optim_kernels.cuh"

namespace {

thread_local std::string g_last_error;

int fail(const std::string& msg) {
    g_last_error = msg;
    return SOAR_ERROR;
}

#define SOAR_CUDA_TRY(expr)                                                              \
    do {                                                                                 \
        cudaError_t e_ = (expr);                                                         \
        if (e_ != cudaSuccess) return fail(std::string(#expr) + ": " + cudaGetErrorString(e_)); \
    } while (0)

// Makes the optimizer's device current for the scope of one call.
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

constexpr size_t kSlabAlign = 256;
constexpr uint32_t kBcCap = 1u << 22;  // bias-correction table entries before it must converge

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct TensorRec {
    void* param;
    void* grad;
    uint64_t numel;
    float wd;
    uint64_t state_off;  // element offset of this tensor's master/m/v slices
    uint64_t vec_from;   // first element of the 16-byte-aligned vector part (numel: none)
};

// Lists of at most kDirectMaxRuns tensors with a vector part and at most this
// many elements update with the register-fed kernel (k_apply_direct) instead
// of the bulk-copy pipeline: there a step lasts a few to tens of
// microseconds and the pipeline's set-up and drain are a large share of it.
// Measured on B200 (one flat tensor, plain update): the direct kernel is
// faster at 1M-16M elements in both layouts (1M fp32 back to back: 6.7 vs
// 9.7 us; 8M: 39.5 vs 41.3 us) and the pipeline from 32M on.
#ifndef SOAR_DIRECT_MAX_ELEMS
#define SOAR_DIRECT_MAX_ELEMS (16ull << 20)
#endif
constexpr uint64_t kDirectMaxElems = SOAR_DIRECT_MAX_ELEMS;

// One set of gradient buffers for the optimizer's tensors, with the chunk
// tables (and direct-kernel runs) that point into it. Set 0 is the one given
// at create time; more are added with soar_optim_add_grads.
struct GradSet {
    std::vector<void*> grads;
    soarb::Chunk* chunks = nullptr;        // update table (device)
    soarb::Chunk* sumsq_chunks = nullptr;  // norm-pass table (device)
    soarb::DirectRuns druns{};
    void* alloc = nullptr;                 // device block of an added set's tables
};

struct Optim {
    int device = 0;
    bool mixed = false;
    bool sgd = false;            // SGD (momentum buffer in m) instead of AdamW
    float momentum = 0.0f, dampening = 0.0f;
    bool nesterov = false;
    soar_adamw_opts opts{};
    float lr = 1e-3f;
    float pending_coef = 1.0f;   // from a standalone clip_grad_norm (mixed layout)
    float async_clip = 0.0f;     // > 0: clip_grad_norm_async enqueued the norm pass; the
                                 // next step clips by this norm from Ctl::sumsq
    uint64_t host_calls = 0;     // step() calls issued: an upper bound of the device t

    std::vector<TensorRec> tensors;
    uint64_t state_elems = 0;

    char* slab = nullptr;
    float* master = nullptr;     // mixed only
    float* m = nullptr;
    float* v = nullptr;
    soarb::Chunk* chunks = nullptr;
    int n_chunks = 0;
    int n_vec = 0;               // vector chunks come first in the table
    bool dyn = false;            // the update hands chunks out dynamically (see choose_dynamic)
    double* partials = nullptr;
    soarb::Ctl* ctl = nullptr;
    double* sumsq_scratch = nullptr;
    soar_step_info* info_stage = nullptr;  // device staging of soar_optim_get_info_async

    float* ema = nullptr;        // weight-EMA shadow (separate allocation, state layout)
    float ema_decay = 0.0f;
    float2* bc = nullptr;        // separate allocation (it can grow)
    uint32_t bc_len = 0;
    bool bc_converged = false;

    int grid_sumsq = 1;
    int grid_apply = 1;
    bool direct = false;         // update with k_apply_direct (short lists)
    soarb::DirectRuns druns{};   // of the gradient set in use
    int grid_direct = 1;
    std::vector<GradSet> grad_sets;
    int grad_set = 0;            // the set step / clip / zero_grad use
    uint32_t chunk_elems = soarb::kChunkElems;  // adaptive: see choose_chunk_elems
    std::vector<soarb::Chunk> host_chunks;
    // The norm pass and the in-place fp32 clip walk the table before the tail
    // was cut into pieces (k_grad_sumsq keeps several loads in flight per
    // thread only on full-length chunks); same layout, same invariants.
    soarb::Chunk* sumsq_chunks = nullptr;
    int n_sumsq_chunks = 0;
    std::vector<soarb::Chunk> host_sumsq_chunks;
};

struct Cosine {
    Optim* opt;
    float base_lr;
    float eta_min;
    uint64_t total_steps;
    uint64_t warmup_steps;
    uint64_t current_step = 0;
};

size_t elem_bytes(const Optim& o) { return o.mixed ? 2 : 4; }

// bc[t] = (1 - beta1^t, sqrt(1 - beta2^t)) with the reference's own host
// expressions (adamw.cpp:68-70), so the device reads the reference's bits.
std::vector<float2> bias_table(float beta1, float beta2, uint32_t len, bool* converged) {
    std::vector<float2> tab(len);
    tab[0] = make_float2(1.0f, 1.0f);  // t = 0 is never used
    *converged = false;
    uint32_t ones_run = 0;
    for (uint32_t t = 1; t < len; ++t) {
        const float bias_correction1 = 1.0f - std::pow(beta1, static_cast<float>(t));
        const float bias_correction2 = 1.0f - std::pow(beta2, static_cast<float>(t));
        tab[t] = make_float2(bias_correction1, std::sqrt(bias_correction2));
        ones_run = (bias_correction1 == 1.0f && bias_correction2 == 1.0f) ? ones_run + 1 : 0;
        // Both corrections are exactly 1 from here on (beta^t only shrinks);
        // keep 4096 such entries as a margin and stop.
        if (ones_run == 4096) {
            tab.resize(t + 1);
            *converged = true;
            break;
        }
    }
    return tab;
}

int upload_bias_table(Optim& o, uint32_t len) {
    bool conv = false;
    std::vector<float2> tab = bias_table(o.opts.beta1, o.opts.beta2, len, &conv);
    float2* d = nullptr;
    SOAR_CUDA_TRY(cudaMalloc(&d, tab.size() * sizeof(float2)));
    cudaError_t e = cudaMemcpy(d, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(d);
        return fail(std::string("bias table upload: ") + cudaGetErrorString(e));
    }
    if (o.bc) {
        cudaDeviceSynchronize();  // earlier steps may still read the old table
        cudaFree(o.bc);
    }
    o.bc = d;
    o.bc_len = static_cast<uint32_t>(tab.size());
    o.bc_converged = conv;
    return SOAR_OK;
}

// Splits every tensor with a gradient into chunks.
//
// A tensor whose param and grad share the same phase modulo 16 bytes is cut
// at absolute grad-address boundaries: chunk starts fall where the grad
// address is a multiple of the chunk size in bytes (16384 elements; for
// tensors under 8 chunks, of the 1024-element tile), and its fp32 state
// slices are placed so the same element index is aligned in the state arrays
// too. Bulk copies of a tile then never straddle the tile-sized boundaries of
// any stream, which measurably keeps HBM at full rate (misaligned 25M buckets
// lost ~7 % in k_apply). The ragged start before the first boundary becomes a
// scalar head (< 16 bytes of elements) plus one shorter vector chunk.
//
// A tensor whose param and grad phases differ runs the scalar path. Vector
// chunks go first in the table (they feed the bulk-copy pipeline), scalar
// chunks after them.
// Chunk length: about 8 chunks per update CTA so small tensor lists still
// spread over every SM and k_grad_sumsq's grid-stride tail stays short, a power of two
// between one tile and kChunkElems (large lists keep kChunkElems).
uint32_t choose_chunk_elems(uint64_t total_elems, int grid) {
    const uint64_t target = total_elems / (8ull * static_cast<uint64_t>(std::max(grid, 1)));
    uint32_t c = soarb::kChunkElems;
    while (c > static_cast<uint32_t>(soarb::kTile) && c > target) c >>= 1;
    return c;
}

void build_chunks(Optim& o) {
    const size_t eb = elem_bytes(o);
    const uint32_t kChunk = o.chunk_elems;
    std::vector<soarb::Chunk> vec, scalar;
    uint64_t cursor = 0;
    for (size_t ti = 0; ti < o.tensors.size(); ++ti) {
        TensorRec& t = o.tensors[ti];
        const uintptr_t pa = reinterpret_cast<uintptr_t>(t.param);
        const uintptr_t ga = reinterpret_cast<uintptr_t>(t.grad);
        const uint64_t pphase = (pa % soarb::kVecBytes) / eb;
        const uint64_t gphase = t.grad ? (ga % soarb::kVecBytes) / eb : pphase;
        const bool vec_ok = t.grad && t.numel > 0 && pphase == gphase;
        uint64_t h16 = 0, e0 = 0;  // first 16-byte aligned index, first boundary index
        if (vec_ok) {
            const uint64_t align_elems = t.numel >= 8ull * kChunk ? kChunk : soarb::kTile;
            const uint64_t ab = align_elems * eb;
            const uint64_t h16_raw = ((soarb::kVecBytes - ga % soarb::kVecBytes) % soarb::kVecBytes) / eb;
            const uint64_t e0_raw = ((ab - ga % ab) % ab) / eb;  // >= h16_raw, same phase mod 16 B
            // Element e0_raw sits on an align_elems boundary of the state arrays.
            // Placing by the unclipped index keeps every 16-byte aligned grad
            // position 16-byte aligned in the state too, also when the tensor
            // ends before its first boundary.
            t.state_off = align_up(cursor + e0_raw, align_elems) - e0_raw;
            h16 = std::min<uint64_t>(h16_raw, t.numel);
            e0 = std::min<uint64_t>(e0_raw, t.numel);
            t.vec_from = h16;
        } else {
            // 256-byte aligned slice start, shifted by the param's element phase
            t.state_off = align_up(cursor, 64) + pphase;
            t.vec_from = t.numel;
        }
        cursor = t.state_off + t.numel;
        if (!t.grad || t.numel == 0) continue;
        auto add = [&](uint64_t start, uint64_t len, bool is_vec) {
            soarb::Chunk c{};
            c.param = static_cast<char*>(t.param) + start * eb;
            c.grad = static_cast<const char*>(t.grad) + start * eb;
            c.n = static_cast<uint32_t>(len);
            c.wd = t.wd;
            c.flags = is_vec ? soarb::kChunkVec : 0u;
            c.tensor = static_cast<uint32_t>(ti);
            // master/m/v pointers are filled once the slab exists
            c.master = reinterpret_cast<float*>(static_cast<uintptr_t>(t.state_off + start));
            (is_vec ? vec : scalar).push_back(c);
        };
        auto add_run = [&](uint64_t from, uint64_t to, bool is_vec) {
            for (uint64_t s = from; s < to; s += kChunk)
                add(s, std::min<uint64_t>(kChunk, to - s), is_vec);
        };
        if (!vec_ok) {
            add_run(0, t.numel, false);
            continue;
        }
        add_run(0, h16, false);         // < 16 bytes before the first aligned element
        add_run(h16, e0, true);         // aligned, up to the first chunk boundary
        add_run(e0, t.numel, true);     // boundary-aligned chunks
    }
    o.state_elems = align_up(cursor, 64);
    o.n_vec = static_cast<int>(vec.size());
    o.host_chunks = std::move(vec);
    o.host_chunks.insert(o.host_chunks.end(), scalar.begin(), scalar.end());
}

// Whether the update hands its chunks out dynamically (one atomic per chunk)
// or walks them statically (grid-strided). Measured on B200: the fp32 layout
// is faster dynamic at every size (+10 % at 16M-256M params, +12 % on
// config 2); the bf16-mixed layout is faster static on a few large tensors
// (config 4: 0.865 vs 0.875 ms; one 256M tensor: 1.10 vs 1.15 ms) but dynamic
// on long lists of unequal tensors (config 3's 400 tensors: 0.251 vs
// 0.271 ms), where a static walk leaves some CTAs with more work.
bool choose_dynamic(const Optim& o, int grid) {
    if (!o.mixed) return true;
    int with_grad = 0;
    uint64_t total = 0;
    for (const TensorRec& t : o.tensors)
        if (t.grad && t.numel) {
            ++with_grad;
            total += t.numel;
        }
    // one to four tensors (the config-5 shape): dynamic measured ~3-4 % faster at
    // 16M-64M params, static faster at <= 4M (fewer atomics per tile) and at
    // >= 200M. (ZeRO-1 shards, a handful of bucket slices, keep the static walk
    // measured on NVLink.)
    constexpr uint64_t kDynLo = 8ull << 20, kDynHi = 96ull << 20;
    return with_grad >= std::max(grid, 1) / 4 ||
           (with_grad <= 4 && total >= kDynLo && total < kDynHi);
}

// The dynamic hand-out goes from the top of the vector part of the table
// down, so the chunks at its bottom are the last to be taken. Cut those into
// short pieces (two tiles) until they hold kTailTilesPerCta tiles per update
// CTA: the end of the step then balances at the granularity of a piece rather
// than of a whole chunk, whatever the CTAs' relative speeds. The pieces start
// at tile multiples of a vector chunk's start, so they stay 16-byte aligned
// in every stream.
constexpr uint64_t kTailTilesPerCta = 24;

void split_tail(Optim& o, int grid) {
    const size_t eb = elem_bytes(o);
    const uint64_t piece = std::min<uint64_t>(2ull * soarb::kTile, o.chunk_elems);
    const uint64_t want = kTailTilesPerCta * static_cast<uint64_t>(std::max(grid, 1));
    std::vector<soarb::Chunk> out;
    int k = 0;
    uint64_t tiles = 0;
    for (; k < o.n_vec && tiles < want; ++k) {
        const soarb::Chunk& c = o.host_chunks[k];
        for (uint64_t s = 0; s < c.n; s += piece) {
            soarb::Chunk p = c;
            p.n = static_cast<uint32_t>(std::min<uint64_t>(piece, c.n - s));
            p.param = static_cast<char*>(c.param) + s * eb;
            p.grad = static_cast<const char*>(c.grad) + s * eb;
            // still the state offset (pointers are filled once the slab exists)
            p.master = reinterpret_cast<float*>(reinterpret_cast<uintptr_t>(c.master) + s);
            out.push_back(p);
        }
        tiles += (c.n + soarb::kTile - 1) / soarb::kTile;
    }
    const int pieces = static_cast<int>(out.size());
    out.insert(out.end(), o.host_chunks.begin() + k, o.host_chunks.end());
    o.n_vec += pieces - k;
    o.host_chunks = std::move(out);
}

// Host-side check of the invariants the bulk-copy pipeline relies on, run on
// the final chunk table before it is uploaded: every vector chunk is
// non-empty, at most kChunkElems long, and all five of its streams start on a
// 16-byte boundary (tile offsets are multiples of kTile elements, so every
// tile of the chunk is then aligned too).
bool chunks_valid(const Optim& o, std::string* why) {
    auto a16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % soarb::kVecBytes == 0; };
    for (int i = 0; i < static_cast<int>(o.host_chunks.size()); ++i) {
        const soarb::Chunk& c = o.host_chunks[i];
        const bool vec = (c.flags & soarb::kChunkVec) != 0;
        if (vec != (i < o.n_vec)) {
            *why = "chunk " + std::to_string(i) + ": vector chunks must lead the table";
            return false;
        }
        if (c.n == 0 || c.n > o.chunk_elems) {
            *why = "chunk " + std::to_string(i) + ": bad length";
            return false;
        }
        if (vec && !(a16(c.param) && a16(c.grad) && a16(c.master) && a16(c.m) && a16(c.v))) {
            *why = "chunk " + std::to_string(i) + ": vector chunk not 16-byte aligned";
            return false;
        }
    }
    return true;
}

// The direct kernel's runs: the vector part [vec_from, numel) of every
// tensor with a gradient (exactly the elements the table's vector chunks
// cover), for the gradient buffers `grads`. Returns false when the list has
// more runs than the kernel takes.
bool build_direct_runs(const Optim& o, const std::vector<void*>& grads, soarb::DirectRuns* out) {
    soarb::DirectRuns r{};
    const size_t eb = elem_bytes(o);
    uint64_t vecs = 0;
    for (size_t i = 0; i < o.tensors.size(); ++i) {
        const TensorRec& t = o.tensors[i];
        if (!grads[i] || t.vec_from >= t.numel) continue;
        if (r.n_runs == soarb::kDirectMaxRuns) return false;
        soarb::DirectRun& d = r.run[r.n_runs];
        d.param = static_cast<char*>(t.param) + t.vec_from * eb;
        d.grad = static_cast<const char*>(grads[i]) + t.vec_from * eb;
        d.master = o.mixed ? o.master + t.state_off + t.vec_from
                           : static_cast<float*>(t.param) + t.vec_from;
        d.m = o.m + t.state_off + t.vec_from;
        d.v = o.v + t.state_off + t.vec_from;
        d.n = t.numel - t.vec_from;
        d.wd = t.wd;
        r.start[r.n_runs] = vecs;
        vecs += (d.n + 3) / 4;
        ++r.n_runs;
    }
    r.start[r.n_runs] = vecs;
    *out = r;
    return true;
}

struct SgdParams {
    float momentum, dampening;
    bool nesterov;
};

int create_impl(const soar_tensor_desc* tensors, int n, const soar_adamw_opts* opts,
                void** out, const SgdParams* sgd = nullptr) {
    if (!opts || !out || n < 0 || (n > 0 && !tensors)) return fail("null argument");
    *out = nullptr;
    if (opts->layout != SOAR_LAYOUT_FP32 && opts->layout != SOAR_LAYOUT_BF16_MIXED)
        return fail("unknown layout");
    if (opts->use_loss_scaler && !(opts->init_scale > 0.0f)) return fail("init_scale must be > 0");
    if (opts->use_loss_scaler && opts->growth_interval <= 0) return fail("growth_interval must be > 0");

    auto* o = new Optim();
    o->opts = *opts;
    if (sgd) {
        o->sgd = true;
        o->momentum = sgd->momentum;
        o->dampening = sgd->dampening;
        o->nesterov = sgd->nesterov;
    }
    o->device = opts->device;
    o->mixed = opts->layout == SOAR_LAYOUT_BF16_MIXED;
    o->lr = opts->lr;
    const size_t eb = elem_bytes(*o);
    for (int i = 0; i < n; ++i) {
        const soar_tensor_desc& d = tensors[i];
        if (d.numel > 0 && !d.param) {
            delete o;
            return fail("tensor " + std::to_string(i) + ": null param");
        }
        if ((reinterpret_cast<uintptr_t>(d.param) % eb) || (reinterpret_cast<uintptr_t>(d.grad) % eb)) {
            delete o;
            return fail("tensor " + std::to_string(i) + ": pointer not aligned to its element size");
        }
        o->tensors.push_back({d.param, d.grad, d.numel, d.weight_decay, 0, d.numel});
    }

    DeviceGuard g(o->device);
    if (!g.ok) {
        delete o;
        return fail("cannot select device " + std::to_string(opts->device));
    }
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, o->device) != cudaSuccess ||
        sms <= 0) {
        delete o;
        return fail("cannot query the SM count");
    }
    if (cudaError_t pe = soarb::prepare_kernels(); pe != cudaSuccess) {
        delete o;
        return fail(std::string("kernel set-up: ") + cudaGetErrorString(pe));
    }
    {
        uint64_t total = 0;
        for (const TensorRec& t : o->tensors)
            if (t.grad) total += t.numel;
        o->chunk_elems =
            choose_chunk_elems(total, sms * soarb::occupancy_apply(o->mixed, false, o->sgd));
    }
    build_chunks(*o);
    o->host_sumsq_chunks = o->host_chunks;
    o->n_sumsq_chunks = static_cast<int>(o->host_sumsq_chunks.size());
    {
        const int grid = sms * soarb::occupancy_apply(o->mixed, false, o->sgd);
        o->dyn = choose_dynamic(*o, grid);
        if (o->dyn) split_tail(*o, grid);  // (the static walk measured faster on whole chunks)
    }
    o->n_chunks = static_cast<int>(o->host_chunks.size());
    const int cap = std::max(1, o->n_chunks);
    o->grid_sumsq =
        std::min(sms * soarb::occupancy_grad_sumsq(o->mixed), std::max(1, o->n_sumsq_chunks));
    o->grid_apply = std::min(sms * soarb::occupancy_apply(o->mixed, false, o->sgd), cap);

    // Slab: [master | m | v | chunks | partials | ctl | clip scratch]
    const size_t state_bytes = o->state_elems * sizeof(float);
    size_t off = 0;
    const size_t off_master = off;
    if (o->mixed) off = align_up(off + state_bytes, kSlabAlign);
    const size_t off_m = off;
    off = align_up(off + state_bytes, kSlabAlign);
    const size_t off_v = off;
    if (!o->sgd) off = align_up(off + state_bytes, kSlabAlign);  // SGD has no second moment
    const size_t off_chunks = off;
    off = align_up(off + o->host_chunks.size() * sizeof(soarb::Chunk), kSlabAlign);
    const size_t off_sumsq_chunks = off;
    off = align_up(off + o->host_sumsq_chunks.size() * sizeof(soarb::Chunk), kSlabAlign);
    const size_t off_partials = off;
    off = align_up(off + o->grid_sumsq * sizeof(double), kSlabAlign);
    const size_t off_ctl = off;
    off = align_up(off + sizeof(soarb::Ctl), kSlabAlign);
    const size_t off_scratch = off;
    off = align_up(off + sizeof(double), kSlabAlign);
    const size_t off_info = off;
    off = align_up(off + sizeof(soar_step_info), kSlabAlign);

    cudaError_t e = cudaMalloc(&o->slab, off);
    if (e != cudaSuccess) {
        delete o;
        return fail(std::string("optimizer slab (") + std::to_string(off) + " bytes): " +
                    cudaGetErrorString(e));
    }
    o->master = o->mixed ? reinterpret_cast<float*>(o->slab + off_master) : nullptr;
    o->m = reinterpret_cast<float*>(o->slab + off_m);
    o->v = o->sgd ? nullptr : reinterpret_cast<float*>(o->slab + off_v);
    o->chunks = reinterpret_cast<soarb::Chunk*>(o->slab + off_chunks);
    o->sumsq_chunks = reinterpret_cast<soarb::Chunk*>(o->slab + off_sumsq_chunks);
    o->partials = reinterpret_cast<double*>(o->slab + off_partials);
    o->ctl = reinterpret_cast<soarb::Ctl*>(o->slab + off_ctl);
    o->sumsq_scratch = reinterpret_cast<double*>(o->slab + off_scratch);
    o->info_stage = reinterpret_cast<soar_step_info*>(o->slab + off_info);

    for (auto* table : {&o->host_chunks, &o->host_sumsq_chunks}) {
        for (soarb::Chunk& c : *table) {
            const uint64_t s = static_cast<uint64_t>(reinterpret_cast<uintptr_t>(c.master));
            c.master = o->mixed ? o->master + s : static_cast<float*>(c.param);
            c.m = o->m + s;
            c.v = o->sgd ? nullptr : o->v + s;
        }
    }

    auto cleanup = [&](const std::string& msg) {
        cudaFree(o->slab);
        if (o->bc) cudaFree(o->bc);
        delete o;
        return fail(msg);
    };
    {
        std::string why;
        if (!chunks_valid(*o, &why)) return cleanup("internal chunk-table check failed: " + why);
    }
    if ((e = cudaMemcpy(o->chunks, o->host_chunks.data(),
                        o->host_chunks.size() * sizeof(soarb::Chunk), cudaMemcpyHostToDevice)) !=
            cudaSuccess ||
        (e = cudaMemcpy(o->sumsq_chunks, o->host_sumsq_chunks.data(),
                        o->host_sumsq_chunks.size() * sizeof(soarb::Chunk),
                        cudaMemcpyHostToDevice)) != cudaSuccess)
        return cleanup(std::string("chunk table upload: ") + cudaGetErrorString(e));
    if ((e = cudaMemset(o->m, 0, state_bytes)) != cudaSuccess ||
        (o->v && (e = cudaMemset(o->v, 0, state_bytes)) != cudaSuccess))
        return cleanup(std::string("state zero-fill: ") + cudaGetErrorString(e));
    soarb::Ctl ctl{};
    ctl.scale = opts->use_loss_scaler ? opts->init_scale : 1.0f;
    ctl.last_clip_coef = 1.0f;
    ctl.last_lr = opts->lr;
    if ((e = cudaMemcpy(o->ctl, &ctl, sizeof ctl, cudaMemcpyHostToDevice)) != cudaSuccess)
        return cleanup(std::string("control block upload: ") + cudaGetErrorString(e));
    if (o->mixed) {
        // master = float(bf16 param): exact
        if ((e = cudaMemset(o->master, 0, state_bytes)) != cudaSuccess)
            return cleanup(std::string("master zero-fill: ") + cudaGetErrorString(e));
        for (const TensorRec& t : o->tensors) {
            if (!t.numel) continue;
            if ((e = soarb::launch_bf16_to_f32(static_cast<const uint16_t*>(t.param),
                                               o->master + t.state_off, t.numel, nullptr)) !=
                cudaSuccess)
                return cleanup(std::string("master init: ") + cudaGetErrorString(e));
        }
    }
    {
        // sized for the first 64K steps, grown on demand until it converges
        const int rc = upload_bias_table(*o, 1u << 16);
        if (rc != SOAR_OK) return cleanup(g_last_error);
    }
    {
        GradSet g0;
        for (const TensorRec& t : o->tensors) g0.grads.push_back(t.grad);
        g0.chunks = o->chunks;
        g0.sumsq_chunks = o->sumsq_chunks;
        uint64_t total = 0;
        for (const TensorRec& t : o->tensors)
            if (t.grad) total += t.numel;
        o->direct = !o->sgd && total > 0 && total <= kDirectMaxElems &&
                    build_direct_runs(*o, g0.grads, &g0.druns);
        if (o->direct) {
            // as many CTAs as are resident at once, fewer when the vectors do
            // not fill them (one vector per thread)
            const uint64_t vecs = g0.druns.start[g0.druns.n_runs];
            const uint64_t per_cta = static_cast<uint64_t>(soarb::kDirectThreads);
            const uint64_t want = std::max<uint64_t>(1, (vecs + per_cta - 1) / per_cta);
            const uint64_t cap = static_cast<uint64_t>(sms) * soarb::occupancy_apply_direct(o->mixed);
            o->grid_direct = static_cast<int>(std::min(want, cap));
        }
        o->druns = g0.druns;
        o->grad_sets.push_back(std::move(g0));
    }
    if ((e = cudaDeviceSynchronize()) != cudaSuccess)
        return cleanup(std::string("create: ") + cudaGetErrorString(e));
    *out = o;
    return SOAR_OK;
}

int ensure_bias_table(Optim& o) {
    if (o.bc_converged || o.host_calls + 1 < o.bc_len) return SOAR_OK;
    const uint64_t want = std::min<uint64_t>(static_cast<uint64_t>(o.bc_len) * 2, kBcCap);
    if (want <= o.bc_len) return fail("bias-correction table cap reached without converging");
    return upload_bias_table(o, static_cast<uint32_t>(want));
}

soarb::ApplyArgs apply_args(const Optim& o, const double* parts, int n_parts,
                            float max_norm) {
    soarb::ApplyArgs a{};
    a.lr = o.lr;
    a.beta1 = o.opts.beta1;
    a.beta2 = o.opts.beta2;
    a.eps = o.opts.eps;
    // adamw.cpp:100-101 evaluate (1.0f - beta) in float on the host
    a.omb1 = 1.0f - o.opts.beta1;
    a.omb2 = 1.0f - o.opts.beta2;
    a.max_norm = max_norm;
    a.pending_coef = o.pending_coef;
    a.growth = o.opts.growth_factor;
    a.backoff = o.opts.backoff_factor;
    a.interval = o.opts.growth_interval;
    a.use_scaler = o.opts.use_loss_scaler;
    a.n_parts = n_parts;
    a.parts = parts;
    a.bc = o.bc;
    a.bc_len = o.bc_len;
    if (o.sgd) {
        a.momentum = o.momentum;
        a.omdamp = 1.0f - o.dampening;  // sgd.cpp:79 evaluates (1.0f - dampening) in float
        a.nesterov = o.nesterov ? 1 : 0;
    }
    if (o.ema) {
        a.ema_decay = o.ema_decay;
        a.ema_omd = 1.0f - o.ema_decay;  // ema.hpp:25 evaluates (1.0f - decay_) in float
        a.ema_delta = static_cast<long long>(o.ema - o.m);
    }
    return a;
}

int apply_impl(Optim& o, const double* parts, int n_parts, cudaStream_t s,
               const soarb::AgArgs* ag = nullptr, const int* skip_if = nullptr,
               float max_norm = -1.0f) {
    if (n_parts < 0 || (n_parts > 0 && !parts)) return fail("bad partial sums");
    int rc = ensure_bias_table(o);
    if (rc != SOAR_OK) return rc;
    soarb::ApplyArgs a =
        apply_args(o, parts, n_parts, max_norm >= 0.0f ? max_norm : o.opts.max_grad_norm);
    a.skip_if = skip_if;
    if (o.direct && !ag && !o.ema) {
        SOAR_CUDA_TRY(soarb::launch_apply_direct(o.mixed, o.druns, o.chunks, o.n_chunks, o.n_vec,
                                                 o.ctl, a, o.grid_direct, s));
    } else {
        SOAR_CUDA_TRY(soarb::launch_apply(o.mixed, o.chunks, o.n_chunks, o.n_vec, o.ctl, a,
                                          o.grid_apply, s, ag, o.ema != nullptr, o.sgd, o.dyn));
    }
    o.host_calls += 1;
    o.pending_coef = 1.0f;
    return SOAR_OK;
}

int sumsq_impl(Optim& o, double* out, cudaStream_t s) {
    SOAR_CUDA_TRY(soarb::launch_grad_sumsq(o.mixed, o.sumsq_chunks, o.n_sumsq_chunks, o.ctl, o.partials,
                                           o.grid_sumsq, o.opts.use_loss_scaler, out, s));
    return SOAR_OK;
}

Optim* as_optim(void* h) { return static_cast<Optim*>(h); }

}  // namespace

namespace {
// Packs the control block into the public soar_step_info layout, on the stream.
__global__ void k_pack_info(const soarb::Ctl* c, soar_step_info* out) {
    out->step = c->t;
    out->skipped = c->skipped;
    out->grad_norm = c->last_norm;
    out->found_inf = c->last_found_inf;
    out->clip_coef = c->last_clip_coef;
    out->loss_scale = c->scale;
    out->growth_tracker = c->tracker;
    out->lr = c->last_lr;
    out->error = c->error;
}
}  // namespace

namespace soarb {
// Lets other translation units of the library report through soar_last_error().
void record_error(const std::string& msg) { g_last_error = msg; }

// The update with the fused data-parallel all-gather (zero1.cu).
int optim_apply_allgather(void* optim, const double* parts, int n_parts, cudaStream_t stream,
                          const AgArgs& ag, const int* skip_if) {
    Optim& o = *as_optim(optim);
    DeviceGuard g(o.device);
    return apply_impl(o, parts, n_parts, stream, &ag, skip_if);
}

// Tensor `index`'s param/grad/numel and the optimizer's layout, control block
// and device (index -1: only the latter three).
bool optim_tensor_info(void* optim, int index, void** param, void** grad, uint64_t* numel,
                       bool* mixed, Ctl** ctl, int* device) {
    Optim& o = *as_optim(optim);
    *mixed = o.mixed;
    *ctl = o.ctl;
    *device = o.device;
    if (index < 0) return index == -1;
    if (static_cast<size_t>(index) >= o.tensors.size()) return false;
    *param = o.tensors[index].param;
    *grad = o.tensors[index].grad;
    *numel = o.tensors[index].numel;
    return true;
}
}  // namespace soarb

extern "C" {

SOAR_API void soar_adamw_default_opts(soar_adamw_opts* out) {
    if (!out) return;
    std::memset(out, 0, sizeof *out);
    out->lr = 1e-3f;
    out->beta1 = 0.9f;
    out->beta2 = 0.999f;
    out->eps = 1e-8f;
    out->weight_decay = 1e-2f;
    out->layout = SOAR_LAYOUT_FP32;
    out->max_grad_norm = 0.0f;
    out->use_loss_scaler = 0;
    out->init_scale = 65536.0f;
    out->growth_factor = 2.0f;
    out->backoff_factor = 0.5f;
    out->growth_interval = 200;
    out->device = 0;
}

SOAR_API int soar_optim_create(const soar_tensor_desc* tensors, int n_tensors,
                               const soar_adamw_opts* opts, void** out_handle) {
    try {
        return create_impl(tensors, n_tensors, opts, out_handle);
    } catch (const std::exception& ex) {
        return fail(ex.what());
    } catch (...) {
        return fail("unknown exception");
    }
}

SOAR_API int soar_optim_create_uniform(void* const* params, void* const* grads,
                                       const uint64_t* numel, int n_tensors,
                                       const soar_adamw_opts* opts, void** out_handle) {
    if (!opts || n_tensors < 0 || (n_tensors > 0 && (!params || !numel)))
        return fail("null argument");
    try {
        std::vector<soar_tensor_desc> d(static_cast<size_t>(n_tensors));
        for (int i = 0; i < n_tensors; ++i)
            d[i] = {params[i], grads ? grads[i] : nullptr, numel[i], opts->weight_decay};
        return create_impl(d.data(), n_tensors, opts, out_handle);
    } catch (...) {
        return fail("exception in create_uniform");
    }
}

SOAR_API void soar_sgd_default_opts(soar_sgd_opts* out) {
    if (!out) return;
    std::memset(out, 0, sizeof *out);
    out->lr = 1e-2f;  // SGDOptions defaults, sgd.hpp:9-15
    out->layout = SOAR_LAYOUT_FP32;
    out->init_scale = 65536.0f;
    out->growth_factor = 2.0f;
    out->backoff_factor = 0.5f;
    out->growth_interval = 200;
}

SOAR_API int soar_sgd_create(const soar_tensor_desc* tensors, int n_tensors,
                             const soar_sgd_opts* opts, void** out_handle) {
    if (!opts) return fail("null argument");
    try {
        soar_adamw_opts a;
        soar_adamw_default_opts(&a);
        a.lr = opts->lr;
        a.weight_decay = opts->weight_decay;
        a.layout = opts->layout;
        a.max_grad_norm = opts->max_grad_norm;
        a.use_loss_scaler = opts->use_loss_scaler;
        a.init_scale = opts->init_scale;
        a.growth_factor = opts->growth_factor;
        a.backoff_factor = opts->backoff_factor;
        a.growth_interval = opts->growth_interval;
        a.device = opts->device;
        const SgdParams sp{opts->momentum, opts->dampening, opts->nesterov != 0};
        return create_impl(tensors, n_tensors, &a, out_handle, &sp);
    } catch (const std::exception& ex) {
        return fail(ex.what());
    } catch (...) {
        return fail("unknown exception");
    }
}

SOAR_API int soar_optim_destroy(void* handle) {
    if (!handle) return fail("null handle");
    Optim* o = as_optim(handle);
    {
        DeviceGuard g(o->device);
        cudaDeviceSynchronize();
        cudaFree(o->slab);
        if (o->bc) cudaFree(o->bc);
        if (o->ema) cudaFree(o->ema);
        for (GradSet& gs : o->grad_sets)
            if (gs.alloc) cudaFree(gs.alloc);
    }
    delete o;
    return SOAR_OK;
}

SOAR_API int soar_optim_step(void* handle, void* stream) {
    if (!handle) return fail("null handle");
    Optim& o = *as_optim(handle);
    DeviceGuard g(o.device);
    if (!g.ok) return fail("cannot select the optimizer's device");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (o.async_clip > 0.0f) {
        // clip_grad_norm_async left the norm pass's sum in Ctl::sumsq
        const float max_norm = o.async_clip;
        o.async_clip = 0.0f;
        return apply_impl(o, &o.ctl->sumsq, 1, s, nullptr, nullptr, max_norm);
    }
    const bool need_norm = o.opts.use_loss_scaler || o.opts.max_grad_norm > 0.0f;
    if (need_norm) {
        double* d_sumsq = &o.ctl->sumsq;
        int rc = sumsq_impl(o, d_sumsq, s);
        if (rc != SOAR_OK) return rc;
        return apply_impl(o, d_sumsq, 1, s);
    }
    return apply_impl(o, nullptr, 0, s);
}

SOAR_API int soar_optim_grad_sumsq(void* handle, double* d_sumsq, void* stream) {
    if (!handle || !d_sumsq) return fail("null argument");
    Optim& o = *as_optim(handle);
    DeviceGuard g(o.device);
    return sumsq_impl(o, d_sumsq, static_cast<cudaStream_t>(stream));
}

SOAR_API int soar_optim_apply(void* handle, const double* d_parts, int n_parts, void* stream) {
    if (!handle) return fail("null handle");
    Optim& o = *as_optim(handle);
    DeviceGuard g(o.device);
    return apply_impl(o, d_parts, n_parts, static_cast<cudaStream_t>(stream));
}

SOAR_API int soar_optim_clip_grad_norm(void* handle, float max_norm, float* out_norm,
                                       void* stream) {
    if (!handle || !out_norm) return fail("null argument");
    Optim& o = *as_optim(handle);
    DeviceGuard g(o.device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int rc = sumsq_impl(o, o.sumsq_scratch, s);
    if (rc != SOAR_OK) return rc;
    double total = 0.0;
    SOAR_CUDA_TRY(cudaMemcpyAsync(&total, o.sumsq_scratch, sizeof total, cudaMemcpyDeviceToHost, s));
    SOAR_CUDA_TRY(cudaStreamSynchronize(s));
    // adamw.cpp:42-44
    const float total_norm = static_cast<float>(std::sqrt(total));
    if (total_norm > max_norm && total_norm > 1e-6f) {
        const float clip_coef = max_norm / total_norm;
        if (o.mixed) {
            o.pending_coef = clip_coef;
        } else {
            SOAR_CUDA_TRY(soarb::launch_scale_grads_f32(o.sumsq_chunks, o.n_sumsq_chunks, clip_coef,
                                                        o.grid_apply, s));
        }
    }
    *out_norm = total_norm;
    return SOAR_OK;
}

SOAR_API int soar_optim_clip_grad_norm_async(void* handle, float max_norm, void* stream) {
    if (!handle) return fail("null handle");
    if (!(max_norm > 0.0f)) return fail("max_norm must be > 0");
    Optim& o = *as_optim(handle);
    DeviceGuard g(o.device);
    const int rc = sumsq_impl(o, &o.ctl->sumsq, static_cast<cudaStream_t>(stream));
    if (rc != SOAR_OK) return rc;
    o.async_clip = max_norm;
    return SOAR_OK;
}

SOAR_API int soar_optim_zero_grad(void* handle, void* stream) {
    if (!handle) return fail("null handle");
    Optim& o = *as_optim(handle);
    DeviceGuard g(o.device);
    const size_t eb = elem_bytes(o);
    // coalesce adjacent gradient buffers into single memsets
    std::vector<std::pair<char*, size_t>> r;
    for (const TensorRec& t : o.tensors)
        if (t.grad && t.numel) r.emplace_back(static_cast<char*>(t.grad), t.numel * eb);
    std::sort(r.begin(), r.end());
    size_t i = 0;
    while (i < r.size()) {
        char* p = r[i].first;
        char* end = p + r[i].second;
        size_t j = i + 1;
        while (j < r.size() && r[j].first <= end) {
            end = std::max(end, r[j].first + r[j].second);
            ++j;
        }
        SOAR_CUDA_TRY(cudaMemsetAsync(p, 0, static_cast<size_t>(end - p),
                                      static_cast<cudaStream_t>(stream)));
        i = j;
    }
    return SOAR_OK;
}

SOAR_API int soar_optim_set_lr(void* handle, float lr) {
    if (!handle) return fail("null handle");
    as_optim(handle)->lr = lr;
    return SOAR_OK;
}

SOAR_API int soar_optim_get_lr(void* handle, float* out_lr) {
    if (!handle || !out_lr) return fail("null argument");
    *out_lr = as_optim(handle)->lr;
    return SOAR_OK;
}

SOAR_API int soar_optim_get_info(void* handle, soar_step_info* out, void* stream) {
    if (!handle || !out) return fail("null argument");
    Optim& o = *as_optim(handle);
    DeviceGuard g(o.device);
    soarb::Ctl c{};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    SOAR_CUDA_TRY(cudaMemcpyAsync(&c, o.ctl, sizeof c, cudaMemcpyDeviceToHost, s));
    SOAR_CUDA_TRY(cudaStreamSynchronize(s));
    out->step = c.t;
    out->skipped = c.skipped;
    out->grad_norm = c.last_norm;
    out->found_inf = c.last_found_inf;
    out->clip_coef = c.last_clip_coef;
    out->loss_scale = c.scale;
    out->growth_tracker = c.tracker;
    out->lr = c.last_lr;
    out->error = c.error;
    return SOAR_OK;
}

SOAR_API int soar_optim_get_info_async(void* handle, soar_step_info* out, void* stream) {
    if (!handle || !out) return fail("null argument");
    Optim& o = *as_optim(handle);
    DeviceGuard g(o.device);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    k_pack_info<<<1, 1, 0, s>>>(o.ctl, o.info_stage);
    SOAR_CUDA_TRY(cudaGetLastError());
    SOAR_CUDA_TRY(cudaMemcpyAsync(out, o.info_stage, sizeof *out, cudaMemcpyDeviceToHost, s));
    return SOAR_OK;
}

SOAR_API int soar_optim_set_counters(void* handle, uint64_t step, uint64_t skipped,
                                     float loss_scale, int32_t growth_tracker, void* stream) {
    if (!handle) return fail("null handle");
    Optim& o = *as_optim(handle);
    DeviceGuard g(o.device);
    SOAR_CUDA_TRY(soarb::launch_set_counters(o.ctl, step, skipped, loss_scale, growth_tracker,
                                             static_cast<cudaStream_t>(stream)));
    o.host_calls = std::max(o.host_calls, step + skipped);
    return ensure_bias_table(o);
}

SOAR_API int soar_optim_state_ptr(void* handle, int index, int kind, void** out_ptr) {
    if (!handle || !out_ptr) return fail("null argument");
    Optim& o = *as_optim(handle);
    if (index < 0 || static_cast<size_t>(index) >= o.tensors.size()) return fail("bad tensor index");
    const TensorRec& t = o.tensors[index];
    switch (kind) {
        case SOAR_STATE_MASTER:
            *out_ptr = o.mixed ? static_cast<void*>(o.master + t.state_off) : t.param;
            return SOAR_OK;
        case SOAR_STATE_M:
            *out_ptr = o.m + t.state_off;
            return SOAR_OK;
        case SOAR_STATE_V:
            if (!o.v) return fail("SGD has no second-moment state");
            *out_ptr = o.v + t.state_off;
            return SOAR_OK;
        case SOAR_STATE_EMA:
            if (!o.ema) return fail("weight EMA is not enabled");
            *out_ptr = o.ema + t.state_off;
            return SOAR_OK;
        default:
            return fail("bad state kind");
    }
}

SOAR_API int soar_optim_read_state(void* handle, int index, int kind, float* host_dst) {
    void* p = nullptr;
    if (!host_dst) return fail("null argument");
    int rc = soar_optim_state_ptr(handle, index, kind, &p);
    if (rc != SOAR_OK) return rc;
    Optim& o = *as_optim(handle);
    DeviceGuard g(o.device);
    SOAR_CUDA_TRY(cudaDeviceSynchronize());
    SOAR_CUDA_TRY(cudaMemcpy(host_dst, p, o.tensors[index].numel * sizeof(float),
                             cudaMemcpyDeviceToHost));
    return SOAR_OK;
}

SOAR_API int soar_optim_write_state(void* handle, int index, int kind, const float* host_src) {
    void* p = nullptr;
    if (!host_src) return fail("null argument");
    int rc = soar_optim_state_ptr(handle, index, kind, &p);
    if (rc != SOAR_OK) return rc;
    Optim& o = *as_optim(handle);
    DeviceGuard g(o.device);
    SOAR_CUDA_TRY(cudaDeviceSynchronize());
    SOAR_CUDA_TRY(cudaMemcpy(p, host_src, o.tensors[index].numel * sizeof(float),
                             cudaMemcpyHostToDevice));
    return SOAR_OK;
}

SOAR_API int soar_optim_enable_ema(void* handle, float decay, void* stream) {
    if (!handle) return fail("null handle");
    Optim& o = *as_optim(handle);
    DeviceGuard g(o.device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!o.ema) {
        float* e = nullptr;
        SOAR_CUDA_TRY(cudaMalloc(&e, std::max<uint64_t>(o.state_elems, 1) * sizeof(float)));
        o.ema = e;
    }
    o.ema_decay = decay;
    // ModelEMA::init_shadow (ema.hpp:49-57): the shadow starts as a copy of the weights
    for (const TensorRec& t : o.tensors) {
        if (!t.numel) continue;
        const float* w = o.mixed ? o.master + t.state_off : static_cast<const float*>(t.param);
        SOAR_CUDA_TRY(cudaMemcpyAsync(o.ema + t.state_off, w, t.numel * sizeof(float),
                                      cudaMemcpyDeviceToDevice, s));
    }
    return SOAR_OK;
}

SOAR_API int soar_optim_ema_apply_to(void* handle, void* stream) {
    if (!handle) return fail("null handle");
    Optim& o = *as_optim(handle);
    if (!o.ema) return fail("weight EMA is not enabled");
    DeviceGuard g(o.device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // ModelEMA::apply_to (ema.hpp:31-38): the weights become the shadow
    for (const TensorRec& t : o.tensors) {
        if (!t.numel) continue;
        if (o.mixed) {
            SOAR_CUDA_TRY(cudaMemcpyAsync(o.master + t.state_off, o.ema + t.state_off,
                                          t.numel * sizeof(float), cudaMemcpyDeviceToDevice, s));
            SOAR_CUDA_TRY(soarb::launch_f32_to_bf16(o.ema + t.state_off,
                                                    static_cast<uint16_t*>(t.param), t.numel, s));
        } else {
            SOAR_CUDA_TRY(cudaMemcpyAsync(t.param, o.ema + t.state_off, t.numel * sizeof(float),
                                          cudaMemcpyDeviceToDevice, s));
        }
    }
    return SOAR_OK;
}

SOAR_API int soar_optim_loss_scale_ptr(void* handle, float** out_ptr) {
    if (!handle || !out_ptr) return fail("null argument");
    *out_ptr = &as_optim(handle)->ctl->scale;
    return SOAR_OK;
}

// ---- optimizer-state checkpoint -------------------------------------------
// The reference's weight-file record layout (src/nn/soar_model.cpp:427-463):
// u32 magic 'SOAR', u32 version, u32 variant, u32 count, then per record
// char name[128], u32 ndim, u32 shape[4], u64 bytes, raw bytes. Version 2
// adds the optimizer's records; the reference's loader skips names it does not
// know (soar_model.cpp:508-518), so a model-weights reader still works.

namespace {
constexpr uint32_t kSoarMagic = 0x534F4152u;
constexpr uint32_t kStateVersion = 2;
constexpr const char* kKindName[4] = {"master", "m", "v", "ema"};

struct Counters {  // payload of the "optim.counters" record
    uint64_t t, skipped, host_calls;
    float scale;
    int32_t tracker;
    float lr;
    uint32_t layout;
    uint64_t n_tensors;
};

bool write_record(FILE* f, const std::string& name, uint64_t numel, const void* data,
                  uint64_t bytes) {
    char nb[128]{0};
    std::strncpy(nb, name.c_str(), 127);
    const uint32_t ndim = 1;
    uint32_t shape[4] = {static_cast<uint32_t>(numel), 1, 1, 1};
    return std::fwrite(nb, 128, 1, f) == 1 && std::fwrite(&ndim, 4, 1, f) == 1 &&
           std::fwrite(shape, 16, 1, f) == 1 && std::fwrite(&bytes, 8, 1, f) == 1 &&
           (bytes == 0 || std::fwrite(data, 1, bytes, f) == bytes);
}
}  // namespace

SOAR_API int soar_optim_save_state(void* handle, const char* path) {
    if (!handle || !path) return fail("null argument");
    Optim& o = *as_optim(handle);
    DeviceGuard g(o.device);
    SOAR_CUDA_TRY(cudaDeviceSynchronize());
    soarb::Ctl c{};
    SOAR_CUDA_TRY(cudaMemcpy(&c, o.ctl, sizeof c, cudaMemcpyDeviceToHost));
    FILE* f = std::fopen(path, "wb");
    if (!f) return fail(std::string("cannot open ") + path);
    std::vector<int> kinds = {SOAR_STATE_MASTER, SOAR_STATE_M};
    if (!o.sgd) kinds.push_back(SOAR_STATE_V);
    if (o.ema) kinds.push_back(SOAR_STATE_EMA);
    const uint32_t n_records = 1 + static_cast<uint32_t>(kinds.size() * o.tensors.size());
    const uint32_t hdr[4] = {kSoarMagic, kStateVersion, 0u, n_records};
    bool ok = std::fwrite(hdr, 4, 4, f) == 4;
    Counters ct{c.t, c.skipped, o.host_calls, c.scale, c.tracker, o.lr,
                static_cast<uint32_t>(o.opts.layout) | (o.sgd ? 0x100u : 0u), o.tensors.size()};
    ok = ok && write_record(f, "optim.counters", sizeof ct / 4, &ct, sizeof ct);
    std::vector<float> buf;
    for (size_t i = 0; ok && i < o.tensors.size(); ++i) {
        const TensorRec& t = o.tensors[i];
        buf.resize(t.numel);
        for (int k : kinds) {
            if (!ok) break;
            void* p = nullptr;
            soar_optim_state_ptr(handle, static_cast<int>(i), k, &p);
            if (t.numel && cudaMemcpy(buf.data(), p, t.numel * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
                ok = false;
            ok = ok && write_record(f, std::string("optim.") + kKindName[k] + "." + std::to_string(i),
                                    t.numel, buf.data(), t.numel * 4);
        }
    }
    ok = (std::fclose(f) == 0) && ok;
    return ok ? SOAR_OK : fail(std::string("writing ") + path + " failed");
}

SOAR_API int soar_optim_load_state(void* handle, const char* path, void* stream) {
    if (!handle || !path) return fail("null argument");
    Optim& o = *as_optim(handle);
    DeviceGuard g(o.device);
    FILE* f = std::fopen(path, "rb");
    if (!f) return fail(std::string("cannot open ") + path);
    uint32_t hdr[4]{};
    if (std::fread(hdr, 4, 4, f) != 4 || hdr[0] != kSoarMagic) {
        std::fclose(f);
        return fail("not a SOAR file (bad magic)");
    }
    if (hdr[1] < kStateVersion) {
        std::fclose(f);
        return fail("weights-only file (version < 2): no optimizer state");
    }
    std::map<std::string, std::pair<int, int>> want;  // name -> (tensor, kind)
    std::vector<int> kinds = {SOAR_STATE_MASTER, SOAR_STATE_M};
    if (!o.sgd) kinds.push_back(SOAR_STATE_V);
    if (o.ema) kinds.push_back(SOAR_STATE_EMA);
    for (size_t i = 0; i < o.tensors.size(); ++i)
        for (int k : kinds)
            want[std::string("optim.") + kKindName[k] + "." + std::to_string(i)] = {static_cast<int>(i), k};
    bool have_counters = false;
    Counters ct{};
    size_t loaded = 0;
    std::vector<float> buf;
    SOAR_CUDA_TRY(cudaDeviceSynchronize());
    for (uint32_t r = 0; r < hdr[3]; ++r) {
        char nb[128]{0};
        uint32_t ndim = 0, shape[4]{};
        uint64_t bytes = 0;
        if (std::fread(nb, 128, 1, f) != 1 || std::fread(&ndim, 4, 1, f) != 1 ||
            std::fread(shape, 16, 1, f) != 1 || std::fread(&bytes, 8, 1, f) != 1)
            break;
        nb[127] = 0;
        const std::string name(nb);
        if (name == "optim.counters" && bytes == sizeof ct) {
            have_counters = std::fread(&ct, sizeof ct, 1, f) == 1;
            continue;
        }
        auto it = want.find(name);
        if (it == want.end() || bytes != o.tensors[it->second.first].numel * 4) {
            std::fseek(f, static_cast<long>(bytes), SEEK_CUR);  // skip, as the reference's loader
            continue;
        }
        buf.resize(bytes / 4);
        if (bytes && std::fread(buf.data(), 1, bytes, f) != bytes) break;
        void* p = nullptr;
        soar_optim_state_ptr(handle, it->second.first, it->second.second, &p);
        if (bytes && cudaMemcpy(p, buf.data(), bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
            std::fclose(f);
            return fail("state upload failed");
        }
        ++loaded;
    }
    std::fclose(f);
    if (!have_counters) return fail("no optim.counters record");
    if (ct.n_tensors != o.tensors.size() ||
        ct.layout != (static_cast<uint32_t>(o.opts.layout) | (o.sgd ? 0x100u : 0u)))
        return fail("checkpoint was written by an optimizer with a different tensor list or layout");
    if (loaded != kinds.size() * o.tensors.size())
        return fail("checkpoint is missing optimizer records (" + std::to_string(loaded) + " of " +
                    std::to_string(kinds.size() * o.tensors.size()) + ")");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (o.mixed) {  // bf16 params follow the restored fp32 master
        for (size_t i = 0; i < o.tensors.size(); ++i) {
            const TensorRec& t = o.tensors[i];
            SOAR_CUDA_TRY(soarb::launch_f32_to_bf16(o.master + t.state_off,
                                                    static_cast<uint16_t*>(t.param), t.numel, s));
        }
    }
    SOAR_CUDA_TRY(soarb::launch_set_counters(o.ctl, ct.t, ct.skipped, ct.scale, ct.tracker, s));
    o.host_calls = std::max(ct.host_calls, ct.t + ct.skipped);
    o.lr = ct.lr;
    o.pending_coef = 1.0f;
    SOAR_CUDA_TRY(cudaStreamSynchronize(s));
    return ensure_bias_table(o);
}

SOAR_API int soar_cosine_create(void* optim_handle, uint64_t total_steps, float eta_min,
                                uint64_t warmup_steps, void** out_handle) {
    if (!optim_handle || !out_handle) return fail("null argument");
    Optim* o = as_optim(optim_handle);
    // adamw.cpp:119-121: base lr is the optimizer's lr at construction
    *out_handle = new (std::nothrow) Cosine{o, o->lr, eta_min, total_steps, warmup_steps, 0};
    return *out_handle ? SOAR_OK : fail("out of host memory");
}

SOAR_API int soar_cosine_step(void* sched_handle) {
    if (!sched_handle) return fail("null handle");
    Cosine& c = *static_cast<Cosine*>(sched_handle);
    // adamw.cpp:123-142, same types and expressions
    c.current_step++;
    if (c.current_step <= c.warmup_steps && c.warmup_steps > 0) {
        const float lr = c.base_lr * static_cast<float>(c.current_step) /
                         static_cast<float>(c.warmup_steps);
        c.opt->lr = lr;
        return SOAR_OK;
    }
    const uint64_t adjusted_step = c.current_step - c.warmup_steps;
    const uint64_t adjusted_total = c.total_steps - c.warmup_steps;
    if (adjusted_step > adjusted_total) {
        c.opt->lr = c.eta_min;
        return SOAR_OK;
    }
    constexpr float pi = 3.14159265358979323846f;
    const float progress = static_cast<float>(adjusted_step) / static_cast<float>(adjusted_total);
    const float lr = c.eta_min + 0.5f * (c.base_lr - c.eta_min) * (1.0f + std::cos(progress * pi));
    c.opt->lr = lr;
    return SOAR_OK;
}

SOAR_API int soar_cosine_destroy(void* sched_handle) {
    if (!sched_handle) return fail("null handle");
    delete static_cast<Cosine*>(sched_handle);
    return SOAR_OK;
}

SOAR_API int soar_selftest_bounded_wait(uint64_t limit_ns, int device, int* out_timed_out,
                                        uint64_t* out_waited_ns) {
    if (!out_timed_out || !out_waited_ns) return fail("null argument");
    DeviceGuard g(device);
    if (!g.ok) return fail("cannot select device");
    int* d_err = nullptr;
    SOAR_CUDA_TRY(cudaMalloc(&d_err, 64));
    unsigned long long* d_ns = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(d_err) + 32);
    cudaError_t e = soarb::launch_wait_selftest(limit_ns, d_err, d_ns, nullptr);
    int err = 0;
    unsigned long long ns = 0;
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(&err, d_err, sizeof err, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(&ns, d_ns, sizeof ns, cudaMemcpyDeviceToHost);
    cudaFree(d_err);
    if (e != cudaSuccess) return fail(std::string("selftest: ") + cudaGetErrorString(e));
    *out_timed_out = err;
    *out_waited_ns = ns;
    return SOAR_OK;
}

SOAR_API int soar_optim_add_grads(void* handle, void* const* grads, int* out_set) {
    if (!handle || !grads || !out_set) return fail("null argument");
    Optim& o = *as_optim(handle);
    const GradSet& g0 = o.grad_sets.front();
    const size_t eb = elem_bytes(o);
    std::vector<void*> ng(grads, grads + o.tensors.size());
    for (size_t i = 0; i < ng.size(); ++i) {
        const uintptr_t a = reinterpret_cast<uintptr_t>(ng[i]);
        const uintptr_t b = reinterpret_cast<uintptr_t>(g0.grads[i]);
        if ((ng[i] == nullptr) != (b == 0))
            return fail("tensor " + std::to_string(i) + ": gradient presence differs from the "
                        "optimizer's first gradient set");
        if (ng[i] && (a % eb || a % soarb::kVecBytes != b % soarb::kVecBytes))
            return fail("tensor " + std::to_string(i) + ": gradient alignment (address modulo 16 "
                        "bytes) differs from the optimizer's first gradient set");
    }
    // the tables of set 0 with every gradient pointer moved to the new buffers
    auto moved = [&](std::vector<soarb::Chunk> tab) {
        for (soarb::Chunk& c : tab) {
            const char* old_base = static_cast<const char*>(g0.grads[c.tensor]);
            c.grad = static_cast<const char*>(ng[c.tensor]) +
                     (static_cast<const char*>(c.grad) - old_base);
        }
        return tab;
    };
    const std::vector<soarb::Chunk> up = moved(o.host_chunks), ns = moved(o.host_sumsq_chunks);
    GradSet gs;
    gs.grads = ng;
    if (o.direct && !build_direct_runs(o, ng, &gs.druns)) return fail("internal: direct runs");
    DeviceGuard g(o.device);
    const size_t up_bytes = align_up(up.size() * sizeof(soarb::Chunk), kSlabAlign);
    const size_t bytes = up_bytes + ns.size() * sizeof(soarb::Chunk);
    SOAR_CUDA_TRY(cudaMalloc(&gs.alloc, std::max<size_t>(bytes, 64)));
    gs.chunks = static_cast<soarb::Chunk*>(gs.alloc);
    gs.sumsq_chunks = reinterpret_cast<soarb::Chunk*>(static_cast<char*>(gs.alloc) + up_bytes);
    cudaError_t e = cudaMemcpy(gs.chunks, up.data(), up.size() * sizeof(soarb::Chunk),
                               cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(gs.sumsq_chunks, ns.data(), ns.size() * sizeof(soarb::Chunk),
                       cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(gs.alloc);
        return fail(std::string("gradient-set tables: ") + cudaGetErrorString(e));
    }
    o.grad_sets.push_back(std::move(gs));
    *out_set = static_cast<int>(o.grad_sets.size()) - 1;
    return SOAR_OK;
}

SOAR_API int soar_optim_use_grads(void* handle, int set) {
    if (!handle) return fail("null handle");
    Optim& o = *as_optim(handle);
    if (set < 0 || set >= static_cast<int>(o.grad_sets.size())) return fail("bad gradient set");
    const GradSet& gs = o.grad_sets[set];
    o.chunks = gs.chunks;
    o.sumsq_chunks = gs.sumsq_chunks;
    o.druns = gs.druns;
    for (size_t i = 0; i < o.tensors.size(); ++i) o.tensors[i].grad = gs.grads[i];
    o.grad_set = set;
    return SOAR_OK;
}

SOAR_API int soar_optim_kernel_path(void* handle, int* out_path) {
    if (!handle || !out_path) return fail("null argument");
    const Optim& o = *as_optim(handle);
    *out_path = (o.direct && !o.ema) ? 1 : 0;
    return SOAR_OK;
}

SOAR_API int soar_kernel_arch(int device, int* out_compiled, int* out_loaded) {
    if (!out_compiled) return fail("null argument");
    // the architectures nvcc compiled the kernels for (first entry), e.g. 1000
    constexpr int kArchs[] = {__CUDA_ARCH_LIST__};
    *out_compiled = kArchs[0];
    if (device < 0) return SOAR_OK;
    if (!out_loaded) return fail("null argument");
    DeviceGuard g(device);
    if (!g.ok) return fail("cannot select device " + std::to_string(device));
    cudaFuncAttributes attr{};
    SOAR_CUDA_TRY(soarb::apply_kernel_attributes(&attr));
    *out_loaded = attr.binaryVersion;
    return SOAR_OK;
}

SOAR_API const char* soar_last_error(void) { return g_last_error.c_str(); }

}  // extern "C"
