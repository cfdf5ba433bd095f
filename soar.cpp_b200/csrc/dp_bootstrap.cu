// Data-parallel bootstrap in the library: an NCCL communicator per process
// (one process per GPU) and the fused ZeRO-1 optimizer built over it, so a
// C++ host (the reference's Trainer is C++, src/engine/trainer.cpp) gets the
// fused data-parallel step without Python.
//
// soar_dp_init wraps ncclCommInitRank; the caller moves the 128-byte unique id
// from rank 0 to the other ranks over any host channel (a file, MPI, a TCP
// store), as with NCCL itself. soar_dp_zero1_create then does, collectively:
//   1. allocates this rank's flat bf16 parameter and gradient buffers and its
//      signal block (soar_ipc_alloc: cudaMalloc + CUDA IPC handle);
//   2. all-gathers the three 64-byte IPC handles over the communicator and
//      opens every peer's buffers (soar_ipc_open), so all R buffers are
//      addressable from this GPU at identical offsets;
//   3. plans the buckets: rank r owns the contiguous r-th 1/R slice of every
//      bucket (the last bucket may be shorter, slices are ceil(size / R));
//   4. creates the bf16-mixed optimizer over the owned slices (its fp32
//      master starts from the initial params) and binds it to the buffers
//      (soar_zero1_create, soar_zero1_set_signals);
//   5. a barrier, so no rank steps before every signal block is in place.
// Every phase ends with an agreement (a 1-element all-reduce of the failure
// flag), so a failure on one rank makes every rank clean up and return the
// error instead of leaving the others inside a collective.
//
// NCCL is opened with dlopen at the first soar_dp_init (libnccl.so.2: the
// system library in a C++ process, or the one already loaded by the host
// framework), so the optimizer library itself has no load-time dependency on
// it. Only the types come from nccl.h.
#include <dlfcn.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <cuda_runtime.h>
#include <nccl.h>

#include "../../include/soar_optim.h"

namespace soarb {
void record_error(const std::string& msg);  // optim_capi.cu
}

namespace {

static_assert(sizeof(ncclUniqueId) == SOAR_DP_UNIQUE_ID_BYTES, "NCCL unique id size");

int fail(const std::string& m) {
    soarb::record_error(m);
    return SOAR_ERROR;
}

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

struct Nccl {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
};

const Nccl* nccl(std::string* why) {
    static std::once_flag once;
    static Nccl api;
    static std::string err;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            err = std::string("cannot load libnccl.so.2: ") + dlerror();
            return;
        }
        auto sym = [&](const char* name) { return dlsym(h, name); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        if (!api.get_unique_id || !api.comm_init_rank || !api.comm_destroy || !api.all_gather ||
            !api.all_reduce || !api.error_string)
            err = "libnccl.so.2 lacks an expected entry point";
    });
    if (!err.empty()) {
        *why = err;
        return nullptr;
    }
    return &api;
}

struct DpComm {
    const Nccl* api;
    ncclComm_t comm;
    int rank, world, device;
    cudaStream_t stream;   // the library's own stream for set-up collectives
    int* d_flag;           // 1 int: barrier and agreement word
};

int nccl_fail(const Nccl* api, const char* what, ncclResult_t r) {
    return fail(std::string(what) + ": " + api->error_string(r));
}

// Stream-ordered barrier: a 1-element all-reduce on `stream`.
ncclResult_t barrier_on(DpComm& c, cudaStream_t stream) {
    return c.api->all_reduce(c.d_flag, c.d_flag, 1, ncclInt32, ncclMax, c.comm, stream);
}

// Collective agreement on the host: true when every rank passes ok = true.
// All ranks must call it at the same point of their sequence.
bool agree(DpComm& c, bool ok, std::string* why) {
    const int flag = ok ? 0 : 1;
    if (cudaMemcpyAsync(c.d_flag, &flag, sizeof flag, cudaMemcpyHostToDevice, c.stream) !=
        cudaSuccess) {
        *why = "agreement upload failed";
        return false;
    }
    const ncclResult_t r = barrier_on(c, c.stream);
    int all = 1;
    if (r != ncclSuccess ||
        cudaMemcpyAsync(&all, c.d_flag, sizeof all, cudaMemcpyDeviceToHost, c.stream) !=
            cudaSuccess ||
        cudaStreamSynchronize(c.stream) != cudaSuccess) {
        *why = "agreement collective failed";
        return false;
    }
    if (all != 0 && why->empty()) *why = "failed on another rank";
    return all == 0;
}

struct Bucket {
    uint64_t own_start, own_size;
};

// Rank `rank`'s owned slices: the rank-th ceil(size / world) slice of every
// bucket of `bucket` elements (the last bucket may be shorter).
std::vector<Bucket> plan_buckets(uint64_t n, uint64_t bucket, int world, int rank) {
    std::vector<Bucket> out;
    for (uint64_t start = 0; start < n; start += bucket) {
        const uint64_t size = std::min(bucket, n - start);
        const uint64_t shard = (size + world - 1) / world;
        const uint64_t lo = std::min(size, static_cast<uint64_t>(rank) * shard);
        const uint64_t hi = std::min(size, static_cast<uint64_t>(rank + 1) * shard);
        out.push_back({start + lo, hi - lo});
    }
    return out;
}

struct DpZero1 {
    DpComm* comm;
    int sync_mode;
    uint64_t n = 0, shard = 0;
    void* local[3] = {nullptr, nullptr, nullptr};  // grads (set 0), params, signals (set 0)
    std::vector<void*> extra;                       // further gradient buffers and signal blocks
    std::vector<void*> peers;                       // opened peer mappings
    void* optim = nullptr;
    std::vector<void*> zero1;                       // one fused-step handle per gradient set
    std::vector<void*> grads;                       // this rank's buffer of each gradient set
    int cur = 0;                                    // the set the next steps reduce
    std::vector<void*> param_bases;                 // every rank's parameter buffer
    std::vector<soar_zero1_shard> shards;
    double* d_part = nullptr;                       // sync mode 1: own partial + R partials
};

// Allocates `n` symmetric buffers of bytes[k] on every rank, exchanges their
// IPC handles over the communicator and opens the peers' (collective; every
// phase agreed on). bases[k][q] is rank q's buffer k as seen from here; the
// local buffers go to `locals`, the peer mappings to z.peers.
bool symmetric_alloc(DpZero1& z, int n, const size_t* bytes, std::vector<void*>* bases,
                     std::vector<void*>& locals, std::string* why) {
    DpComm& c = *z.comm;
    std::vector<unsigned char> mine(static_cast<size_t>(n) * SOAR_IPC_HANDLE_BYTES);
    bool ok = true;
    for (int k = 0; k < n && ok; ++k) {
        void* p = nullptr;
        ok = soar_ipc_alloc(bytes[k], c.device, &p, mine.data() + k * SOAR_IPC_HANDLE_BYTES) ==
             SOAR_OK;
        if (ok) locals.push_back(p);
        else *why = soar_last_error();
    }
    if (!agree(c, ok, why)) return false;
    std::vector<unsigned char> all(static_cast<size_t>(c.world) * mine.size());
    {
        unsigned char* d_buf = nullptr;
        cudaError_t e = cudaMalloc(&d_buf, all.size());
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(d_buf + c.rank * mine.size(), mine.data(), mine.size(),
                                cudaMemcpyHostToDevice, c.stream);
        ncclResult_t r = ncclSuccess;
        if (e == cudaSuccess)
            r = c.api->all_gather(d_buf + c.rank * mine.size(), d_buf, mine.size(), ncclUint8,
                                  c.comm, c.stream);
        if (e == cudaSuccess && r == ncclSuccess)
            e = cudaMemcpyAsync(all.data(), d_buf, all.size(), cudaMemcpyDeviceToHost, c.stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c.stream);
        if (d_buf) cudaFree(d_buf);
        ok = e == cudaSuccess && r == ncclSuccess;
        if (!ok) *why = "handle exchange failed";
    }
    for (int k = 0; k < n; ++k) bases[k].assign(c.world, nullptr);
    for (int q = 0; q < c.world && ok; ++q) {
        for (int k = 0; k < n && ok; ++k) {
            if (q == c.rank) {
                bases[k][q] = locals[locals.size() - n + k];
                continue;
            }
            const unsigned char* h = all.data() + (q * n + k) * SOAR_IPC_HANDLE_BYTES;
            void* p = nullptr;
            ok = soar_ipc_open(h, c.device, &p) == SOAR_OK;
            if (ok) {
                z.peers.push_back(p);
                bases[k][q] = p;
            } else {
                *why = soar_last_error();
            }
        }
    }
    return agree(c, ok, why);
}

// Releases what `z` holds. Collective (every rank calls it): no rank frees
// its buffers while a peer may still map them.
void release(DpZero1& z) {
    DpComm& c = *z.comm;
    DeviceGuard g(c.device);
    cudaDeviceSynchronize();
    for (void* h : z.zero1) soar_zero1_destroy(h);
    z.zero1.clear();
    if (z.optim) soar_optim_destroy(z.optim);
    z.optim = nullptr;
    for (void* p : z.peers) soar_ipc_close(p, c.device);
    z.peers.clear();
    barrier_on(c, c.stream);
    cudaStreamSynchronize(c.stream);
    for (void*& p : z.local) {
        if (p) soar_ipc_free(p, c.device);
        p = nullptr;
    }
    for (void* p : z.extra) soar_ipc_free(p, c.device);
    z.extra.clear();
    if (z.d_part) cudaFree(z.d_part);
    z.d_part = nullptr;
}

}  // namespace

extern "C" {

SOAR_API int soar_dp_unique_id(void* out_id) {
    if (!out_id) return fail("null argument");
    std::string why;
    const Nccl* api = nccl(&why);
    if (!api) return fail(why);
    const ncclResult_t r = api->get_unique_id(static_cast<ncclUniqueId*>(out_id));
    return r == ncclSuccess ? SOAR_OK : nccl_fail(api, "ncclGetUniqueId", r);
}

SOAR_API int soar_dp_init(int rank, int world, const void* unique_id, int device,
                          void** out_comm) {
    if (!unique_id || !out_comm) return fail("null argument");
    if (world < 1 || world > 8 || rank < 0 || rank >= world)
        return fail("soar_dp_init: world must be 1..8 and rank inside it");
    *out_comm = nullptr;
    std::string why;
    const Nccl* api = nccl(&why);
    if (!api) return fail(why);
    DeviceGuard g(device);
    if (!g.ok) return fail("cannot select device " + std::to_string(device));
    auto* c = new DpComm{api, nullptr, rank, world, device, nullptr, nullptr};
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof id);
    cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&c->d_flag, 256);
    if (e == cudaSuccess) e = cudaMemset(c->d_flag, 0, 256);
    if (e != cudaSuccess) {
        if (c->stream) cudaStreamDestroy(c->stream);
        if (c->d_flag) cudaFree(c->d_flag);
        delete c;
        return fail(std::string("soar_dp_init: ") + cudaGetErrorString(e));
    }
    const ncclResult_t r = api->comm_init_rank(&c->comm, world, id, rank);
    if (r != ncclSuccess) {
        cudaStreamDestroy(c->stream);
        cudaFree(c->d_flag);
        delete c;
        return nccl_fail(api, "ncclCommInitRank", r);
    }
    *out_comm = c;
    return SOAR_OK;
}

SOAR_API int soar_dp_destroy(void* comm) {
    if (!comm) return fail("null handle");
    auto* c = static_cast<DpComm*>(comm);
    {
        DeviceGuard g(c->device);
        cudaStreamSynchronize(c->stream);
        c->api->comm_destroy(c->comm);
        cudaStreamDestroy(c->stream);
        cudaFree(c->d_flag);
    }
    delete c;
    return SOAR_OK;
}

SOAR_API int soar_dp_barrier(void* comm, void* stream) {
    if (!comm) return fail("null handle");
    auto& c = *static_cast<DpComm*>(comm);
    DeviceGuard g(c.device);
    const ncclResult_t r = barrier_on(c, static_cast<cudaStream_t>(stream));
    return r == ncclSuccess ? SOAR_OK : nccl_fail(c.api, "barrier", r);
}

SOAR_API int soar_dp_allgather_f64(void* comm, const double* d_send, double* d_recv,
                                   uint64_t count, void* stream) {
    if (!comm || !d_send || !d_recv) return fail("null argument");
    auto& c = *static_cast<DpComm*>(comm);
    DeviceGuard g(c.device);
    const ncclResult_t r = c.api->all_gather(d_send, d_recv, count, ncclFloat64, c.comm,
                                             static_cast<cudaStream_t>(stream));
    return r == ncclSuccess ? SOAR_OK : nccl_fail(c.api, "ncclAllGather", r);
}

SOAR_API int soar_dp_zero1_create(void* comm, uint64_t n_params, uint64_t bucket,
                                  const soar_adamw_opts* opts, const void* init_params,
                                  int sync_mode, void** out_handle) {
    if (!comm || !opts || !out_handle) return fail("null argument");
    *out_handle = nullptr;
    if (n_params == 0 || bucket == 0) return fail("soar_dp_zero1_create: empty model or bucket");
    if (opts->layout != SOAR_LAYOUT_BF16_MIXED)
        return fail("soar_dp_zero1_create: the data-parallel step uses the bf16-mixed layout");
    if (sync_mode != SOAR_DP_SYNC_DEVICE && sync_mode != SOAR_DP_SYNC_NCCL)
        return fail("soar_dp_zero1_create: unknown sync mode");
    auto& c = *static_cast<DpComm*>(comm);
    if (opts->device != c.device)
        return fail("soar_dp_zero1_create: opts->device differs from the communicator's device");
    DeviceGuard g(c.device);
    auto* z = new DpZero1{};
    z->comm = &c;
    z->sync_mode = sync_mode;
    z->n = n_params;
    std::string why;
    // 1-2. local buffers, their IPC handles exchanged, the peers' opened
    const size_t bytes[3] = {2 * n_params, 2 * n_params, SOAR_ZERO1_SIGNAL_BYTES};
    std::vector<void*> bases[3], locals;
    bool ok = symmetric_alloc(*z, 3, bytes, bases, locals, &why);
    for (size_t k = 0; k < locals.size(); ++k) z->local[k] = locals[k];
    if (!ok) {
        release(*z);
        delete z;
        return fail("soar_dp_zero1_create: " + why);
    }
    if (init_params &&
        cudaMemcpy(z->local[1], init_params, 2 * n_params, cudaMemcpyDefault) != cudaSuccess) {
        ok = false;
        why = "initial params copy failed";
    }
    if (ok && cudaMalloc(&z->d_part, sizeof(double) * (1 + c.world)) != cudaSuccess) {
        ok = false;
        why = "partial-sum buffer";
    }
    if (!agree(c, ok, &why)) {
        release(*z);
        delete z;
        return fail("soar_dp_zero1_create: " + why);
    }
    // 3-4. the owned slices, the shard optimizer and the fused step's handle
    const std::vector<Bucket> plan = plan_buckets(n_params, bucket, c.world, c.rank);
    std::vector<soar_tensor_desc> descs;
    std::vector<soar_zero1_shard>& shards = z->shards;
    for (const Bucket& b : plan) {
        if (!b.own_size) continue;
        soar_tensor_desc d{};
        d.param = static_cast<uint16_t*>(z->local[1]) + b.own_start;
        d.grad = static_cast<uint16_t*>(z->local[0]) + b.own_start;
        d.numel = b.own_size;
        d.weight_decay = opts->weight_decay;
        shards.push_back({b.own_start, b.own_size, static_cast<int32_t>(descs.size())});
        descs.push_back(d);
        z->shard += b.own_size;
    }
    ok = soar_optim_create(descs.data(), static_cast<int>(descs.size()), opts, &z->optim) ==
         SOAR_OK;
    void* z1 = nullptr;
    if (ok)
        ok = soar_zero1_create(z->optim, c.rank, c.world, bases[0].data(), bases[1].data(),
                               shards.data(), static_cast<int>(shards.size()), &z1) == SOAR_OK;
    if (ok) {
        z->zero1.push_back(z1);
        z->grads.push_back(z->local[0]);
        z->param_bases = bases[1];
    }
    if (ok && sync_mode == SOAR_DP_SYNC_DEVICE)
        ok = soar_zero1_set_signals(z1, bases[2].data()) == SOAR_OK;
    if (!ok) why = soar_last_error();
    // 5. every rank's signal block is zeroed and bound before any rank steps
    if (!agree(c, ok, &why)) {
        release(*z);
        delete z;
        return fail("soar_dp_zero1_create: " + why);
    }
    *out_handle = z;
    return SOAR_OK;
}

SOAR_API int soar_dp_zero1_get_info(void* handle, soar_dp_zero1_info* out) {
    if (!handle || !out) return fail("null argument");
    const auto& z = *static_cast<DpZero1*>(handle);
    out->params = z.local[1];
    out->grads = z.grads[z.cur];
    out->optimizer = z.optim;
    out->zero1 = z.zero1[z.cur];
    out->n_params = z.n;
    out->shard_params = z.shard;
    out->rank = z.comm->rank;
    out->world = z.comm->world;
    return SOAR_OK;
}

SOAR_API int soar_dp_zero1_step(void* handle, void* stream) {
    if (!handle) return fail("null handle");
    auto& z = *static_cast<DpZero1*>(handle);
    void* z1 = z.zero1[z.cur];
    if (z.sync_mode == SOAR_DP_SYNC_DEVICE) return soar_zero1_step(z1, stream);
    // synchronised by NCCL between the launches
    DpComm& c = *z.comm;
    int rc = soar_dp_barrier(&c, stream);                        // every rank's grads complete
    if (rc == SOAR_OK) rc = soar_zero1_reduce_sumsq(z1, z.d_part, stream);
    if (rc == SOAR_OK) rc = soar_dp_allgather_f64(&c, z.d_part, z.d_part + 1, 1, stream);
    if (rc == SOAR_OK) rc = soar_zero1_apply_allgather(z1, z.d_part + 1, c.world, stream);
    if (rc == SOAR_OK) rc = soar_dp_barrier(&c, stream);         // peers' param writes landed
    return rc;
}

SOAR_API int soar_dp_zero1_add_grads(void* handle, int* out_index) {
    if (!handle || !out_index) return fail("null argument");
    auto& z = *static_cast<DpZero1*>(handle);
    DpComm& c = *z.comm;
    DeviceGuard g(c.device);
    std::string why;
    // a gradient buffer and a signal block of their own, symmetric
    const size_t bytes[2] = {2 * z.n, SOAR_ZERO1_SIGNAL_BYTES};
    std::vector<void*> bases[2];
    if (!symmetric_alloc(z, 2, bytes, bases, z.extra, &why))
        return fail("soar_dp_zero1_add_grads: " + why);
    void* gbuf = bases[0][c.rank];
    // the shard optimizer reads the owned slices of the new buffer as a
    // gradient set of its own; the new fused-step handle is bound while that
    // set is in use (it checks the optimizer's slices against the buffer)
    std::vector<void*> slices;
    for (const soar_zero1_shard& s : z.shards)
        slices.push_back(static_cast<uint16_t*>(gbuf) + s.offset);
    int set = -1;
    void* z1 = nullptr;
    bool ok = soar_optim_add_grads(z.optim, slices.data(), &set) == SOAR_OK &&
              set == static_cast<int>(z.zero1.size()) &&
              soar_optim_use_grads(z.optim, set) == SOAR_OK;
    if (ok)
        ok = soar_zero1_create(z.optim, c.rank, c.world, bases[0].data(), z.param_bases.data(),
                               z.shards.data(), static_cast<int>(z.shards.size()), &z1) ==
             SOAR_OK;
    if (ok && z.sync_mode == SOAR_DP_SYNC_DEVICE)
        ok = soar_zero1_set_signals(z1, bases[1].data()) == SOAR_OK;
    if (!ok) why = soar_last_error();
    soar_optim_use_grads(z.optim, z.cur);
    // every rank's new signal block is bound before any rank steps on it, and
    // the set exists on every rank or on none (an unused optimizer gradient
    // set and the buffers stay until destroy)
    if (!agree(c, ok, &why)) {
        if (z1) soar_zero1_destroy(z1);
        return fail("soar_dp_zero1_add_grads: " + why);
    }
    z.zero1.push_back(z1);
    z.grads.push_back(gbuf);
    *out_index = static_cast<int>(z.zero1.size()) - 1;
    return SOAR_OK;
}

SOAR_API int soar_dp_zero1_use_grads(void* handle, int index) {
    if (!handle) return fail("null handle");
    auto& z = *static_cast<DpZero1*>(handle);
    if (index < 0 || index >= static_cast<int>(z.zero1.size()))
        return fail("bad gradient buffer index");
    const int rc = soar_optim_use_grads(z.optim, index);
    if (rc != SOAR_OK) return rc;
    z.cur = index;
    return SOAR_OK;
}

SOAR_API int soar_dp_zero1_grads(void* handle, int index, void** out_grads) {
    if (!handle || !out_grads) return fail("null argument");
    const auto& z = *static_cast<DpZero1*>(handle);
    if (index < 0 || index >= static_cast<int>(z.grads.size()))
        return fail("bad gradient buffer index");
    *out_grads = z.grads[index];
    return SOAR_OK;
}

SOAR_API int soar_dp_zero1_destroy(void* handle) {
    if (!handle) return fail("null handle");
    auto* z = static_cast<DpZero1*>(handle);
    release(*z);
    delete z;
    return SOAR_OK;
}

}  // extern "C"
