"""ZeRO-1 data-parallel optimizer step (one process per GPU).

Layout: the model's parameters and this rank's gradients are flat bf16
buffers of N elements, cut into buckets of `bucket` elements (the last may be
shorter). Rank r of R owns the contiguous 1/R slice of every bucket; fp32
master, m and v exist only for owned slices (16 B x N/R per rank), held by one
fused optimizer whose tensor list is the owned slices.

One step:
  1. reduce-scatter(avg) of every gradient bucket -> this rank's bf16 slice;
  2. sum of squared unscaled grads over the owned slices (fp64, one number);
  3. all-gather of the R partial sums, which every rank adds in rank order --
     identical bits everywhere, so every rank takes the same skip/clip
     decision (it also carries inf/NaN);
  4. the fused unscale/clip/AdamW update of the owned slices, writing their
     bf16 params in place inside the full parameter buffer;
  5. all-gather of every bucket's bf16 params.
At R = 1 steps 1, 3 and 5 are identities and are skipped.

Two drivers:
* ZeroOneAdamW -- the collectives of steps 1 and 5 are library calls through a
  `Comm` object (torch.distributed / NCCL by default; gloo with a CPU stand-in
  optimizer in the host-logic tests).
* FusedZeroOneAdamW -- steps 1-2 are one kernel and steps 4-5 are one kernel
  over peer memory (soar_zero1_*), set up by the library's data-parallel
  bootstrap (soar_dp_init / soar_dp_zero1_create, usable from C or C++
  without Python): the parameter and gradient buffers are allocated by the
  library and opened by every rank through CUDA IPC. The ranks synchronise
  either inside the kernels, through epoch flags in a symmetric signal block
  (sync="device", no host collective in the step), or through an 8-byte
  partial all-gather and two 4-byte barriers over NCCL (sync="nccl").
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Bucket:
    index: int
    start: int      # element offset of the bucket in the flat buffers
    size: int       # elements in the bucket
    shard: int      # elements per rank (size is padded up to R * shard)
    own_start: int  # element offset of this rank's slice in the flat buffers
    own_size: int   # elements of this rank's slice that are real (<= shard)


def plan_buckets(n: int, bucket: int, world: int, rank: int) -> list[Bucket]:
    """Buckets of `bucket` elements; each split into `world` equal shards
    (the bucket is padded to a multiple of world). Rank `rank` owns shard
    `rank` of every bucket."""
    if n < 0 or bucket <= 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError("bad bucket plan arguments")
    out = []
    b = 0
    for start in range(0, n, bucket):
        size = min(bucket, n - start)
        shard = -(-size // world)
        own_lo = min(size, rank * shard)
        own_hi = min(size, (rank + 1) * shard)
        out.append(Bucket(b, start, size, shard, start + own_lo, own_hi - own_lo))
        b += 1
    return out


class TorchComm:
    """Collectives over a torch.distributed process group."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def reduce_scatter_avg(self, out, inp):
        self.dist.reduce_scatter_tensor(out, inp, op=self.dist.ReduceOp.AVG, group=self.group)

    def all_gather(self, out, inp):
        self.dist.all_gather_into_tensor(out, inp, group=self.group)


class ZeroOneAdamW:
    """ZeRO-1 driver around the fused optimizer.

    params: flat bf16 CUDA tensor of N elements (the full model, replicated);
    grads:  flat bf16 CUDA tensor of N elements (this rank's local gradient);
    make_optimizer(shard_params, shard_grads) -> object with
            grad_sumsq(ptr) and apply(ptr, n_parts) (soar_b200.AdamW).
    Buckets whose size is not a multiple of R are padded inside private
    staging buffers; in the common case (R divides the bucket) the
    reduce-scatter writes straight into the optimizer's gradient slices and the
    all-gather reads straight from the updated parameter slices.
    """

    def __init__(self, params, grads, bucket: int, make_optimizer, comm=None):
        import torch
        self.torch = torch
        self.params = params
        self.grads = grads
        self.n = params.numel()
        self.comm = comm
        self.world = comm.world if comm else 1
        self.rank = comm.rank if comm else 0
        self.buckets = plan_buckets(self.n, bucket, self.world, self.rank)
        dev = params.device
        self.padded = any(b.size % self.world for b in self.buckets)
        if self.world == 1:
            shard_p = [params[b.start:b.start + b.size] for b in self.buckets]
            shard_g = [grads[b.start:b.start + b.size] for b in self.buckets]
        else:
            # this rank's gradient slices (reduce-scatter output)
            self.gshard = torch.empty(sum(b.shard for b in self.buckets), dtype=grads.dtype,
                                      device=dev)
            shard_g, shard_p, off = [], [], 0
            for b in self.buckets:
                shard_g.append(self.gshard[off:off + b.own_size])
                shard_p.append(params[b.own_start:b.own_start + b.own_size])
                off += b.shard
            if self.padded:
                self.pad_in = torch.zeros(max(b.shard for b in self.buckets) * self.world,
                                          dtype=grads.dtype, device=dev)
                self.pad_out = torch.zeros_like(self.pad_in)
        self.shard_params = shard_p
        self.shard_grads = shard_g
        self.opt = make_optimizer(shard_p, shard_g)
        self.part = torch.zeros(1, dtype=torch.float64, device=dev)
        self.parts = torch.zeros(self.world, dtype=torch.float64, device=dev)

    # -- the five phases (separately callable for timing) -------------------
    def reduce_scatter(self):
        if self.world == 1:
            return
        off = 0
        for b in self.buckets:
            out = self.gshard[off:off + b.shard]
            src = self.grads[b.start:b.start + b.size]
            if b.size % self.world:
                self.pad_in[:b.size].copy_(src)
                self.pad_in[b.size:b.shard * self.world].zero_()
                self.comm.reduce_scatter_avg(out, self.pad_in[:b.shard * self.world])
            else:
                self.comm.reduce_scatter_avg(out, src)
            off += b.shard

    def norm_partials(self):
        self.opt.grad_sumsq(self.part.data_ptr())
        if self.world == 1:
            return self.part
        self.comm.all_gather(self.parts, self.part)
        return self.parts

    def update(self, parts):
        self.opt.apply(parts.data_ptr(), parts.numel())

    def all_gather(self):
        if self.world == 1:
            return
        for b in self.buckets:
            full = self.params[b.start:b.start + b.size]
            mine = self.params[b.own_start:b.own_start + b.shard]
            if b.size % self.world or b.own_size != b.shard:
                self.pad_out[:b.own_size].copy_(self.params[b.own_start:b.own_start + b.own_size])
                self.comm.all_gather(self.pad_in[:b.shard * self.world], self.pad_out[:b.shard])
                full.copy_(self.pad_in[:b.size])
            else:
                self.comm.all_gather(full, mine)

    def step(self):
        self.reduce_scatter()
        parts = self.norm_partials()
        self.update(parts)
        self.all_gather()


class _DevView:
    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


class FusedZeroOneAdamW:
    """ZeRO-1 step with the reduce-scatter fused into the norm pass and the
    all-gather fused into the update (see the module docstring): a thin
    caller of the library's data-parallel bootstrap (soar_dp_init /
    soar_dp_zero1_create), which allocates and exchanges the symmetric buffers,
    plans the buckets and owns the shard optimizer. torch.distributed only
    carries NCCL's 128-byte unique id from rank 0 to the other ranks.

    `params` / `grads` are flat bf16 CUDA tensors viewing library-owned
    symmetric buffers: fill `grads` with this rank's gradient before step();
    after step() `params` holds the updated full model on every rank. The
    rank's own slice of `grads` is overwritten with the reduced average.
    `options` / max_grad_norm / loss_scaler configure the bf16-mixed AdamW of
    the owned slices (every slice takes options.weight_decay); init_params
    (n bf16 values, any device) is copied into `params` before the optimizer
    is created, so its fp32 master weights start from them.

    sync="device" (default) synchronises the ranks inside the kernels through
    epoch flags in a small symmetric signal block (no host collective in the
    step); sync="nccl" issues the three synchronisation points as small NCCL
    collectives between the launches (over the library's communicator).
    close() is collective: every rank calls it."""

    def __init__(self, n: int, bucket: int, options=None, *, max_grad_norm: float = 0.0,
                 loss_scaler=None, group=None, device: int | None = None, init_params=None,
                 sync: str = "device"):
        import ctypes as C

        import torch
        import torch.distributed as dist

        from . import optim as _o
        if sync not in ("device", "nccl"):
            raise ValueError("sync must be 'device' or 'nccl'")
        self.torch, self.dist, self.group = torch, dist, group
        self.lib = _o.lib()
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = torch.cuda.current_device() if device is None else device
        self.n = n
        self.sync = sync
        self.buckets = plan_buckets(n, bucket, self.world, self.rank)
        self.handle = self.comm = None
        # NCCL's unique id, from rank 0 to every rank over torch.distributed
        uid = (C.c_ubyte * _o.DP_UNIQUE_ID_BYTES)()
        if self.rank == 0:
            _o._check(self.lib.soar_dp_unique_id(uid), "soar_dp_unique_id")
        if self.world > 1:
            box = [bytes(uid)]
            src = dist.get_global_rank(group, 0) if group is not None else 0
            dist.broadcast_object_list(box, src=src, group=group)
            uid = (C.c_ubyte * _o.DP_UNIQUE_ID_BYTES).from_buffer_copy(box[0])
        comm = C.c_void_p()
        _o._check(self.lib.soar_dp_init(self.rank, self.world, uid, self.device, C.byref(comm)),
                  "soar_dp_init")
        self.comm = comm
        options = options or _o.AdamWOptions()
        o = _o.AdamWOpts()
        self.lib.soar_adamw_default_opts(C.byref(o))
        o.lr, o.beta1, o.beta2, o.eps = options.lr, options.beta1, options.beta2, options.eps
        o.weight_decay = options.weight_decay
        o.layout = _o.LAYOUT_BF16_MIXED
        o.max_grad_norm = max_grad_norm
        if loss_scaler is not None:
            o.use_loss_scaler = 1
            o.init_scale = loss_scaler.init_scale
            o.growth_factor = loss_scaler.growth_factor
            o.backoff_factor = loss_scaler.backoff_factor
            o.growth_interval = loss_scaler.growth_interval
        o.device = self.device
        init = None
        if init_params is not None:
            init_params = init_params.contiguous()
            init = init_params.data_ptr()
        h = C.c_void_p()
        rc = self.lib.soar_dp_zero1_create(comm, n, bucket, C.byref(o), init,
                                           _o.DP_SYNC_DEVICE if sync == "device"
                                           else _o.DP_SYNC_NCCL, C.byref(h))
        if rc != 0:
            msg = self.lib.soar_last_error().decode(errors="replace")
            self.lib.soar_dp_destroy(comm)
            self.comm = None
            raise _o.SoarError(f"soar_dp_zero1_create failed: {msg}")
        self.handle = h
        info = _o.DpZero1Info()
        _o._check(self.lib.soar_dp_zero1_get_info(h, C.byref(info)), "soar_dp_zero1_get_info")
        dev = f"cuda:{self.device}"
        self.grads = torch.as_tensor(_DevView(info.grads, n, "<i2"), device=dev).view(
            torch.bfloat16)
        self.params = torch.as_tensor(_DevView(info.params, n, "<i2"), device=dev).view(
            torch.bfloat16)
        mine = [b for b in self.buckets if b.own_size > 0]
        self.shard_params = [self.params[b.own_start:b.own_start + b.own_size] for b in mine]
        self.shard_grads = [self.grads[b.own_start:b.own_start + b.own_size] for b in mine]
        self.opt = _o.AdamW.borrow(info.optimizer, [b.own_size for b in mine], self.device)
        self.zero1 = C.c_void_p(info.zero1)
        self.grad_buffers = [self.grads]
        self._mine = mine
        self.part = torch.zeros(1, dtype=torch.float64, device=dev)
        self.parts = torch.zeros(self.world, dtype=torch.float64, device=dev)

    def _stream(self):
        return self.torch.cuda.current_stream().cuda_stream

    def add_grads(self) -> int:
        """Collective: another symmetric gradient buffer (soar_dp_zero1_add_grads),
        so the next step's gradient can be written while a step reads the
        current one. Returns its index; its view is grad_buffers[index]."""
        import ctypes as C

        from . import optim as _o
        k = C.c_int()
        _o._check(self.lib.soar_dp_zero1_add_grads(self.handle, C.byref(k)),
                  "soar_dp_zero1_add_grads")
        ptr = C.c_void_p()
        _o._check(self.lib.soar_dp_zero1_grads(self.handle, k.value, C.byref(ptr)),
                  "soar_dp_zero1_grads")
        self.grad_buffers.append(self.torch.as_tensor(
            _DevView(ptr.value, self.n, "<i2"), device=f"cuda:{self.device}").view(
            self.torch.bfloat16))
        return k.value

    def use_grads(self, index: int) -> None:
        """The gradient buffer the next steps reduce (every rank the same)."""
        import ctypes as C

        from . import optim as _o
        _o._check(self.lib.soar_dp_zero1_use_grads(self.handle, index), "soar_dp_zero1_use_grads")
        info = _o.DpZero1Info()
        _o._check(self.lib.soar_dp_zero1_get_info(self.handle, C.byref(info)),
                  "soar_dp_zero1_get_info")
        self.zero1 = C.c_void_p(info.zero1)
        self.grads = self.grad_buffers[index]
        self.shard_grads = [self.grads[b.own_start:b.own_start + b.own_size] for b in self._mine]

    def barrier(self):
        """Stream-ordered barrier: completes on this GPU only after every
        rank's earlier work on its stream has completed."""
        from . import optim as _o
        if self.world > 1:
            _o._check(self.lib.soar_dp_barrier(self.comm, self._stream()), "soar_dp_barrier")

    def reduce(self):
        from . import optim as _o
        _o._check(self.lib.soar_zero1_reduce_sumsq(self.zero1, self.part.data_ptr(),
                                                    self._stream()), "soar_zero1_reduce_sumsq")

    def gather_partials(self):
        from . import optim as _o
        if self.world > 1:
            _o._check(self.lib.soar_dp_allgather_f64(self.comm, self.part.data_ptr(),
                                                      self.parts.data_ptr(), 1, self._stream()),
                      "soar_dp_allgather_f64")
            return self.parts
        return self.part

    def update(self, parts):
        from . import optim as _o
        _o._check(self.lib.soar_zero1_apply_allgather(self.zero1, parts.data_ptr(), parts.numel(),
                                                       self._stream()),
                  "soar_zero1_apply_allgather")

    def step(self):
        from . import optim as _o
        _o._check(self.lib.soar_dp_zero1_step(self.handle, self._stream()), "soar_dp_zero1_step")

    def error(self) -> int:
        import ctypes as C

        from . import optim as _o
        out = C.c_int()
        _o._check(self.lib.soar_zero1_error(self.zero1, C.byref(out)), "soar_zero1_error")
        return out.value

    def close(self):
        """Collective: every rank calls it (no rank frees while a peer maps)."""
        if getattr(self, "handle", None) is not None:
            self.torch.cuda.synchronize(self.device)
            self.opt.close()
            self.lib.soar_dp_zero1_destroy(self.handle)
            self.handle = None
        if getattr(self, "comm", None) is not None:
            self.lib.soar_dp_destroy(self.comm)
            self.comm = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
