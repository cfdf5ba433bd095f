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
  over peer memory (soar_zero1_*): the parameter and gradient buffers are
  allocated by the library and opened by every rank through CUDA IPC. The
  ranks synchronise either inside the kernels, through epoch flags in a
  symmetric signal block (sync="device", no host collective in the step), or
  through an 8-byte partial all-gather and two 4-byte barriers over NCCL
  (sync="nccl").
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
    all-gather fused into the update (see the module docstring).

    `params` / `grads` are flat bf16 CUDA tensors viewing library-owned
    symmetric buffers: fill `grads` with this rank's gradient before step();
    after step() `params` holds the updated full model on every rank. The
    rank's own slice of `grads` is overwritten with the reduced average.
    make_optimizer(shard_params, shard_grads) -> soar_b200.AdamW (bf16_mixed).
    init_params (n bf16 values, any device) is copied into `params` before the
    optimizer is created, so its fp32 master weights start from them.

    sync="device" (default) synchronises the ranks inside the kernels through
    epoch flags in a small symmetric signal block (soar_zero1_step: no host
    collective in the step); sync="nccl" issues the three synchronisation
    points as small NCCL collectives between the launches.
    """

    def __init__(self, n: int, bucket: int, make_optimizer, group=None, device: int | None = None,
                 init_params=None, sync: str = "device"):
        import ctypes as C

        import torch
        import torch.distributed as dist

        from . import optim as _o
        self.torch, self.dist, self.group = torch, dist, group
        self.lib = _o.lib()
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = torch.cuda.current_device() if device is None else device
        self.n = n
        self.buckets = plan_buckets(n, bucket, self.world, self.rank)
        self._local, self._peers, self.zero1 = [], [], None
        if sync not in ("device", "nccl"):
            raise ValueError("sync must be 'device' or 'nccl'")
        self.sync = sync
        bases = {}
        sizes = {"grads": 2 * n, "params": 2 * n}
        if sync == "device":
            sizes["signals"] = _o.ZERO1_SIGNAL_BYTES
        for name, nbytes in sizes.items():
            ptr = C.c_void_p()
            handle = (C.c_ubyte * _o.IPC_HANDLE_BYTES)()
            _o._check(self.lib.soar_ipc_alloc(nbytes, self.device, C.byref(ptr), handle),
                      "soar_ipc_alloc")
            self._local.append(ptr.value)
            handles = [None] * self.world
            if self.world > 1:
                dist.all_gather_object(handles, bytes(handle), group=group)
            else:
                handles = [bytes(handle)]
            row = []
            for q, h in enumerate(handles):
                if q == self.rank:
                    row.append(ptr.value)
                    continue
                peer = C.c_void_p()
                buf = (C.c_ubyte * _o.IPC_HANDLE_BYTES).from_buffer_copy(h)
                _o._check(self.lib.soar_ipc_open(buf, self.device, C.byref(peer)), "soar_ipc_open")
                self._peers.append(peer.value)
                row.append(peer.value)
            bases[name] = row
        dev = f"cuda:{self.device}"
        self.grads = torch.as_tensor(_DevView(bases["grads"][self.rank], n, "<i2"),
                                     device=dev).view(torch.bfloat16)
        self.params = torch.as_tensor(_DevView(bases["params"][self.rank], n, "<i2"),
                                      device=dev).view(torch.bfloat16)
        if init_params is not None:
            self.params.copy_(init_params)
        mine = [b for b in self.buckets if b.own_size > 0]
        self.shard_params = [self.params[b.own_start:b.own_start + b.own_size] for b in mine]
        self.shard_grads = [self.grads[b.own_start:b.own_start + b.own_size] for b in mine]
        self.opt = make_optimizer(self.shard_params, self.shard_grads)
        shards = (_o.Zero1Shard * max(1, len(mine)))()
        for i, b in enumerate(mine):
            shards[i].offset, shards[i].count, shards[i].tensor = b.own_start, b.own_size, i
        gb = (C.c_void_p * self.world)(*bases["grads"])
        pb = (C.c_void_p * self.world)(*bases["params"])
        h = C.c_void_p()
        _o._check(self.lib.soar_zero1_create(self.opt.handle, self.rank, self.world, gb, pb,
                                             shards, len(mine), C.byref(h)), "soar_zero1_create")
        self.zero1 = h
        if sync == "device":
            sb = (C.c_void_p * self.world)(*bases["signals"])
            _o._check(self.lib.soar_zero1_set_signals(h, sb), "soar_zero1_set_signals")
        self.part = torch.zeros(1, dtype=torch.float64, device=dev)
        self.parts = torch.zeros(self.world, dtype=torch.float64, device=dev)
        self.flag = torch.zeros(1, dtype=torch.float32, device=dev)

    def _stream(self):
        return self.torch.cuda.current_stream().cuda_stream

    def barrier(self):
        """Stream-ordered barrier: completes on this GPU only after every
        rank's earlier work on its stream has completed."""
        if self.world > 1:
            self.dist.all_reduce(self.flag, group=self.group)

    def reduce(self):
        from . import optim as _o
        _o._check(self.lib.soar_zero1_reduce_sumsq(self.zero1, self.part.data_ptr(),
                                                    self._stream()), "soar_zero1_reduce_sumsq")

    def gather_partials(self):
        if self.world > 1:
            self.dist.all_gather_into_tensor(self.parts, self.part, group=self.group)
            return self.parts
        return self.part

    def update(self, parts):
        from . import optim as _o
        _o._check(self.lib.soar_zero1_apply_allgather(self.zero1, parts.data_ptr(), parts.numel(),
                                                       self._stream()),
                  "soar_zero1_apply_allgather")

    def step(self):
        if self.sync == "device":
            from . import optim as _o
            _o._check(self.lib.soar_zero1_step(self.zero1, self._stream()), "soar_zero1_step")
            return
        self.barrier()                        # every rank's gradients are complete
        self.reduce()                         # reduce-scatter + sum of squares
        self.update(self.gather_partials())   # update + all-gather
        self.barrier()                        # every peer's parameter writes landed

    def error(self) -> int:
        import ctypes as C

        from . import optim as _o
        out = C.c_int()
        _o._check(self.lib.soar_zero1_error(self.zero1, C.byref(out)), "soar_zero1_error")
        return out.value

    def close(self):
        if getattr(self, "zero1", None) is None and not getattr(self, "_local", None):
            return
        self.torch.cuda.synchronize(self.device)
        if self.zero1 is not None:
            self.lib.soar_zero1_destroy(self.zero1)
            self.zero1 = None
        if getattr(self, "opt", None) is not None:
            self.opt.close()
        for p in self._peers:
            self.lib.soar_ipc_close(p, self.device)
        self._peers = []
        for p in self._local:
            self.lib.soar_ipc_free(p, self.device)
        self._local = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
