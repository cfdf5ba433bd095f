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

The collectives go through a `Comm` object (torch.distributed by default), so
the same driver runs over NCCL on GPUs and over gloo with a CPU stand-in
optimizer in the host-logic tests.
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
