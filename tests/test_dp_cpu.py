"""Host logic of the ZeRO-1 data-parallel step on CPU: world_size-2 gloo ranks run
the real driver (soar_b200.dp.ZeroOneAdamW) with the port oracle standing in for
the device optimizer, and the result is checked against one process running
the oracle over the averaged gradients. Covers bucket planning (ragged last
bucket, buckets not divisible by the world size), the reduce-scatter /
partial-sum all-gather / param all-gather sequence and the identical
skip/clip decision on every rank. CPU only, no GPU."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from soar_b200 import dp, synth

N = 5003          # params: ragged buckets
BUCKET = 1001     # not a multiple of the world size
STEPS = 6
INF_STEP = 4      # rank 1 injects +inf at this step: every rank must skip it


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def _grads(rank, step, scale):
    g = synth.normal(synth.seed_of(40, rank, step), N, 0.5) * np.float32(scale)
    if step == INF_STEP and rank == 1:
        g[17] = np.inf
    return synth.to_bf16_bits(g.astype(np.float32))


class GlooComm:
    """Reference collectives over gloo: the reduce-scatter averages in fp32 in
    rank order and rounds to bf16 once (the oracle's definition)."""

    def __init__(self):
        self.world = dist.get_world_size()
        self.rank = dist.get_rank()

    def _gather(self, inp):
        # gloo moves no 16-bit integers: carry the bf16 bits as int32
        wire = inp.contiguous().view(torch.int16).to(torch.int32)
        parts = [torch.empty_like(wire) for _ in range(self.world)]
        dist.all_gather(parts, wire)
        return [p.to(torch.int16).view(inp.dtype) for p in parts]

    def reduce_scatter_avg(self, out, inp):
        parts = self._gather(inp)
        s = torch.zeros(inp.numel(), dtype=torch.float32)
        for p in parts:
            s = s + p.float()
        avg = (s * torch.tensor(1.0 / self.world, dtype=torch.float32)).to(torch.bfloat16)
        n = out.numel()
        out.copy_(avg[self.rank * n:(self.rank + 1) * n])

    def all_gather(self, out, inp):
        if inp.dtype == torch.float64:
            parts = [torch.empty_like(inp) for _ in range(self.world)]
            dist.all_gather(parts, inp.contiguous())
        else:
            parts = self._gather(inp)
        out.copy_(torch.cat(parts))


def _worker(rank, world, port, q):
    from oracle import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        p0 = synth.to_bf16_bits(synth.normal(synth.seed_of(41), N, 0.02))
        params = _bf16(p0.copy())
        grads = _bf16(np.zeros(N, np.uint16))
        cfg = oracle.StepConfig(layout=1, max_norm=1.0, use_scaler=True, growth_interval=3)

        def make(shard_p, shard_g):
            np_p = [t.view(torch.int16).numpy().view(np.uint16) for t in shard_p]
            np_g = [t.view(torch.int16).numpy().view(np.uint16) for t in shard_g]
            return oracle.PortShard(np_p, np_g, [0.01] * len(np_p), cfg, init_scale=256.0)

        z = dp.ZeroOneAdamW(params, grads, BUCKET, make, GlooComm())
        hist = []
        for t in range(1, STEPS + 1):
            grads.copy_(_bf16(_grads(rank, t, z.opt.state.scale)))
            z.step()
            st = z.opt.state
            hist.append((st.skipped, st.scale, st.t))
        q.put((rank, params.view(torch.int16).numpy().view(np.uint16).copy(), hist))
    finally:
        dist.destroy_process_group()


def test_zero1_two_gloo_ranks_match_single_process_oracle(oracle_mod):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    import queue
    import time
    deadline = time.time() + 240
    while len(results) < world and time.time() < deadline:
        try:
            r, params, hist = q.get(timeout=2)
            results[r] = (params, hist)
        except queue.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    for p in procs:
        if p.is_alive() and len(results) < world:
            p.terminate()
    assert len(results) == world, "a rank failed"
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # every rank ends with the same full params and the same decisions
    np.testing.assert_array_equal(results[0][0], results[1][0])
    assert results[0][1] == results[1][1]

    # single process: average the two ranks' grads (oracle definition), one
    # optimizer over the same buckets
    o = oracle_mod
    buckets = dp.plan_buckets(N, BUCKET, 1, 0)
    p_full = synth.to_bf16_bits(synth.normal(synth.seed_of(41), N, 0.02))
    views = [p_full[b.start:b.start + b.size] for b in buckets]
    cfg = o.StepConfig(layout=1, max_norm=1.0, use_scaler=True, growth_interval=3)
    ref = o.PortOptimizer(views, [0.01] * len(views), cfg, init_scale=256.0)
    ref.params = views
    hist = []
    for t in range(1, STEPS + 1):
        g = o.reduce_avg_bf16([_grads(r, t, ref.state.scale) for r in range(world)])
        ref.step([g[b.start:b.start + b.size] for b in buckets])
        hist.append((ref.state.skipped, ref.state.scale, ref.state.t))
    assert hist == results[0][1], (hist, results[0][1])
    assert hist[INF_STEP - 1][0] == 1  # the injected step was skipped everywhere
    got = results[0][0].astype(np.int32)
    want = p_full.astype(np.int32)
    assert np.abs(got - want).max() <= 1  # <= 1 bf16 ulp (norm summation order differs)


def test_plan_buckets_covers_every_element():
    for n, bucket, world in [(5003, 1001, 2), (100, 7, 4), (25_000_000 * 8, 25_000_000, 8),
                             (1, 1000, 8), (0, 10, 2)]:
        seen = np.zeros(n, np.int32)
        for r in range(world):
            for b in dp.plan_buckets(n, bucket, world, r):
                assert b.own_size <= b.shard and b.size <= bucket
                seen[b.own_start:b.own_start + b.own_size] += 1
        assert (seen == 1).all()
    with pytest.raises(ValueError):
        dp.plan_buckets(10, 0, 2, 0)
