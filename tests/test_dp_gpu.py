"""ZeRO-1 on 2 GPUs over NCCL, through the real driver and the CUDA optimizer.

Each rank brings its own bf16 gradient; the step reduce-scatters it (NCCL,
avg), runs the fused update on the rank's shard and all-gathers the params.
The reduce-scatter has no reference counterpart and NCCL's summation order is
its own, so parity is taken on what the optimizer received: every step the
ranks' post-reduce-scatter shards are read back, reassembled, and fed to the
single-process oracle. Checks: identical params on both ranks, skip /
loss-scale / step sequences bit-exact, params within 1 bf16 ulp, and the
reduce-scatter within bf16 rounding of the fp64 mean. The fused path (both
synchronisation modes) and its bounded device-side waits are tested below.
Skipped below 2 GPUs."""
import datetime
import os
import queue
import socket
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N = 3_000_017
BUCKET = 1_000_000
STEPS = 5
INF_STEP = 3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _grads(rank, step, scale):
    from soar_b200 import synth
    g = synth.normal(synth.seed_of(50, rank, step), N, 0.01) * np.float32(scale)
    if step == INF_STEP and rank == 1:
        g[123] = np.inf
    return synth.to_bf16_bits(g.astype(np.float32))


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    import soar_b200 as sb
    from soar_b200 import dp, synth
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        bf = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()
        params = bf(synth.to_bf16_bits(synth.normal(synth.seed_of(51), N, 0.02)))
        grads = torch.empty_like(params)

        def make(sp, sg):
            return sb.AdamW([sb.ParamGroup(sp, 0.01)], layout="bf16_mixed", max_grad_norm=1.0,
                            loss_scaler=sb.LossScalerOptions(init_scale=1024.0,
                                                             growth_interval=2),
                            grads=sg, device=rank)

        z = dp.ZeroOneAdamW(params, grads, BUCKET, make, dp.TorchComm())
        scale = 1024.0
        shards, hist = [], []
        for t in range(1, STEPS + 1):
            grads.copy_(bf(_grads(rank, t, scale)))
            z.reduce_scatter()
            shards.append(z.gshard.view(torch.int16).cpu().numpy().view(np.uint16).copy())
            z.update(z.norm_partials())
            z.all_gather()
            info = z.opt.info()
            scale = info.loss_scale
            hist.append((info.skipped, info.loss_scale, info.step))
        torch.cuda.synchronize()
        out = params.view(torch.int16).cpu().numpy().view(np.uint16).copy()
        q.put((rank, out, hist, shards, [(b.shard, b.own_size) for b in z.buckets]))
        del z
    finally:
        dist.destroy_process_group()


def test_zero1_two_gpus_nccl(oracle_mod):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from soar_b200 import dp, synth
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    deadline = time.time() + 300
    while len(res) < world and time.time() < deadline:
        try:
            r, *rest = q.get(timeout=2)
            res[r] = rest
        except queue.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    for p in procs:
        if p.is_alive() and len(res) < world:
            p.terminate()
        p.join(timeout=60)
    assert len(res) == world, "a rank failed"
    np.testing.assert_array_equal(res[0][0], res[1][0])
    assert res[0][1] == res[1][1]

    # reassemble each step's reduced gradient from the ranks' shards
    o = oracle_mod
    full_buckets = dp.plan_buckets(N, BUCKET, 1, 0)
    p_full = synth.to_bf16_bits(synth.normal(synth.seed_of(51), N, 0.02))
    views = [p_full[b.start:b.start + b.size] for b in full_buckets]
    cfg = o.StepConfig(layout=1, max_norm=1.0, use_scaler=True, growth_interval=2)
    ref = o.PortOptimizer(views, [0.01] * len(views), cfg, init_scale=1024.0)
    ref.params = views
    hist = []
    for t in range(STEPS):
        reduced = np.empty(N, np.uint16)
        for b_full in full_buckets:
            shard = -(-b_full.size // world)
            for r in range(world):
                off = sum(sh for sh, _ in res[r][3][:b_full.index])
                lo = min(b_full.size, r * shard)
                hi = min(b_full.size, (r + 1) * shard)
                reduced[b_full.start + lo:b_full.start + hi] = res[r][2][t][off:off + hi - lo]
        # the reduce-scatter itself: within bf16 rounding of the fp64 mean
        ins = [synth.from_bf16_bits(_grads(r, t + 1, ref.state.scale)).astype(np.float64)
               for r in range(world)]
        mean = sum(ins) / world
        got = synth.from_bf16_bits(reduced).astype(np.float64)
        fin = np.isfinite(mean)
        assert np.all(np.abs(got[fin] - mean[fin]) <= np.abs(mean[fin]) * 2.0 ** -7 + 1e-30)
        ref.step([reduced[b.start:b.start + b.size] for b in full_buckets])
        hist.append((ref.state.skipped, ref.state.scale, ref.state.t))
    assert hist == res[0][1], (hist, res[0][1])
    assert hist[INF_STEP - 1][0] == 1
    diff = np.abs(res[0][0].astype(np.int32) - p_full.astype(np.int32))
    assert diff.max() <= 1


def _fused_worker(rank, world, port, q, sync="nccl"):
    import torch
    import torch.distributed as dist

    import soar_b200 as sb
    from soar_b200 import dp, synth
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    fz = None
    try:
        bf = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()
        p0 = bf(synth.to_bf16_bits(synth.normal(synth.seed_of(51), N, 0.02)))
        fz = dp.FusedZeroOneAdamW(N, BUCKET, sb.AdamWOptions(weight_decay=0.01),
                                  max_grad_norm=1.0,
                                  loss_scaler=sb.LossScalerOptions(init_scale=1024.0,
                                                                   growth_interval=2),
                                  device=rank, init_params=p0, sync=sync)
        scale = 1024.0
        reduced, hist = [], []
        own = lambda: [fz.grads[b.own_start:b.own_start + b.own_size].view(torch.int16).cpu()
                       .numpy().view(np.uint16).copy() for b in fz.buckets]
        for t in range(1, STEPS + 1):
            fz.grads.copy_(bf(_grads(rank, t, scale)))
            if sync == "device":
                fz.step()  # the reduce leaves the averaged slice in place
                torch.cuda.synchronize()
                reduced.append(own())
            else:
                fz.barrier()
                fz.reduce()
                torch.cuda.synchronize()
                reduced.append(own())
                fz.update(fz.gather_partials())
                fz.barrier()
            info = fz.opt.info()
            scale = info.loss_scale
            hist.append((info.skipped, info.loss_scale, info.step))
        torch.cuda.synchronize()
        out = fz.params.view(torch.int16).cpu().numpy().view(np.uint16).copy()
        q.put((rank, out, hist, reduced, fz.error()))
    finally:
        if fz is not None:
            fz.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("sync", ["nccl", "device"])
def test_fused_zero1_two_gpus(oracle_mod, sync):
    """The fused path: reduce-scatter inside the norm kernel and all-gather
    inside the update, over peer memory; the ranks synchronised by small NCCL
    collectives between the launches or by device-side epoch flags. Its
    reduce is defined exactly as the oracle's (fp32 sum in rank order, one
    rounding), so the reduced shards are checked bit-for-bit; the step against
    the single-process oracle."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from soar_b200 import dp, synth
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, world, port, q, sync))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    deadline = time.time() + 300
    while len(res) < world and time.time() < deadline:
        try:
            r, *rest = q.get(timeout=2)
            res[r] = rest
        except queue.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    for p in procs:
        if p.is_alive() and len(res) < world:
            p.terminate()
        p.join(timeout=60)
    assert len(res) == world, "a rank failed"
    assert res[0][3] == 0 and res[1][3] == 0, "device-side wait timed out"
    np.testing.assert_array_equal(res[0][0], res[1][0])
    assert res[0][1] == res[1][1]

    o = oracle_mod
    full_buckets = dp.plan_buckets(N, BUCKET, 1, 0)
    p_full = synth.to_bf16_bits(synth.normal(synth.seed_of(51), N, 0.02))
    views = [p_full[b.start:b.start + b.size] for b in full_buckets]
    cfg = o.StepConfig(layout=1, max_norm=1.0, use_scaler=True, growth_interval=2)
    ref = o.PortOptimizer(views, [0.01] * len(views), cfg, init_scale=1024.0)
    ref.params = views
    hist = []
    for t in range(STEPS):
        avg = o.reduce_avg_bf16([_grads(r, t + 1, ref.state.scale) for r in range(world)])
        for r in range(world):
            for b, got in zip(dp.plan_buckets(N, BUCKET, world, r), res[r][2][t]):
                np.testing.assert_array_equal(got, avg[b.own_start:b.own_start + b.own_size])
        ref.step([avg[b.start:b.start + b.size] for b in full_buckets])
        hist.append((ref.state.skipped, ref.state.scale, ref.state.t))
    assert hist == res[0][1], (hist, res[0][1])
    assert hist[INF_STEP - 1][0] == 1
    diff = np.abs(res[0][0].astype(np.int32) - p_full.astype(np.int32))
    assert diff.max() <= 1


def _absent_peer_worker(rank, world, port, q):
    """Rank 0 steps; rank 1 is alive but never steps. Rank 0's bounded waits
    (the ready flags, then the done flags: 1 s each; the partial exchange is
    skipped once a wait failed) run out, the update is skipped and the error
    flag is set; nothing waits forever."""
    import torch
    import torch.distributed as dist

    import soar_b200 as sb
    from soar_b200 import dp, synth
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    fz = None
    try:
        bf = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()
        p0 = bf(synth.to_bf16_bits(synth.normal(synth.seed_of(51), N, 0.02)))

        fz = dp.FusedZeroOneAdamW(N, BUCKET, sb.AdamWOptions(weight_decay=0.01), device=rank,
                                  init_params=p0, sync="device")
        fz.grads.copy_(bf(_grads(rank, 1, 1.0)))
        dist.barrier()
        out = None
        if rank == 0:
            before = fz.params.view(torch.int16).cpu().numpy().copy()
            t0 = time.time()
            fz.step()
            torch.cuda.synchronize()
            waited = time.time() - t0
            after = fz.params.view(torch.int16).cpu().numpy()
            info = fz.opt.info()
            out = (fz.error(), waited, bool((before == after).all()), info.step, info.skipped)
        dist.barrier()  # rank 1 keeps its buffers mapped until rank 0 is done
        q.put((rank, out))
    finally:
        if fz is not None:
            fz.close()
        dist.destroy_process_group()


def test_device_sync_wait_times_out_and_reports():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_absent_peer_worker, args=(r, world, port, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    deadline = time.time() + 300
    while len(res) < world and time.time() < deadline:
        try:
            r, out = q.get(timeout=2)
            res[r] = out
        except queue.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    for p in procs:
        if p.is_alive() and len(res) < world:
            p.terminate()
        p.join(timeout=60)
    assert len(res) == world, "a rank failed"
    err, waited, unchanged, step, skipped = res[0]
    assert err == 1
    assert 1.5 < waited < 30.0, waited      # two bounded waits of 1 s (ready, then done)
    assert unchanged                        # the update was skipped
    assert (step, skipped) == (0, 1)        # and counted as a skipped step


N4, B4 = 200_000_000, 25_000_000   # config 4 in full


def _full_c4_worker(rank, world, port, q):
    """Config 4 at full size on 2 GPUs (device-synchronised fused step) against
    a single-GPU step on the average gradient (the oracle's reduce: fp32 sum in
    rank order, one multiply by 1/R, one bf16 rounding), on rank 0."""
    import torch
    import torch.distributed as dist

    import soar_b200 as sb
    from soar_b200 import dp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    fz = ref = None
    try:
        gen = torch.Generator(device="cuda")
        gen.manual_seed(4000 + rank)
        p0 = (torch.randn(N4, device="cuda", generator=gen) * 0.02).bfloat16()
        dist.broadcast(p0, 0)
        scaler = sb.LossScalerOptions(init_scale=65536.0)

        def make(sp, sg):
            return sb.AdamW([sb.ParamGroup(sp, 0.01)], layout="bf16_mixed", max_grad_norm=1.0,
                            loss_scaler=scaler, grads=sg, device=rank)

        fz = dp.FusedZeroOneAdamW(N4, B4, sb.AdamWOptions(weight_decay=0.01), max_grad_norm=1.0,
                                  loss_scaler=scaler, device=rank, init_params=p0, sync="device")
        full = dp.plan_buckets(N4, B4, 1, 0)
        if rank == 0:
            ref_p = p0.clone()
            ref_g = torch.empty_like(ref_p)
            ref = make([ref_p[b.start:b.start + b.size] for b in full],
                       [ref_g[b.start:b.start + b.size] for b in full])
        scale = 65536.0
        for t in range(1, 4):
            fz.grads.copy_((torch.randn(N4, device="cuda", generator=gen) * (1e-3 * scale))
                           .bfloat16())
            if t == 2 and rank == 1:
                fz.grads[123_456_789] = float("inf")
            if rank == 1:
                dist.send(fz.grads.clone(), 0)
            else:
                other = torch.empty_like(fz.grads)
                dist.recv(other, 1)
                ref_g.copy_(((fz.grads.float() + other.float()) * 0.5).bfloat16())
                del other
            fz.step()
            if ref is not None:
                ref.step()
            scale = fz.opt.info().loss_scale
        torch.cuda.synchronize()
        i = fz.opt.info()
        out = {"info": (i.step, i.skipped, i.loss_scale), "err": fz.error()}
        if rank == 1:
            dist.send(fz.params.clone(), 0)
        else:
            other = torch.empty_like(fz.params)
            dist.recv(other, 1)
            out["ranks_equal"] = bool(torch.equal(other.view(torch.int16),
                                                  fz.params.view(torch.int16)))
            del other

            def ordered(x):
                x = x.view(torch.int16).int()
                return torch.where(x < 0, -(x & 0x7FFF), x)
            d = (ordered(fz.params) - ordered(ref_p)).abs()
            out["max_ulp"] = int(d.max())
            out["ulp_mismatches"] = int((d > 0).sum())
            ri = ref.info()
            out["ref_info"] = (ri.step, ri.skipped, ri.loss_scale)
            worst = 0.0
            mine = [b for b in fz.buckets if b.own_size > 0]
            for k, b in enumerate(mine):
                lo = b.own_start - full[b.index].start
                for kind in (sb.STATE_MASTER, sb.STATE_M, sb.STATE_V):
                    a = fz.opt.state(k, kind).double()
                    r = ref.state(b.index, kind)[lo:lo + b.own_size].double()
                    den = r.abs().clamp_min(1e-30)
                    worst = max(worst, float(((a - r).abs() / den).max()))
            out["state_max_rel"] = worst
        q.put((rank, out))
    finally:
        if ref is not None:
            ref.close()
        if fz is not None:
            fz.close()
        dist.destroy_process_group()


def test_config4_full_size_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_full_c4_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    deadline = time.time() + 400
    while len(res) < world and time.time() < deadline:
        try:
            r, out = q.get(timeout=2)
            res[r] = out
        except queue.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    for p in procs:
        if p.is_alive() and len(res) < world:
            p.terminate()
        p.join(timeout=60)
    assert len(res) == world, "a rank failed"
    r0 = res[0]
    print("CONFIG4_FULL_DP2", r0)
    assert r0["err"] == 0 and res[1]["err"] == 0
    assert r0["info"] == res[1]["info"] == r0["ref_info"] == (2, 1, 32768.0)
    assert r0["ranks_equal"]
    assert r0["max_ulp"] <= 1
    assert r0["state_max_rel"] <= 1e-6
