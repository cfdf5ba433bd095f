"""The fused ZeRO-1 kernels at world sizes 3, 4 and 8 on ONE GPU.

All R ranks' flat gradient and parameter buffers live on the same device and
every "rank" has its own shard optimizer and soar_zero1 handle over them,
exactly as R processes would over peer memory. The caller-synchronised entry
points need no concurrent kernels (no kernel here waits on another), so the
ranks run one after another in stream order: every rank's reduce-scatter,
then the rank-ordered partials, then every rank's update with the all-gather.

Checks: each rank's reduced slice is bit-identical to the oracle's reduce
(fp32 sum in rank order, one multiply by 1/R rounded as a float, one bf16
rounding -- 1/3 is inexact, so R = 3 pins the rounding); all R parameter
buffers end identical; the step sequence, skip and loss scale match the
single-process oracle run on the average gradient, with params within 1 bf16
ulp. Ragged shards (N not divisible by R) and a 16-byte-misaligned bucket
size are included. One case (two ranks, 19,461 elements each) ends each
rank's vector run with a tile of fewer than 8 elements after three full ones,
so a group of updated params leaves for the peers closed by a tile that has no
vector part."""
import ctypes as C

import numpy as np
import pytest

from gpu_helpers import ulp_diff_bf16

import soar_b200 as sb
from soar_b200 import dp, synth
from soar_b200 import optim as _o

pytestmark = pytest.mark.gpu

N = 1_000_003
BUCKET = 250_001
STEPS = 4
INF_STEP = 2


def _grads(rank, step, scale, n=N):
    g = synth.normal(synth.seed_of(60, rank, step), n, 0.01) * np.float32(scale)
    if step == INF_STEP and rank == 0:
        g[77] = np.inf
    return synth.to_bf16_bits(g.astype(np.float32))


@pytest.mark.parametrize("world,n,bucket", [(3, N, BUCKET), (4, N, BUCKET), (8, N, BUCKET),
                                            (2, 2 * 19_461, 2 * 19_461)],
                         ids=["w3", "w4", "w8", "w2-short-tail"])
def test_zero1_kernels_emulated_world(oracle_mod, cuda, world, n, bucket):
    torch = cuda
    lib = _o.lib()
    bf = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()
    bits = lambda t: t.view(torch.int16).cpu().numpy().view(np.uint16).copy()
    p0 = synth.to_bf16_bits(synth.normal(synth.seed_of(61), n, 0.02))
    def aligned_empty(count):
        # a view starting on a 2048-byte boundary: where the chunk planner's
        # tile boundaries fall is then fixed by the shard offsets alone
        buf = torch.empty(count + 1024, dtype=torch.bfloat16, device="cuda")
        off = (-buf.data_ptr() % 2048) // 2
        return buf[off:off + count]
    grads = [aligned_empty(n) for _ in range(world)]
    params = [bf(p0) for _ in range(world)]
    gb = (C.c_void_p * world)(*[g.data_ptr() for g in grads])
    pb = (C.c_void_p * world)(*[p.data_ptr() for p in params])
    scaler = sb.LossScalerOptions(init_scale=1024.0, growth_interval=2)
    opts, handles, plans = [], [], []
    for r in range(world):
        plan = [b for b in dp.plan_buckets(n, bucket, world, r) if b.own_size > 0]
        opt = sb.AdamW([sb.ParamGroup([params[r][b.own_start:b.own_start + b.own_size]
                                       for b in plan], 0.01)],
                       layout="bf16_mixed", max_grad_norm=1.0, loss_scaler=scaler,
                       grads=[grads[r][b.own_start:b.own_start + b.own_size] for b in plan])
        shards = (_o.Zero1Shard * max(1, len(plan)))()
        for i, b in enumerate(plan):
            shards[i].offset, shards[i].count, shards[i].tensor = b.own_start, b.own_size, i
        h = C.c_void_p()
        _o._check(lib.soar_zero1_create(opt.handle, r, world, gb, pb, shards, len(plan),
                                        C.byref(h)), "soar_zero1_create")
        opts.append(opt)
        handles.append(h)
        plans.append(plan)
    part = torch.zeros(world, dtype=torch.float64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    full = dp.plan_buckets(n, bucket, 1, 0)
    ref = oracle_mod.PortOptimizer([p0[b.start:b.start + b.size] for b in full],
                                   [0.01] * len(full),
                                   oracle_mod.StepConfig(layout=1, max_norm=1.0, use_scaler=True,
                                                         growth_interval=2),
                                   init_scale=1024.0)
    scale = 1024.0
    try:
        for t in range(1, STEPS + 1):
            ins = [_grads(r, t, scale, n) for r in range(world)]
            for r in range(world):
                grads[r].copy_(bf(ins[r]))
            for r in range(world):   # every rank's reduce-scatter + partial
                _o._check(lib.soar_zero1_reduce_sumsq(
                    handles[r], C.c_void_p(part.data_ptr() + 8 * r), C.c_void_p(stream)),
                    "soar_zero1_reduce_sumsq")
            torch.cuda.synchronize()
            avg = oracle_mod.reduce_avg_bf16(ins)
            for r in range(world):
                got = bits(grads[r])
                for b in plans[r]:
                    np.testing.assert_array_equal(got[b.own_start:b.own_start + b.own_size],
                                                  avg[b.own_start:b.own_start + b.own_size])
            for r in range(world):   # every rank's update + all-gather
                _o._check(lib.soar_zero1_apply_allgather(
                    handles[r], C.c_void_p(part.data_ptr()), world, C.c_void_p(stream)),
                    "soar_zero1_apply_allgather")
            torch.cuda.synchronize()
            ref.step([avg[b.start:b.start + b.size] for b in full])
            infos = [o.info() for o in opts]
            assert len({(i.step, i.skipped, i.loss_scale) for i in infos}) == 1
            assert (infos[0].step, infos[0].skipped, infos[0].loss_scale) == \
                (ref.state.t, ref.state.skipped, ref.state.scale)
            scale = infos[0].loss_scale
        assert ref.state.skipped == 1
        final = [bits(p) for p in params]
        for r in range(1, world):
            np.testing.assert_array_equal(final[r], final[0])
        assert ulp_diff_bf16(final[0], np.concatenate(ref.params)).max() <= 1
        for r in range(world):
            err = C.c_int()
            _o._check(lib.soar_zero1_error(handles[r], C.byref(err)), "soar_zero1_error")
            assert err.value == 0
    finally:
        for h in handles:
            lib.soar_zero1_destroy(h)
        for o in opts:
            o.close()
