"""Parity of the CUDA optimizer step (through the C-ABI) against the CPU oracle
on identical seeded inputs.

Bar (written here): skip decisions, loss-scale
sequence and step counts bit-exact; fp32 params / master / m / v within max
relative error 1e-6; bf16 params within 1 bf16 ulp. The kernels follow the
reference's operation order with IEEE-rounded intrinsics, so in practice the
results are bit-identical; the tests also assert that where it is guaranteed
(no clipping: nothing depends on the summation order)."""
import numpy as np
import pytest

import cases
from gpu_helpers import GpuRun, max_rel_err, to_device, to_host, ulp_diff_bf16
from test_oracle import run_port

import soar_b200 as sb

pytestmark = pytest.mark.gpu

FP32_RTOL = 1e-6
BF16_ULP = 1


def compare(oracle, run: GpuRun, port, exact: bool):
    case = run.case
    gp = run.params_host()
    for i in range(len(case.sizes)):
        if case.sizes[i] == 0:
            continue
        if case.layout == 1:
            d = ulp_diff_bf16(gp[i], port.params[i])
            assert d.max(initial=0) <= BF16_ULP, f"param {i}: {d.max()} bf16 ulp"
            if exact:
                np.testing.assert_array_equal(gp[i], port.params[i], f"param {i} bits")
            master = run.state_host(i, sb.STATE_MASTER)
            assert max_rel_err(master, port.master[i]) <= FP32_RTOL, f"master {i}"
            if exact:
                np.testing.assert_array_equal(master.view(np.uint32),
                                              port.master[i].view(np.uint32))
        else:
            assert max_rel_err(gp[i], port.params[i]) <= FP32_RTOL, f"param {i}"
            if exact:
                np.testing.assert_array_equal(gp[i].view(np.uint32),
                                              port.params[i].view(np.uint32), f"param {i} bits")
        for kind, ref in ((sb.STATE_M, port.m[i]), (sb.STATE_V, port.v[i])):
            got = run.state_host(i, kind)
            assert max_rel_err(got, ref) <= FP32_RTOL, f"state {kind} of tensor {i}"
            if exact:
                np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def run_both(oracle, torch, case, steps=None, offsets=None):
    steps = steps or case.steps
    port, hist = run_port(oracle, case, steps)
    run = GpuRun(torch, case, offsets=offsets)
    scale = case.init_scale
    for t in range(1, steps + 1):
        info = run.step(t, scale)
        scale = info.loss_scale
    # step bookkeeping: bit-exact
    assert [h[1] for h in run.hist] == list(np.cumsum([h[0] for h in hist])), "skip sequence"
    if case.use_scaler:
        assert [h[2] for h in run.hist] == [h[1] for h in hist], "loss-scale sequence"
    assert [h[0] for h in run.hist] == [h[2] for h in hist], "step counts"
    return run, port, hist


def test_kat_adamw_parity_gpu(oracle_mod, cuda):
    """tests/test_optimizers.cpp:12-49 on the device: p=1, g=0.5 -> 0.99899."""
    torch = cuda
    p = torch.ones(1, device="cuda")
    g = torch.full((1,), 0.5, device="cuda")
    opt = sb.AdamW([p], sb.AdamWOptions(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8,
                                        weight_decay=1e-2), grads=[g])
    opt.step()
    got = p.cpu().numpy()
    assert abs(got[0] - np.float32(0.99899)) < 1e-6
    q = np.array([1.0], np.float32)
    oracle_mod.PortOptimizer([q], [1e-2], oracle_mod.StepConfig(layout=0)).step(
        [np.array([0.5], np.float32)])
    port_q = oracle_mod.PortOptimizer([np.array([1.0], np.float32)], [1e-2],
                                      oracle_mod.StepConfig(layout=0))
    port_q.step([np.array([0.5], np.float32)])
    assert got.view(np.uint32)[0] == port_q.params[0].view(np.uint32)[0]


def test_kat_gradient_clipping_gpu(cuda):
    """tests/test_optimizers.cpp:97-119: norm 5 returned, grads scaled to norm 2.5."""
    torch = cuda
    p = torch.tensor([3.0, 4.0], device="cuda")
    g = torch.tensor([3.0, 4.0], device="cuda")
    opt = sb.AdamW([p], grads=[g])
    norm = opt.clip_grad_norm(2.5)
    assert abs(norm - 5.0) < 1e-5
    gg = g.cpu().numpy().astype(np.float64)
    assert abs(np.sqrt((gg ** 2).sum()) - 2.5) < 1e-5
    np.testing.assert_array_equal(g.cpu().numpy(), np.array([1.5, 2.0], np.float32))


@pytest.mark.parametrize("case", [cases.c1_small(), cases.c1_full(),
                                  cases.c2(limit=40, steps=100), cases.c2(steps=3)],
                         ids=lambda c: f"{c.name}x{c.steps}")
def test_fp32_bitexact(oracle_mod, cuda, case):
    """fp32 layout without clipping: nothing depends on reduction order, so the
    device must reproduce the oracle's bits (configs 1 and 2)."""
    run, port, _ = run_both(oracle_mod, cuda, case)
    compare(oracle_mod, run, port, exact=True)


@pytest.mark.parametrize("case", [cases.fp32_edge(), cases.mixed_small(steps=14)],
                         ids=lambda c: c.name)
def test_edge_cases(oracle_mod, cuda, case):
    """Chunk-table edges (1, 3, 4, 7, 8, 16383-16385, 65535-65537, 0 elements),
    a tensor without grad, clip, skip on inf, backoff and growth."""
    run, port, hist = run_both(oracle_mod, cuda, case)
    compare(oracle_mod, run, port, exact=False)


def test_config3_reduced(oracle_mod, cuda):
    """Config 3 at 2M params / 400 tensors for 200 steps: +inf at steps 97 and
    194 skip the step and halve the scale; clip 1.0 every step."""
    case = cases.c3(scale_total=2_000_000, steps=200)
    run, port, hist = run_both(oracle_mod, cuda, case)
    assert sum(h[0] for h in hist) == 2
    assert run.hist[-1][2] == 65536.0 / 4
    compare(oracle_mod, run, port, exact=False)


def test_config3b_growth(oracle_mod, cuda):
    """Sub-config 3b: injection stops, the scale doubles after the growth
    interval of clean steps (interval 25 here to keep it short)."""
    case = cases.c3(scale_total=300_000, steps=130, n=40, inf_until=97, growth_interval=25)
    run, port, hist = run_both(oracle_mod, cuda, case)
    scales = [h[2] for h in run.hist]
    assert min(scales) < max(scales[97:])  # grew again after the last skip
    compare(oracle_mod, run, port, exact=False)


@pytest.mark.parametrize("offsets", [[1, 2, 3, 5, 6, 7, 9],
                                     [(1, 2), (3, 1), (0, 1), (2, 2), (1, 0), (5, 3), (7, 6)]],
                         ids=["same-phase", "mixed-phase"])
def test_misaligned_tensors(oracle_mod, cuda, offsets):
    """Tensors starting off the 16-byte boundary: same-phase param/grad get a
    scalar head then vector chunks; different phases take the scalar path."""
    case = cases.mixed_small(steps=6)
    run, port, _ = run_both(oracle_mod, cuda, case, offsets=offsets)
    compare(oracle_mod, run, port, exact=False)
    case32 = cases.Case("fp32_off", 0, [5, 70000, 33, 16390, 4, 9, 100], [0.01] * 7, 4, seed=9)
    run, port, _ = run_both(oracle_mod, cuda, case32, offsets=offsets)
    compare(oracle_mod, run, port, exact=True)


def test_standalone_clip_then_step_matches_fused(oracle_mod, cuda):
    """clip_grad_norm(max) followed by step() equals the fused step with
    max_grad_norm=max, in both layouts."""
    torch = cuda
    for layout in (0, 1):
        case = cases.Case("clip", layout, [1000, 37, 4096], [0.01, 0.0, 0.05], 3, max_norm=0.05,
                          grad_std=0.01, seed=11)
        fused = GpuRun(torch, case)
        plain_case = cases.Case("clip", layout, [1000, 37, 4096], [0.01, 0.0, 0.05], 3,
                                grad_std=0.01, seed=11)
        plain = GpuRun(torch, plain_case)
        for t in range(1, 4):
            fused.step(t, 1.0)
            plain.load_grads(plain_case.grads(t, 1.0))
            norm = plain.opt.clip_grad_norm(0.05)
            plain.opt.step()
            assert norm == pytest.approx(fused.opt.info().grad_norm, rel=0, abs=0)
        for a, b in zip(fused.params_host(), plain.params_host()):
            np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("sizes", [[1000, 37, 4096], [1000, 37, 4096, 70001, 5, 16385]],
                         ids=["direct", "pipeline"])
def test_async_clip_matches_fused_and_standalone(oracle_mod, cuda, sizes):
    """clip_grad_norm_async(max) + step() equals the fused step with
    max_grad_norm=max and the synchronous clip_grad_norm(max) + step(), bit for
    bit, in both layouts and on both update kernels, with the loss scaler on
    (its skip decision then comes from the async norm pass too); the
    gradients are left untouched."""
    torch = cuda
    for layout in (0, 1):
        wd = [0.01, 0.0, 0.05, 0.01, 0.0, 0.02][:len(sizes)]
        kw = dict(grad_std=0.01, seed=12, use_scaler=layout == 1, init_scale=1024.0,
                  inf_every=3 if layout == 1 else 0)
        fused = GpuRun(torch, cases.Case("c", layout, sizes, wd, 5, max_norm=0.05, **kw))
        plain_case = cases.Case("c", layout, sizes, wd, 5, **kw)
        sync, asyn = GpuRun(torch, plain_case), GpuRun(torch, plain_case)
        assert asyn.opt.kernel_path == fused.opt.kernel_path
        scale = 1024.0
        for t in range(1, 6):
            fused.step(t, scale)
            for run in (sync, asyn):
                run.load_grads(plain_case.grads(t, scale))
            sync.opt.clip_grad_norm(0.05)
            sync.opt.step()
            before = [g.clone() for g in asyn.grads if g is not None]
            asyn.opt.clip_grad_norm_async(0.05)
            asyn.opt.step()
            after = [g for g in asyn.grads if g is not None]
            assert all(torch.equal(a, b) for a, b in zip(before, after))
            fi, si, ai = fused.opt.info(), sync.opt.info(), asyn.opt.info()
            assert (ai.step, ai.skipped, ai.loss_scale, ai.grad_norm, ai.clip_coef) == \
                (fi.step, fi.skipped, fi.loss_scale, fi.grad_norm, fi.clip_coef)
            scale = fi.loss_scale
        assert fused.opt.info().skipped >= (1 if layout == 1 else 0)
        for a, b, c in zip(fused.params_host(), asyn.params_host(), sync.params_host()):
            np.testing.assert_array_equal(a, b)
            np.testing.assert_array_equal(a, c)


def test_dp_split_api_matches_step(oracle_mod, cuda):
    """grad_sumsq + apply(1 partial) is exactly step()."""
    torch = cuda
    case = cases.mixed_small(steps=7)
    a = GpuRun(torch, case)
    b = GpuRun(torch, case)
    part = torch.zeros(1, dtype=torch.float64, device="cuda")
    scale = case.init_scale
    for t in range(1, 8):
        a.step(t, scale)
        b.load_grads(case.grads(t, scale))
        b.opt.grad_sumsq(part.data_ptr())
        b.opt.apply(part.data_ptr(), 1)
        scale = a.opt.info().loss_scale
        assert b.opt.info().loss_scale == scale
    for x, y in zip(a.params_host(), b.params_host()):
        np.testing.assert_array_equal(x, y)


def test_zero_grad_and_determinism(oracle_mod, cuda):
    torch = cuda
    case = cases.c2(limit=30, steps=2)
    r1, r2 = GpuRun(torch, case), GpuRun(torch, case)
    for t in (1, 2):
        r1.step(t, 1.0)
        r2.step(t, 1.0)
    for x, y in zip(r1.params_host(), r2.params_host()):
        np.testing.assert_array_equal(x, y)
    r1.opt.zero_grad()
    torch.cuda.synchronize()
    assert all(float(g.abs().max()) == 0.0 for g in r1.grads if g is not None and g.numel())


def test_cosine_matches_oracle(oracle_mod, cuda):
    torch = cuda
    p = torch.zeros(4, device="cuda")
    g = torch.zeros(4, device="cuda")
    for total, eta, warm, base in [(100, 1e-5, 0, 1e-3), (20, 1e-6, 5, 3e-4)]:
        opt = sb.AdamW([p], sb.AdamWOptions(lr=base), grads=[g])
        s = sb.CosineAnnealingLR(opt, total, eta, warm)
        for step in range(1, total + 5):
            s.step()
            assert np.float32(opt.get_lr()) == np.float32(
                oracle_mod.cosine_lr(base, eta, total, warm, step))


def test_errors_are_reported(cuda):
    torch = cuda
    p = torch.zeros(4, device="cuda")
    with pytest.raises(sb.SoarError):
        sb.AdamW([p], layout="bf16_mixed", grads=[torch.zeros(4, device="cuda")],
                 loss_scaler=sb.LossScalerOptions(init_scale=-1.0))


def test_async_info_matches_sync(cuda):
    """soar_optim_get_info_async: the readback enqueued on the stream (pinned
    host memory, read after an event) equals the synchronous readback, step by
    step, through skips and scale changes."""
    torch = cuda
    case = cases.mixed_small(steps=8)
    run = GpuRun(torch, case)
    scale = case.init_scale
    for t in range(1, case.steps + 1):
        run.load_grads(case.grads(t, scale))
        run.opt.step()
        info, ev = run.opt.info_async()
        ev.synchronize()
        want = run.opt.info()
        assert (info.step, info.skipped, info.loss_scale, info.found_inf, info.growth_tracker,
                info.error) == (want.step, want.skipped, want.loss_scale, want.found_inf,
                                want.growth_tracker, want.error)
        assert info.grad_norm == want.grad_norm and info.clip_coef == want.clip_coef
        scale = want.loss_scale
    run.opt.close()


def test_loaded_kernels_are_sm100a(cuda):
    """The update kernel runs as sm_100a SASS on the device (binaryVersion 100),
    and the library reports the architecture it was compiled for."""
    import ctypes
    compiled, loaded = ctypes.c_int(), ctypes.c_int()
    assert sb.lib().soar_kernel_arch(0, ctypes.byref(compiled), ctypes.byref(loaded)) == 0
    assert compiled.value == 1000
    assert loaded.value == 100
