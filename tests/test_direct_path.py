"""The register-fed update (k_apply_direct, short tensor lists) and gradient
sets, through the C-ABI, against the port oracle.

Bar as in tests/test_gpu_parity.py: skip decisions, loss-scale sequence and
step counts bit-exact; fp32 state within max relative error 1e-6 (bit-exact
where no clip coefficient depends on the summation order); bf16 params within
1 bf16 ulp."""
import numpy as np
import pytest

import cases
from gpu_helpers import GpuRun, to_device
from test_gpu_parity import compare, run_both

import soar_b200 as sb

pytestmark = pytest.mark.gpu

DIRECT_CASES = [
    # mixed layout: clip, scaler with skips (every 5th step), backoff and growth
    # (interval 4), wd mask, a 5-element tensor (one partial vector), odd sizes
    cases.Case("direct_mixed", 1, [4097, 1_000_003, 5], [0.01, 0.0, 0.05], 14, max_norm=1.0,
               use_scaler=True, init_scale=1024.0, growth_interval=4, grad_std=1e-1,
               inf_every=5, seed=21),
    # fp32, four runs plus a tensor without a gradient, clip
    cases.Case("direct_fp32_runs", 0, [4099, 17, 1024, 333, 70001], [0.01, 0.0, 0.05, 0.0, 0.01],
               4, max_norm=0.5, null_grad=[1], seed=22),
    # more vectors than one pass of the grid holds (the kernel loops)
    cases.Case("direct_fp32_passes", 0, [3_000_001], [0.01], 3, seed=23),
    cases.Case("direct_mixed_passes", 1, [3_500_002], [0.01], 3, max_norm=1.0, use_scaler=True,
               grad_std=1e-3, seed=24),
]


@pytest.mark.parametrize("case", DIRECT_CASES, ids=lambda c: c.name)
def test_direct_path_matches_oracle(oracle_mod, cuda, case):
    run, port, hist = run_both(oracle_mod, cuda, case)
    assert run.opt.kernel_path == "direct"
    compare(oracle_mod, run, port, exact=case.max_norm == 0.0)
    if case.inf_every:
        assert sum(h[0] for h in hist) >= 2  # the skip branch ran


@pytest.mark.parametrize("offsets", [[1, 3, 6], [(1, 2), (3, 3), (2, 0)]],
                         ids=["same-phase", "mixed-phase"])
def test_direct_path_misaligned(oracle_mod, cuda, offsets):
    """Scalar heads of misaligned tensors and mixed-phase tensors (scalar chunks
    beside the direct kernel's runs)."""
    case = cases.Case("direct_off", 1, [70001, 33, 4101], [0.01, 0.0, 0.05], 6, max_norm=1.0,
                      use_scaler=True, init_scale=1024.0, grad_std=1e-1, inf_every=4, seed=25)
    run, port, _ = run_both(oracle_mod, cuda, case, offsets=offsets)
    assert run.opt.kernel_path == "direct"
    compare(oracle_mod, run, port, exact=False)


def test_large_and_long_lists_use_the_pipeline(cuda):
    torch = cuda
    big = [torch.zeros(20_000_000, device="cuda")]
    opt = sb.AdamW(big, grads=[torch.zeros_like(big[0])])
    assert opt.kernel_path == "pipeline"
    many = [torch.zeros(100, device="cuda") for _ in range(5)]
    opt2 = sb.AdamW(many, grads=[torch.zeros_like(p) for p in many])
    assert opt2.kernel_path == "pipeline"
    small = [torch.zeros(100, device="cuda")]
    opt3 = sb.AdamW(small, grads=[torch.zeros_like(small[0])])
    assert opt3.kernel_path == "direct"
    opt3.enable_ema(0.9)  # the weight EMA runs in the pipeline kernel
    assert opt3.kernel_path == "pipeline"


@pytest.mark.parametrize("case", [DIRECT_CASES[0], cases.mixed_small(steps=10),
                                  cases.fp32_edge()], ids=lambda c: c.name)
def test_gradient_sets_alternate(oracle_mod, cuda, case):
    """Two gradient sets used alternately (odd steps set 0, even steps set 1):
    every step reads the set in use, zero_grad clears only that set, and the
    result is the oracle's on the same gradient sequence."""
    torch = cuda
    from test_oracle import run_port
    port, hist = run_port(oracle_mod, case, case.steps)
    run = GpuRun(torch, case)
    other = [None if g is None else torch.zeros_like(g) for g in run.grads]
    k = run.opt.add_grads(other)
    assert k == 1
    sets = [run.grads, other]
    scale = case.init_scale
    seen = []
    for t in range(1, case.steps + 1):
        which = (t + 1) % 2
        for g_dev, g in zip(sets[which], case.grads(t, scale)):
            if g_dev is not None and g is not None and g.size:
                g_dev.copy_(to_device(torch, g, case.layout))
        run.opt.use_grads(which)
        run.opt.step()
        info = run.opt.info()
        seen.append((info.step, info.skipped, info.loss_scale))
        scale = info.loss_scale
    assert [s[0] for s in seen] == [h[2] for h in hist], "step counts"
    if case.use_scaler:
        assert [s[2] for s in seen] == [h[1] for h in hist], "loss-scale sequence"
    compare(oracle_mod, run, port, exact=False)
    # zero_grad clears the set in use only
    run.opt.use_grads(1)
    run.opt.zero_grad()
    torch.cuda.synchronize()
    assert all(float(g.abs().max()) == 0.0 for g in other if g is not None and g.numel())
    assert any(float(g.float().abs().max()) > 0.0 for g in run.grads if g is not None and g.numel())


def test_gradient_set_checks(cuda):
    torch = cuda
    p = [torch.zeros(1000, device="cuda"), torch.zeros(10, device="cuda")]
    g = [torch.zeros_like(x) for x in p]
    opt = sb.AdamW(p, grads=g)
    buf = torch.zeros(2000, device="cuda")
    with pytest.raises(sb.SoarError, match="alignment"):
        opt.add_grads([buf[1:1001], torch.zeros(10, device="cuda")])
    with pytest.raises(sb.SoarError, match="presence"):
        opt.add_grads([torch.zeros(1000, device="cuda"), None])
    with pytest.raises(sb.SoarError, match="bad gradient set"):
        opt.use_grads(3)
    assert opt.add_grads([torch.zeros(1000, device="cuda"), torch.zeros(10, device="cuda")]) == 1
