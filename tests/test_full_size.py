"""Parity at the BASELINE configs' full sizes on one GPU.

* config 3 in full (50M mixed params in 400 tensors, clip 1.0, loss scaler)
  and config 4's single-GPU step (200M params in 8 buckets of 25M): the CUDA
  step against the port oracle element for element, with an injected +inf so
  a skip step, the scaler backoff and the clip all run at full size.
* config 5's largest size (2B params, both layouts): the oracle cannot hold
  2B elements of state on the host in a test's time, so the check uses the
  path's elementwise independence (no clip, no scaler: every element's update
  depends only on its own param, grad, m, v and the step): a seeded sample of
  2^20 elements is read back before and after two steps and replayed through
  the oracle, which must agree bit for bit.
Bars as in test_gpu_parity: skip / scale / step sequences bit-exact, fp32
state within 1e-6 relative, bf16 params within 1 ulp."""
import dataclasses

import numpy as np
import pytest

import cases
from gpu_helpers import ulp_diff_bf16
from test_gpu_parity import compare, run_both

import soar_b200 as sb

pytestmark = pytest.mark.gpu


def test_config3_full_size(oracle_mod, cuda):
    case = dataclasses.replace(cases.c3(steps=4), inf_every=3)
    assert sum(case.sizes) == 50_000_000 and len(case.sizes) == 400
    run, port, hist = run_both(oracle_mod, cuda, case)
    assert [h[0] for h in hist] == [0, 0, 1, 0]          # step 3 skipped
    compare(oracle_mod, run, port, exact=False)
    run.opt.close()


def test_config4_single_gpu_full_size(oracle_mod, cuda):
    case = cases.Case("c4", 1, [25_000_000] * 8, [0.01] * 8, 3, max_norm=1.0, use_scaler=True,
                      grad_std=1e-3, inf_every=2, inf_until=2, seed=44)
    run, port, hist = run_both(oracle_mod, cuda, case)
    assert [h[0] for h in hist] == [0, 1, 0]              # step 2 skipped, scale halved
    assert hist[-1][1] == 32768.0
    compare(oracle_mod, run, port, exact=False)
    run.opt.close()


@pytest.mark.parametrize("layout", ["bf16_mixed", "fp32"])
def test_config5_2b_sampled(oracle_mod, cuda, layout):
    torch = cuda
    n = 2_000_000_000
    mixed = layout == "bf16_mixed"
    dt = torch.bfloat16 if mixed else torch.float32
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5005)

    def fill(t, std):
        step = 1 << 28
        for a in range(0, n, step):
            b = min(n, a + step)
            t[a:b] = (torch.randn(b - a, device="cuda", generator=gen) * std).to(dt)

    p = torch.empty(n, dtype=dt, device="cuda")
    g = torch.empty(n, dtype=dt, device="cuda")
    fill(p, 0.02)
    rng = np.random.default_rng(5)
    idx_np = np.unique(rng.integers(0, n, size=1 << 20, dtype=np.int64))
    idx_np[0], idx_np[-1] = 0, n - 1                       # both ends of the buffer
    idx = torch.from_numpy(idx_np).cuda()

    def sample(t):
        s = t[idx]
        if mixed:
            return s.view(torch.int16).cpu().numpy().view(np.uint16).copy()
        return s.cpu().numpy().copy()

    p0 = sample(p)
    opt = sb.AdamW([sb.ParamGroup([p], 0.01)], sb.AdamWOptions(lr=1e-3), layout=layout,
                   grads=[g])
    gs = []
    for _ in range(2):
        fill(g, 1e-2)
        gs.append(sample(g))
        opt.step()
    torch.cuda.synchronize()
    got_p = sample(p)
    got = {k: opt.state(0, k)[idx].cpu().numpy() for k in (sb.STATE_M, sb.STATE_V)}
    if mixed:
        got[sb.STATE_MASTER] = opt.state(0, sb.STATE_MASTER)[idx].cpu().numpy()
    assert opt.info().step == 2
    opt.close()
    del p, g

    cfg = oracle_mod.StepConfig(layout=1 if mixed else 0)
    port = oracle_mod.PortOptimizer([p0], [0.01], cfg)
    for gg in gs:
        assert port.step([gg]) == 0
    if mixed:
        assert ulp_diff_bf16(got_p, port.params[0]).max() == 0
        np.testing.assert_array_equal(got[sb.STATE_MASTER].view(np.uint32),
                                      port.master[0].view(np.uint32))
    else:
        np.testing.assert_array_equal(got_p.view(np.uint32), port.params[0].view(np.uint32))
    np.testing.assert_array_equal(got[sb.STATE_M].view(np.uint32), port.m[0].view(np.uint32))
    np.testing.assert_array_equal(got[sb.STATE_V].view(np.uint32), port.v[0].view(np.uint32))
