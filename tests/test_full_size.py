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


def test_config3_full_1000_steps(oracle_mod, cuda):
    """Config 3 as BASELINE.json states it: 50M bf16-mixed params in 400
    tensors (one flat buffer, so most tensors start off the 16-byte boundary),
    clip 1.0, loss scale 65536 with growth after 200 clean steps, +inf into one
    seeded gradient element every 97th step, 1000 steps.

    Gradients: four seeded sets of N(0, 1e-3) fp32 values, cycled (fresh on
    consecutive steps), scaled by the live loss scale and rounded to bf16 on
    the device each step. The scale is a power of two, so the unscaled bf16
    gradient of a set is the same at every scale and the host knows each
    set's fp64 sum of squares exactly. Checked against the oracle:
      - the skip / loss-scale / step-count sequence of all 1000 steps, bit for
        bit (skips at 97, 194, ..., 970: ten backoffs, no growth);
      - every step's global norm, bit for bit with the host's fp64 norm;
      - the final master / m / v / bf16 params on a 65K-element sample (and
        every tensor's first and last element), replayed through the oracle
        over the same 1000 steps, bit for bit."""
    torch = cuda
    case = cases.c3(steps=1000)
    sizes = case.sizes
    n = sum(sizes)
    assert n == 50_000_000 and len(sizes) == 400
    offs = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    p0 = case.params0()
    flat_p0 = np.concatenate(p0)
    params = torch.from_numpy(flat_p0.view(np.int16)).view(torch.bfloat16).cuda()
    grads = torch.empty_like(params)
    views_p = [params[offs[i]:offs[i + 1]] for i in range(400)]
    views_g = [grads[offs[i]:offs[i + 1]] for i in range(400)]
    opt = sb.AdamW([sb.ParamGroup([p], 0.01) for p in views_p], sb.AdamWOptions(lr=1e-3),
                   layout="bf16_mixed", max_grad_norm=1.0,
                   loss_scaler=sb.LossScalerOptions(init_scale=65536.0, growth_interval=200),
                   grads=views_g)
    gen = torch.Generator(device="cuda")
    pool = []
    for k in range(4):
        gen.manual_seed(3000 + k)
        pool.append(torch.randn(n, device="cuda", generator=gen) * 1e-3)
    tmp = torch.empty(n, dtype=torch.float32, device="cuda")

    # host side: each set's unscaled bf16 values (exact at every power-of-two
    # scale) and their fp64 sum of squares, and the sample
    rng = np.random.default_rng(33)
    idx = np.unique(np.concatenate([rng.integers(0, n, 1 << 16), offs[:-1], offs[1:] - 1]))
    unscaled = []
    sumsq = []
    for k in range(4):
        u = oracle_mod.bf16_to_f32(oracle_mod.f32_to_bf16(pool[k].cpu().numpy()))
        sumsq.append(float(np.sum(u.astype(np.float64) ** 2)))
        unscaled.append(u[idx].copy())

    def inject(t):
        i = t % 400
        j = int(rng_inj.integers(0, sizes[i]))
        return int(offs[i] + j)

    rng_inj = np.random.default_rng(97)
    inf_at = {t: inject(t) for t in range(97, 1001, 97)}

    dev_hist = []
    scale = 65536.0
    for t in range(1, 1001):
        k = t % 4
        torch.mul(pool[k], scale, out=tmp)
        grads.copy_(tmp)                          # round to nearest even bf16
        if t in inf_at:
            grads[inf_at[t]] = float("inf")
        opt.step()
        info = opt.info()
        dev_hist.append((info.step, info.skipped, info.loss_scale, info.grad_norm,
                         info.found_inf))
        scale = info.loss_scale
    got_p = params.view(torch.int16)[torch.from_numpy(idx).cuda()].cpu().numpy().view(np.uint16)

    def state(kind):
        v = torch.cat([opt.state(i, kind) for i in range(400)])
        return v[torch.from_numpy(idx).cuda()].cpu().numpy()

    got = {"master": state(sb.STATE_MASTER), "m": state(sb.STATE_M), "v": state(sb.STATE_V)}
    opt.close()

    # the oracle over the same 1000 steps on the sample
    cfg = oracle_mod.StepConfig(layout=1, lr=1e-3, max_norm=1.0, use_scaler=True,
                                growth_interval=200)
    g_s = np.zeros(idx.size, np.uint16)
    ps = oracle_mod.PortShard([flat_p0[idx].copy()], [g_s], [0.01], cfg, init_scale=65536.0)
    for t in range(1, 1001):
        k = t % 4
        s = np.float32(ps.state.scale)
        g_s[:] = oracle_mod.f32_to_bf16(unscaled[k] * s)   # exact: s is a power of two
        total = float("inf") if t in inf_at else sumsq[k]
        ps.apply_sumsq(total)
        d = dev_hist[t - 1]
        assert (d[0], d[1], d[2]) == (ps.state.t, ps.state.skipped, ps.state.scale), \
            f"step {t}: device {d[:3]} vs oracle {(ps.state.t, ps.state.skipped, ps.state.scale)}"
        if t not in inf_at:
            assert np.float32(d[3]) == np.float32(ps.state.last_norm), f"norm at step {t}"
    assert ps.state.skipped == 10 and ps.state.t == 990
    assert ps.state.scale == 65536.0 / 2 ** 10
    np.testing.assert_array_equal(got_p, ps.params[0])
    for key, want in (("master", ps.master[0]), ("m", ps.m[0]), ("v", ps.v[0])):
        np.testing.assert_array_equal(got[key].view(np.uint32), want.view(np.uint32), key)
