"""Pins the CPU oracles: the C restatement (port) against the reference's own
compiled AdamW (oracle/_ref) and against the reference's known answers
(tests/test_optimizers.cpp:12-49, :97-119). CPU only."""
import ctypes
import math

import numpy as np
import pytest

import cases
from soar_b200 import synth


def run_port(oracle, case, steps=None):
    cfg = oracle.StepConfig(layout=case.layout, lr=case.lr, beta1=case.beta1, beta2=case.beta2,
                            eps=case.eps, max_norm=case.max_norm, use_scaler=case.use_scaler,
                            growth_interval=case.growth_interval)
    opt = oracle.PortOptimizer(case.params0(), case.wd, cfg, init_scale=case.init_scale)
    hist = []
    lr = case.lr
    for t in range(1, (steps or case.steps) + 1):
        skipped = opt.step(case.grads(t, opt.state.scale), lr)
        hist.append((skipped, opt.state.scale, opt.state.t, opt.state.last_norm))
        if case.cosine:
            lr = oracle.cosine_lr(case.lr, case.cosine[1], case.cosine[0], case.cosine[2], t)
    return opt, hist


def run_ref(oracle, case, steps=None):
    cfg = oracle.StepConfig(layout=case.layout, lr=case.lr, beta1=case.beta1, beta2=case.beta2,
                            eps=case.eps, max_norm=case.max_norm, use_scaler=case.use_scaler,
                            growth_interval=case.growth_interval)
    opt = oracle.RefComposite(case.params0(), case.wd, cfg, init_scale=case.init_scale,
                              null_grad=case.null_grad)
    sched = None
    if case.cosine:
        # drive the reference scheduler on the instances that step
        scheds = [oracle.RefCosine(o, case.cosine[0], case.cosine[1], case.cosine[2])
                  for o in opt.opts.values()]
    hist = []
    for t in range(1, (steps or case.steps) + 1):
        lr = next(iter(opt.opts.values())).get_lr()
        skipped = opt.step(case.grads(t, opt.state.scale), lr)
        hist.append((skipped, opt.state.scale, opt.state.t, opt.state.last_norm))
        if case.cosine:
            for s in scheds:
                s.step()
    return opt, hist


# ------------------------------------------------------- reference KATs ------

def test_kat_adamw_parity_port(oracle_mod):
    """tests/test_optimizers.cpp:12-49: p=1, g=0.5, one step -> 0.99899 (1e-6)."""
    o = oracle_mod
    cfg = o.StepConfig(layout=0, lr=1e-3)
    opt = o.PortOptimizer([np.array([1.0], np.float32)], [1e-2], cfg)
    opt.step([np.array([0.5], np.float32)])
    assert abs(opt.params[0][0] - np.float32(0.99899)) < 1e-6


def test_kat_adamw_parity_ref(ref_oracle):
    o = ref_oracle
    p = np.array([1.0], np.float32)
    g = np.array([0.5], np.float32)
    opt = o.RefAdamW([p], [g], lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=1e-2)
    opt.step()
    assert abs(p[0] - np.float32(0.99899)) < 1e-6
    # the port gives the same bits
    q = np.array([1.0], np.float32)
    opt2 = o.PortOptimizer([q], [1e-2], o.StepConfig(layout=0, lr=1e-3))
    opt2.step([g])
    assert q.view(np.uint32)[0] == p.view(np.uint32)[0]


def test_kat_gradient_clipping(ref_oracle):
    """tests/test_optimizers.cpp:97-119: grads (3,4), max 2.5 -> norm 5, clipped norm 2.5."""
    o = ref_oracle
    p = np.array([3.0, 4.0], np.float32)
    g = np.array([3.0, 4.0], np.float32)
    opt = o.RefAdamW([p], [g])
    norm = opt.clip_grad_norm(2.5)
    assert abs(norm - 5.0) < 1e-5
    assert abs(math.sqrt(float(g[0]) ** 2 + float(g[1]) ** 2) - 2.5) < 1e-5
    # port: same norm and same coefficient bits
    pn = o.port()
    s = pn.oracle_sumsq_f32(np.array([3.0, 4.0], np.float32), 2, 0.0)
    n2 = pn.oracle_norm_from_sumsq(s)
    assert np.float32(n2) == np.float32(norm)
    flag = ctypes.c_int()
    coef = pn.oracle_clip_coef(n2, 2.5, ctypes.byref(flag))
    assert flag.value == 1
    g2 = np.array([3.0, 4.0], np.float32)
    pn.oracle_scale_f32(g2, 2, coef)
    np.testing.assert_array_equal(g2.view(np.uint32), g.view(np.uint32))


# --------------------------------------------------- port vs reference -------

def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == np.float32 else np.uint16)


@pytest.mark.parametrize("case", [cases.c1_small(), cases.c2(limit=25, steps=6),
                                  cases.fp32_edge(), cases.mixed_small()],
                         ids=lambda c: c.name)
def test_port_matches_reference_bitexact(ref_oracle, case):
    o = ref_oracle
    po, ph = run_port(o, case)
    ro, rh = run_ref(o, case)
    assert [h[0] for h in ph] == [h[0] for h in rh], "skip decisions differ"
    assert [h[1] for h in ph] == [h[1] for h in rh], "loss-scale sequences differ"
    assert [h[2] for h in ph] == [h[2] for h in rh], "step counts differ"
    for i in range(len(case.sizes)):
        np.testing.assert_array_equal(_bits(po.params[i]), _bits(ro.params[i]), f"param {i}")
        if case.layout == 1:
            np.testing.assert_array_equal(_bits(po.master[i]), _bits(ro.master[i]), f"master {i}")
        if i in case.null_grad:
            continue
        np.testing.assert_array_equal(_bits(po.m[i]), _bits(ro.moment(i, 0)), f"m {i}")
        np.testing.assert_array_equal(_bits(po.v[i]), _bits(ro.moment(i, 1)), f"v {i}")


def test_cosine_port_matches_reference(ref_oracle):
    o = ref_oracle
    for total, eta, warm, base in [(100, 1e-5, 0, 1e-3), (50, 1e-6, 5, 3e-4), (10, 0.0, 3, 1.0)]:
        p = np.zeros(1, np.float32)
        r = o.RefAdamW([p], [p.copy()], lr=base)
        s = o.RefCosine(r, total, eta, warm)
        for step in range(1, total + 8):
            s.step()
            want = r.get_lr()
            got = o.cosine_lr(base, eta, total, warm, step)
            assert np.float32(got) == np.float32(want), (total, step)


def test_null_grad_param_untouched(ref_oracle):
    """A param without grad is skipped by step() and clip_grad_norm()."""
    o = ref_oracle
    p0 = np.ones(5, np.float32)
    p1 = np.ones(5, np.float32)
    g1 = np.full(5, 0.25, np.float32)
    r = o.RefAdamW([p0, p1], [None, g1])
    r.clip_grad_norm(0.1)
    r.step()
    np.testing.assert_array_equal(p0, np.ones(5, np.float32))
    assert not np.array_equal(p1, np.ones(5, np.float32))


# -------------------------------------------------------- restated parts -----

def test_bf16_rne_matches_torch(oracle_mod):
    import torch
    x = np.concatenate([synth.normal(7, 100000, 3.0),
                        np.array([0.0, -0.0, 1e-40, -1e-40, 3.4e38, -3.4e38, np.inf, -np.inf,
                                  1.00390625, 1.01171875, 65504.0, 1e-45], np.float32)])
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    got = oracle_mod.f32_to_bf16(x)
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(synth.to_bf16_bits(x), want)
    # NaN -> canonical 0x7FFF
    assert oracle_mod.f32_to_bf16(np.array([np.nan], np.float32))[0] == 0x7FFF
    back = oracle_mod.bf16_to_f32(got)
    np.testing.assert_array_equal(back, synth.from_bf16_bits(got))


def test_scaler_sequence_config3(oracle_mod):
    """Config 3's schedule: inf every 97th step halves the scale; growth after
    200 clean steps is never reached with period 97; with the injection stopped
    (sub-config 3b) the scale doubles every 200 clean steps."""
    o = oracle_mod
    st = o.StepState(scale=65536.0)
    seq = []
    for t in range(1, 1001):
        found = t % 97 == 0
        o.port().oracle_scaler_update(ctypes.byref(st), int(found), 2.0, 0.5, 200)
        seq.append(st.scale)
    assert seq[95] == 65536.0 and seq[96] == 32768.0 and seq[193] == 16384.0
    assert max(seq) == 65536.0
    st = o.StepState(scale=65536.0)
    seq = []
    for t in range(1, 1001):
        found = t % 97 == 0 and t <= 300
        o.port().oracle_scaler_update(ctypes.byref(st), int(found), 2.0, 0.5, 200)
        seq.append(st.scale)
    # halvings at 97, 194, 291 -> 8192; growth 200 clean steps after 291 -> step 491
    assert seq[290] == 8192.0 and seq[489] == 8192.0 and seq[490] == 16384.0
    assert seq[690] == 32768.0 and seq[890] == 65536.0


def test_mixed_skip_leaves_state(oracle_mod):
    """A skipped step leaves params, master, m, v and t unchanged."""
    o = oracle_mod
    case = cases.mixed_small(steps=4)
    opt, hist = run_port(o, case)
    before = ([p.copy() for p in opt.params], [m.copy() for m in opt.master],
              [m.copy() for m in opt.m], [v.copy() for v in opt.v], opt.state.t)
    skipped = opt.step(case.grads(5, opt.state.scale))  # step 5 injects +inf
    assert skipped == 1
    for a, b in zip(before[0], opt.params):
        np.testing.assert_array_equal(a, b)
    for a, b in zip(before[1], opt.master):
        np.testing.assert_array_equal(a, b)
    for a, b in zip(before[2], opt.m):
        np.testing.assert_array_equal(a, b)
    for a, b in zip(before[3], opt.v):
        np.testing.assert_array_equal(a, b)
    assert opt.state.t == before[4]


def test_reduce_avg_bf16(oracle_mod):
    ins = [synth.to_bf16_bits(synth.normal(100 + r, 1000, 1.0)) for r in range(4)]
    out = oracle_mod.reduce_avg_bf16(ins)
    f = sum(synth.from_bf16_bits(x).astype(np.float32) for x in ins)
    want = synth.to_bf16_bits((f * np.float32(0.25)).astype(np.float32))
    np.testing.assert_array_equal(out, want)


def test_kat_model_ema_ref(ref_oracle):
    """tests/test_metrics_preprocess.cpp:103-123: decay 0.9, a weight moved by
    +10 -> shadow 0.9*orig + 0.1*(orig+10) within 1e-4; apply_to copies it."""
    o = ref_oracle
    p = synth.normal(synth.seed_of(70), 16, 0.02)
    orig = float(p[0])
    e = o.RefEma([p], 0.9)
    p[0] = np.float32(orig + 10.0)
    e.update()
    expected = 0.9 * orig + 0.1 * (orig + 10.0)
    assert abs(e.shadow(0)[0] - expected) < 1e-4
    e.apply_to()
    assert abs(p[0] - expected) < 1e-4


def test_ema_port_matches_reference_bitexact(ref_oracle):
    o = ref_oracle
    ws = [synth.normal(synth.seed_of(71, i), n, 1.0) for i, n in enumerate([7, 1000, 4097])]
    e = o.RefEma(ws, 0.999)
    shadow = [w.copy() for w in ws]
    for step in range(5):
        for i, w in enumerate(ws):
            w += synth.normal(synth.seed_of(72, i, step), w.size, 0.1)
        e.update()
        for sh, w in zip(shadow, ws):
            o.port().oracle_ema_update(sh, w, w.size, 0.999)
    for i, sh in enumerate(shadow):
        np.testing.assert_array_equal(sh.view(np.uint32), e.shadow(i).view(np.uint32))


def test_kat_sgd_parity_ref(ref_oracle):
    """tests/test_optimizers.cpp:51-95: p=2, lr 0.1, momentum 0.9, wd 0.01;
    g=0.4 -> 1.958, then g=0.2 -> 1.898242 (1e-6)."""
    o = ref_oracle
    p = np.array([2.0], np.float32)
    g = np.array([0.4], np.float32)
    r = o.RefSGD([p], [g], lr=0.1, momentum=0.9, weight_decay=0.01)
    r.step()
    assert abs(p[0] - np.float32(1.958)) < 1e-6
    g[0] = 0.2
    r.step()
    assert abs(p[0] - np.float32(1.898242)) < 1e-6


@pytest.mark.parametrize("momentum,dampening,nesterov,wd", [
    (0.0, 0.0, False, 0.0), (0.9, 0.0, False, 0.01), (0.9, 0.1, False, 0.0),
    (0.9, 0.0, True, 0.05), (0.5, 0.25, True, 0.0)])
def test_sgd_port_matches_reference_bitexact(ref_oracle, momentum, dampening, nesterov, wd):
    o = ref_oracle
    sizes = [1, 7, 1000, 4099]
    p_ref = [synth.normal(synth.seed_of(80, i), n, 0.5) for i, n in enumerate(sizes)]
    g_ref = [np.zeros(n, np.float32) for n in sizes]
    r = o.RefSGD(p_ref, g_ref, lr=0.05, momentum=momentum, dampening=dampening,
                 weight_decay=wd, nesterov=nesterov)
    port = o.PortSGD([p.copy() for p in p_ref], [wd] * len(sizes),
                     o.StepConfig(layout=0, lr=0.05), momentum, dampening, nesterov)
    for t in range(1, 5):
        gs = [synth.normal(synth.seed_of(81, i, t), n, 0.1) for i, n in enumerate(sizes)]
        for dst, src in zip(g_ref, gs):
            dst[:] = src
        r.step()
        port.step(gs)
    for a, b in zip(port.params, p_ref):
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))


def test_port_matches_reference_on_random_hyperparameters(ref_oracle):
    """Property check of the pin: for seeded random hyperparameters (lr, betas,
    eps, per-tensor wd incl. 0, clip on or off), tensor sizes and layouts,
    the port and the reference's own compiled code agree bit for bit."""
    import dataclasses
    rng = np.random.default_rng(2024)
    for k in range(24):
        n_t = int(rng.integers(1, 5))
        sizes = [int(x) for x in rng.integers(1, 5000, size=n_t)]
        case = cases.Case(
            f"rand{k}", int(rng.integers(0, 2)), sizes,
            [float(rng.choice([0.0, 0.01, 0.1, 0.5])) for _ in sizes], int(rng.integers(1, 6)),
            lr=float(10 ** rng.uniform(-5, -1)), beta1=float(rng.choice([0.0, 0.5, 0.9, 0.99])),
            beta2=float(rng.choice([0.9, 0.99, 0.999, 0.9999])),
            eps=float(10 ** rng.uniform(-10, -4)),
            max_norm=float(rng.choice([0.0, 0.05, 1.0, 100.0])),
            grad_std=float(10 ** rng.uniform(-4, 0)), seed=1000 + k)
        if case.layout == 1:
            case = dataclasses.replace(case, use_scaler=bool(rng.integers(0, 2)),
                                       init_scale=float(2.0 ** rng.integers(0, 17)),
                                       inf_every=int(rng.choice([0, 2, 3])), growth_interval=2)
        o = ref_oracle
        po, ph = run_port(o, case)
        ro, rh = run_ref(o, case)
        assert [h[:3] for h in ph] == [h[:3] for h in rh], case
        for i in range(len(case.sizes)):
            np.testing.assert_array_equal(_bits(po.params[i]), _bits(ro.params[i]), str(case))
            np.testing.assert_array_equal(_bits(po.m[i]), _bits(ro.moment(i, 0)), str(case))
            np.testing.assert_array_equal(_bits(po.v[i]), _bits(ro.moment(i, 1)), str(case))
