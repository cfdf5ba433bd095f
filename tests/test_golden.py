"""Golden vectors from the reference's own AdamW (tests/golden/make_golden.py):
the port oracle must reproduce them bit-for-bit on the CPU, and the device
through the C-ABI on the GPU (bit-exact in fp32; the mixed case within the
parity tolerances: bf16 params 1 ulp, fp32 state 1e-6 relative, skip/scale
sequence exact). The fixtures carry their inputs, so neither check depends on
the input generator or on the reference tree being present."""
import ctypes
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def split(flat, sizes):
    out, o = [], 0
    for n in sizes:
        out.append(flat[o:o + n])
        o += n
    return out


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == np.float32 else np.uint16)


# ------------------------------------------------------------------ port -----

def test_golden_kats_port(oracle_mod):
    o = oracle_mod
    d = load("kat_adamw")
    opt = o.PortOptimizer([d["p0"].copy()], [float(d["wd"])], o.StepConfig(layout=0, lr=float(d["lr"])))
    opt.step([d["g"]])
    assert bits(opt.params[0])[0] == bits(d["p1"])[0]
    assert bits(opt.m[0])[0] == bits(d["m1"])[0] and bits(opt.v[0])[0] == bits(d["v1"])[0]
    c = load("kat_clip")
    pn = o.port()
    norm = pn.oracle_norm_from_sumsq(pn.oracle_sumsq_f32(c["g0"], 2, 0.0))
    assert np.float32(norm) == c["norm"]
    flag = ctypes.c_int()
    coef = pn.oracle_clip_coef(norm, float(c["max_norm"]), ctypes.byref(flag))
    g = c["g0"].copy()
    pn.oracle_scale_f32(g, 2, coef)
    np.testing.assert_array_equal(bits(g), bits(c["g1"]))


def _run_port_fp32(o, d):
    sizes = [int(x) for x in d["sizes"]]
    total, eta, warm = d["cosine"]
    opt = o.PortOptimizer(split(d["p0"].copy(), sizes), d["wd"], o.StepConfig(layout=0))
    lr = 1e-3
    for t, g in enumerate(d["grads"], start=1):
        opt.step(split(g, sizes), lr)
        if total:
            lr = o.cosine_lr(1e-3, float(eta), int(total), int(warm), t)
    return opt, sizes


@pytest.mark.parametrize("name", ["c1", "c2"])
def test_golden_fp32_port(oracle_mod, name):
    d = load(name)
    opt, sizes = _run_port_fp32(oracle_mod, d)
    np.testing.assert_array_equal(bits(np.concatenate(opt.params)), bits(d["p1"]))
    np.testing.assert_array_equal(bits(np.concatenate(opt.m)), bits(d["m1"]))
    np.testing.assert_array_equal(bits(np.concatenate(opt.v)), bits(d["v1"]))


def test_golden_mixed_port(oracle_mod):
    o = oracle_mod
    d = load("mixed")
    sizes = [int(x) for x in d["sizes"]]
    cfg = o.StepConfig(layout=1, max_norm=1.0, use_scaler=True, growth_interval=4)
    opt = o.PortOptimizer(split(d["p0"].copy(), sizes), d["wd"], cfg, init_scale=1024.0)
    hist = []
    for g in d["grads"]:
        s = opt.step(split(g, sizes))
        hist.append((s, opt.state.scale, opt.state.t))
    np.testing.assert_array_equal(np.array(hist, np.float64), d["hist"])
    np.testing.assert_array_equal(bits(np.concatenate(opt.params)), bits(d["p1"]))
    np.testing.assert_array_equal(bits(np.concatenate(opt.master)), bits(d["master1"]))
    np.testing.assert_array_equal(bits(np.concatenate(opt.m)), bits(d["m1"]))
    np.testing.assert_array_equal(bits(np.concatenate(opt.v)), bits(d["v1"]))


def test_golden_cosine_port(oracle_mod):
    d = load("cosine")
    for k in (0, 1):
        total, eta, warm, base = d[f"cfg{k}"]
        got = [oracle_mod.cosine_lr(float(base), float(eta), int(total), int(warm), t)
               for t in range(1, len(d[f"lrs{k}"]) + 1)]
        np.testing.assert_array_equal(np.array(got, np.float32), d[f"lrs{k}"])


# ------------------------------------------------------------------ device ---

def _device_run(torch, d, layout, cfg_kwargs, init_scale=None):
    import soar_b200 as sb
    sizes = [int(x) for x in d["sizes"]]
    if layout == 1:
        to_dev = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(
            torch.bfloat16).cuda()
    else:
        to_dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    params = [to_dev(p) for p in split(d["p0"], sizes)]
    grads = [torch.empty_like(p) for p in params]
    scaler = sb.LossScalerOptions(init_scale=init_scale, growth_interval=4) if init_scale else None
    opt = sb.AdamW([sb.ParamGroup([p], float(w)) for p, w in zip(params, d["wd"])],
                   layout="bf16_mixed" if layout else "fp32", grads=grads, loss_scaler=scaler,
                   **cfg_kwargs)
    cos = d.get("cosine")
    sched = sb.CosineAnnealingLR(opt, int(cos[0]), float(cos[1]), int(cos[2])) \
        if cos is not None and cos[0] else None
    hist = []
    for g in d["grads"]:
        for gd, gh in zip(grads, split(g, sizes)):
            gd.copy_(to_dev(gh))
        opt.step()
        info = opt.info()
        hist.append((info.found_inf and init_scale is not None, info.loss_scale, info.step))
        if sched:
            sched.step()
    return opt, params, sizes


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["c1", "c2"])
def test_golden_fp32_device(cuda, name):
    import soar_b200 as sb
    d = load(name)
    opt, params, sizes = _device_run(cuda, d, 0, {})
    got = np.concatenate([p.cpu().numpy() for p in params])
    np.testing.assert_array_equal(bits(got), bits(d["p1"]))
    m = np.concatenate([opt.read_state(i, sb.STATE_M) for i in range(len(sizes))])
    v = np.concatenate([opt.read_state(i, sb.STATE_V) for i in range(len(sizes))])
    np.testing.assert_array_equal(bits(m), bits(d["m1"]))
    np.testing.assert_array_equal(bits(v), bits(d["v1"]))


@pytest.mark.gpu
def test_golden_mixed_device(cuda):
    import soar_b200 as sb
    torch = cuda
    d = load("mixed")
    opt, params, sizes = _device_run(torch, d, 1, {"max_grad_norm": 1.0}, init_scale=1024.0)
    info = opt.info()
    assert info.skipped == int(d["hist"][:, 0].sum())
    assert info.loss_scale == d["hist"][-1, 1] and info.step == int(d["hist"][-1, 2])
    got = np.concatenate([p.view(torch.int16).cpu().numpy().view(np.uint16) for p in params])
    assert np.abs(got.astype(np.int32) - d["p1"].astype(np.int32)).max() <= 1
    for kind, key in ((sb.STATE_MASTER, "master1"), (sb.STATE_M, "m1"), (sb.STATE_V, "v1")):
        st = np.concatenate([opt.read_state(i, kind) for i in range(len(sizes))]).astype(np.float64)
        ref = d[key].astype(np.float64)
        assert np.max(np.abs(st - ref) / np.maximum(np.abs(ref), 1e-30)) <= 1e-6, key
