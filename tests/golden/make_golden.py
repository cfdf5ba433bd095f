"""Generates tests/golden/*.npz: seeded inputs and the outputs of the
reference's own, unmodified AdamW (src/optim/adamw.cpp compiled by
oracle/Makefile into oracle/_ref) for small cases of every part of the
optimizer-step path. Each fixture stores its inputs, so the golden check does
not depend on the input generator.

  python tests/golden/make_golden.py      (needs the reference sources to build oracle/_ref)

Cases:
  kat_adamw   the reference's own known answer, tests/test_optimizers.cpp:12-49
  kat_clip    tests/test_optimizers.cpp:97-119
  c1          config 1 shape, 1027 params, 10 steps, fresh grads each step
  c2          first 6 tensors of the config-2 list, wd 0.05 on conv weights only,
              cosine 1e-3 -> 1e-5 over 100 steps (5 steps taken)
  mixed       bf16 params/grads, fp32 master, loss scaler (init 1024, growth
              interval 4), +inf injected at step 5, clip 1.0, per-tensor wd
  cosine      learning-rate sequences of CosineAnnealingLR
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "soar.cpp_b200"))
sys.path.insert(0, str(ROOT))

from oracle import oracle  # noqa: E402
from soar_b200 import synth  # noqa: E402


def kat_adamw():
    p = np.array([1.0], np.float32)
    g = np.array([0.5], np.float32)
    r = oracle.RefAdamW([p], [g], lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=1e-2)
    r.step()
    return dict(p0=np.array([1.0], np.float32), g=g, lr=np.float32(1e-3), wd=np.float32(1e-2),
                p1=p, m1=r.moment(0, 0), v1=r.moment(0, 1))


def kat_clip():
    p = np.array([3.0, 4.0], np.float32)
    g = np.array([3.0, 4.0], np.float32)
    r = oracle.RefAdamW([p], [g])
    norm = r.clip_grad_norm(2.5)
    return dict(g0=np.array([3.0, 4.0], np.float32), max_norm=np.float32(2.5),
                norm=np.float32(norm), g1=g)


def fp32_case(sizes, wd, steps, seed, grad_std, cosine=None):
    params = [synth.normal(synth.seed_of(seed, i, 0), n, 0.02) for i, n in enumerate(sizes)]
    p0 = [p.copy() for p in params]
    grads = [np.zeros(n, np.float32) for n in sizes]
    groups = {}
    for i, w in enumerate(wd):
        groups.setdefault(float(np.float32(w)), []).append(i)
    opts = {w: oracle.RefAdamW([params[i] for i in idx], [grads[i] for i in idx], lr=1e-3,
                               weight_decay=w) for w, idx in groups.items()}
    scheds = [oracle.RefCosine(o, *cosine) for o in opts.values()] if cosine else []
    g_hist = []
    for t in range(1, steps + 1):
        for i, n in enumerate(sizes):
            grads[i][:] = synth.normal(synth.seed_of(seed, i, t), n, grad_std)
        g_hist.append(np.concatenate(grads))
        for o in opts.values():
            o.step()
        for s in scheds:
            s.step()
    m = np.concatenate([opts[float(np.float32(wd[i]))].moment(groups[float(np.float32(wd[i]))].index(i), 0)
                        for i in range(len(sizes))])
    v = np.concatenate([opts[float(np.float32(wd[i]))].moment(groups[float(np.float32(wd[i]))].index(i), 1)
                        for i in range(len(sizes))])
    return dict(sizes=np.array(sizes, np.int64), wd=np.array(wd, np.float32),
                p0=np.concatenate(p0), grads=np.stack(g_hist), p1=np.concatenate(params), m1=m,
                v1=v, cosine=np.array(cosine if cosine else (0, 0, 0), np.float64))


def mixed_case():
    sizes = [1, 3, 7, 8, 1000, 4097]
    wd = [0.01, 0.0, 0.05, 0.0, 0.01, 0.0]
    steps, inf_step = 12, 5
    cfg = oracle.StepConfig(layout=1, max_norm=1.0, use_scaler=True, growth_interval=4)
    p0 = [synth.to_bf16_bits(synth.normal(synth.seed_of(60, i, 0), n, 0.02))
          for i, n in enumerate(sizes)]
    ref = oracle.RefComposite([p.copy() for p in p0], wd, cfg, init_scale=1024.0)
    g_hist, hist = [], []
    for t in range(1, steps + 1):
        gs = []
        for i, n in enumerate(sizes):
            g = synth.normal(synth.seed_of(60, i, t), n, 0.1) * np.float32(ref.state.scale)
            if t == inf_step and i == 4:
                g[3] = np.inf
            gs.append(synth.to_bf16_bits(g.astype(np.float32)))
        g_hist.append(np.concatenate(gs))
        skipped = ref.step(gs)
        hist.append((skipped, ref.state.scale, ref.state.t))
    return dict(sizes=np.array(sizes, np.int64), wd=np.array(wd, np.float32),
                p0=np.concatenate(p0), grads=np.stack(g_hist),
                p1=np.concatenate(ref.params), master1=np.concatenate(ref.master),
                m1=np.concatenate([ref.moment(i, 0) for i in range(len(sizes))]),
                v1=np.concatenate([ref.moment(i, 1) for i in range(len(sizes))]),
                hist=np.array(hist, np.float64))


def cosine_case():
    out = {}
    for k, (total, eta, warm, base) in enumerate([(100, 1e-5, 0, 1e-3), (50, 1e-6, 5, 3e-4)]):
        p = np.zeros(1, np.float32)
        r = oracle.RefAdamW([p], [p.copy()], lr=base)
        s = oracle.RefCosine(r, total, eta, warm)
        lrs = []
        for _ in range(total + 5):
            s.step()
            lrs.append(r.get_lr())
        out[f"lrs{k}"] = np.array(lrs, np.float32)
        out[f"cfg{k}"] = np.array([total, eta, warm, base], np.float64)
    return out


def main():
    oracle.build(ref=True)
    if not oracle.ref_available():
        sys.exit("oracle/_ref not built: the reference sources are needed")
    cases = {
        "kat_adamw": kat_adamw(),
        "kat_clip": kat_clip(),
        "c1": fp32_case([1027], [0.01], 10, 61, 1e-2),
        "c2": fp32_case([int(np.prod(s)) for _, s in synth.config2_shapes()[:6]],
                        [0.05 if k in ("dw", "pw") else 0.0 for k, _ in synth.config2_shapes()[:6]],
                        5, 62, 1e-3, cosine=(100, 1e-5, 0)),
        "mixed": mixed_case(),
        "cosine": cosine_case(),
    }
    for name, d in cases.items():
        np.savez_compressed(HERE / f"{name}.npz", **d)
        print(name, (HERE / f"{name}.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
