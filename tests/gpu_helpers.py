"""Drives a seeded Case through the CUDA optimizer (C-ABI via soar_b200) and
reads its results back for comparison with the port oracle."""
from __future__ import annotations

import numpy as np

import soar_b200 as sb


def to_device(torch, arr: np.ndarray, layout: int):
    if layout == 1:
        t = torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).view(torch.bfloat16)
    else:
        t = torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32))
    return t.to("cuda")


def to_host(t, layout: int) -> np.ndarray:
    if layout == 1:
        return t.view(__import__("torch").int16).cpu().numpy().view(np.uint16)
    return t.cpu().numpy()


class GpuRun:
    """One CUDA optimizer over a Case's tensors, stepped with the Case's grads."""

    def __init__(self, torch, case, offsets=None):
        self.torch = torch
        self.case = case
        lay = case.layout
        p0 = case.params0()
        if offsets:
            # place tensors at element offsets inside larger buffers (misaligned starts)
            self.pbufs, self.params, self.gbufs, self.grads = [], [], [], []
            for i, (p, off) in enumerate(zip(p0, offsets)):
                goff = off[1] if isinstance(off, tuple) else off
                poff = off[0] if isinstance(off, tuple) else off
                pb = to_device(torch, np.concatenate([np.zeros(poff, p.dtype), p]), lay)
                self.pbufs.append(pb)
                self.params.append(pb[poff:])
                gb = torch.zeros(goff + p.size, dtype=pb.dtype, device="cuda")
                self.gbufs.append(gb)
                self.grads.append(None if i in case.null_grad else gb[goff:])
        else:
            self.params = [to_device(torch, p, lay) for p in p0]
            self.grads = [None if i in case.null_grad else torch.zeros_like(p)
                          for i, p in enumerate(self.params)]
        groups = [sb.ParamGroup([p], w) for p, w in zip(self.params, case.wd)]
        scaler = sb.LossScalerOptions(init_scale=case.init_scale,
                                      growth_interval=case.growth_interval) \
            if case.use_scaler else None
        self.opt = sb.AdamW(groups, sb.AdamWOptions(lr=case.lr, beta1=case.beta1,
                                                    beta2=case.beta2, eps=case.eps),
                            layout="bf16_mixed" if lay == 1 else "fp32",
                            max_grad_norm=case.max_norm, loss_scaler=scaler, grads=self.grads)
        self.sched = sb.CosineAnnealingLR(self.opt, case.cosine[0], case.cosine[1],
                                          case.cosine[2]) if case.cosine else None
        self.hist = []

    def load_grads(self, grads):
        for g_dev, g in zip(self.grads, grads):
            if g_dev is not None and g is not None and g.size:
                g_dev.copy_(to_device(self.torch, g, self.case.layout))

    def step(self, t: int, scale: float):
        self.load_grads(self.case.grads(t, scale))
        self.opt.step()
        info = self.opt.info()
        self.hist.append((info.step, info.skipped, info.loss_scale, info.found_inf,
                          info.grad_norm))
        if self.sched:
            self.sched.step()
        return info

    def params_host(self):
        return [to_host(p, self.case.layout) for p in self.params]

    def state_host(self, i, kind):
        return self.opt.read_state(i, kind)


def ulp_diff_bf16(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """|a - b| in bf16 ulps (sign-magnitude ordering)."""
    def ordered(x):
        x = x.astype(np.int32)
        return np.where(x & 0x8000, -(x & 0x7FFF), x)
    return np.abs(ordered(a) - ordered(b))


def max_rel_err(a: np.ndarray, b: np.ndarray) -> float:
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    den = np.maximum(np.abs(b), 1e-30)
    return float(np.max(np.abs(a - b) / den)) if a.size else 0.0
