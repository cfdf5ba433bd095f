"""Seeded parity cases shared by the oracle tests, the golden-vector generator
and the GPU parity tests. Every input comes from soar_b200.synth, so the host
oracle and the device see identical bits."""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from soar_b200 import synth


@dataclass
class Case:
    name: str
    layout: int                      # 0 fp32, 1 bf16 mixed
    sizes: list[int]
    wd: list[float]
    steps: int
    lr: float = 1e-3
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    max_norm: float = 0.0
    use_scaler: bool = False
    init_scale: float = 65536.0
    growth_interval: int = 200
    grad_std: float = 1e-2
    param_std: float = 0.02
    inf_every: int = 0               # inject +inf into one grad element every k-th step
    inf_until: int = 1 << 62         # ... only up to this step
    cosine: tuple | None = None      # (total_steps, eta_min, warmup)
    seed: int = 0
    null_grad: list[int] = field(default_factory=list)

    def params0(self) -> list[np.ndarray]:
        out = []
        for i, n in enumerate(self.sizes):
            p = synth.normal(synth.seed_of(self.seed, i, 0), n, self.param_std)
            out.append(synth.to_bf16_bits(p) if self.layout == 1 else p)
        return out

    def grads(self, step: int, scale: float) -> list[np.ndarray | None]:
        """Grads of 1-based `step`; the mixed layout multiplies by the live loss
        scale (as a scaled backward would) and rounds to bf16."""
        out = []
        for i, n in enumerate(self.sizes):
            if i in self.null_grad:
                out.append(None)
                continue
            g = synth.normal(synth.seed_of(self.seed, i, step), n, self.grad_std)
            if self.use_scaler:
                g = (g * np.float32(scale)).astype(np.float32)
            if self.inf_every and step % self.inf_every == 0 and step <= self.inf_until \
                    and i == step % len(self.sizes) and n > 0:
                j = int(synth.uniform_int(synth.seed_of(self.seed, 777, step), 1, 0, n - 1)[0])
                g[j] = np.inf
            out.append(synth.to_bf16_bits(g) if self.layout == 1 else g)
        return out


def c1_small(n: int = 4099, steps: int = 10) -> Case:
    """Config 1 at a CPU-quick size: one fp32 tensor, wd 0.01, no clip/scaler."""
    return Case("c1_small", 0, [n], [0.01], steps, seed=1)


def c1_full() -> Case:
    return Case("c1", 0, [1_048_576], [0.01], 10, seed=1)


def c2(limit: int | None = None, steps: int = 100) -> Case:
    """Config 2: segmentation-net tensor list, wd 0.05 on conv weights only,
    cosine 1e-3 -> 1e-5 over 100 steps."""
    shapes = synth.config2_shapes()
    if limit:
        shapes = shapes[:limit]
    sizes = [int(np.prod(s)) for _, s in shapes]
    wd = [0.05 if k in ("dw", "pw") else 0.0 for k, _ in shapes]
    return Case("c2" if not limit else f"c2_{limit}", 0, sizes, wd, steps, grad_std=1e-3,
                cosine=(100, 1e-5, 0), seed=2)


def c3(scale_total: int = 50_000_000, steps: int = 1000, n: int = 400, inf_until=1 << 62,
       growth_interval: int = 200) -> Case:
    """Config 3: mixed precision, clip 1.0, scaler 65536, +inf every 97th step."""
    sizes = synth.config3_sizes(total=scale_total, n=n, lo=max(1, 16384 * scale_total // 50_000_000),
                                hi=max(2, 262144 * scale_total // 50_000_000))
    return Case("c3", 1, sizes, [0.01] * len(sizes), steps, max_norm=1.0, use_scaler=True,
                grad_std=1e-3, inf_every=97, inf_until=inf_until,
                growth_interval=growth_interval, seed=3)


def mixed_small(steps: int = 12) -> Case:
    """Small mixed case that exercises every branch: skip on inf, backoff,
    growth (interval 4), clip, wd mask, odd sizes."""
    return Case("mixed_small", 1, [1, 3, 4, 7, 8, 1000, 4097], [0.01, 0.0, 0.05, 0.0, 0.01, 0.01, 0.0],
                steps, max_norm=1.0, use_scaler=True, init_scale=1024.0, growth_interval=4,
                grad_std=1e-1, inf_every=5, seed=4)


def fp32_edge() -> Case:
    """fp32 tensor list over the chunk-table edge sizes."""
    sizes = [1, 3, 4, 7, 8, 65535, 65536, 65537, 0, 16383, 16384, 16385]
    wd = [0.01 if i % 2 == 0 else 0.0 for i in range(len(sizes))]
    return Case("fp32_edge", 0, sizes, wd, 3, max_norm=0.5, seed=5, null_grad=[3])
