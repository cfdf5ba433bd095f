"""Weight EMA fused into the update kernel (soar_optim_enable_ema), against the
oracle's restatement of ModelEMA::update (pinned to the reference's own
ema.hpp in test_oracle.py). fp32 layout: bit-exact; mixed layout (EMA of the
fp32 master, no update on skipped steps): within 1e-6 relative, skip sequence
exact. apply_to makes the weights the shadow."""
import numpy as np
import pytest

import cases
from gpu_helpers import GpuRun, max_rel_err
from test_oracle import run_port

import soar_b200 as sb

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case,decay", [(cases.c2(limit=30, steps=8), 0.99),
                                        (cases.mixed_small(steps=12), 0.9),
                                        (cases.fp32_edge(), 0.999)],
                         ids=lambda x: getattr(x, "name", str(x)))
def test_fused_ema_matches_oracle(oracle_mod, cuda, case, decay):
    o = oracle_mod
    cfg = o.StepConfig(layout=case.layout, lr=case.lr, max_norm=case.max_norm,
                       use_scaler=case.use_scaler, growth_interval=case.growth_interval)
    port = o.PortOptimizer(case.params0(), case.wd, cfg, init_scale=case.init_scale)
    port.enable_ema(decay)
    run = GpuRun(cuda, case)
    run.opt.enable_ema(decay)
    scale = case.init_scale
    lr = case.lr
    for t in range(1, case.steps + 1):
        port.step(case.grads(t, port.state.scale), lr)
        scale = run.step(t, scale).loss_scale
        if case.cosine:
            lr = o.cosine_lr(case.lr, case.cosine[1], case.cosine[0], case.cosine[2], t)
    for i, n in enumerate(case.sizes):
        if n == 0:
            continue
        got = run.opt.read_state(i, sb.STATE_EMA)
        if case.layout == 0:
            np.testing.assert_array_equal(got.view(np.uint32), port.ema[i].view(np.uint32))
        else:
            assert max_rel_err(got, port.ema[i]) <= 1e-6
    # apply_to: weights become the shadow
    run.opt.ema_apply_to()
    cuda.cuda.synchronize()
    for i, n in enumerate(case.sizes):
        if n == 0:
            continue
        w = run.opt.read_state(i, sb.STATE_MASTER)
        np.testing.assert_array_equal(w, run.opt.read_state(i, sb.STATE_EMA))
