"""SGD on the fused device step (soar_sgd_create) against the port oracle,
which is pinned bit-for-bit to the reference's own src/optim/sgd.cpp in
test_oracle.py. fp32 layout: bit-exact; mixed layout with loss scaler and clip:
within the parity tolerances, skip/scale sequence exact."""
import numpy as np
import pytest

import cases
from gpu_helpers import max_rel_err, to_device, to_host, ulp_diff_bf16

import soar_b200 as sb

pytestmark = pytest.mark.gpu


def test_kat_sgd_parity_gpu(cuda):
    """tests/test_optimizers.cpp:51-95 on the device: 1.958, then 1.898242."""
    torch = cuda
    p = torch.tensor([2.0], device="cuda")
    g = torch.tensor([0.4], device="cuda")
    opt = sb.SGD([p], sb.SGDOptions(lr=0.1, momentum=0.9, weight_decay=0.01), grads=[g])
    opt.step()
    assert abs(p.item() - np.float32(1.958)) < 1e-6
    g.fill_(0.2)
    opt.step()
    assert abs(p.item() - np.float32(1.898242)) < 1e-6


@pytest.mark.parametrize("layout,momentum,dampening,nesterov", [
    (0, 0.0, 0.0, False), (0, 0.9, 0.0, False), (0, 0.9, 0.1, True),
    (1, 0.9, 0.0, False), (1, 0.5, 0.25, True)])
def test_sgd_matches_oracle(oracle_mod, cuda, layout, momentum, dampening, nesterov):
    torch = cuda
    o = oracle_mod
    mixed = layout == 1
    case = cases.Case("sgd", layout, [1, 3, 8, 1000, 70001, 16385], [0.01, 0.0, 0.05, 0.0, 0.01, 0.0],
                      9, max_norm=1.0 if mixed else 0.0, use_scaler=mixed, init_scale=1024.0,
                      growth_interval=3, grad_std=0.1, inf_every=5 if mixed else 0, seed=90)
    cfg = o.StepConfig(layout=layout, lr=0.05, max_norm=case.max_norm, use_scaler=mixed,
                       growth_interval=3)
    port = o.PortSGD(case.params0(), case.wd, cfg, momentum, dampening, nesterov,
                     init_scale=case.init_scale)
    params = [to_device(torch, p, layout) for p in case.params0()]
    grads = [torch.empty_like(p) for p in params]
    opt = sb.SGD([sb.ParamGroup([p], w) for p, w in zip(params, case.wd)],
                 sb.SGDOptions(lr=0.05, momentum=momentum, dampening=dampening,
                               nesterov=nesterov),
                 layout="bf16_mixed" if mixed else "fp32", max_grad_norm=case.max_norm,
                 loss_scaler=sb.LossScalerOptions(init_scale=1024.0, growth_interval=3)
                 if mixed else None, grads=grads)
    for t in range(1, case.steps + 1):
        gs = case.grads(t, port.state.scale)
        for d, g in zip(grads, gs):
            d.copy_(to_device(torch, g, layout))
        port.step(gs)
        opt.step()
        info = opt.info()
        assert (info.skipped, info.loss_scale, info.step) == (
            port.state.skipped, port.state.scale, port.state.t)
    for i, p in enumerate(params):
        got = to_host(p, layout)
        if mixed:
            assert ulp_diff_bf16(got, port.params[i]).max() <= 1
            assert max_rel_err(opt.read_state(i, sb.STATE_MASTER), port.master[i]) <= 1e-6
        else:
            np.testing.assert_array_equal(got.view(np.uint32), port.params[i].view(np.uint32))
        if momentum:
            buf = opt.read_state(i, sb.STATE_M)
            if mixed:
                assert max_rel_err(buf, port.m[i]) <= 1e-6
            else:
                np.testing.assert_array_equal(buf.view(np.uint32), port.m[i].view(np.uint32))
    with pytest.raises(sb.SoarError):
        opt.read_state(0, sb.STATE_V)
