"""The fused step captured once into a CUDA graph and replayed, against the
same steps run eagerly: identical skip / loss-scale / step sequences and
bit-identical params, master, m and v. The case has clipping, the dynamic
loss scaler, injected inf (skip + backoff) and growth, so every device-side
decision is exercised on replay."""
import numpy as np
import pytest

import cases
from gpu_helpers import GpuRun

import soar_b200 as sb

pytestmark = pytest.mark.gpu


def test_captured_step_replays_like_eager(cuda):
    torch = cuda
    case = cases.mixed_small(steps=14)
    eager = GpuRun(torch, case)
    graphed = GpuRun(torch, case)
    s = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        graphed.opt.step(s)
    torch.cuda.synchronize()
    scale_e = scale_g = case.init_scale
    for t in range(1, case.steps + 1):
        scale_e = eager.step(t, scale_e).loss_scale
        graphed.load_grads(case.grads(t, scale_g))
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        info = graphed.opt.info()
        graphed.hist.append((info.step, info.skipped, info.loss_scale, info.found_inf,
                             info.grad_norm))
        scale_g = info.loss_scale
    assert [h[:4] for h in graphed.hist] == [h[:4] for h in eager.hist]
    assert any(h[3] for h in eager.hist) and eager.hist[-1][1] > 0   # skips happened
    for i in range(len(case.sizes)):
        np.testing.assert_array_equal(graphed.params_host()[i], eager.params_host()[i])
        for kind in (sb.STATE_MASTER, sb.STATE_M, sb.STATE_V):
            np.testing.assert_array_equal(graphed.state_host(i, kind).view(np.uint32),
                                          eager.state_host(i, kind).view(np.uint32))
    del graph
    eager.opt.close()
    graphed.opt.close()
