"""GPU test of soar_grad_sumsq_noalloc, the allocation-free entry point.

It exists for callers that cannot call cudaMalloc -- a runtime that reserves all
of a GPU's memory up front in its own pool, or a latency-sensitive loop that
cannot take cudaMalloc's device-wide synchronisation -- and keeps its scratch in
a static device array shared by every call. This checks, through the C-ABI, that
it returns the same gradient sum of squares as the allocating path (an
optimizer handle's soar_optim_grad_sumsq), within the fp32 tolerance the parity
tests use (1e-6 relative), on two calls in a row, so a second call sees the
array as the first left it. Kept in its own file, collected last.
"""
import ctypes

import numpy as np
import pytest

import soar_b200 as sb
from soar_b200 import synth

pytestmark = pytest.mark.gpu

RTOL = 1e-6
INIT_SCALE = 1024.0


def _device_grads(torch, layout, sizes, call):
    """Seeded grads, one of them starting off the 16-byte boundary."""
    out, keep = [], []
    for i, n in enumerate(sizes):
        g = synth.normal(synth.seed_of(77, i, call), n, 0.5) * np.float32(INIT_SCALE)
        if layout == sb.LAYOUT_BF16_MIXED:
            t = torch.from_numpy(synth.to_bf16_bits(g).view(np.int16)).view(torch.bfloat16)
        else:
            t = torch.from_numpy(g.astype(np.float32))
        off = 1 if i == 2 else 0
        buf = torch.zeros(n + off, dtype=t.dtype, device="cuda")
        buf[off:].copy_(t.cuda())
        keep.append(buf)
        out.append(buf[off:])
    return out, keep


@pytest.mark.parametrize("layout", [sb.LAYOUT_FP32, sb.LAYOUT_BF16_MIXED], ids=["fp32", "bf16"])
def test_noalloc_sumsq_matches_allocating_path(cuda, layout):
    torch = cuda
    lib = sb.lib()
    sizes = [1, 3, 4097, 100_000, 65_537]
    dtype = torch.bfloat16 if layout == sb.LAYOUT_BF16_MIXED else torch.float32
    grads, keep = _device_grads(torch, layout, sizes, call=0)
    params = [torch.zeros(n, dtype=dtype, device="cuda") for n in sizes]
    opt = sb.AdamW(params, layout="bf16_mixed" if layout else "fp32", grads=grads,
                   loss_scaler=sb.LossScalerOptions(init_scale=INIT_SCALE))
    inv_scale = np.float32(1.0) / np.float32(INIT_SCALE)
    ptrs = (ctypes.c_void_p * len(sizes))(*[g.data_ptr() for g in grads])
    numel = (ctypes.c_uint64 * len(sizes))(*sizes)
    allocating = torch.zeros(1, dtype=torch.float64, device="cuda")
    no_alloc = torch.zeros(1, dtype=torch.float64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for call in (1, 2):
        fresh, keep2 = _device_grads(torch, layout, sizes, call)
        for g, f in zip(grads, fresh):
            g.copy_(f)
        opt.grad_sumsq(allocating.data_ptr())
        rc = lib.soar_grad_sumsq_noalloc(ptrs, numel, len(sizes), layout, float(inv_scale),
                                         no_alloc.data_ptr(), stream)
        assert rc == 0, lib.soar_last_error()
        torch.cuda.synchronize()
        a, b = float(allocating[0]), float(no_alloc[0])
        assert a > 0 and abs(b - a) <= RTOL * a, (call, a, b)
        # and both against a host fp64 sum
        host = sum(float(np.sum((g.float().cpu().numpy().astype(np.float64) * inv_scale) ** 2))
                   for g in grads)
        assert abs(b - host) <= RTOL * host, (call, b, host)


def test_noalloc_rejects_too_many_tensors(cuda):
    torch = cuda
    lib = sb.lib()
    n = 65  # one more than SOAR_NOALLOC_MAX_TENSORS
    g = torch.ones(n, device="cuda")
    ptrs = (ctypes.c_void_p * n)(*[g.data_ptr() + 4 * i for i in range(n)])
    numel = (ctypes.c_uint64 * n)(*([1] * n))
    out = torch.zeros(1, dtype=torch.float64, device="cuda")
    rc = lib.soar_grad_sumsq_noalloc(ptrs, numel, n, sb.LAYOUT_FP32, 1.0, out.data_ptr(),
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == -1
    assert b"at most 64" in lib.soar_last_error()
