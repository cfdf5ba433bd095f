"""Optimizer-state checkpoint/resume (soar_optim_save_state / load_state).

The reference saves model weights only (src/nn/soar_model.cpp:427-463), so a
resumed run loses Adam's moments, the step count and (here) the loss scale.
A run interrupted at step 6, saved, restored into a freshly created optimizer
and continued must end bit-identical to the uninterrupted run -- through a
skipped step and a loss-scale growth. The file must parse with the
reference's weight-record layout, and a weights-only (version 1) file must be
refused with an error."""
import struct

import numpy as np
import pytest

import cases
from gpu_helpers import GpuRun

import soar_b200 as sb

pytestmark = pytest.mark.gpu


def _state(run):
    out = [p.copy() for p in run.params_host()]
    for i in range(len(run.case.sizes)):
        for k in (sb.STATE_MASTER, sb.STATE_M, sb.STATE_V):
            out.append(run.opt.read_state(i, k))
    return out


def _parse_soar(path):
    """The reference's reader loop (soar_model.cpp:466-523)."""
    with open(path, "rb") as f:
        magic, version, variant, count = struct.unpack("<4I", f.read(16))
        recs = {}
        for _ in range(count):
            name = f.read(128).split(b"\0")[0].decode()
            ndim = struct.unpack("<I", f.read(4))[0]
            shape = struct.unpack("<4I", f.read(16))
            nbytes = struct.unpack("<Q", f.read(8))[0]
            recs[name] = (ndim, shape, f.read(nbytes))
    return magic, version, recs


@pytest.mark.parametrize("case", [cases.mixed_small(steps=12), cases.fp32_edge()],
                         ids=lambda c: c.name)
def test_resume_is_bit_identical(cuda, tmp_path, case):
    torch = cuda
    steps = case.steps if case.layout == 0 else 12
    cut = steps // 2
    full = GpuRun(torch, case)
    scale = case.init_scale
    for t in range(1, steps + 1):
        scale = full.step(t, scale).loss_scale

    first = GpuRun(torch, case)
    scale = case.init_scale
    for t in range(1, cut + 1):
        scale = first.step(t, scale).loss_scale
    path = tmp_path / "optim.soar"
    first.opt.save_state(path)
    info_saved = first.opt.info()
    del first

    resumed = GpuRun(torch, case)          # fresh params and zero state
    resumed.opt.load_state(path)
    info = resumed.opt.info()
    assert (info.step, info.skipped, info.loss_scale, info.growth_tracker) == (
        info_saved.step, info_saved.skipped, info_saved.loss_scale, info_saved.growth_tracker)
    for t in range(cut + 1, steps + 1):
        scale = resumed.step(t, scale).loss_scale

    a, b = full.opt.info(), resumed.opt.info()
    assert (a.step, a.skipped, a.loss_scale) == (b.step, b.skipped, b.loss_scale)
    for x, y in zip(_state(full), _state(resumed)):
        np.testing.assert_array_equal(x, y)

    magic, version, recs = _parse_soar(path)
    assert magic == 0x534F4152 and version == 2
    assert "optim.counters" in recs
    for i, n in enumerate(case.sizes):
        for k in ("master", "m", "v"):
            ndim, shape, data = recs[f"optim.{k}.{i}"]
            assert ndim == 1 and shape[0] == n and len(data) == 4 * n


def test_weights_only_file_is_refused(cuda, tmp_path):
    torch = cuda
    p = torch.zeros(4, device="cuda")
    g = torch.zeros(4, device="cuda")
    opt = sb.AdamW([p], grads=[g])
    path = tmp_path / "weights.soar"
    with open(path, "wb") as f:  # a version-1 file as SOARModel::save_weights writes it
        f.write(struct.pack("<4I", 0x534F4152, 1, 0, 1))
        f.write(b"stem.conv.weight".ljust(128, b"\0"))
        f.write(struct.pack("<I4IQ", 1, 4, 1, 1, 1, 16))
        f.write(np.ones(4, np.float32).tobytes())
    with pytest.raises(sb.SoarError, match="version"):
        opt.load_state(path)
