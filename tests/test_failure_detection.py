"""Failure detection, tested without faulting, trapping or hanging a GPU.

* Device: every pipeline wait is bounded. The self-test waits on an mbarrier
  nothing arrives at with a 20 ms limit: the kernel must give up, report it to
  the host, and leave the context usable (a normal optimizer step then runs).
* Host, CPU only: a data-parallel rank that dies before the step makes the
  surviving rank's collective end with an error within the process-group
  timeout instead of hanging (gloo ranks)."""
import ctypes
import datetime
import os
import queue
import socket
import time

import numpy as np
import pytest
import torch

import soar_b200 as sb


@pytest.mark.gpu
def test_bounded_wait_times_out_and_reports(cuda):
    lib = sb.lib()
    timed_out = ctypes.c_int(-1)
    waited = ctypes.c_uint64(0)
    limit = 20_000_000  # 20 ms
    assert lib.soar_selftest_bounded_wait(limit, 0, ctypes.byref(timed_out),
                                          ctypes.byref(waited)) == 0, lib.soar_last_error()
    assert timed_out.value == 1
    assert limit <= waited.value < 50 * limit
    # the context is intact: a real step still works
    p = cuda.ones(1, device="cuda")
    g = cuda.full((1,), 0.5, device="cuda")
    opt = sb.AdamW([p], grads=[g])
    opt.step()
    assert abs(p.item() - np.float32(0.99899)) < 1e-6
    assert opt.info().error == 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, port, q):
    import torch.distributed as dist

    from soar_b200 import dp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        q.put((1, "left"))  # dies between steps, with no collective in flight
        q.close()
        q.join_thread()
        os._exit(0)
    t0 = time.time()
    try:
        parts = torch.zeros(2, dtype=torch.float64)
        part = torch.zeros(1, dtype=torch.float64)
        dist.all_gather_into_tensor(parts, part) if hasattr(dist, "all_gather_into_tensor") \
            else dist.all_gather([torch.zeros(1, dtype=torch.float64)] * 2, part)
        q.put((0, "no error"))
    except Exception as ex:  # the expected path
        q.put((0, f"error after {time.time() - t0:.1f}s: {type(ex).__name__}"))


def test_dead_rank_is_detected_on_host():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.time() + 120
    while len(got) < 2 and time.time() < deadline:
        try:
            r, msg = q.get(timeout=2)
            got[r] = msg
        except queue.Empty:
            pass
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.terminate()
    assert got.get(1) == "left"
    assert got.get(0, "").startswith("error after"), got
