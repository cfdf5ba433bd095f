"""Benchmark of the fused optimizer step (ZeRO-1 DP).

Workload: 200M parameters, bf16 params and bf16 grads (N(0,1e-3) x loss scale
65536, seeded per rank), fp32 master/m/v, 25M-element gradient buckets,
global-norm clip 1.0, dynamic loss scaler, lr 1e-3, wd 0.01. At N GPUs each
rank brings its own full 200M-element gradient; a step reduce-scatters it, runs
the fused unscale/norm/clip/AdamW on the rank's 1/N shard and all-gathers the
bf16 params -- by default with both collectives fused into the kernels over
peer memory and the ranks synchronised by device-side flags (--dp fused; with
small NCCL collectives as the synchronisation instead: --dp fused-nccl), or
with NCCL around the kernels (--dp nccl). Unit:
one parameter-gradient of one rank reduced and applied, so each GPU's input is
fixed as N grows ("weak"); at N = 1 it is simply parameters updated per
second.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Rank 0 prints one JSON line. `--impl reference` times the reference's own CPU
AdamW (oracle/_ref: the unmodified src/optim/adamw.cpp; the port oracle if that
was not built) on a bounded sample of the same workload with all host threads.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT / "soar.cpp_b200", ROOT):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

N_PARAMS = 200_000_000
BUCKET = 25_000_000
BYTES_PER_PARAM = 28          # algorithmic: read g 2 + master/m/v 12, write master/m/v 12 + param 2
METRIC = "AdamW Gparams/s (fused ZeRO-1 optimizer step, 200M bf16-mixed params)"
UNIT = "Gparams/s"
# dram__bytes_read.sum + dram__bytes_write.sum of one k_apply launch on the full
# 200M workload at N=1 (profiles/k_apply_config4.md: 2,801,499,392 read +
# 2,740,448,512 written). Reported only for the workload it was measured on.
APPLY_TRAFFIC_BYTES = {200_000_000: 5_541_141_760}


def measured_peak_hbm() -> tuple[float, str]:
    try:
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--params", type=int, default=N_PARAMS)
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true",
                    help="config 5: flat 1M..2B params in both layouts, one JSON line each "
                         "(not the headline line)")
    ap.add_argument("--sweep-sizes", default="1000000,16000000,256000000,1000000000,2000000000")
    ap.add_argument("--cpu-sample", action="store_true",
                    help="print the CPU reference sample of --params params as JSON and exit "
                         "(threads from OMP_NUM_THREADS; the 1-thread baseline row runs this)")
    ap.add_argument("--configs", action="store_true",
                    help="configs 1-3 at their own shapes on one GPU, one JSON line each "
                         "(not the headline line)")
    ap.add_argument("--dp", default="fused", choices=["fused", "fused-nccl", "nccl"],
                    help="N>1: collectives fused into the kernels over peer memory, the ranks "
                         "synchronised by device-side flags (default) or by small NCCL "
                         "collectives between the launches (fused-nccl); or NCCL "
                         "reduce-scatter / all-gather around the kernels (nccl)")
    return ap.parse_args()


# ------------------------------------------------------------ CPU baseline --

def cpu_reference_sample(n: int, steps: int, warmup: int = 1) -> dict:
    """The reference's clip_grad_norm(1.0) + step() (adamw.cpp:87-176) on one
    fp32 bucket of n params (the unscaled grads and fp32 master of the mixed
    workload), OpenMP over all host threads. Returns Gparams/s."""
    import numpy as np

    from oracle import oracle
    from soar_b200 import synth
    threads = int(os.environ.get("OMP_NUM_THREADS", "0")) or (os.cpu_count() or 1)
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    p = synth.normal(synth.seed_of(4, 0), n, 0.02)
    g = synth.normal(synth.seed_of(4, 1, 0), n, 1e-3)
    if oracle.ref_available():
        opt = oracle.RefAdamW([p], [g], lr=1e-3, weight_decay=0.01)
        kind = "reference"

        def one():
            opt.clip_grad_norm(1.0)
            opt.step()
    else:
        cfg = oracle.StepConfig(layout=0, max_norm=1.0)
        opt = oracle.PortOptimizer([p], [0.01], cfg)
        kind = "port"

        def one():
            opt.step([g])
    for _ in range(warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    dt = time.perf_counter() - t0
    return {"value": n * steps / dt / 1e9, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{steps} steps of clip_grad_norm(1.0)+step() on one fp32 bucket of "
                      f"{n} params (host arrays, unscale/bf16 cast not timed)",
            "ms_per_step": dt / steps * 1e3}


def cpu_single_thread_sample(n: int, steps: int = 3) -> dict | None:
    """The same sample on one host thread, in a child process (OpenMP reads
    OMP_NUM_THREADS when the library starts)."""
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run([sys.executable, str(Path(__file__).resolve()), "--cpu-sample",
                        "--params", str(n), "--steps", str(steps)],
                       env=env, capture_output=True, text=True, timeout=300)
    lines = [x for x in r.stdout.splitlines() if x.startswith("{")]
    if r.returncode != 0 or not lines:
        return None
    d = json.loads(lines[-1])
    return {"value": d["value"], "cores": d["cores"], "sample": d["sample"]}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    n = min(BUCKET, args.params)
    t0 = time.perf_counter()
    res = cpu_reference_sample(n, args.steps, args.warmup)
    line = {"impl": "reference", "metric": METRIC, "value": res["value"], "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config4 sample: one 25M bucket, fp32 reference AdamW",
                       "params": n},
            "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": res["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "wall_s": time.perf_counter() - t0}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ clocks --

class ClockSampler:
    """SM clocks and clock-event reasons of the GPUs in use, sampled during the
    timed region (reads only; no setting is touched). An NVML thread samples
    every ~5 ms, so even a timed region of a few tens of ms gets several
    samples; without NVML, `nvidia-smi -lms 200` into a temporary file."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    FIELDS = ("index,clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, devices: list[int]):
        self.devices = devices
        self.samples = []          # (time, device position, sm MHz, reason names)
        self.max_mhz = []
        self.window = [None, None]
        self.thread = self.proc = None
        self.stopping = False

    def _nvml_handles(self, nvml):
        import torch
        out = []
        for d in self.devices:
            p = torch.cuda.get_device_properties(d)
            for i in range(nvml.nvmlDeviceGetCount()):
                h = nvml.nvmlDeviceGetHandleByIndex(i)
                pci = nvml.nvmlDeviceGetPciInfo(h)
                if (pci.domain, pci.bus, pci.device) == (p.pci_domain_id, p.pci_bus_id,
                                                          p.pci_device_id):
                    out.append(h)
                    break
            else:
                raise RuntimeError("no NVML device for cuda:%d" % d)
        return out

    def start(self):
        import threading
        try:
            import pynvml as nvml
            nvml.nvmlInit()
            handles = self._nvml_handles(nvml)
            self.max_mhz = [nvml.nvmlDeviceGetMaxClockInfo(h, nvml.NVML_CLOCK_SM) for h in handles]
            masks = [(name, getattr(nvml, const)) for name, const in self.REASONS]

            def run():
                while not self.stopping:
                    t = time.perf_counter()
                    for k, h in enumerate(handles):
                        try:
                            sm = nvml.nvmlDeviceGetClockInfo(h, nvml.NVML_CLOCK_SM)
                            r = nvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        except Exception:
                            continue
                        self.samples.append((t, k, float(sm), [n for n, m in masks if r & m]))
                    time.sleep(0.005)

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
        except Exception:
            self.thread = None
            self._start_smi()

    def _start_smi(self):
        import tempfile
        try:
            self.fh = tempfile.NamedTemporaryFile("w+", suffix=".csv")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def begin(self):
        self.window[0] = time.perf_counter()

    def end(self):
        self.window[1] = time.perf_counter()

    def stop(self) -> dict | None:
        if self.thread is not None:
            self.stopping = True
            self.thread.join(5)
            lo, hi = self.window
            inside = [x for x in self.samples if lo is not None and hi is not None and
                      lo - 0.005 <= x[0] <= hi + 0.005]
            if not inside and self.samples and hi is not None:   # the nearest sample after the end
                after = [x for x in self.samples if x[0] >= hi]
                inside = after[:len(self.devices)] or self.samples[-len(self.devices):]
            if not inside:
                return None
            reasons = sorted({n for x in inside for n in x[3]})
            return {"sm_mhz": statistics.median(x[2] for x in inside),
                    "sm_max_mhz": max(self.max_mhz), "reasons": reasons,
                    "samples": len(inside), "source": "nvml"}
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except Exception:
            self.proc.kill()
        self.fh.seek(0)
        sm, mx, reasons = [], [], set()
        names = [n for n, _ in self.REASONS]
        for line in self.fh.read().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 7 or not f[0].isdigit() or int(f[0]) not in self.devices:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[3:7]):
                if v.lower() == "active":
                    reasons.add(nm)
        self.fh.close()
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi"}


# ----------------------------------------------------------------- our arm --

def run_ours(args):
    import numpy as np
    import torch

    import soar_b200 as sb
    from soar_b200 import dp, synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    comm = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        comm = dp.TorchComm()
    n = args.params
    dev = torch.device("cuda", local)

    # params: identical on every rank; grads: per rank
    p_host = synth.to_bf16_bits(synth.normal(synth.seed_of(4, 0), n, 0.02))
    g_host = synth.to_bf16_bits(synth.normal(synth.seed_of(4, 1, 0, rank), n, 1e-3)
                                * np.float32(65536.0))
    params = torch.from_numpy(p_host.view(np.int16)).view(torch.bfloat16).to(dev)
    grads = torch.from_numpy(g_host.view(np.int16)).view(torch.bfloat16).to(dev)

    def make_opt(sp, sg):
        return sb.AdamW([sb.ParamGroup(sp, 0.01)], sb.AdamWOptions(lr=1e-3, weight_decay=0.01),
                        layout="bf16_mixed", max_grad_norm=1.0,
                        loss_scaler=sb.LossScalerOptions(init_scale=65536.0), grads=sg,
                        device=local)

    fused = world > 1 and args.dp.startswith("fused")
    dev_sync = fused and args.dp == "fused"
    if fused:
        z = dp.FusedZeroOneAdamW(n, BUCKET, make_opt, device=local, init_params=params,
                                 sync="device" if dev_sync else "nccl")
        del params, grads
        params, grads = z.params, z.grads
        grads.copy_(torch.from_numpy(g_host.view(np.int16)).view(torch.bfloat16).to(dev))
        # k_rs_sumsq, k_apply<all-gather> (+ the end-of-step flag wait)
        launches_per_step = 3 if dev_sync else 2
    else:
        z = dp.ZeroOneAdamW(params, grads, BUCKET, make_opt, comm)
        launches_per_step = 2
    stream = torch.cuda.current_stream()
    shard_params = sum(b.own_size for b in z.buckets)

    def barrier():
        if comm:
            torch.distributed.barrier(device_ids=[local])

    def one_step(ev=None):
        if dev_sync:
            z.step()  # one call: no host collective, so no event inside the step
            return
        if fused:
            z.barrier()
            z.reduce()
            parts = z.gather_partials()
        else:
            z.reduce_scatter()
            parts = z.norm_partials()
        if ev is not None:
            ev[0].record(stream)
        z.update(parts)
        if ev is not None:
            ev[1].record(stream)
        if fused:
            z.barrier()
        else:
            z.all_gather()

    for _ in range(args.warmup):
        one_step()
    # the clock sampler starts before the barrier, so no rank enters the timed
    # region while another is still setting it up; rank 0 samples every GPU
    clocks = ClockSampler(list(range(world))) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    apply_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if clocks:
        clocks.begin()
    start.record(stream)
    for k in range(args.steps):
        one_step(apply_ev[k])
    end.record(stream)
    torch.cuda.synchronize()
    if clocks:
        clocks.end()   # the device work of the timed region is done here
    barrier()
    torch.cuda.synchronize()
    clock_info = clocks.stop() if clocks else None

    ms = start.elapsed_time(end)
    apply_ms = None if dev_sync else [a.elapsed_time(b) for a, b in apply_ev]

    # per-phase breakdown (a separate loop after the timed region, not part of
    # `value`): CUDA events around each phase of the step on this rank (the
    # fused path runs its caller-synchronised form here, so the phases split)
    phase_names = (["barrier", "reduce_scatter+sumsq", "partial_allgather", "update+allgather",
                    "barrier2"] if fused else
                   ["reduce_scatter", "sumsq+partial_allgather", "update", "param_allgather"])
    pev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(phase_names) + 1)]
           for _ in range(10)]
    barrier()  # (rank 0 stopped the clock sampler: start the ranks together)
    torch.cuda.synchronize()
    for ev in pev:
        ev[0].record(stream)
        if fused:
            z.barrier(); ev[1].record(stream)
            z.reduce(); ev[2].record(stream)
            parts = z.gather_partials(); ev[3].record(stream)
            z.update(parts); ev[4].record(stream)
            z.barrier(); ev[5].record(stream)
        else:
            z.reduce_scatter(); ev[1].record(stream)
            parts = z.norm_partials(); ev[2].record(stream)
            z.update(parts); ev[3].record(stream)
            z.all_gather(); ev[4].record(stream)
    torch.cuda.synchronize()
    ph = torch.tensor([statistics.mean(e[i].elapsed_time(e[i + 1]) for e in pev)
                       for i in range(len(phase_names))], dtype=torch.float64, device=dev)
    if comm:
        torch.distributed.all_reduce(ph, op=torch.distributed.ReduceOp.MAX)
    phases = {k: round(float(v), 4) for k, v in zip(phase_names, ph.tolist())}
    nvl = None
    if fused:
        try:  # a reported roofline, never a reason to lose the bench line
            nvl = nvlink_rates(torch, world, rank, local, 2 * shard_params, phases)
        except Exception as ex:
            nvl = {"error": str(ex)[:300]}
    if apply_ms is None:  # device-synchronised step: the update phase of the loop above
        apply_ms = [float(ph[phase_names.index("update+allgather")])]
    t = torch.tensor([ms, statistics.mean(apply_ms)], dtype=torch.float64, device=dev)
    if comm:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms_max, apply_ms_max = float(t[0]), float(t[1])
    info = z.opt.info()

    # ---- end to end through the public API with host buffers -------------
    g_pin = torch.from_numpy(g_host.view(np.int16)).view(torch.bfloat16).pin_memory()
    p_pin = torch.empty(n, dtype=torch.bfloat16).pin_memory()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    # the step's result read back: each rank's own updated shard of the bf16
    # params (the ranks' shards together are the whole model once; at N = 1
    # the whole model)
    own = [(b.own_start, b.own_size) for b in z.buckets if b.own_size > 0]
    for _ in range(args.e2e_steps):
        grads.copy_(g_pin, non_blocking=True)
        z.step()
        for lo, sz in own:
            p_pin[lo:lo + sz].copy_(params[lo:lo + sz], non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if comm:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    e2e_ms = float(t[0])

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_reference_sample(min(BUCKET, n), 5)
            cpu.pop("ms_per_step", None)
            cpu["single_thread"] = cpu_single_thread_sample(min(BUCKET, n) // 5)
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"error": str(ex)}

    if fused:
        z.close()
    if comm:
        torch.distributed.barrier(device_ids=[local])
        torch.distributed.destroy_process_group()
    if rank != 0:
        return 0
    peak, peak_kind = measured_peak_hbm()
    apply_bytes = BYTES_PER_PARAM * shard_params
    achieved = apply_bytes / (apply_ms_max * 1e-3) / 1e9
    units = world * n * args.steps
    line = {
        "metric": METRIC,
        "value": units / (ms_max * 1e-3) / 1e9,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "config4: ZeRO-1 fused AdamW step, 200M params bf16 params+grads, "
                               "fp32 master/m/v, 25M buckets, clip 1.0, loss scaler 65536",
                   "params": n, "bucket": BUCKET, "params_per_rank_shard": shard_params,
                   "parallelism": f"dp{world} zero1" + (
                       " (collectives fused into the kernels over peer memory, device-side "
                       "flag synchronisation)" if dev_sync else
                       " (collectives fused into the kernels over peer memory, NCCL "
                       "synchronisation)" if fused else
                       " (NCCL reduce-scatter/all-gather)" if world > 1 else ""),
                   "global_batch": None, "seq_len": None,
                   "l2": "inputs larger than L2 (16 B/param resident state = "
                         f"{16 * shard_params / 1e9:.1f} GB per rank)"},
        "roofline": {"bound": "hbm", "kernel": "k_apply", "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": APPLY_TRAFFIC_BYTES.get(shard_params),
                     "algorithmic_bytes_per_launch": apply_bytes,
                     "apply_ms": apply_ms_max},
        "cpu_baseline": cpu,
        "e2e": {"value": world * n * args.e2e_steps / (e2e_ms * 1e-3) / 1e9, "unit": UNIT,
                "h2d_bytes_per_step": 2 * n, "d2h_bytes_per_step": 2 * shard_params,
                "transfers": "per rank: H2D of its full bf16 gradient from pinned memory, D2H "
                             "of its updated shard of the bf16 params",
                "ms_per_step": e2e_ms / args.e2e_steps},
        "clocks": clock_info,
        "gpu_launches": launches_per_step * args.steps,
        "phases_ms": phases,
        "nvlink": nvl,
        "final_info": {"step": info.step, "skipped": info.skipped, "loss_scale": info.loss_scale,
                       "grad_norm": info.grad_norm},
    }
    print(json.dumps(line), flush=True)
    return 0


def nvlink_rates(torch, world, rank, local, shard_bytes, phases):
    """The fused kernels' NVLink rates against the raw rates of their access
    patterns on this box (soar_nvlink_probe: all ranks at once, no arithmetic,
    the same bytes per peer as the step). GB/s per direction per rank; max
    time over ranks."""
    import ctypes as C

    import torch.distributed as dist

    from soar_b200 import optim as _o
    lib = _o.lib()
    tile_lcm = 64 * 1024
    bpp = max(tile_lcm, shard_bytes // tile_lcm * tile_lcm)
    ptr = C.c_void_p()
    handle = (C.c_ubyte * _o.IPC_HANDLE_BYTES)()
    _o._check(lib.soar_ipc_alloc(world * bpp, local, C.byref(ptr), handle), "soar_ipc_alloc")
    handles = [None] * world
    dist.all_gather_object(handles, bytes(handle))
    bases, opened = [], []
    for q, h in enumerate(handles):
        if q == rank:
            bases.append(ptr.value)
            continue
        peer = C.c_void_p()
        buf = (C.c_ubyte * _o.IPC_HANDLE_BYTES).from_buffer_copy(h)
        _o._check(lib.soar_ipc_open(buf, local, C.byref(peer)), "soar_ipc_open")
        bases.append(peer.value)
        opened.append(peer.value)
    arr = (C.c_void_p * world)(*bases)
    err = torch.zeros(1, dtype=torch.int32, device=f"cuda:{local}")
    stream = torch.cuda.current_stream()
    sms = torch.cuda.get_device_properties(local).multi_processor_count
    gbs = lambda ms: (world - 1) * bpp / (ms * 1e-3) / 1e9

    def timed(mode, tile, stages, grid, reps=5):
        def launch():
            _o._check(lib.soar_nvlink_probe(arr, world, rank, bpp, mode, tile, stages, grid,
                                            C.c_void_p(err.data_ptr()),
                                            C.c_void_p(stream.cuda_stream)), "soar_nvlink_probe")
        for _ in range(2):
            launch()
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            launch()
        b.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) / reps], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return round(gbs(float(t[0])), 1)

    pull = {f"tile{tile}_stages{st}_grid{g}": timed(0, tile, st, g)
            for tile, st, g in ((4096, 4, sms), (2048, 8, 2 * sms))
            if st * tile * (world - 1) <= 200 * 1024}
    push = {f"tile{tile}_grid{g}": timed(1, tile, 0, g)
            for tile, g in ((2048, 2 * sms), (8192, sms))}
    torch.cuda.synchronize()
    failed = int(err.item())
    dist.barrier(device_ids=[local])
    for pp in opened:
        lib.soar_ipc_close(C.c_void_p(pp), local)
    dist.barrier(device_ids=[local])
    lib.soar_ipc_free(ptr, local)
    rs = (world - 1) * shard_bytes / (phases["reduce_scatter+sumsq"] * 1e-3) / 1e9
    ag = (world - 1) * shard_bytes / (phases["update+allgather"] * 1e-3) / 1e9
    p_pull, p_push = max(pull.values()), max(push.values())
    return {"unit": "GB/s per direction per rank", "bytes_per_peer": shard_bytes,
            "k_rs_sumsq": {"achieved": round(rs, 1), "peak": p_pull, "frac": round(rs / p_pull, 3),
                           "peak_kind": "measured: soar_nvlink_probe pull, all ranks at once"},
            "k_apply_allgather": {"achieved": round(ag, 1), "peak": p_push,
                                  "frac": round(ag / p_push, 3),
                                  "peak_kind": "measured: soar_nvlink_probe push, all ranks at once"},
            "probe": {"pull": pull, "push": push, "wait_error": failed}}


def run_sweep(args):
    """one flat tensor of N params, fp32 layout (fp32 param,
    grad, m, v) and mixed layout (bf16 param and grad, fp32 master/m/v), no
    clip or scaler (the plain update), K timed steps after 3 warm-up, back to
    back on one stream. Prints one JSON line per (layout, N): Gparams/s and
    k_apply's achieved GB/s at 28 B/param against the measured HBM peak, and
    the same K steps replayed from a CUDA graph (`graph`: device time, without
    the per-step host launch cost that dominates below ~4M params). Under
    torchrun every rank runs the same sweep on its own GPU as an independent
    replica (the update has no cross-GPU term without a reduce): the ranks
    start each timed region together and the time is the max over ranks;
    `value` counts all ranks' params."""
    import torch

    import soar_b200 as sb
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def sync_max(x):
        """Barrier-free max over ranks of a host float (one tiny all-reduce)."""
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0])

    def together():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier(device_ids=[local])
            torch.cuda.synchronize()

    peak, peak_kind = measured_peak_hbm()
    free = sync_max(-torch.cuda.mem_get_info()[0]) * -1  # the smallest free memory of any rank
    for layout in ("fp32", "bf16_mixed"):
        for n in [int(x) for x in args.sweep_sizes.split(",")]:
            need = 16 * n + (12 * n if layout == "bf16_mixed" else 8 * n)
            if need > 0.9 * free:
                if rank == 0:
                    print(json.dumps({"sweep": True, "layout": layout, "params": n,
                                      "skipped": f"needs {need / 1e9:.1f} GB"}), flush=True)
                continue
            dt = torch.bfloat16 if layout == "bf16_mixed" else torch.float32
            p = (torch.randn(n, device="cuda") * 0.02).to(dt)
            g = (torch.randn(n, device="cuda") * 1e-3).to(dt)
            opt = sb.AdamW([p], sb.AdamWOptions(lr=1e-3, weight_decay=0.01), layout=layout,
                           grads=[g], device=local)
            s = torch.cuda.Stream()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(s):
                for _ in range(3):
                    opt.step(s)
            together()
            with torch.cuda.stream(s):
                # K steps back to back through the API (host launch overhead included
                # wherever it exceeds a step's device time)
                a.record(s)
                for _ in range(args.steps):
                    opt.step(s)
                b.record(s)
            torch.cuda.synchronize()
            ms = sync_max(a.elapsed_time(b) / args.steps)
            # the same K steps captured once in a CUDA graph and replayed: device time
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                for _ in range(args.steps):
                    opt.step(s)
            with torch.cuda.stream(s):
                graph.replay()
            together()
            with torch.cuda.stream(s):
                a.record(s)
                graph.replay()
                b.record(s)
            torch.cuda.synchronize()
            gms = sync_max(a.elapsed_time(b) / args.steps)
            del graph
            gbs = BYTES_PER_PARAM * n / (ms * 1e-3) / 1e9
            ggbs = BYTES_PER_PARAM * n / (gms * 1e-3) / 1e9
            if rank == 0:
                print(json.dumps({"sweep": True, "metric": "AdamW Gparams/s (config 5 sweep)",
                                  "layout": layout, "params": n, "n_gpus": world,
                                  "scaling": "weak", "steps": args.steps, "warmup": 3,
                                  "ms_per_step": ms, "value": world * n / (ms * 1e-3) / 1e9,
                                  "unit": "Gparams/s", "achieved_gbs_per_gpu": gbs,
                                  "peak_gbs": peak, "peak_kind": peak_kind, "frac": gbs / peak,
                                  "graph": {"ms_per_step": gms,
                                            "value": world * n / (gms * 1e-3) / 1e9,
                                            "achieved_gbs_per_gpu": ggbs, "frac": ggbs / peak},
                                  "l2": "larger than L2" if 16 * n > 126e6 else "fits in L2"}),
                      flush=True)
            opt.close()
            del p, g, opt
            torch.cuda.empty_cache()
    if dist is not None:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def run_configs(args):
    """BASELINE configs 1-3 at their own shapes on one GPU, K steps back to back
    through the API after 3 warm-up, one JSON line each: Gparams/s, step ms and
    k_apply-equivalent GB/s (28 B/param) against the measured HBM copy.
      c1  1 fp32 tensor of 1,048,576 params, no clip/scaler;
      c2  the 240-tensor segmentation-net list (~12M fp32), wd 0.05 on conv
          weights / 0 on norms and biases, cosine 1e-3 -> 1e-5 over 100 steps
          (the scheduler steps after every step, on the host);
      c3  400 bf16-mixed tensors summing to 50M, clip 1.0, loss scaler 65536.
    Inputs are device-generated; the numerics of these configs are pinned by
    the parity tests, not here."""
    import math

    import torch

    import soar_b200 as sb
    from soar_b200 import synth
    torch.cuda.set_device(0)
    peak, peak_kind = measured_peak_hbm()

    def rnd(n, std, dt):
        return (torch.randn(n, device="cuda") * std).to(dt)

    c2_shapes = synth.config2_shapes()
    cfgs = {
        "c1": dict(sizes=[1_048_576], wd=[0.01], layout="fp32", clip=0.0, scaler=None,
                   cosine=None),
        "c2": dict(sizes=[int(math.prod(sh)) for _, sh in c2_shapes],
                   wd=[0.05 if k in ("dw", "pw") else 0.0 for k, _ in c2_shapes],
                   layout="fp32", clip=0.0, scaler=None, cosine=(100, 1e-5, 0)),
        "c3": dict(sizes=synth.config3_sizes(), wd=None, layout="bf16_mixed", clip=1.0,
                   scaler=sb.LossScalerOptions(init_scale=65536.0), cosine=None),
    }
    for name, c in cfgs.items():
        dt = torch.bfloat16 if c["layout"] == "bf16_mixed" else torch.float32
        ps = [rnd(n, 0.02, dt) for n in c["sizes"]]
        gs = [rnd(n, 1e-3 * (65536.0 if c["scaler"] else 1.0), dt) for n in c["sizes"]]
        wds = c["wd"] or [0.01] * len(ps)
        groups = [sb.ParamGroup([p], w) for p, w in zip(ps, wds)]
        opt = sb.AdamW(groups, sb.AdamWOptions(lr=1e-3), layout=c["layout"],
                       max_grad_norm=c["clip"], loss_scaler=c["scaler"], grads=gs)
        sched = sb.CosineAnnealingLR(opt, *c["cosine"]) if c["cosine"] else None
        s = torch.cuda.Stream()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            for _ in range(3):
                opt.step(s)
            torch.cuda.synchronize()
            a.record(s)
            for _ in range(args.steps):
                opt.step(s)
                if sched:
                    sched.step()
            b.record(s)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / args.steps
        n = sum(c["sizes"])
        gbs = BYTES_PER_PARAM * n / (ms * 1e-3) / 1e9
        info = opt.info()
        print(json.dumps({"config": name, "metric": "AdamW Gparams/s (BASELINE configs 1-3)",
                          "params": n, "tensors": len(c["sizes"]), "layout": c["layout"],
                          "steps": args.steps, "warmup": 3, "ms_per_step": ms,
                          "value": n / (ms * 1e-3) / 1e9, "unit": "Gparams/s",
                          "achieved_gbs": gbs, "peak_gbs": peak, "peak_kind": peak_kind,
                          "frac": gbs / peak, "final_step": info.step,
                          "skipped": info.skipped}), flush=True)
        if sched:
            sched.close()
        opt.close()
        del ps, gs, opt
        torch.cuda.empty_cache()
    return 0


def main():
    args = parse()
    if args.cpu_sample:
        res = cpu_reference_sample(args.params, args.steps)
        print(json.dumps(res), flush=True)
        return 0
    if args.impl == "reference":
        return run_reference(args)
    if args.sweep:
        return run_sweep(args)
    if args.configs:
        return run_configs(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
