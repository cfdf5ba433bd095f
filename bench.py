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

Rank 0 prints one JSON line. Besides the timed step it carries:
  e2e       the same step through the public API with host buffers: every
            step copies the rank's gradient in from pinned memory and its
            updated params out, on two copy streams so that the read-back of
            step s overlaps the upload of step s+1;
  roofline  k_apply against the measured HBM copy peak at N = 1; at N > 1 the
            slower of the two fused kernels against its binding resource
            (NVLink or HBM; both kernels under `rooflines`);
  parity    after the timed region, one more step checked against the CPU
            oracle on a sample of rank 0's shard, plus bit-identical params and
            counters on every rank;
  configs   (N = 1) BASELINE configs 1-3 and config-5 sizes, cold-L2 steps
            back to back over several copies, and one cold step alone.

`--impl reference` times the reference's own CPU AdamW (oracle/_ref: the
unmodified src/optim/adamw.cpp; the port oracle if that was not built) on the
same 200M-parameter workload (8 fp32 buckets of 25M) with every host thread,
in a child process that loads nothing of this package.
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
# dram__bytes_read.sum + dram__bytes_write.sum of one k_apply launch on the
# full 200M-parameter shard at N = 1, from a one-pass ncu capture of this
# bench's own command (2,801,499,392 read + 2,740,448,512 written). Reported
# only for the workload it was measured on.
APPLY_TRAFFIC_BYTES = {200_000_000: 5_541_141_760}
# DRAM read + write per launch of the data-parallel kernels, per element of the
# rank's shard, at 8 ranks: one-GPU ncu capture of the 8 ranks' kernels
# (bench.py --emulate-world 8 --params 50000000: shard 6.25M elements, 8
# launches of each kernel averaged). With every rank's buffers on one GPU, a
# kernel's DRAM bytes are the per-GPU HBM bytes of its multi-GPU launch; the
# writes that are still in L2 when the kernel ends are not in the count.
DP_TRAFFIC_PER_ELEM = {8: {"k_rs_sumsq": (100_074_400 + 1_204_672) / 6_250_000,
                           "k_apply<all-gather>": (87_755_008 + 123_064_736) / 6_250_000}}
# NVLink references of this pool (per direction per GPU): the measured peer
# copy and NVLink 5's specification.
NVLINK_PEER_COPY_GBS = 770.0
NVLINK_SPEC_GBS = 900.0
# B200 HBM3e specification (DGX figure), reported beside the measured copy peak
HBM_SPEC_GBS = 8000.0
L2_FLUSH_BYTES = 256 << 20    # twice the 126 MB L2


def measured_peak_hbm() -> tuple[float, str]:
    try:
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def host_threads() -> int:
    """Every host CPU this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--params", type=int, default=N_PARAMS)
    # 40: the pipeline's fill and drain (the first upload and the last
    # read-back run alone) amortise to ~0.2 ms of a ~9 ms step
    ap.add_argument("--e2e-steps", type=int, default=40)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="leave the configs key out of the N=1 line")
    ap.add_argument("--sweep", action="store_true",
                    help="config 5: flat 1M..2B params in both layouts, one JSON line each "
                         "(not the headline line)")
    ap.add_argument("--sweep-sizes", default="1000000,16000000,256000000,1000000000,2000000000")
    ap.add_argument("--cpu-sample", action="store_true",
                    help="(child process) time the CPU reference on --params params and print "
                         "JSON; threads from OMP_NUM_THREADS")
    ap.add_argument("--configs", action="store_true",
                    help="configs 1-3 and config-5 sizes on one GPU, one JSON line each "
                         "(not the headline line)")
    ap.add_argument("--emulate-world", type=int, default=0,
                    help="run the fused data-parallel kernels of R ranks on ONE GPU (every "
                         "rank's buffers local, ranks in stream order) with --params params: "
                         "the small case an ncu capture of k_rs_sumsq / k_apply<all-gather> "
                         "runs on (not the headline line)")
    ap.add_argument("--dp", default="fused", choices=["fused", "fused-nccl", "nccl"],
                    help="N>1: collectives fused into the kernels over peer memory, the ranks "
                         "synchronised by device-side flags (default) or by small NCCL "
                         "collectives between the launches (fused-nccl); or NCCL "
                         "reduce-scatter / all-gather around the kernels (nccl)")
    return ap.parse_args()


# ------------------------------------------------------------ CPU baseline --

def cpu_reference_sample(n: int, steps: int, warmup: int = 1) -> dict:
    """The reference's clip_grad_norm(1.0) + step() (adamw.cpp:28-117) on n
    fp32 params cut into 25M-element buckets (the unscaled grads and fp32
    master of the mixed workload), OpenMP over OMP_NUM_THREADS threads. Inputs
    come from numpy; nothing of this package is loaded. Returns Gparams/s."""
    import numpy as np

    from oracle import oracle
    threads = int(os.environ.get("OMP_NUM_THREADS", "0")) or host_threads()
    rng = np.random.Generator(np.random.PCG64(4))
    sizes = [min(BUCKET, n - s) for s in range(0, n, BUCKET)]
    ps = [rng.standard_normal(k, dtype=np.float32) * np.float32(0.02) for k in sizes]
    gs = [rng.standard_normal(k, dtype=np.float32) * np.float32(1e-3) for k in sizes]
    if oracle.ref_available():
        opt = oracle.RefAdamW(ps, gs, lr=1e-3, weight_decay=0.01)
        kind = "reference"

        def one():
            opt.clip_grad_norm(1.0)
            opt.step()
    else:
        cfg = oracle.StepConfig(layout=0, max_norm=1.0)
        opt = oracle.PortOptimizer(ps, [0.01] * len(ps), cfg)
        kind = "port"

        def one():
            opt.step(gs)
    for _ in range(warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    dt = time.perf_counter() - t0
    return {"value": n * steps / dt / 1e9, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{steps} steps (after {warmup} warm-up) of clip_grad_norm(1.0)+step() on "
                      f"{n} fp32 params in {len(sizes)} buckets (host arrays; the unscale and "
                      "bf16 cast, which the reference lacks, not timed)",
            "ms_per_step": dt / steps * 1e3, "params": n}


def cpu_child(n: int, steps: int, warmup: int, threads: int, timeout: float = 900) -> dict:
    """cpu_reference_sample in a fresh child process with OMP_NUM_THREADS set
    before any OpenMP runtime starts (a torchrun parent sets it to 1)."""
    env = dict(os.environ, OMP_NUM_THREADS=str(threads))
    r = subprocess.run([sys.executable, str(Path(__file__).resolve()), "--cpu-sample",
                        "--params", str(n), "--steps", str(steps), "--warmup", str(warmup)],
                       env=env, capture_output=True, text=True, timeout=timeout)
    lines = [x for x in r.stdout.splitlines() if x.startswith("{")]
    if r.returncode != 0 or not lines:
        raise RuntimeError(f"CPU reference child failed ({r.returncode}): {r.stderr[-400:]}")
    return json.loads(lines[-1])


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    t0 = time.perf_counter()
    threads = host_threads()
    res = cpu_child(args.params, args.steps, args.warmup, threads)
    line = {"impl": "reference", "metric": METRIC, "value": res["value"], "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config4 on the host: the reference's clip_grad_norm(1.0) + "
                                   "step() over 200M fp32 params in 25M buckets",
                       "params": args.params, "bucket": BUCKET, "same_config": True,
                       "threads": threads},
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
        z = dp.FusedZeroOneAdamW(n, BUCKET, sb.AdamWOptions(lr=1e-3, weight_decay=0.01),
                                 max_grad_norm=1.0,
                                 loss_scaler=sb.LossScalerOptions(init_scale=65536.0),
                                 device=local, init_params=params,
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
    probe = nvlink_probe_rates(torch, world, rank, local, 2 * shard_params) if fused else None
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
    # the step's result read back: each rank's own updated shard of the bf16
    # params (the ranks' shards together are the whole model once; at N = 1
    # the whole model)
    own = [(b.own_start, b.own_size) for b in z.buckets if b.own_size > 0]
    grad_bufs, use_set = [grads], None
    if world == 1:
        # a second gradient buffer registered with the optimizer as gradient
        # set 1: the upload of step s+1 lands there while step s reads set 0
        grads2 = torch.empty_like(grads)
        z.opt.add_grads([grads2[b.start:b.start + b.size] for b in z.buckets])
        grad_bufs, use_set = [grads, grads2], z.opt.use_grads
    elif fused:
        # the same with a second symmetric gradient buffer of the fused step
        z.add_grads()
        grads2 = z.grad_buffers[1]
        grad_bufs, use_set = [z.grad_buffers[0], grads2], z.use_grads
    barrier()
    torch.cuda.synchronize()
    e2e_ms, e2e_copies = e2e_overlapped(torch, z.step, stream, grad_bufs, use_set, params,
                                        g_pin, p_pin, own, args.e2e_steps)
    barrier()
    torch.cuda.synchronize()
    pcie_ms = pcie_floor(torch, stream, grad_bufs[0], g_pin, params, p_pin, own)
    if use_set is not None:
        use_set(0)
        del grad_bufs, grads2
    t = torch.tensor([e2e_ms, pcie_ms], dtype=torch.float64, device=dev)
    if comm:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    e2e_ms, pcie_ms = float(t[0]), float(t[1])

    # ---- parity of one more step: oracle replay on rank 0, identity on all --
    barrier()
    torch.cuda.synchronize()
    parity = parity_check(torch, np, z, world, rank, comm, g_pin, grads, params)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_child(BUCKET, 5, 1, host_threads())
            cpu.pop("ms_per_step", None)
            cpu.pop("params", None)
            one = cpu_child(BUCKET // 5, 3, 1, 1)
            cpu["single_thread"] = {"value": one["value"], "cores": one["cores"],
                                    "sample": one["sample"]}
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"error": str(ex)[:300]}

    if fused:
        z.close()
    del z
    torch.cuda.empty_cache()
    peak, peak_kind = measured_peak_hbm()
    configs = None
    if not args.no_configs and (world == 1 or comm):
        # N = 1: configs 1-3 and config 5; N > 1: config 5 as one replica per
        # GPU (the update has no cross-GPU term without a reduce), max over ranks
        def together():
            torch.cuda.synchronize()
            torch.distributed.barrier(device_ids=[local])

        def reduce_max(x):
            v = torch.tensor([x], dtype=torch.float64, device=dev)
            torch.distributed.all_reduce(v, op=torch.distributed.ReduceOp.MAX)
            return float(v[0])
        names = None if world == 1 else [k for k in config_specs() if k.startswith("c5")]
        try:
            configs = measure_configs(torch, peak, steps=20, names=names,
                                      together=together if comm else None,
                                      reduce_max=reduce_max if comm else None, world=world)
        except Exception as ex:  # reported beside the headline, never a reason to lose it
            configs = {"error": str(ex)[:300]}
    if comm:
        torch.distributed.barrier(device_ids=[local])
        torch.distributed.destroy_process_group()
    if rank != 0:
        return 0
    apply_bytes = BYTES_PER_PARAM * shard_params
    achieved = apply_bytes / (apply_ms_max * 1e-3) / 1e9
    hbm = {"bound": "hbm", "kernel": "k_apply", "achieved": achieved, "peak": peak,
           "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
           "peak_spec": HBM_SPEC_GBS, "frac_spec": achieved / HBM_SPEC_GBS,
           "traffic": APPLY_TRAFFIC_BYTES.get(shard_params),
           "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one k_apply "
                             "launch of this command at N=1" if shard_params in
                             APPLY_TRAFFIC_BYTES else None,
           "algorithmic_bytes_per_launch": apply_bytes, "apply_ms": apply_ms_max}
    per_kernel = None
    if world == 1:
        roofline = hbm
    else:
        roofline, per_kernel = dp_rooflines(world, shard_params, phases, peak)
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
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": {"value": world * n * args.e2e_steps / (e2e_ms * 1e-3) / 1e9, "unit": UNIT,
                "h2d_bytes_per_step": 2 * n, "d2h_bytes_per_step": 2 * shard_params,
                "transfers": "per rank: H2D of its full bf16 gradient from pinned memory, D2H "
                             "of its updated shard of the bf16 params (from a device snapshot); "
                             "two copy streams, so the read-back of step s overlaps the upload "
                             "of step s+1" + (", which lands in a second gradient buffer "
                                              "while step s runs" if world == 1 or fused
                                              else ""),
                "steps": args.e2e_steps, "ms_per_step": e2e_ms / args.e2e_steps,
                "copies": e2e_copies,
                "roofline": {"bound": "pcie", "floor_ms_per_step": pcie_ms,
                             "frac": pcie_ms / (e2e_ms / args.e2e_steps),
                             "floor": "the same H2D and D2H bytes as one step, both directions "
                                      "at once on two copy streams, no step (all ranks at "
                                      "once), max over ranks"}},
        "clocks": clock_info,
        "gpu_launches": launches_per_step * args.steps,
        "phases_ms": phases,
        "parity": parity,
        "final_info": {"step": info.step, "skipped": info.skipped, "loss_scale": info.loss_scale,
                       "grad_norm": info.grad_norm},
    }
    if world > 1:
        line["rooflines"] = per_kernel
        line["composite_roofline"] = composite_roofline(world, n, shard_params,
                                                        ms_max / args.steps, peak)
        line["nvlink_probe"] = probe
    if configs is not None:
        line["configs"] = configs
    print(json.dumps(line), flush=True)
    return 0


def e2e_overlapped(torch, step, stream, grad_bufs, use_set, params, g_pin, p_pin, own,
                   steps) -> tuple[float, dict]:
    """`steps` steps through the public API with host buffers, timed on
    `stream` with CUDA events. Step s uploads the gradient into buffer s mod B
    (B = len(grad_bufs); with B = 2 the optimizer alternates between two
    registered gradient sets, so the upload of step s+1 overlaps step s) on one
    copy stream, once the step that last read that buffer is done; runs the
    step on `stream`; copies the updated params into one of two device
    snapshots (a device-to-device copy), which a second copy stream reads back
    to the host. Both PCIe directions run at once and the step never waits
    for a read-back. Returns (ms for all steps, copy timings)."""
    nb = len(grad_bufs)
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    snaps = [torch.empty_like(params), torch.empty_like(params)]
    ev = lambda timing=False: torch.cuda.Event(enable_timing=timing)
    up, used, done, back = ([ev() for _ in range(steps)] for _ in range(4))
    t_up = [(ev(True), ev(True)) for _ in range(steps)]
    t_back = [(ev(True), ev(True)) for _ in range(steps)]
    e0, e1 = ev(True), ev(True)
    e0.record(stream)
    for s in range(steps):
        b = s % nb
        h2d.wait_event(used[s - nb] if s >= nb else e0)   # buffer b consumed by its last step
        t_up[s][0].record(h2d)
        with torch.cuda.stream(h2d):
            grad_bufs[b].copy_(g_pin, non_blocking=True)
        t_up[s][1].record(h2d)
        up[s].record(h2d)
        stream.wait_event(up[s])
        if use_set is not None:
            use_set(b)
        step()
        used[s].record(stream)
        if s >= 2:
            stream.wait_event(back[s - 2])                # snapshot s % 2 read back
        for lo, sz in own:
            snaps[s % 2][lo:lo + sz].copy_(params[lo:lo + sz])
        done[s].record(stream)
        d2h.wait_event(done[s])
        t_back[s][0].record(d2h)
        with torch.cuda.stream(d2h):
            for lo, sz in own:
                p_pin[lo:lo + sz].copy_(snaps[s % 2][lo:lo + sz], non_blocking=True)
        t_back[s][1].record(d2h)
        back[s].record(d2h)
    stream.wait_event(back[steps - 1])
    e1.record(stream)
    torch.cuda.synchronize()
    h2d_ms = statistics.mean(a.elapsed_time(b) for a, b in t_up)
    d2h_ms = statistics.mean(a.elapsed_time(b) for a, b in t_back)
    gb_up = g_pin.numel() * g_pin.element_size() / 1e9
    gb_back = sum(sz for _, sz in own) * params.element_size() / 1e9
    copies = {"h2d_ms": round(h2d_ms, 3), "d2h_ms": round(d2h_ms, 3),
              "h2d_gbs": round(gb_up / (h2d_ms * 1e-3), 1),
              "d2h_gbs": round(gb_back / (d2h_ms * 1e-3), 1), "grad_buffers": nb}
    del snaps
    return e0.elapsed_time(e1), copies


def pcie_floor(torch, stream, dst, g_pin, src, p_pin, own, reps=3) -> float:
    """The PCIe floor of one end-to-end step: the step's upload (g_pin ->
    dst) and read-back (src's owned slices -> p_pin) on two copy streams at
    once, with no step, `reps` times; ms per repetition on `stream`."""
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    h2d.wait_event(e0)
    d2h.wait_event(e0)
    for _ in range(reps):
        with torch.cuda.stream(h2d):
            dst.copy_(g_pin, non_blocking=True)
        with torch.cuda.stream(d2h):
            for lo, sz in own:
                p_pin[lo:lo + sz].copy_(src[lo:lo + sz], non_blocking=True)
    for s in (h2d, d2h):
        done = torch.cuda.Event()
        done.record(s)
        stream.wait_event(done)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def parity_check(torch, np, z, world, rank, comm, g_pin, grads, params) -> dict:
    """One more step after the timed work, checked three ways (every rank runs
    the same collectives):
      params_identical  a checksum of every rank's full bf16 parameter buffer
                        agrees across ranks;
      counters_equal    (step, skipped, loss scale, growth tracker, norm bits)
                        agree across ranks and with the oracle;
      sampled replay    the oracle (oracle/, the port of the reference's
                        src/optim/adamw.cpp:28-117 plus the loss scaler)
                        replays the step on ~65536 seeded elements of rank 0's
                        shard from its state before the step and the averaged
                        gradient the step consumed; master/m/v and the bf16
                        params are compared with the device.
    The reduce is compared with the oracle's rank-ordered reduce of the R raw
    gradients on the same sample, and the device's global norm with an fp64
    norm of the averaged gradients computed independently with torch."""
    import torch.distributed as tdist

    from oracle import oracle
    from soar_b200.dp import plan_buckets
    dev = grads.device
    out = {"sample": 0, "checked_rank": 0}
    try:
        # rank 0's tensors (its owned slices, in bucket order) and a seeded sample
        b0 = [b for b in plan_buckets(z.n, BUCKET, world, 0) if b.own_size > 0]
        rng = np.random.Generator(np.random.PCG64(20260))
        per = max(1, 65536 // max(1, len(b0)))
        picks = []  # (k-th tensor of rank 0, offset)
        for k, b in enumerate(b0):
            offs = np.unique(np.concatenate([rng.integers(0, b.own_size, per),
                                             [0, b.own_size - 1]]))
            picks.extend((k, int(o)) for o in offs)
        flat = torch.tensor([b0[k].own_start + o for k, o in picks], dtype=torch.int64,
                            device=dev)
        out["sample"] = len(picks)
        by_t = {}
        for k, o in picks:
            by_t.setdefault(k, []).append(o)

        def sample_state(kind):
            nz = [i for i, sg in enumerate(z.shard_grads) if sg.numel() > 0]
            return np.concatenate([z.opt.state(nz[k], kind)[torch.tensor(by_t[k], device=dev)]
                                   .cpu().numpy() for k in sorted(by_t)])

        # fresh raw gradients on every rank, and their values on rank 0's sample
        grads.copy_(g_pin)
        torch.cuda.synchronize()
        raw = grads.view(torch.int16)[flat].contiguous()
        raws = [raw]
        if world > 1:  # moved as bf16 (the same bytes: NCCL has no int16)
            got = [torch.empty_like(raw).view(torch.bfloat16) for _ in range(world)]
            tdist.all_gather(got, raw.view(torch.bfloat16))
            raws = [r.view(torch.int16) for r in got]
        info_b = z.opt.info()
        if rank == 0:
            st = {key: sample_state(kind) for kind, key in ((0, "master"), (1, "m"), (2, "v"))}
            p_before = params.view(torch.int16)[flat].cpu().numpy().view(np.uint16)
        torch.cuda.synchronize()
        if comm:
            tdist.barrier()
        z.step()
        torch.cuda.synchronize()
        info = z.opt.info()
        # the averaged gradient the step consumed (in place in the own slices
        # for the fused reduce-scatter, the shard buffer for NCCL): an
        # independent fp64 norm over every rank's shard
        ss = torch.zeros(1, dtype=torch.float64, device=dev)
        for sg in z.shard_grads:
            if sg.numel():
                ss += ((sg.to(torch.float64) / info_b.loss_scale) ** 2).sum()
        if world > 1:
            tdist.all_reduce(ss)
        norm64 = float(torch.sqrt(ss)[0])
        out["norm_rel_err_vs_fp64"] = abs(info.grad_norm - norm64) / max(norm64, 1e-30)
        # identity across ranks
        w = params.view(torch.int32).to(torch.int64)
        pos = torch.arange(w.numel(), device=dev, dtype=torch.int64) % 65521 + 1
        cks = torch.stack([w.sum(), ((w & 0xFFFFFFFF) * pos).sum()])
        del w, pos
        bits = lambda x: int(np.float32(x).view(np.int32))
        cnt = torch.tensor([info.step, info.skipped, bits(info.loss_scale), info.growth_tracker,
                            bits(info.grad_norm)], dtype=torch.int64, device=dev)
        all_cks, all_cnt = [cks], [cnt]
        if world > 1:
            all_cks = [torch.empty_like(cks) for _ in range(world)]
            all_cnt = [torch.empty_like(cnt) for _ in range(world)]
            tdist.all_gather(all_cks, cks)
            tdist.all_gather(all_cnt, cnt)
        out["params_identical"] = all(bool(torch.equal(c, all_cks[0])) for c in all_cks)
        counters_same = all(bool(torch.equal(c, all_cnt[0])) for c in all_cnt)
        if rank != 0:
            return out
        nz = [i for i, sg in enumerate(z.shard_grads) if sg.numel() > 0]
        avg = np.concatenate([z.shard_grads[nz[k]][torch.tensor(by_t[k], device=dev)]
                              .view(torch.int16).cpu().numpy().view(np.uint16)
                              for k in sorted(by_t)])
        raw_np = [r.cpu().numpy().view(np.uint16) for r in raws]
        red = oracle.reduce_avg_bf16(raw_np) if world > 1 else raw_np[0]
        out["reduce_bit_exact"] = bool(np.array_equal(red, avg))
        out["reduce_max_ulp"] = int(np.abs(red.astype(np.int32) - avg.astype(np.int32)).max())
        # the oracle's step on the sample, from the device's state before it
        cfg = oracle.StepConfig(layout=1, lr=1e-3, max_norm=1.0, use_scaler=True)
        ps = oracle.PortShard([p_before.copy()], [avg.copy()], [0.01], cfg,
                              init_scale=info_b.loss_scale)
        ps.master[0][:] = st["master"]
        ps.m[0][:] = st["m"]
        ps.v[0][:] = st["v"]
        ps.state.t, ps.state.skipped = info_b.step, info_b.skipped
        ps.state.tracker = info_b.growth_tracker
        norm = np.float64(np.float32(info.grad_norm))
        ps.apply_sumsq(float(norm * norm))  # the square of a float is exact: same fp32 norm
        got_p = params.view(torch.int16)[flat].cpu().numpy().view(np.uint16)
        got = {key: sample_state(kind) for kind, key in ((0, "master"), (1, "m"), (2, "v"))}
        want = {"master": ps.master[0], "m": ps.m[0], "v": ps.v[0]}
        rel, exact = 0.0, True
        for k in want:
            a, b = got[k].astype(np.float64), want[k].astype(np.float64)
            rel = max(rel, float(np.max(np.abs(a - b) / np.maximum(np.abs(b), 1e-30))))
            exact = exact and bool(np.array_equal(got[k].view(np.uint32),
                                                  want[k].view(np.uint32)))
        out["max_ulp"] = int(np.abs(got_p.astype(np.int32) - ps.params[0].astype(np.int32)).max())
        out["state_max_rel_err"] = rel
        out["state_bit_exact"] = exact
        oc = (ps.state.t, ps.state.skipped, float(ps.state.scale), ps.state.tracker)
        dc = (info.step, info.skipped, float(info.loss_scale), info.growth_tracker)
        out["counters_equal"] = counters_same and oc == dc
        out["tolerance"] = "bf16 params <= 1 ulp; fp32 state max rel err <= 1e-6"
        out["pass"] = bool(out["params_identical"] and out["counters_equal"] and
                           out["max_ulp"] <= 1 and rel <= 1e-6 and
                           out["norm_rel_err_vs_fp64"] <= 1e-6)
    except Exception as ex:  # reported, never a reason to lose the bench line
        out["error"] = f"{type(ex).__name__}: {str(ex)[:300]}"
    return out


def composite_roofline(world, n, shard_params, step_ms, hbm_peak) -> dict:
    """The whole data-parallel step against the sum of its two phases' floors
    (the phases cannot overlap: the global norm decides the clip between them).
    Each phase's floor is its binding resource, as in dp_rooflines:
      reduce-scatter  max((R+1) x shard x 2 B / HBM, (R-1) x shard x 2 B / NVLink)
      update + AG     max((28 x shard + (R-1) x shard x 2 B) / HBM,
                          (R-1) x shard x 2 B / NVLink)
    with NVLink bytes per rank and direction. `additive` is the sum of the
    shard update at the HBM peak and both collectives at the NVLink peak: no
    lower bound here, since the fused kernels overlap the two (at 2 GPUs the
    step runs below it). Measured peaks (HBM copy, peer copy) and the
    specifications (8 TB/s HBM, 900 GB/s NVLink per direction)."""
    nvl = (world - 1) * shard_params * 2
    upd = BYTES_PER_PARAM * shard_params

    def floors(hbm, link):
        rs = max((world + 1) * shard_params * 2 / hbm, nvl / link)
        ag = max((upd + nvl) / hbm, nvl / link)
        return (rs + ag) * 1e3 / 1e9, (upd / hbm + 2 * nvl / link) * 1e3 / 1e9

    f, add = floors(hbm_peak, NVLINK_PEER_COPY_GBS)
    fs, adds = floors(HBM_SPEC_GBS, NVLINK_SPEC_GBS)
    return {"floor": "per phase, the slower of HBM and NVLink; summed over reduce-scatter and "
                     "update + all-gather",
            "params": n, "floor_ms": round(f, 4), "frac": f / step_ms,
            "floor_ms_spec": round(fs, 4), "frac_spec": fs / step_ms,
            "peaks": {"hbm": hbm_peak, "nvlink": NVLINK_PEER_COPY_GBS},
            "peaks_spec": {"hbm": HBM_SPEC_GBS, "nvlink": NVLINK_SPEC_GBS},
            "additive": {"formula": "28 B x N/R / HBM + 2 x (R-1)/R x 2 B x N / NVLink",
                         "ms": round(add, 4), "ms_spec": round(adds, 4)}}


def dp_rooflines(world, shard_params, phases, hbm_peak) -> tuple[dict, dict]:
    """Rooflines of the data-parallel step's two kernels at N > 1, each against
    its own binding resource (the larger of its two floors), from phases_ms:
      k_rs_sumsq            NVLink: it pulls (R-1) x shard x 2 B from the peers
                            while they pull as much from this GPU; HBM: own
                            shard read + average written + the peers' pulls
                            served, (R+1) x shard x 2 B;
      k_apply<all-gather>   NVLink: it pushes (R-1) x shard x 2 B into the
                            peers and receives as much; HBM: the 28 B/param
                            update of the shard + the peers' pushes landing
                            here, 28 x shard + (R-1) x shard x 2 B.
    NVLink peak: the pool's measured peer copy, 770 GB/s per direction (spec
    900); HBM peak: the measured copy. Returns (the slower kernel's roofline,
    both)."""
    nvl = (world - 1) * shard_params * 2
    fused = "update+allgather" in phases
    if fused:
        times = {"k_rs_sumsq": phases["reduce_scatter+sumsq"],
                 "k_apply<all-gather>": phases["update+allgather"]}
    else:  # NCCL collectives around the kernels: time the update phase with them
        times = {"k_rs_sumsq": phases["reduce_scatter"],
                 "k_apply<all-gather>": phases["update"] + phases["param_allgather"]}
    hbm_bytes = {"k_rs_sumsq": (world + 1) * shard_params * 2,
                 "k_apply<all-gather>": BYTES_PER_PARAM * shard_params + nvl}
    out = {}
    for k, ms in times.items():
        floors = {"nvlink": nvl / (NVLINK_PEER_COPY_GBS * 1e9),
                  "hbm": hbm_bytes[k] / (hbm_peak * 1e9)}
        bound = max(floors, key=floors.get)
        nbytes = nvl if bound == "nvlink" else hbm_bytes[k]
        peak = NVLINK_PEER_COPY_GBS if bound == "nvlink" else hbm_peak
        achieved = nbytes / (ms * 1e-3) / 1e9
        out[k] = {"bound": bound, "kernel": k, "achieved": achieved, "peak": peak,
                  "peak_kind": "measured peer copy of this pool, per direction per GPU"
                               if bound == "nvlink" else "measured HBM copy",
                  "unit": "GB/s" + (" per direction per rank" if bound == "nvlink" else ""),
                  "frac": achieved / peak, "bytes_per_launch": nbytes,
                  "nvlink_bytes_per_direction": nvl, "hbm_bytes": hbm_bytes[k], "ms": ms,
                  "floor_ms": {b: round(f * 1e3, 4) for b, f in floors.items()}}
        per = DP_TRAFFIC_PER_ELEM.get(world, {}).get(k)
        out[k]["traffic"] = round(per * shard_params) if per and fused else None
        if out[k]["traffic"] is not None:
            out[k]["traffic_source"] = ("HBM bytes per launch: one-GPU ncu capture of the "
                                        f"{world} ranks' kernels (--emulate-world {world}, "
                                        "shard 6.25M), scaled to this shard; compare hbm_bytes")
        spec = NVLINK_SPEC_GBS if bound == "nvlink" else HBM_SPEC_GBS
        out[k]["peak_spec"] = spec
        out[k]["frac_spec"] = achieved / spec
        if not fused:
            out[k]["kernel"] += " (NCCL around it)"
    dominant = max(out.values(), key=lambda r: r["ms"])
    return dominant, out


def nvlink_probe_rates(torch, world, rank, local, shard_bytes) -> dict:
    """Raw rates of the fused kernels' two peer access patterns on this box
    (the bench-only probe library: all ranks at once, no arithmetic, the same
    bytes per peer as the step). GB/s per direction per rank; max time over
    ranks. A failure on any rank is agreed on by every rank before the next
    collective, so the ranks never run different collectives, and the buffers
    are released whatever happens."""
    import ctypes as C

    import torch.distributed as dist

    from soar_b200 import optim as _o
    lib = _o.lib()
    tile_lcm = 64 * 1024
    bpp = max(tile_lcm, shard_bytes // tile_lcm * tile_lcm)
    dev = f"cuda:{local}"
    err = None

    def agree(ok: bool) -> bool:
        f = torch.tensor([0 if ok else 1], dtype=torch.int32, device=dev)
        dist.all_reduce(f, op=dist.ReduceOp.MAX)
        return int(f.item()) == 0

    ptr = C.c_void_p()
    handle = (C.c_ubyte * _o.IPC_HANDLE_BYTES)()
    opened = []
    allocated = False
    try:
        probe = None
        try:
            probe = _o.probe_lib()
            _o._check(lib.soar_ipc_alloc(world * bpp, local, C.byref(ptr), handle),
                      "soar_ipc_alloc")
            allocated = True
            ok = True
        except Exception as ex:
            err, ok = str(ex)[:200], False
        if not agree(ok):
            return {"error": err or "failed on another rank"}
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle))
        bases = []
        try:
            for q, h in enumerate(handles):
                if q == rank:
                    bases.append(ptr.value)
                    continue
                peer = C.c_void_p()
                buf = (C.c_ubyte * _o.IPC_HANDLE_BYTES).from_buffer_copy(h)
                _o._check(lib.soar_ipc_open(buf, local, C.byref(peer)), "soar_ipc_open")
                bases.append(peer.value)
                opened.append(peer.value)
            ok = True
        except Exception as ex:
            err, ok = str(ex)[:200], False
        if not agree(ok):
            return {"error": err or "failed on another rank"}
        arr = (C.c_void_p * world)(*bases)
        d_err = torch.zeros(1, dtype=torch.int32, device=dev)
        stream = torch.cuda.current_stream()
        sms = torch.cuda.get_device_properties(local).multi_processor_count
        failed = [False]

        def launch(mode, tile, stages, grid):
            if failed[0]:
                return  # the collectives below still run: every rank takes the same steps
            rc = probe.soar_nvlink_probe(arr, world, rank, bpp, mode, tile, stages, grid,
                                         C.c_void_p(d_err.data_ptr()),
                                         C.c_void_p(stream.cuda_stream))
            failed[0] = rc != 0

        def timed(mode, tile, stages, grid, reps=5):
            for _ in range(2):
                launch(mode, tile, stages, grid)
            torch.cuda.synchronize()
            dist.barrier(device_ids=[local])
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(reps):
                launch(mode, tile, stages, grid)
            b.record(stream)
            torch.cuda.synchronize()
            t = torch.tensor([a.elapsed_time(b) / reps], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return round((world - 1) * bpp / (float(t[0]) * 1e-3) / 1e9, 1)

        pull = {f"tile{tile}_stages{st}_grid{g}": timed(0, tile, st, g)
                for tile, st, g in ((4096, 4, sms), (2048, 8, 2 * sms))
                if st * tile * (world - 1) <= 200 * 1024}
        push = {f"tile{tile}_grid{g}": timed(1, tile, 0, g)
                for tile, g in ((2048, 2 * sms), (8192, sms))}
        torch.cuda.synchronize()
        if not agree(not failed[0] and int(d_err.item()) == 0):
            return {"error": "a probe launch failed or a wait timed out on some rank"}
        return {"unit": "GB/s per direction per rank, all ranks at once",
                "bytes_per_peer": bpp, "pull": pull, "push": push}
    finally:
        torch.cuda.synchronize()
        for pp in opened:
            lib.soar_ipc_close(C.c_void_p(pp), local)
        dist.barrier(device_ids=[local])  # no rank frees while a peer still maps it
        if allocated:
            lib.soar_ipc_free(ptr, local)


# ----------------------------------------------------------- configs 1-3, 5 --

def config_specs(sizes5=(1_000_000, 16_000_000, 256_000_000)):
    """BASELINE configs at their own shapes:
      c1  1 fp32 tensor of 1,048,576 params, no clip/scaler, wd 0.01;
      c2  the 240-tensor segmentation-net list (~12M fp32), wd 0.05 on conv
          weights / 0 on norms and biases, cosine 1e-3 -> 1e-5 over 100 steps
          (the scheduler steps after every step, on the host);
      c3  400 bf16-mixed tensors summing to 50M, clip 1.0, loss scaler 65536;
      c5  one flat tensor of N params in both layouts, plain update."""
    import math

    from soar_b200 import synth
    c2_shapes = synth.config2_shapes()
    specs = {
        "c1": dict(sizes=[1_048_576], wd=[0.01], layout="fp32", clip=0.0, scaler=False,
                   cosine=None),
        "c2": dict(sizes=[int(math.prod(sh)) for _, sh in c2_shapes],
                   wd=[0.05 if k in ("dw", "pw") else 0.0 for k, _ in c2_shapes],
                   layout="fp32", clip=0.0, scaler=False, cosine=(100, 1e-5, 0)),
        "c3": dict(sizes=synth.config3_sizes(), wd=None, layout="bf16_mixed", clip=1.0,
                   scaler=True, cosine=None),
    }
    for n in sizes5:
        for lay, tag in (("fp32", "fp32"), ("bf16_mixed", "mixed")):
            specs[f"c5_{tag}_{n // 1_000_000}M"] = dict(sizes=[n], wd=[0.01], layout=lay,
                                                        clip=0.0, scaler=False, cosine=None)
    return specs


def measure_configs(torch, peak: float, steps: int = 20, names=None, together=None,
                    reduce_max=None, world: int = 1) -> dict:
    """Each config, two ways, 3 warm-up steps first:
      us_per_step  steps back to back over R independent copies of the config,
                   stepped in turn, with R chosen so the copies' resident state
                   together exceeds 3x the 126 MB L2: every step finds its own
                   data evicted by the R-1 steps before it (inputs larger than
                   L2), as in training, where the forward and backward passes
                   run between two optimizer steps; CUDA events around all
                   `steps` x R steps;
      isolated_us  one step timed alone (CUDA events) after an L2 flush (a
                   256 MB write followed by a 256 MB read, so the lines left in
                   L2 are clean and the step is not charged for the flush's
                   write-backs): the latency of a single cold step, launch
                   included.
    Inputs are device-generated; the numerics of these configs are pinned by
    the parity tests. Under torchrun every rank measures its own replica
    (`together` starts the ranks' timed regions together, `reduce_max` takes
    the slowest rank's time) and Gparams/s counts all `world` replicas.
    Returns {name: figures}."""
    import soar_b200 as sb
    specs = config_specs()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    sink = torch.empty(1, dtype=torch.float32, device="cuda")
    out = {}
    for name, c in specs.items():
        if names and name not in names:
            continue
        n = sum(c["sizes"])
        dt = torch.bfloat16 if c["layout"] == "bf16_mixed" else torch.float32
        resident = n * 16                                   # param, grad, master/m/v
        reps = max(1, -(-3 * 126_000_000 // resident))
        copies = []
        for _ in range(reps):
            ps = [(torch.randn(k, device="cuda") * 0.02).to(dt) for k in c["sizes"]]
            gs = [(torch.randn(k, device="cuda") * (1e-3 * (65536.0 if c["scaler"] else 1.0)))
                  .to(dt) for k in c["sizes"]]
            wds = c["wd"] or [0.01] * len(ps)
            opt = sb.AdamW([sb.ParamGroup([p], w) for p, w in zip(ps, wds)],
                           sb.AdamWOptions(lr=1e-3), layout=c["layout"],
                           max_grad_norm=c["clip"],
                           loss_scaler=sb.LossScalerOptions(init_scale=65536.0) if c["scaler"]
                           else None, grads=gs)
            sched = sb.CosineAnnealingLR(opt, *c["cosine"]) if c["cosine"] else None
            copies.append((ps, gs, opt, sched))
        s = torch.cuda.Stream()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        iso = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(10)]
        with torch.cuda.stream(s):
            for _ in range(3):
                for _, _, opt, _ in copies:
                    opt.step(s)
            torch.cuda.synchronize()
            if together is not None:
                together()
            a.record(s)
            for _ in range(steps):
                for _, _, opt, sched in copies:
                    opt.step(s)
                    if sched:
                        sched.step()
            b.record(s)
            opt0 = copies[0][2]
            for e0, e1 in iso:
                flush.fill_(1.0)
                torch.sum(flush, 0, out=sink)
                e0.record(s)
                opt0.step(s)
                e1.record(s)
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / (steps * reps)
        iso_us = [e0.elapsed_time(e1) * 1e3 for e0, e1 in iso]
        if reduce_max is not None:
            us = reduce_max(us)
        gbs = BYTES_PER_PARAM * n / (us * 1e-6) / 1e9
        info = opt0.info()
        out[name] = {"params": n, "tensors": len(c["sizes"]), "layout": c["layout"],
                     "kernel": opt0.kernel_path, "copies": reps,
                     "us_per_step": round(us, 2),
                     "gparams_s": round(world * n / (us * 1e-6) / 1e9, 2),
                     "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 3),
                     "isolated_us": round(statistics.median(iso_us), 2),
                     "isolated_frac": round(BYTES_PER_PARAM * n / (statistics.median(iso_us)
                                                                   * 1e-6) / 1e9 / peak, 3),
                     "steps": steps, "final_step": info.step, "skipped": info.skipped}
        for _, _, opt, sched in copies:
            if sched:
                sched.close()
            opt.close()
        del copies
        torch.cuda.empty_cache()
    out["_how"] = ("us_per_step: steps back to back over `copies` independent copies of the "
                   "config stepped in turn (together > 3x L2, so each step's data is cold); "
                   "isolated_us: median of one step timed alone after an L2 flush (256 MB "
                   f"write + 256 MB read); frac of the measured {peak:.0f} GB/s HBM copy at "
                   "28 B/param")
    return out


def run_configs(args):
    """BASELINE configs 1-3 and the config-5 sizes on one GPU, one JSON line
    each (see measure_configs)."""
    import torch
    torch.cuda.set_device(0)
    peak, peak_kind = measured_peak_hbm()
    res = measure_configs(torch, peak, steps=args.steps)
    how = res.pop("_how")
    for name, r in res.items():
        print(json.dumps({"config": name, "metric": "AdamW Gparams/s (BASELINE configs)",
                          "peak_kind": peak_kind, "how": how, **r}), flush=True)
    return 0


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


def run_emulated_world(args):
    """The fused ZeRO-1 kernels of R ranks on one GPU: every rank's flat bf16
    gradient and parameter buffers and shard optimizer on this device, the
    caller-synchronised entry points in stream order (rank 0..R-1
    reduce-scatter + norm, then rank 0..R-1 update + all-gather), config 4's
    hyperparameters. Each kernel moves through HBM exactly the bytes its
    multi-GPU launch moves through NVLink plus local HBM, so a one-GPU ncu
    capture gives the per-launch traffic of the multi-GPU kernels. Prints one
    JSON line with the mean duration of each kernel over `--steps` steps."""
    import ctypes as C

    import torch

    import soar_b200 as sb
    from soar_b200 import dp
    from soar_b200 import optim as _o
    world, n = args.emulate_world, args.params
    torch.cuda.set_device(0)
    lib = _o.lib()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(404)
    p0 = (torch.randn(n, device="cuda", generator=gen) * 0.02).bfloat16()
    grads = [(torch.randn(n, device="cuda", generator=gen) * (1e-3 * 65536.0)).bfloat16()
             for _ in range(world)]
    params = [p0.clone() for _ in range(world)]
    gb = (C.c_void_p * world)(*[g.data_ptr() for g in grads])
    pb = (C.c_void_p * world)(*[p.data_ptr() for p in params])
    opts, handles = [], []
    for r in range(world):
        plan = [b for b in dp.plan_buckets(n, BUCKET, world, r) if b.own_size > 0]
        opt = sb.AdamW([sb.ParamGroup([params[r][b.own_start:b.own_start + b.own_size]
                                       for b in plan], 0.01)], sb.AdamWOptions(lr=1e-3),
                       layout="bf16_mixed", max_grad_norm=1.0,
                       loss_scaler=sb.LossScalerOptions(init_scale=65536.0),
                       grads=[grads[r][b.own_start:b.own_start + b.own_size] for b in plan])
        shards = (_o.Zero1Shard * max(1, len(plan)))()
        for i, b in enumerate(plan):
            shards[i].offset, shards[i].count, shards[i].tensor = b.own_start, b.own_size, i
        h = C.c_void_p()
        _o._check(lib.soar_zero1_create(opt.handle, r, world, gb, pb, shards, len(plan),
                                        C.byref(h)), "soar_zero1_create")
        opts.append(opt)
        handles.append(h)
    part = torch.zeros(world, dtype=torch.float64, device="cuda")
    s = torch.cuda.current_stream()
    ev = lambda: torch.cuda.Event(enable_timing=True)
    rs_ms, ag_ms = [], []
    for k in range(args.warmup + args.steps):
        marks = [ev() for _ in range(2 * world + 1)]
        marks[0].record(s)
        for r in range(world):
            _o._check(lib.soar_zero1_reduce_sumsq(handles[r], C.c_void_p(part.data_ptr() + 8 * r),
                                                  C.c_void_p(s.cuda_stream)), "reduce")
            marks[1 + r].record(s)
        for r in range(world):
            _o._check(lib.soar_zero1_apply_allgather(handles[r], C.c_void_p(part.data_ptr()),
                                                     world, C.c_void_p(s.cuda_stream)), "update")
            marks[1 + world + r].record(s)
        torch.cuda.synchronize()
        if k >= args.warmup:
            rs_ms += [marks[r].elapsed_time(marks[r + 1]) for r in range(world)]
            ag_ms += [marks[world + r].elapsed_time(marks[world + r + 1]) for r in range(world)]
    shard = n // world
    print(json.dumps({"emulated_world": world, "params": n, "bucket": BUCKET,
                      "shard_params": shard, "steps": args.steps,
                      "k_rs_sumsq_ms": statistics.mean(rs_ms),
                      "k_apply_allgather_ms": statistics.mean(ag_ms),
                      "rs_bytes_per_launch": world * shard * 2 + shard * 2,
                      "ag_bytes_per_launch": BYTES_PER_PARAM * shard + (world - 1) * shard * 2,
                      "info": opts[0].info().as_dict()}), flush=True)
    for h in handles:
        lib.soar_zero1_destroy(h)
    for o in opts:
        o.close()
    return 0


def main():
    args = parse()
    if args.cpu_sample:
        res = cpu_reference_sample(args.params, args.steps, args.warmup)
        print(json.dumps(res), flush=True)
        return 0
    if args.impl == "reference":
        return run_reference(args)
    if args.sweep:
        return run_sweep(args)
    if args.configs:
        return run_configs(args)
    if args.emulate_world:
        return run_emulated_world(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
