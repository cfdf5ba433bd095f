"""Host-side pieces of bench.py that need no GPU: the clock summary taken
during the timed region (NVML samples and the nvidia-smi fallback) and the
CPU reference sample used by the baseline rows."""
import io
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_clock_summary_uses_only_samples_inside_the_timed_region():
    cs = bench.ClockSampler([0, 1])
    cs.thread = type("T", (), {"join": lambda self, t=None: None})()  # no real thread
    cs.max_mhz = [1965, 1965]
    # idle before, loaded inside [10, 11], a throttle reason only outside
    cs.samples = [(9.0, 0, 600.0, []), (9.0, 1, 600.0, ["sw_power_cap"]),
                  (10.1, 0, 1965.0, []), (10.1, 1, 1950.0, ["sw_power_cap"]),
                  (10.6, 0, 1965.0, []), (10.6, 1, 1965.0, []),
                  (12.0, 0, 700.0, ["hw_slowdown"])]
    cs.window = [10.0, 11.0]
    out = cs.stop()
    assert out["samples"] == 4
    assert out["sm_mhz"] == 1965.0
    assert out["sm_max_mhz"] == 1965
    assert out["reasons"] == ["sw_power_cap"]
    assert out["source"] == "nvml"


def test_clock_summary_falls_back_to_the_nearest_sample_after_a_short_region():
    cs = bench.ClockSampler([0])
    cs.thread = type("T", (), {"join": lambda self, t=None: None})()
    cs.max_mhz = [1965]
    cs.samples = [(1.0, 0, 500.0, []), (2.02, 0, 1965.0, []), (3.0, 0, 1800.0, [])]
    cs.window = [2.0, 2.01]  # shorter than the sampling period, nothing inside
    out = cs.stop()
    assert out["samples"] == 1 and out["sm_mhz"] == 1965.0


def test_clock_summary_parses_the_nvidia_smi_fallback(tmp_path):
    cs = bench.ClockSampler([0, 1])
    cs.fh = io.StringIO("0, 1965, 1965, Not Active, Not Active, Not Active, Active\n"
                        "1, 1900, 1965, Active, Not Active, Not Active, Not Active\n"
                        "2, 100, 1965, Active, Active, Active, Active\n"   # not our GPU
                        "garbage line\n")

    class P:
        def terminate(self):
            pass

        def wait(self, t=None):
            return 0
    cs.proc = P()
    out = cs.stop()
    assert out["samples"] == 2
    assert out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["hw_slowdown", "sw_power_cap"]
    assert out["source"] == "nvidia-smi"


def test_cpu_reference_sample_reports_the_reference_kind_and_threads():
    res = bench.cpu_reference_sample(200_000, 2, warmup=1)
    assert res["value"] > 0 and res["unit"] == bench.UNIT
    assert res["kind"] in ("reference", "port") and res["cores"] >= 1


def test_cpu_sample_child_runs_on_one_thread():
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--cpu-sample", "--params",
                        "100000", "--steps", "2"], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads([x for x in r.stdout.splitlines() if x.startswith("{")][-1])
    assert d["cores"] == 1 and d["value"] > 0


def test_reference_arm_uses_every_host_thread_under_torchrun_settings():
    """torchrun sets OMP_NUM_THREADS=1; the reference arm still times the
    reference on every host CPU (the child gets its own OMP_NUM_THREADS), on
    the config's own workload, and the line says so."""
    env = dict(os.environ, OMP_NUM_THREADS="1", RANK="0", WORLD_SIZE="2")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                        "--params", "300000", "--steps", "2", "--warmup", "1", "--gpus", "2"],
                       env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads([x for x in r.stdout.splitlines() if x.startswith("{")][-1])
    assert d["impl"] == "reference" and d["config"]["same_config"] is True
    assert d["cpu_baseline"]["cores"] == bench.host_threads() == d["config"]["threads"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["value"] == d["e2e"]["value"]


def test_reference_arm_other_ranks_exit_without_work():
    env = dict(os.environ, RANK="3", WORLD_SIZE="4")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference"],
                       env=env, capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and not r.stdout.strip()


def test_reference_sample_loads_nothing_of_the_package():
    """The reference's timing process maps only oracle libraries: no library
    of this package (the input generator included)."""
    code = ("import sys; sys.path.insert(0, %r); import bench; "
            "bench.cpu_reference_sample(100000, 1); "
            "print('\\n'.join(l for l in open('/proc/self/maps').read().splitlines() "
            "if '.so' in l))" % str(ROOT))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    ours = [l for l in r.stdout.splitlines() if str(ROOT) in l]
    assert ours and all("/oracle/" in l for l in ours), ours
    assert "soar_b200" not in r.stdout and "soar.cpp_b200" not in r.stdout


def test_dp_rooflines_are_recomputable_from_the_phases():
    phases = {"barrier": 0.01, "reduce_scatter+sumsq": 0.55, "partial_allgather": 0.02,
              "update+allgather": 0.57, "barrier2": 0.01}
    shard = 25_000_000
    dom, both = bench.dp_rooflines(8, shard, phases, 6552.0)
    nvl = 7 * shard * 2
    rs, ag = both["k_rs_sumsq"], both["k_apply<all-gather>"]
    assert rs["bound"] == ag["bound"] == "nvlink" and dom is ag   # 8 GPUs: NVLink-bound
    assert abs(rs["achieved"] - nvl / 0.55e-3 / 1e9) < 1e-6
    assert abs(ag["frac"] - ag["achieved"] / bench.NVLINK_PEER_COPY_GBS) < 1e-12
    assert abs(ag["frac_spec"] - ag["achieved"] / bench.NVLINK_SPEC_GBS) < 1e-12
    # 2 GPUs: the update of a 100M shard is HBM-bound (28 B x 100M + 200 MB received)
    phases2 = {"barrier": 0.016, "reduce_scatter+sumsq": 0.327, "partial_allgather": 0.014,
               "update+allgather": 0.512, "barrier2": 0.019}
    dom2, both2 = bench.dp_rooflines(2, 100_000_000, phases2, 6552.0)
    assert both2["k_rs_sumsq"]["bound"] == "nvlink"
    assert dom2["bound"] == "hbm" and dom2["kernel"] == "k_apply<all-gather>"
    assert dom2["bytes_per_launch"] == 28 * 100_000_000 + 200_000_000
    assert abs(dom2["frac_spec"] - dom2["achieved"] / bench.HBM_SPEC_GBS) < 1e-12


def test_composite_roofline_is_a_lower_bound_of_the_phases():
    # 8 GPUs: both phases NVLink-bound, so the floor is 2 x 350 MB at the link rate
    c = bench.composite_roofline(8, 200_000_000, 25_000_000, 1.153, 6552.0)
    assert abs(c["floor_ms"] - 2 * 350e6 / (bench.NVLINK_PEER_COPY_GBS * 1e9) * 1e3) < 1e-3
    assert abs(c["frac"] - c["floor_ms"] / 1.153) < 1e-3
    assert c["floor_ms"] <= c["additive"]["ms"] and c["floor_ms_spec"] < c["floor_ms"]
    # 2 GPUs: the update phase is HBM-bound; the per-phase floor stays below the
    # measured step where the additive form (no overlap) would exceed it
    c2 = bench.composite_roofline(2, 200_000_000, 100_000_000, 0.834, 6552.0)
    rs = 200e6 / (bench.NVLINK_PEER_COPY_GBS * 1e9)
    ag = (28 * 100e6 + 200e6) / (6552.0 * 1e9)
    assert abs(c2["floor_ms"] - (rs + ag) * 1e3) < 1e-3
    assert c2["frac"] < 1.0 < c2["additive"]["ms"] / 0.834
