"""The C++ API (include/soar_optim.hpp): compiles with g++ as C++17 and C++20
(CPU); on the GPU the reference's optimizer tests ported to it pass, a
Trainer-shaped driver runs clip -> step -> zero_grad without host
synchronisation, and the data-parallel bootstrap runs the fused ZeRO-1 step
from C++ in two processes on two GPUs."""
import subprocess
from pathlib import Path

import pytest

from soar_b200 import _build

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "cpp" / "test_optimizers_gpu.cpp"
TRAINER = ROOT / "tests" / "cpp" / "test_trainer_gpu.cpp"
DP = ROOT / "tests" / "cpp" / "test_dp_gpu.cpp"
CUDA = Path("/usr/local/cuda")


def _compile(out: Path, std: str, src: Path = SRC) -> None:
    lib = _build.build()
    cxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"
    subprocess.run([cxx, f"-std={std}", "-O2", "-Wall", "-Wextra", "-I", str(ROOT / "include"),
                    "-I", str(CUDA / "include"), str(src), "-o", str(out),
                    str(lib), f"-Wl,-rpath,{lib.parent}", "-L", str(CUDA / "lib64"),
                    f"-Wl,-rpath,{CUDA / 'lib64'}", "-lcudart"], check=True)


@pytest.mark.parametrize("std", ["c++17", "c++20"])
@pytest.mark.parametrize("src", [SRC, TRAINER, DP], ids=lambda p: p.stem)
def test_cpp_api_compiles(tmp_path, std, src):
    _compile(tmp_path / "t", std, src)


@pytest.mark.gpu
def test_cpp_api_reference_tests_on_gpu(tmp_path, cuda):
    exe = tmp_path / "t"
    _compile(exe, "c++20")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL OPTIMIZER TESTS PASSED" in r.stdout


@pytest.mark.gpu
def test_cpp_trainer_driver_on_gpu(tmp_path, cuda):
    exe = tmp_path / "trainer"
    _compile(exe, "c++20", TRAINER)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "TRAINER DRIVER TEST PASSED" in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("sync", ["device", "nccl"])
def test_cpp_data_parallel_two_processes(tmp_path, cuda, sync):
    """Two processes, two GPUs, no Python in them: the C-ABI bootstrap and 5
    fused ZeRO-1 steps against the single-GPU step on the averaged gradient."""
    import os
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    exe = tmp_path / "dp"
    _compile(exe, "c++20", DP)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    idf, out = tmp_path / "uid", tmp_path / "params"
    procs = [subprocess.Popen([str(exe), str(r), "2", str(idf), str(out), sync], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
             for r in range(2)]
    outs = []
    for p in procs:
        try:
            outs.append(p.communicate(timeout=240)[0])
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
    print("\n".join(outs))
    assert all(p.returncode == 0 for p in procs), outs
    assert all("DP C++ TEST PASSED" in o for o in outs)
