"""The C++ API (include/soar_optim.hpp): compiles with g++ as C++17 and C++20
(CPU), and the reference's optimizer tests ported to it pass on the GPU."""
import subprocess
from pathlib import Path

import pytest

from soar_b200 import _build

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "cpp" / "test_optimizers_gpu.cpp"
CUDA = Path("/usr/local/cuda")


def _compile(out: Path, std: str) -> None:
    lib = _build.build()
    cxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"
    subprocess.run([cxx, f"-std={std}", "-O2", "-Wall", "-Wextra", "-I", str(ROOT / "include"),
                    "-I", str(CUDA / "include"), str(SRC), "-o", str(out),
                    str(lib), f"-Wl,-rpath,{lib.parent}", "-L", str(CUDA / "lib64"),
                    f"-Wl,-rpath,{CUDA / 'lib64'}", "-lcudart"], check=True)


@pytest.mark.parametrize("std", ["c++17", "c++20"])
def test_cpp_api_compiles(tmp_path, std):
    _compile(tmp_path / "t", std)


@pytest.mark.gpu
def test_cpp_api_reference_tests_on_gpu(tmp_path, cuda):
    exe = tmp_path / "t"
    _compile(exe, "c++20")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL OPTIMIZER TESTS PASSED" in r.stdout
