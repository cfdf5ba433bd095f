"""The C-ABI library builds for sm_100a, loads without a GPU and exports every
symbol include/*.h declares (no compute calls). CPU only."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

import soar_b200 as sb
from soar_b200 import _build, optim

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        for m in re.finditer(r"SOAR_API\s+[\w\s\*]+?\b(\w+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    assert {"soar_optim_create", "soar_optim_step", "soar_optim_clip_grad_norm",
            "soar_optim_zero_grad", "soar_optim_set_lr", "soar_optim_get_lr",
            "soar_cosine_create", "soar_cosine_step"} <= names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_build.build()))
    missing = [n for n in sorted(declared_symbols()) if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding covers the same set
    assert declared_symbols() == set(optim.SIGNATURES)


def test_library_is_sm100a():
    """The kernels were compiled for sm_100a (the library reports its build
    architecture; the loaded SASS version is checked on the GPU in
    tests/test_gpu_parity.py)."""
    compiled = ctypes.c_int()
    assert sb.lib().soar_kernel_arch(-1, ctypes.byref(compiled), None) == 0
    assert compiled.value == 1000
    assert "arch=compute_100a,code=sm_100a" in " ".join(_build.NVCC_FLAGS)


def test_default_opts_match_reference_defaults():
    """AdamWOptions defaults, include/soar/optim/adamw.hpp:10-16."""
    o = optim.AdamWOpts()
    sb.lib().soar_adamw_default_opts(ctypes.byref(o))
    assert (o.lr, o.beta1, o.beta2, o.eps, o.weight_decay) == (
        ctypes.c_float(1e-3).value, ctypes.c_float(0.9).value, ctypes.c_float(0.999).value,
        ctypes.c_float(1e-8).value, ctypes.c_float(1e-2).value)
    a = sb.AdamWOptions()
    assert (a.lr, a.beta1, a.beta2, a.eps, a.weight_decay) == (1e-3, 0.9, 0.999, 1e-8, 1e-2)


def test_null_arguments_return_error():
    """The reference's convention: -1 for a NULL handle (src/api/c_api.cpp:51,80,143)."""
    lib = sb.lib()
    assert lib.soar_optim_step(None, None) == -1
    assert b"null" in lib.soar_last_error()
    assert lib.soar_optim_set_lr(None, 1.0) == -1
    assert lib.soar_optim_get_info_async(None, None, None) == -1
    assert lib.soar_cosine_step(None) == -1
    out = ctypes.c_void_p()
    assert lib.soar_optim_create(None, 1, None, ctypes.byref(out)) == -1


def test_data_parallel_entry_points_reject_bad_arguments():
    """Argument checks that run before any CUDA call (no GPU needed)."""
    lib = sb.lib()
    assert lib.soar_zero1_step(None, None) == -1
    assert b"null" in lib.soar_last_error()
    assert lib.soar_zero1_set_signals(None, None) == -1
    assert lib.soar_zero1_error(None, None) == -1


def test_data_parallel_bootstrap_rejects_bad_arguments():
    """soar_dp_* argument checks run before NCCL or CUDA is touched (no GPU)."""
    lib = sb.lib()
    out = ctypes.c_void_p()
    uid = (ctypes.c_ubyte * optim.DP_UNIQUE_ID_BYTES)()
    assert lib.soar_dp_unique_id(None) == -1
    assert lib.soar_dp_init(0, 2, None, 0, ctypes.byref(out)) == -1
    assert b"null" in lib.soar_last_error()
    assert lib.soar_dp_init(2, 2, uid, 0, ctypes.byref(out)) == -1      # rank outside the world
    assert b"rank" in lib.soar_last_error()
    assert lib.soar_dp_init(0, 9, uid, 0, ctypes.byref(out)) == -1      # at most 8 ranks
    assert lib.soar_dp_destroy(None) == -1
    assert lib.soar_dp_barrier(None, None) == -1
    assert lib.soar_dp_allgather_f64(None, None, None, 1, None) == -1
    opts = optim.AdamWOpts()
    lib.soar_adamw_default_opts(ctypes.byref(opts))
    assert lib.soar_dp_zero1_create(None, 10, 5, ctypes.byref(opts), None, 0,
                                    ctypes.byref(out)) == -1
    assert lib.soar_dp_zero1_step(None, None) == -1
    assert lib.soar_dp_zero1_destroy(None) == -1
    info = optim.DpZero1Info()
    assert lib.soar_dp_zero1_get_info(None, ctypes.byref(info)) == -1
    k = ctypes.c_int()
    assert lib.soar_dp_zero1_add_grads(None, ctypes.byref(k)) == -1
    assert lib.soar_dp_zero1_use_grads(None, 0) == -1
    assert lib.soar_dp_zero1_grads(None, 0, ctypes.byref(out)) == -1


def test_bench_probe_is_a_separate_library_and_checks_arguments():
    """The NVLink probe is a bench-only library (csrc/bench_probe.h), not an
    entry point of the optimizer's C-ABI; its argument checks need no GPU."""
    assert not hasattr(sb.lib(), "soar_nvlink_probe")
    lib = optim.probe_lib()
    lib.soar_last_error = lib.soar_probe_last_error
    err = ctypes.c_int()
    bases = (ctypes.c_void_p * 2)(16, 32)
    # world must be 2..8, rank inside it, mode 0 or 1
    assert lib.soar_nvlink_probe(bases, 1, 0, 1 << 20, 0, 4096, 2, 1, ctypes.byref(err), None) == -1
    assert lib.soar_nvlink_probe(bases, 2, 2, 1 << 20, 0, 4096, 2, 1, ctypes.byref(err), None) == -1
    assert lib.soar_nvlink_probe(bases, 2, 0, 1 << 20, 2, 4096, 2, 1, ctypes.byref(err), None) == -1
    # tiles: multiples of 16 that divide the per-peer bytes
    assert lib.soar_nvlink_probe(bases, 2, 0, 1 << 20, 1, 4000, 0, 1, ctypes.byref(err), None) == -1
    assert b"tile" in lib.soar_last_error()
    assert lib.soar_nvlink_probe(bases, 2, 0, 1000, 1, 4096, 0, 1, ctypes.byref(err), None) == -1
    # the pull ring must fit: stages x tile x (world - 1) <= 200 KB
    big = (ctypes.c_void_p * 8)(*[16 * (i + 1) for i in range(8)])
    assert lib.soar_nvlink_probe(big, 8, 0, 1 << 20, 0, 16384, 2, 1, ctypes.byref(err), None) == -1
    assert b"ring" in lib.soar_last_error()


def test_header_is_plain_c_and_links(tmp_path):
    """include/soar_optim.h is a C header (C99, pedantic) and a C program links
    against the library with it."""
    import shutil
    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        pytest.skip("no C compiler")
    src = tmp_path / "c_user.c"
    src.write_text('#include "soar_optim.h"\n'
                   "int main(void) {\n"
                   "    soar_adamw_opts o;\n"
                   "    soar_adamw_default_opts(&o);\n"
                   "    return soar_optim_step(0, 0) == SOAR_ERROR && o.lr > 0.0f ? 0 : 1;\n"
                   "}\n")
    lib = _build.build()
    inc = Path(__file__).resolve().parents[1] / "include"
    exe = tmp_path / "c_user"
    r = subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", str(inc),
                        str(src), "-o", str(exe), "-L", str(lib.parent), "-lsoar_optim",
                        f"-Wl,-rpath,{lib.parent}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stderr


def test_ctypes_structs_match_the_c_layout(tmp_path):
    """The Python binding's structs (soar_b200/optim.py) have the C header's
    size and field offsets, as a C compiler lays them out."""
    import shutil
    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        pytest.skip("no C compiler")
    pairs = [("soar_tensor_desc", optim.TensorDesc), ("soar_adamw_opts", optim.AdamWOpts),
             ("soar_sgd_opts", optim.SGDOpts), ("soar_step_info", optim.StepInfo),
             ("soar_zero1_shard", optim.Zero1Shard), ("soar_dp_zero1_info", optim.DpZero1Info)]
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "soar_optim.h"',
             "int main(void) {"]
    for cname, py in pairs:
        lines.append(f'    printf("{cname} size %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'    printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines += ["    return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    r = subprocess.run([cc, "-std=c99", "-I", str(ROOT / "include"), str(src), "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    got = {}
    for ln in subprocess.run([str(exe)], capture_output=True, text=True).stdout.splitlines():
        name, field, val = ln.split()
        got[(name, field)] = int(val)
    for cname, py in pairs:
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for f, _ in py._fields_:
            assert got[(cname, f)] == getattr(py, f).offset, (cname, f)
