"""The C-ABI library builds for sm_100a, loads without a GPU and exports every
symbol include/*.h declares (no compute calls). CPU only."""
import ctypes
import re
import subprocess
from pathlib import Path

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
    out = subprocess.run(["cuobjdump", "--list-elf", str(_build.LIB)], capture_output=True,
                         text=True)
    if out.returncode != 0:
        import pytest
        pytest.skip("cuobjdump unavailable")
    assert "sm_100a" in out.stdout


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
    """The reference's convention: -1 for a NULL handle (src/api/c_api.cpp:100,129)."""
    lib = sb.lib()
    assert lib.soar_optim_step(None, None) == -1
    assert b"null" in lib.soar_last_error()
    assert lib.soar_optim_set_lr(None, 1.0) == -1
    assert lib.soar_cosine_step(None) == -1
    out = ctypes.c_void_p()
    assert lib.soar_optim_create(None, 1, None, ctypes.byref(out)) == -1
