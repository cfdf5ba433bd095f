"""TEST INFRASTRUCTURE ONLY: Python access to the two CPU oracles.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module, and only as the checker. The product library never loads it.

* ``Port``  -- oracle/liboracle_port.so, the plain-C restatement in
  oracle/adamw_port.c (always buildable: gcc only).
* ``RefAdamW`` / ``RefCosine`` -- oracle/_ref/libsoar_ref_adamw.so, the
  reference's own unmodified src/optim/adamw.cpp behind an extern "C" shim
  (oracle/ref_shim.cpp). Built only where the reference tree is present; the
  built .so is git-ignored and travels with the working tree.
* ``RefComposite`` -- the fused step (unscale, inf detect, clip, per-tensor
  wd, AdamW, bf16 write-back, scaler) computed with every AdamW/clip
  floating-point operation done by the reference's own code (one reference
  AdamW per distinct wd value, one more over all params for the clip), for
  pinning the port's composite ``PortOptimizer``.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_SO = HERE / "liboracle_port.so"
REF_SO = HERE / "_ref" / "libsoar_ref_adamw.so"
REF_CUDA_SO = HERE / "_ref" / "libsoar_ref_cuda.so"


def _ref_root() -> Path | None:
    """Root of the reference source tree: $SOAR_REF_ROOT, else the
    `reference_path` recorded in the repository's BASELINE.json. None when
    neither names an existing tree (the compiled oracle then comes from an
    earlier build, or is absent)."""
    cand = os.environ.get("SOAR_REF_ROOT")
    if not cand:
        try:
            import json
            cand = json.loads((HERE.parent / "BASELINE.json").read_text()).get("reference_path")
        except (OSError, ValueError):
            cand = None
    if cand and (Path(cand) / "src" / "optim" / "adamw.cpp").exists():
        return Path(cand)
    return None


REF_ROOT = _ref_root()

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")


def build(ref: bool | None = None) -> None:
    """Compile the port (always) and the reference oracle (when its sources exist)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "port"], check=True)
    if ref is None:
        ref = REF_ROOT is not None
    if ref:
        if REF_ROOT is None:
            raise FileNotFoundError("reference sources not found: set SOAR_REF_ROOT")
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", "refcuda", f"REF_ROOT={REF_ROOT}"],
                       check=True)


def ref_available() -> bool:
    return REF_SO.exists()


def ref_cuda():
    """The reference's CUDA AdamW kernels for sm_100a (secondary GPU baseline)."""
    if not REF_CUDA_SO.exists():
        raise FileNotFoundError(f"{REF_CUDA_SO} not built (needs the reference sources)")
    lib = C.CDLL(str(REF_CUDA_SO))
    lib.soar_refcuda_adamw_multi_tensor.argtypes = [
        C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
        C.POINTER(C.c_void_p), C.POINTER(C.c_int64), C.c_int, C.c_float, C.c_float, C.c_float,
        C.c_float, C.c_float, C.c_float, C.c_float, C.c_void_p]
    lib.soar_refcuda_adamw_step.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                            C.c_float, C.c_float, C.c_float, C.c_float, C.c_float,
                                            C.c_float, C.c_float, C.c_uint64, C.c_void_p]
    return lib


class StepState(C.Structure):
    """Mirror of oracle_step_state in adamw_port.c."""

    _fields_ = [
        ("scale", C.c_float),
        ("tracker", C.c_int32),
        ("t", C.c_uint64),
        ("skipped", C.c_uint64),
        ("last_norm", C.c_float),
        ("last_found_inf", C.c_int32),
        ("last_clip_coef", C.c_float),
    ]


def _load_port() -> C.CDLL:
    if not PORT_SO.exists():
        build(ref=False)
    lib = C.CDLL(str(PORT_SO))
    lib.oracle_bf16_to_f32.restype = C.c_float
    lib.oracle_bf16_to_f32.argtypes = [C.c_uint16]
    lib.oracle_f32_to_bf16.restype = C.c_uint16
    lib.oracle_f32_to_bf16.argtypes = [C.c_float]
    lib.oracle_f32_to_bf16_array.argtypes = [_f32p, _u16p, C.c_size_t]
    lib.oracle_bf16_to_f32_array.argtypes = [_u16p, _f32p, C.c_size_t]
    lib.oracle_adamw_coeffs.argtypes = [C.c_float, C.c_float, C.c_float, C.c_uint64,
                                        C.POINTER(C.c_float), C.POINTER(C.c_float)]
    lib.oracle_adamw_update_f32.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_size_t,
                                            C.c_float, C.c_float, C.c_float, C.c_float,
                                            C.c_float, C.c_float, C.c_float]
    lib.oracle_sumsq_f32.restype = C.c_double
    lib.oracle_sumsq_f32.argtypes = [_f32p, C.c_size_t, C.c_double]
    lib.oracle_norm_from_sumsq.restype = C.c_float
    lib.oracle_norm_from_sumsq.argtypes = [C.c_double]
    lib.oracle_clip_coef.restype = C.c_float
    lib.oracle_clip_coef.argtypes = [C.c_float, C.c_float, C.POINTER(C.c_int)]
    lib.oracle_scale_f32.argtypes = [_f32p, C.c_size_t, C.c_float]
    lib.oracle_cosine_lr.restype = C.c_float
    lib.oracle_cosine_lr.argtypes = [C.c_float, C.c_float, C.c_uint64, C.c_uint64, C.c_uint64]
    lib.oracle_unscale_bf16.restype = C.c_int
    lib.oracle_unscale_bf16.argtypes = [_u16p, C.c_size_t, C.c_float, _f32p]
    lib.oracle_scaler_update.argtypes = [C.POINTER(StepState), C.c_int, C.c_float, C.c_float,
                                         C.c_int32]
    lib.oracle_step.restype = C.c_int
    lib.oracle_step.argtypes = [C.c_int, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                C.POINTER(C.c_void_p), C.POINTER(C.c_uint64),
                                C.POINTER(C.c_float), C.c_float, C.c_float, C.c_float,
                                C.c_float, C.c_float, C.c_int, C.c_float, C.c_float,
                                C.c_int32, C.POINTER(StepState), _f32p]
    lib.oracle_reduce_avg_bf16.argtypes = [C.c_int, C.POINTER(C.c_void_p), C.c_size_t, _u16p]
    lib.oracle_ema_update.argtypes = [_f32p, _f32p, C.c_size_t, C.c_float]
    lib.oracle_sgd_apply_with_sumsq.restype = C.c_int
    lib.oracle_sgd_apply_with_sumsq.argtypes = [
        C.c_int, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
        C.POINTER(C.c_void_p), C.POINTER(C.c_uint64), C.POINTER(C.c_float), C.c_float, C.c_float,
        C.c_float, C.c_int, C.c_float, C.c_int, C.c_float, C.c_float, C.c_int32, C.c_double,
        C.POINTER(StepState), _f32p]
    lib.oracle_grad_sumsq.restype = C.c_double
    lib.oracle_grad_sumsq.argtypes = [C.c_int, C.c_int, C.POINTER(C.c_void_p),
                                      C.POINTER(C.c_uint64), C.c_float, C.POINTER(C.c_int), _f32p]
    lib.oracle_apply_with_sumsq.restype = C.c_int
    lib.oracle_apply_with_sumsq.argtypes = [C.c_int, C.c_int, C.POINTER(C.c_void_p),
                                            C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                            C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                            C.POINTER(C.c_uint64), C.POINTER(C.c_float),
                                            C.c_float, C.c_float, C.c_float, C.c_float,
                                            C.c_float, C.c_int, C.c_float, C.c_float, C.c_int32,
                                            C.c_double, C.POINTER(StepState), _f32p]
    return lib


_port: C.CDLL | None = None


def port() -> C.CDLL:
    global _port
    if _port is None:
        _port = _load_port()
    return _port


def _ptrs(arrs):
    return (C.c_void_p * len(arrs))(*[a.ctypes.data if a is not None else None for a in arrs])


# ---------------------------------------------------------------- port API ---

def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    port().oracle_f32_to_bf16_array(x.ravel(), out.ravel(), x.size)
    return out


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, np.float32)
    port().oracle_bf16_to_f32_array(h.ravel(), out.ravel(), h.size)
    return out


def adamw_coeffs(lr: float, beta1: float, beta2: float, t: int) -> tuple[float, float]:
    s, q = C.c_float(), C.c_float()
    port().oracle_adamw_coeffs(lr, beta1, beta2, t, C.byref(s), C.byref(q))
    return s.value, q.value


def cosine_lr(base_lr, eta_min, total, warmup, current) -> float:
    return port().oracle_cosine_lr(base_lr, eta_min, total, warmup, current)


@dataclass
class StepConfig:
    """Hyperparameters of one fused optimizer step."""

    layout: int = 0  # 0 fp32, 1 mixed bf16
    lr: float = 1e-3
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    max_norm: float = 0.0  # <= 0: no clip
    use_scaler: bool = False
    growth_factor: float = 2.0
    backoff_factor: float = 0.5
    growth_interval: int = 200


class PortOptimizer:
    """Port oracle state for a tensor list: params (fp32 or bf16 uint16),
    fp32 master (mixed), m, v, per-tensor wd, and the step state."""

    def __init__(self, params, wd, cfg: StepConfig, init_scale: float = 1.0):
        self.cfg = cfg
        self.params = [np.ascontiguousarray(p) for p in params]
        self.numel = [int(p.size) for p in self.params]
        self.wd = np.asarray(wd, dtype=np.float32)
        if cfg.layout == 1:
            self.master = [bf16_to_f32(p) for p in self.params]
        else:
            self.master = [None] * len(self.params)
        self.m = [np.zeros(n, np.float32) for n in self.numel]
        self.v = [np.zeros(n, np.float32) for n in self.numel]
        self.state = StepState(scale=init_scale if cfg.use_scaler else 1.0)
        self.scratch = np.zeros(max(self.numel + [1]), np.float32)
        self.ema = None
        self.ema_decay = 0.0

    def weights(self, i: int) -> np.ndarray:
        """fp32 weights of tensor i (the master in the mixed layout)."""
        return self.master[i] if self.cfg.layout == 1 else self.params[i]

    def enable_ema(self, decay: float):
        """ModelEMA: the shadow starts as a copy of the weights (ema.hpp:49-57)."""
        self.ema = [self.weights(i).astype(np.float32).copy() for i in range(len(self.params))]
        self.ema_decay = decay

    def step(self, grads, lr: float | None = None) -> int:
        c = self.cfg
        n = len(self.params)
        grads = [None if g is None else np.ascontiguousarray(g) for g in grads]
        numel = (C.c_uint64 * n)(*self.numel)
        wd = (C.c_float * n)(*self.wd.tolist())
        skipped = port().oracle_step(
            c.layout, n, _ptrs(self.params), _ptrs(grads), _ptrs(self.master), _ptrs(self.m),
            _ptrs(self.v), numel, wd, c.lr if lr is None else lr, c.beta1, c.beta2, c.eps,
            c.max_norm, int(c.use_scaler), c.growth_factor, c.backoff_factor,
            c.growth_interval, C.byref(self.state), self.scratch)
        if self.ema is not None and not skipped:
            # the fused EMA follows the weights the step updated (tensors with a grad)
            for i, g in enumerate(grads):
                if g is not None and self.numel[i]:
                    port().oracle_ema_update(self.ema[i], np.ascontiguousarray(self.weights(i)),
                                             self.numel[i], self.ema_decay)
        return skipped


class PortSGD(PortOptimizer):
    """Port oracle of the fused SGD step (oracle_sgd_apply_with_sumsq); the
    momentum buffers live in self.m."""

    def __init__(self, params, wd, cfg: StepConfig, momentum=0.0, dampening=0.0, nesterov=False,
                 init_scale: float = 1.0):
        super().__init__(params, wd, cfg, init_scale)
        self.momentum, self.dampening, self.nesterov = momentum, dampening, nesterov

    def step(self, grads, lr: float | None = None) -> int:
        c = self.cfg
        n = len(self.params)
        grads = [None if g is None else np.ascontiguousarray(g) for g in grads]
        numel = (C.c_uint64 * n)(*self.numel)
        inv = (np.float32(1.0) / np.float32(self.state.scale)) if c.use_scaler else np.float32(1.0)
        found = C.c_int()
        sumsq = port().oracle_grad_sumsq(c.layout, n, _ptrs(grads), numel, float(inv),
                                         C.byref(found), self.scratch)
        return port().oracle_sgd_apply_with_sumsq(
            c.layout, n, _ptrs(self.params), _ptrs(grads), _ptrs(self.master), _ptrs(self.m),
            numel, (C.c_float * n)(*self.wd.tolist()), c.lr if lr is None else lr,
            self.momentum, self.dampening, int(self.nesterov), c.max_norm, int(c.use_scaler),
            c.growth_factor, c.backoff_factor, c.growth_interval, sumsq, C.byref(self.state),
            self.scratch)


class PortShard(PortOptimizer):
    """The port oracle behind the data-parallel split API (grad_sumsq / apply
    with rank-ordered partial sums), over numpy views of a rank's shards.
    Stands in for the device optimizer in host-logic tests."""

    def __init__(self, params, grads, wd, cfg: StepConfig, init_scale: float = 1.0):
        super().__init__(params, wd, cfg, init_scale)
        self.params = list(params)  # keep the caller's views: updates land in place
        self.grads = list(grads)

    def _inv(self):
        return (np.float32(1.0) / np.float32(self.state.scale)) if self.cfg.use_scaler \
            else np.float32(1.0)

    def grad_sumsq_value(self) -> float:
        n = len(self.params)
        found = C.c_int()
        return port().oracle_grad_sumsq(self.cfg.layout, n, _ptrs(self.grads),
                                        (C.c_uint64 * n)(*self.numel), float(self._inv()),
                                        C.byref(found), self.scratch)

    def grad_sumsq(self, out_ptr: int, stream=None):
        C.c_double.from_address(out_ptr).value = self.grad_sumsq_value()

    def apply_sumsq(self, total: float, lr: float | None = None) -> int:
        c = self.cfg
        n = len(self.params)
        return port().oracle_apply_with_sumsq(
            c.layout, n, _ptrs(self.params), _ptrs(self.grads), _ptrs(self.master),
            _ptrs(self.m), _ptrs(self.v), (C.c_uint64 * n)(*self.numel),
            (C.c_float * n)(*self.wd.tolist()), c.lr if lr is None else lr, c.beta1, c.beta2,
            c.eps, c.max_norm, int(c.use_scaler), c.growth_factor, c.backoff_factor,
            c.growth_interval, total, C.byref(self.state), self.scratch)

    def apply(self, parts_ptr: int, n_parts: int, stream=None):
        total = 0.0
        if n_parts:
            parts = (C.c_double * n_parts).from_address(parts_ptr)
            for x in parts:  # rank order, as the device sums them
                total += x
        return self.apply_sumsq(total)


def reduce_avg_bf16(inputs: list[np.ndarray]) -> np.ndarray:
    n = inputs[0].size
    out = np.empty(n, np.uint16)
    arrs = [np.ascontiguousarray(a, dtype=np.uint16) for a in inputs]
    port().oracle_reduce_avg_bf16(len(arrs), _ptrs(arrs), n, out)
    return out


# ----------------------------------------------------------- reference API ---

_ref: C.CDLL | None = None


def ref() -> C.CDLL:
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} not built (needs the reference sources)")
        lib = C.CDLL(str(REF_SO))
        lib.soar_ref_adamw_create.restype = C.c_void_p
        lib.soar_ref_adamw_create.argtypes = [C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                              C.POINTER(C.c_uint64), C.c_int, C.c_float,
                                              C.c_float, C.c_float, C.c_float, C.c_float]
        for name in ("destroy", "step", "zero_grad"):
            getattr(lib, f"soar_ref_adamw_{name}").argtypes = [C.c_void_p]
        lib.soar_ref_adamw_clip_grad_norm.restype = C.c_float
        lib.soar_ref_adamw_clip_grad_norm.argtypes = [C.c_void_p, C.c_float]
        lib.soar_ref_adamw_set_lr.argtypes = [C.c_void_p, C.c_float]
        lib.soar_ref_adamw_get_lr.restype = C.c_float
        lib.soar_ref_adamw_get_lr.argtypes = [C.c_void_p]
        lib.soar_ref_adamw_get_step.restype = C.c_uint64
        lib.soar_ref_adamw_get_step.argtypes = [C.c_void_p]
        lib.soar_ref_adamw_set_step.argtypes = [C.c_void_p, C.c_uint64]
        lib.soar_ref_adamw_get_moment.restype = C.c_int
        lib.soar_ref_adamw_get_moment.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p]
        lib.soar_ref_adamw_set_moment.restype = C.c_int
        lib.soar_ref_adamw_set_moment.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p]
        lib.soar_ref_cosine_create.restype = C.c_void_p
        lib.soar_ref_cosine_create.argtypes = [C.c_void_p, C.c_uint64, C.c_float, C.c_uint64]
        lib.soar_ref_cosine_step.argtypes = [C.c_void_p]
        lib.soar_ref_cosine_destroy.argtypes = [C.c_void_p]
        _ref = lib
    return _ref


class RefAdamW:
    """The reference's soar::optim::AdamW over numpy fp32 buffers (in place)."""

    def __init__(self, params, grads, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8,
                 weight_decay=1e-2):
        self.params = params
        self.grads = grads
        n = len(params)
        numel = (C.c_uint64 * n)(*[p.size for p in params])
        self.h = ref().soar_ref_adamw_create(_ptrs(params), _ptrs(grads), numel, n, lr, beta1,
                                             beta2, eps, weight_decay)

    def __del__(self):
        if getattr(self, "h", None):
            ref().soar_ref_adamw_destroy(self.h)
            self.h = None

    def step(self):
        ref().soar_ref_adamw_step(self.h)

    def clip_grad_norm(self, max_norm: float) -> float:
        return ref().soar_ref_adamw_clip_grad_norm(self.h, max_norm)

    def zero_grad(self):
        ref().soar_ref_adamw_zero_grad(self.h)

    def set_lr(self, lr):
        ref().soar_ref_adamw_set_lr(self.h, lr)

    def get_lr(self) -> float:
        return ref().soar_ref_adamw_get_lr(self.h)

    @property
    def step_count(self) -> int:
        return ref().soar_ref_adamw_get_step(self.h)

    @step_count.setter
    def step_count(self, t):
        ref().soar_ref_adamw_set_step(self.h, t)

    def moment(self, idx: int, which: int) -> np.ndarray:
        out = np.empty(self.params[idx].size, np.float32)
        assert ref().soar_ref_adamw_get_moment(self.h, idx, which, out) == 0
        return out

    def set_moment(self, idx: int, which: int, val: np.ndarray):
        assert ref().soar_ref_adamw_set_moment(self.h, idx, which,
                                               np.ascontiguousarray(val, np.float32)) == 0


class RefSGD:
    """The reference's soar::optim::SGD over numpy fp32 buffers (in place)."""

    def __init__(self, params, grads, lr=1e-2, momentum=0.0, dampening=0.0, weight_decay=0.0,
                 nesterov=False):
        lib = ref()
        if not hasattr(lib, "_sgd_bound"):
            lib.soar_ref_sgd_create.restype = C.c_void_p
            lib.soar_ref_sgd_create.argtypes = [C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                                C.POINTER(C.c_uint64), C.c_int, C.c_float,
                                                C.c_float, C.c_float, C.c_float, C.c_int]
            lib.soar_ref_sgd_step.argtypes = [C.c_void_p]
            lib.soar_ref_sgd_destroy.argtypes = [C.c_void_p]
            lib.soar_ref_sgd_set_lr.argtypes = [C.c_void_p, C.c_float]
            lib.soar_ref_sgd_clip_grad_norm.restype = C.c_float
            lib.soar_ref_sgd_clip_grad_norm.argtypes = [C.c_void_p, C.c_float]
            lib._sgd_bound = True
        self.params, self.grads = params, grads
        n = len(params)
        self.h = lib.soar_ref_sgd_create(_ptrs(params), _ptrs(grads),
                                         (C.c_uint64 * n)(*[p.size for p in params]), n, lr,
                                         momentum, dampening, weight_decay, int(nesterov))

    def step(self):
        ref().soar_ref_sgd_step(self.h)

    def clip_grad_norm(self, max_norm):
        return ref().soar_ref_sgd_clip_grad_norm(self.h, max_norm)

    def __del__(self):
        if getattr(self, "h", None):
            ref().soar_ref_sgd_destroy(self.h)
            self.h = None


class RefEma:
    """The reference's soar::utils::ModelEMA over numpy fp32 weights (in place)."""

    def __init__(self, params, decay):
        lib = ref()
        if not hasattr(lib, "_ema_bound"):
            lib.soar_ref_ema_create.restype = C.c_void_p
            lib.soar_ref_ema_create.argtypes = [C.POINTER(C.c_void_p), C.POINTER(C.c_uint64),
                                                C.c_int, C.c_float]
            for nm in ("update", "apply_to", "destroy"):
                getattr(lib, f"soar_ref_ema_{nm}").argtypes = [C.c_void_p]
            lib.soar_ref_ema_shadow.restype = C.c_int
            lib.soar_ref_ema_shadow.argtypes = [C.c_void_p, C.c_int, _f32p]
            lib._ema_bound = True
        self.params = params
        n = len(params)
        self.h = lib.soar_ref_ema_create(_ptrs(params), (C.c_uint64 * n)(*[p.size for p in params]),
                                         n, decay)

    def update(self):
        ref().soar_ref_ema_update(self.h)

    def apply_to(self):
        ref().soar_ref_ema_apply_to(self.h)

    def shadow(self, i) -> np.ndarray:
        out = np.empty(self.params[i].size, np.float32)
        assert ref().soar_ref_ema_shadow(self.h, i, out) == 0
        return out

    def __del__(self):
        if getattr(self, "h", None):
            ref().soar_ref_ema_destroy(self.h)
            self.h = None


class RefCosine:
    """The reference's CosineAnnealingLR bound to a RefAdamW."""

    def __init__(self, opt: RefAdamW, total_steps, eta_min=1e-6, warmup_steps=0):
        self.opt = opt
        self.h = ref().soar_ref_cosine_create(opt.h, total_steps, eta_min, warmup_steps)

    def __del__(self):
        if getattr(self, "h", None):
            ref().soar_ref_cosine_destroy(self.h)
            self.h = None

    def step(self):
        ref().soar_ref_cosine_step(self.h)


class RefComposite:
    """The fused step with every AdamW/clip float op done by the reference.

    Mirrors PortOptimizer: one reference AdamW per distinct weight decay (each
    instance sees only its own tensors, adamw.cpp's loop is per tensor and
    independent), plus one instance over all tensors used only for
    clip_grad_norm. Unscale, inf detection, the scaler and bf16 RNE are the
    port's (the reference has none)."""

    def __init__(self, params, wd, cfg: StepConfig, init_scale: float = 1.0, null_grad=()):
        self.cfg = cfg
        self.params = [np.ascontiguousarray(p) for p in params]
        if cfg.layout == 1:
            self.master = [bf16_to_f32(p) for p in self.params]
        else:
            self.master = self.params
        # tensors without a gradient are skipped by the reference (adamw.cpp:30-31,74-75)
        self.gbuf = [None if i in null_grad else np.zeros(p.size, np.float32)
                     for i, p in enumerate(self.params)]
        self.wd = [float(np.float32(w)) for w in wd]
        self.groups: dict[float, list[int]] = {}
        for i, w in enumerate(self.wd):
            self.groups.setdefault(w, []).append(i)
        self.opts = {w: RefAdamW([self.master[i] for i in idx], [self.gbuf[i] for i in idx],
                                 cfg.lr, cfg.beta1, cfg.beta2, cfg.eps, w)
                     for w, idx in self.groups.items()}
        self.clipper = RefAdamW(self.master, self.gbuf, cfg.lr)
        self.state = StepState(scale=init_scale if cfg.use_scaler else 1.0)

    def moment(self, i: int, which: int) -> np.ndarray:
        w = self.wd[i]
        return self.opts[w].moment(self.groups[w].index(i), which)

    def step(self, grads, lr: float | None = None) -> int:
        c = self.cfg
        st = self.state
        inv = np.float32(1.0) / np.float32(st.scale) if c.use_scaler else np.float32(1.0)
        found = False
        for i, g in enumerate(grads):
            if self.gbuf[i] is None:
                continue
            gf = bf16_to_f32(g) if c.layout == 1 else np.asarray(g, np.float32)
            np.multiply(gf, inv, out=self.gbuf[i], dtype=np.float32)
            found |= not np.isfinite(self.gbuf[i]).all()
        st.last_found_inf = int(found)
        if c.use_scaler and found:
            st.skipped += 1
            st.last_clip_coef = 1.0
            port().oracle_scaler_update(C.byref(st), 1, c.growth_factor, c.backoff_factor,
                                        c.growth_interval)
            return 1
        if c.max_norm > 0:
            st.last_norm = self.clipper.clip_grad_norm(c.max_norm)
            norm, mx = np.float32(st.last_norm), np.float32(c.max_norm)
            clipped = norm > mx and norm > np.float32(1e-6)
            st.last_clip_coef = float(mx / norm) if clipped else 1.0
        for w, o in self.opts.items():
            o.set_lr(c.lr if lr is None else lr)
            o.step()
        st.t += 1
        if c.layout == 1:
            for p, mst, b in zip(self.params, self.master, self.gbuf):
                if b is not None:
                    p[:] = f32_to_bf16(mst)
        if c.use_scaler:
            port().oracle_scaler_update(C.byref(st), 0, c.growth_factor, c.backoff_factor,
                                        c.growth_interval)
        return 0
