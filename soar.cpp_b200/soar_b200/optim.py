"""Python mirror of the reference's optimizer API over the sm_100a C-ABI.

The reference binds its C-ABI with ctypes (soar/__init__.py:48-95); this
module binds include/soar_optim.h the same way and mirrors
soar::optim::AdamW / AdamWOptions / CosineAnnealingLR
(include/soar/optim/adamw.hpp:10-57): same class names, the same methods
(step, zero_grad, clip_grad_norm, set_lr, get_lr) with the same argument
meaning, and failures raised as exceptions (the reference's C++ layer throws;
its C-ABI maps any failure to -1, which this wrapper turns back into an
exception carrying soar_last_error()).

Parameters and gradients are CUDA tensors (anything with ``data_ptr()``,
``numel()`` and, for params, ``.grad``); the optimizer state lives in the
library's own device slab. There is no CPU fallback: without the compiled
library every call fails.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from pathlib import Path

from . import _build

LAYOUT_FP32 = 0
LAYOUT_BF16_MIXED = 1
STATE_MASTER, STATE_M, STATE_V, STATE_EMA = 0, 1, 2, 3


class SoarError(RuntimeError):
    pass


class TensorDesc(C.Structure):
    _fields_ = [("param", C.c_void_p), ("grad", C.c_void_p), ("numel", C.c_uint64),
                ("weight_decay", C.c_float)]


class AdamWOpts(C.Structure):
    _fields_ = [("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float),
                ("eps", C.c_float), ("weight_decay", C.c_float), ("layout", C.c_int32),
                ("max_grad_norm", C.c_float), ("use_loss_scaler", C.c_int32),
                ("init_scale", C.c_float), ("growth_factor", C.c_float),
                ("backoff_factor", C.c_float), ("growth_interval", C.c_int32),
                ("device", C.c_int32)]


class SGDOpts(C.Structure):
    _fields_ = [("lr", C.c_float), ("momentum", C.c_float), ("dampening", C.c_float),
                ("weight_decay", C.c_float), ("nesterov", C.c_int32), ("layout", C.c_int32),
                ("max_grad_norm", C.c_float), ("use_loss_scaler", C.c_int32),
                ("init_scale", C.c_float), ("growth_factor", C.c_float),
                ("backoff_factor", C.c_float), ("growth_interval", C.c_int32),
                ("device", C.c_int32)]


class StepInfo(C.Structure):
    _fields_ = [("step", C.c_uint64), ("skipped", C.c_uint64), ("grad_norm", C.c_float),
                ("found_inf", C.c_int32), ("clip_coef", C.c_float), ("loss_scale", C.c_float),
                ("growth_tracker", C.c_int32), ("lr", C.c_float), ("error", C.c_int32)]

    def as_dict(self) -> dict:
        return {k: getattr(self, k) for k, _ in self._fields_}


_lib: C.CDLL | None = None

# name -> (restype, argtypes); every symbol include/soar_optim.h declares
SIGNATURES: dict[str, tuple] = {
    "soar_adamw_default_opts": (None, [C.POINTER(AdamWOpts)]),
    "soar_optim_create": (C.c_int, [C.POINTER(TensorDesc), C.c_int, C.POINTER(AdamWOpts),
                                    C.POINTER(C.c_void_p)]),
    "soar_optim_create_uniform": (C.c_int, [C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                            C.POINTER(C.c_uint64), C.c_int,
                                            C.POINTER(AdamWOpts), C.POINTER(C.c_void_p)]),
    "soar_optim_destroy": (C.c_int, [C.c_void_p]),
    "soar_sgd_default_opts": (None, [C.POINTER(SGDOpts)]),
    "soar_sgd_create": (C.c_int, [C.POINTER(TensorDesc), C.c_int, C.POINTER(SGDOpts),
                                  C.POINTER(C.c_void_p)]),
    "soar_optim_step": (C.c_int, [C.c_void_p, C.c_void_p]),
    "soar_optim_clip_grad_norm": (C.c_int, [C.c_void_p, C.c_float, C.POINTER(C.c_float),
                                            C.c_void_p]),
    "soar_optim_clip_grad_norm_async": (C.c_int, [C.c_void_p, C.c_float, C.c_void_p]),
    "soar_optim_zero_grad": (C.c_int, [C.c_void_p, C.c_void_p]),
    "soar_optim_set_lr": (C.c_int, [C.c_void_p, C.c_float]),
    "soar_optim_get_lr": (C.c_int, [C.c_void_p, C.POINTER(C.c_float)]),
    "soar_optim_get_info": (C.c_int, [C.c_void_p, C.POINTER(StepInfo), C.c_void_p]),
    "soar_optim_get_info_async": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p]),
    "soar_optim_set_counters": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint64, C.c_float,
                                          C.c_int32, C.c_void_p]),
    "soar_optim_state_ptr": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "soar_optim_read_state": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "soar_optim_write_state": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "soar_optim_loss_scale_ptr": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "soar_optim_enable_ema": (C.c_int, [C.c_void_p, C.c_float, C.c_void_p]),
    "soar_optim_ema_apply_to": (C.c_int, [C.c_void_p, C.c_void_p]),
    "soar_optim_save_state": (C.c_int, [C.c_void_p, C.c_char_p]),
    "soar_optim_load_state": (C.c_int, [C.c_void_p, C.c_char_p, C.c_void_p]),
    "soar_optim_grad_sumsq": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p]),
    "soar_optim_apply": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    "soar_cosine_create": (C.c_int, [C.c_void_p, C.c_uint64, C.c_float, C.c_uint64,
                                     C.POINTER(C.c_void_p)]),
    "soar_cosine_step": (C.c_int, [C.c_void_p]),
    "soar_cosine_destroy": (C.c_int, [C.c_void_p]),
    "soar_grad_sumsq_noalloc": (C.c_int, [C.POINTER(C.c_void_p), C.POINTER(C.c_uint64),
                                          C.c_int, C.c_int, C.c_float, C.c_void_p,
                                          C.c_void_p]),
    "soar_ipc_alloc": (C.c_int, [C.c_size_t, C.c_int, C.POINTER(C.c_void_p), C.c_void_p]),
    "soar_ipc_free": (C.c_int, [C.c_void_p, C.c_int]),
    "soar_ipc_open": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_void_p)]),
    "soar_ipc_close": (C.c_int, [C.c_void_p, C.c_int]),
    "soar_zero1_create": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_void_p),
                                    C.POINTER(C.c_void_p), C.c_void_p, C.c_int,
                                    C.POINTER(C.c_void_p)]),
    "soar_zero1_reduce_sumsq": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p]),
    "soar_zero1_apply_allgather": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    "soar_zero1_set_signals": (C.c_int, [C.c_void_p, C.c_void_p]),
    "soar_zero1_step": (C.c_int, [C.c_void_p, C.c_void_p]),
    "soar_zero1_error": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "soar_zero1_destroy": (C.c_int, [C.c_void_p]),
    "soar_selftest_bounded_wait": (C.c_int, [C.c_uint64, C.c_int, C.POINTER(C.c_int),
                                             C.POINTER(C.c_uint64)]),
    "soar_kernel_arch": (C.c_int, [C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "soar_dp_unique_id": (C.c_int, [C.c_void_p]),
    "soar_dp_init": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_int, C.POINTER(C.c_void_p)]),
    "soar_dp_destroy": (C.c_int, [C.c_void_p]),
    "soar_dp_barrier": (C.c_int, [C.c_void_p, C.c_void_p]),
    "soar_dp_allgather_f64": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64,
                                        C.c_void_p]),
    "soar_dp_zero1_create": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint64, C.c_void_p,
                                       C.c_void_p, C.c_int, C.POINTER(C.c_void_p)]),
    "soar_dp_zero1_get_info": (C.c_int, [C.c_void_p, C.c_void_p]),
    "soar_dp_zero1_step": (C.c_int, [C.c_void_p, C.c_void_p]),
    "soar_dp_zero1_add_grads": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "soar_dp_zero1_use_grads": (C.c_int, [C.c_void_p, C.c_int]),
    "soar_dp_zero1_grads": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_void_p)]),
    "soar_dp_zero1_destroy": (C.c_int, [C.c_void_p]),
    "soar_optim_add_grads": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_int)]),
    "soar_optim_use_grads": (C.c_int, [C.c_void_p, C.c_int]),
    "soar_optim_kernel_path": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "soar_last_error": (C.c_char_p, []),
}

IPC_HANDLE_BYTES = 64
DP_UNIQUE_ID_BYTES = 128
DP_SYNC_DEVICE, DP_SYNC_NCCL = 0, 1


class DpZero1Info(C.Structure):
    _fields_ = [("params", C.c_void_p), ("grads", C.c_void_p), ("optimizer", C.c_void_p),
                ("zero1", C.c_void_p), ("n_params", C.c_uint64), ("shard_params", C.c_uint64),
                ("rank", C.c_int32), ("world", C.c_int32)]
ZERO1_SIGNAL_BYTES = 4096


class Zero1Shard(C.Structure):
    _fields_ = [("offset", C.c_uint64), ("count", C.c_uint64), ("tensor", C.c_int32)]


def library_path() -> Path:
    return _build.LIB


_probe: C.CDLL | None = None


def probe_lib() -> C.CDLL:
    """The bench-only NVLink probe library (bench_probe.h), built on first use."""
    global _probe
    if _probe is None:
        handle = C.CDLL(str(_build.build_probe()))
        handle.soar_nvlink_probe.restype = C.c_int
        handle.soar_nvlink_probe.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_uint64, C.c_int,
                                             C.c_uint32, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        handle.soar_probe_last_error.restype = C.c_char_p
        handle.soar_probe_last_error.argtypes = []
        _probe = handle
    return _probe


def lib() -> C.CDLL:
    """The loaded C-ABI library (built on first use if the .so is absent or stale)."""
    global _lib
    if _lib is None:
        path = _build.build()
        handle = C.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().soar_last_error().decode(errors="replace")
        raise SoarError(f"{what} failed: {msg}")


def _stream_handle(stream) -> int | None:
    """cudaStream_t of `stream` (torch.cuda.Stream, int, None -> torch's current)."""
    if stream is None:
        try:
            import torch
            if torch.cuda.is_available() and torch.cuda.is_initialized():
                return torch.cuda.current_stream().cuda_stream
        except Exception:  # pragma: no cover - torch absent
            pass
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


class _DeviceArray:
    """__cuda_array_interface__ view of library-owned device memory."""

    def __init__(self, ptr: int, n: int, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


@dataclass
class AdamWOptions:
    """include/soar/optim/adamw.hpp:10-16, same defaults."""

    lr: float = 1e-3
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    weight_decay: float = 1e-2


@dataclass
class SGDOptions:
    """include/soar/optim/sgd.hpp:9-15, same defaults."""

    lr: float = 1e-2
    momentum: float = 0.0
    dampening: float = 0.0
    weight_decay: float = 0.0
    nesterov: bool = False


@dataclass
class LossScalerOptions:
    """Dynamic loss scaler (no reference counterpart)."""

    init_scale: float = 65536.0
    growth_factor: float = 2.0
    backoff_factor: float = 0.5
    growth_interval: int = 200


@dataclass
class ParamGroup:
    """A list of params sharing one weight decay (the per-group wd mask)."""

    params: list
    weight_decay: float | None = None
    extra: dict = field(default_factory=dict)


class AdamW:
    """soar::optim::AdamW on the GPU.

    ``params`` is a list of CUDA tensors with ``.grad`` (or ParamGroup objects
    giving their own weight decay). ``layout`` is "fp32" (the reference's
    layout) or "bf16_mixed" (bf16 params/grads, fp32 master/m/v). With
    ``max_grad_norm`` > 0, step() clips first exactly as clip_grad_norm() would.
    ``grads`` optionally gives the gradient buffers explicitly (else ``p.grad``).
    """

    def __init__(self, params, options: AdamWOptions | None = None, *, layout: str = "fp32",
                 max_grad_norm: float = 0.0, loss_scaler: LossScalerOptions | None = None,
                 device: int | None = None, grads=None):
        options = options or AdamWOptions()
        o = AdamWOpts()
        lib().soar_adamw_default_opts(C.byref(o))
        o.lr, o.beta1, o.beta2, o.eps = options.lr, options.beta1, options.beta2, options.eps
        o.weight_decay = options.weight_decay
        self._create(params, grads, options.weight_decay, o, layout, max_grad_norm, loss_scaler,
                     device, lib().soar_optim_create, "soar_optim_create")

    def _create(self, params, grads, default_wd, o, layout, max_grad_norm, loss_scaler, device,
                create_fn, create_name):
        tensors, wds = [], []
        for p in params:
            if isinstance(p, ParamGroup):
                wd = default_wd if p.weight_decay is None else p.weight_decay
                for q in p.params:
                    tensors.append(q)
                    wds.append(wd)
            else:
                tensors.append(p)
                wds.append(default_wd)
        self.params = tensors
        # gradients: explicit list (same order as the flattened params) or .grad
        self.grads = list(grads) if grads is not None else [getattr(p, "grad", None)
                                                             for p in tensors]
        if len(self.grads) != len(tensors):
            raise ValueError("one gradient (or None) per parameter")
        self.layout = {"fp32": LAYOUT_FP32, "bf16_mixed": LAYOUT_BF16_MIXED}[layout]
        o.layout = self.layout
        o.max_grad_norm = max_grad_norm
        if loss_scaler is not None:
            o.use_loss_scaler = 1
            o.init_scale = loss_scaler.init_scale
            o.growth_factor = loss_scaler.growth_factor
            o.backoff_factor = loss_scaler.backoff_factor
            o.growth_interval = loss_scaler.growth_interval
        if device is None:
            dev = getattr(tensors[0], "device", None) if tensors else None
            device = dev.index if dev is not None and dev.index is not None else 0
        o.device = device
        self.device = device
        self.opts = o
        n = len(tensors)
        descs = (TensorDesc * max(n, 1))()
        for i, (p, g, wd) in enumerate(zip(tensors, self.grads, wds)):
            descs[i].param = p.data_ptr()
            descs[i].grad = g.data_ptr() if g is not None else None
            descs[i].numel = p.numel()
            descs[i].weight_decay = wd
        self.numel = [p.numel() for p in tensors]
        self.weight_decays = wds
        h = C.c_void_p()
        _check(create_fn(descs, n, C.byref(o), C.byref(h)), create_name)
        self.handle = h

    @classmethod
    def borrow(cls, handle: int, numel: list[int], device: int, layout: str = "bf16_mixed"):
        """A view of an optimizer another object owns (the shard optimizer of
        soar_dp_zero1_create): every method but close(), which does nothing."""
        self = cls.__new__(cls)
        self.handle = C.c_void_p(handle)
        self.numel = list(numel)
        self.device = device
        self.layout = {"fp32": LAYOUT_FP32, "bf16_mixed": LAYOUT_BF16_MIXED}[layout]
        self.params, self.grads, self.weight_decays = [], [], []
        self._borrowed = True
        return self

    def close(self):
        if getattr(self, "_borrowed", False):
            self.handle = None
            return
        if getattr(self, "handle", None):
            lib().soar_optim_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- the reference's methods (adamw.hpp:25-30) --------------------------
    def step(self, stream=None) -> None:
        _check(lib().soar_optim_step(self.handle, _stream_handle(stream)), "soar_optim_step")

    def zero_grad(self, stream=None) -> None:
        _check(lib().soar_optim_zero_grad(self.handle, _stream_handle(stream)),
               "soar_optim_zero_grad")

    def clip_grad_norm(self, max_norm: float, stream=None) -> float:
        out = C.c_float()
        _check(lib().soar_optim_clip_grad_norm(self.handle, max_norm, C.byref(out),
                                               _stream_handle(stream)),
               "soar_optim_clip_grad_norm")
        return out.value

    def clip_grad_norm_async(self, max_norm: float, stream=None) -> None:
        """clip_grad_norm without the host round trip: the next step() clips
        by max_norm from the norm computed here (grads left untouched)."""
        _check(lib().soar_optim_clip_grad_norm_async(self.handle, max_norm,
                                                      _stream_handle(stream)),
               "soar_optim_clip_grad_norm_async")

    def set_lr(self, lr: float) -> None:
        _check(lib().soar_optim_set_lr(self.handle, lr), "soar_optim_set_lr")

    def get_lr(self) -> float:
        out = C.c_float()
        _check(lib().soar_optim_get_lr(self.handle, C.byref(out)), "soar_optim_get_lr")
        return out.value

    # -- extensions ---------------------------------------------------------
    def info(self, stream=None) -> StepInfo:
        out = StepInfo()
        _check(lib().soar_optim_get_info(self.handle, C.byref(out), _stream_handle(stream)),
               "soar_optim_get_info")
        return out

    def info_async(self, stream=None):
        """Enqueue the bookkeeping readback without synchronising the host.
        Returns (info, event): `info` is a StepInfo in pinned host memory,
        valid once `event` (recorded on the stream after the readback) has
        completed."""
        import torch
        buf = torch.empty(C.sizeof(StepInfo), dtype=torch.uint8).pin_memory()
        _check(lib().soar_optim_get_info_async(self.handle, buf.data_ptr(), _stream_handle(stream)),
               "soar_optim_get_info_async")
        ev = torch.cuda.Event()
        s = torch.cuda.current_stream(self.device) if stream is None else stream
        if isinstance(s, int):
            s = torch.cuda.ExternalStream(s)
        ev.record(s)
        info = StepInfo.from_address(buf.data_ptr())
        info._keepalive = buf
        return info, ev

    def set_counters(self, step: int, skipped: int, loss_scale: float, growth_tracker: int,
                     stream=None) -> None:
        _check(lib().soar_optim_set_counters(self.handle, step, skipped, loss_scale,
                                             growth_tracker, _stream_handle(stream)),
               "soar_optim_set_counters")

    def state_ptr(self, index: int, kind: int) -> int:
        out = C.c_void_p()
        _check(lib().soar_optim_state_ptr(self.handle, index, kind, C.byref(out)),
               "soar_optim_state_ptr")
        return out.value

    def state(self, index: int, kind: int):
        """Zero-copy torch view of tensor `index`'s master / m / v."""
        import torch
        arr = _DeviceArray(self.state_ptr(index, kind), self.numel[index])
        return torch.as_tensor(arr, device=f"cuda:{self.device}")

    def read_state(self, index: int, kind: int):
        import numpy as np
        out = np.empty(self.numel[index], np.float32)
        _check(lib().soar_optim_read_state(self.handle, index, kind, out.ctypes.data),
               "soar_optim_read_state")
        return out

    def write_state(self, index: int, kind: int, values) -> None:
        import numpy as np
        v = np.ascontiguousarray(values, dtype=np.float32)
        if v.size != self.numel[index]:
            raise ValueError("size mismatch")
        _check(lib().soar_optim_write_state(self.handle, index, kind, v.ctypes.data),
               "soar_optim_write_state")

    def enable_ema(self, decay: float = 0.9999, stream=None) -> None:
        """Weight EMA fused into the update (ModelEMA: shadow starts as the weights)."""
        _check(lib().soar_optim_enable_ema(self.handle, decay, _stream_handle(stream)),
               "soar_optim_enable_ema")

    def ema_apply_to(self, stream=None) -> None:
        _check(lib().soar_optim_ema_apply_to(self.handle, _stream_handle(stream)),
               "soar_optim_ema_apply_to")

    def save_state(self, path) -> None:
        """Optimizer-state checkpoint (master/m/v + counters), SOAR v2 records."""
        _check(lib().soar_optim_save_state(self.handle, str(path).encode()),
               "soar_optim_save_state")

    def load_state(self, path, stream=None) -> None:
        _check(lib().soar_optim_load_state(self.handle, str(path).encode(),
                                           _stream_handle(stream)), "soar_optim_load_state")

    def add_grads(self, grads) -> int:
        """Registers another set of gradient buffers (one per tensor, in the
        order the optimizer was created with; None where it had none) and
        returns its index; the creating list is set 0."""
        n = len(self.numel)
        if len(grads) != n:
            raise ValueError(f"{n} gradient buffers expected")
        arr = (C.c_void_p * n)(*[None if g is None else g.data_ptr() for g in grads])
        out = C.c_int()
        _check(lib().soar_optim_add_grads(self.handle, arr, C.byref(out)), "soar_optim_add_grads")
        self._grad_sets = getattr(self, "_grad_sets", []) + [list(grads)]  # keep them alive
        return out.value

    def use_grads(self, index: int) -> None:
        """Makes gradient set `index` the one the next steps use."""
        _check(lib().soar_optim_use_grads(self.handle, index), "soar_optim_use_grads")

    @property
    def kernel_path(self) -> str:
        """'pipeline' (k_apply) or 'direct' (k_apply_direct)."""
        out = C.c_int()
        _check(lib().soar_optim_kernel_path(self.handle, C.byref(out)), "soar_optim_kernel_path")
        return "direct" if out.value == 1 else "pipeline"

    def loss_scale_ptr(self) -> int:
        out = C.c_void_p()
        _check(lib().soar_optim_loss_scale_ptr(self.handle, C.byref(out)),
               "soar_optim_loss_scale_ptr")
        return out.value

    def grad_sumsq(self, out_ptr: int, stream=None) -> None:
        _check(lib().soar_optim_grad_sumsq(self.handle, out_ptr, _stream_handle(stream)),
               "soar_optim_grad_sumsq")

    def apply(self, parts_ptr: int | None, n_parts: int, stream=None) -> None:
        _check(lib().soar_optim_apply(self.handle, parts_ptr, n_parts, _stream_handle(stream)),
               "soar_optim_apply")


class SGD(AdamW):
    """soar::optim::SGD (include/soar/optim/sgd.hpp:21-38) on the same fused
    device step: momentum, dampening, Nesterov, coupled weight decay (per
    ParamGroup), with the same layouts, fused clip and loss scaler. The
    momentum buffer is state kind STATE_M; there is no STATE_V."""

    def __init__(self, params, options: SGDOptions | None = None, *, layout: str = "fp32",
                 max_grad_norm: float = 0.0, loss_scaler: LossScalerOptions | None = None,
                 device: int | None = None, grads=None):
        options = options or SGDOptions()
        o = SGDOpts()
        lib().soar_sgd_default_opts(C.byref(o))
        o.lr, o.momentum, o.dampening = options.lr, options.momentum, options.dampening
        o.weight_decay, o.nesterov = options.weight_decay, int(options.nesterov)
        self._create(params, grads, options.weight_decay, o, layout, max_grad_norm, loss_scaler,
                     device, lib().soar_sgd_create, "soar_sgd_create")


class CosineAnnealingLR:
    """soar::optim::CosineAnnealingLR (adamw.hpp:45-57), bound to an AdamW."""

    def __init__(self, optimizer: AdamW, total_steps: int, eta_min: float = 1e-6,
                 warmup_steps: int = 0):
        self.optimizer = optimizer
        h = C.c_void_p()
        _check(lib().soar_cosine_create(optimizer.handle, total_steps, eta_min, warmup_steps,
                                        C.byref(h)), "soar_cosine_create")
        self.handle = h

    def step(self) -> None:
        _check(lib().soar_cosine_step(self.handle), "soar_cosine_step")

    def close(self):
        if getattr(self, "handle", None):
            lib().soar_cosine_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
