"""soar_b200: the B200 (sm_100a) optimizer-step hot path of pomagrenate/soar.cpp.

A drop-in for the reference's soar::optim::AdamW / CosineAnnealingLR update
step: one fused multi-tensor CUDA step (unscale, inf/NaN detect, global norm,
clip, AdamW with per-tensor weight decay on fp32 master/m/v, bf16 write-back,
dynamic loss scaling) behind the C-ABI in include/soar_optim.h, bound here with
ctypes, plus the ZeRO-1 data-parallel driver (dp.py).
"""
from .optim import (SGD, AdamW, AdamWOptions, CosineAnnealingLR, LossScalerOptions, ParamGroup,
                    SGDOptions,
                    SoarError, StepInfo, LAYOUT_FP32, LAYOUT_BF16_MIXED, STATE_MASTER,
                    STATE_M, STATE_V, STATE_EMA, lib, library_path)

__all__ = ["SGD", "SGDOptions", "AdamW", "AdamWOptions", "CosineAnnealingLR", "LossScalerOptions", "ParamGroup",
           "SoarError", "StepInfo", "LAYOUT_FP32", "LAYOUT_BF16_MIXED", "STATE_MASTER",
           "STATE_M", "STATE_V", "STATE_EMA", "lib", "library_path"]
