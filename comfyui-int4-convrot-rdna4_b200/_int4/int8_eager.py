"""Torch ConvRot W8A8 helpers (the int8 middle tier of mixed precision).

Same rotation as int4; plain int8 storage [N, K] and scale = absmax / 127
(reference: _int4/int8_eager.py:19-57). These define the bytes of int8 layers
and of the activation codes where the fused kernel does not apply; the W8A8
forward itself is ``_int4.convrot_w8a8_linear`` (CUDA kernels only).
"""
from __future__ import annotations

import torch

from .eager import _build_hadamard, _rotate_weight

_INT8_MAX = 127


def quantize_signed_int8_rowwise(x: torch.Tensor):
    """Row-wise symmetric int8: (int8 [R, C], scale f32 [R]), in x.dtype."""
    scale = x.abs().amax(dim=-1, keepdim=True).clamp(min=1e-10) / _INT8_MAX
    q = (x / scale).round_().clamp_(-_INT8_MAX, _INT8_MAX).to(torch.int8)
    return q, scale.reshape(x.shape[0]).to(torch.float32)


def quantize_convrot_w8a8_weight(weight: torch.Tensor, convrot_groupsize: int):
    if weight.dim() != 2:
        raise ValueError(f"ConvRot W8A8 expects a 2D tensor, got {tuple(weight.shape)}")
    if weight.shape[-1] % convrot_groupsize:
        raise ValueError(f"in_features {weight.shape[-1]} not divisible by "
                         f"convrot_groupsize {convrot_groupsize}")
    h = _build_hadamard(convrot_groupsize, device=weight.device, dtype=weight.dtype)
    return quantize_signed_int8_rowwise(_rotate_weight(weight, h, convrot_groupsize))


def dequantize_convrot_w8a8_weight(qdata: torch.Tensor, scales: torch.Tensor, convrot_groupsize: int,
                                   output_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    w = qdata.to(torch.float32) * scales.to(qdata.device, torch.float32).reshape(-1, 1)
    h = _build_hadamard(convrot_groupsize, device=qdata.device, dtype=torch.float32)
    return _rotate_weight(w, h, convrot_groupsize).to(output_dtype)

