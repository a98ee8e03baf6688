"""Torch (device-agnostic) ConvRot helpers: the load-time weight quantizer.

These functions define the bytes of a quantized weight, so they follow the
reference's eager arithmetic op for op (_int4/eager.py:20-197): the weight is
rotated with a torch matmul in its own dtype (fp16 in the reference loader,
int4_ops.py:342-349) and quantized row-wise in that dtype. Running them on the
same device and dtype as the reference therefore gives byte-identical packed
weights and scales. They are not on the per-step path: ``convrot_w4a4_linear``
in ``_int4/__init__.py`` always runs the CUDA kernels.
"""
from __future__ import annotations

import math

import torch

from ._codec import _INT4_GROUP_SIZE, _INT4_MAX, _pack_int4_row_major, _unpack_int4_row_major

_HADAMARD_CACHE: dict = {}


def _regular_hadamard_signs(size: int) -> torch.Tensor:
    """kron(H4, ..., H4) with H4 = ones(4,4) - 2 * antidiag, as float64 +-1."""
    h4 = torch.ones(4, 4, dtype=torch.float64) - 2 * torch.eye(4, dtype=torch.float64).flip(1)
    h = h4
    while h.shape[0] < size:
        h = torch.kron(h, h4)
    return h


def _build_hadamard(size: int, device="cpu", dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Normalised regular Hadamard matrix of order ``size`` (a power of 4).

    Entries are +-1/sqrt(size), exact powers of two in every float dtype.
    """
    key = (size, str(device), dtype)
    cached = _HADAMARD_CACHE.get(key)
    if cached is not None:
        return cached
    if size < 4 or size & (size - 1) or (size.bit_length() - 1) % 2:
        raise ValueError(f"Regular Hadamard size must be a power of 4, got {size}")
    h = (_regular_hadamard_signs(size) / math.sqrt(size)).to(device=device, dtype=dtype)
    _HADAMARD_CACHE[key] = h
    return h


def _rotate_weight(weight: torch.Tensor, h: torch.Tensor, group_size: int) -> torch.Tensor:
    """W [N, K] -> W_g @ H^T per group of ``group_size`` input channels."""
    n, k = weight.shape
    if k % group_size:
        raise ValueError(f"in_features {k} not divisible by group_size {group_size}")
    grouped = weight.reshape(n, k // group_size, group_size)
    rotated = torch.matmul(grouped, h.T.to(dtype=weight.dtype, device=weight.device))
    return rotated.reshape(n, k)


def _rotate_activation(x: torch.Tensor, h: torch.Tensor, group_size: int) -> torch.Tensor:
    """x [..., K] -> x_g @ H per group, in x.dtype."""
    k = x.shape[-1]
    if k % group_size:
        raise ValueError(f"features {k} not divisible by group_size {group_size}")
    grouped = x.reshape(-1, k // group_size, group_size)
    return torch.matmul(grouped, h.to(dtype=x.dtype, device=x.device)).reshape(x.shape)


def validate_w4a4_shape(tensor: torch.Tensor, convrot_groupsize: int, quant_group_size: int) -> None:
    if tensor.dim() != 2:
        raise ValueError(f"ConvRot W4A4 expects a 2D tensor, got shape {tuple(tensor.shape)}")
    k = tensor.shape[-1]
    if k % convrot_groupsize:
        raise ValueError(f"in_features {k} not divisible by convrot_groupsize {convrot_groupsize}")
    if k % quant_group_size:
        raise ValueError(f"in_features {k} not divisible by quant_group_size {quant_group_size}")


def _round_int4(scaled: torch.Tensor, stochastic_rounding: int | None = 0) -> torch.Tensor:
    """Round half-to-even, or floor(x + U[0,1)) from a generator seeded with
    ``stochastic_rounding`` when it is a positive seed; clamp to [-7, 7]."""
    if stochastic_rounding is not None and stochastic_rounding > 0:
        gen = torch.Generator(device=scaled.device)
        gen.manual_seed(stochastic_rounding)
        noise = torch.rand(scaled.shape, dtype=scaled.dtype, layout=scaled.layout,
                           device=scaled.device, generator=gen)
        return scaled.add_(noise).floor_().clamp_(-_INT4_MAX, _INT4_MAX).to(torch.int8)
    return scaled.round_().clamp_(-_INT4_MAX, _INT4_MAX).to(torch.int8)


def quantize_signed_int4_rowwise(x: torch.Tensor, stochastic_rounding: int | None = 0):
    """Row-wise symmetric int4: (packed int8 [R, C/2], scale f32 [R]), in x.dtype."""
    scale = x.abs().amax(dim=-1, keepdim=True).clamp(min=1e-10) / _INT4_MAX
    codes = _round_int4(x / scale, stochastic_rounding=stochastic_rounding)
    return _pack_int4_row_major(codes), scale.reshape(x.shape[0]).to(torch.float32)


def quantize_convrot_w4a4_weight(weight: torch.Tensor, convrot_groupsize: int = 256,
                                 quant_group_size: int = _INT4_GROUP_SIZE,
                                 stochastic_rounding: int | None = 0):
    """Rotate a weight [N, K] with ConvRot and quantize it to packed signed int4."""
    if quant_group_size != _INT4_GROUP_SIZE:
        raise ValueError(f"int4 MMA kernel requires quant_group_size {_INT4_GROUP_SIZE}")
    validate_w4a4_shape(weight, convrot_groupsize, quant_group_size)
    h = _build_hadamard(convrot_groupsize, device=weight.device, dtype=weight.dtype)
    return quantize_signed_int4_rowwise(_rotate_weight(weight, h, convrot_groupsize),
                                        stochastic_rounding=stochastic_rounding)


def dequantize_convrot_w4a4_weight(qdata: torch.Tensor, scales: torch.Tensor,
                                   convrot_groupsize: int = 256,
                                   quant_group_size: int = _INT4_GROUP_SIZE,
                                   output_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Unpack, rescale and rotate back to the original basis (H is orthogonal, symmetric)."""
    if quant_group_size != _INT4_GROUP_SIZE:
        raise ValueError(f"int4 MMA kernel requires quant_group_size {_INT4_GROUP_SIZE}")
    w = _unpack_int4_row_major(qdata).to(torch.float32)
    w = w * scales.to(device=qdata.device, dtype=torch.float32).reshape(-1, 1)
    h = _build_hadamard(convrot_groupsize, device=qdata.device, dtype=torch.float32)
    return _rotate_weight(w, h, convrot_groupsize).to(output_dtype)
