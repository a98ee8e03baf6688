"""Torch restatement of the reference's eager linears -- TEST AND BASELINE INFRASTRUCTURE.

Only ``tests/`` and the CPU-baseline legs of ``bench.py`` use this module. It
restates, op for op in torch, the reference's pure-torch forward of the path
(paths relative to the reference project):

* ``convrot_w4a4_linear``  ``_int4/eager.py:172-197`` (rotation ``:65-79``,
  row-wise int4 quantizer ``:104-120``, ``int4_linear`` ``:154-169``: the
  integer product is formed in the activation dtype, then x-scale, w-scale and
  bias are applied in that dtype)
* ``convrot_w8a8_linear``  ``_int4/int8_eager.py:60-89`` (int8 quantizer
  ``:22-27``; product and epilogue in fp32, one cast at the end)

It is what the reference runs on a host without its HIP kernel, so ``bench.py``
times it as the CPU baseline when the reference package itself is not
installed (``kind: "port"``). The numpy oracle (``convrot_oracle.py``), not
this module, is the bit-level parity checker of the CUDA kernels: the eager
product rounds its accumulators to bf16.
"""
from __future__ import annotations

import math

import torch

_HADAMARD: dict = {}


def hadamard(group: int, dtype: torch.dtype, device="cpu") -> torch.Tensor:
    """kron(H4, ..., H4) / sqrt(group), H4 = ones - 2 * antidiag (``_int4/eager.py:20-46``)."""
    key = (group, dtype, str(device))
    if key not in _HADAMARD:
        h4 = torch.ones(4, 4, dtype=torch.float64) - 2 * torch.eye(4, dtype=torch.float64).flip(1)
        h = h4
        while h.shape[0] < group:
            h = torch.kron(h, h4)
        _HADAMARD[key] = (h / math.sqrt(group)).to(device=device, dtype=dtype)
    return _HADAMARD[key]


def rotate(x2d: torch.Tensor, group: int) -> torch.Tensor:
    """x [M, K] -> per-group x_g @ H in x.dtype (``_int4/eager.py:65-79``)."""
    m, k = x2d.shape
    return torch.matmul(x2d.reshape(m, k // group, group), hadamard(group, x2d.dtype, x2d.device)).reshape(m, k)


def quantize_rowwise(x: torch.Tensor, qmax: int):
    """absmax / qmax scale in x.dtype, round half to even, clamp (``_int4/eager.py:112-120``,
    ``_int4/int8_eager.py:22-27``): (int8 codes [R, C], f32 scale [R])."""
    scale = x.abs().amax(dim=-1, keepdim=True).clamp(min=1e-10) / qmax
    q = (x / scale).round_().clamp_(-qmax, qmax).to(torch.int8)
    return q, scale.reshape(x.shape[0]).to(torch.float32)


def unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    """[R, K/2] int8 -> [R, K] int8; low nibble = even column, sign-extended (``_int4/_codec.py:27-36``)."""
    p = packed.to(torch.int16)
    lo = ((p & 0xF) ^ 8) - 8
    hi = (((p >> 4) & 0xF) ^ 8) - 8
    return torch.stack([lo, hi], dim=-1).reshape(packed.shape[0], -1).to(torch.int8)


def pack_int4(codes: torch.Tensor) -> torch.Tensor:
    """[R, K] codes in [-8, 7] -> [R, K/2] int8, even column in the low nibble (``_int4/_codec.py:19-25``)."""
    c = codes.to(torch.int16) & 0xF
    return (c[:, 0::2] | (c[:, 1::2] << 4)).to(torch.uint8).view(torch.int8)


def convrot_w4a4_linear(x, qweight, wscales, bias=None, convrot_groupsize: int = 256):
    """The reference's eager W4A4 linear: rotate, quantize and pack the activation,
    unpack both operands, product and epilogue in the activation dtype."""
    shape = x.shape
    x2d = x.reshape(-1, shape[-1]).contiguous()
    q, xs = quantize_rowwise(rotate(x2d, convrot_groupsize).contiguous(), 7)
    qact = pack_int4(q)
    dt = x.dtype
    out = unpack_int4(qact).to(dt) @ unpack_int4(qweight).to(dt).t()
    out = out * xs.reshape(-1, 1).to(dt)
    out = out * wscales.reshape(1, -1).to(dt)
    if bias is not None:
        out = out + bias.to(dt).reshape(1, -1)
    return out.reshape(*shape[:-1], qweight.shape[0])


def convrot_w8a8_linear(x, qweight, wscales, bias=None, convrot_groupsize: int = 256):
    """The reference's eager W8A8 linear: int8 activation codes, fp32 product and epilogue."""
    shape = x.shape
    x2d = x.reshape(-1, shape[-1]).contiguous()
    q, xs = quantize_rowwise(rotate(x2d, convrot_groupsize).contiguous(), 127)
    out = q.to(torch.float32) @ qweight.to(torch.float32).t()
    out = out * xs.reshape(-1, 1) * wscales.to(torch.float32).reshape(1, -1)
    if bias is not None:
        out = out + bias.to(torch.float32).reshape(1, -1)
    return out.to(x.dtype).reshape(*shape[:-1], qweight.shape[0])
