"""Signed-int4 nibble codec and quantizer constants of the ConvRot W4A4 format.

Same byte layout as the reference codec (_int4/_codec.py:12-36): a row of K
int4 values is stored as K/2 int8 bytes, column 2j in the low nibble and column
2j+1 in the high nibble, two's complement. The quantizer emits [-7, 7]; -8 is
decodable but never produced, which keeps dequantization symmetric.
"""
from __future__ import annotations

import torch

_INT4_GROUP_SIZE = 64   # divisibility requirement on in_features (not a scale group)
_INT4_MAX = 7           # symmetric range [-7, 7], scale = absmax / 7


def _pack_int4_row_major(values: torch.Tensor) -> torch.Tensor:
    """(..., K) integer values in [-8, 7] -> (..., K // 2) int8."""
    if values.shape[-1] % 2 != 0:
        raise ValueError(f"last dim must be even, got {values.shape[-1]}")
    pairs = values.to(torch.int32).reshape(*values.shape[:-1], values.shape[-1] // 2, 2) & 0xF
    return (pairs[..., 0] | (pairs[..., 1] << 4)).to(torch.uint8).view(torch.int8)


def _unpack_int4_row_major(packed: torch.Tensor) -> torch.Tensor:
    """(..., K // 2) int8 -> (..., K) int8 in [-8, 7] (sign-extended nibbles)."""
    b = packed.view(torch.uint8).to(torch.int32)
    both = torch.stack([b & 0xF, b >> 4], dim=-1)
    both = both - ((both & 0x8) << 1)
    return both.reshape(*packed.shape[:-1], packed.shape[-1] * 2).to(torch.int8)
