"""A quantized Linear with the forward contract of the node's operator.

Mirrors ``Int4ConvRotOps.Linear.forward`` and ``_apply_dyn_lora``
(int4_ops.py:366-383, :181-192) without ComfyUI: the weight is held as packed
int4 codes ``_q`` [N, K/2] with per-row scales ``_qs`` [N] and an fp16 bias, and
every forward runs the B200 kernels. Dynamic-LoRA adapters (down [r, K],
up [N, r], alpha, strength) are fused into the GEMM epilogue instead of being
added after it.
"""
from __future__ import annotations

import torch

from . import convrot_w4a4_linear, convrot_w4a4_linear_lora, pick_groupsize
from .eager import quantize_convrot_w4a4_weight


class Int4ConvRotLinear(torch.nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None,
                 convrot_groupsize: int | None = None):
        super().__init__()
        g = convrot_groupsize or pick_groupsize(in_features)
        if g is None or in_features % 64:
            raise ValueError(f"in_features {in_features} is not quantizable (needs a multiple of 64)")
        self.in_features, self.out_features, self._qgs = in_features, out_features, g
        self.register_buffer("_q", torch.zeros(out_features, in_features // 2, dtype=torch.int8, device=device))
        self.register_buffer("_qs", torch.ones(out_features, dtype=torch.float32, device=device))
        self.register_buffer("bias", torch.zeros(out_features, dtype=torch.float16, device=device) if bias else None)
        self._dyn_lora: list[tuple[torch.Tensor, torch.Tensor, float]] = []

    @classmethod
    def from_linear(cls, linear: torch.nn.Linear, stochastic_rounding: int | None = 0,
                    device=None) -> "Int4ConvRotLinear":
        """Quantize like the node's on-the-fly load path: fp16 weight on the device
        (int4_ops.py:340-356), fp16 bias."""
        device = device or linear.weight.device
        mod = cls(linear.in_features, linear.out_features, linear.bias is not None, device=device)
        q, s = quantize_convrot_w4a4_weight(linear.weight.detach().to(device, torch.float16), mod._qgs,
                                            stochastic_rounding=stochastic_rounding)
        mod._q.copy_(q)
        mod._qs.copy_(s)
        if linear.bias is not None:
            mod.bias.copy_(linear.bias.detach().to(device, torch.float16))
        return mod

    def set_dynamic_lora(self, adapters) -> None:
        """adapters: iterable of (down [r, K], up [N, r], alpha, strength); scale = alpha / r * strength."""
        prepared = []
        for down, up, alpha, strength in adapters:
            r = down.shape[0]
            prepared.append((down.to(self._q.device, torch.bfloat16), up.to(self._q.device, torch.bfloat16),
                             float(alpha) / r * float(strength)))
        self._dyn_lora = prepared

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._dyn_lora:
            return convrot_w4a4_linear_lora(x, self._q, self._qs, self.bias, self._dyn_lora, self._qgs)
        return convrot_w4a4_linear(x, self._q, self._qs, self.bias, convrot_groupsize=self._qgs)
