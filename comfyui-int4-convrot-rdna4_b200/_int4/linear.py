"""A quantized Linear with the forward contract of the node's operator.

Mirrors ``Int4ConvRotOps.Linear.forward`` and ``_apply_dyn_lora``
(int4_ops.py:366-383, :181-192) without ComfyUI: the weight is held as packed
int4 codes ``_q`` [N, K/2] (or int8 codes [N, K] for the W8A8 tier) with
per-row scales ``_qs`` [N] and an fp16 bias, and every forward runs the B200
kernels. Dynamic-LoRA adapters (down [r, K], up [N, r], alpha, strength) are
fused into the int4 GEMM epilogue instead of being added after it.

The state dict is the node's prequantized checkpoint form (``weight``,
``weight_scale``, ``comfy_quant``, ``bias``; see ``_int4.checkpoint``), so
``load_state_dict`` takes the tensors of a file the node saved and
``state_dict`` gives back the same tensors.
"""
from __future__ import annotations

import torch

from . import (checkpoint, convrot_w4a4_linear, convrot_w4a4_linear_lnmod, convrot_w4a4_linear_lora,
               convrot_w8a8_linear_lora, cuda_loader, pick_groupsize)
from .eager import quantize_convrot_w4a4_weight

_CKPT_KEYS = ("weight", "weight_scale", "comfy_quant", "bias")


class Int4ConvRotLinear(torch.nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None,
                 convrot_groupsize: int | None = None, mode: str = "int4"):
        super().__init__()
        g = convrot_groupsize or pick_groupsize(in_features)
        if g is None or in_features % 64:
            raise ValueError(f"in_features {in_features} is not quantizable (needs a multiple of 64)")
        if mode not in ("int4", "int8"):
            raise ValueError(f"mode must be 'int4' or 'int8', got {mode!r}")
        self.in_features, self.out_features, self._qgs, self._qmode = in_features, out_features, g, mode
        cols = in_features // 2 if mode == "int4" else in_features
        self.register_buffer("_q", torch.zeros(out_features, cols, dtype=torch.int8, device=device))
        self.register_buffer("_qs", torch.ones(out_features, dtype=torch.float32, device=device))
        self.register_buffer("bias", torch.zeros(out_features, dtype=torch.float16, device=device) if bias else None)
        self._dyn_lora: list[tuple[torch.Tensor, torch.Tensor, float]] = []

    # ---- checkpoint form (int4_ops.py:223-284 on load, int4_save.py:110-133 on save)
    def _save_to_state_dict(self, destination, prefix, keep_vars):
        def out(t):
            return t if keep_vars else t.detach()
        destination[prefix + "weight"] = out(self._q)
        destination[prefix + "weight_scale"] = out(self._qs.reshape(-1, 1) if self._qmode == "int8" else self._qs)
        destination[prefix + "comfy_quant"] = checkpoint.quant_tag(self._qmode, self._qgs)
        if self.bias is not None:
            destination[prefix + "bias"] = out(self.bias)

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                              unexpected_keys, error_msgs):
        if strict:
            for k in state_dict:
                if k.startswith(prefix) and "." not in k[len(prefix):] and k[len(prefix):] not in _CKPT_KEYS:
                    unexpected_keys.append(k)
        if prefix + "weight" not in state_dict:
            missing_keys.extend(prefix + k for k in ("weight", "weight_scale"))
            return
        had_bias = prefix + "bias" in state_dict
        pw = checkpoint.take_prequantized(state_dict, prefix, self.in_features, device=self._qs.device)
        if pw is None:
            error_msgs.append(f"{prefix}weight: {tuple(state_dict[prefix + 'weight'].shape)} is not a ConvRot "
                              f"int4/int8 layout for in_features={self.in_features}")
            return
        if pw.q.shape[0] != self.out_features or pw.scale.numel() != self.out_features:
            error_msgs.append(f"{prefix}weight: {pw.q.shape[0]} rows, expected out_features={self.out_features}")
            return
        self._q, self._qs, self._qgs, self._qmode = pw.q, pw.scale, pw.groupsize, pw.mode
        if pw.bias is not None:
            self.bias = pw.bias
        elif self.bias is not None and not had_bias:
            missing_keys.append(prefix + "bias")

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
            prepared.append((down.to(self._q.device, torch.float16), up.to(self._q.device, torch.float16),
                             float(alpha) / r * float(strength)))
        self._dyn_lora = prepared

    def forward_lnmod(self, x: torch.Tensor, shift: torch.Tensor | None, scale: torch.Tensor | None,
                      eps: float = 1e-6) -> torch.Tensor:
        """``self((1 + scale) * layer_norm(x) + shift)``, the input a Flux block feeds its QKV and
        MLP-up projections. Plain int4 layers on bf16 rows of whole tiles run it in one pass
        over x (``_int4.convrot_w4a4_linear_lnmod``: the normalised rows never reach memory);
        int8 layers and layers with Dynamic-LoRA adapters normalise in torch first."""
        if self._qmode == "int4" and not self._dyn_lora and cuda_loader.lnmod_supported(x, self._qgs):
            return convrot_w4a4_linear_lnmod(x, self._q, self._qs, self.bias, shift=shift, scale=scale, eps=eps,
                                             convrot_groupsize=self._qgs)
        xn = torch.nn.functional.layer_norm(x, (x.shape[-1],), eps=eps)
        if scale is not None:
            xn = xn * (1 + scale)
        if shift is not None:
            xn = xn + shift
        return self(xn)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._qmode == "int8":
            return convrot_w8a8_linear_lora(x, self._q, self._qs, self.bias, self._dyn_lora, self._qgs)
        if self._dyn_lora:
            return convrot_w4a4_linear_lora(x, self._q, self._qs, self.bias, self._dyn_lora, self._qgs)
        return convrot_w4a4_linear(x, self._q, self._qs, self.bias, convrot_groupsize=self._qgs)
