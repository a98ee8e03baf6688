"""ConvRot W4A4 forward path for NVIDIA B200 (sm_100a).

Drop-in replacement for the ``_int4`` package of ComfyUI-INT4-ConvRot-RDNA4
(reference API: _int4/__init__.py:9-14, :35-42). The node code calls

    quantize_convrot_w4a4_weight(weight, convrot_groupsize) -> (qweight_i8, scale_f32)
    convrot_w4a4_linear(x, qweight, wscales, bias, convrot_groupsize) -> tensor
    is_available() -> bool          # sm_100 device + loadable CUDA library
    pick_groupsize(in_features) -> int | None

with the same signatures, packed-weight layout and errors. Every int4 forward
runs two CUDA kernels from libconvrot_b200.so (fused rotate+quantize, then the
tcgen05 GEMM with the dequant/bias epilogue); there is no torch or CPU
fallback, so a missing library raises.
"""
from __future__ import annotations

import torch

from ._codec import _INT4_GROUP_SIZE
from . import cuda_loader, weight_cache
from .cuda_loader import convrot_quant_int4, int4_convrot_gemm, int4_convrot_gemm_lora
from .cuda_loader import convrot_quant_int8, int8_convrot_gemm
from .cuda_loader import is_available as _lib_available
from .eager import (
    _build_hadamard,
    _rotate_activation,
    dequantize_convrot_w4a4_weight,
    quantize_convrot_w4a4_weight,
    quantize_signed_int4_rowwise,
)
from .int8_eager import quantize_signed_int8_rowwise as _quantize_int8_rowwise

__all__ = [
    "quantize_convrot_w4a4_weight",
    "dequantize_convrot_w4a4_weight",
    "convrot_w4a4_linear",
    "convrot_w8a8_linear",
    "convrot_w4a4_linear_lora",
    "set_unpacked_weights",
    "is_available",
    "pick_groupsize",
]

# Output dtypes the GEMM epilogue writes directly; others compute f32 then cast.
_NATIVE_OUT = frozenset({torch.float32, torch.bfloat16})
# With the unpacked-weight cache switched on (opt-in), layers run on unpacked
# codes (int8 pipeline) from this many rows, and few-row layers (N <= _FEW_ROWS_N:
# a dozen swapped 256-row tiles leave most SMs idle) already from 5 tokens once
# M * K >= _FEW_ROWS_MIN_MK (measured on 3072 x 3072 .. 12288 x 4096 weights).
# Without it, ck_convrot_w4a4_linear picks the form itself: the A8 form (int8
# activation codes, packed weights) for 129+ bf16 rows, packed codes below.
_UNPACKED_MIN_ROWS = 129
_FEW_ROWS_N = 4096
_FEW_ROWS_MIN_MK = 8 * 12288
# rows from which the LoRA linear runs the A8 form (the fused linear's threshold)
_A8_MIN_ROWS = 129


def _use_unpacked(x2d: torch.Tensor, qweight: torch.Tensor, convrot_groupsize: int) -> bool:
    """Whether this call runs on cached unpacked weight codes (the opt-in cache)."""
    if not weight_cache.enabled():
        return False
    m, k = x2d.shape
    few_rows = qweight.shape[0] <= _FEW_ROWS_N and m >= 5 and m * k >= _FEW_ROWS_MIN_MK
    if m < _UNPACKED_MIN_ROWS and not few_rows:
        return False
    return cuda_loader.unpacked_path_supported(x2d, convrot_groupsize)


def _use_a8(x2d: torch.Tensor, convrot_groupsize: int) -> bool:
    return x2d.shape[0] >= _A8_MIN_ROWS and cuda_loader.unpacked_path_supported(x2d, convrot_groupsize)


def set_unpacked_weights(enabled: bool = True) -> None:
    """Opt in to (or out of, the default) cached unpacked weight copies: faster
    many-token layers at twice the weight bytes."""
    weight_cache.enable(enabled)


def pick_groupsize(in_features: int) -> int | None:
    """Largest supported ConvRot group size (256, 64, 16) dividing in_features."""
    for g in (256, 64, 16):
        if in_features % g == 0:
            return g
    return None


def _is_sm100() -> bool:
    if not torch.cuda.is_available():
        return False
    try:
        major, _minor = torch.cuda.get_device_capability(0)
    except Exception:
        return False
    return major == 10


def is_available() -> bool:
    """True only on an sm_100 (B200-class) CUDA device with a loadable library."""
    return _is_sm100() and _lib_available()


def _validate(x, qweight, convrot_groupsize, quant_group_size, linear_dtype) -> None:
    if linear_dtype not in ("int4", "int8"):
        raise ValueError(f"ConvRot W4A4 linear_dtype must be 'int4' or 'int8', got {linear_dtype!r}")
    if quant_group_size != _INT4_GROUP_SIZE:
        raise ValueError(f"int4 MMA kernel requires quant_group_size {_INT4_GROUP_SIZE}")
    if x.shape[-1] != qweight.shape[-1] * 2:
        raise ValueError(f"Input K={x.shape[-1]} does not match qweight K={qweight.shape[-1] * 2}")
    if x.shape[-1] % convrot_groupsize != 0:
        raise ValueError(f"Input K={x.shape[-1]} not divisible by convrot_groupsize {convrot_groupsize}")


def convrot_w4a4_linear(
    x: torch.Tensor,
    qweight: torch.Tensor,
    wscales: torch.Tensor,
    bias: torch.Tensor | None = None,
    convrot_groupsize: int = 256,
    quant_group_size: int = _INT4_GROUP_SIZE,
    linear_dtype: str = "int4",
) -> torch.Tensor:
    """``x @ W.T + bias`` through the B200 int4 ConvRot kernels.

    x [..., K] (bf16, fp16 or fp32, CUDA), qweight int8 [N, K/2] packed,
    wscales [N], bias [N] or None. Returns [..., N] in x.dtype.
    ``linear_dtype='int8'`` is accepted like the reference, whose eager path
    computes the same int4 product for it (_int4/eager.py:172-197).
    """
    _validate(x, qweight, convrot_groupsize, quant_group_size, linear_dtype)
    shape = x.shape
    x2d = x.reshape(-1, shape[-1]).contiguous()
    out_dtype = x.dtype if x.dtype in _NATIVE_OUT else torch.float32
    if _use_unpacked(x2d, qweight, convrot_groupsize):
        # opt-in cache: both operands as int8 codes on the int8 tensor-core pipeline
        # (same accumulators, same results); the weight's codes are cached
        codes = weight_cache.unpacked(qweight)
        out = cuda_loader.convrot_w4a4_linear_unpacked(x2d, codes, wscales, bias, out_dtype, convrot_groupsize)
    else:
        # packed weights; the fused entry picks the A8 form for many bf16 rows
        out = cuda_loader.convrot_w4a4_linear(x2d, qweight, wscales, bias, out_dtype, convrot_groupsize)
    if out.dtype != x.dtype:
        out = out.to(x.dtype)
    return out.reshape(*shape[:-1], qweight.shape[0])


def convrot_w4a4_linear_lnmod(
    x: torch.Tensor,
    qweight: torch.Tensor,
    wscales: torch.Tensor,
    bias: torch.Tensor | None = None,
    shift: torch.Tensor | None = None,
    scale: torch.Tensor | None = None,
    eps: float = 1e-6,
    convrot_groupsize: int = 256,
) -> torch.Tensor:
    """``convrot_w4a4_linear((1 + scale) * LayerNorm(x) + shift, ...)`` in one pass over x.

    The rotation moved into the producer of x: a Flux block's QKV and MLP-up
    projections take ``(1 + mod.scale) * norm(x) + mod.shift`` (LayerNorm
    without affine, eps 1e-6), and here the normalisation and modulation run in
    the kernel that rotates and quantizes the rows, so the normalised bf16
    tensor never goes to memory. x bf16 [..., K] (K % 256 == 0, K <= 6144), shift /
    scale bf16 [K] (one vector for all rows; None = zeros). The statistics use a
    fixed fp32 order (``ck_convrot_quant_int4_lnmod``), within rounding of
    torch's LayerNorm. Returns [..., N] in bf16.
    """
    _validate(x, qweight, convrot_groupsize, _INT4_GROUP_SIZE, "int4")
    if not cuda_loader.lnmod_supported(x, convrot_groupsize):
        raise ValueError("the fused LayerNorm linear takes bf16 CUDA rows of whole 256-column tiles "
                         "(K <= 6144, convrot_groupsize 64 or 256)")
    shape = x.shape
    x2d = x.reshape(-1, shape[-1]).contiguous()
    out = cuda_loader.convrot_w4a4_linear_lnmod(x2d, qweight, wscales, bias, scale, shift, eps, torch.bfloat16,
                                                convrot_groupsize)
    return out.reshape(*shape[:-1], qweight.shape[0])


_MAX_LORA_RANK = 64
# Unit roundoff of the side path's operand type (T = x.A^T and B enter the
# tensor cores in fp16, the reference's adapter dtype, int4_ops.py:165-167): the
# bound a caller's tolerance on the LoRA term needs.
LORA_OPERAND_UNIT = 2.0 ** -11


def convrot_w4a4_linear_lora(
    x: torch.Tensor,
    qweight: torch.Tensor,
    wscales: torch.Tensor,
    bias: torch.Tensor | None,
    adapters,
    convrot_groupsize: int = 256,
) -> torch.Tensor:
    """``convrot_w4a4_linear`` plus Dynamic-LoRA side paths fused into the GEMM epilogue.

    adapters: iterable of (down [r, K], up [N, r], scale) with scale = (alpha / r) * strength,
    the low-rank "bypass" of the node's forward (int4_ops.py:181-192). The down
    projection T = fp16(x) @ down^T runs on the tensor cores (ck_lora_down: x read
    once, converted to fp16 in shared memory, fp32 accumulation); the up projection and the add
    run on fp16 tensor-core MMAs inside the int4 GEMM, fp32 accumulation, added
    before the single output rounding (the reference adds the adapter's output to
    the already rounded int4 output, int4_ops.py:183-192; one rounding is the
    more accurate of the two and a deliberate difference). The adapters are in
    fp16, as the reference prepares them (int4_ops.py:165-167). Several adapters
    are stacked along the rank (total rank <= 64); with more than one, each scale
    is folded into its up matrix in fp16.
    """
    adapters = list(adapters)
    if not adapters:
        return convrot_w4a4_linear(x, qweight, wscales, bias, convrot_groupsize)
    _validate(x, qweight, convrot_groupsize, _INT4_GROUP_SIZE, "int4")
    shape = x.shape
    x2d = x.reshape(-1, shape[-1]).contiguous()
    lora_t, up, scale = _lora_operands(x2d, adapters, qweight.shape[0])
    out_dtype = x.dtype if x.dtype in _NATIVE_OUT else torch.float32
    if _use_unpacked(x2d, qweight, convrot_groupsize):
        qact, x_scale = cuda_loader.convrot_quant_int4_unpacked(x2d, convrot_groupsize)
        out = cuda_loader.int8_convrot_gemm_lora(qact, weight_cache.unpacked(qweight), x_scale, wscales, bias,
                                                 out_dtype, lora_t, up, scale)
    elif _use_a8(x2d, convrot_groupsize):
        qact, x_scale = cuda_loader.convrot_quant_int4_unpacked(x2d, convrot_groupsize)
        out = cuda_loader.int4_convrot_gemm_a8(qact, qweight, x_scale, wscales, bias, out_dtype, lora_t, up, scale)
    else:
        qact, x_scale = convrot_quant_int4(x2d, convrot_groupsize)
        out = int4_convrot_gemm_lora(qact, qweight, x_scale, wscales, bias, out_dtype, lora_t, up, scale)
    if out.dtype != x.dtype:
        out = out.to(x.dtype)
    return out.reshape(*shape[:-1], qweight.shape[0])


def _lora_operands(x2d: torch.Tensor, adapters, n: int):
    """(T = fp16(x) @ down^T [M, r] fp16, up [N, r] fp16, scale) for the fused side path;
    several adapters are stacked along the rank, each scale folded into its up
    matrix in fp16; the rank is padded to a multiple of 8."""
    if len(adapters) == 1:
        down, up, scale = adapters[0]
        down = down.to(device=x2d.device, dtype=torch.float16)
        up = up.to(device=x2d.device, dtype=torch.float16)
    else:
        down = torch.cat([d.to(device=x2d.device, dtype=torch.float16) for d, _, _ in adapters], dim=0)
        up = torch.cat([(u.to(device=x2d.device, dtype=torch.float32) * float(s)).to(torch.float16)
                        for _, u, s in adapters], dim=1)
        scale = 1.0
    rank = down.shape[0]
    if rank > _MAX_LORA_RANK or up.shape != (n, rank) or down.shape[1] != x2d.shape[-1]:
        raise ValueError(f"LoRA down {tuple(down.shape)} / up {tuple(up.shape)} do not fit this layer "
                         f"(total rank must be <= {_MAX_LORA_RANK})")
    pad = (-rank) % 8
    if pad:
        down = torch.nn.functional.pad(down, (0, 0, 0, pad))
        up = torch.nn.functional.pad(up, (0, pad))
    return cuda_loader.lora_down(x2d, down), up, scale


def convrot_w8a8_linear(
    x: torch.Tensor,
    qweight: torch.Tensor,
    wscales: torch.Tensor,
    bias: torch.Tensor | None = None,
    convrot_groupsize: int = 256,
) -> torch.Tensor:
    """``x @ W.T + bias`` for int8 ConvRot layers (qweight int8 [N, K], wscales [N]) -- the W8A8
    middle tier (reference: _int4/__init__.py:141-175).

    bf16 rows of whole 256-column tiles (G = 64/256) are rotated and int8-quantized by
    one kernel (ck_convrot_quant_int8); other activations take the torch rotation and
    quantizer on the device, as the reference's layer does where its fused kernel does
    not apply. The product always runs on the int8 tensor cores (ck_int8_convrot_gemm).
    """
    return convrot_w8a8_linear_lora(x, qweight, wscales, bias, (), convrot_groupsize)


def convrot_w8a8_linear_lora(x, qweight, wscales, bias, adapters, convrot_groupsize: int = 256) -> torch.Tensor:
    """``convrot_w8a8_linear`` plus Dynamic-LoRA side paths (as ``convrot_w4a4_linear_lora``)
    fused into the int8 GEMM's epilogue; no adapters: the plain W8A8 linear."""
    if x.shape[-1] != qweight.shape[-1]:
        raise ValueError(f"Input K={x.shape[-1]} does not match qweight K={qweight.shape[-1]}")
    if x.shape[-1] % convrot_groupsize != 0:
        raise ValueError(f"Input K={x.shape[-1]} not divisible by convrot_groupsize {convrot_groupsize}")
    if not x.is_cuda:
        raise ValueError("the B200 ConvRot kernels need CUDA tensors")
    adapters = list(adapters)
    shape = x.shape
    x2d = x.reshape(-1, shape[-1]).contiguous()
    lora = _lora_operands(x2d, adapters, qweight.shape[0]) if adapters else None
    if cuda_loader.int8_quant_supported(x2d, convrot_groupsize):
        qact, x_scale = cuda_loader.convrot_quant_int8(x2d, convrot_groupsize)
    else:
        h = _build_hadamard(convrot_groupsize, device=x2d.device, dtype=x2d.dtype)
        qact, x_scale = _quantize_int8_rowwise(_rotate_activation(x2d, h, convrot_groupsize).contiguous())
    out_dtype = x.dtype if x.dtype in _NATIVE_OUT else torch.float32
    if lora is not None:
        out = cuda_loader.int8_convrot_gemm_lora(qact, qweight, x_scale, wscales, bias, out_dtype, *lora)
    else:
        out = cuda_loader.int8_convrot_gemm(qact, qweight, x_scale, wscales, bias, out_dtype)
    if out.dtype != x.dtype:
        out = out.to(x.dtype)
    return out.reshape(*shape[:-1], qweight.shape[0])
