"""CPU oracle for the ConvRot W4A4 linear path -- TEST INFRASTRUCTURE ONLY.

This module is the parity checker for the B200 kernels. Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
it. The product path (``_int4`` and the CUDA library) never calls it and fails
loudly when the CUDA library is missing.

It restates, in numpy, the reference algorithm of
0xDELUXA/ComfyUI-INT4-ConvRot-RDNA4 (paths below are relative to that project):

* Hadamard matrix            ``_int4/eager.py:20-46``
* activation rotation        ``_int4/eager.py:65-79``  (x.reshape(-1,K/G,G) @ H)
* row-wise int4 quantizer    ``_int4/eager.py:104-120`` (absmax/7, round half even, clamp +-7)
* nibble codec               ``_int4/_codec.py:19-36``  (low nibble = even column)
* fused rotate+quant kernel  ``_int4/int4_gemm.hip:348-408`` (radix-4 fp32 butterflies)
* int4 GEMM + epilogue       ``_int4/int4_gemm.hip:152-169`` (acc*xs*ws + bias in fp32)

Pinning: the tests in ``tests/test_oracle_golden.py`` check every function here
against golden vectors produced by running the reference's own eager code
(``tests/golden/make_golden.py``); the reference ships no golden vectors of its own.

Rounding contract (what "bit-exact" means for this path):

* Rotation: each 256-element tile is a 16x16 matrix ``A[a][b]`` (i = 16a + b).
  The kernel applies H4 along b0, then b1, then (G=256) a0, a1 or (G=64) a0,
  each H4 step as ``S = (v0+v1)+(v2+v3); out_i = S - 2*v_(3-i)`` in IEEE fp32
  (the subtraction is one rounding: it is an FMA with an exact -2*v).  The
  result is scaled by 1/sqrt(G) (a power of two, exact) and rounded once to the
  activation dtype.  ``rotate`` below performs exactly these operations.
* Quantizer: the eager arithmetic in the activation dtype: absmax (exact),
  clamp(min=1e-10) (in the dtype), ``scale = dtype(fp32(absmax/7))``,
  ``q = rint(dtype(fp32(x/scale)))`` clamped to +-7.
* GEMM: exact integer dot products; epilogue ``((float(D) * xs) * ws) + bias``
  in IEEE fp32, then one rounding to the output dtype.
"""
from __future__ import annotations

import math

import numpy as np

INT4_MAX = 7
INT8_MAX = 127
QUANT_GROUP_SIZE = 64          # _int4/_codec.py:15 -- divisibility only, not a scale group
SUPPORTED_GROUPS = (256, 64, 16)

# ---------------------------------------------------------------------------
# 16-bit float helpers (bf16 has no numpy dtype; it travels as uint16 bits)
# ---------------------------------------------------------------------------


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 values (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (NaN kept quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), rounded)
    return rounded


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 value, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def round_to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to the activation dtype and return them as float32."""
    if dtype == "bf16":
        return round_to_bf16(x)
    if dtype == "f16":
        with np.errstate(over="ignore"):
            return x.astype(np.float16).astype(np.float32)
    if dtype == "f32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(f"unknown dtype {dtype!r}")


def to_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    """Activation storage (uint16 bits for bf16, float16, float32) -> float32."""
    if dtype == "bf16":
        return bf16_bits_to_f32(x)
    return np.asarray(x).astype(np.float32)


def from_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values already representable in ``dtype`` -> storage array."""
    if dtype == "bf16":
        return f32_to_bf16_bits(x)
    if dtype == "f16":
        return x.astype(np.float16)
    return np.asarray(x, dtype=np.float32)


# ---------------------------------------------------------------------------
# Hadamard (``_int4/eager.py:20-46``)
# ---------------------------------------------------------------------------

_H4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.int8)


def pick_groupsize(in_features: int) -> int | None:
    """Largest of 256/64/16 dividing ``in_features`` (``_int4/__init__.py:69-74``)."""
    for g in SUPPORTED_GROUPS:
        if in_features % g == 0:
            return g
    return None


def hadamard_signs(size: int) -> np.ndarray:
    """kron(H4, ..., H4) as an int8 +-1 matrix; ``size`` must be a power of 4 >= 4."""
    if size < 4 or size & (size - 1) or round(math.log(size, 4)) != math.log(size, 4):
        raise ValueError(f"Regular Hadamard size must be a power of 4, got {size}")
    h = _H4
    while h.shape[0] < size:
        h = np.kron(h, _H4).astype(np.int8)
    return h


def hadamard(size: int) -> np.ndarray:
    """Normalised regular Hadamard kron(H4,...)/sqrt(size) in float64."""
    return hadamard_signs(size).astype(np.float64) / math.sqrt(size)


# ---------------------------------------------------------------------------
# Rotation: the fixed fp32 radix-4 butterfly order of the CUDA kernel
# ---------------------------------------------------------------------------


def _h4_step(v: np.ndarray, axis: int) -> np.ndarray:
    """One H4 application along a length-4 axis, in the kernel's fp32 order."""
    v0, v1, v2, v3 = (np.take(v, i, axis=axis) for i in range(4))
    s = (v0 + v1) + (v2 + v3)
    two = np.float32(2.0)
    return np.stack([s - two * v3, s - two * v2, s - two * v1, s - two * v0], axis=axis)


def rotate_f32(x: np.ndarray, group: int) -> np.ndarray:
    """ConvRot rotation of ``x`` [M, K] (float32 values) in fp32, before rounding.

    K must be a multiple of ``group``. Works on 256-element tiles (16x16,
    i = 16a + b); a K that is not a multiple of 256 (group 16 or 64) is padded
    with zeros to the next tile, which changes no value of the real groups.
    """
    if group not in SUPPORTED_GROUPS:
        raise ValueError(f"group must be one of {SUPPORTED_GROUPS}, got {group}")
    x = np.asarray(x, dtype=np.float32)
    m, k = x.shape
    if k % group:
        raise ValueError(f"K={k} not divisible by group {group}")
    kp = -(-k // 256) * 256
    if kp != k:
        x = np.concatenate([x, np.zeros((m, kp - k), np.float32)], axis=1)
    # axes: (m, tile, a1, a0, b1, b0)
    t = x.reshape(m, kp // 256, 4, 4, 4, 4)
    t = _h4_step(t, 5)          # b0
    t = _h4_step(t, 4)          # b1
    if group >= 64:
        t = _h4_step(t, 3)      # a0
    if group == 256:
        t = _h4_step(t, 2)      # a1
    t = t * np.float32(1.0 / math.sqrt(group))
    return np.ascontiguousarray(t.reshape(m, kp)[:, :k])


def rotate(x: np.ndarray, group: int, dtype: str = "bf16") -> np.ndarray:
    """Rotated activation rounded to ``dtype``; input/outputs in storage form."""
    return from_f32(round_to_dtype(rotate_f32(to_f32(x, dtype), group), dtype), dtype)


# ---------------------------------------------------------------------------
# Quantizer (``_int4/eager.py:104-120``) and codec (``_int4/_codec.py:19-36``)
# ---------------------------------------------------------------------------


def quantize_rowwise(xr: np.ndarray, dtype: str = "bf16") -> tuple[np.ndarray, np.ndarray]:
    """Eager row-wise symmetric int4 quantizer in the activation dtype.

    Returns (codes int8 [M, K] in [-7, 7], scale float32 [M]).
    """
    return _quantize_rowwise(xr, dtype, INT4_MAX)


def quantize_rowwise_int8(xr: np.ndarray, dtype: str = "bf16") -> tuple[np.ndarray, np.ndarray]:
    """Eager row-wise symmetric int8 quantizer of the W8A8 tier
    (``_int4/int8_eager.py:22-27``): the int4 arithmetic with 127 for 7.

    Returns (codes int8 [M, K] in [-127, 127], scale float32 [M]).
    """
    return _quantize_rowwise(xr, dtype, INT8_MAX)


def _quantize_rowwise(xr: np.ndarray, dtype: str, qmax: int) -> tuple[np.ndarray, np.ndarray]:
    v = to_f32(xr, dtype)
    absmax = np.abs(v).max(axis=1, keepdims=True) if v.shape[1] else np.zeros((v.shape[0], 1), np.float32)
    floor = round_to_dtype(np.array([1e-10], np.float32), dtype)[0]
    absmax = np.maximum(absmax, floor)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        scale = round_to_dtype(absmax / np.float32(qmax), dtype)
        t = round_to_dtype(v / scale, dtype)
    # An all-zero fp16 row has scale 0 (the 1e-10 floor underflows in fp16), so its
    # values are 0/0 = NaN; the reference's NaN -> int8 cast gives code 0 there
    # (row 3 of the golden case q_g256_f16 in tests/golden/int8.npz).
    t = np.where(np.isnan(t), np.float32(0), t)
    q = np.clip(np.rint(t), -qmax, qmax).astype(np.int8)
    return q, scale.reshape(-1).astype(np.float32)


def layernorm_modulate(x_bits: np.ndarray, scale_bits=None, shift_bits=None, eps: float = 1e-6) -> np.ndarray:
    """(1 + scale) * LayerNorm(x) + shift of bf16 rows (storage bits in, bits out).

    The producer of x before a Flux block's QKV and MLP-up projections (LayerNorm
    without affine, biased variance; per-channel modulation vectors [K]), in the
    fixed fp32 order of the fused kernel ``ck_convrot_quant_int4_lnmod``: the row
    is cut into 128-value segments (half a 256-column tile each, in order); a
    segment's sum is a binary tree over its sixteen 8-value chunks of binary-tree
    chunk sums; the segment sums are added in order; mean = sum / K; the squared
    deviations (x - mean)^2 (two roundings) the same way; rstd =
    1 / sqrt(var + eps), each step rounded; xn = bf16((x - mean) * rstd);
    y = bf16(bf16(bf16(1 + scale) * xn) + shift). The model code behind it
    (ComfyUI's Flux blocks) is not part of the reference; this is the fused
    kernel's own definition, close to torch.nn.functional.layer_norm followed
    by the bf16 modulation (``tests/test_oracle_lnmod.py``).
    """
    f32 = np.float32
    v = bf16_bits_to_f32(x_bits)
    m, k = v.shape
    if k % 256:
        raise ValueError("K must be a multiple of 256")

    def warp_sum(vals):
        c = vals.reshape(m, k // 128, 16, 8)
        while c.shape[-1] > 1:                      # chunk sums: pairs, quads, all 8
            c = (c[..., 0::2] + c[..., 1::2]).astype(f32)
        c = c[..., 0]
        while c.shape[-1] > 1:                      # segment sums over the 16 chunks
            c = (c[..., 0::2] + c[..., 1::2]).astype(f32)
        part = c[..., 0]
        acc = part[:, 0]
        for i in range(1, part.shape[1]):
            acc = (acc + part[:, i]).astype(f32)
        return acc

    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        mean = (warp_sum(v) / f32(k)).astype(f32)
        d = (v - mean[:, None]).astype(f32)
        var = (warp_sum((d * d).astype(f32)) / f32(k)).astype(f32)
        rstd = (f32(1.0) / np.sqrt((var + f32(eps)).astype(f32))).astype(f32)
        xn = round_to_bf16((d * rstd[:, None]).astype(f32))
        s1 = np.ones(k, f32) if scale_bits is None else round_to_bf16((f32(1.0) + bf16_bits_to_f32(scale_bits)).astype(f32))
        sh = np.zeros(k, f32) if shift_bits is None else bf16_bits_to_f32(shift_bits)
        t2 = round_to_bf16((s1[None, :] * xn).astype(f32))
        y = round_to_bf16((t2 + sh[None, :]).astype(f32))
    return f32_to_bf16_bits(y)


def convrot_quant_int4_lnmod(x_bits, scale_bits, shift_bits, eps: float, group: int):
    """Packed codes and scales of the modulated LayerNorm of x (``ck_convrot_quant_int4_lnmod``)."""
    return convrot_quant_int4(layernorm_modulate(x_bits, scale_bits, shift_bits, eps), group, "bf16")


def pack_int4(codes: np.ndarray) -> np.ndarray:
    """[..., K] int4 values -> [..., K/2] int8; even column in the low nibble."""
    codes = np.asarray(codes)
    if codes.shape[-1] % 2:
        raise ValueError(f"last dim must be even, got {codes.shape[-1]}")
    c = codes.astype(np.int32)
    lo = c[..., 0::2] & 0xF
    hi = c[..., 1::2] & 0xF
    return (lo | (hi << 4)).astype(np.uint8).view(np.int8)


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """Inverse of ``pack_int4``; nibbles are read as two's complement [-8, 7]."""
    p = np.asarray(packed).astype(np.int8).view(np.uint8).astype(np.int32)
    lo = p & 0xF
    hi = p >> 4
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), np.int8)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out


def convrot_quant_int4(x: np.ndarray, group: int, dtype: str = "bf16") -> tuple[np.ndarray, np.ndarray]:
    """Fused rotation + quantization + packing: (packed int8 [M,K/2], scale f32 [M])."""
    q, s = quantize_rowwise(rotate(x, group, dtype), dtype)
    return pack_int4(q), s


def quant_int4_prerotated(xr: np.ndarray, dtype: str = "bf16") -> tuple[np.ndarray, np.ndarray]:
    """Quantize + pack an already rotated activation (rotation skipped)."""
    q, s = quantize_rowwise(xr, dtype)
    return pack_int4(q), s


# ---------------------------------------------------------------------------
# GEMM (``_int4/int4_gemm.hip:152-169``)
# ---------------------------------------------------------------------------


def int4_gemm_acc(xp: np.ndarray, wp: np.ndarray) -> np.ndarray:
    """Exact int32 accumulators D[m, n] = sum_k X[m,k] * W[n,k] of packed codes.

    float32 BLAS is exact here: products are <= 64 and every partial sum stays
    below 2**24 for K < 262144, so any summation order gives the same integers.
    """
    xi = unpack_int4(xp).astype(np.float32)
    wi = unpack_int4(wp).astype(np.float32)
    if xi.shape[1] >= 262144:
        raise ValueError("K too large for the exact float32 oracle")
    return (xi @ wi.T).astype(np.int32)


def int8_gemm_acc(xq: np.ndarray, wq: np.ndarray) -> np.ndarray:
    """Exact int32 accumulators D[m, n] = sum_k X[m,k] * W[n,k] of int8 values
    (``_int4/int4_gemm.hip:421-492``). float64 BLAS is exact: |products| <= 2**14
    and |D| < 2**31 < 2**53 for K <= 65536."""
    xi = np.asarray(xq).astype(np.int8).astype(np.float64)
    wi = np.asarray(wq).astype(np.int8).astype(np.float64)
    if xi.shape[1] > 65536:
        raise ValueError("K too large for int32 accumulators")
    return (xi @ wi.T).astype(np.int32)


def convrot_quant_int8(x: np.ndarray, group: int, dtype: str = "bf16") -> tuple[np.ndarray, np.ndarray]:
    """W8A8 activation path: rotation, then the int8 quantizer (codes not packed)."""
    return quantize_rowwise_int8(rotate(x, group, dtype), dtype)


def int4_gemm_epilogue(acc: np.ndarray, xs: np.ndarray, ws: np.ndarray,
                       bias: np.ndarray | None, out_dtype: str = "bf16") -> np.ndarray:
    """out = ((float(D) * xs[m]) * ws[n]) + bias[n] in fp32, rounded to out_dtype.

    Returns float32 values for out_dtype 'f32', bf16 bit patterns for 'bf16'.
    """
    v = acc.astype(np.float32) * np.asarray(xs, np.float32).reshape(-1, 1)
    v = v * np.asarray(ws, np.float32).reshape(1, -1)
    # The reference kernel always adds (bias or 0.0f): -0.0 becomes +0.0.
    v = v + (np.asarray(bias, np.float32).reshape(1, -1) if bias is not None else np.float32(0.0))
    if out_dtype == "f32":
        return v.astype(np.float32)
    if out_dtype == "bf16":
        return f32_to_bf16_bits(v)
    raise ValueError(f"unknown out dtype {out_dtype!r}")


def int4_gemm_epilogue_lora(acc, xs, ws, bias, lora_t, lora_b, scale: float,
                            out_dtype: str = "bf16") -> np.ndarray:
    """Epilogue with the Dynamic-LoRA side path:
    (((float(D) * xs) * ws) + bias) + fp32(fp32(T . B^T) * scale), one output rounding.

    T . B^T is formed in float64 and rounded once to fp32; the tensor cores
    accumulate it in fp32 in an unspecified order, so the kernel may differ in
    the last fp32 bits of that term (tests use a tolerance for this path).
    """
    v = acc.astype(np.float32) * np.asarray(xs, np.float32).reshape(-1, 1)
    v = v * np.asarray(ws, np.float32).reshape(1, -1)
    v = v + (np.asarray(bias, np.float32).reshape(1, -1) if bias is not None else np.float32(0.0))
    lora = (np.asarray(lora_t, np.float64) @ np.asarray(lora_b, np.float64).T).astype(np.float32)
    v = v + lora * np.float32(scale)
    if out_dtype == "f32":
        return v.astype(np.float32)
    return f32_to_bf16_bits(v)


def int4_convrot_gemm(xp, wp, xs, ws, bias, out_dtype: str = "bf16") -> np.ndarray:
    """Packed X [M,K/2] x packed W [N,K/2] -> dequantized output [M,N]."""
    return int4_gemm_epilogue(int4_gemm_acc(xp, wp), xs, ws, bias, out_dtype)


def lora_side_path(x: np.ndarray, a: np.ndarray, b: np.ndarray, scale: float) -> np.ndarray:
    """Dynamic-LoRA contribution (x @ A^T) @ B^T * scale, computed in float64.

    ComfyUI's adapter arithmetic (``int4_ops.py:181-192`` calls ``v.h(x, out)``)
    is not vendored in the reference and no version is pinned, so this side
    path has no pinned golden vectors; it is the mathematical definition.
    """
    t = np.asarray(x, np.float64) @ np.asarray(a, np.float64).T
    return (t @ np.asarray(b, np.float64).T) * float(scale)


def convrot_w4a4_linear(x: np.ndarray, wp: np.ndarray, ws: np.ndarray, bias=None,
                        group: int = 256, dtype: str = "bf16") -> np.ndarray:
    """Whole forward: rotate + quantize x [M,K], GEMM with packed W, epilogue.

    Output is in the activation dtype (bf16 bits, or f32 values computed as f32
    then rounded for f16), like ``_int4/__init__.py:134-138``.
    """
    xp, xs = convrot_quant_int4(x, group, dtype)
    if dtype == "bf16":
        return int4_convrot_gemm(xp, wp, xs, ws, bias, "bf16")
    out = int4_convrot_gemm(xp, wp, xs, ws, bias, "f32")
    return out.astype(np.float16) if dtype == "f16" else out


def decode_weight(wp: np.ndarray) -> np.ndarray:
    """Packed weight [N, K/2] -> its codes as a float32 [N, K] matrix (decode once, reuse)."""
    return unpack_int4(wp).astype(np.float32)


def convrot_w4a4_linear_decoded(x: np.ndarray, w_codes: np.ndarray, ws: np.ndarray, bias=None,
                                group: int = 256) -> np.ndarray:
    """``convrot_w4a4_linear`` (bf16) with the weight codes already decoded to float32.

    Same arithmetic: exact integer products (float32 BLAS is exact for these
    magnitudes), the fp32 epilogue, bf16 output bits.
    """
    xp, xs = convrot_quant_int4(x, group, "bf16")
    acc = unpack_int4(xp).astype(np.float32) @ w_codes.T
    return int4_gemm_epilogue(acc.astype(np.int32), xs, ws, bias, "bf16")


# ---------------------------------------------------------------------------
# Weight quantization (``_int4/eager.py:49-62``, ``:123-135``), in fp16 like
# the reference load path (``int4_ops.py:342-349`` casts the weight to fp16)
# ---------------------------------------------------------------------------


def quantize_weight(w: np.ndarray, group: int, dtype: str = "f16") -> tuple[np.ndarray, np.ndarray]:
    """Rotate + quantize a weight [N, K] (storage form of ``dtype``).

    The reference rotates with a library fp16 matmul; this oracle uses the
    kernel's fp32 butterfly order, so codes can differ at rare rounding ties.
    """
    return convrot_quant_int4(w, group, dtype)


def dequantize_weight(wp: np.ndarray, ws: np.ndarray, group: int) -> np.ndarray:
    """Unpack, scale and rotate back (H is symmetric and orthogonal): float64 [N, K]."""
    wi = unpack_int4(wp).astype(np.float64) * np.asarray(ws, np.float64).reshape(-1, 1)
    n, k = wi.shape
    h = hadamard(group)
    return (wi.reshape(n, k // group, group) @ h.T).reshape(n, k)


def convrot_w8a8_linear(x: np.ndarray, qweight: np.ndarray, wscales: np.ndarray,
                        bias: np.ndarray | None, group: int, dtype: str = "bf16") -> np.ndarray:
    """W8A8 linear (``_int4/int8_eager.py:60-89`` with the int8 GEMM's exact int32
    accumulator and fp32 epilogue, ``_int4/int4_gemm.hip:421-492``)."""
    xq, xs = convrot_quant_int8(x, group, dtype)
    return int4_gemm_epilogue(int8_gemm_acc(xq, qweight), xs, wscales, bias, dtype)
