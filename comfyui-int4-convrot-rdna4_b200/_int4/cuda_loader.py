"""ctypes binding of libconvrot_b200.so (the sm_100a kernels).

Counterpart of the reference's hip_loader.py (_int4/hip_loader.py:42-207):
same Python functions, same argument meaning, outputs allocated by torch on
the input's device, calls issued on torch's current stream, RuntimeError on a
nonzero return code. There is no fallback: if the library cannot be loaded
every call raises.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import build as _build

_lib = None
_lock = threading.Lock()

_OUT_DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1}
_IN_DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_P = ctypes.c_void_p
_I = ctypes.c_int
_SIGNATURES = {
    "ck_convrot_quant_int4": [_P, _I, _P, _P, _I, _I, _I, _P],
    "ck_int4_quant_rowwise": [_P, _I, _P, _P, _I, _I, _P],
    "ck_int4_convrot_gemm": [_P] * 6 + [_I] * 4 + [_P],
    "ck_int4_convrot_gemm_splitk": [_P] * 5 + [_I] * 4 + [_P],
    "ck_int4_convrot_gemm_lora": [_P] * 5 + [_I, _P] + [_I] * 4 + [_P, _P, _I, ctypes.c_float, _P],
    "ck_convrot_w4a4_linear": [_P, _I, _P, _P, _P, _I, _P] + [_I] * 5 + [_P, ctypes.c_size_t, _P],
    "ck_convrot_w4a4_linear_workspace_size": [_I, _I],
    "ck_convrot_w4a4_linear_noalloc": [_P, _I, _P, _P, _P, _I, _P] + [_I] * 5 + [_P],
    "ck_int4_gemm_s32": [_P, _P, _P, _I, _I, _I, _P],
    "ck_convrot_quant_int8": [_P, _I, _P, _P, _I, _I, _I, _P],
    "ck_int8_convrot_gemm": [_P] * 6 + [_I] * 4 + [_P],
    "ck_int8_gemm_s32": [_P, _P, _P, _I, _I, _I, _P],
    "ck_int8_convrot_gemm_lora": [_P] * 5 + [_I, _P] + [_I] * 4 + [_P, _P, _I, ctypes.c_float, _P],
    "ck_int4_unpack": [_P, _P, ctypes.c_longlong, _I, _P],
    "ck_lora_down": [_P, _I, _P, _P, _I, _I, _I, _P],
    "ck_convrot_quant_int4_lnmod": [_P, _P, _P, ctypes.c_float, _P, _P, _I, _I, _I, _I, _P],
    "ck_convrot_w4a4_linear_lnmod": [_P, _P, _P, ctypes.c_float, _P, _P, _P, _I, _P] + [_I] * 5
                                    + [_P, ctypes.c_size_t, _P],
    "ck_peer_buffer_alloc": [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), _P],
    "ck_peer_buffer_open": [_P, ctypes.POINTER(ctypes.c_void_p)],
    "ck_peer_buffer_close": [_P],
    "ck_peer_buffer_free": [_P],
    "ck_peer_barrier": [_P, _I, _I, _P, ctypes.c_longlong, _P],
    "ck_peer_copy_columns": [_P, _I, _P] + [ctypes.c_longlong] * 4 + [_P],
    "ck_int4_convrot_gemm_a8_peers": [_P] * 5 + [_I, _P] + [_I] * 7 + [_P, _P, _I, ctypes.c_float, _P],
    "ck_int4_convrot_gemm_a8": [_P] * 5 + [_I, _P] + [_I] * 4 + [_P, _P, _I, ctypes.c_float, _P],
    "ck_convrot_quant_int4_unpacked": [_P, _I, _P, _P, _I, _I, _I, _P],
    "ck_convrot_w4a4_linear_unpacked_workspace_size": [_I, _I],
    "ck_convrot_w4a4_linear_unpacked": [_P, _I, _P, _P, _P, _I, _P] + [_I] * 5 + [_P, ctypes.c_size_t, _P],
    "ck_convrot_device_status": [_P, ctypes.POINTER(ctypes.c_int)],
    "ck_convrot_selftest_wait_timeout": [ctypes.c_longlong, _P],
    "ck_convrot_last_error": [],
}


def _load():
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = _build.lib_path()
            if not __import__("os").path.exists(path):
                _build.build()
            lib = ctypes.CDLL(path)
            for name, argtypes in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = {"ck_convrot_last_error": ctypes.c_char_p,
                              "ck_convrot_w4a4_linear_workspace_size": ctypes.c_size_t,
                              "ck_convrot_w4a4_linear_unpacked_workspace_size": ctypes.c_size_t}.get(name, ctypes.c_int)
            _lib = lib
    return _lib


def library():
    """The loaded ctypes library (builds it first if the .so is missing)."""
    return _load()


def _check(name: str, rc: int) -> None:
    if rc == 0:
        return
    if rc == -1:
        msg = _load().ck_convrot_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} rejected its arguments: {msg}")
    raise RuntimeError(f"{name} failed, cudaError={rc}")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("the B200 ConvRot kernels need CUDA tensors")


def convrot_quant_int4(x: torch.Tensor, convrot_groupsize: int):
    """Fused rotation + row-wise int4 quantization: (packed int8 [M, K/2], scale f32 [M])."""
    lib = _load()
    if convrot_groupsize not in (16, 64, 256):
        raise ValueError("fused convrot_quant_int4 supports groupsize 16/64/256")
    _require_cuda(x)
    if x.dtype not in _IN_DTYPE_CODE:
        raise ValueError(f"unsupported activation dtype {x.dtype}")
    x = x.contiguous()
    m, k = x.shape
    qout = torch.empty((m, k // 2), dtype=torch.int8, device=x.device)
    scale = torch.empty((m,), dtype=torch.float32, device=x.device)
    rc = lib.ck_convrot_quant_int4(x.data_ptr(), _IN_DTYPE_CODE[x.dtype], qout.data_ptr(),
                                   scale.data_ptr(), m, k, convrot_groupsize, _stream(x))
    _check("ck_convrot_quant_int4", rc)
    return qout, scale


def int4_quant_rowwise(x_rot: torch.Tensor):
    """Row-wise int4 quantization of an already rotated activation."""
    lib = _load()
    _require_cuda(x_rot)
    if x_rot.dtype not in _IN_DTYPE_CODE:
        raise ValueError(f"unsupported activation dtype {x_rot.dtype}")
    x_rot = x_rot.contiguous()
    m, k = x_rot.shape
    qout = torch.empty((m, k // 2), dtype=torch.int8, device=x_rot.device)
    scale = torch.empty((m,), dtype=torch.float32, device=x_rot.device)
    rc = lib.ck_int4_quant_rowwise(x_rot.data_ptr(), _IN_DTYPE_CODE[x_rot.dtype], qout.data_ptr(),
                                   scale.data_ptr(), m, k, _stream(x_rot))
    _check("ck_int4_quant_rowwise", rc)
    return qout, scale


def _packed_pair(x_packed: torch.Tensor, w_packed: torch.Tensor):
    _require_cuda(x_packed, w_packed)
    x_packed = x_packed.contiguous()
    w_packed = w_packed.contiguous()
    m, kp = x_packed.shape
    n, kp2 = w_packed.shape
    if kp != kp2:
        raise ValueError(f"K mismatch: x {tuple(x_packed.shape)} w {tuple(w_packed.shape)}")
    return x_packed, w_packed, m, n, kp * 2


def int4_convrot_gemm(x_packed, w_packed, x_scale, w_scale, bias, out_dtype):
    """out[M,N] = (Xint @ Wint^T) * x_scale[:,None] * w_scale[None,:] (+ bias)."""
    lib = _load()
    if out_dtype not in _OUT_DTYPE_CODE:
        raise ValueError(f"int4 gemm output dtype must be float32/bfloat16, got {out_dtype}")
    x_packed, w_packed, m, n, k = _packed_pair(x_packed, w_packed)
    x_scale = x_scale.to(torch.float32).contiguous()
    w_scale = w_scale.to(torch.float32).contiguous()
    out = torch.empty((m, n), dtype=out_dtype, device=x_packed.device)
    bias_ptr = 0
    if bias is not None:
        bias = bias.to(torch.float32).contiguous()
        bias_ptr = bias.data_ptr()
    rc = lib.ck_int4_convrot_gemm(x_packed.data_ptr(), w_packed.data_ptr(), x_scale.data_ptr(),
                                  w_scale.data_ptr(), bias_ptr, out.data_ptr(), m, n, k,
                                  _OUT_DTYPE_CODE[out_dtype], _stream(x_packed))
    _check("ck_int4_convrot_gemm", rc)
    return out


def int4_convrot_gemm_lora(x_packed, w_packed, x_scale, w_scale, bias, out_dtype, lora_t, lora_b, lora_scale):
    """int4_convrot_gemm plus lora_scale * (lora_t @ lora_b^T), fused in the epilogue.

    lora_t: fp16 [M, r] (= x @ A^T), lora_b: fp16 [N, r], r a multiple of 8 up to 64.
    """
    x_packed, w_packed, m, n, k = _packed_pair(x_packed, w_packed)
    return _gemm_lora("ck_int4_convrot_gemm_lora", x_packed, w_packed, m, n, k, x_scale, w_scale, bias,
                      out_dtype, lora_t, lora_b, lora_scale)


def int8_convrot_gemm_lora(x_int8, w_int8, x_scale, w_scale, bias, out_dtype, lora_t, lora_b, lora_scale):
    """int4_convrot_gemm_lora on int8 operands [M, K] / [N, K] (the W8A8 tier, or
    unpacked int4 codes: same accumulators, same output bits)."""
    x_int8, w_int8, m, n, k = _int8_pair(x_int8, w_int8)
    return _gemm_lora("ck_int8_convrot_gemm_lora", x_int8, w_int8, m, n, k, x_scale, w_scale, bias,
                      out_dtype, lora_t, lora_b, lora_scale)


def _gemm_lora(name, xq, wq, m, n, k, x_scale, w_scale, bias, out_dtype, lora_t, lora_b, lora_scale):
    lib = _load()
    if out_dtype not in _OUT_DTYPE_CODE:
        raise ValueError(f"LoRA gemm output dtype must be float32/bfloat16, got {out_dtype}")
    _require_cuda(lora_t, lora_b)
    lora_t = lora_t.to(torch.float16).contiguous()
    lora_b = lora_b.to(torch.float16).contiguous()
    r = lora_t.shape[1]
    if tuple(lora_t.shape) != (m, r) or tuple(lora_b.shape) != (n, r):
        raise ValueError(f"LoRA shapes {tuple(lora_t.shape)} / {tuple(lora_b.shape)} do not match M={m}, N={n}")
    x_scale = x_scale.to(torch.float32).contiguous()
    w_scale = w_scale.to(torch.float32).contiguous()
    out = torch.empty((m, n), dtype=out_dtype, device=xq.device)
    bias, bias_ptr, bias_code = _bias_arg(bias)
    rc = getattr(lib, name)(xq.data_ptr(), wq.data_ptr(), x_scale.data_ptr(), w_scale.data_ptr(), bias_ptr,
                            bias_code, out.data_ptr(), m, n, k, _OUT_DTYPE_CODE[out_dtype], lora_t.data_ptr(),
                            lora_b.data_ptr(), r, float(lora_scale), _stream(xq))
    _check(name, rc)
    return out


def int4_convrot_gemm_a8(x_codes, w_packed, x_scale, w_scale, bias, out_dtype,
                         lora_t=None, lora_b=None, lora_scale: float = 0.0):
    """The int4 GEMM on int8 activation codes [M, K] (one sign-extended code per byte,
    from convrot_quant_int4_unpacked) and packed int4 weights [N, K/2]: the same
    accumulators and output bits as int4_convrot_gemm on the packed codes. With
    lora_t / lora_b (fp16 [M, r] / [N, r]) the Dynamic-LoRA side path is fused as in
    int4_convrot_gemm_lora. out_dtype torch.int32 returns the exact accumulators."""
    lib = _load()
    _require_cuda(x_codes, w_packed, x_scale, w_scale)
    x_codes = x_codes.contiguous()
    w_packed = w_packed.contiguous()
    m, k = x_codes.shape
    n, kp = w_packed.shape
    if k != 2 * kp:
        raise ValueError(f"K mismatch: codes {tuple(x_codes.shape)} packed weights {tuple(w_packed.shape)}")
    codes = {**_OUT_DTYPE_CODE, torch.int32: 3}
    if out_dtype not in codes:
        raise ValueError(f"A8 gemm output dtype must be float32/bfloat16/int32, got {out_dtype}")
    x_scale = x_scale.to(torch.float32).contiguous()
    w_scale = w_scale.to(torch.float32).contiguous()
    bias, bias_ptr, bias_code = _bias_arg(bias)
    lt_ptr = lb_ptr = 0
    r = 0
    if lora_t is not None:
        _require_cuda(lora_t, lora_b)
        lora_t = lora_t.to(torch.float16).contiguous()
        lora_b = lora_b.to(torch.float16).contiguous()
        r = lora_t.shape[1]
        if tuple(lora_t.shape) != (m, r) or tuple(lora_b.shape) != (n, r):
            raise ValueError(f"LoRA shapes {tuple(lora_t.shape)} / {tuple(lora_b.shape)} do not match M={m}, N={n}")
        lt_ptr, lb_ptr = lora_t.data_ptr(), lora_b.data_ptr()
    out = torch.empty((m, n), dtype=out_dtype, device=x_codes.device)
    rc = lib.ck_int4_convrot_gemm_a8(x_codes.data_ptr(), w_packed.data_ptr(), x_scale.data_ptr(),
                                     w_scale.data_ptr(), bias_ptr, bias_code, out.data_ptr(), m, n, k,
                                     codes[out_dtype], lt_ptr, lb_ptr, r, float(lora_scale), _stream(x_codes))
    _check("ck_int4_convrot_gemm_a8", rc)
    return out


def _bias_arg(bias):
    """(tensor kept alive, pointer, dtype code): f32/bf16/f16 bias is read as is by the kernels."""
    if bias is None:
        return None, 0, 0
    if bias.dtype not in _IN_DTYPE_CODE:
        bias = bias.to(torch.float32)
    bias = bias.contiguous()
    return bias, bias.data_ptr(), _IN_DTYPE_CODE[bias.dtype]


def convrot_w4a4_linear(x, w_packed, w_scale, bias, out_dtype, convrot_groupsize: int = 256):
    """x [M, K] @ W^T + bias through the fused entry ck_convrot_w4a4_linear.

    Rotation + quantization into a workspace, then the int4 GEMM (a programmatic
    dependent launch of the quantizer); the bias is read in its own dtype.
    """
    lib = _load()
    if out_dtype not in _OUT_DTYPE_CODE:
        raise ValueError(f"int4 gemm output dtype must be float32/bfloat16, got {out_dtype}")
    if convrot_groupsize not in (16, 64, 256):
        raise ValueError("fused convrot_quant_int4 supports groupsize 16/64/256")
    _require_cuda(x, w_packed)
    if x.dtype not in _IN_DTYPE_CODE:
        raise ValueError(f"unsupported activation dtype {x.dtype}")
    x = x.contiguous()
    w_packed = w_packed.contiguous()
    m, k = x.shape
    n, kp = w_packed.shape
    if kp * 2 != k:
        raise ValueError(f"K mismatch: x {tuple(x.shape)} w {tuple(w_packed.shape)}")
    w_scale = w_scale.to(torch.float32).contiguous()
    bias, bias_ptr, bias_code = _bias_arg(bias)
    out = torch.empty((m, n), dtype=out_dtype, device=x.device)
    ws_bytes = lib.ck_convrot_w4a4_linear_workspace_size(m, k)
    workspace = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=x.device)
    rc = lib.ck_convrot_w4a4_linear(x.data_ptr(), _IN_DTYPE_CODE[x.dtype], w_packed.data_ptr(),
                                    w_scale.data_ptr(), bias_ptr, bias_code, out.data_ptr(),
                                    _OUT_DTYPE_CODE[out_dtype], m, n, k, convrot_groupsize,
                                    workspace.data_ptr(), ws_bytes, _stream(x))
    _check("ck_convrot_w4a4_linear", rc)
    return out


def convrot_w4a4_linear_noalloc(x, w_packed, w_scale, bias, out_dtype, convrot_groupsize: int = 256):
    """As convrot_w4a4_linear, through ck_convrot_w4a4_linear_noalloc: the library
    allocates nothing (its static per-device scratch holds the quantized
    activations); only the output tensor is allocated here, by torch."""
    lib = _load()
    if out_dtype not in _OUT_DTYPE_CODE:
        raise ValueError(f"int4 gemm output dtype must be float32/bfloat16, got {out_dtype}")
    _require_cuda(x, w_packed)
    if x.dtype not in _IN_DTYPE_CODE:
        raise ValueError(f"unsupported activation dtype {x.dtype}")
    x = x.contiguous()
    w_packed = w_packed.contiguous()
    m, k = x.shape
    n = w_packed.shape[0]
    w_scale = w_scale.to(torch.float32).contiguous()
    bias, bias_ptr, bias_code = _bias_arg(bias)
    out = torch.empty((m, n), dtype=out_dtype, device=x.device)
    rc = lib.ck_convrot_w4a4_linear_noalloc(x.data_ptr(), _IN_DTYPE_CODE[x.dtype], w_packed.data_ptr(),
                                            w_scale.data_ptr(), bias_ptr, bias_code, out.data_ptr(),
                                            _OUT_DTYPE_CODE[out_dtype], m, n, k, convrot_groupsize, _stream(x))
    _check("ck_convrot_w4a4_linear_noalloc", rc)
    return out


def int4_convrot_gemm_splitk(x_packed, w_packed, x_scale, w_scale, accum, nsplit: int = 1):
    """accum += (Xint @ Wint^T) * x_scale[:,None] * w_scale[None,:] (f32, in place)."""
    lib = _load()
    x_packed, w_packed, m, n, k = _packed_pair(x_packed, w_packed)
    if accum.dtype != torch.float32 or tuple(accum.shape) != (m, n) or not accum.is_contiguous():
        raise ValueError("accum must be a contiguous float32 [M, N] tensor")
    x_scale = x_scale.to(torch.float32).contiguous()
    w_scale = w_scale.to(torch.float32).contiguous()
    rc = lib.ck_int4_convrot_gemm_splitk(x_packed.data_ptr(), w_packed.data_ptr(), x_scale.data_ptr(),
                                         w_scale.data_ptr(), accum.data_ptr(), m, n, k, nsplit,
                                         _stream(x_packed))
    _check("ck_int4_convrot_gemm_splitk", rc)
    return accum


def int4_gemm_s32(x_packed, w_packed):
    """Exact int32 accumulators [M, N] of the packed-code product."""
    lib = _load()
    x_packed, w_packed, m, n, k = _packed_pair(x_packed, w_packed)
    acc = torch.empty((m, n), dtype=torch.int32, device=x_packed.device)
    rc = lib.ck_int4_gemm_s32(x_packed.data_ptr(), w_packed.data_ptr(), acc.data_ptr(), m, n, k,
                              _stream(x_packed))
    _check("ck_int4_gemm_s32", rc)
    return acc


def selftest_wait_timeout(limit_ns: int, device=None) -> None:
    """Launch the failure-path self test (a bounded wait nothing ends); afterwards
    device_status() returns 5."""
    lib = _load()
    stream = torch.cuda.current_stream(device).cuda_stream
    _check("ck_convrot_selftest_wait_timeout", lib.ck_convrot_selftest_wait_timeout(int(limit_ns), stream))


def device_status(device=None) -> int:
    """Read and clear the kernels' bounded-wait status word (0 = ok)."""
    lib = _load()
    st = ctypes.c_int(0)
    stream = torch.cuda.current_stream(device).cuda_stream
    _check("ck_convrot_device_status", lib.ck_convrot_device_status(stream, ctypes.byref(st)))
    return st.value


def is_available() -> bool:
    try:
        _load()
        return True
    except Exception:
        return False


# --------------------------------------------------------------------- W8A8 tier


def int8_quant_supported(x: torch.Tensor, convrot_groupsize: int) -> bool:
    """Shapes the native int8 quantizer takes: bf16 rows of whole 256-column tiles, G = 64/256."""
    k = x.shape[-1]
    return (x.dtype == torch.bfloat16 and convrot_groupsize in (64, 256) and k % 256 == 0
            and k // 256 <= 192)


def convrot_quant_int8(x: torch.Tensor, convrot_groupsize: int):
    """Fused rotation + row-wise int8 quantization: (int8 [M, K], scale f32 [M]).

    Mirrors hip_loader.convrot_quant_int8 (_int4/hip_loader.py:95-113).
    """
    lib = _load()
    if convrot_groupsize not in (16, 64, 256):
        raise ValueError("fused convrot_quant_int8 supports groupsize 16/64/256")
    _require_cuda(x)
    if x.dtype not in _IN_DTYPE_CODE:
        raise ValueError(f"unsupported activation dtype {x.dtype}")
    x = x.contiguous()
    m, k = x.shape
    qout = torch.empty((m, k), dtype=torch.int8, device=x.device)
    scale = torch.empty((m,), dtype=torch.float32, device=x.device)
    rc = lib.ck_convrot_quant_int8(x.data_ptr(), _IN_DTYPE_CODE[x.dtype], qout.data_ptr(),
                                   scale.data_ptr(), m, k, convrot_groupsize, _stream(x))
    _check("ck_convrot_quant_int8", rc)
    return qout, scale


def _int8_pair(x_int8: torch.Tensor, w_int8: torch.Tensor):
    _require_cuda(x_int8, w_int8)
    x_int8 = x_int8.contiguous()
    w_int8 = w_int8.contiguous()
    m, k = x_int8.shape
    n, kw = w_int8.shape
    if k != kw:
        raise ValueError(f"K mismatch: x {tuple(x_int8.shape)} w {tuple(w_int8.shape)}")
    return x_int8, w_int8, m, n, k


def int8_convrot_gemm(x_int8, w_int8, x_scale, w_scale, bias, out_dtype):
    """out[M,N] = (X @ W^T) * x_scale[:,None] * w_scale[None,:] (+ bias), int8 operands.

    Mirrors hip_loader.int8_convrot_gemm (_int4/hip_loader.py:116-150).
    """
    lib = _load()
    if out_dtype not in _OUT_DTYPE_CODE:
        raise ValueError(f"int8 gemm output dtype must be float32/bfloat16, got {out_dtype}")
    x_int8, w_int8, m, n, k = _int8_pair(x_int8, w_int8)
    x_scale = x_scale.to(torch.float32).contiguous()
    w_scale = w_scale.to(torch.float32).contiguous()
    out = torch.empty((m, n), dtype=out_dtype, device=x_int8.device)
    bias_ptr = 0
    if bias is not None:
        bias = bias.to(torch.float32).contiguous()
        bias_ptr = bias.data_ptr()
    rc = lib.ck_int8_convrot_gemm(x_int8.data_ptr(), w_int8.data_ptr(), x_scale.data_ptr(),
                                  w_scale.data_ptr(), bias_ptr, out.data_ptr(), m, n, k,
                                  _OUT_DTYPE_CODE[out_dtype], _stream(x_int8))
    _check("ck_int8_convrot_gemm", rc)
    return out


def int8_gemm_s32(x_int8, w_int8):
    """Exact int32 accumulators [M, N] of the int8 product."""
    lib = _load()
    x_int8, w_int8, m, n, k = _int8_pair(x_int8, w_int8)
    acc = torch.empty((m, n), dtype=torch.int32, device=x_int8.device)
    rc = lib.ck_int8_gemm_s32(x_int8.data_ptr(), w_int8.data_ptr(), acc.data_ptr(), m, n, k, _stream(x_int8))
    _check("ck_int8_gemm_s32", rc)
    return acc


# --------------------------------------------------------------------- LayerNorm + modulation fused


def _mod_vector(v, k: int, device):
    if v is None:
        return None, None
    v = v.reshape(-1).to(device=device, dtype=torch.bfloat16).contiguous()
    if v.numel() != k:
        raise ValueError(f"modulation vector of {v.numel()} values for K={k}")
    return v, v.data_ptr()


def convrot_quant_int4_lnmod(x, scale, shift, eps: float, convrot_groupsize: int, unpacked: bool = False):
    """Codes and scales of bf16((1 + scale) * LayerNorm(x) + shift), rotated and quantized in
    one pass over x (ck_convrot_quant_int4_lnmod): packed [M, K/2] or one int8 per code [M, K]."""
    lib = _load()
    _require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise ValueError("the fused LayerNorm quantizer takes bf16 activations")
    x = x.contiguous()
    m, k = x.shape
    sc, sc_ptr = _mod_vector(scale, k, x.device)
    sh, sh_ptr = _mod_vector(shift, k, x.device)
    q = torch.empty((m, k if unpacked else k // 2), dtype=torch.int8, device=x.device)
    s = torch.empty((m,), dtype=torch.float32, device=x.device)
    rc = lib.ck_convrot_quant_int4_lnmod(x.data_ptr(), sc_ptr, sh_ptr, float(eps), q.data_ptr(), s.data_ptr(), m, k,
                                         convrot_groupsize, 1 if unpacked else 0, _stream(x))
    _check("ck_convrot_quant_int4_lnmod", rc)
    return q, s


def convrot_w4a4_linear_lnmod(x, w_packed, w_scale, bias, scale, shift, eps: float, out_dtype,
                              convrot_groupsize: int = 256):
    """The int4 linear of bf16((1 + scale) * LayerNorm(x) + shift) (ck_convrot_w4a4_linear_lnmod)."""
    lib = _load()
    _require_cuda(x, w_packed)
    if x.dtype != torch.bfloat16:
        raise ValueError("the fused LayerNorm linear takes bf16 activations")
    x = x.contiguous()
    w_packed = w_packed.contiguous()
    m, k = x.shape
    n, kp = w_packed.shape
    if kp * 2 != k:
        raise ValueError(f"K mismatch: x {tuple(x.shape)} w {tuple(w_packed.shape)}")
    sc, sc_ptr = _mod_vector(scale, k, x.device)
    sh, sh_ptr = _mod_vector(shift, k, x.device)
    w_scale = w_scale.to(torch.float32).contiguous()
    bias, bias_ptr, bias_code = _bias_arg(bias)
    out = torch.empty((m, n), dtype=out_dtype, device=x.device)
    ws_bytes = lib.ck_convrot_w4a4_linear_workspace_size(m, k)
    workspace = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=x.device)
    rc = lib.ck_convrot_w4a4_linear_lnmod(x.data_ptr(), sc_ptr, sh_ptr, float(eps), w_packed.data_ptr(),
                                          w_scale.data_ptr(), bias_ptr, bias_code, out.data_ptr(),
                                          _OUT_DTYPE_CODE[out_dtype], m, n, k, convrot_groupsize,
                                          workspace.data_ptr(), ws_bytes, _stream(x))
    _check("ck_convrot_w4a4_linear_lnmod", rc)
    return out


def lnmod_supported(x: torch.Tensor, convrot_groupsize: int) -> bool:
    """bf16 CUDA rows of whole 256-column tiles, K <= 6144, G in {64, 256}."""
    k = x.shape[-1]
    return (x.is_cuda and x.dtype == torch.bfloat16 and convrot_groupsize in (64, 256) and k % 256 == 0
            and k <= 6144)


# --------------------------------------------------------------------- Dynamic-LoRA down projection


def lora_down(x: torch.Tensor, down: torch.Tensor) -> torch.Tensor:
    """T = fp16(x) @ down^T as fp16 [M, R] on the tensor cores (ck_lora_down).

    x [M, K] bf16 or fp16 (f32 is cast to fp16 first), down [R, K] fp16 with R a
    multiple of 8 in [8, 64]; fp32 accumulation, one rounding to fp16."""
    lib = _load()
    _require_cuda(x, down)
    if x.dtype == torch.float32:
        x = x.to(torch.float16)
    x = x.contiguous()
    down = down.to(torch.float16).contiguous()
    m, k = x.shape
    r = down.shape[0]
    t = torch.empty((m, r), dtype=torch.float16, device=x.device)
    rc = lib.ck_lora_down(x.data_ptr(), _IN_DTYPE_CODE[x.dtype], down.data_ptr(), t.data_ptr(), m, k, r, _stream(x))
    _check("ck_lora_down", rc)
    return t


# --------------------------------------------------------------------- peer memory (column split)


def peer_buffer_alloc(nbytes: int) -> tuple[int, bytes]:
    """A zeroed device buffer of this process and its CUDA IPC handle (64 bytes)."""
    lib = _load()
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    _check("ck_peer_buffer_alloc", lib.ck_peer_buffer_alloc(nbytes, ctypes.byref(ptr), handle))
    return int(ptr.value), bytes(handle.raw)


def peer_buffer_open(handle: bytes) -> int:
    """This process's mapping of another process's buffer (from peer_buffer_alloc's handle)."""
    lib = _load()
    ptr = ctypes.c_void_p()
    _check("ck_peer_buffer_open", lib.ck_peer_buffer_open(ctypes.create_string_buffer(handle, 64), ctypes.byref(ptr)))
    return int(ptr.value)


def peer_buffer_close(ptr: int) -> None:
    _check("ck_peer_buffer_close", _load().ck_peer_buffer_close(ptr))


def peer_buffer_free(ptr: int) -> None:
    _check("ck_peer_buffer_free", _load().ck_peer_buffer_free(ptr))


def _ptr_array(ptrs):
    return (ctypes.c_void_p * len(ptrs))(*ptrs)


def peer_barrier(flag_ptrs, rank: int, counter_ptr: int, timeout_ns: int, device) -> None:
    """Flag barrier after peer stores (ck_peer_barrier) on the device's current stream."""
    lib = _load()
    stream = torch.cuda.current_stream(device).cuda_stream
    _check("ck_peer_barrier", lib.ck_peer_barrier(_ptr_array(flag_ptrs), len(flag_ptrs), rank, counter_ptr,
                                                  int(timeout_ns), stream))


def peer_copy_columns(dsts, src_ptr: int, pitch_bytes: int, offset_bytes: int, width_bytes: int, rows: int,
                      stream) -> None:
    """2D copies of a column block from src to every destination (ck_peer_copy_columns)."""
    lib = _load()
    _check("ck_peer_copy_columns", lib.ck_peer_copy_columns(_ptr_array(dsts), len(dsts), src_ptr, pitch_bytes,
                                                            offset_bytes, width_bytes, rows, stream.cuda_stream))


def int4_convrot_gemm_a8_peers(x_codes, w_packed, x_scale, w_scale, bias, out_dtype, outs, ldo: int, col0: int,
                               lora_t=None, lora_b=None, lora_scale: float = 0.0) -> None:
    """ck_int4_convrot_gemm_a8_peers: the A8 GEMM storing its [M, N] block at columns
    col0 .. col0 + N of the [M, ldo] matrices at the device pointers ``outs``."""
    lib = _load()
    _require_cuda(x_codes, w_packed)
    m, k = x_codes.shape
    n, kp = w_packed.shape
    if kp * 2 != k:
        raise ValueError(f"K mismatch: codes {tuple(x_codes.shape)} w {tuple(w_packed.shape)}")
    x_scale = x_scale.to(torch.float32).contiguous()
    w_scale = w_scale.to(torch.float32).contiguous()
    bias, bias_ptr, bias_code = _bias_arg(bias)
    r = 0
    if lora_t is not None:
        lora_t = lora_t.to(torch.float16).contiguous()
        lora_b = lora_b.to(torch.float16).contiguous()
        r = lora_t.shape[1]
    rc = lib.ck_int4_convrot_gemm_a8_peers(
        x_codes.data_ptr(), w_packed.data_ptr(), x_scale.data_ptr(), w_scale.data_ptr(), bias_ptr, bias_code,
        _ptr_array(outs), len(outs), ldo, col0, m, n, k, _OUT_DTYPE_CODE[out_dtype],
        lora_t.data_ptr() if lora_t is not None else None, lora_b.data_ptr() if lora_b is not None else None,
        r, float(lora_scale), _stream(x_codes))
    _check("ck_int4_convrot_gemm_a8_peers", rc)


# --------------------------------------------------------------------- unpacked-code path


def int4_unpack(packed: torch.Tensor) -> torch.Tensor:
    """packed int4 [R, K/2] -> int8 codes [R, K] on the device (ck_int4_unpack)."""
    lib = _load()
    _require_cuda(packed)
    packed = packed.contiguous()
    rows, kp = packed.shape
    codes = torch.empty((rows, 2 * kp), dtype=torch.int8, device=packed.device)
    rc = lib.ck_int4_unpack(packed.data_ptr(), codes.data_ptr(), rows, 2 * kp, _stream(packed))
    _check("ck_int4_unpack", rc)
    return codes


def unpacked_path_supported(x: torch.Tensor, convrot_groupsize: int) -> bool:
    """Activations the unpacked-code quantizer takes (bf16 whole tiles, G = 64/256)."""
    return int8_quant_supported(x, convrot_groupsize)


def convrot_quant_int4_unpacked(x: torch.Tensor, convrot_groupsize: int):
    """Rotation + int4 quantization with one int8 per code: (codes [M, K], scale f32 [M])."""
    lib = _load()
    _require_cuda(x)
    x = x.contiguous()
    m, k = x.shape
    qout = torch.empty((m, k), dtype=torch.int8, device=x.device)
    scale = torch.empty((m,), dtype=torch.float32, device=x.device)
    rc = lib.ck_convrot_quant_int4_unpacked(x.data_ptr(), _IN_DTYPE_CODE.get(x.dtype, -1), qout.data_ptr(),
                                            scale.data_ptr(), m, k, convrot_groupsize, _stream(x))
    _check("ck_convrot_quant_int4_unpacked", rc)
    return qout, scale


def convrot_w4a4_linear_unpacked(x, w_codes, w_scale, bias, out_dtype, convrot_groupsize: int = 256):
    """The W4A4 linear on unpacked codes (ck_convrot_w4a4_linear_unpacked): x [M, K] bf16,
    w_codes int8 [N, K] from int4_unpack; results identical to convrot_w4a4_linear."""
    lib = _load()
    if out_dtype not in _OUT_DTYPE_CODE:
        raise ValueError(f"int4 gemm output dtype must be float32/bfloat16, got {out_dtype}")
    _require_cuda(x, w_codes)
    x = x.contiguous()
    w_codes = w_codes.contiguous()
    m, k = x.shape
    n, kw = w_codes.shape
    if kw != k:
        raise ValueError(f"K mismatch: x {tuple(x.shape)} w {tuple(w_codes.shape)}")
    w_scale = w_scale.to(torch.float32).contiguous()
    bias, bias_ptr, bias_code = _bias_arg(bias)
    out = torch.empty((m, n), dtype=out_dtype, device=x.device)
    ws_bytes = lib.ck_convrot_w4a4_linear_unpacked_workspace_size(m, k)
    workspace = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=x.device)
    rc = lib.ck_convrot_w4a4_linear_unpacked(x.data_ptr(), _IN_DTYPE_CODE.get(x.dtype, -1), w_codes.data_ptr(),
                                             w_scale.data_ptr(), bias_ptr, bias_code, out.data_ptr(),
                                             _OUT_DTYPE_CODE[out_dtype], m, n, k, convrot_groupsize,
                                             workspace.data_ptr(), ws_bytes, _stream(x))
    _check("ck_convrot_w4a4_linear_unpacked", rc)
    return out
