"""C-ABI and host-logic checks that need no GPU.

The library must load and export every function declared in
include/convrot_b200.h; precondition failures return -1 before any CUDA call
(the reference's convention, _int4/int4_gemm.hip:637, :653, :715).
"""
import ctypes
import os
import re

import pytest
import torch

import _int4
from _int4 import build as libbuild
from _int4 import cuda_loader

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "convrot_b200.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"\b(?:int|size_t|const char\*)\s+(ck_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(libbuild.lib_path()):
        libbuild.build()
    return cuda_loader.library()


def test_header_symbols_exported(lib):
    names = header_functions()
    assert len(names) >= 7
    raw = ctypes.CDLL(libbuild.lib_path())
    for n in names:
        assert hasattr(raw, n), n


def test_only_header_symbols_are_public(lib):
    """-fvisibility=hidden: nothing but the ck_* API leaks from the library."""
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", libbuild.lib_path()], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("nm unavailable")
    ck = {line.split()[-1] for line in out.stdout.splitlines() if " T ck_" in line}
    assert ck == set(header_functions())


@pytest.mark.parametrize("k", [0, 48, 65568])
def test_gemm_rejects_bad_k(lib, k):
    rc = lib.ck_int4_convrot_gemm(16, 16, 16, 16, 0, 16, 4, 4, k, 1, None)
    assert rc == -1
    assert b"K" in lib.ck_convrot_last_error()


def test_gemm_rejects_bad_out_dtype_and_alignment(lib):
    assert lib.ck_int4_convrot_gemm(16, 16, 16, 16, 0, 16, 4, 4, 64, 7, None) == -1
    assert lib.ck_int4_convrot_gemm(17, 16, 16, 16, 0, 16, 4, 4, 64, 1, None) == -1
    assert b"aligned" in lib.ck_convrot_last_error()
    assert lib.ck_int4_convrot_gemm(0, 0, 16, 16, 0, 16, 4, 4, 64, 1, None) == -1


def test_gemm_empty_is_noop(lib):
    assert lib.ck_int4_convrot_gemm(16, 16, 16, 16, 0, 16, 0, 4, 64, 1, None) == 0
    assert lib.ck_int4_gemm_s32(16, 16, 16, 4, 0, 64, None) == 0


def test_splitk_rejects_bad_nsplit(lib):
    assert lib.ck_int4_convrot_gemm_splitk(16, 16, 16, 16, 16, 4, 4, 64, 0, None) == -1


@pytest.mark.parametrize("g,k", [(32, 512), (256, 320), (64, 96)])
def test_quant_rejects_bad_group(lib, g, k):
    assert lib.ck_convrot_quant_int4(16, 1, 16, 16, 4, k, g, None) == -1


def test_quant_rejects_bad_dtype_and_k(lib):
    assert lib.ck_convrot_quant_int4(16, 3, 16, 16, 4, 256, 256, None) == -1
    assert lib.ck_int4_quant_rowwise(16, 1, 16, 16, 4, 24, None) == -1
    assert lib.ck_convrot_quant_int4(16, 1, 16, 16, 0, 256, 256, None) == 0


def test_linear_workspace_size(lib):
    f = lib.ck_convrot_w4a4_linear_workspace_size
    up = lambda v: (v + 255) // 256 * 256
    for m, k in [(1, 64), (7, 12288), (128, 3072)]:              # packed codes
        assert f(m, k) == up(m * k // 2) + up(4 * m)
    for m, k in [(129, 3072), (4608, 3072), (18432, 12288)]:    # one int8 per code (A8 form)
        assert f(m, k) == up(m * k) + up(4 * m)
    assert f(0, 3072) == 0


def test_gemm_a8_rejects_bad_arguments(lib):
    f = lib.ck_int4_convrot_gemm_a8
    ok = dict(x=256, w=256, xs=256, ws=256, b=0, bd=0, out=256, m=4, n=8, k=256, od=1, lt=0, lb=0, r=0)

    def call(**kw):
        a = {**ok, **kw}
        return f(a["x"], a["w"], a["xs"], a["ws"], a["b"], a["bd"], a["out"], a["m"], a["n"], a["k"], a["od"],
                 a["lt"], a["lb"], a["r"], 1.0, None)
    assert call(k=192) == -1 and b"128" in lib.ck_convrot_last_error()     # K % 128
    assert call(od=2) == -1
    assert call(bd=4) == -1
    assert call(x=264) == -1 and b"aligned" in lib.ck_convrot_last_error()
    assert call(lt=256, lb=256, r=12) == -1                                 # rank not a multiple of 8
    assert call(lt=256, lb=256, r=64, od=3) == -1                           # no LoRA on raw accumulators
    assert call(m=0) == 0 and call(n=0) == 0


def test_linear_rejects_bad_arguments(lib):
    f = lib.ck_convrot_w4a4_linear
    ws = lib.ck_convrot_w4a4_linear_workspace_size(4, 256)
    ok = dict(x=256, ind=1, w=256, s=256, b=256, bd=1, out=256, od=1, m=4, n=8, k=256, g=256, wk=4096, wsz=ws)

    def call(**kw):
        a = {**ok, **kw}
        return f(a["x"], a["ind"], a["w"], a["s"], a["b"], a["bd"], a["out"], a["od"], a["m"], a["n"], a["k"],
                 a["g"], a["wk"], a["wsz"], None)
    assert call(g=32) == -1
    assert call(k=320) == -1                                  # not divisible by G
    assert call(ind=3) == -1
    assert call(od=2) == -1
    assert call(bd=5) == -1
    assert call(wk=4100) == -1 and b"256-byte" in lib.ck_convrot_last_error()
    assert call(wsz=ws - 1) == -1 and b"workspace" in lib.ck_convrot_last_error()
    assert call(m=0) == 0 and call(n=0) == 0                  # empty: nothing launched


def test_selftest_wait_rejects_bad_limit(lib):
    assert lib.ck_convrot_selftest_wait_timeout(0, None) == -1
    assert lib.ck_convrot_selftest_wait_timeout(200_000_000, None) == -1
    assert b"limit_ns" in lib.ck_convrot_last_error()


def test_int8_lora_rejects_bad_arguments(lib):
    f = lib.ck_int8_convrot_gemm_lora
    assert f(16, 16, 16, 16, 0, 0, 16, 256, 256, 256, 1, 16, 16, 12, 1.0, None) == -1   # rank not a multiple of 8
    assert f(16, 16, 16, 16, 0, 0, 16, 256, 256, 250, 1, 16, 16, 64, 1.0, None) == -1   # K % 16
    assert f(16, 16, 16, 16, 0, 3, 16, 256, 256, 256, 1, 16, 16, 64, 1.0, None) == -1   # bias dtype
    assert f(16, 16, 16, 16, 0, 0, 16, 0, 256, 256, 1, 16, 16, 64, 1.0, None) == 0      # empty


def test_unpacked_path_rejects_bad_arguments(lib):
    assert lib.ck_convrot_w4a4_linear_unpacked_workspace_size(4608, 3072) == 4608 * 3072 + 4608 * 4
    assert lib.ck_int4_unpack(16, 16, 4, 48, None) == -1                       # K % 32
    assert lib.ck_int4_unpack(16, 17, 4, 64, None) == -1                       # alignment
    assert lib.ck_int4_unpack(16, 16, 0, 64, None) == 0                        # empty
    assert lib.ck_convrot_quant_int4_unpacked(16, 0, 16, 16, 4, 512, 256, None) == -1   # not bf16
    assert lib.ck_convrot_quant_int4_unpacked(16, 1, 16, 16, 4, 320, 64, None) == -1    # ragged tile
    f = lib.ck_convrot_w4a4_linear_unpacked
    ws = lib.ck_convrot_w4a4_linear_unpacked_workspace_size(4, 256)
    assert f(256, 1, 256, 256, 0, 0, 256, 1, 4, 8, 256, 16, 256, ws, None) == -1    # G = 16
    assert f(256, 1, 256, 256, 0, 0, 256, 1, 4, 8, 256, 256, 256, ws - 1, None) == -1
    assert b"workspace" in lib.ck_convrot_last_error()
    assert f(256, 1, 256, 256, 0, 0, 256, 1, 0, 8, 256, 256, 256, ws, None) == 0


def test_python_api_validation_errors():
    x = torch.zeros(4, 512, dtype=torch.bfloat16)
    qw = torch.zeros(8, 256, dtype=torch.int8)
    ws = torch.ones(8)
    with pytest.raises(ValueError, match="linear_dtype"):
        _int4.convrot_w4a4_linear(x, qw, ws, linear_dtype="fp8")
    with pytest.raises(ValueError, match="quant_group_size"):
        _int4.convrot_w4a4_linear(x, qw, ws, quant_group_size=32)
    with pytest.raises(ValueError, match="does not match"):
        _int4.convrot_w4a4_linear(x, qw[:, :128], ws)
    with pytest.raises(ValueError, match="divisible"):
        _int4.convrot_w4a4_linear(torch.zeros(4, 320, dtype=torch.bfloat16), qw[:, :160], ws, convrot_groupsize=256)
    with pytest.raises(ValueError, match="CUDA"):
        _int4.convrot_w4a4_linear(x, qw, ws)


def test_pick_groupsize_and_availability():
    assert _int4.pick_groupsize(3072) == 256
    assert _int4.pick_groupsize(15360) == 256
    assert _int4.pick_groupsize(320) == 64
    assert _int4.pick_groupsize(48) == 16
    assert _int4.pick_groupsize(40) is None
    if not torch.cuda.is_available():
        assert _int4.is_available() is False


def test_lora_down_preconditions(lib):
    f = lib.ck_lora_down
    assert f(256, 1, 256, 256, 16, 260, 8, None) == -1 and b"K" in lib.ck_convrot_last_error()    # K % 8
    assert f(256, 1, 256, 256, 16, 256, 12, None) == -1                                          # rank % 8
    assert f(256, 1, 256, 256, 16, 256, 72, None) == -1                                          # rank > 64
    assert f(256, 0, 256, 256, 16, 256, 8, None) == -1 and b"dtype" in lib.ck_convrot_last_error()
    assert f(264, 1, 256, 256, 16, 256, 8, None) == -1 and b"aligned" in lib.ck_convrot_last_error()
    assert f(256, 1, 256, 256, 0, 256, 8, None) == 0                                             # M = 0: no launch


def test_lnmod_preconditions(lib):
    f = lib.ck_convrot_quant_int4_lnmod
    assert f(256, 0, 0, 1e-6, 256, 256, 4, 320, 64, 0, None) == -1 and b"256" in lib.ck_convrot_last_error()
    assert f(256, 0, 0, 1e-6, 256, 256, 4, 8192, 256, 0, None) == -1                 # K > 6144
    assert f(256, 0, 0, 1e-6, 256, 256, 4, 3072, 16, 0, None) == -1                  # G = 16
    assert f(264, 0, 0, 1e-6, 256, 256, 4, 3072, 256, 0, None) == -1 and b"aligned" in lib.ck_convrot_last_error()
    assert f(256, 0, 0, -1.0, 256, 256, 4, 3072, 256, 0, None) == -1                 # eps < 0
    assert f(256, 0, 0, 1e-6, 256, 256, 0, 3072, 256, 0, None) == 0                  # M = 0: no launch


def test_peer_entry_preconditions(lib):
    outs = (ctypes.c_void_p * 2)(256, 512)
    f = lib.ck_int4_convrot_gemm_a8_peers
    assert f(256, 256, 256, 256, 0, 0, outs, 9, 3072, 0, 16, 1536, 3072, 1, 0, 0, 0, ctypes.c_float(0), None) == -1
    assert f(256, 256, 256, 256, 0, 0, outs, 2, 3000, 1536, 16, 1536, 3072, 1, 0, 0, 0, ctypes.c_float(0), None) == -1
    assert f(256, 256, 256, 256, 0, 0, outs, 2, 3072, 4, 16, 1536, 3072, 1, 0, 0, 0, ctypes.c_float(0), None) == -1
    flags = (ctypes.c_void_p * 2)(256, 512)
    assert lib.ck_peer_barrier(flags, 9, 0, 256, 1000, None) == -1
    assert lib.ck_peer_barrier(flags, 2, 2, 256, 1000, None) == -1
    assert lib.ck_peer_barrier(flags, 2, 0, 256, 0, None) == -1
    assert lib.ck_peer_copy_columns(flags, 1, 256, 64, 32, 64, 4, None) == -1     # offset + width > pitch
