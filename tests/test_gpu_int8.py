"""GPU parity tests of the W8A8 tier: the int8 rotate+quantize kernel, the int8
tensor-core GEMM and the int8 linear, against the oracle (bit-exact) and the
reference's eager W8A8 linear (golden vectors, 1e-2 relative L2).
"""
import os

import numpy as np
import pytest
import torch

from oracle import convrot_oracle as orc
from oracle import eager_torch

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def ck():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import _int4
    from _int4 import cuda_loader
    assert _int4.is_available()
    return cuda_loader


def bits(t):
    t = t.detach().cpu().contiguous()
    return t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()


def activation(m, k, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    x[:, torch.randperm(k, generator=g)[: max(1, k // 100)]] *= 20
    return x.to(torch.bfloat16).cuda()


# ------------------------------------------------------------------ quantizer

@pytest.mark.parametrize("m,k,g", [(1, 768, 256), (7, 3072, 256), (129, 512, 64), (300, 3072, 64),
                                   (3, 12288, 256), (2, 15360, 256), (1000, 12288, 256), (2000, 3072, 256)])
def test_int8_quant_bit_exact_vs_oracle(ck, m, k, g):
    x = activation(m, k, m + k)
    q, s = ck.convrot_quant_int8(x, g)
    torch.cuda.synchronize()
    qo, so = orc.convrot_quant_int8(bits(x), g, "bf16")
    assert np.array_equal(bits(s).view(np.uint32), so.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), qo)


def test_int8_quant_zero_tiny_and_large_rows(ck):
    x = activation(24, 3072, 7).float()
    x[3] = 0.0
    x[7] = 1e-30
    x[8, ::7] = -3e-39
    x[11] *= 1e30
    x = x.to(torch.bfloat16)
    q, s = ck.convrot_quant_int8(x, 256)
    torch.cuda.synchronize()
    qo, so = orc.convrot_quant_int8(bits(x), 256, "bf16")
    assert np.array_equal(bits(s).view(np.uint32), so.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), qo)


def test_int8_quant_rejects_unsupported_shapes(ck):
    with pytest.raises(RuntimeError, match="int8 quantizer"):
        ck.convrot_quant_int8(activation(4, 320, 1), 64)                      # ragged tile
    with pytest.raises(RuntimeError, match="int8 quantizer"):
        ck.convrot_quant_int8(activation(4, 512, 1).to(torch.float16), 256)   # not bf16


# ------------------------------------------------------------------ GEMM

def rand_i8(rows, k, seed, lo=-128):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, 128, (rows, k), generator=g, dtype=torch.int8).cuda()


# 256x128 and 256x256 pair tiles (staged and direct stores), tails in M, N and K
# (K not a multiple of the 128-byte k-stage), M below one pair tile.
I8_SHAPES = [(1, 64, 64), (5, 96, 48), (129, 384, 512), (300, 1000, 1040), (512, 3072, 3072),
             (4608, 256, 64), (1024, 3072, 4096), (2048, 2304, 1536)]


@pytest.mark.parametrize("m,n,k", I8_SHAPES)
def test_int8_gemm_accumulators_exact(ck, m, n, k):
    x, w = rand_i8(m, k, m), rand_i8(n, k, n + 1)
    acc = ck.int8_gemm_s32(x, w)
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy(), orc.int8_gemm_acc(x.cpu().numpy(), w.cpu().numpy()))


@pytest.mark.parametrize("m,n,k", [(77, 300, 1024), (515, 2056, 320), (1024, 3072, 3072), (256, 512, 6144)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("with_bias", [True, False])
def test_int8_gemm_epilogue_bit_exact(ck, m, n, k, out_dtype, with_bias):
    g = torch.Generator().manual_seed(m * 7 + n)
    x, w = rand_i8(m, k, m, lo=-127), rand_i8(n, k, n, lo=-127)
    xs = (torch.rand(m, generator=g) * 0.05 + 1e-3).cuda()
    ws = (torch.rand(n, generator=g) * 0.01 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).cuda() if with_bias else None
    out = ck.int8_convrot_gemm(x, w, xs, ws, bias, out_dtype)
    torch.cuda.synchronize()
    acc = orc.int8_gemm_acc(x.cpu().numpy(), w.cpu().numpy())
    ref = orc.int4_gemm_epilogue(acc, xs.cpu().numpy(), ws.cpu().numpy(),
                                 bias.cpu().numpy() if with_bias else None,
                                 "bf16" if out_dtype == torch.bfloat16 else "f32")
    assert np.array_equal(bits(out), ref)


# ------------------------------------------------------------------ linear

@pytest.mark.parametrize("case", ["g256", "g64", "cfg0"])
def test_w8a8_linear_vs_reference_and_oracle(ck, case):
    import _int4
    g = np.load(os.path.join(GOLD, "int8.npz"))
    grp, k, n, m = (int(v) for v in g[f"l_{case}_meta"])
    x = torch.from_numpy(g[f"l_{case}_x"].view(np.int16)).view(torch.bfloat16).cuda()
    qw = torch.from_numpy(g[f"l_{case}_qw"]).cuda()
    ws = torch.from_numpy(g[f"l_{case}_ws"]).cuda()
    bias = torch.from_numpy(g[f"l_{case}_bias"].view(np.int16)).view(torch.bfloat16).cuda().to(torch.float16)
    out = _int4.convrot_w8a8_linear(x, qw, ws, bias=bias, convrot_groupsize=grp)
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16 and out.shape == (m, n)
    ora = orc.convrot_w8a8_linear(g[f"l_{case}_x"], g[f"l_{case}_qw"], g[f"l_{case}_ws"],
                                  bits(bias.float()), grp)
    assert np.array_equal(bits(out), ora)
    ref = orc.bf16_bits_to_f32(g[f"l_{case}_out"])
    got = orc.bf16_bits_to_f32(bits(out))
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-2


def test_w8a8_linear_other_shapes_take_torch_quant_then_native_gemm(ck):
    """fp16 activations (not taken by the int8 quant kernel) still run the int8 GEMM."""
    import _int4
    x = activation(33, 512, 3).to(torch.float16)
    w = (torch.randn(64, 512) * 0.02).to(torch.float16).cuda()
    from _int4 import int8_eager
    qw, ws = int8_eager.quantize_convrot_w8a8_weight(w, 256)
    out = _int4.convrot_w8a8_linear(x, qw, ws)
    ref = eager_torch.convrot_w8a8_linear(x, qw, ws)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16
    rel = (out.float() - ref.float()).norm() / ref.float().norm()
    assert rel < 1e-2, rel


# ------------------------------------------------------------------ unpacked-code path (int4 on the int8 pipeline)

def test_int4_unpack_matches_codec(ck):
    p = rand_i8(333, 1536, 9)                                   # packed [R, K/2]
    codes = ck.int4_unpack(p)
    torch.cuda.synchronize()
    assert np.array_equal(codes.cpu().numpy(), orc.unpack_int4(p.cpu().numpy()))


@pytest.mark.parametrize("m,k,g", [(129, 3072, 256), (300, 768, 64), (4608, 3072, 256), (5, 12288, 256)])
def test_int4_quant_unpacked_equals_packed(ck, m, k, g):
    x = activation(m, k, m + 3)
    qu, su = ck.convrot_quant_int4_unpacked(x, g)
    qp, sp = ck.convrot_quant_int4(x, g)
    torch.cuda.synchronize()
    assert torch.equal(su, sp)
    assert np.array_equal(qu.cpu().numpy(), orc.unpack_int4(qp.cpu().numpy()))


@pytest.mark.parametrize("m,k,n", [(129, 3072, 3072), (300, 768, 520), (4608, 3072, 12288), (1024, 12288, 3072),
                                   (700, 3840, 15360)])
@pytest.mark.parametrize("bias_dtype", [None, torch.float16, torch.float32])
def test_int4_linear_unpacked_equals_packed(ck, m, k, n, bias_dtype):
    g = torch.Generator().manual_seed(n)
    x = activation(m, k, m)
    wp = rand_i8(n, k // 2, n)
    ws = (torch.rand(n, generator=g) * 0.01 + 1e-4).cuda()
    bias = None if bias_dtype is None else (torch.randn(n, generator=g) * 0.1).to(bias_dtype).cuda()
    a = ck.convrot_w4a4_linear_unpacked(x, ck.int4_unpack(wp), ws, bias, torch.bfloat16, 256)
    b = ck.convrot_w4a4_linear(x, wp, ws, bias, torch.bfloat16, 256)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_public_linear_takes_unpacked_path_for_many_tokens(ck):
    import _int4
    from _int4 import weight_cache
    was = weight_cache.enabled()
    weight_cache.enable(True)
    x = activation(512, 3072, 1)
    w = (torch.randn(1024, 3072) * 0.02).to(torch.float16).cuda()
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, 256)
    before = weight_cache.cached_bytes()
    y = _int4.convrot_w4a4_linear(x, qw, ws)
    assert weight_cache.cached_bytes() == before + 1024 * 3072
    weight_cache.enable(False)
    y_packed = _int4.convrot_w4a4_linear(x, qw, ws)
    weight_cache.enable(was)
    torch.cuda.synchronize()
    assert torch.equal(y, y_packed)
    ora = orc.convrot_w4a4_linear(bits(x), qw.cpu().numpy(), ws.cpu().numpy(), None, 256)
    assert np.array_equal(bits(y), ora)


@pytest.mark.parametrize("m,k,n,unpacked", [(64, 12288, 3072, True), (32, 3072, 3072, True),
                                           (16, 3072, 3072, False), (64, 3072, 12288, False),
                                           (4, 3072, 3072, False)])
def test_public_linear_few_rows_dispatch(ck, m, k, n, unpacked):
    """5..128 tokens: few-row layers (N <= 4096, M * K >= 8 * 12288) take the unpacked
    path, others stay packed; the output bits are the packed path's either way."""
    import _int4
    from _int4 import weight_cache
    was = weight_cache.enabled()
    weight_cache.enable(True)
    x = activation(m, k, m + n)
    w = (torch.randn(n, k) * 0.02).to(torch.float16).cuda()
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, 256)
    before = weight_cache.cached_bytes()
    y = _int4.convrot_w4a4_linear(x, qw, ws)
    assert weight_cache.cached_bytes() == before + (n * k if unpacked else 0)
    weight_cache.enable(False)
    y_packed = _int4.convrot_w4a4_linear(x, qw, ws)
    weight_cache.enable(was)
    torch.cuda.synchronize()
    assert torch.equal(y, y_packed)
