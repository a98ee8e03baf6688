"""GPU tests of the A8 form: the int4 GEMM on int8 activation codes (one per byte)
and packed int4 weights expanded in shared memory (ck_int4_convrot_gemm_a8).

Its integer accumulators must equal the oracle's exact products, and its outputs
(plain and with the fused Dynamic-LoRA side path) must equal, bit for bit, the
packed-code GEMM's on the same codes; the fused linear that dispatches to it
(many bf16 rows) must match the oracle.
"""
import numpy as np
import pytest
import torch

from oracle import convrot_oracle as orc

pytestmark = pytest.mark.gpu


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


def operands(m, n, k, seed):
    """Random packed activation codes in [-7, 7] (the quantizer's range) in both
    forms, random packed weights, scales and bias."""
    g = torch.Generator().manual_seed(seed)
    codes = torch.randint(-7, 8, (m, k), generator=g, dtype=torch.int8)
    xp = torch.from_numpy(orc.pack_int4(codes.numpy()))
    wp = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int8)
    xs = torch.rand(m, generator=g) * 0.05 + 1e-3
    ws = torch.rand(n, generator=g) * 0.01 + 1e-4
    bias = torch.randn(n, generator=g) * 0.1
    return codes.cuda(), xp.cuda(), wp.cuda(), xs.cuda(), ws.cuda(), bias.cuda()


@pytest.mark.parametrize("m,n,k", [(129, 256, 256), (256, 512, 128), (300, 520, 768), (517, 264, 3072),
                                   (1024, 1000, 12288), (640, 3072, 15360)])
def test_a8_accumulators_exact_vs_oracle(ck, m, n, k):
    codes, xp, wp, _, _, _ = operands(m, n, k, m + n + k)
    acc = ck.int4_convrot_gemm_a8(codes, wp, torch.ones(m, device="cuda"), torch.ones(n, device="cuda"),
                                  None, torch.int32)
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy().astype(np.int64), orc.int4_gemm_acc(xp.cpu().numpy(), wp.cpu().numpy()))


def test_a8_accumulators_full_size_match_packed(ck):
    """Config-1 MLP up (4608 x 3072 -> 12288): every accumulator equals the packed GEMM's."""
    m, n, k = 4608, 12288, 3072
    codes, xp, wp, _, _, _ = operands(m, n, k, 5)
    a = ck.int4_convrot_gemm_a8(codes, wp, torch.ones(m, device="cuda"), torch.ones(n, device="cuda"),
                                None, torch.int32)
    b = ck.int4_gemm_s32(xp, wp)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("m,n,k", [(129, 264, 256), (700, 3072, 3072), (4608, 9216, 3072), (2048, 3072, 12288),
                                   (333, 15360, 3840)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("bias_dtype", [None, torch.float16, torch.float32])
def test_a8_output_equals_packed_gemm(ck, m, n, k, out_dtype, bias_dtype):
    codes, xp, wp, xs, ws, bias = operands(m, n, k, n + k)
    bias = None if bias_dtype is None else bias.to(bias_dtype)
    a = ck.int4_convrot_gemm_a8(codes, wp, xs, ws, bias, out_dtype)
    b = ck.int4_convrot_gemm(xp, wp, xs, ws, None if bias is None else bias.float(), out_dtype)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("m,n,k", [(2000, 2004, 1024), (1500, 3001, 512), (4608, 3072, 3072), (777, 9000, 256)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32, torch.int32])
def test_a8_many_tiles_ragged_equals_packed(ck, m, n, k, out_dtype):
    """Shapes with enough tiles for the weights-in-TMEM form, with ragged token and
    weight edges, N not a multiple of 8 (direct stores) and odd N."""
    codes, xp, wp, xs, ws, bias = operands(m, n, k, m * 3 + n)
    if out_dtype == torch.int32:
        a = ck.int4_convrot_gemm_a8(codes, wp, torch.ones(m, device="cuda"), torch.ones(n, device="cuda"),
                                    None, torch.int32)
        b = ck.int4_gemm_s32(xp, wp)
    else:
        a = ck.int4_convrot_gemm_a8(codes, wp, xs, ws, bias, out_dtype)
        b = ck.int4_convrot_gemm(xp, wp, xs, ws, bias, out_dtype)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert ck.device_status() == 0


def test_a8_output_vs_oracle_epilogue(ck):
    m, n, k = 300, 520, 768
    codes, xp, wp, xs, ws, bias = operands(m, n, k, 17)
    out = ck.int4_convrot_gemm_a8(codes, wp, xs, ws, bias, torch.bfloat16)
    torch.cuda.synchronize()
    ref = orc.int4_convrot_gemm(xp.cpu().numpy(), wp.cpu().numpy(), xs.cpu().numpy(), ws.cpu().numpy(),
                                bias.cpu().numpy(), "bf16")
    assert np.array_equal(bits(out), ref)


@pytest.mark.parametrize("m,n,k,r", [(256, 256, 512, 64), (300, 1000, 1024, 16), (2048, 3072, 3072, 64),
                                     (1024, 12288, 3072, 64), (4608, 3072, 12288, 32)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_a8_lora_equals_packed_lora(ck, m, n, k, r, out_dtype):
    """Same side-path operands and MMAs as the packed LoRA GEMM: the same bits."""
    codes, xp, wp, xs, ws, bias = operands(m, n, k, m + r)
    g = torch.Generator().manual_seed(r)
    lt = (torch.randn(m, r, generator=g) * 0.5).to(torch.float16).cuda()
    lb = (torch.randn(n, r, generator=g) * 0.01).to(torch.float16).cuda()
    a = ck.int4_convrot_gemm_a8(codes, wp, xs, ws, bias, out_dtype, lt, lb, 0.75)
    b = ck.int4_convrot_gemm_lora(xp, wp, xs, ws, bias, out_dtype, lt, lb, 0.75)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("m,k,n", [(129, 3072, 3072), (512, 3072, 3072), (4608, 3072, 12288), (1024, 12288, 3072)])
@pytest.mark.parametrize("g", [256, 64])
def test_fused_linear_a8_vs_oracle(ck, m, k, n, g):
    """ck_convrot_w4a4_linear with 129+ bf16 rows runs the A8 form; sampled rows are
    exact against the oracle (the quantizer is row-wise)."""
    gen = torch.Generator().manual_seed(m + n)
    x = torch.randn(m, k, generator=gen)
    x[:, torch.randperm(k, generator=gen)[: k // 100]] *= 20
    x = x.to(torch.bfloat16).cuda()
    wp = torch.randint(-128, 128, (n, k // 2), generator=gen, dtype=torch.int8).cuda()
    ws = (torch.rand(n, generator=gen) * 0.01 + 1e-4).cuda()
    bias = (torch.randn(n, generator=gen) * 0.1).to(torch.float16).cuda()
    out = ck.convrot_w4a4_linear(x, wp, ws, bias, torch.bfloat16, g)
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([np.random.default_rng(m).choice(m, 48, replace=False), [0, m - 1]]))
    ref = orc.convrot_w4a4_linear(bits(x)[rows], wp.cpu().numpy(), ws.cpu().numpy(), bias.float().cpu().numpy(), g)
    assert np.array_equal(bits(out)[rows], ref)
    assert ck.device_status() == 0



@pytest.mark.parametrize("m", [5, 17, 64, 65, 100, 128])
@pytest.mark.parametrize("k,n", [(3072, 18432), (12288, 3072), (256, 264)])
def test_public_linear_small_m_a8t_vs_oracle(m, k, n):
    """The public linear at 5 to 128 bf16 rows (swapped-tile GEMMs on packed codes) against
    the oracle at config-sized layers and a ragged one: bf16 bits equal."""
    import _int4
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = torch.Generator().manual_seed(m * 31 + k + n)
    x = torch.randn(m, k, generator=g)
    x[:, torch.randperm(k, generator=g)[: max(1, k // 100)]] *= 20
    x = x.to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.float16).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.float16).cuda()
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, 256)
    out = _int4.convrot_w4a4_linear(x, qw, ws, bias=bias, convrot_groupsize=256)
    torch.cuda.synchronize()
    xb = x.cpu().view(torch.int16).numpy().view(np.uint16)
    ref = orc.convrot_w4a4_linear(xb, qw.cpu().numpy(), ws.cpu().numpy(), bias.float().cpu().numpy(), 256)
    assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), ref)


@pytest.mark.parametrize("m,k,n", [(2304, 12288, 3072), (2304, 3072, 3072), (2200, 3072, 3072)])
def test_public_linear_192_token_tiles_vs_oracle(m, k, n):
    """Layers whose 256-token A8T grid leaves the last wave mostly empty take 192-token
    tiles (a token split of config 1 over two GPUs): sampled rows bit-exact."""
    import _int4
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = torch.Generator().manual_seed(m + k + n)
    x = torch.randn(m, k, generator=g)
    x[:, torch.randperm(k, generator=g)[: k // 100]] *= 20
    x = x.to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.float16).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.float16).cuda()
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, 256)
    out = _int4.convrot_w4a4_linear(x, qw, ws, bias=bias, convrot_groupsize=256)
    torch.cuda.synchronize()
    rows = np.unique(np.r_[np.random.default_rng(m).choice(m, 48, replace=False), 0, m - 1])
    xb = x.cpu().view(torch.int16).numpy().view(np.uint16)[rows]
    ref = orc.convrot_w4a4_linear(xb, qw.cpu().numpy(), ws.cpu().numpy(), bias.float().cpu().numpy(), 256)
    assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16)[rows], ref)
