"""GPU tests of the Dynamic-LoRA side path fused into the int4 GEMM epilogue.

The side path's arithmetic belongs to ComfyUI's LoRA adapter, which the
reference does not vendor (int4_ops.py:181-192 calls ``v.h(x, out)``), so it has
no pinned golden vectors; it is checked against the oracle's definition
(oracle.int4_gemm_epilogue_lora) and against a plain fp32 torch reference. Its
operands are fp16, the dtype the reference prepares adapters in
(int4_ops.py:165-167).

Tolerance: the tensor cores accumulate L = T . B^T in fp32 in an unspecified
order, so the fused output may differ from the oracle by at most one unit in the
last place of the output dtype, on a small fraction of elements.
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


def check_close_bf16(got_bits, ref_bits, summand_mag, max_frac=1e-3):
    """One bf16 ulp of the result, plus fp32 accumulation noise of the summands
    (sum of absolute products; matters only where the terms cancel)."""
    g = orc.bf16_bits_to_f32(got_bits)
    r = orc.bf16_bits_to_f32(ref_bits)
    tol = np.maximum(np.abs(g), np.abs(r)) * np.float32(2.0 ** -7) + summand_mag * np.float32(2.0 ** -18)
    assert np.all(np.abs(g - r) <= tol)
    assert np.count_nonzero(got_bits != ref_bits) <= max(2, int(max_frac * g.size))


@pytest.mark.parametrize("m,n,k,r", [(256, 256, 512, 64), (300, 1000, 1024, 16), (1024, 3072, 3072, 64),
                                     (129, 264, 256, 8), (2048, 3072, 256, 32)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_fused_lora_epilogue_vs_oracle(ck, m, n, k, r, out_dtype):
    g = torch.Generator().manual_seed(m + n + r)
    xp = torch.randint(-128, 128, (m, k // 2), generator=g, dtype=torch.int8).cuda()
    wp = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int8).cuda()
    xs = (torch.rand(m, generator=g) * 0.05 + 1e-3).cuda()
    ws = (torch.rand(n, generator=g) * 0.01 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).cuda()
    lt = (torch.randn(m, r, generator=g) * 0.5).to(torch.float16).cuda()
    lb = (torch.randn(n, r, generator=g) * 0.01).to(torch.float16).cuda()
    scale = 0.75
    out = ck.int4_convrot_gemm_lora(xp, wp, xs, ws, bias, out_dtype, lt, lb, scale)
    torch.cuda.synchronize()
    acc = orc.int4_gemm_acc(bits(xp), bits(wp))
    ref = orc.int4_gemm_epilogue_lora(acc, bits(xs), bits(ws), bits(bias), lt.float().cpu().numpy(),
                                      lb.float().cpu().numpy(), scale,
                                      "bf16" if out_dtype == torch.bfloat16 else "f32")
    mag = (np.abs(acc.astype(np.float64) * bits(xs).reshape(-1, 1) * bits(ws).reshape(1, -1))
           + np.abs(bits(bias)).reshape(1, -1)
           + (np.abs(lt.float().cpu().numpy().astype(np.float64)) @ np.abs(lb.float().cpu().numpy()).T) * scale)
    if out_dtype == torch.bfloat16:
        check_close_bf16(bits(out), ref, mag)
    else:
        got = bits(out)
        assert np.all(np.abs(got - ref) <= 2.0 ** -22 * np.abs(ref) + 2.0 ** -18 * mag)


def test_fused_lora_zero_side_path_matches_plain_gemm(ck):
    """With B = 0 the fused kernel must reproduce the plain GEMM bit for bit."""
    m, n, k, r = 512, 1024, 1024, 64
    g = torch.Generator().manual_seed(3)
    xp = torch.randint(-128, 128, (m, k // 2), generator=g, dtype=torch.int8).cuda()
    wp = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int8).cuda()
    xs = torch.rand(m, generator=g).cuda()
    ws = torch.rand(n, generator=g).cuda() * 0.01
    bias = torch.randn(n, generator=g).cuda() * 0.01
    lt = torch.randn(m, r, generator=g).to(torch.float16).cuda()
    lb = torch.zeros(n, r, dtype=torch.float16, device="cuda")
    a = ck.int4_convrot_gemm_lora(xp, wp, xs, ws, bias, torch.bfloat16, lt, lb, 1.0)
    b = ck.int4_convrot_gemm(xp, wp, xs, ws, bias, torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_lora_api_single_and_stacked_adapters(ck):
    import _int4
    m, k, n = 384, 768, 512
    g = torch.Generator().manual_seed(9)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.float16).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.float16).cuda()
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, 256)
    a1 = ((torch.randn(32, k, generator=g) * 0.01).cuda(), (torch.randn(n, 32, generator=g) * 0.01).cuda(), 2.0)
    a2 = ((torch.randn(16, k, generator=g) * 0.01).cuda(), (torch.randn(n, 16, generator=g) * 0.01).cuda(), 0.5)
    base = _int4.convrot_w4a4_linear(x, qw, ws, bias).float()
    for adapters in ([a1], [a1, a2]):
        out = _int4.convrot_w4a4_linear_lora(x, qw, ws, bias, adapters).float()
        side = sum(s * ((x.float() @ d.float().t()) @ u.float().t()) for d, u, s in adapters)
        ref = base + side
        rel = (out - ref).norm() / ref.norm()
        assert rel < 1e-2, rel
        # the side path is actually present
        assert (out - base).norm() / side.norm() > 0.9


def test_lora_rejects_bad_rank(ck):
    m, n, k = 64, 64, 64
    xp = torch.zeros(m, k // 2, dtype=torch.int8, device="cuda")
    wp = torch.zeros(n, k // 2, dtype=torch.int8, device="cuda")
    s = torch.ones(max(m, n), device="cuda")
    lt = torch.zeros(m, 72, dtype=torch.float16, device="cuda")
    lb = torch.zeros(n, 72, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="rank"):
        ck.int4_convrot_gemm_lora(xp, wp, s[:m], s[:n], None, torch.bfloat16, lt, lb, 1.0)


# ------------------------------------------------------------------ int8 operands (W8A8 tier, unpacked int4 codes)

# 256 x 128 tiles (few tiles) and 256 x 256 tiles (at least one per SM), ragged edges
@pytest.mark.parametrize("m,n,k,r", [(256, 256, 512, 64), (300, 1000, 1024, 16), (1024, 3072, 3072, 64),
                                     (129, 264, 256, 8), (700, 3072, 12288, 64), (2304, 4096, 1024, 64),
                                     (4608, 3072, 3072, 32), (2000, 3000, 2048, 64)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_int8_lora_on_unpacked_codes_equals_packed(ck, m, n, k, r, out_dtype):
    """Same accumulators (sign-extended codes), same LoRA MMAs (a rank step of K = 16
    per output element, whatever the tile width), same epilogue: bit-identical to the
    packed kernel."""
    g = torch.Generator().manual_seed(m * 3 + n + r)
    xp = torch.randint(-128, 128, (m, k // 2), generator=g, dtype=torch.int8).cuda()
    wp = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int8).cuda()
    xs = (torch.rand(m, generator=g) * 0.05 + 1e-3).cuda()
    ws = (torch.rand(n, generator=g) * 0.01 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.float16).cuda()
    lt = (torch.randn(m, r, generator=g) * 0.5).to(torch.float16).cuda()
    lb = (torch.randn(n, r, generator=g) * 0.01).to(torch.float16).cuda()
    a = ck.int8_convrot_gemm_lora(ck.int4_unpack(xp), ck.int4_unpack(wp), xs, ws, bias, out_dtype, lt, lb, 0.75)
    b = ck.int4_convrot_gemm_lora(xp, wp, xs, ws, bias, out_dtype, lt, lb, 0.75)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_public_lora_linear_many_tokens_takes_unpacked_path(ck):
    """With the opt-in cache the LoRA linear runs on unpacked weights; without it,
    the A8 form on the packed weights: the same bits."""
    import _int4
    from _int4 import weight_cache
    was = weight_cache.enabled()
    weight_cache.enable(True)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(512, 3072, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(1024, 3072, generator=g) * 0.02).to(torch.float16).cuda()
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, 256)
    ad = [((torch.randn(64, 3072, generator=g) * 0.01).cuda(), (torch.randn(1024, 64, generator=g) * 0.01).cuda(), 1.0)]
    before = weight_cache.cached_bytes()
    y = _int4.convrot_w4a4_linear_lora(x, qw, ws, None, ad)
    assert weight_cache.cached_bytes() == before + 1024 * 3072
    weight_cache.enable(False)
    y_packed = _int4.convrot_w4a4_linear_lora(x, qw, ws, None, ad)
    weight_cache.enable(was)
    torch.cuda.synchronize()
    assert torch.equal(y, y_packed)


def test_w8a8_lora_api_and_int8_module(ck):
    """W8A8 tier with adapters: the side path fused into the int8 GEMM epilogue, against
    the plain W8A8 linear plus an fp32 torch side path (1e-2 relative L2), also through
    Int4ConvRotLinear in int8 mode."""
    import _int4
    from _int4 import int8_eager
    from _int4.linear import Int4ConvRotLinear
    m, k, n = 384, 768, 512
    g = torch.Generator().manual_seed(11)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.float16).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.float16).cuda()
    qw, ws = int8_eager.quantize_convrot_w8a8_weight(w, 256)
    a1 = ((torch.randn(32, k, generator=g) * 0.01).cuda(), (torch.randn(n, 32, generator=g) * 0.01).cuda(), 2.0)
    base = _int4.convrot_w8a8_linear(x, qw, ws, bias).float()
    side = 2.0 * ((x.float() @ a1[0].float().t()) @ a1[1].float().t())
    out = _int4.convrot_w8a8_linear_lora(x, qw, ws, bias, [a1]).float()
    ref = base + side
    assert (out - ref).norm() / ref.norm() < 1e-2
    assert (out - base).norm() / side.norm() > 0.9
    mod = Int4ConvRotLinear(k, n, device="cuda")
    mod.load_state_dict({"weight": qw, "weight_scale": ws, "bias": bias})
    assert mod._qmode == "int8"
    mod.set_dynamic_lora([(a1[0], a1[1], 64, 2.0 * 32 / 64)])       # alpha / r * strength = 2.0
    assert torch.equal(mod(x), _int4.convrot_w8a8_linear_lora(x, qw, ws, bias, [a1]))
