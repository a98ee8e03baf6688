"""GPU tests of the rotation fused into the producer of x (LayerNorm + modulation).

``ck_convrot_quant_int4_lnmod`` normalises and modulates each bf16 row, then
rotates and quantizes it, in one pass over x. Codes and scales must equal the
oracle's ``convrot_quant_int4(layernorm_modulate(x))`` bit for bit (packed and
one-int8-per-code forms, both group sizes, ragged row counts, rows that are
constant, zero, tiny or large, no modulation vectors), and the fused linear
must equal the oracle's linear of the same modulated rows. Against torch's own
LayerNorm followed by the modulation and the unfused public linear, the output
stays within the bf16 rounding of the statistics.
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


def rows(m, k, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g) * 2 + 0.3
    x[:, torch.randperm(k, generator=g)[: k // 100]] *= 20
    scale = (torch.randn(k, generator=g) * 0.2).to(torch.bfloat16)
    shift = (torch.randn(k, generator=g) * 0.2).to(torch.bfloat16)
    return x.to(torch.bfloat16).cuda(), scale.cuda(), shift.cuda()


@pytest.mark.parametrize("group", [256, 64])
@pytest.mark.parametrize("unpacked", [False, True], ids=["packed", "unpacked"])
@pytest.mark.parametrize("m,k", [(1, 3072), (7, 3072), (130, 3840), (4608, 3072), (333, 6144), (64, 256)])
def test_lnmod_quant_bit_exact_vs_oracle(ck, m, k, group, unpacked):
    x, scale, shift = rows(m, k, seed=m + k + group)
    q, s = ck.convrot_quant_int4_lnmod(x, scale, shift, 1e-6, group, unpacked)
    torch.cuda.synchronize()
    sel = np.arange(m) if m <= 512 else np.unique(np.r_[np.random.default_rng(m).choice(m, 64), 0, m - 1])
    qo, so = orc.convrot_quant_int4_lnmod(bits(x)[sel], bits(scale), bits(shift), 1e-6, group)
    assert np.array_equal(bits(s)[sel].view(np.uint32), so.view(np.uint32))
    qg = bits(q)[sel]
    assert np.array_equal(orc.pack_int4(qg) if unpacked else qg, qo)


def test_lnmod_quant_special_rows_and_no_modulation(ck):
    x, _, _ = rows(6, 3072, seed=3)
    xf = x.float().cpu()
    xf[0] = 0.0                      # all zero: var 0, scale floor
    xf[1] = 4.0                      # constant row
    xf[2] = 1e-30                    # tiny
    xf[3, ::5] = 3e4                 # large values
    xf[4] *= 1e20
    x = xf.to(torch.bfloat16).cuda()
    for scale, shift in ((None, None), (torch.full((3072,), 0.5, dtype=torch.bfloat16).cuda(), None)):
        q, s = ck.convrot_quant_int4_lnmod(x, scale, shift, 1e-6, 256, False)
        torch.cuda.synchronize()
        qo, so = orc.convrot_quant_int4_lnmod(bits(x), None if scale is None else bits(scale), None, 1e-6, 256)
        assert np.array_equal(bits(s).view(np.uint32), so.view(np.uint32))
        assert np.array_equal(bits(q), qo)


@pytest.mark.parametrize("m,k,n", [(4096, 3072, 9216), (512, 3072, 12288), (3, 3072, 3072)])
def test_lnmod_linear_vs_oracle(ck, m, k, n):
    import _int4
    x, scale, shift = rows(m, k, seed=n)
    g = torch.Generator().manual_seed(k)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.float16).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.float16).cuda()
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, 256)
    out = _int4.convrot_w4a4_linear_lnmod(x, qw, ws, bias, shift=shift, scale=scale)
    torch.cuda.synchronize()
    sel = np.arange(m) if m <= 64 else np.unique(np.r_[np.random.default_rng(n).choice(m, 48), 0, m - 1])
    y = orc.layernorm_modulate(bits(x)[sel], bits(scale), bits(shift), 1e-6)
    ref = orc.convrot_w4a4_linear(y, qw.cpu().numpy(), ws.cpu().numpy(), bias.float().cpu().numpy(), 256)
    assert np.array_equal(bits(out)[sel], ref)


def test_lnmod_linear_close_to_torch_layernorm_then_linear(ck):
    """Same result as the model's unfused sequence up to the statistics' rounding."""
    import _int4
    m, k, n = 1024, 3072, 3072
    x, scale, shift = rows(m, k, seed=11)
    g = torch.Generator().manual_seed(12)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.float16).cuda()
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, 256)
    fused = _int4.convrot_w4a4_linear_lnmod(x, qw, ws, None, shift=shift, scale=scale)
    xn = torch.nn.functional.layer_norm(x.float(), (k,), eps=1e-6).to(torch.bfloat16)
    unfused = _int4.convrot_w4a4_linear((1 + scale) * xn + shift, qw, ws, None)
    torch.cuda.synchronize()
    rel = (fused.float() - unfused.float()).norm() / unfused.float().norm()
    assert float(rel) < 5e-3


def test_lnmod_rejects_bad_shapes(ck):
    x = torch.zeros(4, 320, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError):
        ck.convrot_quant_int4_lnmod(x, None, None, 1e-6, 64, False)      # K % 256
    x = torch.zeros(4, 8192, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError):
        ck.convrot_quant_int4_lnmod(x, None, None, 1e-6, 256, False)     # K > 6144


def test_module_forward_lnmod(ck):
    """Int4ConvRotLinear.forward_lnmod: the fused pass for plain int4 layers; with a
    Dynamic-LoRA adapter, torch normalises first and the LoRA linear runs."""
    import _int4
    from _int4.linear import Int4ConvRotLinear
    m, k, n = 300, 3072, 1024
    x, scale, shift = rows(m, k, seed=21)
    g = torch.Generator().manual_seed(22)
    lin = Int4ConvRotLinear(k, n, True, device="cuda")
    qw, ws = _int4.quantize_convrot_w4a4_weight((torch.randn(n, k, generator=g) * 0.02).to(torch.float16).cuda(), 256)
    lin._q.copy_(qw)
    lin._qs.copy_(ws)
    got = lin.forward_lnmod(x, shift, scale)
    want = _int4.convrot_w4a4_linear_lnmod(x, qw, ws, lin.bias, shift=shift, scale=scale)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    down = (torch.randn(16, k, generator=g) * 0.01).cuda()
    up = (torch.randn(n, 16, generator=g) * 0.01).cuda()
    lin.set_dynamic_lora([(down, up, 16.0, 1.0)])
    got = lin.forward_lnmod(x, shift, scale)
    xn = torch.nn.functional.layer_norm(x, (k,), eps=1e-6) * (1 + scale) + shift
    want = lin(xn)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
