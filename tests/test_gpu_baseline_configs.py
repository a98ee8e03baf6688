"""The public linear at every BASELINE configuration's shapes, against the oracle.

``_int4.convrot_w4a4_linear`` is run on the full activation of each layer the
benchmark times (config 0, the four config-1 layers at M = 4608, config 3's
3840 <-> 15360 MLP at M = 1024 and 4096, config 4's LoRA layers at M = 18432),
in both dispatch modes: the default (packed weights: the A8 form, int8
activation codes with in-kernel weight expansion, for M > 128) and with the
opt-in unpacked-weight cache (the int8-form GEMM on unpacked codes).
The quantizer is row-wise and every output row depends only on its own input
row, so the oracle run on a seeded sample of 64 rows (first and last included)
checks those rows exactly: bf16 bits equal. The LoRA layers are checked within
the side path's stated tolerance (see ``check_lora_rows``).
"""
import numpy as np
import pytest
import torch

from oracle import convrot_oracle as orc

pytestmark = pytest.mark.gpu

SAMPLE_ROWS = 64

# (config, M, K, N)
SHAPES = [
    ("config0", 512, 3072, 3072),
    ("config1_qkv", 4608, 3072, 9216),
    ("config1_attn_out", 4608, 3072, 3072),
    ("config1_mlp_up", 4608, 3072, 12288),
    ("config1_mlp_down", 4608, 12288, 3072),
    ("config3_up_m1024", 1024, 3840, 15360),
    ("config3_down_m1024", 1024, 15360, 3840),
    ("config3_up_m4096", 4096, 3840, 15360),
    ("config3_down_m4096", 4096, 15360, 3840),
]


@pytest.fixture(scope="module")
def api():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import _int4
    assert _int4.is_available()
    return _int4


def bits(t):
    t = t.detach().cpu().contiguous()
    return t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()


def synth_layer(m, k, n, seed):
    """The benchmark's value recipe: x ~ N(0,1) with 1 % of channels x20, W ~ N(0, 0.02)
    quantized by the load-time quantizer from fp16, bias ~ N(0, 0.01) stored fp16."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    x[:, torch.randperm(k, generator=g)[: k // 100]] *= 20
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.float16)
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).to(torch.float16)
    return x.to(torch.bfloat16).cuda(), w.cuda(), bias.cuda()


def sample_rows(m, seed):
    rng = np.random.default_rng(seed)
    rows = rng.choice(m, size=min(m, SAMPLE_ROWS), replace=False)
    return np.unique(np.concatenate([rows, [0, m - 1]]))


@pytest.mark.parametrize("unpacked", [False, True], ids=["default", "cached"])
@pytest.mark.parametrize("name,m,k,n", SHAPES, ids=[s[0] for s in SHAPES])
def test_public_linear_vs_oracle_on_sampled_rows(api, name, m, k, n, unpacked):
    x, w, bias = synth_layer(m, k, n, seed=m + k + n)
    qw, ws = api.quantize_convrot_w4a4_weight(w, 256)
    api.set_unpacked_weights(unpacked)
    try:
        assert api._use_unpacked(x, qw, 256) == unpacked
        out = api.convrot_w4a4_linear(x, qw, ws, bias=bias, convrot_groupsize=256)
        torch.cuda.synchronize()
    finally:
        api.set_unpacked_weights(False)
    rows = sample_rows(m, seed=n)
    ref = orc.convrot_w4a4_linear(bits(x)[rows], qw.cpu().numpy(), ws.cpu().numpy(),
                                  bias.float().cpu().numpy(), 256)
    got = bits(out)[rows]
    assert out.shape == (m, n) and out.dtype == torch.bfloat16
    assert np.array_equal(got, ref), f"{name}: {np.count_nonzero(got != ref)} of {got.size} sampled values differ"


def check_lora_rows(got_bits, x_rows, qw, ws, bias, down, up, scale, t_unit):
    """Fused LoRA output vs the oracle: int4 epilogue + the exact side path
    (x.A^T).B^T * scale, one rounding. Allowed difference: one bf16 unit of the
    result; the side path's operand rounding (T = x.A^T and B to a type of unit
    roundoff t_unit); the fp32 accumulation of T over K (bounded by
    K * 2^-24 * |x|.|A|^T); fp32 accumulation noise of all summands."""
    xp, xs = orc.convrot_quant_int4(x_rows, 256, "bf16")
    acc = orc.int4_gemm_acc(xp, qw)
    xf = orc.bf16_bits_to_f32(x_rows).astype(np.float64)
    t_exact = xf @ down.astype(np.float64).T
    ref = orc.int4_gemm_epilogue_lora(acc, xs, ws, bias, t_exact, up, scale, "f32")
    g = orc.bf16_bits_to_f32(got_bits).astype(np.float64)
    r = ref.astype(np.float64)
    up_abs = np.abs(up.astype(np.float64)).T
    side_mag = (np.abs(t_exact) @ up_abs) * abs(scale)
    t_acc = (np.abs(xf) @ np.abs(down.astype(np.float64)).T) * (down.shape[1] * 2.0 ** -24)
    mag = (np.abs(acc.astype(np.float64) * xs.reshape(-1, 1) * ws.reshape(1, -1))
           + np.abs(bias).reshape(1, -1) + side_mag)
    tol = (np.maximum(np.abs(g), np.abs(r)) * 2.0 ** -7 + side_mag * 2 * t_unit
           + (t_acc @ up_abs) * abs(scale) + mag * 2.0 ** -18)
    bad = np.abs(g - r) > tol
    assert not bad.any(), f"{np.count_nonzero(bad)} sampled values outside the LoRA tolerance"


@pytest.mark.parametrize("unpacked", [False, True], ids=["default", "cached"])
@pytest.mark.parametrize("k,n", [(3072, 12288), (12288, 3072)], ids=["mlp_up", "mlp_down"])
def test_public_lora_linear_config4_vs_oracle_on_sampled_rows(api, k, n, unpacked):
    """Config 4: M = 18432, rank-64 adapter, A, B ~ N(0, 0.01), alpha = 64."""
    m, r = 18432, 64
    x, w, bias = synth_layer(m, k, n, seed=k + n)
    g = torch.Generator().manual_seed(7)
    down = (torch.randn(r, k, generator=g) * 0.01).to(torch.bfloat16).cuda()
    up = (torch.randn(n, r, generator=g) * 0.01).to(torch.bfloat16).cuda()
    scale = 64.0 / r
    qw, ws = api.quantize_convrot_w4a4_weight(w, 256)
    api.set_unpacked_weights(unpacked)
    try:
        out = api.convrot_w4a4_linear_lora(x, qw, ws, bias, [(down, up, scale)], 256)
        torch.cuda.synchronize()
    finally:
        api.set_unpacked_weights(False)
    rows = sample_rows(m, seed=n + 1)
    check_lora_rows(bits(out)[rows], bits(x)[rows], qw.cpu().numpy(), ws.cpu().numpy(),
                    bias.float().cpu().numpy(), down.float().cpu().numpy(), up.float().cpu().numpy(),
                    scale, api.LORA_OPERAND_UNIT)
