"""GPU tests of the public linear with one to four bf16 rows (the GEMV path).

``_int4.convrot_w4a4_linear`` quantizes such rows (one launch) and streams the
packed weights through the few-token GEMV (a second, programmatic dependent
launch). Its output must equal the oracle's bit for bit for every rows-per-warp
plan of the GEMV (K up to 15360, both group sizes), with and without bias, in
bf16 and f32, including the quantizer's edge rows (all-zero rows: the scale
floor; subnormal-range rows; values near the top of the range), and when calls
are chained in one CUDA graph with each input the previous call's output.
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


def layer(m, k, n, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    x[:, torch.randperm(k, generator=g)[: max(1, k // 100)]] *= 20
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.float16)
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.float16)
    return x.to(torch.bfloat16).cuda(), w.cuda(), bias.cuda()


def oracle_linear(x, qw, ws, bias, group, out_dtype="bf16"):
    xp, xs = orc.convrot_quant_int4(bits(x), group, "bf16")
    acc = orc.int4_gemm_acc(xp, qw.cpu().numpy())
    b = None if bias is None else bias.float().cpu().numpy()
    return orc.int4_gemm_epilogue(acc, xs, ws.cpu().numpy(), b, out_dtype)


# K picks the rows-per-warp plan: <= 4096 four rows a warp, <= 8192 two, else one
@pytest.mark.parametrize("m", [1, 2, 3, 4])
@pytest.mark.parametrize("k,n,group", [(3072, 18432, 256), (256, 1000, 256), (768, 2056, 64), (6144, 3072, 256),
                                       (12288, 3072, 256), (15360, 1544, 64)])
def test_few_token_linear_vs_oracle(ck, m, k, n, group):
    x, w, bias = layer(m, k, n, seed=m * 7 + k + n)
    import _int4
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, group)
    out = _int4.convrot_w4a4_linear(x, qw, ws, bias=bias, convrot_groupsize=group)
    torch.cuda.synchronize()
    assert np.array_equal(bits(out), oracle_linear(x, qw, ws, bias, group))


@pytest.mark.parametrize("group", [256, 64])
def test_few_token_linear_f32_out_no_bias(ck, group):
    import _int4
    x, w, _ = layer(3, 3072, 4104, seed=group)
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, group)
    out = ck.convrot_w4a4_linear(x, qw, ws, None, torch.float32, group)
    torch.cuda.synchronize()
    assert np.array_equal(bits(out).view(np.uint32), oracle_linear(x, qw, ws, None, group, "f32").view(np.uint32))


@pytest.mark.parametrize("group", [256, 64])
def test_few_token_linear_zero_tiny_and_huge_rows(ck, group):
    import _int4
    k, n = 3072, 2048
    _, w, bias = layer(4, k, n, seed=5)
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, group)
    x = torch.randn(4, k)
    x[0] = 0.0
    x[1] = 1e-30
    x[1, ::7] = -3e-39
    x[2] *= 1e30
    x[2, 5] = 1e35
    x = x.to(torch.bfloat16).cuda()
    out = _int4.convrot_w4a4_linear(x, qw, ws, bias=bias, convrot_groupsize=group)
    torch.cuda.synchronize()
    assert np.array_equal(bits(out), oracle_linear(x, qw, ws, bias, group))


def test_few_token_linear_equals_quantizer_then_gemm(ck):
    """The fused entry gives the bits of the two reference-style calls."""
    import _int4
    x, w, bias = layer(4, 3072, 9216, seed=9)
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, 256)
    fused = _int4.convrot_w4a4_linear(x, qw, ws, bias=bias, convrot_groupsize=256)
    xq, xs = ck.convrot_quant_int4(x, 256)
    two = ck.int4_convrot_gemm(xq, qw, xs, ws, bias.float(), torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(fused.view(torch.int16), two.view(torch.int16))


def test_few_token_linear_back_to_back_in_a_graph(ck):
    """Calls chained in one CUDA graph, each input the previous output (programmatic
    dependent launches back to back), equal to the same chain run eagerly."""
    import _int4
    k = n = 3072
    x0, w, bias = layer(1, k, n, seed=21)
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, 256)
    steps = 6
    outs = []
    xin = x0
    for _ in range(steps):                       # eager reference chain
        xin = _int4.convrot_w4a4_linear(xin, qw, ws, bias=bias, convrot_groupsize=256)
        outs.append(xin)
    torch.cuda.synchronize()
    static_x = x0.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = static_x
        g_outs = []
        for _ in range(steps):
            y = _int4.convrot_w4a4_linear(y, qw, ws, bias=bias, convrot_groupsize=256)
            g_outs.append(y)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        for a, b in zip(outs, g_outs):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16))
