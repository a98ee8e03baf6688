"""GPU parity tests: the sm_100a kernels against the CPU oracle and the reference goldens.

Bar (per stage):
  * packed int4 codes and f32 scales: bit-exact vs the oracle; bit-exact vs the
    reference eager quantizer when fed its rotated tensor;
  * int32 accumulators: bit-exact vs exact integer products;
  * dequantized output: bit-exact vs the oracle epilogue; within 1e-2 relative
    L2 of the reference eager linear.
"""
import os

import numpy as np
import pytest
import torch

from oracle import convrot_oracle as orc

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


@pytest.fixture(scope="module")
def ck():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import _int4
    from _int4 import cuda_loader
    assert _int4.is_available(), "sm_100 device with the CUDA library required"
    return cuda_loader


def to_storage(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def from_storage(a: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == "bf16":
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a))


def activation(m, k, dtype="bf16", seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    idx = torch.randperm(k, generator=g)[: max(1, k // 100)]
    x[:, idx] *= 20
    return x.to(DT[dtype]).cuda()


def random_packed(rows, k, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(-128, 128, (rows, k // 2), generator=g, dtype=torch.int8).cuda()


# ------------------------------------------------------------------ quantizer

# bf16 rows of whole 256-column tiles with G = 64/256 take the two-threads-per-tile
# kernel (rounds of up to 192 tiles: 16 rows at K = 3072, 4 at 12288, 3 at 15360);
# every other shape, dtype or G takes the half-warp-per-tile kernel.
QUANT_SHAPES = [(1, 768, 256), (7, 3072, 256), (127, 512, 256), (128, 3840, 256), (129, 256, 256),
                (33, 320, 64), (40, 576, 64), (17, 160, 16), (9, 48, 16), (3, 12288, 256), (2, 15360, 256),
                (40, 768, 64), (300, 3072, 64), (5, 256, 64)]


@pytest.mark.parametrize("m,k,g", QUANT_SHAPES)
@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_fused_quant_bit_exact_vs_oracle(ck, m, k, g, dtype):
    x = activation(m, k, dtype, seed=m + k + g)
    q, s = ck.convrot_quant_int4(x, g)
    torch.cuda.synchronize()
    qo, so = orc.convrot_quant_int4(to_storage(x), g, dtype)
    assert np.array_equal(to_storage(s).view(np.uint32), so.view(np.uint32))
    assert np.array_equal(to_storage(q), qo)


def test_fused_quant_large_m(ck):
    x = activation(4608, 3072, "bf16", seed=3)
    q, s = ck.convrot_quant_int4(x, 256)
    torch.cuda.synchronize()
    sl = slice(4000, 4608)
    qo, so = orc.convrot_quant_int4(to_storage(x[sl]), 256, "bf16")
    assert np.array_equal(to_storage(q[sl]), qo)
    assert np.array_equal(to_storage(s[sl]).view(np.uint32), so.view(np.uint32))


@pytest.mark.parametrize("m,k", [(1000, 12288), (2000, 3072), (149, 15360)])
def test_fused_quant_bf16_many_rounds_all_rows(ck, m, k):
    """Several rounds per block, a partial last round, every row checked."""
    x = activation(m, k, "bf16", seed=m)
    q, s = ck.convrot_quant_int4(x, 256)
    torch.cuda.synchronize()
    qo, so = orc.convrot_quant_int4(to_storage(x), 256, "bf16")
    assert np.array_equal(to_storage(s).view(np.uint32), so.view(np.uint32))
    assert np.array_equal(to_storage(q), qo)


@pytest.mark.parametrize("g", [64, 256])
def test_fused_quant_zero_tiny_and_huge_rows(ck, g):
    """All-zero rows (scale floor), subnormal-range rows and large (finite) values."""
    x = activation(24, 3072, "bf16", seed=g).float()
    x[3] = 0.0
    x[7] = 1e-30
    x[8, ::7] = -3e-39
    x[11] *= 1e30
    x[12, 5] = 1e35
    x = x.to(torch.bfloat16)
    q, s = ck.convrot_quant_int4(x, g)
    torch.cuda.synchronize()
    qo, so = orc.convrot_quant_int4(to_storage(x), g, "bf16")
    assert np.array_equal(to_storage(s).view(np.uint32), so.view(np.uint32))
    assert np.array_equal(to_storage(q), qo)


@pytest.mark.parametrize("case", ["g256_bf16", "g64_bf16", "g16_bf16", "g256_f16", "g256_f32", "cfg0_bf16"])
def test_rowwise_quant_bit_exact_vs_reference(ck, case):
    """Given the reference's rotated tensor, codes and scales equal eager's."""
    gold = np.load(os.path.join(GOLD, "quant.npz"))
    dtype = {0: "bf16", 1: "f16", 2: "f32"}[int(gold[f"{case}_meta"][2])]
    xr = from_storage(gold[f"{case}_xrot"], dtype).cuda()
    q, s = ck.int4_quant_rowwise(xr)
    torch.cuda.synchronize()
    assert np.array_equal(to_storage(q), gold[f"{case}_q"])
    assert np.array_equal(to_storage(s).view(np.uint32), gold[f"{case}_scale"].view(np.uint32))


@pytest.mark.parametrize("case", ["g256_bf16", "g64_bf16", "g16_bf16", "g256_f16", "cfg0_bf16"])
def test_fused_quant_vs_reference_eager(ck, case):
    """End to end: only rotation rounding ties may move a code, by one step."""
    gold = np.load(os.path.join(GOLD, "quant.npz"))
    grp, _, dti = (int(v) for v in gold[f"{case}_meta"])
    dtype = {0: "bf16", 1: "f16", 2: "f32"}[dti]
    x = from_storage(gold[f"{case}_x"], dtype).cuda()
    q, _ = ck.convrot_quant_int4(x, grp)
    torch.cuda.synchronize()
    a = orc.unpack_int4(to_storage(q)).astype(np.int32)
    b = orc.unpack_int4(gold[f"{case}_q"]).astype(np.int32)
    assert np.abs(a - b).max() <= 1
    assert np.count_nonzero(a != b) <= max(1, a.size // 100000)


# ------------------------------------------------------------------ GEMM

# Covers every kernel variant: the CUDA-core few-token path for M <= 4 (rows in
# one K slice, in several slices, a shorter last slice, one row per block, and
# K = 65536 where M = 3..4 falls back to the tensor path), swapped tiles (weights
# in TMEM) for M <= 32/64/128, CTA pairs above; partial k-stages (K/2 not a
# multiple of 64), tails in M and N, a pair whose second CTA lies wholly outside
# the matrix.
GEMM_SHAPES = [(1, 64, 64), (7, 100, 96), (128, 256, 3072), (129, 384, 512), (257, 3072, 3072),
               (64, 192, 32), (300, 1000, 1024), (512, 3072, 3072), (16, 128, 12288),
               (33, 520, 160), (100, 300, 224), (65, 18432, 3072), (1, 18432, 3072), (4608, 256, 64),
               (2, 1000, 3072), (3, 520, 160), (4, 2052, 12288), (1, 96, 32768),
               (1, 3072, 12288), (3, 200, 7680), (2, 150, 65536), (4, 37, 3840)]


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
def test_gemm_int32_accumulators_exact(ck, m, n, k):
    xp = random_packed(m, k, seed=m * 7 + k)
    wp = random_packed(n, k, seed=n * 11 + k)
    acc = ck.int4_gemm_s32(xp, wp)
    torch.cuda.synchronize()
    xi = orc.unpack_int4(to_storage(xp)).astype(np.int64)
    wi = orc.unpack_int4(to_storage(wp)).astype(np.int64)
    assert np.array_equal(to_storage(acc).astype(np.int64), xi @ wi.T)


# (2048, 3072): more output tiles than CTA pairs on the GPU (persistent tile loop);
# (515, 2056): staged bf16 stores with tails in M and in the last 64-column box.
@pytest.mark.parametrize("m,n,k", [(1, 64, 64), (77, 300, 1024), (256, 512, 3072), (200, 3072, 12288),
                                   (2048, 3072, 256), (515, 2056, 320), (3, 777, 3072), (4, 18432, 3072),
                                   (1, 3072, 12288), (2, 300, 7680)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("with_bias", [True, False])
def test_gemm_epilogue_bit_exact(ck, m, n, k, out_dtype, with_bias):
    xp = random_packed(m, k, seed=1 + m)
    wp = random_packed(n, k, seed=2 + n)
    g = torch.Generator().manual_seed(m + n)
    xs = (torch.rand(m, generator=g) * 0.1 + 1e-3).cuda()
    ws = (torch.rand(n, generator=g) * 0.01 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).cuda() if with_bias else None
    out = ck.int4_convrot_gemm(xp, wp, xs, ws, bias, out_dtype)
    torch.cuda.synchronize()
    ref = orc.int4_convrot_gemm(to_storage(xp), to_storage(wp), to_storage(xs), to_storage(ws),
                                None if bias is None else to_storage(bias),
                                "bf16" if out_dtype == torch.bfloat16 else "f32")
    got = to_storage(out)
    if out_dtype == torch.float32:
        got, ref = got.view(np.uint32), ref.view(np.uint32)
    assert np.array_equal(got, ref)


def test_gemm_guard_bands_untouched(ck):
    """Writes stay inside [M, N]: canaries around the output survive (tails in M and N)."""
    m, n, k = 131, 200, 512
    xp = random_packed(m, k, 5)
    wp = random_packed(n, k, 6)
    xs = torch.ones(m, device="cuda")
    ws = torch.ones(n, device="cuda")
    pad = 4096
    buf = torch.full((pad + m * n + pad,), 12345.0, device="cuda")
    view = buf[pad:pad + m * n]
    rc = ck.library().ck_int4_convrot_gemm(xp.data_ptr(), wp.data_ptr(), xs.data_ptr(), ws.data_ptr(), 0,
                                           view.data_ptr(), m, n, k, 0,
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.all(buf[:pad] == 12345.0) and torch.all(buf[pad + m * n:] == 12345.0)
    exact = orc.int4_gemm_acc(to_storage(xp), to_storage(wp)).astype(np.float32)
    assert np.array_equal(to_storage(view).reshape(m, n), exact)


def test_splitk_accumulates_deterministically(ck):
    m, n, k = 96, 384, 2048
    xp = random_packed(m, k, 8)
    wp = random_packed(n, k, 9)
    xs = torch.rand(m, device="cuda") * 0.01
    ws = torch.rand(n, device="cuda") * 0.01
    base = torch.randn(m, n, device="cuda")
    acc = base.clone()
    ck.int4_convrot_gemm_splitk(xp, wp, xs, ws, acc, nsplit=4)
    acc2 = base.clone()
    ck.int4_convrot_gemm_splitk(xp, wp, xs, ws, acc2, nsplit=2)
    torch.cuda.synchronize()
    assert torch.equal(acc, acc2)
    d = orc.int4_gemm_acc(to_storage(xp), to_storage(wp))
    ref = to_storage(base) + orc.int4_gemm_epilogue(d, to_storage(xs), to_storage(ws), None, "f32")
    assert np.array_equal(to_storage(acc).view(np.uint32), ref.astype(np.float32).view(np.uint32))


def test_gemm_full_size_checksums(ck):
    """Config-1 MLP-up shape: row and column checksums of D equal exact integer identities."""
    m, n, k = 4608, 12288, 3072
    xp = random_packed(m, k, 21)
    wp = random_packed(n, k, 22)
    acc = ck.int4_gemm_s32(xp, wp).to(torch.int64)
    xi = torch.from_numpy(orc.unpack_int4(to_storage(xp)).astype(np.int64))
    wi = torch.from_numpy(orc.unpack_int4(to_storage(wp)).astype(np.int64))
    rows = acc.sum(dim=1).cpu()
    cols = acc.sum(dim=0).cpu()
    assert torch.equal(rows, xi @ wi.sum(dim=0))
    assert torch.equal(cols, wi @ xi.sum(dim=0))
    g = torch.Generator().manual_seed(0)
    ri = torch.randint(0, m, (64,), generator=g)
    acc_cpu = acc[ri].cpu()
    assert torch.equal(acc_cpu, xi[ri] @ wi.T)


# ------------------------------------------------------------------ full linear

@pytest.mark.parametrize("case", ["g256", "g64", "g16", "cfg0"])
def test_linear_vs_reference_and_oracle(ck, case):
    import _int4
    lin = np.load(os.path.join(GOLD, "linear.npz"))
    grp = int(lin[f"{case}_meta"][0])
    x = from_storage(lin[f"{case}_x"], "bf16").cuda()
    qw = torch.from_numpy(lin[f"{case}_qw"]).cuda()
    ws = torch.from_numpy(lin[f"{case}_ws"]).cuda()
    bias = from_storage(lin[f"{case}_bias"], "bf16").cuda().to(torch.float16)
    out = _int4.convrot_w4a4_linear(x, qw, ws, bias=bias, convrot_groupsize=grp)
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16 and out.shape == (x.shape[0], qw.shape[0])
    got = to_storage(out)
    ora = orc.convrot_w4a4_linear(lin[f"{case}_x"], lin[f"{case}_qw"], lin[f"{case}_ws"],
                                  to_storage(bias.float()), grp)
    assert np.array_equal(got, ora)
    ref = orc.bf16_bits_to_f32(lin[f"{case}_out"])
    g32 = orc.bf16_bits_to_f32(got)
    assert np.linalg.norm(g32 - ref) / np.linalg.norm(ref) < 1e-2


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_linear_other_activation_dtypes(ck, dtype):
    import _int4
    m, k, n = 37, 512, 256
    x = activation(m, k, "bf16", 4).to(dtype)
    w = (torch.randn(n, k) * 0.02).to(torch.float16).cuda()
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, 256)
    out = _int4.convrot_w4a4_linear(x, qw, ws, bias=None)
    torch.cuda.synchronize()
    assert out.dtype == dtype
    key = "f16" if dtype == torch.float16 else "f32"
    ref = orc.convrot_w4a4_linear(to_storage(x), to_storage(qw), to_storage(ws), None, 256, key)
    assert np.array_equal(to_storage(out).view(np.uint8), np.asarray(ref).view(np.uint8))


def test_linear_keeps_leading_dims_and_status_clear(ck):
    import _int4
    x = activation(2 * 3 * 5, 768, "bf16", 9).reshape(2, 3, 5, 768)
    w = (torch.randn(96, 768) * 0.02).to(torch.float16).cuda()
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, 256)
    out = _int4.convrot_w4a4_linear(x, qw, ws)
    assert out.shape == (2, 3, 5, 96)
    assert ck.device_status() == 0


# ------------------------------------------------------------------ fused linear entry

# ck_convrot_w4a4_linear = ck_convrot_quant_int4 then ck_int4_convrot_gemm, with
# the bias read in its own dtype: bit-identical to the two exports with an
# fp32-converted bias, for the few-token path (M <= 4) and both tensor paths.
@pytest.mark.parametrize("m,k,n", [(1, 3072, 3072), (3, 768, 520), (64, 1024, 384), (700, 3072, 1280)])
@pytest.mark.parametrize("bias_dtype", [None, torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_fused_linear_entry_matches_two_calls(ck, m, k, n, bias_dtype, out_dtype):
    g = torch.Generator().manual_seed(m + n)
    x = (torch.randn(m, k, generator=g) * 2).to(torch.bfloat16).cuda()
    wq = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int8).cuda()
    ws = (torch.rand(n, generator=g) * 0.01 + 1e-4).cuda()
    bias = None if bias_dtype is None else (torch.randn(n, generator=g) * 0.1).to(bias_dtype).cuda()
    fused = ck.convrot_w4a4_linear(x, wq, ws, bias, out_dtype, 256)
    q, xs = ck.convrot_quant_int4(x, 256)
    two = ck.int4_convrot_gemm(q, wq, xs, ws, bias, out_dtype)
    torch.cuda.synchronize()
    assert torch.equal(fused, two)
    assert ck.device_status() == 0


def test_fused_linear_entry_back_to_back_in_a_graph(ck):
    """Programmatic dependent launches chained through layers, captured in a
    CUDA graph: each layer consumes the previous layer's output."""
    import _int4
    dims = [3072, 1536, 3072, 768]
    g = torch.Generator().manual_seed(5)
    layers = []
    for a, b in zip(dims[:-1], dims[1:]):
        w = (torch.randn(b, a, generator=g) * 0.02).to(torch.bfloat16).cuda()
        qw, wsc = _int4.quantize_convrot_w4a4_weight(w, 256)
        layers.append((qw, wsc, (torch.randn(b, generator=g) * 0.1).to(torch.bfloat16).cuda()))
    x0 = torch.randn(300, dims[0], generator=g).to(torch.bfloat16).cuda()

    def run(x):
        for qw, wsc, b in layers:
            x = _int4.convrot_w4a4_linear(x, qw, wsc, b)
        return x
    eager = run(x0)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = run(x0)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    # the same chain through the oracle
    ref = to_storage(x0)
    for qw, wsc, b in layers:
        ref = orc.convrot_w4a4_linear(ref, to_storage(qw), to_storage(wsc), to_storage(b.float()), 256)
    assert np.array_equal(to_storage(eager), ref)
