"""GPU tests of the Dynamic-LoRA down projection T = fp16(x) . A^T (ck_lora_down).

The node prepares adapters in fp16 (int4_ops.py:165-167) and the side path's
down projection is an fp16 product with fp32 accumulation. The reference value
here is the exact product of the fp16-rounded operands (float64 on the CPU),
rounded once to fp16. Tolerance, written out in ``check_t``: one fp16 unit of
the result (and the fp16 subnormal step), plus the fp32 accumulation bound
K * 2^-24 * sum |x_k a_k| for the tensor cores' summation order.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ck():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import _int4
    from _int4 import cuda_loader
    assert _int4.is_available()
    return cuda_loader


def exact_t(x16: torch.Tensor, a16: torch.Tensor):
    xf = x16.cpu().double().numpy()
    af = a16.cpu().double().numpy()
    return xf @ af.T, np.abs(xf) @ np.abs(af).T


def check_t(got: torch.Tensor, x16: torch.Tensor, a16: torch.Tensor):
    t, mag = exact_t(x16, a16)
    g = got.cpu().double().numpy()
    k = x16.shape[1]
    tol = np.abs(t) * 2.0 ** -10 + 2.0 ** -24 + mag * (k * 2.0 ** -24)
    bad = np.abs(g - t) > tol
    assert not bad.any(), f"{np.count_nonzero(bad)} of {g.size} values outside the tolerance"


def synth(m, k, r, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    x[:, torch.randperm(k, generator=g)[: max(1, k // 100)]] *= 20
    a = (torch.randn(r, k, generator=g) * 0.01).to(torch.float16)
    return x.to(dtype).cuda(), a.cuda()


# (M, K, R): one row; a K that ends inside a stage (OOB columns); one K stage;
# few M tiles (K split over a cluster); ragged M; config-4 sizes
SHAPES = [(1, 3072, 64), (130, 264, 16), (1024, 64, 8), (100, 256, 8), (4608, 3072, 64), (513, 15360, 24),
          (4000, 12288, 64)]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("m,k,r", SHAPES)
def test_lora_down_vs_exact(ck, m, k, r, dtype):
    x, a = synth(m, k, r, dtype, seed=m + k + r)
    t = ck.lora_down(x, a)
    torch.cuda.synchronize()
    assert t.dtype == torch.float16 and tuple(t.shape) == (m, r)
    rows = np.arange(m) if m <= 600 else np.unique(np.r_[np.random.default_rng(m).choice(m, 96), 0, m - 1])
    check_t(t[rows], x.to(torch.float16)[rows], a)


@pytest.mark.parametrize("m,k,r", [(18432, 12288, 64), (18432, 3072, 64)])
def test_lora_down_config4_sampled_rows(ck, m, k, r):
    x, a = synth(m, k, r, torch.bfloat16, seed=3)
    t = ck.lora_down(x, a)
    torch.cuda.synchronize()
    rows = np.unique(np.r_[np.random.default_rng(5).choice(m, 64), 0, m - 1])
    check_t(t[rows], x.to(torch.float16)[rows], a)


def test_lora_down_repeats_bit_for_bit(ck):
    """Fixed summation order (split-K partials summed in cluster-rank order)."""
    x, a = synth(4608, 3072, 64, torch.bfloat16, seed=11)
    t1 = ck.lora_down(x, a)
    t2 = ck.lora_down(x, a)
    torch.cuda.synchronize()
    assert torch.equal(t1.view(torch.int16), t2.view(torch.int16))


def test_lora_down_matches_fp16_matmul(ck):
    """Against the cast-then-matmul it replaces (fp32 accumulation both)."""
    x, a = synth(2048, 3072, 64, torch.bfloat16, seed=13)
    t = ck.lora_down(x, a)
    ref = x.to(torch.float16) @ a.t()
    torch.cuda.synchronize()
    d = (t.float() - ref.float()).abs()
    assert float(d.max()) <= float((ref.float().abs() * 2.0 ** -9 + 1e-3).max())


def test_lora_down_bf16_beyond_fp16_range(ck):
    """bf16 values beyond the fp16 range become +-inf in the conversion, as in a cast."""
    x, a = synth(128, 256, 8, torch.bfloat16, seed=17)
    x[5, 7] = 1.0e6
    x[9, 100] = -3.0e5
    t = ck.lora_down(x, a)
    ref = x.to(torch.float16).double() @ a.double().t()
    torch.cuda.synchronize()
    got = t.cpu().double()
    ref = ref.cpu()
    assert torch.equal(torch.isinf(got), torch.isinf(ref))
    assert torch.equal(torch.sign(got[torch.isinf(got)]), torch.sign(ref[torch.isinf(ref)]))


def test_lora_down_rejects_bad_shapes(ck):
    x = torch.zeros(16, 260, dtype=torch.bfloat16, device="cuda")
    a = torch.zeros(8, 260, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError):
        ck.lora_down(x, a)                       # K % 8 != 0
    x = torch.zeros(16, 256, dtype=torch.bfloat16, device="cuda")
    a = torch.zeros(12, 256, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError):
        ck.lora_down(x, a)                       # rank not a multiple of 8
