"""The no-allocation linear entry, ck_convrot_w4a4_linear_noalloc.

Callers that cannot allocate device memory (a host framework that owns every
device buffer through its own arena, a plugin ABI with plain pointers and no
allocator) use this entry; it keeps its quantized activations in a static
128 MiB array per device instead of a caller workspace. It must give exactly
what ck_convrot_w4a4_linear gives with a caller workspace, on consecutive calls
that reuse the static scratch (also near its end, and on a second device), and
refuse sizes beyond the scratch before touching CUDA. This file is collected
last so it also runs after every other GPU test in one process (and passes
alone in a fresh one).
"""
import os

import pytest
import torch

from _int4 import build as libbuild
from _int4 import cuda_loader

SCRATCH = 128 << 20


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(libbuild.lib_path()):
        libbuild.build()
    return cuda_loader.library()


def packed_scratch_bytes(m, k):
    """What the entry keeps in its scratch: packed codes and row scales, 256-byte aligned."""
    up = lambda v: (v + 255) // 256 * 256
    return up(m * k // 2) + up(4 * m)


def test_noalloc_rejects_sizes_beyond_the_scratch(lib):
    """Checked on the host before any CUDA call (runs without a GPU)."""
    f = lib.ck_convrot_w4a4_linear_noalloc
    m, k = 32768, 8192                     # 128 MiB of codes + scales: over the limit
    assert packed_scratch_bytes(m, k) > SCRATCH
    assert f(256, 1, 256, 256, 0, 0, 256, 1, m, 64, k, 256, None) == -1
    assert b"128 MiB" in lib.ck_convrot_last_error()
    assert packed_scratch_bytes(18432, 12288) <= SCRATCH
    assert f(256, 1, 256, 256, 0, 0, 256, 1, 0, 64, k, 256, None) == 0      # empty: no launch
    assert f(256, 1, 256, 256, 0, 7, 256, 1, 4, 64, 256, 256, None) == -1   # bad bias dtype


def _case(m, k, n, seed, bias_dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(m, k, generator=g) * 3).to(torch.bfloat16).cuda()
    wq = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int8).cuda()
    ws = (torch.rand(n, generator=g) * 0.01 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.1).to(bias_dtype).cuda()
    return x, wq, ws, bias


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,n", [(1, 3072, 3072), (4, 768, 520), (300, 3072, 1280), (4608, 3072, 3072)])
def test_noalloc_matches_workspace_entry_on_consecutive_calls(lib, m, k, n):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    a = _case(m, k, n, seed=m)
    b = _case(m, k, n, seed=m + 1, bias_dtype=torch.float32)
    # two calls in a row on one stream: the second overwrites the scratch the first used
    na = cuda_loader.convrot_w4a4_linear_noalloc(*a, torch.bfloat16, 256)
    nb = cuda_loader.convrot_w4a4_linear_noalloc(*b, torch.float32, 256)
    wa = cuda_loader.convrot_w4a4_linear(*a, torch.bfloat16, 256)
    wb = cuda_loader.convrot_w4a4_linear(*b, torch.float32, 256)
    torch.cuda.synchronize()
    assert torch.equal(na, wa)
    assert torch.equal(nb, wb)
    assert not torch.equal(na.float(), nb)
    assert cuda_loader.device_status() == 0


@pytest.mark.gpu
def test_noalloc_near_the_scratch_limit(lib):
    """M = 18432, K = 12288: codes and row scales fill ~108 of the 128 MiB, so the
    scale block sits near the end of the array; two calls in a row."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    m, k, n = 18432, 12288, 256
    assert packed_scratch_bytes(m, k) > (100 << 20)
    for seed in (11, 12):
        x, wq, ws, bias = _case(m, k, n, seed=seed)
        na = cuda_loader.convrot_w4a4_linear_noalloc(x, wq, ws, bias, torch.bfloat16, 256)
        wa = cuda_loader.convrot_w4a4_linear(x, wq, ws, bias, torch.bfloat16, 256)
        torch.cuda.synchronize()
        assert torch.equal(na, wa)
    assert cuda_loader.device_status() == 0


@pytest.mark.gpu
def test_noalloc_on_a_second_device(lib):
    """Each device has its own copy of the scratch: a call with device 1 current
    uses device 1's array (no peer access involved)."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    with torch.cuda.device(1):
        a = [t.to("cuda:1") for t in _case(300, 3072, 1280, seed=21)]
        for _ in range(2):
            na = cuda_loader.convrot_w4a4_linear_noalloc(*a, torch.bfloat16, 256)
            wa = cuda_loader.convrot_w4a4_linear(*a, torch.bfloat16, 256)
            torch.cuda.synchronize()
            assert na.device == torch.device("cuda", 1)
            assert torch.equal(na, wa)
