"""The bounded-wait failure path on the GPU, without faulting or hanging it: a
wait that nothing ends gives up after its limit, records its status code, and
the context stays usable for the next launch."""
import time

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


def test_wait_that_nothing_ends_reports_timeout(ck):
    assert ck.device_status() == 0                      # read and clear
    t0 = time.perf_counter()
    ck.selftest_wait_timeout(1_000_000)                 # 1 ms
    assert ck.device_status() == 5                      # kStatusTimeoutSelfTest
    assert time.perf_counter() - t0 < 5.0
    assert ck.device_status() == 0                      # cleared by the read
    # the context still runs the real kernels, bit-exactly
    g = torch.Generator().manual_seed(1)
    xp = torch.randint(-128, 128, (300, 512), generator=g, dtype=torch.int8).cuda()
    wp = torch.randint(-128, 128, (640, 512), generator=g, dtype=torch.int8).cuda()
    a = ck.int4_gemm_s32(xp, wp)
    b = ck.int8_gemm_s32(ck.int4_unpack(xp), ck.int4_unpack(wp))
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert ck.device_status() == 0
