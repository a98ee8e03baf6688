"""Host logic of the unpacked-weight cache (no GPU: a counting fake unpacker)."""
import gc

import pytest
import torch

from _int4 import weight_cache


@pytest.fixture(autouse=True)
def restore_cache_state():
    """The cache is opt-in: every test here leaves it as it found it."""
    was = weight_cache.enabled()
    yield
    weight_cache.enable(was)


class CountingUnpack:
    def __init__(self):
        self.calls = 0

    def __call__(self, packed):
        self.calls += 1
        return torch.zeros(packed.shape[0], 2 * packed.shape[1], dtype=torch.int8)


def test_unpacked_once_per_tensor_and_refreshed_on_write():
    weight_cache.enable(True)
    f = CountingUnpack()
    w = torch.zeros(8, 16, dtype=torch.int8)
    a = weight_cache.unpacked(w, f)
    b = weight_cache.unpacked(w, f)
    assert a is b and f.calls == 1
    w.add_(1)                                  # in-place write: version counter moves
    c = weight_cache.unpacked(w, f)
    assert c is not a and f.calls == 2
    other = torch.zeros(8, 16, dtype=torch.int8)
    weight_cache.unpacked(other, f)
    assert f.calls == 3


def test_copy_dropped_with_its_tensor():
    weight_cache.enable(True)
    f = CountingUnpack()
    w = torch.zeros(4, 32, dtype=torch.int8)
    weight_cache.unpacked(w, f)
    before = weight_cache.cached_bytes()
    assert before >= 4 * 64
    del w
    gc.collect()
    assert weight_cache.cached_bytes() == before - 4 * 64


def test_disable_frees_everything():
    f = CountingUnpack()
    keep = torch.zeros(2, 16, dtype=torch.int8)
    weight_cache.unpacked(keep, f)
    weight_cache.enable(False)
    assert weight_cache.cached_bytes() == 0 and not weight_cache.enabled()
    weight_cache.enable(True)


def test_unpacked_dispatch_rule(monkeypatch):
    import _int4
    from _int4 import cuda_loader
    monkeypatch.setattr(cuda_loader, "unpacked_path_supported", lambda x, g: True)
    weight_cache.enable(True)

    def use(m, n, k=3072):
        return _int4._use_unpacked(torch.zeros(m, k), torch.zeros(n, k // 2, dtype=torch.int8), 256)
    assert use(129, 18432) and use(4608, 3072)                 # many tokens
    assert use(32, 3072) and use(8, 4096, 12288)               # few rows: a dozen swapped tiles
    assert not use(16, 3072) and not use(7, 3072, 12288)       # too little work per weight byte
    assert not use(64, 12288) and not use(128, 4352)           # enough swapped tiles: packed
    assert not use(4, 3072, 65536) and not use(1, 3072)        # few-token GEMV
    weight_cache.enable(False)
    assert not use(4608, 3072)
    weight_cache.enable(True)
