"""Unpacked-code copies of packed int4 weights, one per live weight tensor.

Opt-in speed over memory: with both operands as one sign-extended int8 per
code the int4 layer runs on the plain int8 tensor-core pipeline (identical
results: the accumulators are the same exact integers), about a fifth faster
than the default A8 form on many-token layers, at the price of a second,
unpacked copy of every weight (twice the packed bytes). Off by default: the
weights then stay packed int4 in HBM. ``enable(True)`` (or
``CONVROT_UNPACKED_WEIGHTS=1``) turns it on. A weight is unpacked once, on
first use, and the copy lives exactly as long as the packed tensor object it
came from (a weak reference drops it); an in-place write to the packed tensor
(its version counter moves) or a new storage refreshes the copy.
"""
from __future__ import annotations

import os
import threading
import weakref

import torch

_enabled = os.environ.get("CONVROT_UNPACKED_WEIGHTS", "0") == "1"
_lock = threading.Lock()
_cache: dict[int, tuple] = {}        # id(packed) -> (weakref, version, data_ptr, shape, codes)


def enable(flag: bool = True) -> None:
    """Turn the unpacked-weight path on or off (off frees the cached copies)."""
    global _enabled
    with _lock:
        _enabled = bool(flag)
        if not _enabled:
            _cache.clear()


def enabled() -> bool:
    return _enabled


def cached_bytes() -> int:
    """Device bytes held by the cached unpacked copies."""
    with _lock:
        return sum(entry[4].numel() * entry[4].element_size() for entry in _cache.values())


def _signature(packed: torch.Tensor):
    return packed._version, packed.data_ptr(), tuple(packed.shape)


def unpacked(packed: torch.Tensor, unpack=None) -> torch.Tensor:
    """The int8 codes [N, K] of `packed` [N, K/2], unpacked on first use and cached.

    `unpack` (packed -> codes) defaults to the device kernel; tests pass their own.
    """
    if unpack is None:
        from .cuda_loader import int4_unpack as unpack
    key = id(packed)
    sig = _signature(packed)
    with _lock:
        entry = _cache.get(key)
        if entry is not None and entry[0]() is packed and entry[1:4] == sig:
            return entry[4]
    codes = unpack(packed)
    with _lock:
        ref = weakref.ref(packed, lambda _r, k=key: _drop(k, _r))
        _cache[key] = (ref, *sig, codes)
    return codes


def _drop(key: int, ref) -> None:
    with _lock:
        entry = _cache.get(key)
        if entry is not None and entry[0] is ref:
            del _cache[key]
