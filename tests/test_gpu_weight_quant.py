"""The load-time weight quantizer on the device, against the reference's own code.

``_int4.eager.quantize_convrot_w4a4_weight`` defines the bytes of every int4
weight (reference: _int4/eager.py:123-135, :92-120). Given CUDA tensors it runs
on the GPU, including the stochastic-rounding variant, whose noise comes from a
CUDA ``torch.Generator`` seeded with the given value (reference:
_int4/eager.py:92-109). On the same device and seed it must give the
reference's bytes exactly: the reference package is imported from
``baseline/_ref`` (installed from the reference checkout by
``__graft_entry__.build()``), skipped where that install is absent.
"""
import importlib.util
import os
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref", "_int4")


@pytest.fixture(scope="module")
def ref():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not os.path.exists(os.path.join(REF, "eager.py")):
        pytest.skip("reference package not installed in baseline/_ref")
    name = "convrot_reference_int4_tests"
    spec = importlib.util.spec_from_file_location(name, os.path.join(REF, "__init__.py"),
                                                  submodule_search_locations=[REF])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("seed", [0, 1234, 987654321])
@pytest.mark.parametrize("n,k,g", [(3072, 3072, 256), (640, 1280, 64), (12288, 3072, 256)])
def test_weight_quant_on_device_matches_reference(ref, n, k, g, seed):
    from _int4 import eager
    w = (torch.randn(n, k, generator=torch.Generator().manual_seed(n + k)) * 0.02).to(torch.float16).cuda()
    q, s = eager.quantize_convrot_w4a4_weight(w.clone(), g, stochastic_rounding=seed)
    qr, sr = ref.quantize_convrot_w4a4_weight(w.clone(), g, stochastic_rounding=seed)
    torch.cuda.synchronize()
    assert q.is_cuda and torch.equal(q, qr)
    assert torch.equal(s.view(torch.int32), sr.to(torch.float32).view(torch.int32))


def test_stochastic_rounding_on_device_is_seeded(ref):
    from _int4 import eager
    w = (torch.randn(1024, 3072, generator=torch.Generator().manual_seed(3)) * 0.02).to(torch.float16).cuda()
    a, _ = eager.quantize_convrot_w4a4_weight(w, 256, stochastic_rounding=77)
    b, _ = eager.quantize_convrot_w4a4_weight(w, 256, stochastic_rounding=77)
    c, _ = eager.quantize_convrot_w4a4_weight(w, 256, stochastic_rounding=78)
    d, _ = eager.quantize_convrot_w4a4_weight(w, 256, stochastic_rounding=0)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and not torch.equal(a, c) and not torch.equal(a, d)
