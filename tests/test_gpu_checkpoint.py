"""GPU forward of layers loaded from the reference-written prequantized
checkpoints (tests/golden/ckpt_*.safetensors): bit-exact against the oracle on
the file's own bytes, for the int4 (G = 256 and 64) and int8 layers, on both
the packed (M <= 128) and unpacked (M > 128) int4 paths."""
import numpy as np
import pytest
import torch

from oracle import convrot_oracle as orc
from test_checkpoint import LAYERS, load_fixture

pytestmark = pytest.mark.gpu


def bits(t):
    t = t.detach().cpu().contiguous()
    return t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()


@pytest.fixture(scope="module")
def model():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    m, _ = load_fixture("native", device="cuda")
    return m


@pytest.mark.parametrize("m", [1, 77, 300])
@pytest.mark.parametrize("name", [l[0] for l in LAYERS])
def test_loaded_layer_forward_bit_exact(model, name, m):
    layer = model.get_submodule(name)
    g = torch.Generator().manual_seed(m)
    x = torch.randn(m, layer.in_features, generator=g).to(torch.bfloat16).cuda()
    y = layer(x)
    torch.cuda.synchronize()
    q, ws = layer._q.cpu().numpy(), layer._qs.cpu().numpy()
    bias = None if layer.bias is None else layer.bias.float().cpu().numpy()
    if layer._qmode == "int8":
        ref = orc.convrot_w8a8_linear(bits(x), q, ws, bias, layer._qgs)
    else:
        ref = orc.convrot_w4a4_linear(bits(x), q, ws, bias, layer._qgs)
    assert y.dtype == torch.bfloat16 and np.array_equal(bits(y), ref)
