"""The oracle's LayerNorm + modulation restatement against torch, on the CPU.

``oracle.layernorm_modulate`` defines the fused kernel's arithmetic (a fixed
fp32 order for the row statistics). The model code it stands for (a Flux
block's ``(1 + scale) * norm(x) + shift`` before QKV / MLP-up) is ComfyUI's and
not part of the reference, so the restatement is pinned here to torch's own
``layer_norm`` (fp32 statistics) followed by the modulation in bf16: the
statistics may differ in their last bits, which moves a bf16 result by at
most one unit, on a small fraction of elements; the elementwise modulation is
the same sequence of bf16 roundings.
"""
import numpy as np
import torch

from oracle import convrot_oracle as orc


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def torch_lnmod(x, scale, shift, eps):
    xn = torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), eps=eps).to(torch.bfloat16)
    return (1 + scale) * xn + shift


def test_lnmod_oracle_matches_torch_within_one_unit():
    g = torch.Generator().manual_seed(0)
    for m, k in ((64, 3072), (17, 3840), (8, 256)):
        x = (torch.randn(m, k, generator=g) * 3 + 0.5).to(torch.bfloat16)
        x[:, :: 97] *= 20
        scale = (torch.randn(k, generator=g) * 0.3).to(torch.bfloat16)
        shift = (torch.randn(k, generator=g) * 0.3).to(torch.bfloat16)
        got = orc.bf16_bits_to_f32(orc.layernorm_modulate(bits(x), bits(scale), bits(shift), 1e-6))
        want = torch_lnmod(x, scale, shift, 1e-6).float().numpy()
        ulp = np.abs(want) * 2.0 ** -7 + 2.0 ** -126
        diff = np.abs(got - want)
        assert np.all(diff <= 2 * ulp)
        assert np.count_nonzero(diff) <= 0.02 * diff.size


def test_lnmod_oracle_plain_layernorm_and_constant_rows():
    x = torch.zeros(3, 512, dtype=torch.bfloat16)
    x[1] = 2.5                                             # constant row: var 0, xn 0
    x[2, ::2] = 1.0
    x[2, 1::2] = -1.0                                      # mean 0, var 1
    y = orc.bf16_bits_to_f32(orc.layernorm_modulate(bits(x), None, None, 1e-6))
    assert np.all(y[0] == 0) and np.all(y[1] == 0)
    assert np.allclose(y[2], np.where(np.arange(512) % 2 == 0, 1.0, -1.0), atol=2 ** -7)
