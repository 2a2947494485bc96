"""The dense STE training layer (pentanet_layer.PentaLinear) on the CPU: its
quantisation equals the oracle's for both rules (pentanet, and the ternary
bitnet rule of train_pentagpt.py:33-36), the straight-through gradient
reaches the master weights unchanged, and fast-inference conversion refuses
CPU weights as the reference does (pentanet_layer.py:63-64)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from _util import gen_act
from oracle import oracle as orc
import pentanet_layer as pl


@pytest.mark.parametrize("mode,qmax", [("pentanet", 2), ("bitnet", 1)])
def test_ste_layer_matches_oracle(mode, qmax):
    torch.manual_seed(7)
    layer = pl.PentaLinear(250, 96, bias=True, mode=mode)
    with torch.no_grad():
        layer.bias.copy_(torch.randn(96) * 0.1)
    x = gen_act(5, 250, seed=3).float().requires_grad_(True)
    y = layer(x)
    scale = float(layer.weight.detach().abs().mean().clamp(min=1e-8))
    packed, _, _ = orc.quantize_pack(layer.weight.detach().numpy(), scale, mode=mode)
    q = orc.unpack(packed, 250).astype(np.float32)
    assert np.abs(q).max() <= qmax
    want = F.linear(x.detach(), torch.from_numpy(q) * scale, layer.bias.detach())
    assert torch.allclose(y.detach(), want, rtol=1e-5, atol=1e-5)
    # straight-through: d y / d W is the dense linear's, as if W were used directly
    g = torch.randn_like(y)
    y.backward(g)
    assert torch.allclose(layer.weight.grad, g.t() @ x.detach(), rtol=1e-5, atol=1e-5)
    assert torch.allclose(x.grad, g @ (torch.from_numpy(q) * scale), rtol=1e-5, atol=1e-5)


def test_fast_conversion_needs_cuda():
    with pytest.raises(AssertionError):
        pl.PentaLinear(40, 8).to_fast_inference()
    with pytest.raises(AssertionError):
        pl.PentaLinear(40, 8, mode="ternary")
