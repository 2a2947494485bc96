"""PentaLinear / PentaLinearFast / convert_to_fast_inference on the GPU,
mirroring scripts/benchmark_kernel.py:47-80 (parity vs the STE layer) with the
oracle's tighter bar added."""
import numpy as np
import pytest
import torch
import torch.nn as nn

from _util import assert_close
from oracle import oracle as orc
import penta_kernel as pk
from pentanet_layer import PentaLinear, PentaLinearFast, convert_to_fast_inference

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("K,N", [(768, 2304), (768, 768), (768, 3072), (3072, 768)])
def test_fast_layer_vs_ste(cuda_device, K, N):
    torch.manual_seed(K + N)
    layer = PentaLinear(K, N, bias=True).to(cuda_device)
    with torch.no_grad():
        layer.bias.normal_()
    x = torch.randn(16, K, device=cuda_device)
    with torch.no_grad():
        y_ref = layer(x)                        # dense STE forward (fp32 weights)
    fast = layer.to_fast_inference()
    y = fast(x)                                 # x cast to bf16 as the reference does
    assert y.dtype == torch.bfloat16 and y.shape == (16, N)
    assert (y.float() - y_ref).abs().max() < 0.2          # the reference's own bar
    # tighter: against the oracle on the same bf16 activations
    w8 = orc.unpack(fast.packed_w.cpu().numpy(), K)
    want = orc.matmul_f64(x.to(torch.bfloat16).float().cpu().numpy(), w8, fast.scale)
    want += layer.bias.detach().to(torch.bfloat16).float().cpu().numpy()[None, :]
    got = pk.penta_linear(x.to(torch.bfloat16), fast.packed_w, fast.scale, K, fast.bias, out_dtype=torch.float32)
    assert_close(got.cpu().numpy(), want, what="fast layer fp32")


class QuantLinear(nn.Module):
    """Stand-in with the attributes of train_pentagpt.QuantLinear (train_pentagpt.py:16-40)."""

    def __init__(self, i, o, bias=False, mode="pentanet"):
        super().__init__()
        self.mode = mode
        self.weight = nn.Parameter(torch.randn(o, i) / i ** 0.5)
        self.bias = None

    def forward(self, x):
        scale = self.weight.abs().mean().clamp(min=1e-8)
        qmax = 2 if self.mode == "pentanet" else 1   # train_pentagpt.py:32-36
        w_q = torch.clamp(torch.round(self.weight / scale), -qmax, qmax)
        return nn.functional.linear(x, (w_q * scale - self.weight).detach() + self.weight)


def test_convert_model_with_quantlinear_and_tied(cuda_device):
    torch.manual_seed(0)
    m = nn.Sequential(PentaLinear(64, 128), nn.GELU(), QuantLinear(128, 64), QuantLinear(64, 64, mode="bitnet"))
    head = QuantLinear(64, 96)
    m.append(head)
    m.append(nn.Identity())
    emb = nn.Embedding(96, 64)
    emb.weight = head.weight                     # tie like train_pentagpt.py:115-116
    m = m.to(cuda_device)
    x = torch.randn(5, 64, device=cuda_device)
    # inference runs under bf16 autocast, as train_pentagpt.py evaluates
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        y_ref = m(x)
    convert_to_fast_inference(m)
    assert isinstance(m[0], PentaLinearFast) and isinstance(m[2], PentaLinearFast)
    assert isinstance(m[3], PentaLinearFast)     # ternary (bitnet) layers pack into the same codes
    assert isinstance(m[4], PentaLinearFast)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(x)
    assert (y.float() - y_ref.float()).abs().max() < 0.25


def test_state_dict_keeps_scale_and_k(cuda_device):
    torch.manual_seed(1)
    fast = PentaLinear(96, 40).to(cuda_device).to_fast_inference()
    sd = fast.state_dict()
    assert "scale_buf" in sd and "k_orig_buf" in sd
    clone = PentaLinearFast(torch.zeros_like(fast.packed_w), 1.0, 1, torch.zeros_like(fast.bias))
    clone.load_state_dict(sd)
    assert clone.scale == fast.scale and clone.K_orig == 96
    x = torch.randn(3, 96, device=cuda_device)
    assert torch.equal(clone(x), fast(x))
    assert "in=96, out=40" in repr(fast)
    # resident weights sit at a 16-byte row stride (K_packs = 10 -> 12 words),
    # also after a device round trip
    assert fast.packed_w.shape == (40, 10) and fast.packed_w.stride(0) == 12
    moved = fast.cpu().to(cuda_device)
    assert moved.packed_w.stride(0) == 12 and torch.equal(moved(x), clone(x))


def test_int8_activation_mode(cuda_device):
    torch.manual_seed(2)
    layer = PentaLinear(512, 256).to(cuda_device)
    fast = PentaLinearFast.from_pentalinear(layer, act_quant="int8")
    x = torch.randn(64, 512, device=cuda_device)
    y = fast(x)
    with torch.no_grad():
        y_ref = layer(x)
    # per-token int8 activations: the quantisation error, not kernel error, dominates
    assert (y.float() - y_ref).abs().max() < 0.5


def test_ternary_pack_and_product(cuda_device):
    """mode='bitnet': the ternary rule of QuantLinear (train_pentagpt.py:33-36)
    in the same 3-bit codes; packed bytes equal the oracle's, every code is in
    {1, 2, 3}, and the bf16 product matches the oracle."""
    w = torch.randn(300, 1001, generator=torch.Generator().manual_seed(7)) * 0.02
    packed, K, gamma = pk.quantize_and_pack(w.to(cuda_device), mode="bitnet")
    want, _, g_want = orc.quantize_pack(w.numpy(), mode="bitnet")
    assert np.array_equal(packed.cpu().numpy(), want)
    w8 = orc.unpack(want, K)
    assert w8.min() == -1 and w8.max() == 1
    penta, _, _ = pk.quantize_and_pack(w.to(cuda_device))
    assert not np.array_equal(packed.cpu().numpy(), penta.cpu().numpy())
    x = torch.randn(5, K, generator=torch.Generator().manual_seed(8)).to(torch.bfloat16)
    y = pk.penta_linear(x.to(cuda_device), packed, gamma, K, out_dtype=torch.float32)
    assert_close(y.cpu().numpy(), orc.matmul_f64(x.float().numpy(), w8, gamma), what="ternary")
