"""PentaGPT inference model (pentagpt.py): the packed model's logits against
the same network computed densely with torch (dequantised weights, bf16
activations), on a small configuration."""
import math

import pytest
import torch
import torch.nn.functional as F

import penta_kernel as pk
from pentagpt import PentaGPTConfig, PentaGPTFast

pytestmark = pytest.mark.gpu


def _dense(lin):
    w = pk.unpack_weights(lin.packed_w, lin.K_orig).float() * lin.scale
    return w.to(torch.bfloat16)


def _dense_forward(model, idx):
    cfg = model.cfg
    B, T = idx.shape
    x = (model.wte(idx) + model.wpe(torch.arange(T, device=idx.device))).to(torch.bfloat16)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        for blk in model.h:
            C = cfg.n_embd
            q, k, v = F.linear(blk.ln_1(x).to(torch.bfloat16), _dense(blk.c_attn)).split(C, dim=2)
            sh = lambda t: t.view(B, T, cfg.n_head, C // cfg.n_head).transpose(1, 2)
            att = (sh(q).float() @ sh(k).float().transpose(-2, -1)) / math.sqrt(C // cfg.n_head)
            att = att.masked_fill(torch.ones(T, T, device=idx.device).tril() == 0, float("-inf")).softmax(-1)
            y = (att @ sh(v).float()).to(torch.bfloat16).transpose(1, 2).contiguous().view(B, T, C)
            x = x + F.linear(y, _dense(blk.attn_proj))
            h = F.linear(F.gelu(F.linear(blk.ln_2(x).to(torch.bfloat16), _dense(blk.c_fc))), _dense(blk.mlp_proj))
            x = x + h
        x = model.ln_f(x)
    return F.linear(x.to(torch.bfloat16), _dense(model.lm_head)).float()


def test_small_pentagpt_matches_dense(cuda_device):
    cfg = PentaGPTConfig(n_layer=2, n_head=4, n_embd=128, block_size=64, vocab_size=1000)
    model = PentaGPTFast.random(cfg, seed=42, device=cuda_device)
    idx = torch.randint(0, cfg.vocab_size, (3, 40), generator=torch.Generator().manual_seed(1)).to(cuda_device)
    got = model(idx, all_logits=True).float()
    want = _dense_forward(model, idx)
    assert got.shape == (3, 40, cfg.vocab_size)
    # bf16 activations through the whole network: agreement to bf16 precision
    err = (got - want).abs().max().item()
    assert err <= 2e-2 * want.abs().max().item() + 1e-3, err
    last = model(idx).float()
    assert last.shape == (3, 1, cfg.vocab_size)
    assert torch.allclose(last[:, 0], got[:, -1], rtol=0, atol=0)


def test_pentagpt_124m_shapes(cuda_device):
    model = PentaGPTFast.random(seed=42, device=cuda_device)
    # 12 x (2304 + 768 + 3072) x 768 + 768 x 3072 x 12 packed projection weights, plus the tied lm_head
    assert model.n_packed_params() == 12 * (768 * 2304 + 768 * 768 + 2 * 768 * 3072) + 50257 * 768
    idx = torch.randint(0, 50257, (2, 128), generator=torch.Generator().manual_seed(2)).to(cuda_device)
    out = model(idx)
    assert out.shape == (2, 1, 50257) and torch.isfinite(out.float()).all()
