"""PentaGPT inference model on the packed sm_100a layers.

A GPT-2-style decoder with the architecture of the reference's PentaGPT
(train_pentagpt.py:46-136; GPTConfig size 'large': 12 layers, 12 heads,
d_model 768, MLP 3072, no biases, weight-tied lm_head) in which every
projection -- c_attn, attention c_proj, c_fc, MLP c_proj and the lm_head -- is
a PentaLinearFast (3-bit packed weights, fused dequant-matmul).  For
decode-sized batches the MLP's GELU and both residual adds run in the
epilogues of the projections that produce their inputs (c_fc, attention
c_proj, MLP c_proj), rounded as the separate bf16 ops round them; at prefill
sizes they stay separate torch ops, which are cheaper there (the product's
epilogue runs on the warps of its main loop: for c_fc at 32768 tokens a fused
GELU added ~180 us against ~110 us for F.gelu).  Each LayerNorm is one pass from bf16 to bf16
with fp32 statistics (penta_kernel.layer_norm: what nn.LayerNorm under bf16
autocast plus the cast in front of the projection compute, without the fp32
round trip).  Causal attention is torch's scaled_dot_product_attention, the
memory-efficient equivalent of the reference's masked softmax.

`PentaGPTFast.random(seed)` builds the model from random weights, as used for
throughput measurement; a trained reference model converts with
`pentanet_layer.convert_to_fast_inference`, which packs the same layers.
Forward without targets returns the logits of the last position only, as the
reference does (train_pentagpt.py:129-134).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

try:
    from .pentanet_layer import PentaLinearFast
    from . import penta_kernel as pk
except ImportError:
    from pentanet_layer import PentaLinearFast
    import penta_kernel as pk


@dataclass
class PentaGPTConfig:
    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768
    block_size: int = 1024
    vocab_size: int = 50257


def _packed(w: torch.Tensor, act_quant: str | None) -> PentaLinearFast:
    packed, K, scale = pk.quantize_and_pack(w)
    return PentaLinearFast(packed, scale, K, None, act_quant=act_quant)


# Largest token count whose GELU and residual adds are fused into the products.
FUSE_MAX_TOKENS = 64


class _Block(nn.Module):
    def __init__(self, cfg: PentaGPTConfig, weights: dict, act_quant: str | None):
        super().__init__()
        self.n_head = cfg.n_head
        self.ln_1 = nn.LayerNorm(cfg.n_embd, bias=False)
        self.ln_2 = nn.LayerNorm(cfg.n_embd, bias=False)
        self.c_attn = _packed(weights["c_attn"], act_quant)
        self.attn_proj = _packed(weights["attn_proj"], act_quant)
        self.c_fc = _packed(weights["c_fc"], act_quant)
        self.mlp_proj = _packed(weights["mlp_proj"], act_quant)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, C = x.shape
        h = pk.layer_norm(x, self.ln_1.weight, self.ln_1.bias, self.ln_1.eps)
        q, k, v = self.c_attn(h).split(C, dim=2)
        q = q.view(B, T, self.n_head, C // self.n_head).transpose(1, 2)
        k = k.view(B, T, self.n_head, C // self.n_head).transpose(1, 2)
        v = v.view(B, T, self.n_head, C // self.n_head).transpose(1, 2)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        y = y.transpose(1, 2).contiguous().view(B, T, C)
        if B * T <= FUSE_MAX_TOKENS:
            x = self.attn_proj(y, residual=x)  # x + attn(ln_1(x)), train_pentagpt.py:100
            h = pk.layer_norm(x, self.ln_2.weight, self.ln_2.bias, self.ln_2.eps)
            return self.mlp_proj(self.c_fc(h, act="gelu"), residual=x)  # x + mlp(ln_2(x)), :101
        x = x + self.attn_proj(y)
        h = pk.layer_norm(x, self.ln_2.weight, self.ln_2.bias, self.ln_2.eps)
        return x + self.mlp_proj(F.gelu(self.c_fc(h)))


class PentaGPTFast(nn.Module):
    """PentaGPT for inference with packed projections (bf16 activations, or the
    per-token int8 path with act_quant='int8')."""

    def __init__(self, cfg: PentaGPTConfig, weights: dict, act_quant: str | None = None):
        super().__init__()
        self.cfg = cfg
        self.wte = nn.Embedding(cfg.vocab_size, cfg.n_embd)
        self.wpe = nn.Embedding(cfg.block_size, cfg.n_embd)
        with torch.no_grad():
            self.wte.weight.copy_(weights["wte"])
            self.wpe.weight.copy_(weights["wpe"])
        self.h = nn.ModuleList([_Block(cfg, weights["h"][i], act_quant) for i in range(cfg.n_layer)])
        self.ln_f = nn.LayerNorm(cfg.n_embd, bias=False)
        # weight tying: the lm_head packs the token-embedding matrix
        self.lm_head = _packed(weights["wte"], act_quant)

    @classmethod
    def random(cls, cfg: PentaGPTConfig | None = None, seed: int = 42, device="cuda",
               act_quant: str | None = None) -> "PentaGPTFast":
        """Random N(0, 0.02) weights from `seed` (a throughput model)."""
        cfg = cfg or PentaGPTConfig()
        g = torch.Generator(device=device).manual_seed(seed)
        d = cfg.n_embd

        def rnd(*shape):
            return torch.randn(*shape, device=device, generator=g) * 0.02

        weights = {"wte": rnd(cfg.vocab_size, d), "wpe": rnd(cfg.block_size, d), "h": []}
        for _ in range(cfg.n_layer):
            weights["h"].append({"c_attn": rnd(3 * d, d), "attn_proj": rnd(d, d) / math.sqrt(2 * cfg.n_layer),
                                 "c_fc": rnd(4 * d, d), "mlp_proj": rnd(d, 4 * d) / math.sqrt(2 * cfg.n_layer)})
        model = cls(cfg, weights, act_quant).to(device)
        return model

    def n_packed_params(self) -> int:
        return sum(m.packed_w.shape[0] * m.K_orig for m in self.modules() if isinstance(m, PentaLinearFast))

    @torch.no_grad()
    def forward(self, idx: torch.Tensor, all_logits: bool = False) -> torch.Tensor:
        B, T = idx.shape
        assert T <= self.cfg.block_size
        pos = torch.arange(T, device=idx.device)
        x = (self.wte(idx) + self.wpe(pos)).to(torch.bfloat16)
        for block in self.h:
            x = block(x)
        if not all_logits:
            x = x[:, [-1], :]  # LayerNorm is per position: normalise only what the lm_head reads
        x = pk.layer_norm(x, self.ln_f.weight, self.ln_f.bias, self.ln_f.eps)
        return self.lm_head(x)
