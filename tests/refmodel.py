"""The reference's GPT module tree (train_pentagpt.py:16-176), restated as test
infrastructure so that the drop-in conversion can be checked where the
reference tree is absent.

Same module names, nesting, parameter names and forward arithmetic as
train_pentagpt.PentaGPT: QuantLinear in pentanet mode (fake-quantised
weights, train_pentagpt.py:16-40), causal self-attention with an explicit
masked softmax (:42-71), GELU MLP (:73-87), pre-LayerNorm blocks without
biases (:89-99), tied lm_head and last-position logits (:101-136).  Whether
this restatement computes what the reference computes is itself pinned: the
fixture script (golden/make_pentagpt_golden.py) loads the same weights into
the reference's own module and stores its logits, and the test compares this
module's fp32 forward with them before converting it.

Weights come from `weights(cfg, seed)`: every parameter drawn from its own
seeded CPU generator with the reference's init statistics (N(0, 1/in) for
QuantLinear, N(0, 1) for the position table, LayerNorm gains near one), so
any machine rebuilds them bit for bit.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


class Cfg:
    def __init__(self, n_layer: int, n_head: int, n_embd: int, vocab_size: int = 50257, block_size: int = 256):
        self.n_layer, self.n_head, self.n_embd = n_layer, n_head, n_embd
        self.vocab_size, self.block_size = vocab_size, block_size
        self.bias = False
        self.dropout = 0.0
        self.mode = "pentanet"


class QuantLinear(nn.Module):
    """Class name and `mode` attribute as the reference's, so the converter
    recognises it (train_pentagpt.py:16-40)."""

    def __init__(self, fan_in: int, fan_out: int, mode: str = "pentanet"):
        super().__init__()
        self.in_features, self.out_features, self.mode = fan_in, fan_out, mode
        self.weight = nn.Parameter(torch.empty(fan_out, fan_in))
        self.register_parameter("bias", None)
        # The reference's gamma is torch's fp32 CPU mean, whose last bit depends
        # on the machine's summation order; the fixtures record the values the
        # reference computed, and a test may pin them here.
        self.fixed_gamma = None

    def forward(self, x):
        gamma = (self.weight.abs().mean().clamp(min=1e-8) if self.fixed_gamma is None
                 else torch.tensor(self.fixed_gamma, dtype=self.weight.dtype, device=self.weight.device))
        lim = 2 if self.mode == "pentanet" else 1
        q = torch.clamp(torch.round(self.weight / gamma), -lim, lim)
        return F.linear(x, (q * gamma - self.weight).detach() + self.weight, self.bias)


class CausalSelfAttention(nn.Module):
    def __init__(self, cfg: Cfg):
        super().__init__()
        self.c_attn = QuantLinear(cfg.n_embd, 3 * cfg.n_embd)
        self.c_proj = QuantLinear(cfg.n_embd, cfg.n_embd)
        self.n_head, self.n_embd = cfg.n_head, cfg.n_embd
        mask = torch.tril(torch.ones(cfg.block_size, cfg.block_size)).view(1, 1, cfg.block_size, cfg.block_size)
        self.register_buffer("bias", mask)

    def forward(self, x):
        B, T, C = x.shape
        hd = C // self.n_head
        q, k, v = self.c_attn(x).split(self.n_embd, dim=2)
        q, k, v = (t.view(B, T, self.n_head, hd).transpose(1, 2) for t in (q, k, v))
        att = (q @ k.transpose(-2, -1)) * (1.0 / math.sqrt(hd))
        att = F.softmax(att.masked_fill(self.bias[:, :, :T, :T] == 0, float("-inf")), dim=-1)
        y = (att @ v).transpose(1, 2).contiguous().view(B, T, C)
        return self.c_proj(y)


class MLP(nn.Module):
    def __init__(self, cfg: Cfg):
        super().__init__()
        self.c_fc = QuantLinear(cfg.n_embd, 4 * cfg.n_embd)
        self.gelu = nn.GELU()
        self.c_proj = QuantLinear(4 * cfg.n_embd, cfg.n_embd)

    def forward(self, x):
        return self.c_proj(self.gelu(self.c_fc(x)))


class Block(nn.Module):
    def __init__(self, cfg: Cfg):
        super().__init__()
        self.ln_1 = nn.LayerNorm(cfg.n_embd, bias=False)
        self.attn = CausalSelfAttention(cfg)
        self.ln_2 = nn.LayerNorm(cfg.n_embd, bias=False)
        self.mlp = MLP(cfg)

    def forward(self, x):
        x = x + self.attn(self.ln_1(x))
        return x + self.mlp(self.ln_2(x))


class PentaGPT(nn.Module):
    def __init__(self, cfg: Cfg):
        super().__init__()
        self.config = cfg
        self.transformer = nn.ModuleDict(dict(
            wte=nn.Embedding(cfg.vocab_size, cfg.n_embd),
            wpe=nn.Embedding(cfg.block_size, cfg.n_embd),
            drop=nn.Dropout(0.0),
            h=nn.ModuleList([Block(cfg) for _ in range(cfg.n_layer)]),
            ln_f=nn.LayerNorm(cfg.n_embd, bias=False),
        ))
        self.lm_head = QuantLinear(cfg.n_embd, cfg.vocab_size)
        self.transformer.wte.weight = self.lm_head.weight

    def forward(self, idx, targets=None):
        t = idx.shape[1]
        pos = torch.arange(t, device=idx.device)
        x = self.transformer.drop(self.transformer.wte(idx) + self.transformer.wpe(pos))
        for blk in self.transformer.h:
            x = blk(x)
        x = self.transformer.ln_f(x)
        if targets is None:
            return self.lm_head(x[:, [-1], :]), None
        logits = self.lm_head(x)
        return logits, F.cross_entropy(logits.view(-1, logits.size(-1)), targets.view(-1), ignore_index=-1)


def weights(model: nn.Module, seed: int) -> dict:
    """Deterministic parameters for `model`'s state_dict keys (the reference
    model has the same keys): one CPU generator per key, seeded seed + index."""
    out = {}
    for i, (name, t) in enumerate(model.state_dict().items()):
        g = torch.Generator().manual_seed(seed + i)
        if name.endswith("attn.bias"):      # the causal mask buffer
            out[name] = t.clone()
        elif name.endswith("wpe.weight"):
            out[name] = torch.randn(t.shape, generator=g)
        elif ".ln_" in name or name.startswith("transformer.ln_f"):
            out[name] = 1.0 + 0.1 * torch.randn(t.shape, generator=g)
        else:                                # QuantLinear weights (and the tied table)
            out[name] = torch.randn(t.shape, generator=g) / math.sqrt(t.shape[1])
    # tied: the token table is the lm_head weight (train_pentagpt.py:116)
    out["transformer.wte.weight"] = out["lm_head.weight"]
    return out


def quant_layers(model: nn.Module) -> list:
    """The QuantLinear modules in named_modules() order (tied ones once)."""
    return [m for _, m in model.named_modules() if type(m).__name__ == "QuantLinear"]


def tokens(cfg: Cfg, batch: int, seq: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    idx = torch.randint(0, cfg.vocab_size, (batch, seq), generator=g)
    tgt = torch.randint(0, cfg.vocab_size, (batch, seq), generator=g)
    return idx, tgt


CONFIGS = {
    # two layers of the reference's "small" size at the full GPT-2 vocabulary
    "small2": (Cfg(n_layer=2, n_head=6, n_embd=384), 11, 2, 64),
    # the reference's "large" size: 12 layers, 12 heads, d 768 (PentaNet-124M), a short sequence
    "large": (Cfg(n_layer=12, n_head=12, n_embd=768), 12, 2, 32),
}
