"""pentanet_layer -- drop-in for the reference module of the same name
(pentanet_layer.py): the STE training layer, the packed fast-inference layer
and the model converter, with the fast layer running on the sm_100a kernels.

    PentaLinear(in_features, out_features, bias=True)     pentanet_layer.py:17-65
    PentaLinearFast(packed_w, scale, K_orig, bias=None)    pentanet_layer.py:92-134
    convert_to_fast_inference(model)                       pentanet_layer.py:137-153

Differences, all additive:
  * convert_to_fast_inference also converts the GPT script's
    QuantLinear(mode='pentanet') layers (train_pentagpt.py:16-40), which the
    reference converter skips;
  * PentaLinearFast keeps `scale` and `K_orig` in its state_dict (the
    reference stores them as plain attributes, so a saved fast model loses
    them);
  * PentaLinearFast(..., act_quant='int8') routes prefill through the per-token
    int8 tensor-core path.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

try:
    from . import penta_kernel as _pk
except ImportError:
    import penta_kernel as _pk

quantize_and_pack = _pk.quantize_and_pack
_penta_linear_fast = _pk.penta_linear
_KERNEL_AVAILABLE = True


class PentaLinear(nn.Module):
    """Linear layer constrained to {-2,-1,0,+1,+2} x absmean scale, trained with
    the straight-through estimator (pentanet_layer.py:17-65).  Dense torch math:
    this is the training layer and the dense numeric reference.

    mode='bitnet' (not in the reference's PentaLinear; the ternary rule of its
    GPT script's QuantLinear, train_pentagpt.py:33-36) clamps to {-1, 0, +1}
    instead; to_fast_inference then packs the ternary codes in the same
    format."""

    def __init__(self, in_features, out_features, bias=True, mode='pentanet'):
        super().__init__()
        assert mode in ('pentanet', 'bitnet')
        self.mode = mode
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(torch.randn(out_features, in_features) * (1.0 / in_features ** 0.5))
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.register_parameter('bias', None)

    def forward(self, x):
        scale = self.weight.abs().mean().clamp(min=1e-8)
        qmax = 2 if self.mode == 'pentanet' else 1
        w_quant = torch.clamp(torch.round(self.weight / scale), -qmax, qmax)
        w_ste = (w_quant * scale - self.weight).detach() + self.weight
        return F.linear(x, w_ste, self.bias)

    def to_fast_inference(self) -> 'PentaLinearFast':
        """Convert to a PentaLinearFast for packed inference (pentanet_layer.py:50-65)."""
        assert self.weight.is_cuda, "Weights must be on CUDA"
        return PentaLinearFast.from_pentalinear(self)


class PentaLinearFast(nn.Module):
    """Drop-in replacement for PentaLinear using packed 3-bit weights and the
    fused sm_100a dequant-matmul (pentanet_layer.py:92-134)."""

    def __init__(self, packed_w: torch.Tensor, scale: float, K_orig: int,
                 bias: torch.Tensor | None = None, act_quant: str | None = None):
        super().__init__()
        assert act_quant in (None, 'int8')
        self.register_buffer('packed_w', packed_w)  # (N, K_packs) int32
        self._pad_weights()
        self.scale = float(scale)
        self.K_orig = int(K_orig)
        self.act_quant = act_quant
        if bias is not None:
            self.register_buffer('bias', bias)
        else:
            self.bias = None
        # persisted copies of the python attributes
        self.register_buffer('scale_buf', torch.tensor(self.scale, dtype=torch.float32), persistent=True)
        self.register_buffer('k_orig_buf', torch.tensor(self.K_orig, dtype=torch.int64), persistent=True)

    @classmethod
    def from_pentalinear(cls, layer: nn.Module, act_quant: str | None = None) -> 'PentaLinearFast':
        """Quantize + 3-bit pack the master weights of a trained PentaLinear (or
        QuantLinear in pentanet mode; in bitnet mode with its ternary rule,
        train_pentagpt.py:33-36, in the same codes)."""
        mode = 'bitnet' if getattr(layer, 'mode', 'pentanet') == 'bitnet' else 'pentanet'
        packed, K_orig, scale = quantize_and_pack(layer.weight.detach(), mode=mode)
        bias = layer.bias.detach().clone() if getattr(layer, 'bias', None) is not None else None
        return cls(packed, scale, K_orig, bias, act_quant=act_quant)

    @classmethod
    def from_state_dict(cls, state: dict, prefix: str = '', act_quant: str | None = None) -> 'PentaLinearFast':
        """A layer built from a saved PentaLinearFast state_dict (or the merged
        state of a sharded layer, penta_dist.merge_shards): packed words,
        gamma, K_orig and bias all come from the state."""
        bias = state.get(prefix + 'bias')
        return cls(state[prefix + 'packed_w'].contiguous(), float(state[prefix + 'scale_buf']),
                   int(state[prefix + 'k_orig_buf']), bias.clone() if bias is not None else None, act_quant=act_quant)

    def _pad_weights(self) -> None:
        # Resident CUDA weights are kept at a 16-byte row stride (same shape and
        # values; see penta_kernel.pad_packed) so that the GEMM reads them in
        # place instead of re-pitching them on every call.
        if self.packed_w.is_cuda:
            self.packed_w = _pk.pad_packed(self.packed_w)

    def _apply(self, fn, *args, **kwargs):
        super()._apply(fn, *args, **kwargs)  # device moves copy buffers contiguously
        self._pad_weights()
        return self

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)
        if prefix + 'scale_buf' in state_dict:
            self.scale = float(state_dict[prefix + 'scale_buf'])
        if prefix + 'k_orig_buf' in state_dict:
            self.K_orig = int(state_dict[prefix + 'k_orig_buf'])

    def forward(self, x: torch.Tensor, act: str | None = None, residual: torch.Tensor | None = None) -> torch.Tensor:
        """y = x @ W.T * scale (+ bias); optionally act='gelu' and a bf16
        `residual` added last, both fused into the product's epilogue."""
        if self.act_quant == 'int8':
            return _pk.penta_linear_i8(x, self.packed_w, self.scale, self.K_orig, self.bias, act=act,
                                       residual=residual)
        if x.dtype != torch.bfloat16:
            x = x.to(torch.bfloat16)
        return _penta_linear_fast(x, self.packed_w, self.scale, self.K_orig, self.bias, act=act, residual=residual)

    def extra_repr(self) -> str:
        N, K_packs = self.packed_w.shape
        mb = N * self.K_orig * 3 / 8 / 1e6
        return (f'in={self.K_orig}, out={N}, scale={self.scale:.4f}, '
                f'packed_size={mb:.3f} MB (3-bit)')


def _is_pentanary_layer(module: nn.Module) -> bool:
    if isinstance(module, PentaLinear):
        return True
    # train_pentagpt.QuantLinear (train_pentagpt.py:16-40), pentanet or bitnet mode
    return (type(module).__name__ == 'QuantLinear' and getattr(module, 'mode', None) in ('pentanet', 'bitnet')
            and isinstance(getattr(module, 'weight', None), torch.Tensor) and module.weight.dim() == 2)


def convert_to_fast_inference(model: nn.Module, act_quant: str | None = None) -> nn.Module:
    """Recursively convert every PentaLinear (and QuantLinear, mode 'pentanet'
    or the ternary 'bitnet') layer to PentaLinearFast (pentanet_layer.py:137-153).
    Tied weights are packed once per distinct parameter."""
    cache: dict[int, PentaLinearFast] = {}

    def rec(m: nn.Module) -> None:
        for name, module in list(m.named_children()):
            if _is_pentanary_layer(module):
                key = id(module.weight)
                if key in cache:
                    src = cache[key]
                    bias = module.bias.detach().clone() if getattr(module, 'bias', None) is not None else None
                    fast = PentaLinearFast(src.packed_w, src.scale, src.K_orig, bias, act_quant=act_quant)
                else:
                    fast = PentaLinearFast.from_pentalinear(module, act_quant=act_quant)
                    cache[key] = fast
                setattr(m, name, fast)
            else:
                rec(module)

    rec(model)
    return model
