"""Output-dimension sharding of a packed PentaLinear across the GPUs of one node.

Rank r of a world of P owns the packed rows [r*N/P, (r+1)*N/P): a contiguous
slice of the canonical (N, K_packs) tensor, so sharding needs no repacking.
The per-tensor scale gamma is computed from the whole matrix before sharding
(or, for weights that only exist sharded, from an all-reduce of sum|W| in
float64 and the total element count), so every shard quantises exactly as the
unsharded layer would.  Each rank runs the local tensor-core GEMV/GEMM on its
rows and the shards meet in one NCCL all-gather; the reference has no
multi-GPU path (its multi-"GPU" runs are independent jobs).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

try:
    from . import penta_kernel as pk
except ImportError:
    import penta_kernel as pk


def shard_range(N: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [lo, hi) owned by `rank`; remainders go to the lowest ranks."""
    base, rem = divmod(N, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)


def shard_packed(packed: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    lo, hi = shard_range(packed.shape[0], rank, world)
    return packed[lo:hi]


def global_absmean(local_weight: torch.Tensor, group=None) -> torch.Tensor:
    """gamma of a matrix whose rows are spread over the ranks: one all-reduce of
    (sum|W|, count) in float64, then the same clamp as penta_kernel.py:57."""
    s = torch.stack([local_weight.double().abs().sum(),
                     torch.tensor(float(local_weight.numel()), dtype=torch.float64, device=local_weight.device)])
    dist.all_reduce(s, group=group)
    mean = (s[0] / s[1]).float()
    return mean.clamp(min=1e-8)


def gather_columns(y_local: torch.Tensor, N: int, world: int, group=None,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather per-rank (M, N/P) output blocks into the full (M, N) result.
    Requires N divisible by the world size (all 7B/70B shapes at P <= 8)."""
    M, n_loc = y_local.shape
    assert n_loc * world == N, "gather_columns needs equal shards"
    # rank-major concatenation along dim 0 (the layout every backend accepts)
    buf = torch.empty(world * M, n_loc, dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, y_local.contiguous(), group=group)
    if out is None:
        out = torch.empty(M, N, dtype=y_local.dtype, device=y_local.device)
    out.view(M, world, n_loc).copy_(buf.view(world, M, n_loc).permute(1, 0, 2))
    return out


class ShardedPentaLinear(torch.nn.Module):
    """PentaLinearFast split by output rows over the ranks of `group`; forward
    returns the full (..., N) output on every rank."""

    def __init__(self, packed_local: torch.Tensor, scale: float, K_orig: int, N: int,
                 bias_local: torch.Tensor | None = None, group=None, act_quant: str | None = None):
        super().__init__()
        self.register_buffer("packed_w", packed_local)
        self.scale = float(scale)
        self.K_orig = int(K_orig)
        self.N = int(N)
        self.group = group
        self.world = dist.get_world_size(group)
        self.act_quant = act_quant
        self.bias = bias_local

    @classmethod
    def from_full(cls, packed: torch.Tensor, scale: float, K_orig: int, bias: torch.Tensor | None = None,
                  group=None, act_quant: str | None = None) -> "ShardedPentaLinear":
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        lo, hi = shard_range(packed.shape[0], rank, world)
        b = bias[lo:hi].contiguous() if bias is not None else None
        return cls(packed[lo:hi].contiguous(), scale, K_orig, packed.shape[0], b, group, act_quant)

    def forward_local(self, x: torch.Tensor) -> torch.Tensor:
        if self.act_quant == "int8":
            return pk.penta_linear_i8(x, self.packed_w, self.scale, self.K_orig, self.bias)
        if x.dtype != torch.bfloat16:
            x = x.to(torch.bfloat16)
        return pk.penta_linear(x, self.packed_w, self.scale, self.K_orig, self.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        y_loc = self.forward_local(x.reshape(-1, x.shape[-1]))
        y = gather_columns(y_loc, self.N, self.world, self.group)
        return y.reshape(*lead, self.N)
