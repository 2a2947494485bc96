"""Output-dimension sharding of a packed PentaLinear across the GPUs of one node.

Two ways to assemble the output: `gather_columns` (an NCCL all-gather after
the local GEMM) and `PeerGroup` + `ShardedPentaLinear(..., peers=...)`, where
the GEMM's epilogue stores every output value straight into each GPU's
full-output buffer over NVLink (CUDA IPC mappings) and a cross-GPU barrier
kernel follows -- no separate collective, no extra pass over the output.

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

import ctypes

import torch
import torch.distributed as dist

try:
    from . import penta_kernel as pk
    from . import penta_native as nat
except ImportError:
    import penta_kernel as pk
    import penta_native as nat


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
                 bias_local: torch.Tensor | None = None, group=None, act_quant: str | None = None,
                 peers: "PeerGroup | None" = None, max_tokens: int = 64):
        super().__init__()
        self.register_buffer("packed_w", packed_local)
        self.scale = float(scale)
        self.K_orig = int(K_orig)
        self.N = int(N)
        self.group = group
        self.world = dist.get_world_size(group)
        self.act_quant = act_quant
        self.bias = bias_local
        # Fused mode: outputs stored into every rank's buffer by the GEMM
        # itself (bf16 activations); the returned tensor is a view of that
        # buffer and is overwritten by the next forward of this layer.
        self.peers = peers
        if peers is not None:
            self.col0 = shard_range(self.N, peers.rank, peers.world)[0]
            self.out, self.out_ptrs = peers.buffer((max_tokens, self.N), torch.bfloat16)

    @classmethod
    def from_full(cls, packed: torch.Tensor, scale: float, K_orig: int, bias: torch.Tensor | None = None,
                  group=None, act_quant: str | None = None, peers: "PeerGroup | None" = None,
                  max_tokens: int = 64) -> "ShardedPentaLinear":
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        lo, hi = shard_range(packed.shape[0], rank, world)
        b = bias[lo:hi].contiguous() if bias is not None else None
        return cls(packed[lo:hi].contiguous(), scale, K_orig, packed.shape[0], b, group, act_quant, peers, max_tokens)

    def forward_local(self, x: torch.Tensor) -> torch.Tensor:
        if self.act_quant == "int8":
            return pk.penta_linear_i8(x, self.packed_w, self.scale, self.K_orig, self.bias)
        if x.dtype != torch.bfloat16:
            x = x.to(torch.bfloat16)
        return pk.penta_linear(x, self.packed_w, self.scale, self.K_orig, self.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        if self.peers is not None and self.act_quant is None:
            x2 = x.reshape(-1, x.shape[-1])
            if x2.dtype != torch.bfloat16:
                x2 = x2.to(torch.bfloat16)
            x2 = x2.contiguous()
            M = x2.shape[0]
            assert M <= self.out.shape[0], "more tokens than the peer output buffer holds"
            linear_peers(x2, self.packed_w, self.scale, self.K_orig, self.col0, self.out_ptrs, self.N,
                         bias_local=self.bias)
            self.peers.barrier()
            return self.out[:M].reshape(*lead, self.N)
        y_loc = self.forward_local(x.reshape(-1, x.shape[-1]))
        y = gather_columns(y_loc, self.N, self.world, self.group)
        return y.reshape(*lead, self.N)


class PeerGroup:
    """Peer-mapped output buffers for output-sharded layers, one GPU per rank.

    `buffer(shape, dtype)` allocates a full-output tensor on this GPU and maps
    the same buffer of every other rank (CUDA IPC; the handles travel over
    the process group), returning the local tensor and the peers' device
    pointers.  `barrier(stream)` enqueues the cross-GPU barrier (device-side
    generation counter, so it can be captured in CUDA graphs).  Every rank
    must create buffers in the same order."""

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert 1 <= self.world <= 8, "PeerGroup supports up to 8 GPUs"
        self._lib = nat.load()
        self._opened = {}  # (rank, handle) -> mapped base: an allocation is opened once
        self._keep = []
        self.flags, self._flag_ptrs = self.buffer((self.world,), torch.int32)
        self.flags.zero_()
        self.gen = torch.zeros(1, dtype=torch.int32, device=self.flags.device)
        torch.cuda.synchronize()
        dist.barrier(group=group)

    def _exchange(self, t: torch.Tensor) -> list[int]:
        L = self._lib
        handle = (ctypes.c_char * 64)()
        off = ctypes.c_size_t(0)
        nat.check(L.pn_ipc_handle(t.data_ptr(), handle, ctypes.byref(off)), "pn_ipc_handle")
        mine = (bytes(handle), int(off.value))
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=self.group)
        ptrs = []
        for r, (h, o) in enumerate(allh):
            if r == self.rank:
                ptrs.append(t.data_ptr())
                continue
            key = (r, h)
            if key not in self._opened:
                base = ctypes.c_void_p()
                nat.check(L.pn_ipc_open(h, ctypes.byref(base)), "pn_ipc_open")
                self._opened[key] = base.value
            ptrs.append(self._opened[key] + o)
        return ptrs

    def buffer(self, shape, dtype) -> tuple[torch.Tensor, list[int]]:
        t = torch.zeros(shape, dtype=dtype, device=torch.device("cuda", torch.cuda.current_device()))
        self._keep.append(t)
        return t, self._exchange(t)

    def barrier(self, stream=None) -> None:
        s = stream if stream is not None else torch.cuda.current_stream()
        arr = (ctypes.c_void_p * self.world)(*self._flag_ptrs)
        nat.check(self._lib.pn_peer_barrier(arr, self.world, self.rank, self.gen.data_ptr(), s.cuda_stream),
                  "pn_peer_barrier")

    def close(self) -> None:
        torch.cuda.synchronize()
        for p in self._opened.values():
            self._lib.pn_ipc_close(ctypes.c_void_p(p))
        self._opened.clear()


def linear_peers(x: torch.Tensor, packed_local: torch.Tensor, scale: float, K_orig: int, col0: int,
                 out_ptrs: list[int], ld: int, out_dtype: torch.dtype = torch.bfloat16,
                 bias_local: torch.Tensor | None = None, stream=None) -> None:
    """This rank's output columns [col0, col0 + N_local) of x @ W^T, stored into
    every rank's full-output buffer (row stride ld).  Follow with
    PeerGroup.barrier before reading the buffer."""
    assert x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2
    M, K = x.shape
    assert K == K_orig
    N, KP = packed_local.shape
    L = nat.load()
    ws_bytes = int(L.pn_linear_workspace_size(nat.PN_BF16, M, N, K))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device) if ws_bytes else None
    arr = (ctypes.c_void_p * len(out_ptrs))(*out_ptrs)
    s = stream if stream is not None else torch.cuda.current_stream(x.device)
    b = bias_local.to(torch.bfloat16).contiguous() if bias_local is not None else None
    ydt = nat.PN_F32 if out_dtype == torch.float32 else nat.PN_BF16
    nat.check(L.pn_linear_bf16_peers(x.data_ptr(), M, K, packed_local.data_ptr(), N, KP, ctypes.c_float(scale),
                                     nat.ptr(b), arr, len(out_ptrs), ld, col0, ydt, nat.ptr(ws), ws_bytes,
                                     s.cuda_stream), "pn_linear_bf16_peers")
