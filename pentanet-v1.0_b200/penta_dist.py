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

A column-parallel layer and its row-parallel partner (an MLP's up and down
projections) need no gather at all: `ShardedPentaLinear(gather=False)` keeps
each rank's block of the up projection's outputs on that rank, and
`RowShardedPentaLinear` multiplies that block by its K slice of the down
projection's packed weights, so one all-reduce of fp32 partial products per
pair replaces an all-gather per layer.  Both shard with boundaries on
multiples of 40 columns, so every K slice starts on a packed word.
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


def shard_range(N: int, rank: int, world: int, unit: int = 1) -> tuple[int, int]:
    """Rows [lo, hi) owned by `rank`; remainders go to the lowest ranks.  With
    unit > 1 the boundaries fall on multiples of `unit` (the last shard ends at
    N): a column-parallel layer sharded with unit 40 hands a row-parallel
    partner K slices that start on packed words (10 k each) at 16-byte
    aligned activation offsets."""
    if unit > 1:
        lo_u, hi_u = shard_range((N + unit - 1) // unit, rank, world)
        return min(lo_u * unit, N), min(hi_u * unit, N)
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
                   out: torch.Tensor | None = None, unit: int = 1) -> torch.Tensor:
    """All-gather the per-rank (M, hi - lo) output blocks, rank r owning the
    columns shard_range(N, r, world, unit), into the full (M, N) result.
    Equal shards (all 7B/70B shapes at P <= 8) gather in place; unequal ones
    are padded to the largest shard for the collective."""
    M, n_loc = y_local.shape
    ranges = [shard_range(N, r, world, unit) for r in range(world)]
    lo, hi = ranges[dist.get_rank(group)]
    assert n_loc == hi - lo, f"this rank owns {hi - lo} columns, got {n_loc}"
    n_max = max(b - a for a, b in ranges)
    if out is None:
        out = torch.empty(M, N, dtype=y_local.dtype, device=y_local.device)
    src = y_local.contiguous()
    if n_loc != n_max:
        src = torch.zeros(M, n_max, dtype=y_local.dtype, device=y_local.device)
        src[:, :n_loc] = y_local
    # rank-major concatenation along dim 0 (the layout every backend accepts)
    buf = torch.empty(world * M, n_max, dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, src, group=group)
    if n_max * world == N:
        out.view(M, world, n_max).copy_(buf.view(world, M, n_max).permute(1, 0, 2))
    else:
        blocks = buf.view(world, M, n_max)
        for r, (a, b) in enumerate(ranges):
            out[:, a:b].copy_(blocks[r, :, :b - a])
    return out


SHARD_ROWS, SHARD_K = 0, 1


def _register_shard_state(m: torch.nn.Module, scale: float, K_orig: int, axis: int, lo: int, hi: int, full: int,
                          world: int, unit: int) -> None:
    """Persist what the packed words alone do not say: gamma, K_orig and which
    slice of which layout this rank holds ([axis, lo, hi, full, world, unit];
    axis SHARD_ROWS = output rows [lo, hi) of `full`, SHARD_K = inputs [lo, hi)
    of K_orig = `full`)."""
    m.register_buffer("scale_buf", torch.tensor(float(scale), dtype=torch.float32))
    m.register_buffer("k_orig_buf", torch.tensor(int(K_orig), dtype=torch.int64))
    m.register_buffer("shard_buf", torch.tensor([axis, lo, hi, full, world, unit], dtype=torch.int64))


def _describe_shard(info) -> str:
    axis, lo, hi, full, world, unit = (int(v) for v in info)
    what = "output rows" if axis == SHARD_ROWS else "inputs"
    return f"{what} [{lo}, {hi}) of {full} (world {world}, unit {unit})"


def _check_shard_state(m: torch.nn.Module, state_dict, prefix: str) -> None:
    key = prefix + "shard_buf"
    if key in state_dict:
        got, own = state_dict[key].tolist(), m.shard_buf.tolist()
        assert got == own, (f"checkpoint holds {_describe_shard(got)}, this layer is "
                            f"{_describe_shard(own)}")


def _restore_attrs(m: torch.nn.Module) -> None:
    m.scale = float(m.scale_buf)
    m.K_orig = int(m.k_orig_buf)


def merge_shards(states: list[dict], prefix: str = "") -> dict:
    """The unsharded layer's state (PentaLinearFast's keys: the canonical
    (N, ceil(K/10)) `packed_w`, `scale_buf`, `k_orig_buf` and `bias` when the
    layer has one) from the state_dicts of every rank's shard of one layer,
    given in any order.  Output-row shards concatenate by rows; K shards by
    packed words (their boundaries are word-aligned and the last one holds the
    padded final word)."""
    infos = [[int(v) for v in st[prefix + "shard_buf"].tolist()] for st in states]
    axis, _, _, full, world, unit = infos[0]
    assert len(states) == world, f"{len(states)} shards for a world of {world}"
    assert all(i[0] == axis and i[3] == full and i[4] == world and i[5] == unit for i in infos),         "shards of different layouts"
    order = sorted(range(world), key=lambda r: (infos[r][1], infos[r][2]))
    assert [(infos[r][1], infos[r][2]) for r in order] == [shard_range(full, r, world, unit) for r in range(world)],         "the shards do not tile the layer (missing or repeated ranks)"
    scales = {float(st[prefix + "scale_buf"]) for st in states}
    assert len(scales) == 1, "shards of one layer disagree on gamma"
    parts = [states[r][prefix + "packed_w"].contiguous() for r in order]
    out = {"scale_buf": states[0][prefix + "scale_buf"].clone(), "k_orig_buf": states[0][prefix + "k_orig_buf"].clone()}
    has_bias = prefix + "bias" in states[0]
    if axis == SHARD_ROWS:
        out["packed_w"] = torch.cat(parts, dim=0)
        if has_bias:
            out["bias"] = torch.cat([states[r][prefix + "bias"] for r in order])
    else:
        out["packed_w"] = torch.cat(parts, dim=1)
        if has_bias:
            out["bias"] = states[0][prefix + "bias"].clone()
    assert out["packed_w"].shape[1] == pk._k_packs(int(out["k_orig_buf"])), "merged words do not cover K_orig"
    return out


class ShardedPentaLinear(torch.nn.Module):
    """PentaLinearFast split by output rows over the ranks of `group`; forward
    returns the full (..., N) output on every rank, or with gather=False this
    rank's (..., hi - lo) block of columns [lo, hi) (the input of a
    RowShardedPentaLinear partner, which then needs no gather)."""

    def __init__(self, packed_local: torch.Tensor, scale: float, K_orig: int, N: int,
                 bias_local: torch.Tensor | None = None, group=None, act_quant: str | None = None,
                 peers: "PeerGroup | None" = None, max_tokens: int = 64, gather: bool = True, unit: int = 1):
        super().__init__()
        self.gather = gather
        self.unit = int(unit)
        self.register_buffer("packed_w", packed_local)
        self.scale = float(scale)
        self.K_orig = int(K_orig)
        self.N = int(N)
        self.group = group
        self.world = dist.get_world_size(group)
        self.act_quant = act_quant
        self.register_buffer("bias", bias_local)
        lo, hi = shard_range(self.N, dist.get_rank(group), self.world, self.unit)
        assert packed_local.shape[0] == hi - lo, f"this rank owns {hi - lo} rows, got {packed_local.shape[0]}"
        _register_shard_state(self, self.scale, self.K_orig, SHARD_ROWS, lo, hi, self.N, self.world, self.unit)
        # Fused mode: outputs stored into every rank's buffer by the GEMM
        # itself (bf16 activations); the returned tensor is a view of that
        # buffer and is overwritten by the next forward of this layer.
        self.peers = peers
        if peers is not None:
            assert gather, "peer-mapped outputs are gathered by construction"
            self.col0 = shard_range(self.N, peers.rank, peers.world, self.unit)[0]
            self.out, self.out_ptrs = peers.buffer((max_tokens, self.N), torch.bfloat16)

    @classmethod
    def from_full(cls, packed: torch.Tensor, scale: float, K_orig: int, bias: torch.Tensor | None = None,
                  group=None, act_quant: str | None = None, peers: "PeerGroup | None" = None,
                  max_tokens: int = 64, gather: bool = True, unit: int = 1) -> "ShardedPentaLinear":
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        lo, hi = shard_range(packed.shape[0], rank, world, unit)
        b = bias[lo:hi].contiguous() if bias is not None else None
        return cls(packed[lo:hi].contiguous(), scale, K_orig, packed.shape[0], b, group, act_quant, peers, max_tokens,
                   gather, unit)

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        _check_shard_state(self, state_dict, prefix)
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)
        _restore_attrs(self)

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
        if not self.gather:
            return y_loc.reshape(*lead, y_loc.shape[-1])
        y = gather_columns(y_loc, self.N, self.world, self.group, unit=self.unit)
        return y.reshape(*lead, self.N)


class RowShardedPentaLinear(torch.nn.Module):
    """The row-parallel partner of a column-parallel layer (the MLP's down
    projection after its up projection): the weight's input dimension K is split
    over the ranks at packed-word boundaries, each rank multiplies its slice of
    the activations by its slice of the weights into an fp32 partial product,
    one all-reduce sums the partials, and the bias and the reference's bf16
    rounding (bf16(acc * gamma), then + bf16(bias)) are applied to the sum.
    Paired with a ShardedPentaLinear(gather=False) sharded with the same
    `unit`, the activations never leave their rank: one all-reduce per pair
    instead of an all-gather per layer.  bf16 activations only."""

    def __init__(self, packed_local: torch.Tensor, scale: float, K_local: int, k0: int, K_orig: int,
                 bias: torch.Tensor | None = None, group=None, unit: int = 40):
        super().__init__()
        self.register_buffer("packed_w", packed_local)  # (N, words of this rank's K slice)
        self.scale = float(scale)
        self.K_local = int(K_local)
        self.k0 = int(k0)
        self.K_orig = int(K_orig)
        self.N = int(packed_local.shape[0])
        self.register_buffer("bias", bias)
        self.group = group
        self.world = dist.get_world_size(group)
        _register_shard_state(self, self.scale, self.K_orig, SHARD_K, self.k0, self.k0 + self.K_local, self.K_orig,
                              self.world, unit)

    @staticmethod
    def slice_k(packed: torch.Tensor, K_orig: int, rank: int, world: int, unit: int = 40):
        """Rank `rank`'s K slice [lo, hi) of a packed (N, ceil(K/10)) weight: the
        words covering it (the last rank keeps the padded final word) and lo, hi."""
        assert unit % pk._W_PER_INT32 == 0, "K slices must start on packed words"
        lo, hi = shard_range(K_orig, rank, world, unit)
        w0 = lo // pk._W_PER_INT32
        w1 = packed.shape[1] if hi == K_orig else hi // pk._W_PER_INT32
        if lo == hi:  # a trailing rank without columns holds no words
            w0 = w1 = 0
        local = packed[:, w0:w1].contiguous()
        if local.is_cuda and local.shape[1] > 0:
            local = pk.pad_packed(local)
        return local, lo, hi

    @classmethod
    def from_full(cls, packed: torch.Tensor, scale: float, K_orig: int, bias: torch.Tensor | None = None,
                  group=None, unit: int = 40) -> "RowShardedPentaLinear":
        local, lo, hi = cls.slice_k(packed, K_orig, dist.get_rank(group), dist.get_world_size(group), unit)
        return cls(local, scale, hi - lo, lo, K_orig, bias, group, unit)

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        _check_shard_state(self, state_dict, prefix)
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)
        _restore_attrs(self)

    def forward_local(self, x_local: torch.Tensor) -> torch.Tensor:
        """This rank's fp32 partial product (M, N) = x_local @ W_slice.T * gamma."""
        if self.K_local == 0:
            return torch.zeros(x_local.shape[0], self.N, dtype=torch.float32, device=x_local.device)
        return pk.penta_linear(x_local.to(torch.bfloat16).contiguous(), self.packed_w, self.scale, self.K_local,
                               out_dtype=torch.float32)

    def forward(self, x: torch.Tensor, x_is_local: bool = False) -> torch.Tensor:
        """x: the full (..., K) activations, or with x_is_local=True this rank's
        (..., K_local) slice (a column-parallel layer's gather=False output)."""
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if not x_is_local:
            x2 = x2[:, self.k0:self.k0 + self.K_local]
        assert x2.shape[1] == self.K_local, f"expected {self.K_local} input features on this rank, got {x2.shape[1]}"
        y = self.forward_local(x2)
        if self.world > 1:
            dist.all_reduce(y, group=self.group)
        yb = y.to(torch.bfloat16)
        if self.bias is not None:
            yb = (yb.float() + self.bias.detach().to(device=yb.device, dtype=torch.bfloat16).float()).to(torch.bfloat16)
        return yb.reshape(*lead, self.N)


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

    def barrier(self, stream=None, wait_ns: int = 0) -> None:
        """Enqueue the cross-GPU barrier.  Each rank's wait is bounded (wait_ns
        nanoseconds, 0 = the library default of 2 s); a wait that runs out
        leaves PN_ERR_TIMEOUT in the device status word
        (penta_native.device_status) and the group needs reset()."""
        s = stream if stream is not None else torch.cuda.current_stream()
        arr = (ctypes.c_void_p * self.world)(*self._flag_ptrs)
        nat.check(self._lib.pn_peer_barrier_wait(arr, self.world, self.rank, self.gen.data_ptr(), int(wait_ns),
                                                 s.cuda_stream), "pn_peer_barrier_wait")

    def reset(self) -> None:
        """Bring the barrier back into step after a wait ran out: every rank
        calls it (a host collective).  Each rank first lets its own kernels
        finish (every wait is bounded), the process group's barrier then
        guarantees that no barrier kernel is in flight on any rank, and only
        then does each rank zero its flag array and generation counter; a
        second host barrier keeps any rank from starting a new device
        barrier before all have zeroed."""
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self.flags.zero_()
        self.gen.zero_()
        torch.cuda.synchronize()
        dist.barrier(group=self.group)

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
    ws_bytes = nat.linear_workspace_size(nat.PN_BF16, M, N, K, x.device)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device) if ws_bytes else None
    arr = (ctypes.c_void_p * len(out_ptrs))(*out_ptrs)
    s = stream if stream is not None else torch.cuda.current_stream(x.device)
    b = bias_local.to(torch.bfloat16).contiguous() if bias_local is not None else None
    ydt = nat.PN_F32 if out_dtype == torch.float32 else nat.PN_BF16
    nat.check(L.pn_linear_bf16_peers(x.data_ptr(), M, K, packed_local.data_ptr(), N, KP, ctypes.c_float(scale),
                                     nat.ptr(b), arr, len(out_ptrs), ld, col0, ydt, nat.ptr(ws), ws_bytes,
                                     s.cuda_stream), "pn_linear_bf16_peers")
