"""Output-row sharding (penta_dist.py) on CPU with the gloo backend, world
size 2: shard ranges, the fp64 all-reduce of sum|W| for gamma, the all-gather
of output shards, and a ShardedPentaLinear whose local product is replaced by
the oracle (the CUDA product itself is covered by the GPU tests)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from _util import gen_act, gen_weight
from oracle import oracle as orc
import penta_dist as pd


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_range_covers_rows_once():
    for N in (1, 7, 128, 1000, 28672, 11008):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                lo, hi = pd.shard_range(N, r, world)
                assert 0 <= lo <= hi <= N
                seen.extend(range(lo, hi))
            assert seen == list(range(N))
            sizes = [pd.shard_range(N, r, world)[1] - pd.shard_range(N, r, world)[0] for r in range(world)]
            assert max(sizes) - min(sizes) <= 1


def _worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        N, K, M = 96, 250, 3
        w = gen_weight(N, K, seed=11)
        lo, hi = pd.shard_range(N, rank, world)
        # gamma from the sharded rows equals the whole-matrix absmean
        g_sharded = float(pd.global_absmean(w[lo:hi]))
        g_full = float(orc.absmean_scale(w.numpy()))
        # output shards meet in one all-gather, in column order
        packed, _, _ = orc.quantize_pack(w.numpy(), g_full)
        w8 = orc.unpack(packed, K)
        x = gen_act(M, K, seed=5).float().numpy()
        y_loc = torch.from_numpy(orc.matmul_f64(x, w8[lo:hi], g_full).astype(np.float32))
        y = pd.gather_columns(y_loc, N, world)
        want = orc.matmul_f64(x, w8, g_full).astype(np.float32)
        # ShardedPentaLinear.from_full keeps this rank's rows and gathers
        layer = pd.ShardedPentaLinear.from_full(torch.from_numpy(packed), g_full, K)
        assert layer.packed_w.shape[0] == hi - lo
        assert torch.equal(layer.packed_w, torch.from_numpy(packed[lo:hi]))
        layer.forward_local = lambda xx: torch.from_numpy(
            orc.matmul_f64(xx.float().numpy(), orc.unpack(layer.packed_w.numpy(), K), g_full).astype(np.float32))
        y2 = layer(torch.from_numpy(x).reshape(1, M, K))
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), g_sharded=g_sharded, g_full=g_full, y=y.numpy(),
                 want=want, y2=y2.numpy())
    finally:
        dist.destroy_process_group()


def test_sharded_layer_gloo_world2(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    for r in range(world):
        d = np.load(tmp_path / f"r{r}.npz")
        assert abs(float(d["g_sharded"]) - float(d["g_full"])) <= 1e-7 * float(d["g_full"])
        assert np.array_equal(d["y"], d["want"])
        assert d["y2"].shape == (1,) + d["want"].shape
        assert np.array_equal(d["y2"][0], d["want"])
