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


def test_shard_range_aligned():
    for N in (1, 39, 40, 250, 1000, 2816, 28672):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                lo, hi = pd.shard_range(N, r, world, 40)
                assert 0 <= lo <= hi <= N
                assert (lo % 40 == 0 or lo == N) and (hi % 40 == 0 or hi == N)
                seen.extend(range(lo, hi))
            assert seen == list(range(N))


def _gelu(a: np.ndarray) -> np.ndarray:
    return torch.nn.functional.gelu(torch.from_numpy(a.astype(np.float32))).numpy()


def _pair_worker(rank, world, port, out_dir):
    """Up projection sharded by output column without a gather, GELU on the
    local block, down projection sharded by K with one all-reduce; the local
    products are the oracle's."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        D, H, M = 130, 250, 3
        w_up, w_dn = gen_weight(H, D, seed=21).numpy(), gen_weight(D, H, seed=22).numpy()
        g_up, g_dn = float(orc.absmean_scale(w_up)), float(orc.absmean_scale(w_dn))
        p_up, _, _ = orc.quantize_pack(w_up, g_up)
        p_dn, _, _ = orc.quantize_pack(w_dn, g_dn)
        bias = gen_weight(1, D, seed=23, std=0.5).numpy()[0]
        x = gen_act(M, D, seed=24).float().numpy()

        up = pd.ShardedPentaLinear.from_full(torch.from_numpy(p_up), g_up, D, gather=False, unit=40)
        up.forward_local = lambda xx: torch.from_numpy(
            orc.matmul_f64(xx.float().numpy(), orc.unpack(up.packed_w.numpy(), D), g_up).astype(np.float32))
        dn = pd.RowShardedPentaLinear.from_full(torch.from_numpy(p_dn), g_dn, H, bias=torch.from_numpy(bias), unit=40)
        dn.forward_local = lambda xl: torch.from_numpy(
            orc.matmul_f64(xl.float().numpy(), orc.unpack(dn.packed_w.numpy(), dn.K_local), g_dn).astype(np.float32))
        lo, hi = pd.shard_range(H, rank, world, 40)
        h_loc = up(torch.from_numpy(x)).numpy()
        y = dn(torch.from_numpy(_gelu(h_loc)), x_is_local=True).float().numpy()

        h_full = orc.matmul_f64(x, orc.unpack(p_up, D), g_up).astype(np.float32)
        a_full = _gelu(h_full)
        y_full_in = dn(torch.from_numpy(a_full)).float().numpy()  # slices the full input itself
        acc = orc.matmul_f64(a_full, orc.unpack(p_dn, H), g_dn)
        np.savez(os.path.join(out_dir, f"p{rank}.npz"), lo=lo, hi=hi, k0=dn.k0, K_local=dn.K_local,
                 h_loc=h_loc, h_want=h_full[:, lo:hi], y=y, y_full_in=y_full_in,
                 want=orc.bf16_linear_out(acc.astype(np.float32), bias), pre=acc,
                 words=np.array(dn.packed_w.numpy()), words_want=p_dn[:, lo // 10:(p_dn.shape[1] if hi == H else hi // 10)])
    finally:
        dist.destroy_process_group()


def test_column_row_pairing_gloo_world2(tmp_path):
    from _util import assert_bf16_close
    world = 2
    mp.start_processes(_pair_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    bounds = []
    for r in range(world):
        d = np.load(tmp_path / f"p{r}.npz")
        # the down projection's K slice is exactly the up projection's column block
        assert int(d["k0"]) == int(d["lo"]) and int(d["K_local"]) == int(d["hi"]) - int(d["lo"])
        assert np.array_equal(d["words"], d["words_want"])
        assert np.array_equal(d["h_loc"], d["h_want"])
        # every rank holds the whole all-reduced output, equal whichever way the input came
        assert np.array_equal(d["y"], d["y_full_in"])
        assert_bf16_close(d["y"], d["want"].astype(np.float64), "row-parallel down projection", pre_bias=d["pre"])
        bounds.append((int(d["lo"]), int(d["hi"])))
    assert bounds == [(0, 160), (160, 250)]


def test_k_slices_concatenate_to_packed():
    """K slices of every rank, empty trailing ones included, put back together
    word by word give the packed tensor."""
    for K in (250, 1000, 1376, 41, 7):
        packed, _, _ = orc.quantize_pack(gen_weight(5, K, seed=K).numpy())
        pt = torch.from_numpy(packed)
        for world in (1, 2, 3, 8):
            parts = []
            for r in range(world):
                local, lo, hi = pd.RowShardedPentaLinear.slice_k(pt, K, r, world)
                assert local.shape[1] == (0 if lo == hi else orc.k_packs(hi) - lo // 10)
                parts.append(local)
            assert torch.equal(torch.cat(parts, dim=1), pt)


def _ckpt_worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        N, K = 90, 250
        w = gen_weight(N, K, seed=41).numpy()
        g = float(orc.absmean_scale(w))
        packed = torch.from_numpy(orc.quantize_pack(w, g)[0])
        bias = gen_weight(1, N, seed=42, std=0.5)[0]
        rows = pd.ShardedPentaLinear.from_full(packed, g, K, bias=bias, unit=40)
        ks = pd.RowShardedPentaLinear.from_full(packed, g, K, bias=bias, unit=40)
        torch.save({"rows": rows.state_dict(), "k": ks.state_dict()}, os.path.join(out_dir, f"c{rank}.pt"))
        dist.barrier()
        other = torch.load(os.path.join(out_dir, f"c{1 - rank}.pt"))
        mine = torch.load(os.path.join(out_dir, f"c{rank}.pt"))
        refused = []
        for name, layer in (("rows", rows), ("k", ks)):
            try:
                layer.load_state_dict(other[name])
                refused.append(False)
            except AssertionError:
                refused.append(True)
        # a layer built with a wrong gamma takes gamma and K_orig back from its own shard
        fresh = pd.RowShardedPentaLinear.from_full(packed, 1.0, K, bias=torch.zeros(N), unit=40)
        fresh.load_state_dict(mine["k"])
        np.savez(os.path.join(out_dir, f"s{rank}.npz"), refused=np.array(refused), scale=fresh.scale, g=g,
                 bias_ok=bool(torch.equal(fresh.bias, bias)))
    finally:
        dist.destroy_process_group()


def test_sharded_checkpoint_gloo_world2(tmp_path):
    """Shard info persists: each rank's state_dict names its slice, loading a
    neighbour's shard is refused, and the shards of either layout merge back
    into the unsharded layer's packed words, gamma, K_orig and bias."""
    import pentanet_layer as pl
    world = 2
    mp.start_processes(_ckpt_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    N, K = 90, 250
    w = gen_weight(N, K, seed=41).numpy()
    g = float(orc.absmean_scale(w))
    packed = torch.from_numpy(orc.quantize_pack(w, g)[0])
    bias = gen_weight(1, N, seed=42, std=0.5)[0]
    states = [torch.load(tmp_path / f"c{r}.pt") for r in range(world)]
    assert states[0]["rows"]["shard_buf"].tolist() == [pd.SHARD_ROWS, 0, 80, N, 2, 40]
    assert states[1]["k"]["shard_buf"].tolist() == [pd.SHARD_K, 160, 250, K, 2, 40]
    for name in ("rows", "k"):
        for order in ([0, 1], [1, 0]):
            merged = pd.merge_shards([states[r][name] for r in order])
            assert torch.equal(merged["packed_w"], packed)
            assert float(merged["scale_buf"]) == np.float32(g) and int(merged["k_orig_buf"]) == K
            assert torch.equal(merged["bias"], bias)
        with pytest.raises(AssertionError):
            pd.merge_shards([states[0][name], states[0][name]])
        fast = pl.PentaLinearFast.from_state_dict(pd.merge_shards([s[name] for s in states]))
        assert torch.equal(fast.packed_w, packed) and fast.K_orig == K and fast.scale == float(np.float32(g))
    for r in range(world):
        d = np.load(tmp_path / f"s{r}.npz")
        assert d["refused"].all()
        assert float(d["scale"]) == float(np.float32(d["g"])) and bool(d["bias_ok"])


def _empty_slice_worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        N, K, M = 24, 80, 3
        w = gen_weight(N, K, seed=51).numpy()
        g = float(orc.absmean_scale(w))
        p = orc.quantize_pack(w, g)[0]
        dn = pd.RowShardedPentaLinear.from_full(torch.from_numpy(p), g, K, unit=40)
        if dn.K_local > 0:  # an empty slice keeps the layer's own zero partial
            dn.forward_local = lambda xl: torch.from_numpy(
                orc.matmul_f64(xl.float().numpy(), orc.unpack(dn.packed_w.numpy(), dn.K_local), g).astype(np.float32))
        x = gen_act(M, K, seed=52).float()
        y = dn(x).float().numpy()
        want = orc.bf16_linear_out(orc.matmul_f64(x.numpy(), orc.unpack(p, K), g).astype(np.float32))
        np.savez(os.path.join(out_dir, f"e{rank}.npz"), y=y, want=want, k_local=dn.K_local,
                 words=dn.packed_w.shape[1])
    finally:
        dist.destroy_process_group()


def test_row_parallel_empty_slice_gloo_world3(tmp_path):
    """A world larger than K's 40-column units leaves a rank without columns:
    it holds no words, contributes a zero partial, and every rank still gets
    the full product."""
    from _util import assert_bf16_close
    world = 3
    mp.start_processes(_empty_slice_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    ks = []
    for r in range(world):
        d = np.load(tmp_path / f"e{r}.npz")
        ks.append((int(d["k_local"]), int(d["words"])))
        assert_bf16_close(d["y"], d["want"].astype(np.float64), f"rank {r}")
    assert ks == [(40, 4), (40, 4), (0, 0)]
