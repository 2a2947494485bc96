"""Tensor-parallel pairing without the gather on the GPU: a column-parallel up
projection that keeps its output block on its rank (ShardedPentaLinear with
gather=False) feeding a row-parallel (K-split) down projection
(RowShardedPentaLinear) whose fp32 partial products meet in one all-reduce.

One GPU: the K splits of two and three ranks are emulated by summing the
per-slice partial products on the device, and a world of one runs the layers
end to end.  The two-GPU test (NCCL) runs when the box has two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from _util import assert_bf16_close, gen_act, gen_weight
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("M,N,K", [(1, 1024, 2816), (8, 768, 1000), (64, 512, 1376), (200, 256, 1040)])
def test_k_split_partials_one_gpu(cuda_device, M, N, K, world):
    """Summed fp32 partial products of the K slices, rounded the reference's
    way (bf16(acc * gamma), then + bf16(bias)), equal the oracle's unsplit
    product to within one bf16 ulp."""
    import penta_dist as pd
    import penta_kernel as pk
    w = gen_weight(N, K, seed=N + K + M)
    packed, _, gamma = pk.quantize_and_pack(w.to(cuda_device))
    bias = gen_weight(1, N, seed=M, std=0.5)[0]
    a = gen_act(M, K, seed=N).to(torch.bfloat16)
    a_dev = a.to(cuda_device)
    acc = torch.zeros(M, N, dtype=torch.float32, device=cuda_device)
    for r in range(world):
        local, lo, hi = pd.RowShardedPentaLinear.slice_k(packed, K, r, world)
        assert lo % 40 == 0 and (hi % 40 == 0 or hi == K)
        acc += pk.penta_linear(a_dev[:, lo:hi].contiguous(), local, gamma, hi - lo, out_dtype=torch.float32)
    yb = acc.to(torch.bfloat16)
    y = (yb.float() + bias.to(cuda_device).to(torch.bfloat16).float()).to(torch.bfloat16)
    pre = orc.matmul_f64(a.float().numpy(), orc.unpack(packed.cpu().numpy(), K), float(gamma))
    want = pre + bias.to(torch.bfloat16).float().numpy()[None, :]
    assert_bf16_close(y.float().cpu().numpy(), want, f"K split over {world}", pre_bias=pre)


def _pair_run(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    import penta_dist as pd
    import penta_kernel as pk
    try:
        D, H = 1024, 2816
        p_up, _, g_up = pk.quantize_and_pack(gen_weight(H, D, seed=31).to(dev))
        p_dn, _, g_dn = pk.quantize_and_pack(gen_weight(D, H, seed=32).to(dev))
        bias = gen_weight(1, D, seed=33, std=0.5)[0].to(dev)
        up = pd.ShardedPentaLinear.from_full(p_up, g_up, D, gather=False, unit=40)
        dn = pd.RowShardedPentaLinear.from_full(p_dn, g_dn, H, bias=bias, unit=40)
        lo, hi = pd.shard_range(H, rank, world, 40)
        res = {}
        for M in (1, 8, 64, 200):
            x = gen_act(M, D, seed=M).to(torch.bfloat16).to(dev)
            h_loc = up(x)
            a_loc = torch.nn.functional.gelu(h_loc)
            y = dn(a_loc, x_is_local=True)
            # the same activations gathered, through the unsharded product
            a_full = pd.gather_columns(a_loc, H, world, unit=40)
            y_dense = pk.penta_linear(a_full, p_dn, g_dn, H, bias=bias)
            pre = pk.penta_linear(a_full, p_dn, g_dn, H, out_dtype=torch.float32)
            h_dense = pk.penta_linear(x, p_up, g_up, D)[:, lo:hi]
            torch.cuda.synchronize()
            res[M] = dict(y=y.float().cpu().numpy(), y_dense=y_dense.float().cpu().numpy(),
                          pre=pre.cpu().numpy(), h=h_loc.float().cpu().numpy(), h_dense=h_dense.float().cpu().numpy(),
                          shape=tuple(h_loc.shape), K_local=dn.K_local, k0=dn.k0, lo=lo, hi=hi)
        np.save(os.path.join(out_dir, f"r{rank}.npy"), res, allow_pickle=True)
    finally:
        dist.destroy_process_group()


def _check(out_dir, world):
    from _util import bf16_ulp
    for r in range(world):
        res = np.load(os.path.join(out_dir, f"r{r}.npy"), allow_pickle=True).item()
        for M, d in res.items():
            assert d["k0"] == d["lo"] and d["K_local"] == d["hi"] - d["lo"] and d["shape"] == (M, d["K_local"])
            # fewer output rows change the up projection's k split: within one bf16 ulp
            err = np.abs(d["h"].astype(np.float64) - d["h_dense"])
            assert (err <= bf16_ulp(d["h_dense"]) + 1e-6).all(), f"rank {r} M={M}: up block off by {err.max():.3g}"
            # summed partials vs one unsplit product of the same activations
            bound = 2 * bf16_ulp(d["y_dense"]) + bf16_ulp(d["pre"]) + 1e-3
            err = np.abs(d["y"].astype(np.float64) - d["y_dense"])
            assert (err <= bound).all(), f"rank {r} M={M}: down projection off by {err.max():.3g}"


def test_pairing_world1(cuda_device, tmp_path):
    mp.start_processes(_pair_run, args=(1, _free_port(), str(tmp_path)), nprocs=1, start_method="spawn")
    _check(str(tmp_path), 1)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_pairing_world2(cuda_device, tmp_path):
    mp.start_processes(_pair_run, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    _check(str(tmp_path), 2)
