"""Output-sharded layers with the outputs stored into every GPU's buffer by
the GEMM epilogue (CUDA IPC peer mappings) and the cross-GPU barrier kernel.

A world of one (process group over gloo) runs on any single B200; the
two-GPU test spawns one process per GPU when the box has two or more."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from _util import bf16_ulp, gen_act, gen_weight

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, port, out_dir, cases):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import penta_dist as pd
    import penta_kernel as pk
    import penta_native as nat
    try:
        dev = torch.device("cuda", rank)
        peers = pd.PeerGroup()
        res = {}
        for (M, N, K) in cases:
            w = gen_weight(N, K, seed=N + K).to(dev)
            packed, _, g = pk.quantize_and_pack(w)
            x = gen_act(M, K, seed=M + 1).to(torch.bfloat16).to(dev)
            want = pk.penta_linear(x, packed, g, K)  # unsharded, this GPU
            layer = pd.ShardedPentaLinear.from_full(packed, g, K, peers=peers, max_tokens=64)
            ys = [layer(x).clone() for _ in range(3)]  # repeated calls reuse buffer and barrier
            torch.cuda.synchronize()
            res[f"{M}x{N}x{K}"] = (ys[0].float().cpu().numpy(), want.float().cpu().numpy(),
                                   all(torch.equal(y, ys[0]) for y in ys))
        res["status"] = nat.device_status(reset=True)
        peers.close()
        np.save(os.path.join(out_dir, f"r{rank}.npy"), res, allow_pickle=True)
    finally:
        dist.destroy_process_group()


CASES = [(1, 1024, 3072), (8, 4096, 8192), (64, 768, 4096)]


def _check(out_dir, world):
    for r in range(world):
        res = np.load(os.path.join(out_dir, f"r{r}.npy"), allow_pickle=True).item()
        assert res.pop("status") == 0
        for name, (y, want, same) in res.items():
            assert same, f"rank {r} {name}: repeated calls differ"
            # sharding changes the k-split of tiles, hence the fp32 summation
            # order: the bf16 outputs agree to within one bf16 ulp
            err = np.abs(y.astype(np.float64) - want)
            assert (err <= bf16_ulp(want) + 1e-6).all(), f"rank {r} {name}: max err {err.max():.3g}"


def test_peer_outputs_world1(cuda_device, tmp_path):
    mp.start_processes(_run, args=(1, _free_port(), str(tmp_path), CASES), nprocs=1, start_method="spawn")
    _check(str(tmp_path), 1)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_outputs_world2(cuda_device, tmp_path):
    mp.start_processes(_run, args=(2, _free_port(), str(tmp_path), CASES), nprocs=2, start_method="spawn")
    _check(str(tmp_path), 2)


@pytest.mark.parametrize("M,N,K", [(1, 300, 1000), (16, 256, 4096), (64, 384, 3072), (200, 256, 1600)])
def test_two_outputs_one_gpu(cuda_device, M, N, K):
    """The multi-output epilogue on one GPU: the shard's columns stored into two
    local buffers (row stride ld > N, first column col0) equal the plain product,
    and nothing outside the shard's columns is written."""
    import ctypes
    import penta_kernel as pk
    import penta_native as nat
    import penta_dist as pd
    packed, _, gamma = pk.quantize_and_pack(gen_weight(N, K, seed=M + K).to(cuda_device))
    x = gen_act(M, K, seed=N).to(torch.bfloat16).to(cuda_device)
    want = pk.penta_linear(x, packed, gamma, K)
    ld, col0 = N + 24, 16
    bufs = [torch.full((M, ld), 7.0, dtype=torch.bfloat16, device=cuda_device) for _ in range(2)]
    for _ in range(2):  # two calls in a row
        pd.linear_peers(x, packed, gamma, K, col0, [b.data_ptr() for b in bufs], ld)
        torch.cuda.synchronize()
        for b in bufs:
            assert torch.equal(b[:, col0:col0 + N], want)
            assert bool((b[:, :col0] == 7.0).all()) and bool((b[:, col0 + N:] == 7.0).all())
    assert nat.device_status() == 0
