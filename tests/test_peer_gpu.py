"""Output-sharded layers with the outputs stored into every GPU's buffer by
the GEMM epilogue (CUDA IPC peer mappings) and the cross-GPU barrier kernel.

A world of one (process group over gloo) runs on any single B200; the
multi-GPU tests spawn one process per GPU (2, 4 or 8) when the box has that
many, on the CPU-seeded small cases and on the 70B-class decode layers
(8192->28672 and 28672->8192 at M = 1, 8, 64), each rank checking the full
output assembled by the peer stores against the unsharded product.

The barrier's failure detection is exercised without any GPU fault: a
bounded wait on a flag that nothing sets runs out (one GPU), and a rank that
skips one barrier makes the other rank's wait run out (two GPUs); both
recover through PeerGroup.reset()."""
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


BIG = [(1, 28672, 8192), (8, 28672, 8192), (64, 28672, 8192), (1, 8192, 28672), (8, 8192, 28672),
       (64, 8192, 28672)]


def _big_inputs(M, N, K, dev):
    """70B-class layer and activations from a device generator (same values on
    every rank)."""
    g = torch.Generator(device=dev).manual_seed(N * 7 + K)
    w = torch.randn(N, K, device=dev, generator=g) * 0.02
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    return w, x


def _run(rank, world, port, out_dir, cases, big=()):
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
        for (M, N, K) in big:
            w, x = _big_inputs(M, N, K, dev)
            packed, _, g = pk.quantize_and_pack(w)
            del w
            want = pk.penta_linear(x, packed, g, K)
            layer = pd.ShardedPentaLinear.from_full(packed, g, K, peers=peers, max_tokens=64)
            ys = [layer(x).clone() for _ in range(2)]
            torch.cuda.synchronize()
            res[f"big{M}x{N}x{K}"] = (ys[0].float().cpu().numpy(), want.float().cpu().numpy(),
                                      torch.equal(ys[0], ys[1]))
            del packed, layer
            torch.cuda.empty_cache()
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


def test_peer_outputs_world1_70b(cuda_device, tmp_path):
    mp.start_processes(_run, args=(1, _free_port(), str(tmp_path), [], BIG[:3]), nprocs=1, start_method="spawn")
    _check(str(tmp_path), 1)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_outputs_multi_gpu(cuda_device, tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_run, args=(world, _free_port(), str(tmp_path), CASES, BIG), nprocs=world,
                       start_method="spawn")
    _check(str(tmp_path), world)


def test_barrier_wait_runs_out(cuda_device):
    """A bounded wait on a flag that nothing sets: a world-2 barrier on one GPU
    with both flag arrays local and rank 1 never arriving.  The kernel gives
    up after 20 ms, records PN_ERR_TIMEOUT and returns; the context stays
    usable, and after zeroing the flags and generation (what PeerGroup.reset
    does on every rank) a barrier completes again."""
    import ctypes
    import penta_kernel as pk
    import penta_native as nat
    L = nat.load()
    flags = [torch.zeros(2, dtype=torch.int32, device=cuda_device) for _ in range(2)]
    gen = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    arr = (ctypes.c_void_p * 2)(*[f.data_ptr() for f in flags])
    assert nat.device_status(reset=True) == 0
    s = torch.cuda.current_stream().cuda_stream
    nat.check(L.pn_peer_barrier_wait(arr, 2, 0, gen.data_ptr(), 20_000_000, s), "pn_peer_barrier_wait")
    assert nat.device_status(reset=True) == nat.PN_ERR_TIMEOUT
    # rank 0 posted generation 1 into both arrays before it waited
    assert flags[0].tolist() == [1, 0] and flags[1].tolist() == [1, 0] and gen.item() == 1
    # the context is intact: a product still matches
    w = gen_weight(256, 640, seed=3).to(cuda_device)
    x = gen_act(4, 640, seed=4).to(torch.bfloat16).to(cuda_device)
    packed, _, g = pk.quantize_and_pack(w)
    y = pk.penta_linear(x, packed, g, 640)
    assert torch.isfinite(y.float()).all()
    # reset, then a barrier whose every rank arrives (world 1) completes
    for f in flags:
        f.zero_()
    gen.zero_()
    arr1 = (ctypes.c_void_p * 1)(flags[0].data_ptr())
    nat.check(L.pn_peer_barrier_wait(arr1, 1, 0, gen.data_ptr(), 20_000_000, s), "pn_peer_barrier_wait")
    assert nat.device_status(reset=True) == 0 and gen.item() == 1 and flags[0][0].item() == 1
    assert L.pn_peer_barrier_wait(arr1, 1, 0, gen.data_ptr(), -1, s) == nat.PN_ERR_ARG


def _skip_run(rank, world, port, out_dir):
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
        M, N, K = 8, 4096, 8192
        w = gen_weight(N, K, seed=5).to(dev)
        packed, _, g = pk.quantize_and_pack(w)
        x = gen_act(M, K, seed=6).to(torch.bfloat16).to(dev)
        want = pk.penta_linear(x, packed, g, K)
        layer = pd.ShardedPentaLinear.from_full(packed, g, K, peers=peers, max_tokens=64)
        y0 = layer(x).clone()
        torch.cuda.synchronize()
        # the failure, made on the host: rank 1 skips one barrier, so rank 0's
        # wait (50 ms) runs out; nothing is in flight on rank 1 meanwhile
        if rank == 0:
            peers.barrier(wait_ns=50_000_000)
        st_fail = nat.device_status(reset=True)
        peers.reset()
        y1 = layer(x).clone()
        torch.cuda.synchronize()
        st_after = nat.device_status(reset=True)
        np.save(os.path.join(out_dir, f"r{rank}.npy"),
                {"st_fail": st_fail, "st_after": st_after, "y0": y0.float().cpu().numpy(),
                 "y1": y1.float().cpu().numpy(), "want": want.float().cpu().numpy()}, allow_pickle=True)
        peers.close()
    finally:
        dist.destroy_process_group()


def test_barrier_skipped_rank_world2(cuda_device, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import penta_native as nat
    mp.start_processes(_skip_run, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    for r in range(2):
        d = np.load(os.path.join(str(tmp_path), f"r{r}.npy"), allow_pickle=True).item()
        assert d["st_fail"] == (nat.PN_ERR_TIMEOUT if r == 0 else 0), (r, d["st_fail"])
        assert d["st_after"] == 0
        for y in (d["y0"], d["y1"]):
            err = np.abs(y.astype(np.float64) - d["want"])
            assert (err <= bf16_ulp(d["want"]) + 1e-6).all(), f"rank {r}: max err {err.max():.3g}"


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
