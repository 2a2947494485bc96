"""penta_linear (bf16 activations, kind::f16 tensor-core path and the CUDA-core
path for unaligned K) against the oracle and the reference's golden outputs.

Tolerance (written here as the contract): fp32 outputs within rel 1e-3 / abs
1e-3 of the oracle after scaling; bf16 outputs within one bf16 ulp (+ abs 1e-3)
of the exact value, since bf16 rounding itself is coarser than rel 1e-3."""
import numpy as np
import pytest
import torch

from _util import assert_bf16_close, assert_close, gen_act, gen_weight, golden
from oracle import oracle as orc
import penta_kernel as pk

pytestmark = pytest.mark.gpu
META, G = golden()


def _layer(N, K, seed, dev, std=0.02):
    w = gen_weight(N, K, seed, std)
    packed, _, gamma = pk.quantize_and_pack(w.to(dev))
    w8 = orc.unpack(packed.cpu().numpy(), K)
    return packed, gamma, w8


def _check(x_bf16, packed, gamma, w8, K, bias=None, what=""):
    """Run fp32-out and bf16-out through the C ABI and compare to the oracle."""
    xf = x_bf16.float().cpu().numpy()
    pre = orc.matmul_f64(xf, w8, gamma)
    want = pre
    if bias is not None:
        want = pre + bias.to(torch.bfloat16).float().cpu().numpy()[None, :]
    y32 = pk.penta_linear(x_bf16, packed, gamma, K, bias, out_dtype=torch.float32)
    assert y32.dtype == torch.float32
    assert_close(y32.cpu().numpy(), want, what=what + " fp32")
    y16 = pk.penta_linear(x_bf16, packed, gamma, K, bias)
    assert y16.dtype == torch.bfloat16
    assert_bf16_close(y16.float().cpu().numpy(), want, what=what + " bf16",
                      pre_bias=None if bias is None else pre)
    if bias is None:
        # bf16 output = bf16(acc * scale) of the same accumulator (penta_kernel.py:224)
        assert np.array_equal(y16.float().cpu().numpy(), orc.to_bf16_f32(y32.cpu().numpy()))
    return y32


@pytest.mark.parametrize("shape", [(768, 2304), (768, 768), (768, 3072), (3072, 768)])
@pytest.mark.parametrize("M", [1, 4, 16])
def test_cfg1_decode_sweep(cuda_device, shape, M):
    K, N = shape
    name = f"cfg1.{K}x{N}"
    c = META["cases"][name]
    packed, gamma, w8 = _layer(N, K, c["w_seed"], cuda_device)
    x = gen_act(M, K, c[f"M{M}_x_seed"]).to(torch.bfloat16).to(cuda_device)
    y32 = _check(x, packed, gamma, w8, K, what=f"{name} M={M}")
    # the reference's own CPU kernel output (numba, penta_kernel_cpu.py)
    assert_close(y32.cpu().numpy(), G[f"{name}.M{M}.y_numba"], what=f"{name} M={M} vs numba")


def test_cfg0_shape(cuda_device):
    c = META["cases"]["cfg0"]
    packed, gamma, w8 = _layer(3072, 768, 0, cuda_device)
    x = gen_act(8, 768, c["x_seed"])
    xb = x.to(torch.bfloat16).to(cuda_device)
    _check(xb, packed, gamma, w8, 768, what="cfg0")
    # fp32 activations rounded to bf16 stay within the bar of the fp32 reference on this data
    y = pk.penta_linear(xb, packed, gamma, 768, out_dtype=torch.float32).cpu().numpy()
    assert np.abs(y - G["cfg0.y_numba"]).max() < 0.05


@pytest.mark.parametrize("M,N,K", [
    (1, 1, 16), (2, 130, 160), (3, 257, 1000), (17, 128, 320), (33, 200, 776), (64, 384, 1600),
    (65, 128, 480), (100, 300, 2048), (129, 256, 640), (256, 130, 800), (300, 512, 3072), (1000, 260, 768),
])
def test_tensor_core_shapes(cuda_device, M, N, K):
    packed, gamma, w8 = _layer(N, K, seed=M + N + K, dev=cuda_device, std=0.05)
    x = gen_act(M, K, seed=7 * M + K).to(torch.bfloat16).to(cuda_device)
    _check(x, packed, gamma, w8, K, what=f"M={M} N={N} K={K}")


@pytest.mark.parametrize("M,N,K", [(1, 5, 7), (3, 17, 13), (16, 40, 770), (5, 64, 1001), (40, 33, 10),
                                   (100, 20, 13), (70, 8, 1001)])
def test_unaligned_k(cuda_device, M, N, K):
    """K not a multiple of 8: decode tiles (M <= 64) re-lay the activations with
    plain loads; larger M takes the CUDA-core kernel."""
    packed, gamma, w8 = _layer(N, K, seed=N * K, dev=cuda_device, std=0.05)
    x = gen_act(M, K, seed=M * K).to(torch.bfloat16).to(cuda_device)
    _check(x, packed, gamma, w8, K, what=f"simt M={M} N={N} K={K}")


def test_bias_and_batch_dims(cuda_device):
    N, K = 300, 768
    packed, gamma, w8 = _layer(N, K, seed=3, dev=cuda_device)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(9)).to(cuda_device)
    x = gen_act(2 * 5, K, seed=4).to(torch.bfloat16).to(cuda_device).reshape(2, 5, K)
    y = pk.penta_linear(x, packed, gamma, K, bias)
    assert y.shape == (2, 5, N)
    _check(x.reshape(10, K), packed, gamma, w8, K, bias=bias, what="bias")


def test_small_golden_outputs(cuda_device):
    for name in [n for n in META["cases"] if n.startswith("small.")]:
        c = META["cases"][name]
        packed = torch.from_numpy(G[f"{name}.packed"]).to(cuda_device)
        x = gen_act(3, c["K"], c["x_seed"])
        y = pk.penta_linear(x.to(torch.bfloat16).to(cuda_device), packed, c["scale"], c["K"],
                            out_dtype=torch.float32).cpu().numpy()
        w8 = orc.unpack(G[f"{name}.packed"], c["K"])
        assert_close(y, orc.matmul_f64(x.to(torch.bfloat16).float().numpy(), w8, c["scale"]), what=name)


def test_zero_and_empty(cuda_device):
    packed, gamma, w8 = _layer(64, 160, seed=1, dev=cuda_device)
    x = torch.zeros(5, 160, dtype=torch.bfloat16, device=cuda_device)
    assert torch.count_nonzero(pk.penta_linear(x, packed, gamma, 160)) == 0
    y = pk.penta_linear(torch.zeros(0, 160, dtype=torch.bfloat16, device=cuda_device), packed, gamma, 160)
    assert y.shape == (0, 64)


def test_errors_like_reference(cuda_device):
    packed, gamma, _ = _layer(8, 40, seed=1, dev=cuda_device)
    with pytest.raises(AssertionError, match="bfloat16"):
        pk.penta_linear(torch.zeros(2, 40, device=cuda_device), packed, gamma, 40)
    with pytest.raises(AssertionError, match="K_orig"):
        pk.penta_linear(torch.zeros(2, 30, dtype=torch.bfloat16, device=cuda_device), packed, gamma, 40)


@pytest.mark.parametrize("K,N", [(8192, 28672), (28672, 8192)])
def test_cfg4_full_size(cuda_device, K, N):
    """70B-class decode shapes at full size, M = 1, 8, 64: every output (fp32
    and bf16) against the oracle's float64 product of the unpacked weights,
    plus two size-independent properties: exact linearity under x -> 2x and a
    checksum of checksums (sum over n of y[m, n] = x[m] . colsum(w))."""
    packed, gamma, _ = _layer(N, K, seed=K + N, dev=cuda_device)
    w8 = pk.unpack_weights_i8(packed, K)
    w8_np = w8.cpu().numpy()
    colsum = w8.to(torch.float64).sum(0)
    for M in (1, 8, 64):
        x = gen_act(M, K, seed=K + M).to(torch.bfloat16).to(cuda_device)
        want = orc.matmul_f64(x.float().cpu().numpy(), w8_np, gamma)
        y = pk.penta_linear(x, packed, gamma, K, out_dtype=torch.float32)
        assert_close(y.cpu().numpy(), want, what=f"cfg4 {K}->{N} M={M} fp32")
        yb = pk.penta_linear(x, packed, gamma, K)
        assert_bf16_close(yb.float().cpu().numpy(), want, what=f"cfg4 {K}->{N} M={M} bf16")
        yd = y.double()
        y2 = pk.penta_linear(x * 2, packed, gamma, K, out_dtype=torch.float32).double()
        assert torch.equal(y2, 2 * yd)
        got = yd.sum(1)
        ref = (x.double() @ colsum) * gamma
        assert torch.allclose(got, ref, rtol=1e-6, atol=1e-3 * N ** 0.5)


def test_no_device_timeouts(cuda_device):
    import penta_native as nat
    assert nat.device_status(reset=True) == 0


@pytest.mark.parametrize("M,N,K", [(1, 1024, 8192), (16, 640, 3072), (64, 512, 4096), (300, 512, 3072),
                                   (1000, 260, 768)])
def test_repeat_calls_bit_identical(cuda_device, M, N, K):
    """Ring-slot reuse stress: many repeated launches over several tiles must
    give bit-identical results (a stale-phase race would perturb them)."""
    packed, gamma, w8 = _layer(N, K, seed=N + K, dev=cuda_device)
    x = gen_act(M, K, seed=M).to(torch.bfloat16).to(cuda_device)
    first = pk.penta_linear(x, packed, gamma, K, out_dtype=torch.float32)
    for _ in range(8):
        assert torch.equal(pk.penta_linear(x, packed, gamma, K, out_dtype=torch.float32), first)
    xf = x.float().cpu().numpy()
    rows = [0, N // 2, N - 1]
    assert_close(first[:, rows].cpu().numpy(), orc.matmul_f64(xf, w8[rows], gamma), what="repeat")


@pytest.mark.parametrize("M,N,K", [(1, 384, 28672), (7, 8192, 3072), (64, 200, 8192), (200, 300, 1536),
                                   (33, 1000, 1001)])
def test_split_and_whole_tile_schedules(cuda_device, M, N, K):
    """With the recommended workspace the kernel splits tiles' K ranges over
    SMs (partial sums reduced by the last arriving CTA); with the minimum it
    gives each SM whole tiles.  Both must match the oracle and be repeatable."""
    import ctypes
    import penta_native as nat
    L = nat.load()
    packed, gamma, w8 = _layer(N, K, seed=N + 3 * K, dev=cuda_device)
    x = gen_act(M, K, seed=M + 7).to(torch.bfloat16).to(cuda_device)
    KP = packed.shape[1]
    full = L.pn_linear_workspace_size(nat.PN_BF16, M, N, K)
    least = L.pn_linear_workspace_min_size(nat.PN_BF16, M, N, K)
    assert 0 <= least <= full
    want = orc.matmul_f64(x.float().cpu().numpy(), w8, gamma)
    outs = []
    for nbytes in (full, least):
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=cuda_device)
        runs = []
        for _ in range(3):
            y = torch.empty(M, N, dtype=torch.float32, device=cuda_device)
            st = L.pn_linear_bf16(x.data_ptr(), M, K, packed.data_ptr(), N, KP, ctypes.c_float(gamma), None,
                                  y.data_ptr(), nat.PN_F32, ws.data_ptr(), nbytes, nat.stream_of(x))
            assert st == nat.PN_OK, L.pn_last_error()
            runs.append(y)
        torch.cuda.synchronize()
        assert all(torch.equal(r, runs[0]) for r in runs[1:]), f"workspace {nbytes}: repeat calls differ"
        assert_close(runs[0].cpu().numpy(), want, what=f"M={M} N={N} K={K} workspace {nbytes}")
        outs.append(runs[0])
    if least < full:
        # one byte short of the minimum is refused
        ws = torch.empty(max(least, 1), dtype=torch.uint8, device=cuda_device)
        y = torch.empty(M, N, dtype=torch.float32, device=cuda_device)
        if least > 0:
            st = L.pn_linear_bf16(x.data_ptr(), M, K, packed.data_ptr(), N, KP, ctypes.c_float(gamma), None,
                                  y.data_ptr(), nat.PN_F32, ws.data_ptr(), least - 1, nat.stream_of(x))
            assert st == nat.PN_ERR_WORKSPACE
    assert nat.device_status(reset=True) == 0


@pytest.mark.parametrize("M,N,K", [(1, 300, 770), (16, 256, 4096), (200, 384, 1001), (300, 256, 4096)])
def test_padded_row_stride(cuda_device, M, N, K):
    """Weights stored at a 16-byte row stride (pad_packed, the resident layout
    of PentaLinearFast) give the same bits as the contiguous tensor, which is
    re-pitched per call; any other stride is accepted too."""
    packed, gamma, w8 = _layer(N, K, seed=M + N, dev=cuda_device)
    x = gen_act(M, K, seed=K + 1).to(torch.bfloat16).to(cuda_device)
    padded = pk.pad_packed(packed)
    assert padded.shape == packed.shape and torch.equal(padded, packed)
    assert padded.stride(0) == pk.packed_ld(packed.shape[1]) and padded.stride(0) % 4 == 0
    assert pk.pad_packed(padded) is padded
    wide = torch.zeros(N, packed.shape[1] + 5, dtype=torch.int32, device=cuda_device)
    wide[:, :packed.shape[1]] = packed
    ref = pk.penta_linear(x, packed, gamma, K, out_dtype=torch.float32)
    for pw in (padded, wide[:, :packed.shape[1]]):
        assert torch.equal(pk.penta_linear(x, pw, gamma, K, out_dtype=torch.float32), ref)
        y8, acc8 = pk.penta_linear_i8(x, pw, gamma, K, out_dtype=torch.float32, return_acc=True)
        y8c, acc8c = pk.penta_linear_i8(x, packed, gamma, K, out_dtype=torch.float32, return_acc=True)
        assert torch.equal(acc8, acc8c) and torch.equal(y8, y8c)
    _check(x, padded, gamma, w8, K, what="padded")


@pytest.mark.parametrize("M,N,K", [(1, 200, 10), (2, 300, 170), (5, 256, 1600), (8, 384, 8192), (1, 640, 28672),
                                   (3, 130, 31999), (8, 128, 9984)])
def test_resident_activation_decode(cuda_device, M, N, K):
    """Decode products of at most 8 tokens whose activations fit in shared
    memory keep them resident for the launch (compact unswizzled image); the
    larger shapes here fall back to the streamed slabs."""
    packed, gamma, w8 = _layer(N, K, seed=K + M, dev=cuda_device)
    x = gen_act(M, K, seed=N + 3).to(torch.bfloat16).to(cuda_device)
    _check(x, packed, gamma, w8, K, what=f"resident M={M} K={K}")
    _check(x, pk.pad_packed(packed), gamma, w8, K, what=f"resident padded M={M} K={K}")
