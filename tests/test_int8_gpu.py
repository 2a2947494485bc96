"""Per-token int8 activation quantiser and the int8 tensor-core GEMM against the
oracle: xq, s_x and int32 accumulators bit-exact (= torch._int_mm), outputs
exact to the reference's epilogue formula (penta_avx2_wrapper.py:147)."""
import os

import numpy as np
import pytest
import torch

from _util import assert_bf16_close, gen_act, gen_weight, golden
from oracle import oracle as orc
import penta_kernel as pk

pytestmark = pytest.mark.gpu
META, G = golden()


@pytest.mark.parametrize("name", [n for n in META["cases"] if n.startswith("int8.")])
def test_golden_int8_cases(cuda_device, name):
    c = META["cases"][name]
    x = gen_act(c["M"], c["K"], c["x_seed"]).to(cuda_device)
    xq, s_x, rowsum = pk.quantize_activations_i8(x)
    K = c["K"]
    assert np.array_equal(xq[:, :K].cpu().numpy(), G[f"{name}.xq"])
    assert not xq[:, K:].any()
    assert np.array_equal(s_x.cpu().numpy(), G[f"{name}.sx"])
    assert np.array_equal(rowsum.cpu().numpy(), G[f"{name}.xq"].astype(np.int64).sum(1))
    packed = torch.from_numpy(G[f"{name}.packed"]).to(cuda_device)
    y, acc = pk.penta_linear_i8_prequant(xq, s_x, rowsum, K, packed, c["scale"], out_dtype=torch.float32,
                                         return_acc=True)
    assert np.array_equal(acc.cpu().numpy(), G[f"{name}.acc"])
    assert np.array_equal(y.cpu().numpy(), G[f"{name}.y"])


@pytest.mark.parametrize("M,N,K", [
    (1, 128, 160), (16, 130, 770), (33, 257, 1001), (64, 384, 4096), (200, 256, 320), (256, 128, 3072),
    (257, 300, 1600), (512, 640, 4096),
])
def test_int8_gemm_exact(cuda_device, M, N, K):
    w = gen_weight(N, K, seed=M * 3 + N + K)
    packed, _, gamma = pk.quantize_and_pack(w.to(cuda_device))
    x = gen_act(M, K, seed=M + 5 * K).to(torch.bfloat16)
    y, acc = pk.penta_linear_i8(x.to(cuda_device), packed, gamma, K, out_dtype=torch.float32, return_acc=True)
    xq, sx = orc.quant_act_i8(x.float().numpy())
    w8 = orc.unpack(packed.cpu().numpy(), K)
    want_acc = orc.matmul_i8(xq, w8)
    assert np.array_equal(acc.cpu().numpy(), want_acc)
    assert np.array_equal(y.cpu().numpy(), orc.dequant_i8(want_acc, sx, gamma))
    yb = pk.penta_linear_i8(x.to(cuda_device), packed, gamma, K)
    assert np.array_equal(yb.float().cpu().numpy(), orc.to_bf16_f32(orc.dequant_i8(want_acc, sx, gamma)))


def test_int8_bias_and_zero_rows(cuda_device):
    N, K = 200, 512
    packed, _, gamma = pk.quantize_and_pack(gen_weight(N, K, seed=2).to(cuda_device))
    x = gen_act(6, K, seed=3)
    x[2] = 0
    bias = torch.randn(N, generator=torch.Generator().manual_seed(1))
    y = pk.penta_linear_i8(x.to(cuda_device), packed, gamma, K, bias.to(cuda_device), out_dtype=torch.float32)
    xq, sx = orc.quant_act_i8(x.numpy())
    assert sx[2] == 1.0
    acc = orc.matmul_i8(xq, orc.unpack(packed.cpu().numpy(), K))
    pre = orc.dequant_i8(acc, sx, gamma)
    want = pre + bias.to(torch.bfloat16).float().numpy()[None, :]
    assert np.array_equal(y.cpu().numpy(), want.astype(np.float32))
    yb = pk.penta_linear_i8(x.to(cuda_device), packed, gamma, K, bias.to(cuda_device))
    # exactly the reference's double rounding of the exact epilogue value
    assert np.array_equal(yb.float().cpu().numpy(), orc.bf16_linear_out(pre, bias.numpy()))
    assert_bf16_close(yb.float().cpu().numpy(), want, what="int8 bias bf16", pre_bias=pre)


@pytest.mark.parametrize("K,N", [(4096, 4096), (4096, 11008), (11008, 4096)])
def test_cfg3_full_size(cuda_device, K, N):
    """7B-class prefill shapes at M=4096: every int32 accumulator equal to the
    exact integer product (CPU torch._int_mm of the same int8 activations and
    unpacked weights, in row blocks; the int8 line's own arithmetic,
    penta_avx2_wrapper.py:130-131,147), the exact checksum of checksums
    (sum_n acc[m, n] = xq[m] . colsum(w)), and sampled outputs against the
    oracle's epilogue."""
    M = 4096
    packed, _, gamma = pk.quantize_and_pack(gen_weight(N, K, seed=K * 7 + N).to(cuda_device))
    x = gen_act(M, K, seed=N).to(torch.bfloat16).to(cuda_device)
    xq, s_x, rowsum = pk.quantize_activations_i8(x)
    y, acc = pk.penta_linear_i8_prequant(xq, s_x, rowsum, K, packed, gamma, out_dtype=torch.float32,
                                         return_acc=True)
    w8 = pk.unpack_weights_i8(packed, K)
    acc_c = acc.cpu()
    xq_c = xq[:, :K].cpu()
    wt_c = w8.cpu().t().contiguous()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for r0 in range(0, M, 1024):
        want = torch._int_mm(xq_c[r0:r0 + 1024].contiguous(), wt_c)
        assert torch.equal(acc_c[r0:r0 + 1024], want), f"int32 accumulators differ in rows {r0}..{r0 + 1023}"
    # float64 sums of these integers are exact (all partial sums < 2^53)
    xqd = xq[:, :K].double()
    w8d = w8.double()
    assert torch.equal(acc.double().sum(1), xqd @ w8d.sum(0))
    rows = torch.tensor([0, 1, 2047, M - 1])
    want = orc.matmul_i8(xq[rows, :K].cpu().numpy(), w8.cpu().numpy())
    assert np.array_equal(acc[rows].cpu().numpy(), want)
    assert np.array_equal(y[rows].cpu().numpy(), orc.dequant_i8(want, s_x[rows].cpu().numpy(), gamma))


@pytest.mark.parametrize("M,N,K", [(1, 384, 28672), (100, 1000, 3072), (300, 640, 1600)])
def test_int8_split_and_whole_tile_schedules(cuda_device, M, N, K):
    """The recommended workspace (split K ranges, partial sums) and the minimum
    one (whole tiles per SM) give the same exact int32 accumulators."""
    import ctypes
    import penta_native as nat
    L = nat.load()
    packed, _, gamma = pk.quantize_and_pack(gen_weight(N, K, seed=M + N + K).to(cuda_device))
    x = gen_act(M, K, seed=K + 1).to(torch.bfloat16)
    xq, s_x, rowsum = pk.quantize_activations_i8(x.to(cuda_device))
    want = orc.matmul_i8(orc.quant_act_i8(x.float().numpy())[0], orc.unpack(packed.cpu().numpy(), K))
    for nbytes in (L.pn_linear_workspace_size(nat.PN_I8, M, N, K), L.pn_linear_workspace_min_size(nat.PN_I8, M, N, K)):
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=cuda_device)
        acc = torch.empty(M, N, dtype=torch.int32, device=cuda_device)
        st = L.pn_linear_i8(xq.data_ptr(), xq.shape[1], s_x.data_ptr(), rowsum.data_ptr(), M, K, packed.data_ptr(),
                            N, packed.shape[1], ctypes.c_float(gamma), None, None, nat.PN_F32, acc.data_ptr(),
                            ws.data_ptr(), nbytes, nat.stream_of(xq))
        assert st == nat.PN_OK, L.pn_last_error()
        assert np.array_equal(acc.cpu().numpy(), want), f"workspace {nbytes}"


@pytest.mark.parametrize("K", [8, 16, 96, 768, 1000, 2048, 3072, 4096, 8192, 11008, 28672, 40000])
@pytest.mark.parametrize("M", [1, 7, 33])
def test_quantiser_all_row_lengths(cuda_device, M, K):
    """Every threads-per-token variant of the vectorised quantiser (rows of 8
    to 32768), the scalar kernel (K % 8 != 0, longer rows) and exact
    half-integer quotients (rounded half to even, as the reference's division
    then round)."""
    x = gen_act(M, K, seed=M * 7 + K)
    x[0, :4] = torch.tensor([3.0, -7.5, 4.5, 0.5])   # with s = 3: x / s = 1, -2.5, 1.5, 1/6
    x[0, 4] = 381.0                                   # s = 3 exactly
    if M > 1:
        x[1] = 0                                      # all-zero row: s = 1
    x = x.to(torch.bfloat16)
    xq, s_x, rowsum = pk.quantize_activations_i8(x.to(cuda_device))
    want_q, want_s = orc.quant_act_i8(x.float().numpy())
    assert np.array_equal(xq[:, :K].cpu().numpy(), want_q)
    assert not xq[:, K:].any()
    assert np.array_equal(s_x.cpu().numpy(), want_s)
    assert np.array_equal(rowsum.cpu().numpy(), want_q.astype(np.int64).sum(1))
