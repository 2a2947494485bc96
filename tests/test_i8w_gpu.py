"""pn_matmul_i8w: the reference's CPU matmul ABI (penta_matmul_avx2, fp32 x
times unpacked int8 weights) on the GPU, against the oracle and the
reference's own AVX2 output.

Tolerance: fp32 outputs within rel 1e-3 / abs 1e-3 of the oracle's float64
product (the contract of the reference's paths)."""
import ctypes

import numpy as np
import pytest
import torch

from _util import assert_close, gen_act, gen_weight, golden
from oracle import oracle as orc
import penta_avx2_wrapper as avx
import penta_kernel as pk
import penta_native as nat

pytestmark = pytest.mark.gpu
META, G = golden()


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (8, 3072, 768), (3, 257, 1001), (16, 640, 4096), (5, 33, 30),
                                   (17, 100, 160), (64, 128, 3072), (2, 1000, 13)])
def test_matmul_i8w(cuda_device, M, N, K):
    w = gen_weight(N, K, seed=N + K)
    packed, _, gamma = pk.quantize_and_pack(w.to(cuda_device))
    w8 = pk.unpack_weights_i8(packed, K)
    x = gen_act(M, K, seed=M * 7 + K)
    y = pk.penta_linear_i8w(x.to(cuda_device), w8, gamma)
    assert y.dtype == torch.float32 and y.shape == (M, N)
    assert_close(y.cpu().numpy(), orc.matmul_f64(x.numpy(), w8.cpu().numpy(), gamma), what=f"i8w M={M} N={N} K={K}")


def test_reference_module_names_and_avx2_golden(cuda_device):
    """penta_avx2_wrapper's two functions, as the reference's benchmark calls
    them, against the reference's own AVX2 output for configs[0]."""
    c = META["cases"]["cfg0"]
    w = gen_weight(3072, 768, seed=0)
    packed, K, gamma = pk.quantize_and_pack(w.to(cuda_device))
    w8 = avx.penta_unpack(packed, K)
    assert w8.dtype == torch.int8 and w8.shape == (3072, 768)
    x = gen_act(8, 768, c["x_seed"])
    bias = torch.randn(3072, generator=torch.Generator().manual_seed(3))
    y = avx.penta_linear_avx2(x.to(cuda_device), w8, gamma)
    assert_close(y.cpu().numpy(), G["cfg0.y_avx2"], what="vs the reference AVX2 output")
    yb = avx.penta_linear_avx2(x.to(cuda_device), w8, gamma, bias.to(cuda_device))
    assert_close(yb.cpu().numpy(), G["cfg0.y_avx2"] + bias.numpy()[None, :], what="with bias")


def test_matmul_i8w_abi_errors(cuda_device):
    L = nat.load()
    x = torch.zeros(2, 8, device=cuda_device)
    w = torch.zeros(4, 8, dtype=torch.int8, device=cuda_device)
    y = torch.empty(2, 4, device=cuda_device)
    s = nat.stream_of(x)
    assert L.pn_matmul_i8w(x.data_ptr(), w.data_ptr(), y.data_ptr(), 2, 4, 8, ctypes.c_float(1.0), s) == nat.PN_OK
    assert L.pn_matmul_i8w(x.data_ptr(), w.data_ptr(), y.data_ptr(), -1, 4, 8, ctypes.c_float(1.0), s) == nat.PN_ERR_SHAPE
    assert L.pn_matmul_i8w(None, w.data_ptr(), y.data_ptr(), 2, 4, 8, ctypes.c_float(1.0), s) == nat.PN_ERR_ARG
    assert L.pn_matmul_i8w(x.data_ptr() + 2, w.data_ptr(), y.data_ptr(), 2, 4, 8, ctypes.c_float(1.0), s) == nat.PN_ERR_ALIGN
    # K = 0: zeros
    assert L.pn_matmul_i8w(x.data_ptr(), w.data_ptr(), y.data_ptr(), 2, 4, 0, ctypes.c_float(1.0), s) == nat.PN_OK
    torch.cuda.synchronize()
    assert torch.count_nonzero(y) == 0
    with pytest.raises(AssertionError):
        pk.penta_linear_i8w(x, w[:, :4], 1.0)
