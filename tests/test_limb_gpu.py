"""The limb decode kernel (bf16 products of at most 16 tokens on kind::i8
tensor cores: activations as four int8 limbs of a per-token 32-bit
fixed-point integer, weights as shifted codes) and the kind::f16 decode kernel
beside it, both against the oracle.

Tolerance (the contract of penta_linear): fp32 outputs within rel 1e-3 /
abs 1e-3 of the oracle's float64 product; bf16 outputs within one bf16 ulp
(+ abs 1e-3).  The limb path rounds each activation to a multiple of
2^-25 max|x| of its token, far inside that bar."""
import ctypes

import numpy as np
import pytest
import torch

from _util import assert_bf16_close, assert_close, gen_act, gen_weight
from oracle import oracle as orc
import penta_kernel as pk
import penta_native as nat

pytestmark = pytest.mark.gpu


@pytest.fixture
def limb_limit():
    """Restores the process-wide limb-path limit after the test."""
    L = nat.load()
    prev = L.pn_set_limb_max_tokens(-1)
    yield L
    L.pn_set_limb_max_tokens(prev)


def _layer(N, K, seed, dev, std=0.02):
    w = gen_weight(N, K, seed, std)
    packed, _, gamma = pk.quantize_and_pack(w.to(dev))
    return packed, gamma, orc.unpack(packed.cpu().numpy(), K)


def _check(x, packed, gamma, w8, K, what):
    want = orc.matmul_f64(x.float().cpu().numpy(), w8, gamma)
    y32 = pk.penta_linear(x, packed, gamma, K, out_dtype=torch.float32)
    assert_close(y32.cpu().numpy(), want, what=what + " fp32")
    y16 = pk.penta_linear(x, packed, gamma, K)
    assert_bf16_close(y16.float().cpu().numpy(), want, what=what + " bf16")
    # bf16 output = bf16 rounding of the same fp32 value
    assert np.array_equal(y16.float().cpu().numpy(), orc.to_bf16_f32(y32.cpu().numpy()))
    return y32


SHAPES = [(1, 300, 770), (2, 130, 160), (3, 257, 1000), (4, 1024, 8192), (5, 64, 1001), (8, 384, 8192),
          (9, 200, 3072), (16, 640, 4096), (1, 384, 28672), (8, 256, 28672), (16, 130, 31999), (7, 1, 16)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_limb_path(cuda_device, limb_limit, M, N, K):
    limb_limit.pn_set_limb_max_tokens(16)
    packed, gamma, w8 = _layer(N, K, seed=M * 31 + N + K, dev=cuda_device)
    x = gen_act(M, K, seed=N + 5 * M).to(torch.bfloat16).to(cuda_device)
    y = _check(x, packed, gamma, w8, K, what=f"limb M={M} N={N} K={K}")
    # repeat calls are bit-identical (integer sums, fixed-order corrections)
    assert torch.equal(pk.penta_linear(x, packed, gamma, K, out_dtype=torch.float32), y)
    # the padded resident stride gives the same bits
    assert torch.equal(pk.penta_linear(x, pk.pad_packed(packed), gamma, K, out_dtype=torch.float32), y)


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_f16_decode_path(cuda_device, limb_limit, M, N, K):
    """With the limb path off, the same batches run on the kind::f16 decode
    kernel (bf16 codes and activations, fp32 accumulation)."""
    limb_limit.pn_set_limb_max_tokens(0)
    packed, gamma, w8 = _layer(N, K, seed=M * 31 + N + K, dev=cuda_device)
    x = gen_act(M, K, seed=N + 5 * M).to(torch.bfloat16).to(cuda_device)
    _check(x, packed, gamma, w8, K, what=f"f16 M={M} N={N} K={K}")


@pytest.mark.parametrize("scale", [2.0 ** 100, 2.0 ** -100, 2.0 ** -126])
def test_limb_extreme_scales(cuda_device, limb_limit, scale):
    """Activations far from 1 in magnitude: the per-token exponent follows
    them (no overflow of the limbs, no loss from underflow)."""
    limb_limit.pn_set_limb_max_tokens(16)
    M, N, K = 3, 256, 3000
    packed, gamma, w8 = _layer(N, K, seed=11, dev=cuda_device)
    x = (gen_act(M, K, seed=12) * scale).to(torch.bfloat16).to(cuda_device)
    want = orc.matmul_f64(x.float().cpu().numpy(), w8, gamma)
    y = pk.penta_linear(x, packed, gamma, K, out_dtype=torch.float32).cpu().numpy().astype(np.float64)
    # relative to the scale of the data (the absolute bar is for unit-scale data)
    err = np.abs(y - want) / scale
    assert err.max() <= 1e-3 + 1e-3 * (np.abs(want) / scale).max(), err.max()


def test_limb_outliers(cuda_device, limb_limit):
    """A few activations 2^10 times larger than the rest (outlier features):
    every output still within the bar."""
    limb_limit.pn_set_limb_max_tokens(16)
    M, N, K = 4, 512, 8192
    packed, gamma, w8 = _layer(N, K, seed=21, dev=cuda_device)
    x = gen_act(M, K, seed=22)
    x[:, [5, 777, 4096]] *= 1024.0
    _check(x.to(torch.bfloat16).to(cuda_device), packed, gamma, w8, K, what="outliers")


def test_limb_zero_and_nonfinite(cuda_device, limb_limit):
    limb_limit.pn_set_limb_max_tokens(16)
    M, N, K = 3, 200, 1600
    packed, gamma, w8 = _layer(N, K, seed=31, dev=cuda_device)
    x = gen_act(M, K, seed=32).to(torch.bfloat16)
    x[0] = 0.0
    x[1, 100] = float("inf")
    y = pk.penta_linear(x.to(cuda_device), packed, gamma, K, out_dtype=torch.float32).cpu().numpy()
    assert np.count_nonzero(y[0]) == 0
    assert np.isnan(y[1]).all()  # a token holding inf or NaN gives NaN outputs
    assert_close(y[2], orc.matmul_f64(x[2:3].float().numpy(), w8, gamma)[0], what="finite token")
    assert nat.device_status(reset=True) == 0


def test_limb_limit_setter(limb_limit):
    L = limb_limit
    prev = L.pn_set_limb_max_tokens(-1)  # query only
    assert 0 <= prev <= 16
    assert L.pn_set_limb_max_tokens(40) == prev
    assert L.pn_set_limb_max_tokens(prev) == 16  # clamped


@pytest.mark.parametrize("M,N,K", [(1, 384, 28672), (8, 8192, 3072), (13, 200, 8192)])
def test_limb_split_and_whole_tiles(cuda_device, limb_limit, M, N, K):
    """The recommended workspace (tiles split over SMs, int32 partial sums)
    and the minimum one (whole tiles per SM) give the same bits."""
    L = limb_limit
    L.pn_set_limb_max_tokens(16)
    packed, gamma, w8 = _layer(N, K, seed=N + K, dev=cuda_device)
    x = gen_act(M, K, seed=M + 3).to(torch.bfloat16).to(cuda_device)
    KP = packed.shape[1]
    outs = []
    for nbytes in (L.pn_linear_workspace_size(nat.PN_BF16, M, N, K),
                   L.pn_linear_workspace_min_size(nat.PN_BF16, M, N, K)):
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=cuda_device)
        y = torch.empty(M, N, dtype=torch.float32, device=cuda_device)
        st = L.pn_linear_bf16(x.data_ptr(), M, K, packed.data_ptr(), N, KP, ctypes.c_float(gamma), None,
                              y.data_ptr(), nat.PN_F32, ws.data_ptr(), nbytes, nat.stream_of(x))
        assert st == nat.PN_OK, L.pn_last_error()
        outs.append(y)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    assert_close(outs[0].cpu().numpy(), orc.matmul_f64(x.float().cpu().numpy(), w8, gamma), what="split/whole")
