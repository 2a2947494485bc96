"""The 2-bit ternary format (16 codes per int32; QuantLinear's bitnet rule,
train_pentagpt.py:33-36): packed bytes against the oracle, the same codes as
the 3-bit ternary packing, and the product against the oracle.

Tolerance: packed bytes and unpacked values exact; fp32 outputs within
rel 1e-3 / abs 1e-3 of the oracle's float64 product; bf16 outputs within one
bf16 ulp (+ abs 1e-3)."""
import numpy as np
import pytest
import torch

from _util import assert_bf16_close, assert_close, gen_act, gen_weight
from oracle import oracle as orc
import penta_kernel as pk
import penta_native as nat


def test_oracle_2bit_roundtrip():
    """CPU: the oracle's 2-bit packing round-trips every ternary value."""
    rng = np.random.default_rng(0)
    for K in (1, 15, 16, 17, 100):
        q = rng.integers(-1, 2, size=(7, K)).astype(np.int8)
        p = orc.pack_2bit(q)
        assert p.shape == (7, (K + 15) // 16) and p.dtype == np.int32
        assert np.array_equal(orc.unpack_2bit(p, K), q)
    # padding codes are 1 (q = 0): one weight 1 -> code 2 in the low bits, then 15 x code 1
    assert orc.pack_2bit(np.array([[1]], dtype=np.int8))[0, 0] == np.int32(np.uint32(0x55555556).view(np.int32))


@pytest.mark.gpu
@pytest.mark.parametrize("N,K,dtype", [(5, 1, torch.float32), (64, 15, torch.float32), (33, 16, torch.float32),
                                       (130, 17, torch.bfloat16), (300, 770, torch.float32),
                                       (257, 1001, torch.bfloat16), (1024, 4096, torch.float32)])
def test_pack_2bit_matches_oracle(cuda_device, N, K, dtype):
    w = gen_weight(N, K, seed=N + K)
    if dtype == torch.bfloat16:
        w = w.to(torch.bfloat16)
    packed, K_orig, gamma = pk.quantize_and_pack_2bit(w.to(cuda_device))
    assert K_orig == K and packed.shape == (N, (K + 15) // 16)
    # the oracle's ternary rule with the same gamma
    p3, _, _ = orc.quantize_pack(w.float().numpy(), gamma=gamma, mode="bitnet")
    q = orc.unpack(p3, K)
    assert np.array_equal(packed.cpu().numpy(), orc.pack_2bit(q)), "2-bit packed bytes differ from the oracle"
    assert np.array_equal(pk.unpack_weights_2bit(packed, K).cpu().numpy(), q)
    # the same codes as the 3-bit ternary packing on the GPU
    p3g, _, g3 = pk.quantize_and_pack(w.to(cuda_device), mode="bitnet")
    assert g3 == gamma
    assert torch.equal(pk.unpack_weights_i8(p3g, K), pk.unpack_weights_2bit(packed, K))


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(1, 300, 770), (5, 257, 1001), (16, 640, 4096), (40, 128, 3072), (3, 100, 13),
                                   (8, 2048, 8192)])
def test_linear_2bit(cuda_device, M, N, K):
    w = gen_weight(N, K, seed=M + N)
    packed, _, gamma = pk.quantize_and_pack_2bit(w.to(cuda_device))
    q = orc.unpack_2bit(packed.cpu().numpy(), K)
    x = gen_act(M, K, seed=K + 3).to(torch.bfloat16)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(M)).to(torch.bfloat16)
    pre = orc.matmul_f64(x.float().numpy(), q, gamma)
    y32 = pk.penta_linear_2bit(x.to(cuda_device), packed, gamma, K, out_dtype=torch.float32)
    assert_close(y32.cpu().numpy(), pre, what=f"2bit fp32 M={M} N={N} K={K}")
    y16 = pk.penta_linear_2bit(x.to(cuda_device), packed, gamma, K)
    assert_bf16_close(y16.float().cpu().numpy(), pre, what="2bit bf16")
    assert np.array_equal(y16.float().cpu().numpy(), orc.to_bf16_f32(y32.cpu().numpy()))
    yb = pk.penta_linear_2bit(x.to(cuda_device), packed, gamma, K, bias.to(cuda_device))
    assert_bf16_close(yb.float().cpu().numpy(), pre + bias.float().numpy()[None, :], what="2bit bias", pre_bias=pre)


@pytest.mark.gpu
def test_2bit_errors(cuda_device):
    w = gen_weight(8, 40, seed=1).to(cuda_device)
    packed, K, gamma = pk.quantize_and_pack_2bit(w)
    x = torch.zeros(2, 40, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(AssertionError):
        pk.penta_linear_2bit(x, packed[:, :2], gamma, K)  # K_words does not match K
    with pytest.raises(AssertionError):
        pk.penta_linear_2bit(x.float(), packed, gamma, K)
    assert nat.load().pn_words_2bit(40) == 3 and nat.load().pn_words_2bit(0) == 0
