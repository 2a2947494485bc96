"""Quantise+pack, absmean scale and unpack on the GPU against the oracle and
the reference's golden bytes (bit-exact)."""
import numpy as np
import pytest
import torch

from _util import gen_weight, golden, sha
from oracle import oracle as orc
import penta_kernel as pk

pytestmark = pytest.mark.gpu
META, G = golden()

PACK_CASES = [n for n in META["cases"] if "w_seed" in META["cases"][n] and not n.startswith("roundtrip.")]


def _w(c):
    return gen_weight(c["N"], c["K"], c["w_seed"], c.get("std", 0.02))


@pytest.mark.parametrize("name", PACK_CASES)
def test_pack_bytes_match_reference(cuda_device, name):
    c = META["cases"][name]
    w = _w(c).to(cuda_device)
    # with the reference's gamma: byte-exact
    packed, K, _ = pk.quantize_and_pack(w, scale=c["scale"])
    assert packed.shape == (c["N"], c["K_packs"]) and packed.dtype == torch.int32 and K == c["K"]
    assert sha(packed.cpu().numpy()) == c["packed_sha256"]
    # self-computed gamma: equals the oracle's correctly rounded mean exactly,
    # and within one ulp of torch's fp32 CPU mean
    packed2, _, gamma = pk.quantize_and_pack(w)
    assert gamma == orc.absmean_scale(_w(c).numpy())
    assert abs(int(np.float32(gamma).view(np.int32)) - int(np.float32(c["scale"]).view(np.int32))) <= 1
    assert sha(packed2.cpu().numpy()) == c["packed_sha256"]
    # unpack (int32 like the reference, int8 like the C kernel)
    u = pk.unpack_weights(packed2, K)
    assert u.dtype == torch.int32 and u.shape == (c["N"], K)
    assert sha(u.cpu().numpy().astype(np.int8)) == c["unpacked_sha256"]


def test_ties_and_roundtrip(cuda_device):
    from make_golden_shim import tie_weight
    wt = tie_weight(12, 50).to(cuda_device)
    packed, K, gamma = pk.quantize_and_pack(wt)
    assert gamma == 2.0 ** -4
    assert np.array_equal(pk.unpack_weights_i8(packed, K).cpu().numpy(), G["ties.12x50.unpacked"])
    for name in [n for n in META["cases"] if n.startswith("roundtrip.")]:
        c = META["cases"][name]
        g = torch.Generator().manual_seed(c["w_seed"])
        w_true = torch.randint(-2, 3, (c["N"], c["K"]), dtype=torch.int32, generator=g)
        packed, K, _ = pk.quantize_and_pack(w_true.float().to(cuda_device))
        assert sha(packed.cpu().numpy()) == c["packed_sha256"]
        assert torch.equal(pk.unpack_weights(packed, K).cpu(), w_true)


@pytest.mark.parametrize("N,K", [(1, 1), (3, 9), (2, 11), (129, 1001), (300, 4096), (7, 28672),
                                 (3, 4), (5, 124), (17, 8200), (9, 8192)])
def test_pack_random_shapes_vs_oracle(cuda_device, N, K):
    """Ragged and aligned K, odd word counts, a partial last word: the
    oracle's bytes."""
    w = gen_weight(N, K, seed=N * 31 + K, std=0.3)
    want, _, gamma = orc.quantize_pack(w.numpy())
    got, _, g2 = pk.quantize_and_pack(w.to(cuda_device))
    assert g2 == gamma
    assert np.array_equal(got.cpu().numpy(), want)
    assert np.array_equal(pk.unpack_weights_i8(got, K).cpu().numpy(), orc.unpack(want, K))


def test_pack_bf16_weights(cuda_device):
    w = gen_weight(64, 770, seed=5).to(torch.bfloat16)
    want, _, gamma = orc.quantize_pack(w.float().numpy())
    got, _, g2 = pk.quantize_and_pack(w.to(cuda_device))
    assert g2 == gamma and np.array_equal(got.cpu().numpy(), want)


def test_pack_special_values(cuda_device):
    w = torch.tensor([[0.0, -0.0, float("inf"), -float("inf"), 1e-30, 3.0, -3.0, 0.49, 0.51, 1.0, -1.0, 2.0]])
    # gamma fixed to 1 so the rounding rule is visible directly
    got, K, _ = pk.quantize_and_pack(w.to(cuda_device), scale=1.0)
    want, _, _ = orc.quantize_pack(w.numpy(), 1.0)
    assert np.array_equal(got.cpu().numpy(), want)
    assert pk.unpack_weights(got, K).cpu().tolist() == [[0, 0, 2, -2, 0, 2, -2, 0, 1, 1, -1, 2]]


def test_unpack_arbitrary_bits(cuda_device):
    rng = np.random.default_rng(0)
    raw = rng.integers(-2 ** 31, 2 ** 31, size=(33, 17), dtype=np.int64).astype(np.int32)
    got = pk.unpack_weights_i8(torch.from_numpy(raw).to(cuda_device), 165).cpu().numpy()
    assert np.array_equal(got, orc.unpack(raw, 165))


def test_cfg4_size_pack_property(cuda_device):
    """Full 70B-class matrix: pack -> unpack is idempotent under re-packing and
    the code histogram matches the absmean rule's ~11% +-2 occupancy."""
    w = gen_weight(28672, 8192, seed=11).to(cuda_device)
    packed, K, gamma = pk.quantize_and_pack(w)
    assert packed.shape == (28672, 820)
    q = pk.unpack_weights_i8(packed, K)
    repacked, _, _ = pk.quantize_and_pack(q.float(), scale=1.0)
    assert torch.equal(repacked, packed)
    hist = torch.bincount((q.flatten().to(torch.int64) + 2), minlength=5).double() / q.numel()
    assert 0.09 < hist[0] < 0.14 and 0.09 < hist[4] < 0.14
    # spot rows against the oracle
    rows = [0, 1, 12345, 28671]
    want, _, _ = orc.quantize_pack(w[rows].cpu().numpy(), gamma)
    assert np.array_equal(packed[rows].cpu().numpy(), want)


@pytest.mark.parametrize("gamma", [0.0137, 0.3, 1e-8, 7.77, 0.015953034162521362])
@pytest.mark.parametrize("mode", ["pentanet", "bitnet"])
def test_pack_near_half_integer_quotients(cuda_device, gamma, mode):
    """Weights within a few ulps of gamma * (k + 1/2) for every half-integer the
    clamp can see: the codes must equal those of the IEEE quotient (the oracle
    divides exactly like torch's weight / scale), whichever side of the tie
    each value falls on."""
    g32 = np.float32(gamma)
    vals = []
    for h in (-3.5, -2.5, -1.5, -0.5, 0.5, 1.5, 2.5, 3.5):
        c = np.float32(h) * g32
        for d in range(-4, 5):
            v = c
            step = np.float32(np.inf) if d > 0 else np.float32(-np.inf)
            for _ in range(abs(d)):
                v = np.nextafter(v, step, dtype=np.float32)
            vals.append(v)
    w = np.array(vals, dtype=np.float32).reshape(1, -1)
    w = np.concatenate([w, -w[:, ::-1]], axis=0)
    want, _, _ = orc.quantize_pack(w, float(g32), mode=mode)
    got, K, _ = pk.quantize_and_pack(torch.from_numpy(w).to(cuda_device), scale=float(g32), mode=mode)
    assert np.array_equal(got.cpu().numpy(), want)
