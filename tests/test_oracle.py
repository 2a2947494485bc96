"""The oracle (oracle/penta_oracle.c) pinned against the reference's own outputs.

tests/golden/ holds what the reference produced (penta_kernel.quantize_and_pack,
unpack_weights, memory_stats; penta_kernel_cpu.penta_linear_cpu (numba); the
AVX2 kernel compiled from penta_avx2.c; torch._int_mm for the int8 line), made by
tests/golden/make_golden.py.  No GPU is needed."""
import numpy as np
import pytest

from _util import gen_act, gen_weight, golden, sha
from oracle import oracle as orc

META, G = golden()


def _case_weight(name, c):
    if name.startswith("ties."):
        import make_golden_shim as mg
        return mg.tie_weight(c["N"], c["K"]).numpy()
    if name.startswith("roundtrip."):
        import torch
        g = torch.Generator().manual_seed(c["w_seed"])
        return torch.randint(-2, 3, (c["N"], c["K"]), dtype=torch.int32, generator=g).float().numpy()
    return gen_weight(c["N"], c["K"], c["w_seed"], c.get("std", 0.02)).numpy()


PACK_CASES = [n for n in META["cases"] if "w_seed" in META["cases"][n] or n.startswith("ties.")]


@pytest.mark.parametrize("name", PACK_CASES)
def test_quantize_pack_matches_reference(name):
    c = META["cases"][name]
    w = _case_weight(name, c)
    # Byte-exact with the reference's own gamma ...
    packed, K, gamma = orc.quantize_pack(w, c["scale"])
    assert K == c["K"] and packed.shape == (c["N"], c["K_packs"])
    assert sha(packed) == c["packed_sha256"]
    assert sha(orc.unpack(packed, K)) == c["unpacked_sha256"]
    if f"{name}.packed" in G.files:
        assert np.array_equal(packed, G[f"{name}.packed"])
    # ... and with the oracle's correctly rounded mean, which may sit one ulp
    # from torch's fp32 CPU sum (penta_kernel.py:57): same bytes on every fixture.
    packed2, _, gamma2 = orc.quantize_pack(w)
    ulps = abs(int(np.float32(gamma2).view(np.int32)) - int(np.float32(c["scale"]).view(np.int32)))
    assert ulps <= 1, f"gamma {gamma2!r} vs reference {c['scale']!r}"
    assert sha(packed2) == c["packed_sha256"]


def test_ties_round_half_even():
    c = META["cases"]["ties.12x50"]
    w = _case_weight("ties.12x50", c)
    packed, K, gamma = orc.quantize_pack(w)
    assert gamma == 2.0 ** -4
    assert np.array_equal(orc.unpack(packed, K), G["ties.12x50.unpacked"])
    # 0.5 -> 0, 1.5 -> 2, 2.5 -> 2, -0.5 -> 0, -1.5 -> -2
    q = orc.unpack(packed, K)
    r = w / gamma
    for v, expect in [(0.5, 0), (1.5, 2), (2.5, 2), (-0.5, 0), (-1.5, -2)]:
        assert np.all(q[r == v] == expect)


@pytest.mark.parametrize("name", [n for n in META["cases"] if n.startswith("roundtrip.")])
def test_roundtrip_exact(name):
    c = META["cases"][name]
    assert c["roundtrip_exact"]
    w = _case_weight(name, c)
    packed, K, _ = orc.quantize_pack(w)
    assert np.array_equal(orc.unpack(packed, K), w.astype(np.int8))


def test_unpack_np_matches_c():
    p = G["small.128x770.packed"]
    assert np.array_equal(orc.unpack_np(p, 770), orc.unpack(p, 770))
    # undefined codes 5..7 and the top two bits follow the shift-and-mask rule
    rng = np.random.default_rng(0)
    raw = rng.integers(0, 2 ** 31, size=(9, 7), dtype=np.int64).astype(np.int32)
    assert np.array_equal(orc.unpack_np(raw, 65), orc.unpack(raw, 65))


def test_numba_and_avx2_outputs_cfg0():
    c = META["cases"]["cfg0"]
    w = gen_weight(3072, 768, 0).numpy()
    packed, K, gamma = orc.quantize_pack(w)
    x = gen_act(8, 768, c["x_seed"]).numpy()
    w8 = orc.unpack(packed, K)
    y32 = orc.matmul_f32(x, w8, gamma)
    y64 = orc.matmul_f64(x, w8, gamma)
    # same math, different fp32 summation order than numba (fastmath) / AVX2 (8 lanes)
    assert np.abs(y32 - G["cfg0.y_numba"]).max() < 1e-5
    assert np.abs(y32 - G["cfg0.y_avx2"]).max() < 1e-5
    assert np.abs(y64 - G["cfg0.y_numba"]).max() < 1e-5
    occ = np.bincount((w8.astype(np.int16) + 2).ravel(), minlength=5) / w8.size
    assert np.allclose(occ, c["occupancy_m2_to_p2"])


@pytest.mark.parametrize("shape", [(768, 2304), (768, 768), (768, 3072), (3072, 768)])
def test_cfg1_numba_outputs(shape):
    K, N = shape
    name = f"cfg1.{K}x{N}"
    c = META["cases"][name]
    w = gen_weight(N, K, c["w_seed"]).numpy()
    packed, _, gamma = orc.quantize_pack(w)
    assert sha(packed) == c["packed_sha256"]
    w8 = orc.unpack(packed, K)
    import torch
    for M in (1, 4, 16):
        x = gen_act(M, K, c[f"M{M}_x_seed"]).to(torch.bfloat16).float().numpy()
        y = orc.matmul_f64(x, w8, gamma)
        assert np.abs(y - G[f"{name}.M{M}.y_numba"]).max() < 1e-4


@pytest.mark.parametrize("name", [n for n in META["cases"] if n.startswith("int8.")])
def test_int8_line_exact(name):
    c = META["cases"][name]
    x = gen_act(c["M"], c["K"], c["x_seed"]).numpy()
    xq, sx = orc.quant_act_i8(x)
    assert np.array_equal(xq, G[f"{name}.xq"])
    assert np.array_equal(sx, G[f"{name}.sx"])
    w8 = orc.unpack(G[f"{name}.packed"], c["K"])
    acc = orc.matmul_i8(xq, w8)
    assert np.array_equal(acc, G[f"{name}.acc"])
    assert np.array_equal(orc.matmul_i8_c(xq, w8), acc)
    assert np.array_equal(orc.dequant_i8(acc, sx, c["scale"]), G[f"{name}.y"])


def test_int_mm_fixture():
    acc = orc.matmul_i8(G["intmm.a"], G["intmm.b"])
    assert np.array_equal(acc, G["intmm.acc"])


def test_zero_row_activation_scale():
    x = np.zeros((2, 40), dtype=np.float32)
    x[1, 3] = -5.0
    xq, sx = orc.quant_act_i8(x)
    assert sx[0] == 1.0 and not xq[0].any()
    assert xq[1, 3] == -127


def test_bf16_rounding_helper():
    v = np.array([1.0, 1.00390625, 1.005859375, -3.14159, 65504.0, 1e-20], dtype=np.float32)
    import torch
    want = torch.from_numpy(v).to(torch.bfloat16).float().numpy()
    assert np.array_equal(orc.to_bf16_f32(v), want)


def test_memory_stats_matches_reference():
    import penta_kernel as pk  # the package's module (imports without a GPU)
    for key, stats in META["memory_stats"].items():
        N, K = map(int, key.split("x"))
        assert pk.memory_stats(N, K) == stats


def test_ternary_rule():
    """The oracle's ternary (bitnet) quantiser is clamp(round_half_even(w / gamma),
    -1, 1) with float32 division (train_pentagpt.py:33-36), ties included."""
    w = gen_weight(64, 257, seed=3).numpy()
    w[0, :4] = [0.5, -0.5, 1.5, -2.5]
    gamma = 1.0
    packed, K, _ = orc.quantize_pack(w, gamma, mode="bitnet")
    q = orc.unpack(packed, K)
    want = np.clip(np.rint(w.astype(np.float32) / np.float32(gamma)), -1, 1).astype(np.int8)
    assert np.array_equal(q, want)
    assert list(q[0, :4]) == [0, 0, 1, -1]


@pytest.mark.parametrize("name", ["cfg0"] + [n for n in META["cases"] if n.startswith("small.")][:4])
def test_numba_port_matches_reference_numba(name):
    """oracle/numba_port.py (the timed numba CPU leg) against the reference's own
    numba penta_linear_cpu outputs stored in the fixtures."""
    import torch
    from oracle import numba_port as nbp
    if not nbp.AVAILABLE:
        pytest.skip("numba not importable")
    c = META["cases"][name]
    if name == "cfg0":
        w, x = gen_weight(3072, 768, seed=0), gen_act(8, 768, seed=100)
    else:
        w = gen_weight(c["N"], c["K"], seed=c["w_seed"], std=c["std"])
        x = gen_act(3, c["K"], seed=c["x_seed"])
    packed, _, gamma = orc.quantize_pack(w.numpy())
    y = nbp.penta_linear_cpu(x, torch.from_numpy(packed), gamma, c["K"]).numpy()
    assert np.abs(y - G[f"{name}.y_numba"]).max() < 1e-5
