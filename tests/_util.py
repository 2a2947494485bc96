"""Seeded input generators and tolerance checks shared by the tests.

Inputs are drawn with torch.Generator on the CPU (identical on every machine)
and moved to the GPU, so the oracle and the CUDA path see the same values.
The generators match tests/golden/make_golden.py."""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN_DIR = os.path.join(HERE, "golden")

# Parity bar for floating-point outputs: |gpu - oracle| <= ABS + REL * |oracle|
# after scaling (rel 1e-3 / abs 1e-3).
REL_TOL = 1e-3
ABS_TOL = 1e-3


def gen_weight(N: int, K: int, seed: int, std: float = 0.02) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(N, K, generator=g) * std


def gen_act(M: int, K: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(M, K, generator=g)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def golden():
    meta = json.load(open(os.path.join(GOLDEN_DIR, "golden.json")))
    arrays = np.load(os.path.join(GOLDEN_DIR, "golden.npz"))
    return meta, arrays


def assert_close(got: np.ndarray, want: np.ndarray, rel: float = REL_TOL, abs_: float = ABS_TOL, what: str = ""):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    err = np.abs(got - want)
    bound = abs_ + rel * np.abs(want)
    bad = err > bound
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} outside rel {rel}/abs {abs_}; "
                           f"max err {err.max():.3g} at {np.unravel_index(err.argmax(), err.shape)}")


def bf16_ulp(v: np.ndarray) -> np.ndarray:
    """Spacing of bf16 numbers at |v| (8 significant bits)."""
    a = np.maximum(np.abs(np.asarray(v, dtype=np.float64)), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(a)) - 7)


def assert_bf16_close(got_bf16: np.ndarray, want: np.ndarray, what: str = "", pre_bias: np.ndarray | None = None):
    """bf16 outputs: within one bf16 ulp of the exact value plus the abs bar.

    With a bias the reference rounds twice, bf16(bf16(acc*scale) + bf16(bias))
    (penta_kernel.py:224,275-276), so the first rounding may add up to one ulp
    of the pre-bias value `pre_bias`."""
    got = np.asarray(got_bf16, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    err = np.abs(got - want)
    bound = bf16_ulp(want) + ABS_TOL
    if pre_bias is not None:
        bound = bound + bf16_ulp(pre_bias)
    bad = err > bound
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} beyond 1 bf16 ulp; max err {err.max():.3g}")
