"""Numba restatement of the reference's CPU kernel, for the timed CPU baseline.

TEST INFRASTRUCTURE ONLY (the checker / the CPU baseline): imported by tests/
and by bench.py's CPU legs, never by the shipped package.

``penta_linear_cpu`` follows penta_kernel_cpu.py:63-101 step for step: per call
the packed words are unpacked to int8 (penta_kernel.py:81-90, torch ops), and
the zero-multiplier loop (penta_kernel_cpu.py:35-60: a five-way branch per
weight, x + x for |w| = 2, parallel over output neurons with prange,
fastmath) runs over them; the result is scaled by gamma and the bias added in
fp32.  numba is a third-party dependency of the reference (imported at
penta_kernel_cpu.py:23-28, unpinned there); this restatement was checked
against the reference's own outputs (tests/golden, numba fixtures).
"""
from __future__ import annotations

import numpy as np

try:
    from numba import get_num_threads, njit, prange, set_num_threads
    AVAILABLE = True
except ImportError:  # pragma: no cover - numba is in the image
    AVAILABLE = False


if AVAILABLE:
    @njit(parallel=True, fastmath=True, cache=False)
    def _matmul_branchy(x, w, out):
        N, K = w.shape
        M = x.shape[0]
        for n in prange(N):
            for m in range(M):
                acc = np.float32(0.0)
                for k in range(K):
                    wk = w[n, k]
                    xk = x[m, k]
                    if wk == 1:
                        acc += xk
                    elif wk == -1:
                        acc -= xk
                    elif wk == 2:
                        acc += xk + xk
                    elif wk == -2:
                        acc -= xk + xk
                out[m, n] = acc


def unpack_torch(packed, K_orig: int):
    """penta_kernel.py:81-90: ten strided shift-and-mask passes, minus 2, cut to K."""
    import torch
    N, KP = packed.shape
    out = torch.zeros(N, KP * 10, dtype=torch.int32)
    for i in range(10):
        out[:, i::10] = (packed >> (3 * i)) & 7
    return (out - 2)[:, :K_orig]


def penta_linear_cpu(x, packed, scale: float, K_orig: int, bias=None):
    """penta_kernel_cpu.py:63-101 with torch tensors in and out (fp32)."""
    import torch
    assert AVAILABLE, "numba required"
    shape = x.shape
    x_np = x.contiguous().reshape(-1, shape[-1]).float().numpy().astype(np.float32)
    w_np = unpack_torch(packed, K_orig).numpy().astype(np.int8)
    out = np.empty((x_np.shape[0], w_np.shape[0]), dtype=np.float32)
    _matmul_branchy(x_np, w_np, out)
    y = torch.from_numpy(out) * scale
    if bias is not None:
        y = y + bias.float()
    return y.reshape(*shape[:-1], w_np.shape[0])


def threads(n: int | None = None) -> int:
    """Set numba's thread count (when n is given) and return it."""
    if n is not None:
        set_num_threads(n)
    return get_num_threads()
