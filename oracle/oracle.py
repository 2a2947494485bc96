"""CPU oracle for PentaNet's packed pentanary path.

TEST INFRASTRUCTURE ONLY: this module is the checker.  The shipped package never
imports it; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
do, and only to compare against or to time the reference's CPU path.

Two layers:
  * ctypes bindings to ``libpenta_oracle.so`` (``penta_oracle.c``), the plain-C
    restatement of the reference algorithm, each function citing the reference
    file:line it follows;
  * numpy helpers for sizes where a scalar C loop is too slow (float64 BLAS dot
    products of exact small integers and bf16-exact activations).

``ref_avx2()`` loads ``_ref/penta_avx2.so``: the reference's own AVX2/OpenMP kernel
(penta_avx2.c:41-171) compiled from its source by ``oracle/Makefile``.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PER_WORD = 10  # penta_kernel.py:35

_lib = None
_ref = None


def _build_hint() -> str:
    return f"run `make -C {HERE}` to build the oracle"


def lib() -> ctypes.CDLL:
    """Load libpenta_oracle.so (built by oracle/Makefile)."""
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "libpenta_oracle.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing; {_build_hint()}")
        L = ctypes.CDLL(path)
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        L.pno_k_packs.restype = I64
        L.pno_k_packs.argtypes = [I64]
        L.pno_abs_sum_f64.restype = ctypes.c_double
        L.pno_abs_sum_f64.argtypes = [P, I64]
        L.pno_absmean_scale.restype = ctypes.c_float
        L.pno_absmean_scale.argtypes = [P, I64]
        L.pno_quantize_pack.restype = None
        L.pno_quantize_pack.argtypes = [P, I64, I64, ctypes.c_float, P]
        L.pno_quantize_pack_ternary.restype = None
        L.pno_quantize_pack_ternary.argtypes = [P, I64, I64, ctypes.c_float, P]
        L.pno_unpack.restype = None
        L.pno_unpack.argtypes = [P, I64, I64, I64, P]
        L.pno_matmul_f32.restype = None
        L.pno_matmul_f32.argtypes = [P, P, P, I64, I64, I64, ctypes.c_float]
        L.pno_quant_act_i8.restype = None
        L.pno_quant_act_i8.argtypes = [P, I64, I64, P, P]
        L.pno_matmul_i8.restype = None
        L.pno_matmul_i8.argtypes = [P, P, P, I64, I64, I64]
        L.pno_dequant_i8.restype = None
        L.pno_dequant_i8.argtypes = [P, P, I64, I64, ctypes.c_float, P]
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def k_packs(K: int) -> int:
    """ceil(K / 10) (penta_kernel.py:63-67)."""
    return (K + PER_WORD - 1) // PER_WORD


# ---------------------------------------------------------------- packing ---

def absmean_scale(w: np.ndarray) -> float:
    """gamma = max(mean|W|, 1e-8) as a float32 value (penta_kernel.py:57)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    return float(lib().pno_absmean_scale(_p(w), w.size))


def quantize_pack(w: np.ndarray, gamma: float | None = None, mode: str = "pentanet"):
    """quantize_and_pack (penta_kernel.py:42-78) -> (packed int32 (N,KP), K, gamma).
    mode 'bitnet': the ternary rule of QuantLinear (train_pentagpt.py:33-36),
    clamp to [-1, 1], in the same 3-bit codes."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    if gamma is None:
        gamma = absmean_scale(w)
    packed = np.empty((N, k_packs(K)), dtype=np.int32)
    fn = lib().pno_quantize_pack_ternary if mode == "bitnet" else lib().pno_quantize_pack
    fn(_p(w), N, K, ctypes.c_float(gamma), _p(packed))
    return packed, K, float(np.float32(gamma))


def unpack(packed: np.ndarray, K: int) -> np.ndarray:
    """unpack_weights (penta_kernel.py:81-90) -> int8 (N, K) in {-2..2}."""
    packed = np.ascontiguousarray(packed, dtype=np.int32)
    N, KP = packed.shape
    out = np.empty((N, K), dtype=np.int8)
    lib().pno_unpack(_p(packed), N, KP, K, _p(out))
    return out


def unpack_np(packed: np.ndarray, K: int) -> np.ndarray:
    """Vectorised unpack with the same semantics as ``unpack`` (for large N)."""
    p = np.ascontiguousarray(packed).view(np.uint32)
    N, KP = p.shape
    shifts = (3 * np.arange(PER_WORD, dtype=np.uint32))[None, None, :]
    codes = (p[:, :, None] >> shifts) & np.uint32(7)
    return (codes.reshape(N, KP * PER_WORD)[:, :K].astype(np.int16) - 2).astype(np.int8)


def pack_2bit(q: np.ndarray) -> np.ndarray:
    """Ternary values q (N, K) in {-1, 0, +1} in the library's 2-bit format:
    sixteen codes q + 1 per int32, k = 16g + j at bits 2j..2j+1 of word g,
    padding code 1.  The ternary rule itself is QuantLinear's bitnet mode
    (train_pentagpt.py:33-36), which quantize_pack(..., mode='bitnet')
    restates; the reference has no 2-bit packed format."""
    q = np.asarray(q, dtype=np.int64)
    N, K = q.shape
    KW = (K + 15) // 16
    codes = np.ones((N, KW * 16), dtype=np.uint64)
    codes[:, :K] = q + 1
    words = (codes.reshape(N, KW, 16) << (2 * np.arange(16, dtype=np.uint64))[None, None, :]).sum(axis=2)
    return words.astype(np.uint32).view(np.int32)


def unpack_2bit(packed: np.ndarray, K: int) -> np.ndarray:
    """pack_2bit's inverse -> int8 (N, K); a code 3 reads as 2."""
    p = np.ascontiguousarray(packed).view(np.uint32)
    N, KW = p.shape
    codes = (p[:, :, None] >> (2 * np.arange(16, dtype=np.uint32))[None, None, :]) & np.uint32(3)
    return (codes.reshape(N, KW * 16)[:, :K].astype(np.int16) - 1).astype(np.int8)


# ----------------------------------------------------------------- matmul ---

def matmul_f32(x: np.ndarray, w8: np.ndarray, gamma: float) -> np.ndarray:
    """Zero-multiplier fp32 matmul (penta_kernel_cpu.py:35-60, :97): sequential
    fp32 accumulation, then * gamma.  Scalar C; use for small shapes."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w8 = np.ascontiguousarray(w8, dtype=np.int8)
    M, K = x.shape
    N = w8.shape[0]
    out = np.empty((M, N), dtype=np.float32)
    lib().pno_matmul_f32(_p(x), _p(w8), _p(out), M, N, K, ctypes.c_float(gamma))
    return out


def matmul_f64(x: np.ndarray, w8: np.ndarray, gamma: float) -> np.ndarray:
    """gamma * (x @ w.T) in float64 (exact products, BLAS sum): the
    order-independent value every fp32 accumulation order approximates."""
    return (np.asarray(x, dtype=np.float64) @ np.asarray(w8, dtype=np.float64).T) * float(gamma)


def quant_act_i8(x: np.ndarray):
    """Per-token absmax int8 quantiser (penta_avx2_wrapper.py:130-131 applied
    per row) -> (xq int8 (M,K), s_x float32 (M,))."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    xq = np.empty((M, K), dtype=np.int8)
    sx = np.empty((M,), dtype=np.float32)
    lib().pno_quant_act_i8(_p(x), M, K, _p(xq), _p(sx))
    return xq, sx


def matmul_i8(xq: np.ndarray, w8: np.ndarray) -> np.ndarray:
    """torch._int_mm(xq, w.T) (penta_avx2_wrapper.py:137), exact int32.
    Uses float64 BLAS: every partial sum is an integer below 2^53, so the
    result is exact."""
    acc = np.asarray(xq, dtype=np.float64) @ np.asarray(w8, dtype=np.float64).T
    return acc.astype(np.int64).astype(np.int32)


def matmul_i8_c(xq: np.ndarray, w8: np.ndarray) -> np.ndarray:
    """Scalar-C exact int8 matmul (cross-check of ``matmul_i8``)."""
    xq = np.ascontiguousarray(xq, dtype=np.int8)
    w8 = np.ascontiguousarray(w8, dtype=np.int8)
    M, K = xq.shape
    N = w8.shape[0]
    acc = np.empty((M, N), dtype=np.int32)
    lib().pno_matmul_i8(_p(xq), _p(w8), _p(acc), M, N, K)
    return acc


def dequant_i8(acc: np.ndarray, sx: np.ndarray, gamma: float) -> np.ndarray:
    """y = float(acc) * float32(gamma * s_x) (penta_avx2_wrapper.py:147)."""
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    sx = np.ascontiguousarray(sx, dtype=np.float32)
    M, N = acc.shape
    y = np.empty((M, N), dtype=np.float32)
    lib().pno_dequant_i8(_p(acc), _p(sx), M, N, ctypes.c_float(gamma), _p(y))
    return y


# ------------------------------------------------------- bf16 rounding ----

def to_bf16_f32(a: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest-even), returned as float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32).copy()
    out[nan] = np.nan
    return out


def bf16_linear_out(acc_scaled: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """Output rounding of the reference GPU entry point (penta_kernel.py:224,
    :275-276): bf16(acc * gamma), then + bf16(bias) rounded to bf16 again."""
    y = to_bf16_f32(acc_scaled)
    if bias is not None:
        y = to_bf16_f32(y + to_bf16_f32(np.asarray(bias, dtype=np.float32))[None, :])
    return y


# ------------------------------------------------ reference AVX2 kernel ----

def ref_avx2_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "penta_avx2.so"))


def ref_avx2() -> ctypes.CDLL:
    """The reference's own CPU kernel, compiled from penta_avx2.c into _ref/.
    ABI as bound by the reference wrapper (penta_avx2_wrapper.py:18-34)."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "penta_avx2.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing; {_build_hint()} on a machine with the reference tree")
        L = ctypes.CDLL(path)
        L.penta_unpack_3bit.restype = None
        L.penta_unpack_3bit.argtypes = [ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.penta_matmul_avx2.restype = None
        L.penta_matmul_avx2.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        _ref = L
    return _ref


def ref_omp_threads(n: int | None = None) -> int:
    """Set (when n is given) and return the OpenMP thread count the reference's
    kernel runs with on the calling thread.  Launchers such as torchrun export
    OMP_NUM_THREADS=1, which libgomp reads once at start-up; the timed CPU
    baseline sets the count explicitly instead of inheriting that."""
    ref_avx2()  # loads the libgomp the kernel is linked against
    gomp = ctypes.CDLL("libgomp.so.1")
    if n is not None:
        gomp.omp_set_num_threads(ctypes.c_int(int(n)))
    return int(gomp.omp_get_max_threads())


def ref_avx2_unpack(packed: np.ndarray, K: int) -> np.ndarray:
    """penta_unpack (penta_avx2_wrapper.py:37-53) via the reference C kernel."""
    packed = np.ascontiguousarray(packed, dtype=np.int32)
    N, KP = packed.shape
    out = np.empty((N, K), dtype=np.int8)
    ref_avx2().penta_unpack_3bit(_p(packed), _p(out), N, KP, K)
    return out


def ref_avx2_linear(x: np.ndarray, w8: np.ndarray, gamma: float, out: np.ndarray | None = None) -> np.ndarray:
    """penta_linear_avx2 (penta_avx2_wrapper.py:56-94) without the torch wrap."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    N = w8.shape[0]
    if out is None:
        out = np.empty((M, N), dtype=np.float32)
    ref_avx2().penta_matmul_avx2(_p(x), _p(w8), _p(out), M, N, K, ctypes.c_float(gamma))
    return out
