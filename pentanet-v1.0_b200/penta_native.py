"""ctypes binding of libpentanet_b200.so (the C ABI in include/pentanet_b200.h).

Torch supplies device memory and the current CUDA stream; every compute call
goes through the C ABI into the sm_100a kernels.  There is no CPU fallback:
if the library is missing or the device is not a B200-class sm_100 GPU, calls
raise instead of computing anything elsewhere.
"""
from __future__ import annotations

import ctypes
import functools
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "libpentanet_b200.so"

# enum pn_status_code / pn_dtype (include/pentanet_b200.h)
PN_OK, PN_ERR_ARG, PN_ERR_SHAPE, PN_ERR_ALIGN, PN_ERR_DTYPE = 0, 1, 2, 3, 4
PN_ERR_CUDA, PN_ERR_UNSUPPORTED, PN_ERR_TIMEOUT, PN_ERR_WORKSPACE = 5, 6, 7, 8
PN_F32, PN_BF16, PN_I8, PN_I32 = 0, 1, 2, 3
PN_ACT_NONE, PN_ACT_GELU = 0, 1

# Functions the header declares; tests check the library exports each one.
EXPORTS = (
    "pn_abi_version", "pn_status_string", "pn_last_error", "pn_device_status", "pn_device_sm_count",
    "pn_absmean_workspace_size", "pn_absmean_scale", "pn_quantize_pack", "pn_quantize_pack_ternary", "pn_unpack",
    "pn_linear_workspace_size", "pn_linear_workspace_min_size", "pn_linear_bf16", "pn_linear_bf16_ld", "pn_packed_ld",
    "pn_linear_bf16_nows", "pn_linear_bf16_epi", "pn_act_i8_pitch", "pn_quant_act_i8", "pn_linear_i8",
    "pn_linear_i8_ld", "pn_linear_i8_epi", "pn_layer_norm",
    "pn_ipc_handle", "pn_ipc_open", "pn_ipc_close",
    "pn_linear_bf16_peers", "pn_peer_barrier", "pn_peer_barrier_wait", "pn_set_gemv_max_tokens",
    "pn_set_limb_max_tokens", "pn_matmul_i8w",
    "pn_words_2bit", "pn_quantize_pack_2bit", "pn_unpack_2bit", "pn_linear_bf16_2bit",
)

_lib = None


class PentaNativeError(RuntimeError):
    """A CUDA-side failure reported by the C ABI (status PN_ERR_CUDA / TIMEOUT / UNSUPPORTED)."""


def lib_path() -> str:
    return os.path.join(HERE, LIB_NAME)


def load() -> ctypes.CDLL:
    """Load the shared library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                          f"or `make -C {HERE}`")
    L = ctypes.CDLL(path)
    P, I, I64, F, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
    sig = {
        "pn_abi_version": (I, []),
        "pn_status_string": (ctypes.c_char_p, [I]),
        "pn_last_error": (ctypes.c_char_p, []),
        "pn_device_status": (I, [I, ctypes.POINTER(ctypes.c_int)]),
        "pn_device_sm_count": (I, [ctypes.POINTER(ctypes.c_int)]),
        "pn_absmean_workspace_size": (SZ, []),
        "pn_absmean_scale": (I, [P, I, I64, P, P, SZ, P]),
        "pn_quantize_pack": (I, [P, I, I64, I64, P, P, P]),
        "pn_quantize_pack_ternary": (I, [P, I, I64, I64, P, P, P]),
        "pn_unpack": (I, [P, I64, I64, I64, P, P]),
        "pn_linear_workspace_size": (SZ, [I, I64, I64, I64]),
        "pn_linear_workspace_min_size": (SZ, [I, I64, I64, I64]),
        "pn_linear_bf16": (I, [P, I64, I64, P, I64, I64, F, P, P, I, P, SZ, P]),
        "pn_linear_bf16_ld": (I, [P, I64, I64, P, I64, I64, I64, F, P, P, I, P, SZ, P]),
        "pn_linear_bf16_epi": (I, [P, I64, I64, P, I64, I64, I64, F, P, I, P, I64, P, I, P, SZ, P]),
        "pn_packed_ld": (I64, [I64]),
        "pn_linear_bf16_nows": (I, [P, I64, I64, P, I64, I64, I64, F, P, P, I, P]),
        "pn_act_i8_pitch": (I64, [I64]),
        "pn_quant_act_i8": (I, [P, I, I64, I64, P, I64, P, P, P]),
        "pn_linear_i8": (I, [P, I64, P, P, I64, I64, P, I64, I64, F, P, P, I, P, P, SZ, P]),
        "pn_linear_i8_ld": (I, [P, I64, P, P, I64, I64, P, I64, I64, I64, F, P, P, I, P, P, SZ, P]),
        "pn_linear_i8_epi": (I, [P, I64, P, P, I64, I64, P, I64, I64, I64, F, P, I, P, I64, P, I, P, P, SZ, P]),
        "pn_layer_norm": (I, [P, I, I64, I64, P, P, F, P, I, P]),
        "pn_ipc_handle": (I, [P, P, ctypes.POINTER(SZ)]),
        "pn_ipc_open": (I, [P, ctypes.POINTER(P)]),
        "pn_ipc_close": (I, [P]),
        "pn_linear_bf16_peers": (I, [P, I64, I64, P, I64, I64, F, P, ctypes.POINTER(P), I, I64, I64, I, P, SZ, P]),
        "pn_peer_barrier": (I, [ctypes.POINTER(P), I, I, P, P]),
        "pn_peer_barrier_wait": (I, [ctypes.POINTER(P), I, I, P, I64, P]),
        "pn_set_gemv_max_tokens": (I, [I]),
        "pn_set_limb_max_tokens": (I, [I]),
        "pn_matmul_i8w": (I, [P, P, P, I64, I64, I64, F, P]),
        "pn_words_2bit": (I64, [I64]),
        "pn_quantize_pack_2bit": (I, [P, I, I64, I64, P, P, P]),
        "pn_unpack_2bit": (I, [P, I64, I64, I64, P, P]),
        "pn_linear_bf16_2bit": (I, [P, I64, I64, P, I64, I64, F, P, P, I, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(status: int, what: str) -> None:
    """Map a C-ABI status to the reference's error behaviour: argument, shape,
    dtype and alignment problems raise AssertionError (the reference asserts,
    penta_kernel.py:249-257); device-side failures raise PentaNativeError."""
    if status == PN_OK:
        return
    L = load()
    msg = f"{what}: {L.pn_status_string(status).decode()}: {L.pn_last_error().decode()}"
    if status in (PN_ERR_ARG, PN_ERR_SHAPE, PN_ERR_DTYPE, PN_ERR_ALIGN, PN_ERR_WORKSPACE):
        raise AssertionError(msg)
    raise PentaNativeError(msg)


# The current stream's raw handle without building a torch.cuda.Stream object
# (~0.2 us against ~2 us per call); the public route where torch lacks it.
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(t: torch.Tensor) -> int:
    if _raw_stream is not None:
        return _raw_stream(t.device.index)
    return torch.cuda.current_stream(t.device).cuda_stream


@functools.lru_cache(maxsize=4096)
def _workspace_size(kind: int, M: int, N: int, K: int, device_index: int) -> int:
    with torch.cuda.device(device_index):
        return int(load().pn_linear_workspace_size(kind, M, N, K))


def linear_workspace_size(kind: int, M: int, N: int, K: int, device: torch.device) -> int:
    """pn_linear_workspace_size on `device` (it depends on the device's SM
    count), cached per shape and device."""
    return _workspace_size(kind, M, N, K, device.index)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def device_status(reset: bool = True) -> int:
    """Device-side status word of the current device (PN_ERR_TIMEOUT after a
    kernel abandoned a bounded wait); synchronises the device."""
    v = ctypes.c_int(0)
    check(load().pn_device_status(int(reset), ctypes.byref(v)), "pn_device_status")
    return v.value
