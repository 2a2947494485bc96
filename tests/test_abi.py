"""The C-ABI library: loads, exports every function the header declares, and
validates arguments on the host (no GPU needed: every case below fails before
anything touches CUDA)."""
import ctypes
import os
import re
import subprocess

import pytest

import penta_native as nat

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pentanet_b200.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pn_[a-z0-9_]+)\s*\(", text)))


def test_header_lists_binding():
    assert header_functions() == sorted(nat.EXPORTS)


def test_library_exports_every_header_symbol():
    L = nat.load()
    for name in header_functions():
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", nat.lib_path()], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (pn_\w+)", out))
    assert set(header_functions()) <= exported


def test_status_strings_and_version():
    L = nat.load()
    assert L.pn_abi_version() == 1
    assert L.pn_status_string(nat.PN_OK) == b"ok"
    assert L.pn_status_string(nat.PN_ERR_TIMEOUT).startswith(b"device-side")
    assert L.pn_status_string(99) == b"unknown status"


def test_pitch_and_workspace_queries():
    L = nat.load()
    assert L.pn_act_i8_pitch(1) == 32
    assert L.pn_act_i8_pitch(4096) == 4096
    assert L.pn_act_i8_pitch(11008) == 11008
    assert L.pn_act_i8_pitch(770) == 800
    assert L.pn_absmean_workspace_size() >= 8
    assert L.pn_linear_workspace_size(nat.PN_BF16, 1, 8192, 28672) >= 0


def _call_linear_bf16(**kw):
    a = dict(x=1 << 20, M=1, K=768, packed=1 << 20, N=64, K_packs=77, scale=1.0, bias=None, y=1 << 20,
             y_dtype=nat.PN_BF16, ws=None, ws_bytes=0, stream=None)
    a.update(kw)
    L = nat.load()
    return L.pn_linear_bf16(a["x"], a["M"], a["K"], a["packed"], a["N"], a["K_packs"], ctypes.c_float(a["scale"]),
                            a["bias"], a["y"], a["y_dtype"], a["ws"], a["ws_bytes"], a["stream"])


def test_linear_argument_validation():
    L = nat.load()
    assert _call_linear_bf16(x=None) == nat.PN_ERR_ARG
    assert b"null" in L.pn_last_error()
    assert _call_linear_bf16(y_dtype=nat.PN_I8) == nat.PN_ERR_DTYPE
    assert _call_linear_bf16(K_packs=76) == nat.PN_ERR_SHAPE      # K=768 needs 77 words
    assert b"K_packs=77" in L.pn_last_error()
    assert _call_linear_bf16(M=-1) == nat.PN_ERR_SHAPE
    assert _call_linear_bf16(x=(1 << 20) + 1) == nat.PN_ERR_ALIGN  # bf16 needs 2-byte alignment
    assert _call_linear_bf16(packed=(1 << 20) + 2) == nat.PN_ERR_ALIGN


def test_int8_and_pack_argument_validation():
    L = nat.load()
    P = 1 << 20
    # pitch must cover K and be a multiple of 16
    assert L.pn_quant_act_i8(P, nat.PN_BF16, 4, 100, P, 100, P, P, None) == nat.PN_ERR_SHAPE
    assert L.pn_quant_act_i8(P, nat.PN_I32, 4, 100, P, 128, P, P, None) == nat.PN_ERR_DTYPE
    assert L.pn_linear_i8(P, 96, P, P, 4, 100, P, 8, 10, ctypes.c_float(1.0), None, P, nat.PN_BF16, None,
                          None, 0, None) == nat.PN_ERR_SHAPE                      # pitch < K
    assert L.pn_linear_i8(P, 128, P, P, 4, 100, P, 8, 9, ctypes.c_float(1.0), None, P, nat.PN_BF16, None,
                          None, 0, None) == nat.PN_ERR_SHAPE                      # K_packs mismatch
    assert L.pn_linear_i8(P, 128, P, P, 4, 100, P, 8, 10, ctypes.c_float(1.0), None, None, nat.PN_BF16, None,
                          None, 0, None) == nat.PN_ERR_ARG                        # no output at all
    assert L.pn_quantize_pack(P, nat.PN_F32, 4, 0, P, P, None) == nat.PN_ERR_SHAPE
    assert L.pn_unpack(P, 4, 2, 21, P, None) == nat.PN_ERR_SHAPE                 # K_orig > 10*K_packs
    assert L.pn_absmean_scale(P, nat.PN_F32, 10, P, None, 0, None) == nat.PN_ERR_WORKSPACE
    assert L.pn_device_status(0, None) == nat.PN_ERR_ARG


def test_python_errors_mirror_reference_asserts():
    """Shape/dtype problems raise AssertionError like penta_kernel.py:249-257."""
    with pytest.raises(AssertionError):
        nat.check(nat.PN_ERR_SHAPE, "x")
    with pytest.raises(nat.PentaNativeError):
        nat.check(nat.PN_ERR_TIMEOUT, "x")


def test_no_cpu_fallback():
    """The product path refuses CPU tensors instead of computing elsewhere."""
    import torch
    import penta_kernel as pk
    w = torch.randn(8, 20)
    with pytest.raises(AssertionError, match="CUDA"):
        pk.quantize_and_pack(w)
    with pytest.raises(AssertionError, match="CUDA"):
        pk.penta_linear(torch.randn(2, 20, dtype=torch.bfloat16), torch.zeros(8, 2, dtype=torch.int32), 1.0, 20)


def test_modules_import_without_triton():
    import sys
    import penta_kernel
    import pentanet_layer  # noqa: F401
    src = open(penta_kernel.__file__).read()
    assert "import triton" not in src
