"""penta_kernel -- drop-in for the reference module of the same name
(penta_kernel.py), backed by hand-written sm_100a kernels through a C ABI.

Same public functions, argument meanings and error behaviour:

    quantize_and_pack(weight)                         penta_kernel.py:42-78
    unpack_weights(packed, K_orig)                    penta_kernel.py:81-90
    memory_stats(N, K)                                penta_kernel.py:93-106
    penta_linear(x, packed_w, scale, K_orig, bias)    penta_kernel.py:229-278

plus the int8-activation path of the reference benchmark
(penta_avx2_wrapper.py:130-131,137,147), per token:

    quantize_activations_i8(x)
    penta_linear_i8(x, packed_w, scale, K_orig, bias)

Encoding (penta_kernel.py:7-20): weight q in {-2,-1,0,+1,+2} is stored as the
3-bit code q+2; ten codes per int32 (bits [3i+2:3i] hold column 10g+i; bits
31:30 are zero); K is padded to a multiple of 10 with code 2.  Packed tensors
are byte-identical to the reference's.

Unlike the reference module this one imports without Triton; it needs the
built library and a CUDA device (no CPU fallback).
"""
from __future__ import annotations

import ctypes

import torch

try:
    from . import penta_native as _nat
except ImportError:  # flat import (this directory on sys.path, as a drop-in)
    import penta_native as _nat

# ── Constants (penta_kernel.py:35-37) ─────────────────────────────────────────
_W_PER_INT32 = 10
_BITS_PER_W = 3
_PENTA_OFFSET = 2


def _k_packs(K: int) -> int:
    return (K + _W_PER_INT32 - 1) // _W_PER_INT32


def _require_cuda(t: torch.Tensor, what: str) -> None:
    assert t.is_cuda, f"{what} requires a CUDA tensor (sm_100a kernels; there is no CPU path)"


# ── Packing / unpacking ───────────────────────────────────────────────────────

def absmean_scale(weight: torch.Tensor) -> torch.Tensor:
    """gamma = max(mean|W|, 1e-8) as a 0-dim float32 CUDA tensor (no host sync).
    The sum of |W| runs in double in a fixed order (deterministic)."""
    assert weight.dim() == 2
    _require_cuda(weight, "absmean_scale")
    w = weight.contiguous()
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.float()
    L = _nat.load()
    ws = torch.empty(int(L.pn_absmean_workspace_size()), dtype=torch.uint8, device=w.device)
    out = torch.empty((), dtype=torch.float32, device=w.device)
    dt = _nat.PN_F32 if w.dtype == torch.float32 else _nat.PN_BF16
    _nat.check(L.pn_absmean_scale(w.data_ptr(), dt, w.numel(), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                  _nat.stream_of(w)), "absmean_scale")
    return out


def quantize_and_pack(weight: torch.Tensor, scale: float | torch.Tensor | None = None, mode: str = 'pentanet'
                      ) -> tuple[torch.Tensor, int, float]:
    """Quantize FP32/BF16 master weights to pentanary {-2..+2} and 3-bit pack.

    Args:
        weight : (N, K) FP32/BF16 CUDA tensor
        scale  : optional absmean scale to use instead of computing it (a float
                 or a 0-dim CUDA tensor); the reference always computes it.
        mode   : 'pentanet' (the reference's rule) or 'bitnet': the ternary
                 {-1, 0, +1} rule of QuantLinear(mode='bitnet')
                 (train_pentagpt.py:33-36), stored in the same 3-bit codes so
                 that every product runs it unchanged (not in the reference).

    Returns:
        packed : (N, ceil(K/10)) int32, byte-identical to the reference
        K_orig : K
        scale  : python float (penta_kernel.py:57)
    """
    assert weight.dim() == 2
    assert mode in ('pentanet', 'bitnet'), f"unknown mode {mode!r}"
    _require_cuda(weight, "quantize_and_pack")
    N, K = weight.shape
    w = weight.detach().contiguous()
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.float()
    if scale is None:
        d_scale = absmean_scale(w)
    elif isinstance(scale, torch.Tensor):
        d_scale = scale.detach().to(device=w.device, dtype=torch.float32).reshape(())
    else:
        d_scale = torch.tensor(float(scale), dtype=torch.float32, device=w.device)
    packed = torch.empty(N, _k_packs(K), dtype=torch.int32, device=w.device)
    dt = _nat.PN_F32 if w.dtype == torch.float32 else _nat.PN_BF16
    L = _nat.load()
    fn = L.pn_quantize_pack_ternary if mode == 'bitnet' else L.pn_quantize_pack
    _nat.check(fn(w.data_ptr(), dt, N, K, d_scale.data_ptr(), packed.data_ptr(), _nat.stream_of(w)),
               "quantize_and_pack")
    return packed, K, float(d_scale)


def quantize_and_pack_2bit(weight: torch.Tensor, scale: float | torch.Tensor | None = None
                           ) -> tuple[torch.Tensor, int, float]:
    """The ternary rule of QuantLinear(mode='bitnet') (train_pentagpt.py:33-36)
    packed 16 weights per int32 (2 bits each, code q + 1): 37.5 % fewer bytes
    than the 3-bit format.  Returns (packed (N, ceil(K/16)) int32, K, scale).
    Not in the reference."""
    assert weight.dim() == 2
    _require_cuda(weight, "quantize_and_pack_2bit")
    N, K = weight.shape
    w = weight.detach().contiguous()
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.float()
    if scale is None:
        d_scale = absmean_scale(w)
    elif isinstance(scale, torch.Tensor):
        d_scale = scale.detach().to(device=w.device, dtype=torch.float32).reshape(())
    else:
        d_scale = torch.tensor(float(scale), dtype=torch.float32, device=w.device)
    L = _nat.load()
    packed = torch.empty(N, int(L.pn_words_2bit(K)), dtype=torch.int32, device=w.device)
    dt = _nat.PN_F32 if w.dtype == torch.float32 else _nat.PN_BF16
    _nat.check(L.pn_quantize_pack_2bit(w.data_ptr(), dt, N, K, d_scale.data_ptr(), packed.data_ptr(),
                                       _nat.stream_of(w)), "quantize_and_pack_2bit")
    return packed, K, float(d_scale)


def unpack_weights_2bit(packed: torch.Tensor, K_orig: int) -> torch.Tensor:
    """The 2-bit ternary format back to int8 (N, K_orig) values in {-1, 0, +1}."""
    assert packed.dim() == 2 and packed.dtype == torch.int32
    _require_cuda(packed, "unpack_weights_2bit")
    N, KW = packed.shape
    p = packed.contiguous()
    out = torch.empty(N, K_orig, dtype=torch.int8, device=p.device)
    _nat.check(_nat.load().pn_unpack_2bit(p.data_ptr(), N, KW, K_orig, out.data_ptr(), _nat.stream_of(p)),
               "unpack_weights_2bit")
    return out


def penta_linear_2bit(x: torch.Tensor, packed_w: torch.Tensor, scale: float, K_orig: int,
                      bias: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """penta_linear for weights in the 2-bit ternary format: bf16 x (..., K),
    fp32 sums, then scale, bias and the output rounding of penta_linear."""
    assert x.dtype == torch.bfloat16, "x must be bfloat16"
    assert packed_w.dim() == 2 and packed_w.dtype == torch.int32
    assert x.shape[-1] == K_orig, f"x has K={x.shape[-1]}, expected {K_orig}"
    assert out_dtype in (torch.bfloat16, torch.float32)
    _require_cuda(x, "penta_linear_2bit")
    N, KW = packed_w.shape
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K_orig).contiguous()
    M = x2.shape[0]
    w = packed_w.contiguous()
    b = None if bias is None else bias.to(device=x.device, dtype=torch.bfloat16).contiguous()
    y = torch.empty(M, N, dtype=out_dtype, device=x.device)
    _nat.check(_nat.load().pn_linear_bf16_2bit(x2.data_ptr(), M, K_orig, w.data_ptr(), N, KW, float(scale),
                                               None if b is None else b.data_ptr(), y.data_ptr(),
                                               _nat.PN_F32 if out_dtype == torch.float32 else _nat.PN_BF16,
                                               _nat.stream_of(x2)), "penta_linear_2bit")
    return y.reshape(*lead, N)


def unpack_weights(packed: torch.Tensor, K_orig: int) -> torch.Tensor:
    """Unpack 3-bit tensor -> int32 (N, K_orig) with values in {-2..+2}
    (penta_kernel.py:81-90).  Use unpack_weights_i8 for the int8 form."""
    return unpack_weights_i8(packed, K_orig).to(torch.int32)


def unpack_weights_i8(packed: torch.Tensor, K_orig: int) -> torch.Tensor:
    """Unpack to int8 (N, K_orig), the layout of penta_unpack_3bit (penta_avx2.c:41-59)."""
    assert packed.dim() == 2 and packed.dtype == torch.int32
    _require_cuda(packed, "unpack_weights")
    N, K_packs = packed.shape
    p = packed.contiguous()
    out = torch.empty(N, K_orig, dtype=torch.int8, device=p.device)
    _nat.check(_nat.load().pn_unpack(p.data_ptr(), N, K_packs, K_orig, out.data_ptr(), _nat.stream_of(p)),
               "unpack_weights")
    return out


def penta_linear_i8w(x: torch.Tensor, w_int8: torch.Tensor, scale: float,
                     bias: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 x (..., K) times unpacked int8 weights (N, K) in {-2..+2}, times
    scale, plus an optional bias, in fp32: the GPU form of the reference's
    AVX2 path (penta_linear_avx2, penta_avx2_wrapper.py:58-94, computing
    penta_matmul_avx2, penta_avx2.c:87-171).  w_int8 comes from
    unpack_weights_i8 (the layout of penta_unpack_3bit)."""
    assert w_int8.dim() == 2 and w_int8.dtype == torch.int8, "w_int8 must be an (N, K) int8 tensor"
    _require_cuda(x, "penta_linear_i8w")
    _require_cuda(w_int8, "penta_linear_i8w")
    N, K = w_int8.shape
    assert x.shape[-1] == K, f"x has K={x.shape[-1]}, the weights K={K}"
    lead = x.shape[:-1]
    xf = x.reshape(-1, K).float().contiguous()
    w = w_int8.contiguous()
    M = xf.shape[0]
    y = torch.empty(M, N, dtype=torch.float32, device=x.device)
    _nat.check(_nat.load().pn_matmul_i8w(xf.data_ptr(), w.data_ptr(), y.data_ptr(), M, N, K, float(scale),
                                         _nat.stream_of(xf)), "penta_linear_i8w")
    if bias is not None:
        y = y + bias.float()
    return y.reshape(*lead, N)


def memory_stats(N: int, K: int) -> dict:
    """Memory footprint comparison for an (N, K) weight matrix (penta_kernel.py:93-106):
    nominal 3 bits/weight, as the reference reports it."""
    fp16_bytes = N * K * 2
    packed_bytes = (N * K * _BITS_PER_W + 7) // 8
    ternary_bytes = (N * K * 2 + 7) // 8
    return {
        "fp16_MB": fp16_bytes / 1e6,
        "packed_MB": packed_bytes / 1e6,
        "ternary_MB": ternary_bytes / 1e6,
        "penta_vs_fp16_ratio": round(fp16_bytes / packed_bytes, 2),
        "penta_vs_ternary_ratio": round(ternary_bytes / packed_bytes, 2),
    }


def storage_bytes(N: int, K: int) -> int:
    """Actual bytes of the packed int32 tensor (4 * N * ceil(K/10))."""
    return 4 * N * _k_packs(K)


# ── Resident weight layout ───────────────────────────────────────────────────

def packed_ld(K_packs: int) -> int:
    """Row stride (int32 words) at which the GEMM reads packed rows in place:
    K_packs rounded up to a multiple of 4 (16-byte rows for TMA)."""
    return (int(K_packs) + 3) // 4 * 4


def pad_packed(packed: torch.Tensor) -> torch.Tensor:
    """The same (N, K_packs) packed weights stored at row stride
    packed_ld(K_packs): a view of a zero-padded (N, packed_ld) buffer.  Values
    and shape are unchanged; penta_linear / penta_linear_i8 read such rows in
    place instead of re-pitching the weights on every call (when K_packs is not
    a multiple of 4).  Not in the reference; used for weights kept resident
    (PentaLinearFast)."""
    assert packed.dim() == 2 and packed.dtype == torch.int32
    N, KP = packed.shape
    ld = packed_ld(KP)
    if packed.stride(1) == 1 and packed.stride(0) == ld:
        return packed
    buf = torch.zeros(N, ld, dtype=torch.int32, device=packed.device)
    buf[:, :KP].copy_(packed)
    return buf[:, :KP]


def _packed_rows(packed_w: torch.Tensor) -> tuple[torch.Tensor, int]:
    """(tensor, row stride in words) to hand to the C ABI: strided views with
    unit column stride are passed as they are, anything else is made contiguous."""
    if packed_w.dim() == 2 and packed_w.stride(1) == 1 and packed_w.stride(0) >= packed_w.shape[1]:
        return packed_w, int(packed_w.stride(0))
    pw = packed_w.contiguous()
    return pw, int(pw.shape[1])


# ── Fused dequant-matmul ─────────────────────────────────────────────────────

_ACTS = {None: _nat.PN_ACT_NONE, 'none': _nat.PN_ACT_NONE, 'gelu': _nat.PN_ACT_GELU}


def _epilogue_args(act, residual, lead, N, device):
    """(activation code, residual (M, N) bf16 or None) for the fused epilogue."""
    assert act in _ACTS, f"act must be one of {sorted(k for k in _ACTS if k)} or None, got {act!r}"
    if residual is None:
        return _ACTS[act], None
    assert residual.dtype == torch.bfloat16, "residual must be bfloat16"
    assert residual.device == device, "residual must be on the activations' device"
    assert tuple(residual.shape) == (*lead, N), f"residual shape {tuple(residual.shape)} != {(*lead, N)}"
    return _ACTS[act], residual.contiguous().reshape(-1, N)


def penta_linear(x: torch.Tensor, packed_w: torch.Tensor, scale: float, K_orig: int,
                 bias: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
                 act: str | None = None, residual: torch.Tensor | None = None) -> torch.Tensor:
    """Fast pentanary linear: Y = X @ W.T * scale + bias (penta_kernel.py:229-278).

    Args:
        x        : (..., K) bfloat16 activation on CUDA
        packed_w : (N, K_packs) int32 packed weights on CUDA
        scale    : scalar float (absmean scale from quantize_and_pack)
        K_orig   : original K before padding
        bias     : (N,) optional bias tensor
        out_dtype: torch.bfloat16 (reference rounding) or torch.float32 (the
                   unrounded fp32 result; not in the reference)
        act      : None or 'gelu' -- applied in the epilogue after the bias,
                   rounded as a separate bf16 F.gelu would be (not in the
                   reference's wrapper; its GPT applies nn.GELU after c_fc)
        residual : None or a (..., N) bf16 tensor added last, as the GPT
                   block's `x + proj(..)` (train_pentagpt.py:100-101)

    Returns:
        y : (..., N) of out_dtype
    """
    assert x.is_cuda, "penta_linear requires CUDA"
    assert x.dtype == torch.bfloat16, "Activations must be bfloat16"
    assert packed_w.dtype == torch.int32
    assert out_dtype in (torch.bfloat16, torch.float32)
    orig_shape = x.shape
    x_2d = x.contiguous().reshape(-1, orig_shape[-1])
    M, K = x_2d.shape
    N, K_packs = packed_w.shape
    assert K == K_orig, f"Activation K={K} must match K_orig={K_orig}"
    act_code, res = _epilogue_args(act, residual, orig_shape[:-1], N, x.device)
    pw, ld = _packed_rows(packed_w)
    y = torch.empty(M, N, device=x.device, dtype=out_dtype)
    b = None
    if bias is not None:
        b = bias.detach().to(device=x.device, dtype=torch.bfloat16).contiguous()
        assert b.numel() == N
    L = _nat.load()
    ws_bytes = _nat.linear_workspace_size(_nat.PN_BF16, M, N, K, x.device)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device) if ws_bytes else None
    ydt = _nat.PN_F32 if out_dtype == torch.float32 else _nat.PN_BF16
    if act_code == _nat.PN_ACT_NONE and res is None:
        _nat.check(L.pn_linear_bf16_ld(x_2d.data_ptr(), M, K, pw.data_ptr(), N, K_packs, ld, ctypes.c_float(scale),
                                       _nat.ptr(b), y.data_ptr(), ydt, _nat.ptr(ws), ws_bytes,
                                       _nat.stream_of(x_2d)), "penta_linear")
    else:
        _nat.check(L.pn_linear_bf16_epi(x_2d.data_ptr(), M, K, pw.data_ptr(), N, K_packs, ld, ctypes.c_float(scale),
                                        _nat.ptr(b), act_code, _nat.ptr(res), N, y.data_ptr(), ydt, _nat.ptr(ws),
                                        ws_bytes, _nat.stream_of(x_2d)), "penta_linear")
    return y.reshape(*orig_shape[:-1], N)


def layer_norm(x: torch.Tensor, weight: torch.Tensor | None = None, bias: torch.Tensor | None = None,
               eps: float = 1e-5, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """LayerNorm over the last dimension in one pass, output in out_dtype: what
    nn.LayerNorm under bf16 autocast followed by a cast to bf16 computes (fp32
    statistics, biased variance; train_pentagpt.py:94-96,127), without the
    fp32 round trip.  x: (..., C) bf16/fp32 CUDA; weight, bias: (C,) or None."""
    assert x.is_cuda and x.dtype in (torch.bfloat16, torch.float32)
    assert out_dtype in (torch.bfloat16, torch.float32)
    C = x.shape[-1]
    x2 = x.contiguous().reshape(-1, C)
    wf = weight.detach().to(device=x.device, dtype=torch.float32).contiguous() if weight is not None else None
    bf = bias.detach().to(device=x.device, dtype=torch.float32).contiguous() if bias is not None else None
    assert wf is None or wf.numel() == C
    assert bf is None or bf.numel() == C
    y = torch.empty(x2.shape, dtype=out_dtype, device=x.device)
    dt = lambda t: _nat.PN_F32 if t == torch.float32 else _nat.PN_BF16
    L = _nat.load()
    _nat.check(L.pn_layer_norm(x2.data_ptr(), dt(x2.dtype), x2.shape[0], C, _nat.ptr(wf), _nat.ptr(bf),
                               ctypes.c_float(eps), y.data_ptr(), dt(out_dtype), _nat.stream_of(x2)), "layer_norm")
    return y.reshape(x.shape)


# ── int8 activation path ─────────────────────────────────────────────────────

def quantize_activations_i8(x: torch.Tensor):
    """Per-token absmax int8 quantiser (penta_avx2_wrapper.py:130-131 applied per row).

    Returns (xq, s_x, rowsum): xq (M, pitch) int8 zero-padded past K (pitch =
    ceil(K/32)*32; xq[:, :K] is the quantised activation), s_x (M,) float32,
    rowsum (M,) int32 = xq.sum(1)."""
    assert x.is_cuda and x.dtype in (torch.bfloat16, torch.float32)
    x_2d = x.contiguous().reshape(-1, x.shape[-1])
    M, K = x_2d.shape
    L = _nat.load()
    pitch = int(L.pn_act_i8_pitch(K))
    xq = torch.empty(M, pitch, dtype=torch.int8, device=x.device)
    s_x = torch.empty(M, dtype=torch.float32, device=x.device)
    rowsum = torch.empty(M, dtype=torch.int32, device=x.device)
    dt = _nat.PN_F32 if x_2d.dtype == torch.float32 else _nat.PN_BF16
    _nat.check(L.pn_quant_act_i8(x_2d.data_ptr(), dt, M, K, xq.data_ptr(), pitch, s_x.data_ptr(),
                                 rowsum.data_ptr(), _nat.stream_of(x_2d)), "quantize_activations_i8")
    return xq, s_x, rowsum


def penta_linear_i8_prequant(xq: torch.Tensor, s_x: torch.Tensor, rowsum: torch.Tensor, K_orig: int,
                             packed_w: torch.Tensor, scale: float, bias: torch.Tensor | None = None,
                             out_dtype: torch.dtype | None = torch.bfloat16, return_acc: bool = False,
                             act: str | None = None, residual: torch.Tensor | None = None):
    """int8 x packed-weight GEMM on already-quantised activations.
    acc = xq @ w.T exactly (int32, = torch._int_mm); y = float(acc) * float32(scale * s_x) (+ bias),
    then the fused act / residual of penta_linear."""
    assert xq.is_cuda and xq.dtype == torch.int8 and xq.dim() == 2
    assert packed_w.dtype == torch.int32
    M, pitch = xq.shape
    N, K_packs = packed_w.shape
    assert K_packs == _k_packs(K_orig), "packed weights do not match K_orig"
    act_code, res = _epilogue_args(act, residual, (M,), N, xq.device)
    assert out_dtype is not None or (act_code == _nat.PN_ACT_NONE and res is None), "epilogue ops need an output"
    pw, ld = _packed_rows(packed_w)
    y = torch.empty(M, N, device=xq.device, dtype=out_dtype) if out_dtype is not None else None
    acc = torch.empty(M, N, device=xq.device, dtype=torch.int32) if return_acc else None
    b = bias.detach().to(device=xq.device, dtype=torch.bfloat16).contiguous() if bias is not None else None
    L = _nat.load()
    ws_bytes = _nat.linear_workspace_size(_nat.PN_I8, M, N, K_orig, xq.device)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=xq.device) if ws_bytes else None
    ydt = _nat.PN_F32 if out_dtype == torch.float32 else _nat.PN_BF16
    _nat.check(L.pn_linear_i8_epi(xq.data_ptr(), pitch, s_x.data_ptr(), rowsum.data_ptr(), M, K_orig,
                                  pw.data_ptr(), N, K_packs, ld, ctypes.c_float(scale), _nat.ptr(b), act_code,
                                  _nat.ptr(res), N, _nat.ptr(y), ydt, _nat.ptr(acc), _nat.ptr(ws), ws_bytes,
                                  _nat.stream_of(xq)), "penta_linear_i8")
    return (y, acc) if return_acc else y


def penta_linear_i8(x: torch.Tensor, packed_w: torch.Tensor, scale: float, K_orig: int,
                    bias: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
                    return_acc: bool = False, act: str | None = None, residual: torch.Tensor | None = None):
    """Prefill path: per-token int8 activations x packed weights on the int8
    tensor cores, fused scale epilogue (+ bias, act, residual as penta_linear).
    x: (..., K) bf16/fp32 CUDA."""
    orig_shape = x.shape
    assert orig_shape[-1] == K_orig, f"Activation K={orig_shape[-1]} must match K_orig={K_orig}"
    N = packed_w.shape[0]
    if residual is not None:
        assert tuple(residual.shape) == (*orig_shape[:-1], N), "residual must match the output shape"
        residual = residual.reshape(-1, N)
    xq, s_x, rowsum = quantize_activations_i8(x)
    out = penta_linear_i8_prequant(xq, s_x, rowsum, K_orig, packed_w, scale, bias, out_dtype, return_acc,
                                   act=act, residual=residual)
    if return_acc:
        y, acc = out
        return y.reshape(*orig_shape[:-1], N), acc.reshape(*orig_shape[:-1], N)
    return out.reshape(*orig_shape[:-1], N)
