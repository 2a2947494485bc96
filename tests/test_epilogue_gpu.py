"""Fused epilogue ops of the products (pn_linear_bf16_epi / pn_linear_i8_epi):
bias, GELU and a residual add applied after the product's bf16 rounding, each
rounded to bf16 as the separate torch ops of the reference's GPT block round
them (train_pentagpt.py:80,86,100-101).  The reference for each case is the
unfused product (itself checked against the oracle elsewhere) followed by
those torch ops on the same tensors."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from _util import bf16_ulp, gen_act, gen_weight

pytestmark = pytest.mark.gpu

# decode tiles (M <= 64, permuted activations), prefill tiles with split and
# whole tiles, a ragged last token tile, and the CUDA-core path (K % 8 != 0)
SHAPES = [(1, 3072, 768), (8, 768, 3072), (64, 1000, 2048), (200, 768, 3072), (1024, 3072, 768), (300, 256, 1001)]


def _setup(dev, M, N, K, seed):
    import penta_kernel as pk
    packed, _, gamma = pk.quantize_and_pack(gen_weight(N, K, seed=seed).to(dev))
    x = gen_act(M, K, seed=seed + 1).to(torch.bfloat16).to(dev)
    res = (gen_act(M, N, seed=seed + 2) * 0.5).to(torch.bfloat16).to(dev)
    bias = gen_weight(1, N, seed=seed + 3, std=0.3)[0].to(torch.bfloat16).to(dev)
    return pk, packed, gamma, x, res, bias


def _gelu_close(got, want, what):
    """GELU outputs: equal to torch's bf16 GELU of the same value except where
    the two erff evaluations round differently (at most one bf16 ulp)."""
    g, w = got.float().cpu().numpy().astype(np.float64), want.float().cpu().numpy().astype(np.float64)
    err = np.abs(g - w)
    assert (err <= bf16_ulp(w) + 1e-7).all(), f"{what}: max err {err.max():.3g}"
    assert (err > 0).mean() < 1e-3, f"{what}: {(err > 0).mean():.2%} of outputs differ"


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_bf16_epilogue_ops(cuda_device, M, N, K):
    pk, packed, gamma, x, res, bias = _setup(cuda_device, M, N, K, seed=M + N + K)
    y = pk.penta_linear(x, packed, gamma, K)
    yb = pk.penta_linear(x, packed, gamma, K, bias=bias)
    # residual add and bias + residual: plain bf16 adds, bit-exact
    assert torch.equal(pk.penta_linear(x, packed, gamma, K, residual=res), res + y)
    assert torch.equal(pk.penta_linear(x, packed, gamma, K, bias=bias, residual=res), res + yb)
    # GELU, GELU after bias, GELU then residual
    _gelu_close(pk.penta_linear(x, packed, gamma, K, act="gelu"), F.gelu(y), "gelu")
    _gelu_close(pk.penta_linear(x, packed, gamma, K, bias=bias, act="gelu"), F.gelu(yb), "bias+gelu")
    _gelu_close(pk.penta_linear(x, packed, gamma, K, act="gelu", residual=res), res + F.gelu(y), "gelu+residual")
    # fp32 output: no intermediate rounding
    y32 = pk.penta_linear(x, packed, gamma, K, out_dtype=torch.float32)
    got = pk.penta_linear(x, packed, gamma, K, out_dtype=torch.float32, act="gelu", residual=res)
    want = res.float() + F.gelu(y32)
    assert torch.allclose(got, want, rtol=1e-6, atol=1e-6), (got - want).abs().max().item()


@pytest.mark.parametrize("M,N,K", [(1, 3072, 768), (64, 768, 3072), (1024, 3072, 768), (300, 256, 1024)])
def test_int8_epilogue_ops(cuda_device, M, N, K):
    pk, packed, gamma, x, res, bias = _setup(cuda_device, M, N, K, seed=2 * M + N)
    y = pk.penta_linear_i8(x, packed, gamma, K, bias=bias)
    assert torch.equal(pk.penta_linear_i8(x, packed, gamma, K, bias=bias, residual=res), res + y)
    _gelu_close(pk.penta_linear_i8(x, packed, gamma, K, bias=bias, act="gelu"), F.gelu(y), "int8 bias+gelu")


def test_in_place_residual(cuda_device):
    """The residual may be the output buffer itself (the GPT's x += proj(..))."""
    import ctypes
    import penta_native as nat
    M, N, K = 96, 768, 768
    pk, packed, gamma, x, res, _ = _setup(cuda_device, M, N, K, seed=5)
    want = res + pk.penta_linear(x, packed, gamma, K)
    buf = res.clone()
    pw, ld = pk._packed_rows(packed)
    L = nat.load()
    ws_bytes = int(L.pn_linear_workspace_size(nat.PN_BF16, M, N, K))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda_device)
    nat.check(L.pn_linear_bf16_epi(x.data_ptr(), M, K, pw.data_ptr(), N, packed.shape[1], ld, ctypes.c_float(gamma),
                                   None, nat.PN_ACT_NONE, buf.data_ptr(), N, buf.data_ptr(), nat.PN_BF16,
                                   ws.data_ptr(), ws_bytes, nat.stream_of(x)), "in-place residual")
    torch.cuda.synchronize()
    assert torch.equal(buf, want)


def test_epilogue_argument_errors(cuda_device):
    import ctypes
    import penta_native as nat
    M, N, K = 4, 256, 640
    pk, packed, gamma, x, res, _ = _setup(cuda_device, M, N, K, seed=9)
    with pytest.raises(AssertionError):
        pk.penta_linear(x, packed, gamma, K, act="relu")
    with pytest.raises(AssertionError):
        pk.penta_linear(x, packed, gamma, K, residual=res[:, :100])
    with pytest.raises(AssertionError):
        pk.penta_linear(x, packed, gamma, K, residual=res.float())
    L = nat.load()
    y = torch.empty(M, N, dtype=torch.bfloat16, device=cuda_device)
    ws_bytes = int(L.pn_linear_workspace_size(nat.PN_BF16, M, N, K))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=cuda_device)
    pw, ld = pk._packed_rows(packed)
    common = (x.data_ptr(), M, K, pw.data_ptr(), N, packed.shape[1], ld, ctypes.c_float(gamma), None)
    st = L.pn_linear_bf16_epi(*common, 7, None, 0, y.data_ptr(), nat.PN_BF16, ws.data_ptr(), ws_bytes, None)
    assert st == nat.PN_ERR_ARG
    st = L.pn_linear_bf16_epi(*common, nat.PN_ACT_NONE, res.data_ptr(), N - 1, y.data_ptr(), nat.PN_BF16,
                              ws.data_ptr(), ws_bytes, None)
    assert st == nat.PN_ERR_SHAPE


@pytest.mark.parametrize("B,T", [(2, 32), (1, 7), (2, 256)])
def test_pentagpt_block_fused_matches_unfused(cuda_device, B, T):
    """One PentaGPT block (fused epilogues at decode-sized token counts,
    separate ops above) against the same block run with separate torch ops."""
    from pentagpt import PentaGPTConfig, PentaGPTFast
    cfg = PentaGPTConfig(n_layer=1, n_head=12, n_embd=768, block_size=256, vocab_size=512)
    model = PentaGPTFast.random(cfg, seed=3, device=cuda_device)
    blk = model.h[0]
    x = (gen_act(B * T, 768, seed=4) * 0.3).to(torch.bfloat16).to(cuda_device).view(B, T, 768)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        got = blk(x)
        B, T, C = x.shape
        q, k, v = blk.c_attn(blk.ln_1(x)).split(C, dim=2)
        sh = lambda t: t.view(B, T, blk.n_head, C // blk.n_head).transpose(1, 2)
        yv = F.scaled_dot_product_attention(sh(q), sh(k), sh(v), is_causal=True).transpose(1, 2).contiguous().view(B, T, C)
        x1 = x + blk.attn_proj(yv)
        want = x1 + blk.mlp_proj(F.gelu(blk.c_fc(blk.ln_2(x1))))
    err = (got.float() - want.float()).abs()
    # equal up to one-ulp rounding differences (GELU's erff, the one-pass
    # LayerNorm's fp32 statistics) and what they change downstream
    assert err.mean().item() <= 2e-3 * want.float().abs().mean().item()
    assert err.max().item() <= 0.05 * want.float().abs().max().item()


@pytest.mark.parametrize("M,C", [(1, 768), (300, 768), (64, 1024), (33, 2048), (17, 100), (5, 3000), (4096, 256),
                                 (9, 512), (70, 640)])
@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float32])
def test_layer_norm(cuda_device, M, C, x_dtype):
    """One-pass LayerNorm against torch's fp32 layer_norm of the same values
    (what nn.LayerNorm computes under bf16 autocast), rounded to bf16 or kept
    in fp32."""
    import penta_kernel as pk
    x = (gen_act(M, C, seed=M + C) * 3 + 0.5).to(x_dtype).to(cuda_device)
    w = gen_weight(1, C, seed=C, std=0.3)[0].add(1.0).to(cuda_device)
    b = gen_weight(1, C, seed=C + 1, std=0.1)[0].to(cuda_device)
    for wt, bt in ((w, None), (w, b), (None, None)):
        ref = F.layer_norm(x.float(), (C,), wt, bt, 1e-5)
        got32 = pk.layer_norm(x, wt, bt, 1e-5, out_dtype=torch.float32)
        assert torch.allclose(got32, ref, rtol=2e-5, atol=2e-5), (got32 - ref).abs().max().item()
        got = pk.layer_norm(x, wt, bt, 1e-5)
        assert got.dtype == torch.bfloat16 and got.shape == x.shape
        _gelu_close(got, ref.to(torch.bfloat16), f"layer_norm C={C}")


def test_layer_norm_unaligned_weight(cuda_device):
    """A weight view that is not 16-byte aligned takes the strided kernel."""
    import penta_kernel as pk
    x = gen_act(40, 768, seed=2).to(torch.bfloat16).to(cuda_device)
    w = (gen_weight(1, 769, seed=3, std=0.3)[0] + 1.0).to(cuda_device)[1:]
    assert w.data_ptr() % 16 != 0
    ref = F.layer_norm(x.float(), (768,), w, None, 1e-5)
    got32 = pk.layer_norm(x, w, None, 1e-5, out_dtype=torch.float32)
    assert torch.allclose(got32, ref, rtol=2e-5, atol=2e-5)
