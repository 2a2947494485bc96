"""The CUDA-core decode GEMV (csrc/pn_gemv.cu) against the oracle, for every
token count it takes (1-4), next to the tensor-core kernel on the same inputs.

Same tolerance contract as tests/test_linear_gpu.py: fp32 outputs within rel
1e-3 / abs 1e-3 of the oracle's float64 product, bf16 outputs within one bf16
ulp (+ abs 1e-3)."""
import pytest
import torch

from _util import assert_bf16_close, assert_close, gen_act, gen_weight
from oracle import oracle as orc
import penta_kernel as pk
import penta_native as nat

pytestmark = pytest.mark.gpu


@pytest.fixture
def gemv_limit():
    """Routes products of up to 8 tokens to the GEMV for the test, then restores."""
    L = nat.load()
    prev = L.pn_set_gemv_max_tokens(8)
    yield L
    L.pn_set_gemv_max_tokens(prev)


# (N, K): ragged K, K beyond one 256-word box row, N not a multiple of the row
# tile, several K windows at 8 tokens (K = 28672 > the 8-token window)
SHAPES = [(384, 768), (1000, 1001), (3072, 768), (768, 3072), (200, 10), (96, 4096), (130, 28672), (17, 40000)]


@pytest.mark.parametrize("N,K", SHAPES)
@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8])
def test_gemv_matches_oracle(cuda_device, gemv_limit, M, N, K):
    w = gen_weight(N, K, seed=N * 3 + K)
    packed, _, gamma = pk.quantize_and_pack(w.to(cuda_device))
    padded = pk.pad_packed(packed)  # rows at a 16-byte pitch: the GEMV reads them in place
    w8 = orc.unpack(packed.cpu().numpy(), K)
    x = gen_act(M, K, seed=M + K).to(torch.bfloat16).to(cuda_device)
    want = orc.matmul_f64(x.float().cpu().numpy(), w8, gamma)
    for pw in (padded, packed):
        y32 = pk.penta_linear(x, pw, gamma, K, out_dtype=torch.float32)
        assert_close(y32.cpu().numpy(), want, what=f"gemv M={M} {N}x{K} fp32")
        y16 = pk.penta_linear(x, pw, gamma, K)
        assert_bf16_close(y16.float().cpu().numpy(), want, what=f"gemv M={M} {N}x{K} bf16")
    # the tensor-core kernel on the same inputs agrees to the same bar
    gemv_limit.pn_set_gemv_max_tokens(0)
    ytc = pk.penta_linear(x, padded, gamma, K, out_dtype=torch.float32)
    gemv_limit.pn_set_gemv_max_tokens(8)
    assert_close(ytc.cpu().numpy(), want, what="tensor-core fp32")
    assert nat.device_status() == 0


@pytest.mark.parametrize("M", [1, 3])
def test_gemv_epilogue_ops(cuda_device, gemv_limit, M):
    """Bias (the reference's double rounding), GELU and a residual in the GEMV's epilogue."""
    N, K = 640, 1536
    packed, _, gamma = pk.quantize_and_pack(gen_weight(N, K, seed=9).to(cuda_device))
    packed = pk.pad_packed(packed)
    w8 = orc.unpack(packed[:, :(K + 9) // 10].contiguous().cpu().numpy(), K)
    x = gen_act(M, K, seed=10).to(torch.bfloat16).to(cuda_device)
    bias = (torch.randn(N, generator=torch.Generator().manual_seed(11)) * 0.1).to(torch.bfloat16).to(cuda_device)
    pre = orc.matmul_f64(x.float().cpu().numpy(), w8, gamma)
    y = pk.penta_linear(x, packed, gamma, K, bias)
    want = pre + bias.float().cpu().numpy()[None, :]
    assert_bf16_close(y.float().cpu().numpy(), want, what="gemv bias", pre_bias=pre)
    # fused ops against the same ops applied after the plain GEMV product (bit-exact:
    # the epilogue rounds as the separate bf16 ops do)
    res = gen_act(M, N, seed=12).to(torch.bfloat16).to(cuda_device)
    plain = pk.penta_linear(x, packed, gamma, K, bias)
    fused = pk.penta_linear(x, packed, gamma, K, bias, act="gelu", residual=res)
    ref = (res.float() + torch.nn.functional.gelu(plain.float()).to(torch.bfloat16).float()).to(torch.bfloat16)
    assert torch.equal(fused, ref)


@pytest.mark.parametrize("scale_exp", [-100, -20, 0, 40, 100])
def test_gemv_activation_range(cuda_device, gemv_limit, scale_exp):
    """Per-token exponent: activations scaled by 2^e (exact in bf16) give the
    product scaled by 2^e, for tiny and huge magnitudes alike."""
    N, K, M = 256, 2000, 2
    packed, _, gamma = pk.quantize_and_pack(gen_weight(N, K, seed=13).to(cuda_device))
    packed = pk.pad_packed(packed)
    x = gen_act(M, K, seed=14).to(torch.bfloat16).to(cuda_device)
    y = pk.penta_linear(x, packed, gamma, K, out_dtype=torch.float32)
    ys = pk.penta_linear(x * (2.0 ** scale_exp), packed, gamma, K, out_dtype=torch.float32)
    assert torch.equal(ys, y * (2.0 ** scale_exp))
    # a zero token and a token with one large outlier (2^10: real activation
    # outliers reach ~1e3-1e4).  The codes enter as c = q + 2 and the row sum
    # of 2 x is subtracted at the end, so an outlier adds 2|x| to the partial
    # sums whatever its weight: the fp32 accumulation error grows with the
    # largest |x| of the row (as in the tensor-core decode path, whose
    # correction runs per 160-k block), not only with the output.
    x2 = x.clone()
    x2[0].zero_()
    x2[1, 7] = 2.0 ** 10
    w8 = orc.unpack(packed[:, :(K + 9) // 10].contiguous().cpu().numpy(), K)
    want = orc.matmul_f64(x2.float().cpu().numpy(), w8, gamma)
    got = pk.penta_linear(x2, packed, gamma, K, out_dtype=torch.float32).cpu().numpy()
    assert (got[0] == 0).all()
    assert_close(got[1], want[1], what="outlier token")


def test_gemv_limit_knob(cuda_device):
    L = nat.load()
    prev = L.pn_set_gemv_max_tokens(-1)  # query only
    assert 0 <= prev <= 8
    assert L.pn_set_gemv_max_tokens(9) == prev  # clamped to 8
    assert L.pn_set_gemv_max_tokens(prev) == 8
