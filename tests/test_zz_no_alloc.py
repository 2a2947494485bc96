"""pn_linear_bf16_nows: the packed linear for callers that cannot allocate.

pn_linear_bf16 asks its caller for a scratch workspace whenever a batch has
64 tokens or fewer.  A caller that may not allocate device memory -- code that
runs where no allocator may be called, or an embedding that only hands over raw
input and output pointers -- uses pn_linear_bf16_nows instead, which takes its
scratch from one fixed array compiled into the library.  These tests check that
it gives the same results as the workspace entry point, on two calls in a row
(the array keeps the previous call's bytes), and that it refuses shapes whose
scratch would not fit.  This file is collected last on purpose.
"""
import ctypes

import pytest
import torch

from _util import assert_close, gen_act, gen_weight
import penta_kernel as pk
import penta_native as nat


def _nows(x, packed, scale, K, y, y_dtype=nat.PN_F32):
    M = x.shape[0]
    N, KP = packed.shape
    stream = torch.cuda.current_stream(x.device).cuda_stream
    return nat.load().pn_linear_bf16_nows(x.data_ptr(), M, K, packed.data_ptr(), N, KP, ctypes.c_float(scale),
                                          None, y.data_ptr(), y_dtype, stream)


@pytest.mark.gpu
def test_nows_matches_workspace_entry_point(cuda_device):
    cases = [(1, 1024, 8192), (16, 512, 3072), (64, 384, 28672), (7, 300, 1001)]
    layers = {}
    for (M, N, K) in cases:
        if (N, K) not in layers:
            layers[(N, K)] = pk.quantize_and_pack(gen_weight(N, K, seed=N + K).to(cuda_device))
    for (M, N, K) in cases:
        packed, _, gamma = layers[(N, K)]
        # two calls in a row with different activations: the second must not
        # see anything the first left in the shared scratch
        for call in range(2):
            x = gen_act(M, K, seed=1000 * call + M).to(torch.bfloat16).to(cuda_device)
            want = pk.penta_linear(x, packed, gamma, K, out_dtype=torch.float32)
            y = torch.empty(M, N, dtype=torch.float32, device=cuda_device)
            st = _nows(x, packed, gamma, K, y)
            assert st == nat.PN_OK, nat.load().pn_last_error()
            torch.cuda.synchronize()
            assert_close(y.cpu().numpy(), want.cpu().numpy(), what=f"nows M={M} N={N} K={K} call {call}")
    # bf16 output with a bias goes through the same path
    packed, _, gamma = layers[(512, 3072)]
    x = gen_act(4, 3072, seed=5).to(torch.bfloat16).to(cuda_device)
    bias = torch.randn(512, device=cuda_device).to(torch.bfloat16)
    want = pk.penta_linear(x, packed, gamma, 3072, bias)
    y = torch.empty(4, 512, dtype=torch.bfloat16, device=cuda_device)
    N, KP = packed.shape
    st = nat.load().pn_linear_bf16_nows(x.data_ptr(), 4, 3072, packed.data_ptr(), N, KP, ctypes.c_float(gamma),
                                        bias.data_ptr(), y.data_ptr(), nat.PN_BF16,
                                        torch.cuda.current_stream().cuda_stream)
    assert st == nat.PN_OK
    assert torch.equal(y, want)
    assert nat.device_status(reset=True) == 0


def test_nows_rejects_scratch_beyond_its_array():
    """64 tokens at K = 65536 would need ~8.4 MB of scratch; the array holds
    4 MiB, so the call is refused before anything touches the device."""
    L = nat.load()
    P = 1 << 20
    st = L.pn_linear_bf16_nows(P, 64, 65536, P, 128, 6554, ctypes.c_float(1.0), None, P, nat.PN_BF16, None)
    assert st == nat.PN_ERR_WORKSPACE
    assert b"static array holds" in L.pn_last_error()
