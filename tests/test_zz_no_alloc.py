"""pn_linear_bf16_nows: the packed linear for callers that cannot allocate.

pn_linear_bf16 asks its caller for a scratch workspace.  A caller that may not
allocate device memory -- code that runs where no allocator may be called, or
an embedding that only hands over raw input and output pointers -- uses
pn_linear_bf16_nows instead, which takes its scratch from one fixed array
compiled into the library.  These tests check that it gives the same results
as the workspace entry point, on two calls in a row (the array keeps the
previous call's bytes), including realistic layers whose K_packs is not a
multiple of 4 when their rows are stored at the padded stride, and that it
refuses shapes whose scratch would not fit.  This file is collected last on
purpose.
"""
import ctypes

import pytest
import torch

from _util import assert_close, gen_act, gen_weight
import penta_kernel as pk
import penta_native as nat


def _nows(x, packed, scale, K, y, y_dtype=nat.PN_F32, bias=None):
    """Calls the entry point on `packed`, a (N, K_packs) tensor whose rows may
    sit at a padded stride (packed.stride(0) words apart)."""
    M = x.shape[0]
    N, KP = packed.shape
    stream = torch.cuda.current_stream(x.device).cuda_stream
    return nat.load().pn_linear_bf16_nows(x.data_ptr(), M, K, packed.data_ptr(), N, KP, packed.stride(0),
                                          ctypes.c_float(scale), None if bias is None else bias.data_ptr(),
                                          y.data_ptr(), y_dtype, stream)


@pytest.mark.gpu
def test_nows_matches_workspace_entry_point(cuda_device):
    # (M, N, K, padded rows): K = 8192 / 3072 / 28672 have K_packs % 4 == 0;
    # K = 4096 (410 words), 768 (77) and 1001 (101) do not, and are called with
    # their rows at pn_packed_ld(K_packs), as resident layers store them.
    cases = [(1, 1024, 8192, False), (16, 512, 3072, False), (64, 384, 28672, False), (7, 300, 1001, True),
             (1, 4096, 4096, True), (64, 4096, 4096, True), (8, 11008, 4096, True), (3, 3072, 768, True)]
    layers = {}
    for (M, N, K, pad) in cases:
        if (N, K, pad) not in layers:
            packed, _, gamma = pk.quantize_and_pack(gen_weight(N, K, seed=N + K).to(cuda_device))
            layers[(N, K, pad)] = (pk.pad_packed(packed) if pad else packed, gamma)
    for (M, N, K, pad) in cases:
        packed, gamma = layers[(N, K, pad)]
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
    packed, gamma = layers[(512, 3072, False)]
    x = gen_act(4, 3072, seed=5).to(torch.bfloat16).to(cuda_device)
    bias = torch.randn(512, device=cuda_device).to(torch.bfloat16)
    want = pk.penta_linear(x, packed, gamma, 3072, bias)
    y = torch.empty(4, 512, dtype=torch.bfloat16, device=cuda_device)
    assert _nows(x, packed, gamma, 3072, y, nat.PN_BF16, bias) == nat.PN_OK
    assert torch.equal(y, want)
    assert nat.device_status(reset=True) == 0


@pytest.mark.gpu
def test_nows_unpadded_rows_of_a_large_layer_are_refused(cuda_device):
    """A 4096 -> 4096 layer stored at K_packs = 410 words per row would need a
    6.9 MB re-pitched copy of its weights, more than the array holds: the call
    is refused, and the message names the padded stride that makes it fit."""
    N, K = 4096, 4096
    packed, _, gamma = pk.quantize_and_pack(gen_weight(N, K, seed=3).to(cuda_device))
    assert packed.stride(0) == 410
    x = gen_act(1, K, seed=1).to(torch.bfloat16).to(cuda_device)
    y = torch.zeros(1, N, dtype=torch.float32, device=cuda_device)
    assert _nows(x, packed, gamma, K, y) == nat.PN_ERR_WORKSPACE
    msg = nat.load().pn_last_error()
    assert b"pn_packed_ld" in msg and b"412" in msg, msg
    torch.cuda.synchronize()
    assert torch.count_nonzero(y) == 0  # nothing was enqueued


def test_nows_rejects_scratch_beyond_its_array():
    """64 tokens at K = 65536 would need ~8.4 MB of scratch; the array holds
    4 MiB, so the call is refused before anything touches the device."""
    L = nat.load()
    P = 1 << 20
    st = L.pn_linear_bf16_nows(P, 64, 65536, P, 128, 6554, 6556, ctypes.c_float(1.0), None, P, nat.PN_BF16, None)
    assert st == nat.PN_ERR_WORKSPACE
    assert b"static array holds" in L.pn_last_error()


def test_nows_reports_bad_shapes_as_shape_errors():
    """Shape errors are reported as such, not as a scratch size computed from
    the bad shape."""
    L = nat.load()
    P = 1 << 20
    for (M, K, KP, ld) in ((64, 65536, 6553, 6556), (-1, 4096, 410, 412), (1, 0, 0, 0), (1, 4096, 410, 409)):
        st = L.pn_linear_bf16_nows(P, M, K, P, 128, KP, ld, ctypes.c_float(1.0), None, P, nat.PN_BF16, None)
        assert st == nat.PN_ERR_SHAPE, (M, K, KP, ld, st)
