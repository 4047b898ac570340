"""The stage-1 entry point that allocates nothing (fmka_route_ema_blend_noalloc).

It serves callers that cannot allocate device memory when they call the layer:
a serving runtime that reserved the whole GPU for its own pools, a real-time
path that must not trigger cudaMalloc's implicit synchronisation, or a C
program that links only this library. Its scratch is a fixed 4 MiB device array
inside the library instead of a caller workspace. These tests call it through
the C ABI and check it against the workspace entry point and an fp32
restatement of the gate, EMA and blend on two calls in a row (the array keeps
the previous call's contents, so the second call checks that what must start at
zero is cleared), and that shapes needing more scratch than the array holds are
refused before anything is launched.

This file is named to be collected last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _noalloc(lib, x, logits, b2, l3, beta, h, lam):
    B, T, D = x.shape
    L = logits.shape[1]
    stream = torch.cuda.current_stream().cuda_stream
    return lib.fmka_route_ema_blend_noalloc(
        x.data_ptr(), x.stride(0), x.stride(1), logits.data_ptr(), b2.data_ptr(), None, L,
        l3.data_ptr() if l3 is not None else None, l3.stride(0) if l3 is not None else 0,
        l3.stride(1) if l3 is not None else 0, l3.shape[1] if l3 is not None else 0, beta, B, T, D,
        h.data_ptr(), h.stride(0), h.stride(1), lam.data_ptr(), stream)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    from mka_b200 import _lib, ops

    lib = _lib.load()
    limit = lib.fmka_route_ema_blend_noalloc_scratch_bytes()
    assert limit == 4 << 20
    B, T, D, L = 2, 1000, 1024, 3
    assert lib.fmka_route_ema_blend_workspace_size(B, T, D) <= limit
    g = torch.Generator(device="cuda").manual_seed(21)
    x = torch.randn(B, T, D, generator=g, device="cuda").bfloat16()
    l3 = torch.randn(B, T, D, generator=g, device="cuda").bfloat16()
    logits = torch.randn(B * T, L, generator=g, device="cuda")
    b2 = torch.randn(L, generator=g, device="cuda")
    ref_h, ref_lam = ops.route_ema_blend(x, 0.9, logits=logits, b2=b2, levels=L, l3=l3)
    # an fp32 restatement as well, so that a fault shared by both entry points shows:
    # lam = softmax(logits + b2), L2 = EMA(x) from a zero state, h = lam0 x + lam1 L2 + lam2 L3
    lam32 = torch.softmax(logits + b2, -1).view(B, T, L)
    xf = x.float()
    ema = torch.empty_like(xf)
    st = torch.zeros(B, D, device="cuda")
    for t in range(T):
        st = 0.9 * st + 0.1 * xf[:, t]
        ema[:, t] = st
    h32 = lam32[..., 0:1] * xf + lam32[..., 1:2] * ema + lam32[..., 2:3] * l3.float()
    for _ in range(2):
        h = torch.full_like(x, float("nan"))
        lam = torch.full((B, T, L), float("nan"), device="cuda")
        rc = _noalloc(lib, x, logits, b2, l3, 0.9, h, lam)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        err = ((h.float() - ref_h.float()).abs().max() / ref_h.float().abs().max()).item()
        assert err < TOL
        assert (lam - ref_lam).abs().max().item() < 1e-6
        err32 = ((h.float() - h32).abs().max() / h32.abs().max()).item()
        assert err32 < TOL
        assert (lam - lam32).abs().max().item() < 1e-5
    assert ops.device_status() == 0


def test_noalloc_refuses_shapes_beyond_the_static_scratch():
    from mka_b200 import _lib

    lib = _lib.load()
    B, T, D = 8, 8192, 4096  # needs ~33 MB of scratch
    assert lib.fmka_route_ema_blend_workspace_size(B, T, D) > lib.fmka_route_ema_blend_noalloc_scratch_bytes()
    x = torch.zeros(1, 8, 8, device="cuda", dtype=torch.bfloat16)  # never read: refused before launch
    h = torch.empty_like(x)
    logits = torch.zeros(8, 2, device="cuda")
    lam = torch.empty(1, 8, 2, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.fmka_route_ema_blend_noalloc(x.data_ptr(), T * D, D, logits.data_ptr(), None, None, 2, None, 0, 0, 0,
                                          0.9, B, T, D, h.data_ptr(), T * D, D, lam.data_ptr(), stream)
    assert rc == 2  # FMKA_ERR_UNSUPPORTED
    code, msg = _lib.last_error()
    assert code == 2 and "static array" in msg
