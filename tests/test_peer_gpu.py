"""The kernels of the head-sharded layer's peer exchange, on one GPU with local
destination buffers standing in for the peers' memory:

  * attention whose output rows are split over several buffers equals the plain
    attention output bit for bit, row block by row block;
  * o_proj whose rows are written into several buffers equals the blocked GEMM
    (bit for bit where both take the CTA-pair kernel), and leaves every other
    row of the destinations untouched;
  * the flag barrier passes when every slot has arrived, and when a slot never
    arrives it ends after its time limit with FMKA_STATUS_PEER_TIMEOUT set
    (the wait runs out on a flag that nothing sets; no fault, no hang).

The same kernels across two GPUs are covered by test_sharded_gpu.py.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

PEER_TIMEOUT = 8  # FMKA_STATUS_PEER_TIMEOUT


@pytest.fixture(scope="module")
def ops():
    from mka_b200 import ops as _ops

    _ops.device_status(clear=True)
    return _ops


@pytest.mark.parametrize("B,Hq,Hkv,T,rows,ndst", [(1, 4, 1, 512, 128, 4), (2, 2, 1, 300, 100, 3),
                                                 (1, 8, 2, 640, 320, 2), (1, 2, 2, 200, 256, 1)])
def test_attention_rows_scattered_match_plain_attention(ops, B, Hq, Hkv, T, rows, ndst):
    g = torch.Generator(device="cuda").manual_seed(T + ndst)
    q = torch.randn(B, Hq, T, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, Hkv, T, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, Hkv, T, 128, device="cuda", generator=g).bfloat16()
    ref, _ = ops.attn_prefill(q, k, v, want_lse=False)  # [B, T, Hq, 128]
    # destination j holds rows [j*rows, (j+1)*rows) as [B, rows, Hq, 128]
    dst = [torch.full((B, rows, Hq, 128), 7.0, device="cuda").bfloat16() for _ in range(ndst)]
    ops.attn_prefill_scatter(q, k, v, [d.data_ptr() for d in dst], rows,
                             (dst[0].stride(0), dst[0].stride(1), dst[0].stride(2)))
    torch.cuda.synchronize()
    for j, d in enumerate(dst):
        t0, t1 = j * rows, min((j + 1) * rows, T)
        if t1 > t0:
            assert torch.equal(d[:, : t1 - t0], ref[:, t0:t1]), j
        assert bool((d[:, max(t1 - t0, 0):] == 7.0).all()), j  # rows past T untouched
    assert ops.device_status() == 0


def test_attention_scatter_rejects_uncovered_rows(ops):
    from mka_b200._lib import FastMKAError

    q = torch.zeros(1, 2, 300, 128, device="cuda").bfloat16()
    k = torch.zeros(1, 1, 300, 128, device="cuda").bfloat16()
    d = torch.zeros(1, 100, 2, 128, device="cuda").bfloat16()
    with pytest.raises(FastMKAError):
        ops.attn_prefill_scatter(q, k, k, [d.data_ptr(), d.data_ptr()], 100, (d.stride(0), d.stride(1), d.stride(2)))


@pytest.mark.parametrize("gs,M,width,N,row0,ndst,bias",
                         [(4, 512, 896, 3584, 512, 4, False), (2, 320, 512, 512, 0, 2, True),
                          (3, 200, 128, 640, 77, 3, True), (2, 96, 256, 384, 5, 1, False)])
def test_o_proj_rows_scattered_match_blocked_gemm(ops, gs, M, width, N, row0, ndst, bias):
    g = torch.Generator(device="cuda").manual_seed(M + N + gs)
    K = gs * width
    a = torch.randn(gs, M, width, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).bfloat16()
    b = torch.randn(N, device="cuda", generator=g) if bias else None
    rows_total = row0 + M + 9
    dst = [torch.full((rows_total, N), -3.0, device="cuda").bfloat16() for _ in range(ndst)]
    ops.gemm_kblocked_scatter(a, w, b, [d.data_ptr() for d in dst], row0, N)
    plain = ops.gemm_kblocked(a, w, b)
    ref = torch.cat(list(a.float().unbind(0)), dim=1) @ w.float().t()
    if b is not None:
        ref = ref + b
    torch.cuda.synchronize()
    for d in dst:
        got = d[row0:row0 + M]
        assert ((got.float() - ref).abs().max() / ref.abs().max()).item() < 1e-2
        if M > 128:  # both take the CTA-pair kernel: same sums in the same order
            assert torch.equal(got, plain)
        assert bool((d[:row0] == -3.0).all()) and bool((d[row0 + M:] == -3.0).all())
    assert ops.device_status() == 0


def _barrier(flag_tensors, rank, epoch):
    from mka_b200 import _lib

    arr = (ctypes.c_void_p * len(flag_tensors))(*[t.data_ptr() for t in flag_tensors])
    _lib.call("fmka_peer_barrier", arr, rank, len(flag_tensors), epoch, torch.cuda.current_stream().cuda_stream)


def test_barrier_single_rank_passes(ops):
    own = torch.zeros(8, dtype=torch.int32, device="cuda")
    for e in (1, 2, 3):
        _barrier([own], 0, e)
    torch.cuda.synchronize()
    assert own[0].item() == 3
    assert ops.device_status() == 0


def test_barrier_with_every_slot_arrived_passes(ops):
    # slot 1 already holds a later epoch: a peer that moved on counts as arrived
    own = torch.zeros(8, dtype=torch.int32, device="cuda")
    own[1] = 5
    other = torch.zeros(8, dtype=torch.int32, device="cuda")
    _barrier([own, other], 0, 4)
    torch.cuda.synchronize()
    assert other[0].item() == 4 and own[0].item() == 4
    assert ops.device_status() == 0


def test_barrier_times_out_on_a_missing_rank(ops):
    # rank 1 never arrives: nothing writes slot 1 of rank 0's array, so the
    # wait ends after its 2 s limit with the timeout bit set, and the GPU
    # context stays usable
    own = torch.zeros(8, dtype=torch.int32, device="cuda")
    other = torch.zeros(8, dtype=torch.int32, device="cuda")
    _barrier([own, other], 0, 1)
    torch.cuda.synchronize()
    assert other[0].item() == 1  # the announcement to rank 1 was still made
    assert ops.device_status(clear=True) & PEER_TIMEOUT
    x = torch.ones(4, device="cuda")
    assert (x * 2).sum().item() == 8.0
    assert ops.device_status() == 0
