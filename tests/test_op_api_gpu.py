"""GPU parity of the reference's low-level op API (mka/cuda/ops.py) as exposed by
mka_b200.cuda, against the CPU oracle's restatement of the reference kernels.

  fastmka_attn(q, k, v, causal)            mka/cuda/ops.py:73-77, fastmka_attn.cu:51-131
  fused_route_mka_attn(q, l1, l2, l3, lam, wk, wv)
                                           mka/cuda/ops.py:47-70, fused_route_mka.cu:23-102

Tolerance (bf16 kernels vs the fp32 oracle): max |err| / max |ref| <= 2e-2.
"""
import pytest
import torch

from oracle import fastmka_oracle as orc

pytestmark = pytest.mark.gpu
TOL = 2e-2


def nrel(a, b):
    a = a.detach().float().cpu()
    b = b.detach().float().cpu()
    assert a.shape == b.shape, (a.shape, b.shape)
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()


def _bf16_exact(*shape, gen, scale=1.0):
    return (torch.randn(*shape, generator=gen) * scale).bfloat16().float()


@pytest.mark.parametrize("b,h,hkv,tq,tk,causal", [
    (2, 4, 4, 64, 64, True),      # MHA, square
    (1, 2, 2, 100, 300, True),    # cache in front: causal offset Tk - Tq = 200
    (2, 3, 3, 77, 77, False),     # non-causal, ragged tile
    (2, 4, 4, 1, 513, True),      # one query token: the decode path
    (1, 8, 2, 130, 130, True),    # GQA extension (group of 4)
    (1, 2, 2, 160, 40, True),     # Tq > Tk: the first 120 queries see no key -> zero rows
])
def test_fastmka_attn_matches_oracle(b, h, hkv, tq, tk, causal):
    from mka_b200 import cuda as mka_cuda

    g = torch.Generator().manual_seed(b * 1000 + tq + tk)
    q = _bf16_exact(b, h, tq, 128, gen=g)
    k = _bf16_exact(b, hkv, tk, 128, gen=g)
    v = _bf16_exact(b, hkv, tk, 128, gen=g)
    ref = orc.fastmka_attn_op(q, k, v, causal)
    out = mka_cuda.fastmka_attn(q.cuda().bfloat16(), k.cuda().bfloat16(), v.cuda().bfloat16(), causal)
    assert out.shape == (b, h, tq, 128) and out.dtype == torch.bfloat16
    assert nrel(out, ref) < TOL
    if causal and tq > tk:
        assert out[:, :, : tq - tk].abs().max().item() == 0.0


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_fastmka_attn_returns_input_dtype(dtype):
    """The reference dispatches fp32/fp16 (AT_DISPATCH_FLOATING_TYPES_AND_HALF) and
    returns q's dtype; the B200 op computes in bf16 and converts back."""
    from mka_b200 import cuda as mka_cuda

    g = torch.Generator().manual_seed(11)
    q, k, v = (_bf16_exact(1, 2, 96, 128, gen=g) for _ in range(3))
    out = mka_cuda.fastmka_attn(q.cuda().to(dtype), k.cuda().to(dtype), v.cuda().to(dtype), True)
    assert out.dtype == dtype
    assert nrel(out, orc.fastmka_attn_op(q, k, v, True)) < TOL


@pytest.mark.parametrize("levels", [2, 3])
@pytest.mark.parametrize("b,h,t", [(2, 2, 96), (1, 4, 200)])
def test_fused_route_mka_attn_matches_oracle(levels, b, h, t):
    """MHA (H * Dh == D): fused = sum_l lam_l l_l, k/v = fused wk^T / wv^T, causal
    attention with q; the gate comes from a softmax so it sums to one per token."""
    from mka_b200 import cuda as mka_cuda

    d = h * 128
    g = torch.Generator().manual_seed(levels * 100 + t)
    q = _bf16_exact(b, h, t, 128, gen=g, scale=0.5)
    l1 = _bf16_exact(b, t, d, gen=g)
    l2 = orc.causal_prefix_ema(l1, 0.9).bfloat16().float()
    l3 = _bf16_exact(b, t, d, gen=g, scale=0.5)
    lam = torch.softmax(torch.randn(b, t, levels, generator=g), -1)
    wk = _bf16_exact(d, d, gen=g, scale=d ** -0.5)
    wv = _bf16_exact(d, d, gen=g, scale=d ** -0.5)
    ref = orc.fused_route_mka_op(q, l1, l2, l3, lam, wk, wv)
    out = mka_cuda.fused_route_mka_attn(*(x.cuda() for x in (q, l1, l2, l3, lam, wk, wv)))
    assert out.shape == (b, h, t, 128) and out.dtype == torch.float32
    assert nrel(out, ref) < TOL


def test_fused_route_mka_attn_rejects_reference_errors():
    """The reference's TORCH_CHECKs (fused_route_mka.cu:112-132) surface as RuntimeError."""
    from mka_b200 import cuda as mka_cuda

    dev = "cuda"
    q = torch.zeros(1, 2, 16, 128, device=dev)
    x = torch.zeros(1, 16, 256, device=dev)
    w = torch.zeros(256, 256, device=dev)
    with pytest.raises(RuntimeError, match="2 or 3"):
        mka_cuda.fused_route_mka_attn(q, x, x, x, torch.zeros(1, 16, 4, device=dev), w, w)
    with pytest.raises(RuntimeError, match="shapes must match"):
        mka_cuda.fused_route_mka_attn(q, x, x, torch.zeros(1, 15, 256, device=dev), torch.zeros(1, 16, 2, device=dev),
                                      w, w)
    with pytest.raises(RuntimeError, match="H\\*Dh == D"):
        mka_cuda.fused_route_mka_attn(q[:, :1], x, x, x, torch.zeros(1, 16, 2, device=dev), w, w)
