"""Op-level numerics of every CUDA kernel against a plain PyTorch fp32 reference
of the same op, on small seeded shapes (edge cases included: ragged tiles, GQA,
causal offsets, tails). Module-level parity with the reference algorithm lives
in test_parity_gpu.py."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a = a.float()
    b = b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()


@pytest.fixture(scope="module")
def ops():
    from mka_b200 import ops as _ops

    return _ops


def _ref_attn(q, k, v, causal=True, scale=None):
    """fp32 reference: q [B,Hq,Tq,D], k/v [B,Hkv,Tk,D]; bottom-right causal."""
    B, Hq, Tq, D = q.shape
    Hkv, Tk = k.shape[1], k.shape[2]
    G = Hq // Hkv
    scale = scale or 1.0 / math.sqrt(D)
    kf = k.float().repeat_interleave(G, dim=1)
    vf = v.float().repeat_interleave(G, dim=1)
    s = torch.matmul(q.float(), kf.transpose(-1, -2)) * scale
    if causal:
        qi = torch.arange(Tk - Tq, Tk, device=q.device).view(Tq, 1)
        ki = torch.arange(Tk, device=q.device).view(1, Tk)
        s = s.masked_fill(ki > qi, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.matmul(torch.softmax(s, dim=-1), vf)
    return o, lse


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 384, 256), (1000, 1024, 1024), (77, 136, 3584),
                                   (4096, 2048, 512), (2500, 768, 1536), (40000, 512, 128),
                                   (64, 6144, 4096), (1, 256, 4096), (50, 384, 576), (33, 1000, 128),
                                   (300, 512, 576), (520, 256, 192)])
def test_gemm_plain(ops, M, N, K):
    """Includes odd numbers of 64-wide k-blocks (K = 576, 192) on the CTA-pair and
    split-K kernels, whose last two-k-block box then ends past K and is skipped."""
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g)
    out = ops.gemm(a, w, bias)
    ref = a.float() @ w.float().t() + bias
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("B,T,Hq,R,rope,act", [(2, 100, 2, 64, False, 1), (1, 256, 4, 512, True, 0),
                                                (3, 33, 2, 96, True, 1), (16, 1, 4, 256, True, 0),
                                                (60, 1, 2, 128, True, 1)])
def test_qr_proj(ops, B, T, Hq, R, rope, act):
    D = 256
    L = 3
    g = torch.Generator(device="cuda").manual_seed(7 + T)
    x = torch.randn(B * T, D, device="cuda", generator=g).bfloat16()
    w = (torch.randn(Hq * 128 + R, D, device="cuda", generator=g) / math.sqrt(D)).bfloat16()
    bias = torch.randn(Hq * 128 + R, device="cuda", generator=g) * 0.1
    w2 = torch.randn(L, R, device="cuda", generator=g) / math.sqrt(R)
    cs = None
    if rope:
        pos = torch.arange(T, device="cuda").float()
        inv = 1.0 / (10000 ** (torch.arange(0, 128, 2, device="cuda").float() / 128))
        ang = torch.cat([pos[:, None] * inv[None], pos[:, None] * inv[None]], -1)
        cs = (ang.cos(), ang.sin())
    q, logits = ops.qr_proj(x, w, bias, B, T, Hq, R, w2, L, act, rope=cs)
    full = x.float() @ w.float().t() + bias
    qf = full[:, : Hq * 128].view(B, T, Hq, 128).transpose(1, 2)
    if rope:
        cos, sin = cs
        rot = torch.cat([-qf[..., 64:], qf[..., :64]], -1)
        qf = qf * cos + rot * sin
    hid = full[:, Hq * 128:]
    hid = torch.nn.functional.silu(hid) if act == 0 else torch.nn.functional.gelu(hid)
    lg = hid @ w2.t()
    assert _rel(q, qf) < 1e-2
    assert _rel(logits, lg) < 1e-3


@pytest.mark.parametrize("rope", [False, True])
def test_kv_proj_with_offset(ops, rope):
    B, T, D, Hkv, Tcap, off = 2, 70, 384, 2, 100, 13
    g = torch.Generator(device="cuda").manual_seed(3)
    h = torch.randn(B * T, D, device="cuda", generator=g).bfloat16()
    w = (torch.randn(2 * Hkv * 128, D, device="cuda", generator=g) / math.sqrt(D)).bfloat16()
    bias = torch.randn(2 * Hkv * 128, device="cuda", generator=g) * 0.1
    kc = torch.zeros(B, Hkv, Tcap, 128, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    cs = None
    if rope:
        ang = torch.rand(B, T, 128, device="cuda", generator=g) * 6
        cs = (ang.cos(), ang.sin())
    ops.kv_proj(h, w, bias, B, T, Hkv, rope=cs, k_out=kc, v_out=vc, t_offset=off)
    full = h.float() @ w.float().t() + bias
    kf = full[:, : Hkv * 128].view(B, T, Hkv, 128).transpose(1, 2)
    vf = full[:, Hkv * 128:].view(B, T, Hkv, 128).transpose(1, 2)
    if rope:
        cos, sin = cs[0][:, None], cs[1][:, None]
        kf = kf * cos + torch.cat([-kf[..., 64:], kf[..., :64]], -1) * sin
    assert _rel(kc[:, :, off:off + T], kf) < 1e-2
    assert _rel(vc[:, :, off:off + T], vf) < 1e-2
    assert kc[:, :, :off].abs().max().item() == 0 and kc[:, :, off + T:].abs().max().item() == 0


def _ref_ema(x, beta):
    out = torch.zeros_like(x)
    st = torch.zeros_like(x[:, 0])
    for t in range(x.shape[1]):
        st = beta * st + (1 - beta) * x[:, t]
        out[:, t] = st
    return out


@pytest.mark.parametrize("B,T,D,L,T3,beta", [(2, 64, 256, 2, 0, 0.9), (2, 300, 520, 3, 1, 0.9),
                                             (1, 1000, 1024, 3, 700, 0.99), (3, 5, 264, 3, 9, 0.5),
                                             (1, 4100, 512, 2, 0, 0.999)])
def test_route_ema_blend(ops, B, T, D, L, T3, beta):
    g = torch.Generator(device="cuda").manual_seed(T + D)
    x = torch.randn(B, T, D, device="cuda", generator=g).bfloat16()
    logits = torch.randn(B * T, L, device="cuda", generator=g)
    b2 = torch.randn(L, device="cuda", generator=g)
    l3 = torch.randn(B, T3, D, device="cuda", generator=g).bfloat16() if L == 3 else None
    h, lam = ops.route_ema_blend(x, beta, logits=logits, b2=b2, levels=L, l3=l3)
    lam_ref = torch.softmax(logits + b2, -1).view(B, T, L)
    ema = _ref_ema(x.float(), beta)
    ref = lam_ref[..., 0:1] * x.float() + lam_ref[..., 1:2] * ema
    if L == 3:
        idx = torch.clamp(torch.arange(T, device="cuda"), max=T3 - 1)
        ref = ref + lam_ref[..., 2:3] * l3.float()[:, idx]
    assert ops.device_status() == 0
    assert _rel(lam, lam_ref) < 1e-5
    assert _rel(h, ref) < 1e-2


def test_causal_prefix_ema_op(ops):
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(2, 777, 136, device="cuda", generator=g).bfloat16()
    out = ops.causal_prefix_ema(x, 0.9)
    assert _rel(out, _ref_ema(x.float(), 0.9)) < 1e-2


@pytest.mark.parametrize("B,T,Hkv,rope,off,T3,beta,with_bias", [
    (2, 300, 4, True, 0, 0, 0.9, True), (3, 65, 1, True, 7, 0, 0.9, True), (1, 1, 2, False, 5, 0, 0.9, True),
    (2, 130, 8, True, 0, 0, 0.9, True), (4, 64, 4, False, 0, 0, 0.9, True), (2, 300, 4, True, 0, 1, 0.9, True),
    (3, 65, 1, True, 7, 40, 0.9, True), (2, 1000, 2, True, 3, 0, 0.9, False), (1, 700, 2, False, 0, 300, 0.5, False),
    (2, 600, 1, True, 0, 0, 0.99, True), (2, 500, 3, True, 2, 0, 0.9, True),
    (1, 3000, 2, True, 0, 3000, 0.9, True), (3, 32, 3, True, 4, 20, 0.9, False), (2, 7, 2, True, 9, 0, 0.9, True)])
def test_route_ema_blend_kv(ops, B, T, Hkv, rope, off, T3, beta, with_bias):
    """Stage 1 on y = x [Wk ; Wv]^T: K/V = lam0 y + lam1 EMA(y) (+ lam2 y3) + bias,
    RoPE on K, head-split at token slot t + off; y3 row t is min(t, T3 - 1).
    beta 0.99 takes the full look-back (the general kernel), the others the
    short one (the specialised K/V kernel)."""
    N = 2 * Hkv * 128
    L = 3 if T3 else 2
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + T)
    y = torch.randn(B * T, N, device="cuda", generator=g).bfloat16()
    logits = torch.randn(B * T, L, device="cuda", generator=g)
    b2 = torch.randn(L, device="cuda", generator=g)
    y3 = torch.randn(B, T3, N, device="cuda", generator=g).bfloat16() if T3 else None
    bias = torch.randn(N, device="cuda", generator=g) * 0.1 if with_bias else None
    cs = None
    if rope:
        ang = torch.rand(B, T, 128, device="cuda", generator=g) * 6
        cs = (ang.cos(), ang.sin())
    kc = torch.zeros(B, Hkv, T + off + 3, 128, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    _, _, lam = ops.route_ema_blend_kv(y, beta, logits, b2, B, T, Hkv, bias=bias, rope=cs, k_out=kc, v_out=vc,
                                       t_offset=off, y3=y3)
    lam_ref = torch.softmax(logits + b2, -1).view(B, T, L)
    yf = y.float().view(B, T, N)
    blend = lam_ref[..., 0:1] * yf + lam_ref[..., 1:2] * _ref_ema(yf, beta)
    if bias is not None:
        blend = blend + bias
    if T3:
        idx = torch.clamp(torch.arange(T, device="cuda"), max=T3 - 1)
        blend = blend + lam_ref[..., 2:3] * y3.float()[:, idx]
    kf = blend[..., : N // 2].reshape(B, T, Hkv, 128).transpose(1, 2)
    vf = blend[..., N // 2:].reshape(B, T, Hkv, 128).transpose(1, 2)
    if rope:
        cos, sin = cs[0][:, None], cs[1][:, None]
        kf = kf * cos + torch.cat([-kf[..., 64:], kf[..., :64]], -1) * sin
    assert ops.device_status() == 0
    assert _rel(lam, lam_ref) < 1e-5
    assert _rel(kc[:, :, off:off + T], kf) < 1e-2
    assert _rel(vc[:, :, off:off + T], vf) < 1e-2
    assert kc[:, :, :off].abs().max().item() == 0 if off else True
    assert kc[:, :, off + T:].abs().max().item() == 0 and vc[:, :, off + T:].abs().max().item() == 0


@pytest.mark.parametrize("T1,T2,D,beta", [(173, 127, 3584, 0.9), (64, 1, 136, 0.99), (1, 1, 264, 0.5),
                                         (700, 45, 520, 0.999)])
def test_ema_carried_state(ops, T1, T2, D, beta):
    """Two calls with the state carried equal one call over the whole sequence:
    the EMA of the reference (L2[-1] = 0, session_memory.py:6-22) continued."""
    g = torch.Generator(device="cuda").manual_seed(T1 * 31 + T2)
    B = 2
    x = torch.randn(B, T1 + T2, D, device="cuda", generator=g).bfloat16()
    s1 = torch.empty(B, D, device="cuda")
    s2 = torch.empty(B, D, device="cuda")
    a = ops.causal_prefix_ema(x[:, :T1].contiguous(), beta, state_out=s1)
    b = ops.causal_prefix_ema(x[:, T1:].contiguous(), beta, state=s1, state_out=s2)
    whole = ops.causal_prefix_ema(x, beta)
    ref = _ref_ema(x.float(), beta)
    assert ops.device_status() == 0
    assert _rel(a, ref[:, :T1]) < 1e-2
    assert _rel(b, ref[:, T1:]) < 1e-2
    assert (b.float() - whole[:, T1:].float()).abs().max().item() <= 2 ** -7 * ref.abs().max().item()
    # the carried states are fp32: they match the fp32 recurrence closely
    assert _rel(s1, ref[:, T1 - 1]) < 1e-4
    assert _rel(s2, ref[:, -1]) < 1e-4
    # a state on a blend with a gate and a third level goes through the same scan
    gate = torch.rand(B * T2, 3, device="cuda", generator=g)
    gate = gate / gate.sum(-1, keepdim=True)
    l3 = torch.randn(B, 1, D, device="cuda", generator=g).bfloat16()
    h, _ = ops.route_ema_blend(x[:, T1:].contiguous(), beta, gate=gate, levels=3, l3=l3, ema_state=s1)
    gv = gate.view(B, T2, 3)
    want = gv[..., 0:1] * x[:, T1:].float() + gv[..., 1:2] * ref[:, T1:] + gv[..., 2:3] * l3.float()
    assert _rel(h, want) < 1e-2
    with pytest.raises(Exception):
        ops.causal_prefix_ema(x[:, :T1].contiguous(), beta, state=s1, state_out=s1)


@pytest.mark.parametrize("B,Hq,Hkv,Tq,Tk,causal", [(1, 1, 1, 128, 128, True), (2, 4, 2, 200, 200, True),
                                                   (1, 7, 1, 300, 300, True), (2, 2, 2, 64, 333, True),
                                                   (1, 2, 1, 130, 257, False), (1, 4, 4, 1024, 1024, True),
                                                   (1, 2, 1, 700, 1500, True), (2, 3, 3, 520, 520, False),
                                                   (1, 7, 1, 1536, 1536, True)])
def test_attn_prefill(ops, B, Hq, Hkv, Tq, Tk, causal):
    g = torch.Generator(device="cuda").manual_seed(Tq * 7 + Tk)
    q = torch.randn(B, Hq, Tq, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, Hkv, Tk, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, Hkv, Tk, 128, device="cuda", generator=g).bfloat16()
    o, lse = ops.attn_prefill(q, k, v, causal=causal)
    ro, rlse = _ref_attn(q, k, v, causal)
    assert ops.device_status() == 0
    assert _rel(o, ro.transpose(1, 2)) < 2e-2
    assert (lse - rlse).abs().max().item() < 2e-2


@pytest.mark.parametrize("B,Hq,Hkv,Tk,splits", [(2, 4, 1, 100, 0), (3, 32, 8, 2000, 0), (1, 28, 4, 4096, 3),
                                                (4, 8, 8, 64, 1), (2, 16, 1, 777, 0)])
def test_attn_decode(ops, B, Hq, Hkv, Tk, splits):
    g = torch.Generator(device="cuda").manual_seed(Tk)
    q = torch.randn(B, Hq, 1, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, Hkv, Tk, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, Hkv, Tk, 128, device="cuda", generator=g).bfloat16()
    o, lse = ops.attn_decode(q, k, v, num_splits=splits)
    ro, rlse = _ref_attn(q, k, v, causal=True)
    assert ops.device_status() == 0
    assert _rel(o, ro.transpose(1, 2)) < 2e-2
    assert (lse - rlse[..., 0]).abs().max().item() < 2e-2


@pytest.mark.parametrize("B,Hq,Hkv,Tq,Tk", [(1, 4, 2, 200, 333), (2, 2, 1, 128, 128), (1, 3, 1, 1, 700)])
def test_attention_known_answers(ops, B, Hq, Hkv, Tq, Tk):
    """Closed forms: with every key zero all scores are equal, so a query row
    that sees n keys has lse = log n and its output is the mean of those value
    rows, which is the value row itself when the rows are constant per head."""
    g = torch.Generator(device="cuda").manual_seed(Tq + Tk)
    q = torch.randn(B, Hq, Tq, 128, device="cuda", generator=g).bfloat16()
    k = torch.zeros(B, Hkv, Tk, 128, device="cuda").bfloat16()
    c = torch.randn(B, Hkv, 1, 128, device="cuda", generator=g).bfloat16()
    v = c.expand(B, Hkv, Tk, 128).contiguous()
    G = Hq // Hkv
    want_o = c[:, :, 0].repeat_interleave(G, dim=1)  # [B, Hq, 128]
    o, lse = ops.attn_prefill(q, k, v, causal=True)
    n = torch.arange(Tk - Tq + 1, Tk + 1, device="cuda", dtype=torch.float32)  # keys seen by each row
    assert _rel(o, want_o[:, None].expand(B, Tq, Hq, 128)) < 2e-3
    assert (lse - n.log()).abs().max().item() < 1e-3
    if Tq == 1:
        od, lsed = ops.attn_decode(q, k, v)
        assert _rel(od[:, 0], want_o) < 2e-3
        assert (lsed - math.log(Tk)).abs().max().item() < 1e-3
    assert ops.device_status() == 0


@pytest.mark.parametrize("M,I,K,bias", [(1, 128, 256, False), (64, 384, 512, True), (100, 1408, 256, False),
                                        (300, 256, 1024, True), (1000, 1408, 512, False)])
def test_gemm_swiglu(ops, M, I, K, bias):
    """silu(x Wg^T + bg) * (x Wu^T + bu) from one GEMM over the interleaved weight."""
    g = torch.Generator(device="cuda").manual_seed(M + I + K)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    wg = (torch.randn(I, K, device="cuda", generator=g) / math.sqrt(K)).bfloat16()
    wu = (torch.randn(I, K, device="cuda", generator=g) / math.sqrt(K)).bfloat16()
    bg = torch.randn(I, device="cuda", generator=g) if bias else None
    bu = torch.randn(I, device="cuda", generator=g) if bias else None
    w_gu = ops.interleave_gate_up(wg, wu)
    b_gu = ops.interleave_gate_up(bg, bu) if bias else None
    out = ops.gemm_swiglu(x, w_gu, b_gu)
    gate = x.float() @ wg.float().t() + (bg if bias else 0.0)
    up = x.float() @ wu.float().t() + (bu if bias else 0.0)
    ref = torch.nn.functional.silu(gate) * up
    assert out.shape == (M, I)
    assert ops.device_status() == 0
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("nblk,M,kb,N", [(2, 300, 896, 384), (4, 1024, 128, 512), (1, 77, 256, 256),
                                         (3, 40, 256, 384)])
def test_gemm_kblocked(ops, nblk, M, kb, N):
    """A given as blocks of columns (the all-gathered attention output of a head-sharded layer)."""
    g = torch.Generator(device="cuda").manual_seed(nblk * M)
    blocks = torch.randn(nblk, M, kb, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, nblk * kb, device="cuda", generator=g) / math.sqrt(nblk * kb)).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g)
    out = ops.gemm_kblocked(blocks, w, bias)
    a = blocks.permute(1, 0, 2).reshape(M, nblk * kb).float()
    assert _rel(out, a @ w.float().t() + bias) < 1e-2


@pytest.mark.parametrize("rows,D", [(1, 4096), (300, 4096), (77, 1024), (5, 520), (3, 8192), (1000, 3584)])
def test_rmsnorm_matches_transformers(ops, rows, D):
    """The one-pass RMSNorm against transformers' LlamaRMSNorm on the same bf16
    input and weight (same two roundings; the fp32 sum of squares runs in a
    different order, so a few elements differ by a bf16 step or two) and against
    an fp32 restatement."""
    from transformers.models.llama.modeling_llama import LlamaRMSNorm

    g = torch.Generator(device="cuda").manual_seed(rows + D)
    x = (torch.randn(rows, D, device="cuda", generator=g) * 3).bfloat16()
    norm = LlamaRMSNorm(D, eps=1e-5).cuda().to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(D, device="cuda", generator=g))
        ref = norm(x)
    y = ops.rmsnorm(x, norm.weight.detach(), 1e-5)
    assert y.shape == x.shape and y.dtype == torch.bfloat16
    diff = (y.float() - ref.float()).abs()
    # a sum-order difference can move the first rounding by one step, which the
    # product with the weight carries into y: allow a few bf16 steps, rarely
    assert (diff <= ref.float().abs() * 2 ** -6 + 2 ** -14).all()
    assert (diff == 0).float().mean().item() > 0.99
    xf = x.float()
    r32 = norm.weight.float() * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5))
    assert _rel(y, r32) < 1e-2
    assert ops.device_status() == 0


@pytest.mark.parametrize("shape,inplace", [((96, 512), False), ((3, 1000, 344), True), ((8,), False),
                                           ((257, 14336), True)])
def test_silu_mul_matches_transformers(ops, shape, inplace):
    """bf16(bf16(silu(g)) * u) in one pass against torch's act_fn(gate) * up on
    the same bf16 tensors (two kernels, same roundings; the exponential may
    differ by an fp32 ulp, which can move a rare element by one bf16 step), and
    against an fp32 restatement. inplace: the product overwrites g."""
    n = 1
    for s in shape:
        n *= s
    g = torch.Generator(device="cuda").manual_seed(n)
    gt = (torch.randn(*shape, device="cuda", generator=g) * 4).bfloat16()
    ut = (torch.randn(*shape, device="cuda", generator=g) * 2).bfloat16()
    ref = torch.nn.functional.silu(gt) * ut
    r32 = torch.nn.functional.silu(gt.float()) * ut.float()
    gin = gt.clone()
    y = ops.silu_mul(gin, ut, out=gin if inplace else None)
    if inplace:
        assert y.data_ptr() == gin.data_ptr()
    assert y.shape == gt.shape and y.dtype == torch.bfloat16
    diff = (y.float() - ref.float()).abs()
    assert (diff <= ref.float().abs() * 2 ** -7 + 2 ** -30).all()
    assert (diff == 0).float().mean().item() > 0.99
    assert _rel(y, r32) < 1e-2
    assert ops.device_status() == 0
