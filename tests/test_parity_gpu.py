"""Module-level parity of the B200 path with the FastLM/MKA reference.

Tolerance (bf16 kernels vs the fp32 reference): max |err| / max |ref| <= 2e-2 on
the layer output, k, v and the attention log-sum-exp; the gate lambda within
2e-2 absolute.
  * golden fixtures: the reference modules' own outputs (tests/golden)
  * the single-layer fp32 configuration at full size against the CPU oracle
  * the Qwen-7B-like prefill layer on one whole sequence of 8192 tokens against
    the CPU oracle (out, k, v, gate, LSE)
  * the long-context layer (three levels, per-position L3 memory, GQA, RoPE) at
    full width on one whole sequence of 4096 tokens, and at a small width with
    L3 memories that are truncated, padded and repeated
  * the Qwen-7B-like prefill layer at the full batch (batch 4, seq 8192)
    through size-independent checks: exact softmax rows recomputed in fp32 for
    sampled queries, the EMA/blend recurrence for sampled channels, and the
    causal prefix property
"""
import math

import pytest
import torch
import torch.nn as nn

from oracle import fastmka_oracle as orc
from tests import golden_io

pytestmark = pytest.mark.gpu
TOL = 2e-2


def nrel(a, b):
    a = a.detach().float().cpu()
    b = b.detach().float().cpu()
    assert a.shape == b.shape, (a.shape, b.shape)
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()


def _load_fastmka(case):
    from mka_b200 import FastMKAAttention, FastMKAConfig

    p = golden_io.params(case)
    d = p["wq.weight"].shape[0]
    r = p["router.0.weight"].shape[0]
    cfg = FastMKAConfig(hidden_size=d, num_heads=int(case["heads"]), use_l3=bool(case["use_l3"]),
                        ema_beta=float(case["beta"]), router_hidden=r,
                        router_act="gelu" if int(case["act"]) == 1 else "silu")
    m = FastMKAAttention(cfg)
    m.load_state_dict(p)
    return m.cuda().eval()


@pytest.mark.parametrize("name", ["fastmka_mha_gelu", "fastmka_mha_l3_pad", "fastmka_mha_l3_single",
                                  "fastmka_mha_cache", "fastmka_mha_decode"])
def test_fastmka_golden(name):
    c = golden_io.load(name)
    m = _load_fastmka(c)
    x = c["x"].cuda()
    kw = {}
    if "l3" in c:
        kw["l3_memory"] = c["l3"].cuda()
    if "past_k" in c:
        kw["kv_cache_k"] = c["past_k"].cuda()
        kw["kv_cache_v"] = c["past_v"].cuda()
    out, k, v, lam, lse = m.forward_with_lse(x, **kw)
    assert out.dtype == torch.float32  # returned in the input dtype
    assert nrel(out, c["out"]) < TOL
    assert nrel(k, c["k"]) < TOL
    assert nrel(v, c["v"]) < TOL
    assert (lam.cpu() - c["lam"]).abs().max().item() < TOL
    assert nrel(lse, c["lse"]) < TOL
    from mka_b200 import ops

    assert ops.device_status() == 0


def _hf_module(case, kind):
    from transformers import LlamaConfig, Qwen2Config
    from transformers.models.llama.modeling_llama import LlamaAttention
    from transformers.models.qwen2.modeling_qwen2 import Qwen2Attention, Qwen2RotaryEmbedding

    from mka_b200 import HFFastMKAAttention

    p = golden_io.params(case)
    d = p["q_proj.weight"].shape[1]
    h, hkv = int(case["heads"]), int(case["kv_heads"])
    if kind == "qwen":
        cfg = Qwen2Config(hidden_size=d, num_attention_heads=h, num_key_value_heads=hkv, intermediate_size=1024,
                          vocab_size=128, rope_theta=10000.0)
        att = Qwen2Attention(cfg, layer_idx=0)
        att.rotary_emb = Qwen2RotaryEmbedding(cfg)
    else:
        cfg = LlamaConfig(hidden_size=d, num_attention_heads=h, num_key_value_heads=hkv, intermediate_size=1024,
                          vocab_size=128)
        att = LlamaAttention(cfg, layer_idx=0)
    w = HFFastMKAAttention(att, use_l3=bool(case["use_l3"]), ema_beta=float(case["beta"]))
    r = p["router.0.weight"].shape[0]
    if r != d // 2:
        w.router = nn.Sequential(nn.Linear(d, r), nn.SiLU(), nn.Linear(r, p["router.2.weight"].shape[0]))
    missing, unexpected = w.load_state_dict(p, strict=False)
    assert not unexpected
    assert all(k.startswith("original_attn.") or k.startswith("rotary_emb.") or "rotary_emb" in k
               for k in missing), missing
    return w.cuda().eval()


@pytest.mark.parametrize("name,kind", [("hf_qwen_rope", "qwen"), ("hf_qwen_decode", "qwen"),
                                       ("hf_llama_norope", "llama")])
def test_hf_golden(name, kind):
    c = golden_io.load(name)
    w = _hf_module(c, kind)
    x = c["x"].cuda()
    kw = {"use_cache": True}
    if "cos" in c:
        kw["position_embeddings"] = (c["cos"].cuda(), c["sin"].cuda())
    if "past_k" in c:
        kw["past_key_value"] = (c["past_k"].cuda(), c["past_v"].cuda())
    out, _, present, lse, lam = w.forward_with_lse(x, **kw)
    assert nrel(out, c["out"]) < TOL
    assert nrel(present[0], c["k"]) < TOL
    assert nrel(present[1], c["v"]) < TOL
    assert (lam.cpu() - c["lam"]).abs().max().item() < TOL
    assert nrel(lse, c["lse"]) < TOL


def test_hf_decode_with_static_cache_matches_concat():
    """The in-place cache path gives the same step as the reference's concatenation."""
    from mka_b200 import StaticKVCache

    c = golden_io.load("hf_qwen_decode")
    w = _hf_module(c, "qwen")
    cache = StaticKVCache(batch=2, num_kv_heads=2, capacity=64, num_layers=1, device="cuda")
    cache.load_prefix(0, c["past_k"].cuda().bfloat16(), c["past_v"].cuda().bfloat16())
    out, _, present = w(c["x"].cuda(), position_embeddings=(c["cos"].cuda(), c["sin"].cuda()),
                        past_key_value=cache, use_cache=True)
    assert cache.lengths[0] == c["past_k"].shape[2] + 1
    assert nrel(out, c["out"]) < TOL
    assert nrel(present[0], c["k"]) < TOL


def test_single_layer_fp32_config_full_size():
    """batch 2, seq 512, d_model 1024, 8/8 heads, L1+L2, router 1024->256->2 GELU,
    X ~ N(0,1), Xavier-uniform weights, seed 0: B200 module vs the CPU oracle."""
    from mka_b200 import FastMKAAttention, FastMKAConfig

    torch.manual_seed(0)
    m = FastMKAAttention(FastMKAConfig(hidden_size=1024, num_heads=8, use_l3=False, router_hidden=256,
                                       router_act="gelu"))
    for mod in m.modules():
        if isinstance(mod, nn.Linear):
            nn.init.xavier_uniform_(mod.weight)
    x = torch.randn(2, 512, 1024)
    p = {"wq": m.wq.weight, "wk": m.wk.weight, "wv": m.wv.weight, "wo": m.wo.weight,
         "r1w": m.router[0].weight, "r1b": m.router[0].bias, "r2w": m.router[2].weight, "r2b": m.router[2].bias}
    with torch.no_grad():
        ref = orc.fastmka_forward(x, {k: v.detach() for k, v in p.items()}, 8, False, 0.9, "gelu")
    m = m.cuda().eval()
    out, k, v, lam, lse = m.forward_with_lse(x.cuda())
    assert nrel(out, ref["out"]) < TOL
    assert nrel(k, ref["k_tot"]) < TOL
    assert nrel(v, ref["v_tot"]) < TOL
    assert (lam.cpu() - ref["lam"]).abs().max().item() < TOL
    assert nrel(lse, ref["lse"]) < TOL


def _qwen_like_layer(B, T, seed=0, use_l3=False):
    """The Qwen-7B-like prefill layer: d_model 3584, 28/4 heads, router 3584->512->L,
    weights N(0, 0.02), X ~ N(0,1)/sqrt(3584), seeded."""
    from mka_b200.layers.prepared import prepare

    D, H, HKV, R = 3584, 28, 4, 512
    L = 3 if use_l3 else 2
    g = torch.Generator(device="cuda").manual_seed(seed)
    lin = lambda o, i, bias: nn.Linear(i, o, bias=bias)  # noqa: E731
    mods = {"q": lin(H * 128, D, True), "k": lin(HKV * 128, D, True), "v": lin(HKV * 128, D, True),
            "o": lin(D, H * 128, False)}
    router = nn.Sequential(nn.Linear(D, R), nn.SiLU(), nn.Linear(R, L))
    with torch.no_grad():
        for m in list(mods.values()) + [router[0], router[2]]:
            m.weight.copy_(torch.randn(m.weight.shape, generator=g, device="cuda") * 0.02)
            if m.bias is not None:
                m.bias.copy_(torch.randn(m.bias.shape, generator=g, device="cuda") * 0.02)
    for m in list(mods.values()) + [router]:
        m.cuda()
    W = prepare(mods["q"], mods["k"], mods["v"], mods["o"], router, torch.device("cuda"))
    x = (torch.randn(B, T, D, generator=g, device="cuda") / math.sqrt(D)).bfloat16()
    return mods, router, W, x


def test_qwen_like_prefill_full_size_sampled_rows():
    """Full configuration (batch 4, seq 8192): attention rows recomputed exactly in
    fp32 from the kernel's own q/k/v for sampled queries; the K/V projection and
    EMA/blend for sampled tokens; causal prefix property on the layer output."""
    from mka_b200.layers.forward import fastmka_forward

    B, T = 4, 8192
    mods, router, W, x = _qwen_like_layer(B, T)
    r = fastmka_forward(x, W, 28, 4, 0.9, False)
    q, k, v, lse = r["q"], r["k"], r["v"], r["lse"]
    # attention rows
    rows = [0, 1, 127, 128, 4095, 5000, 8190, 8191]
    from mka_b200 import ops

    o_full, _ = ops.attn_prefill(q, k, v)
    for b in (0, 3):
        for hq in (0, 13, 27):
            kk = k[b, hq // 7].float()
            vv = v[b, hq // 7].float()
            for t in rows:
                s = (kk[: t + 1] @ q[b, hq, t].float()) / math.sqrt(128)
                ref_lse = torch.logsumexp(s, 0)
                ref_o = torch.softmax(s, 0) @ vv[: t + 1]
                assert abs(lse[b, hq, t].item() - ref_lse.item()) < TOL * max(1.0, abs(ref_lse.item()))
                assert nrel(o_full[b, t, hq], ref_o) < TOL
    # EMA / blend / K-projection recurrence for sampled tokens of batch row 1
    xf = x[1].float()
    beta = 0.9
    st = torch.zeros(3584, device="cuda")
    ema = torch.empty(T, 3584, device="cuda")
    for t in range(T):
        st = beta * st + (1 - beta) * xf[t]
        ema[t] = st
    with torch.no_grad():
        qf = mods["q"](xf)
        lam = torch.softmax(router(qf), -1)
        for t in (0, 63, 64, 2047, 8191):
            assert (r["lam"][1, t].float() - lam[t]).abs().max().item() < TOL
            h = lam[t, 0] * xf[t] + lam[t, 1] * ema[t]
            kr = mods["k"](h).view(4, 128)
            assert nrel(k[1, :, t], kr) < TOL
    # causal prefix property: the first half of the sequence does not see the second
    r2 = fastmka_forward(x[:, : T // 2].contiguous(), W, 28, 4, 0.9, False)
    assert nrel(r2["out"], r["out"][:, : T // 2]) < 1e-2
    assert ops.device_status() == 0


def test_decode_llama_like_full_size_sampled_heads():
    """Decode at the full configuration: batch 64, one token against a 32768-long
    cached K/V, 32/8 heads; sampled (batch, head) rows recomputed exactly in fp32."""
    from mka_b200 import ops

    B, HQ, HKV, TK = 64, 32, 8, 32768
    g = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn(B, HQ, 1, 128, generator=g, device="cuda").bfloat16()
    k = torch.randn(B, HKV, TK, 128, generator=g, device="cuda", dtype=torch.bfloat16).mul_(0.1)
    v = torch.randn(B, HKV, TK, 128, generator=g, device="cuda", dtype=torch.bfloat16).mul_(0.1)
    o, lse = ops.attn_decode(q, k, v)
    for b in (0, 31, 63):
        for hq in (0, 5, 31):
            s = (k[b, hq // 4].float() @ q[b, hq, 0].float()) / math.sqrt(128)
            assert abs(lse[b, hq].item() - torch.logsumexp(s, 0).item()) < TOL
            assert nrel(o[b, 0, hq], torch.softmax(s, 0) @ v[b, hq // 4].float()) < TOL
    assert ops.device_status() == 0


def _hf_like_layer(seed=0, D=512, H=4, HKV=2, R=256):
    """A Qwen2-like HF attention module (q/k/v bias, GQA) wrapped by HFFastMKAAttention, on cuda."""
    from mka_b200 import HFFastMKAAttention

    class _Attn(nn.Module):
        def __init__(self):
            super().__init__()
            self.hidden_size, self.num_heads, self.num_key_value_heads = D, H, HKV
            self.q_proj = nn.Linear(D, H * 128, bias=True)
            self.k_proj = nn.Linear(D, HKV * 128, bias=True)
            self.v_proj = nn.Linear(D, HKV * 128, bias=True)
            self.o_proj = nn.Linear(H * 128, D, bias=False)

    torch.manual_seed(seed)
    layer = HFFastMKAAttention(_Attn(), use_l3=False)
    layer.router = nn.Sequential(nn.Linear(D, R), nn.SiLU(), nn.Linear(R, 2))
    with torch.no_grad():
        for m in layer.modules():
            if isinstance(m, nn.Linear):
                m.weight.normal_(0, 0.04)
                if m.bias is not None:
                    m.bias.uniform_(-0.1, 0.1)
    return layer.cuda().eval()


def test_hf_decode_carried_ema_matches_whole_sequence_prefill():
    """With StaticKVCache(carry_ema=True) each decode step continues the L2 EMA
    of the earlier tokens, so the step's output equals the reference forward
    over the whole sequence so far at its last position (hf/attention.py:82-199
    with causal_prefix_ema over all tokens)."""
    from mka_b200 import StaticKVCache

    D, H, HKV = 512, 4, 2
    layer = _hf_like_layer(seed=3, D=D, H=H, HKV=HKV)
    f = lambda t: None if t is None else t.detach().float().cpu()  # noqa: E731
    p = {"wq": f(layer.q_proj.weight), "bq": f(layer.q_proj.bias), "wk": f(layer.k_proj.weight),
         "bk": f(layer.k_proj.bias), "wv": f(layer.v_proj.weight), "bv": f(layer.v_proj.bias),
         "wo": f(layer.o_proj.weight), "r1w": f(layer.router[0].weight), "r1b": f(layer.router[0].bias),
         "r2w": f(layer.router[2].weight), "r2b": f(layer.router[2].bias)}
    g = torch.Generator().manual_seed(5)
    T0, steps = 150, 3
    x = (torch.randn(2, T0 + steps, D, generator=g) * 0.5).bfloat16()
    cache = StaticKVCache(batch=2, num_kv_heads=HKV, capacity=T0 + steps, num_layers=1, device="cuda",
                          carry_ema=True)
    with torch.no_grad():
        out, _, _ = layer(x[:, :T0].cuda(), past_key_value=cache, use_cache=True)
        ref = orc.hf_fastmka_forward(x[:, :T0].float(), p, H, HKV, False, layer.ema_beta, "silu")
        assert nrel(out, ref["out"]) < TOL
        for i in range(steps):
            t = T0 + i
            out, _, _ = layer(x[:, t:t + 1].cuda(), past_key_value=cache, use_cache=True)
            whole = orc.hf_fastmka_forward(x[:, :t + 1].float(), p, H, HKV, False, layer.ema_beta, "silu")
            assert nrel(out, whole["out"][:, -1:]) < TOL, i
    assert cache.lengths[0] == T0 + steps
    # without the carried state a decode step restarts the EMA, as the reference does
    cache2 = StaticKVCache(batch=2, num_kv_heads=HKV, capacity=T0 + 1, num_layers=1, device="cuda")
    with torch.no_grad():
        layer(x[:, :T0].cuda(), past_key_value=cache2, use_cache=True)
        out2, _, _ = layer(x[:, T0:T0 + 1].cuda(), past_key_value=cache2, use_cache=True)
        ref2 = orc.hf_fastmka_forward(x[:, T0:T0 + 1].float(), p, H, HKV, False, layer.ema_beta, "silu",
                                      past=(ref["k"], ref["v"]))
    assert nrel(out2, ref2["out"]) < TOL


class _RopeTables:
    """Stands in for an HF rotary module (its presence makes the wrapper apply
    RoPE, hf/attention.py:113-119); cos/sin are passed as position_embeddings."""

    def __init__(self, theta):
        self.theta = theta

    def tables(self, t):
        inv = 1.0 / (self.theta ** (torch.arange(0, 128, 2, dtype=torch.float64) / 128))
        ang = torch.arange(t, dtype=torch.float64)[:, None] * inv[None]
        ang = torch.cat([ang, ang], -1)
        return ang.cos().float()[None], ang.sin().float()[None]  # [1, T, 128]


def _gqa_l3_layer(D, H, HKV, R, levels, seed, w_std, theta=1.0e6):
    """A Qwen2-like attention (q/k/v bias, GQA, RoPE) wrapped by HFFastMKAAttention
    with a router D -> R -> levels (SiLU); weights and biases N(0, w_std), fp32."""
    from mka_b200 import HFFastMKAAttention

    class _Attn(nn.Module):
        def __init__(self):
            super().__init__()
            self.hidden_size, self.num_heads, self.num_key_value_heads = D, H, HKV
            self.q_proj = nn.Linear(D, H * 128, bias=True)
            self.k_proj = nn.Linear(D, HKV * 128, bias=True)
            self.v_proj = nn.Linear(D, HKV * 128, bias=True)
            self.o_proj = nn.Linear(H * 128, D, bias=False)
            self.rotary_emb = _RopeTables(theta)

    torch.manual_seed(seed)
    layer = HFFastMKAAttention(_Attn(), use_l3=levels == 3)
    layer.router = nn.Sequential(nn.Linear(D, R), nn.SiLU(), nn.Linear(R, levels))
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for m in layer.modules():
            if isinstance(m, nn.Linear):
                m.weight.copy_(torch.randn(m.weight.shape, generator=g) * w_std)
                if m.bias is not None:
                    m.bias.copy_(torch.randn(m.bias.shape, generator=g) * w_std)
    f = lambda t: None if t is None else t.detach().float().clone()  # noqa: E731
    p = {"wq": f(layer.q_proj.weight), "bq": f(layer.q_proj.bias), "wk": f(layer.k_proj.weight),
         "bk": f(layer.k_proj.bias), "wv": f(layer.v_proj.weight), "bv": f(layer.v_proj.bias),
         "wo": f(layer.o_proj.weight), "r1w": f(layer.router[0].weight), "r1b": f(layer.router[0].bias),
         "r2w": f(layer.router[2].weight), "r2b": f(layer.router[2].bias)}
    return layer.cuda().eval(), p


def _check_gqa_layer(layer, p, x, H, HKV, l3=None):
    """The wrapper on the GPU against the oracle's HF forward (hf/attention.py:82-199,
    with the per-position L3 level composed as in fastmka.py:84-89): out, the
    present k/v, the gate and the attention log-sum-exp."""
    B, T, D = x.shape
    cos, sin = layer.rotary_emb.tables(T)
    with torch.no_grad():
        ref = orc.hf_fastmka_forward(x, p, H, HKV, l3 is not None, layer.ema_beta, "silu", cos=cos[:, None],
                                     sin=sin[:, None], l3_memory=l3)
    kw = {"position_embeddings": (cos.cuda(), sin.cuda()), "use_cache": True}
    if l3 is not None:
        kw["l3_memory"] = l3.cuda().bfloat16()
    out, _, present, lse, lam = layer.forward_with_lse(x.cuda().bfloat16(), **kw)
    errs = {"out": nrel(out, ref["out"]), "k": nrel(present[0], ref["k"]), "v": nrel(present[1], ref["v"]),
            "lse": nrel(lse, ref["lse"]), "lam": (lam.float().cpu() - ref["lam"]).abs().max().item()}
    from mka_b200 import ops

    assert ops.device_status() == 0
    assert all(e < TOL for e in errs.values()), errs
    return errs


@pytest.mark.parametrize("t3", ["same", "longer", "shorter", "one"])
def test_hf_gqa_three_levels_per_position_l3(t3):
    """Three levels with a per-position L3 memory on the GQA + RoPE wrapper (the
    long-context configuration's layer at a small size): L3 of T rows, of more
    rows than T (truncated), of fewer (padded with its last row) and of one row
    (repeated), session_memory.py:25-39."""
    B, T, D, H, HKV = 2, 200, 512, 4, 2
    layer, p = _gqa_l3_layer(D, H, HKV, 256, 3, seed=21, w_std=0.05)
    g = torch.Generator().manual_seed(22)
    x = torch.randn(B, T, D, generator=g).bfloat16().float()
    t3n = {"same": T, "longer": T + 40, "shorter": T - 30, "one": 1}[t3]
    l3 = (torch.randn(B, t3n, D, generator=g) * 0.5).bfloat16().float()
    _check_gqa_layer(layer, p, x, H, HKV, l3=l3)


def test_long_context_layer_three_levels_full_width():
    """The long-context configuration's layer at its full width on one whole
    sequence: d_model 3584, 28/4 heads, q/k/v bias, RoPE theta 1e6, router
    3584 -> 512 -> 3, weights N(0, 0.02), X ~ N(0,1)/sqrt(3584), L3 ~ N(0,1)*0.5
    per position, seq 4096."""
    D, H, HKV, T = 3584, 28, 4, 4096
    layer, p = _gqa_l3_layer(D, H, HKV, 512, 3, seed=23, w_std=0.02)
    g = torch.Generator().manual_seed(24)
    x = (torch.randn(1, T, D, generator=g) / math.sqrt(D)).bfloat16().float()
    l3 = (torch.randn(1, T, D, generator=g) * 0.5).bfloat16().float()
    _check_gqa_layer(layer, p, x, H, HKV, l3=l3)


def test_qwen_like_prefill_whole_sequence():
    """The Qwen-7B-like prefill layer (d_model 3584, 28/4 heads, q/k/v bias, RoPE
    theta 1e6, router 3584 -> 512 -> 2, weights N(0, 0.02), X ~ N(0,1)/sqrt(3584))
    on one whole sequence of 8192 tokens: out, k, v, gate and LSE against the
    oracle's fp32 forward of the same sequence."""
    D, H, HKV, T = 3584, 28, 4, 8192
    layer, p = _gqa_l3_layer(D, H, HKV, 512, 2, seed=25, w_std=0.02)
    g = torch.Generator().manual_seed(26)
    x = (torch.randn(1, T, D, generator=g) / math.sqrt(D)).bfloat16().float()
    _check_gqa_layer(layer, p, x, H, HKV)
