"""Generates the golden fixtures by running the FastLM/MKA reference modules.

    python tests/golden/make_golden.py --ref <reference checkout>
    (or set FMKA_REFERENCE_DIR to the checkout and omit --ref)

Needs the reference package on disk (it is not on the GPU box: the fixtures are
committed). Every input is rounded to bf16-representable values before the
reference runs in fp32 on the CPU, so the bf16 CUDA path sees exactly the same
inputs. Outputs are the reference's own tensors; the attention log-sum-exp is
computed here from the reference module's own projections (the reference does
not return it).

Cases (small shapes; the configuration each one mirrors in brackets):
  fastmka_mha_gelu      FastMKAAttention, L1+L2, router D->D/4->2 with GELU   [single-layer fp32 case]
  fastmka_mha_l3_pad    use_l3, L3 memory shorter than T (pad with last row), SiLU router
  fastmka_mha_l3_single use_l3, one-row L3 memory (repeat)
  fastmka_mha_cache     prefill of 8 tokens after a 24-token K/V cache
  fastmka_mha_decode    one token after a 37-token cache
  hf_qwen_rope          HFFastMKAAttention on Qwen2Attention (q/k/v bias), GQA 4/2, RoPE, use_cache
  hf_qwen_decode        one token after hf_qwen_rope's present, RoPE at position 33
  hf_llama_norope       HFFastMKAAttention on LlamaAttention, GQA 4/1, no RoPE, router 512->128->2
  ema                   causal_prefix_ema for three decays, repeat_retrieval_to_length rules
"""
from __future__ import annotations

import argparse
import math
import os
import sys

import numpy as np
import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))


def bf(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


def lse_of(q: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    g = q.shape[1] // k.shape[1]
    k = k.repeat_interleave(g, dim=1)
    tq, tk = q.shape[2], k.shape[2]
    s = (q @ k.transpose(-1, -2)) / math.sqrt(q.shape[-1])
    qp = torch.arange(tk - tq, tk).view(tq, 1)
    kp = torch.arange(tk).view(1, tk)
    return torch.logsumexp(s.masked_fill(kp > qp, float("-inf")), -1)


def round_module(m: nn.Module) -> None:
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(bf(p))


def save(name: str, **arrays) -> None:
    """Tensors whose values are exactly bf16 are stored as their 16-bit words
    under `<key>__bf16` (tests/golden_io.py restores them); others as fp32."""
    out = {}
    for k, v in arrays.items():
        if not torch.is_tensor(v):
            out[k] = np.asarray(v)
            continue
        v = v.detach().to(torch.float32)
        if torch.equal(bf(v), v):
            out[k + "__bf16"] = v.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        else:
            out[k] = v.numpy()
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(f"wrote {name}.npz ({sum(a.nbytes for a in out.values()) / 1e6:.2f} MB raw)")


def state(m: nn.Module, prefix: str = "") -> dict:
    # the HF wrapper's state also lists the wrapped module's projections under
    # original_attn.* (the same tensors as q_proj.* etc.): stored once
    return {prefix + k: v for k, v in m.state_dict().items() if not k.startswith("original_attn.")}


def make_fastmka_cases(mka) -> None:
    from mka.layers.fastmka import FastMKAAttention, FastMKAConfig

    def build(d, h, use_l3, router=None, seed=0):
        torch.manual_seed(seed)
        m = FastMKAAttention(FastMKAConfig(hidden_size=d, num_heads=h, use_l3=use_l3))
        if router is not None:
            m.router = router
        for mod in m.modules():
            if isinstance(mod, nn.Linear):
                nn.init.xavier_uniform_(mod.weight)
                if mod.bias is not None:
                    nn.init.uniform_(mod.bias, -0.1, 0.1)
        round_module(m)
        return m.eval()

    # L1+L2, GELU router (the single-layer fp32 configuration, reduced)
    d, h, b, t = 256, 2, 2, 40
    m = build(d, h, False, nn.Sequential(nn.Linear(d, 64), nn.GELU(), nn.Linear(64, 2)))
    torch.manual_seed(1)
    x = bf(torch.randn(b, t, d))
    with torch.no_grad():
        out, k, v, lam = m(x)
        q = m.wq(x).view(b, t, h, d // h).transpose(1, 2)
    save("fastmka_mha_gelu", x=x, out=out, k=k, v=v, lam=lam, lse=lse_of(q, k), heads=h, act=1, beta=0.9,
         use_l3=0, **state(m, "p."))

    # use_l3 with a shorter L3 memory (pad) and with a single row (repeat), SiLU router
    for name, t3 in (("fastmka_mha_l3_pad", 25), ("fastmka_mha_l3_single", 1)):
        m = build(d, h, True, seed=2)
        torch.manual_seed(3)
        x = bf(torch.randn(b, t, d))
        l3 = bf(torch.randn(b, t3, d) * 0.5)
        with torch.no_grad():
            out, k, v, lam = m(x, l3_memory=l3)
            q = m.wq(x).view(b, t, h, d // h).transpose(1, 2)
        save(name, x=x, l3=l3, out=out, k=k, v=v, lam=lam, lse=lse_of(q, k), heads=h, act=0, beta=0.9,
             use_l3=1, **state(m, "p."))

    # prefill after a cache, and a one-token decode
    for name, tp, tn in (("fastmka_mha_cache", 24, 8), ("fastmka_mha_decode", 37, 1)):
        m = build(d, h, False, seed=4)
        torch.manual_seed(5)
        x = bf(torch.randn(b, tn, d))
        pk = bf(torch.randn(b, h, tp, d // h) * 0.5)
        pv = bf(torch.randn(b, h, tp, d // h) * 0.5)
        with torch.no_grad():
            out, k, v, lam = m(x, kv_cache_k=pk, kv_cache_v=pv)
            q = m.wq(x).view(b, tn, h, d // h).transpose(1, 2)
        save(name, x=x, past_k=pk, past_v=pv, out=out, k=k, v=v, lam=lam, lse=lse_of(q, k), heads=h, act=0,
             beta=0.9, use_l3=0, **state(m, "p."))


def make_hf_cases(mka) -> None:
    from mka.hf.attention import HFFastMKAAttention, _apply_rotary_pos_emb
    from transformers import LlamaConfig, Qwen2Config
    from transformers.models.llama.modeling_llama import LlamaAttention
    from transformers.models.qwen2.modeling_qwen2 import Qwen2Attention, Qwen2RotaryEmbedding

    def shim(att, d, h, hkv, rotary=None):
        # transformers 5.x attention modules no longer carry these attributes,
        # which the reference wrapper reads (mka/hf/attention.py:57-61,68)
        att.hidden_size, att.num_heads, att.num_key_value_heads = d, h, hkv
        att.rotary_emb = rotary
        return att

    def init(m, seed):
        torch.manual_seed(seed)
        for mod in m.modules():
            if isinstance(mod, nn.Linear):
                nn.init.normal_(mod.weight, std=0.04)
                if mod.bias is not None:
                    nn.init.uniform_(mod.bias, -0.1, 0.1)
        round_module(m)

    # Qwen2-like, q/k/v bias, GQA 4/2, RoPE, cache
    d, h, hkv, b, t = 512, 4, 2, 2, 33
    cfg = Qwen2Config(hidden_size=d, num_attention_heads=h, num_key_value_heads=hkv, intermediate_size=1024,
                      vocab_size=128, rope_theta=10000.0)
    rot = Qwen2RotaryEmbedding(cfg)
    att = shim(Qwen2Attention(cfg, layer_idx=0), d, h, hkv, rot)
    w = HFFastMKAAttention(att, use_l3=False)
    init(w, 6)
    w.eval()
    torch.manual_seed(7)
    x = bf(torch.randn(b, t, d) * 0.5)
    pos = torch.arange(t)[None].expand(b, t)
    cos, sin = rot(x, pos)
    cos, sin = cos[:, None], sin[:, None]  # [B,1,T,Dh]: the wrapper does not unsqueeze (hf/attention.py:20-25)
    with torch.no_grad():
        out, _, present = w(x, position_embeddings=(cos, sin), use_cache=True)
        lam = torch.softmax(w.router(w.q_proj(x)), -1)
        q = w.q_proj(x).view(b, t, h, d // h).transpose(1, 2)
        kr = w.k_proj(x).view(b, t, hkv, d // h).transpose(1, 2)  # only for the q rotation
        q, _ = _apply_rotary_pos_emb(q, kr, cos, sin)
    sd = state(w, "p.")
    save("hf_qwen_rope", x=x, cos=cos, sin=sin, out=out, k=present[0], v=present[1], lam=lam,
         lse=lse_of(q, present[0]), heads=h, kv_heads=hkv, act=0, beta=0.9, use_l3=0, **sd)

    # one decode token at position t
    torch.manual_seed(8)
    x1 = bf(torch.randn(b, 1, d) * 0.5)
    pos1 = torch.full((b, 1), t)
    c1, s1 = rot(x1, pos1)
    c1, s1 = c1[:, None], s1[:, None]
    with torch.no_grad():
        out1, _, present1 = w(x1, position_embeddings=(c1, s1), past_key_value=present, use_cache=True)
        lam1 = torch.softmax(w.router(w.q_proj(x1)), -1)
        q1 = w.q_proj(x1).view(b, 1, h, d // h).transpose(1, 2)
        q1, _ = _apply_rotary_pos_emb(q1, q1[:, :hkv], c1, s1)
    # the weights are hf_qwen_rope's (not stored twice)
    save("hf_qwen_decode", x=x1, cos=c1, sin=s1, past_k=present[0], past_v=present[1], out=out1,
         k=present1[0], v=present1[1], lam=lam1, lse=lse_of(q1, present1[0]), heads=h, kv_heads=hkv, act=0,
         beta=0.9, use_l3=0, weights_from="hf_qwen_rope")

    # Llama-like, no bias, GQA 4/1, no RoPE, router overridden to 512 -> 128 -> 2
    d, h, hkv, b, t = 512, 4, 1, 1, 20
    cfg = LlamaConfig(hidden_size=d, num_attention_heads=h, num_key_value_heads=hkv, intermediate_size=1024,
                      vocab_size=128)
    att = shim(LlamaAttention(cfg, layer_idx=0), d, h, hkv, None)
    w = HFFastMKAAttention(att, use_l3=False)
    w.router = nn.Sequential(nn.Linear(d, 128), nn.SiLU(), nn.Linear(128, 2))
    init(w, 9)
    w.eval()
    torch.manual_seed(10)
    x = bf(torch.randn(b, t, d) * 0.5)
    with torch.no_grad():
        out, _, present = w(x, use_cache=True)
        lam = torch.softmax(w.router(w.q_proj(x)), -1)
        q = w.q_proj(x).view(b, t, h, d // h).transpose(1, 2)
    save("hf_llama_norope", x=x, out=out, k=present[0], v=present[1], lam=lam, lse=lse_of(q, present[0]),
         heads=h, kv_heads=hkv, act=0, beta=0.9, use_l3=0, **state(w, "p."))


def make_ema_cases(mka) -> None:
    from mka.layers.session_memory import causal_prefix_ema, repeat_retrieval_to_length

    torch.manual_seed(11)
    x = bf(torch.randn(2, 50, 16))
    arrays = {"x": x}
    for beta in (0.9, 0.5, 0.99):
        arrays[f"ema_{beta}"] = causal_prefix_ema(x, beta=beta)
    mem = bf(torch.randn(2, 7, 16))
    for tl in (7, 3, 12):
        arrays[f"rep_{tl}"] = repeat_retrieval_to_length(mem, tl)
    arrays["rep_single_9"] = repeat_retrieval_to_length(mem[:, :1], 9)
    save("ema", mem=mem, **arrays)


def main() -> None:
    ap = argparse.ArgumentParser()
    env = os.environ.get("FMKA_REFERENCE_DIR")
    ap.add_argument("--ref", default=env, required=env is None,
                    help="the FastLM/MKA checkout (the directory holding the mka package)")
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    import mka  # noqa: F401  (the reference package)

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    make_ema_cases(mka)
    make_fastmka_cases(mka)
    make_hf_cases(mka)


if __name__ == "__main__":
    main()
