"""CPU oracle for the FastMKA attention forward.

TEST INFRASTRUCTURE ONLY. This module restates the FastLM/MKA reference
algorithm in plain fp32 PyTorch on the CPU so that the CUDA path can be checked
against it. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline /
reference arm may import it, and only as the checker or the timed CPU baseline:
the product path (mka_b200) never calls it.

Pinning: every function below is checked against golden vectors produced by
running the reference's own modules (tests/golden/make_golden.py imports the
reference package and records its inputs and outputs; tests/test_oracle.py
compares). The reference has no tests or fixtures of its own.

Each function cites the reference lines it restates. The op sequence mirrors
the reference's CPU path (SDPA for prefill without a cache, the explicit masked
softmax when a cache is present, the Python EMA loop), so timing it is timing
the reference's CPU algorithm.
"""
from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch
import torch.nn.functional as F

Tensor = torch.Tensor


# ------------------------------------------------------------ session memory --
def causal_prefix_ema(x: Tensor, beta: float = 0.9) -> Tensor:
    """mka/layers/session_memory.py:6-22: state_0 = 0,
    state_t = beta * state_{t-1} + (1 - beta) * x_t, out_t = state_t (in x.dtype)."""
    b, t, d = x.shape
    out = torch.zeros_like(x)
    state = torch.zeros((b, d), dtype=x.dtype, device=x.device)
    for i in range(t):
        state = beta * state + (1.0 - beta) * x[:, i, :]
        out[:, i, :] = state
    return out


def repeat_retrieval_to_length(mem: Tensor, target_len: int) -> Tensor:
    """mka/layers/session_memory.py:25-39: [B,T3,D] -> [B,T,D]: identity when
    T3 == T, repeat a single row, truncate a longer one, pad a shorter one with
    its last row."""
    n = mem.size(1)
    if n == target_len:
        return mem
    if n == 1:
        return mem.repeat(1, target_len, 1)
    if n > target_len:
        return mem[:, :target_len, :]
    last = mem[:, -1:, :].repeat(1, target_len - n, 1)
    return torch.cat([mem, last], dim=1)


# -------------------------------------------------------------------- router --
def router_gate(q: Tensor, w1: Tensor, b1: Tensor, w2: Tensor, b2: Tensor, act: str) -> Tensor:
    """lam = softmax(W2 act(W1 q + b1) + b2) over the levels
    (mka/layers/fastmka.py:55-59,91-92; mka/hf/attention.py:71-76,104)."""
    h = F.linear(q, w1, b1)
    h = F.silu(h) if act == "silu" else F.gelu(h)
    return torch.softmax(F.linear(h, w2, b2), dim=-1)


def route_blend(levels, lam: Tensor) -> Tensor:
    """fused = sum_l lam[..., l] * level_l, accumulated left to right from 0.0
    (mka/layers/fastmka.py:94-96; mka/hf/attention.py:105-107)."""
    fused = 0.0
    for i, mem in enumerate(levels):
        fused = fused + lam[..., i:i + 1] * mem
    return fused


# ---------------------------------------------------------------------- RoPE --
def rotate_half(x: Tensor) -> Tensor:
    """mka/hf/attention.py:14-17."""
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def apply_rope(q: Tensor, k: Tensor, cos: Tensor, sin: Tensor) -> Tuple[Tensor, Tensor]:
    """mka/hf/attention.py:20-25 (cos/sin broadcast against [B,H,T,Dh])."""
    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin


# ----------------------------------------------------------------- attention --
def repeat_kv(x: Tensor, n_rep: int) -> Tensor:
    """mka/hf/attention.py:28-33."""
    if n_rep == 1:
        return x
    b, h, s, d = x.shape
    return x[:, :, None].expand(b, h, n_rep, s, d).reshape(b, h * n_rep, s, d)


def attention(q: Tensor, k: Tensor, v: Tensor, use_sdpa: bool) -> Tensor:
    """Causal attention of the reference forward. Without a cache the reference
    calls SDPA(is_causal=True) (fastmka.py:134,157; hf/attention.py:142); with a
    cache it runs the explicit masked softmax with query positions
    [Tk - Tq, Tk) (fastmka.py:166-174; hf/attention.py:188-193)."""
    if use_sdpa:
        return F.scaled_dot_product_attention(q, k, v, attn_mask=None, dropout_p=0.0, is_causal=True)
    t, t_tot = q.size(2), k.size(2)
    scores = torch.matmul(q, k.transpose(-1, -2)) / math.sqrt(q.size(-1))
    q_pos = torch.arange(t_tot - t, t_tot).view(1, 1, t, 1)
    k_pos = torch.arange(t_tot).view(1, 1, 1, t_tot)
    scores = scores.masked_fill(~(k_pos <= q_pos), torch.finfo(scores.dtype).min)
    return torch.matmul(torch.softmax(scores, dim=-1), v)


def attention_lse(q: Tensor, k: Tensor) -> Tensor:
    """Log-sum-exp over keys of the scaled, causally masked scores (bottom-right
    alignment), the second output of the flash kernel: [B, Hq, Tq]. Computed one
    query head at a time so that long sequences stay within host memory."""
    g = q.size(1) // k.size(1)
    t, t_tot = q.size(2), k.size(2)
    q_pos = torch.arange(t_tot - t, t_tot).view(1, t, 1)
    k_pos = torch.arange(t_tot).view(1, 1, t_tot)
    masked = k_pos > q_pos
    out = torch.empty(q.shape[:3], dtype=torch.float32)
    for h in range(q.size(1)):
        s = torch.matmul(q[:, h].float(), k[:, h // g].float().transpose(-1, -2)) / math.sqrt(q.size(-1))
        out[:, h] = torch.logsumexp(s.masked_fill(masked, float("-inf")), dim=-1)
    return out


# ------------------------------------------------------- low-level op API --
def fastmka_attn_op(q: Tensor, k: Tensor, v: Tensor, causal: bool = True) -> Tensor:
    """The reference's fastmka_attn op (mka/cuda/fastmka_attn.cu:51-131, bound at
    mka/cuda/ops.py:73-77): q [B,H,Tq,D], k/v [B,H,Tk,D]; query tq attends keys
    0 .. min(Tk-1, tq + Tk - Tq) when causal, all keys otherwise; a query with no
    key to attend (Tq > Tk) gets zeros (inv_l = 0 at :126-127). Scale 1/sqrt(D).
    A k/v with fewer heads than q is broadcast by head group (the B200 op's GQA
    extension; the reference requires equal head counts)."""
    g = q.size(1) // k.size(1)
    qf, kf, vf = q.float(), repeat_kv(k.float(), g), repeat_kv(v.float(), g)
    tq, tk = qf.size(2), kf.size(2)
    s = torch.matmul(qf, kf.transpose(-1, -2)) / math.sqrt(qf.size(-1))
    if causal:
        q_pos = torch.arange(tk - tq, tk).view(1, 1, tq, 1)
        k_pos = torch.arange(tk).view(1, 1, 1, tk)
        s = s.masked_fill(k_pos > q_pos, float("-inf"))
    p = torch.softmax(s, dim=-1).nan_to_num(0.0)  # rows with every key masked -> zeros
    return torch.matmul(p, vf)


def fused_route_mka_op(q: Tensor, l1: Tensor, l2: Tensor, l3: Tensor, lam: Tensor, wk: Tensor,
                       wv: Tensor) -> Tensor:
    """The reference's fused_route_mka op (mka/cuda/fused_route_mka.cu:23-102,
    bound at mka/cuda/ops.py:47-70): per token fused = lam0 l1 + lam1 l2 (+ lam2 l3
    when lam has 3 levels), k = fused wk^T and v = fused wv^T split into H heads of
    Dh = D / H, then causal attention of q [B,H,T,Dh] over them (offset 0)."""
    b, h, t, dh = q.shape
    d = l1.size(2)
    n_levels = lam.size(2)
    fused = lam[..., 0:1].float() * l1.float() + lam[..., 1:2].float() * l2.float()
    if n_levels > 2:
        fused = fused + lam[..., 2:3].float() * l3.float()
    k = F.linear(fused, wk.float()).view(b, t, h, dh).transpose(1, 2)
    v = F.linear(fused, wv.float()).view(b, t, h, dh).transpose(1, 2)
    assert h * dh == d
    return fastmka_attn_op(q, k, v, causal=True)


# ------------------------------------------------------------- full forwards --
def fastmka_forward(x: Tensor, p: Dict[str, Tensor], num_heads: int, use_l3: bool, beta: float, act: str,
                    l3_memory: Optional[Tensor] = None, kv_cache_k: Optional[Tensor] = None,
                    kv_cache_v: Optional[Tensor] = None, with_lse: bool = True) -> Dict[str, Tensor]:
    """FastMKAAttention.forward (mka/layers/fastmka.py:71-177), MHA, no biases.

    p: wq, wk, wv, wo [D, D]; r1w [R, D], r1b [R], r2w [L, R], r2b [L].
    Returns out, k_tot, v_tot, lam and (with_lse) lse, which the reference
    module does not compute: a timed run of the reference algorithm leaves it out.
    """
    b, t, d = x.shape
    dh = d // num_heads
    q = F.linear(x, p["wq"])
    levels = [x, causal_prefix_ema(x, beta)]
    if use_l3:
        if l3_memory is None:
            l3_memory = torch.zeros((b, 1, d), dtype=x.dtype)
        levels.append(repeat_retrieval_to_length(l3_memory, t))
    lam = router_gate(q, p["r1w"], p["r1b"], p["r2w"], p["r2b"], act)
    fused = route_blend(levels, lam)

    def heads(z):
        return z.view(b, t, num_heads, dh).transpose(1, 2)

    k_new, v_new, qh = heads(F.linear(fused, p["wk"])), heads(F.linear(fused, p["wv"])), heads(q)
    cached = kv_cache_k is not None and kv_cache_v is not None
    k_tot = torch.cat([kv_cache_k, k_new], 2) if cached else k_new
    v_tot = torch.cat([kv_cache_v, v_new], 2) if cached else v_new
    o = attention(qh, k_tot, v_tot, use_sdpa=not cached)
    out = F.linear(o.transpose(1, 2).contiguous().view(b, t, d), p["wo"])
    return {"out": out, "k_tot": k_tot, "v_tot": v_tot, "lam": lam,
            "lse": attention_lse(qh, k_tot) if with_lse else None}


def hf_fastmka_forward(h: Tensor, p: Dict[str, Tensor], num_heads: int, num_kv_heads: int, use_l3: bool,
                       beta: float, act: str, past: Optional[Tuple[Tensor, Tensor]] = None,
                       cos: Optional[Tensor] = None, sin: Optional[Tensor] = None,
                       l3_memory: Optional[Tensor] = None, with_lse: bool = True) -> Dict[str, Tensor]:
    """HFFastMKAAttention.forward (mka/hf/attention.py:82-199): GQA, optional
    q/k/v/o biases (bq, bk, bv, bo in p), RoPE when cos/sin are given
    (:113-119), tuple cache concat (:121-124), present = post-RoPE (k, v).

    l3_memory: the per-position L3 of the cfg-3 workload, composed from the
    reference's own functions as in fastmka.py:84-89; the HF wrapper itself
    always blends zeros (hf/attention.py:100-102), which is l3_memory=None.
    with_lse: also return the attention log-sum-exp (not part of the reference
    forward; a timed run of the reference algorithm leaves it out).
    """
    b, t, d = h.shape
    dh = d // num_heads
    q = F.linear(h, p["wq"], p.get("bq"))
    levels = [h, causal_prefix_ema(h, beta)]
    if use_l3:
        l3 = torch.zeros((b, 1, d), dtype=h.dtype) if l3_memory is None else l3_memory
        levels.append(repeat_retrieval_to_length(l3, t))
    lam = router_gate(q, p["r1w"], p["r1b"], p["r2w"], p["r2b"], act)
    fused = route_blend(levels, lam)
    qs = q.view(b, t, num_heads, dh).transpose(1, 2)
    ks = F.linear(fused, p["wk"], p.get("bk")).view(b, t, num_kv_heads, dh).transpose(1, 2)
    vs = F.linear(fused, p["wv"], p.get("bv")).view(b, t, num_kv_heads, dh).transpose(1, 2)
    if cos is not None:
        qs, ks = apply_rope(qs, ks, cos, sin)
    if past is not None:
        ks = torch.cat([past[0], ks], 2)
        vs = torch.cat([past[1], vs], 2)
    g = num_heads // num_kv_heads
    o = attention(qs, repeat_kv(ks, g), repeat_kv(vs, g), use_sdpa=past is None)
    out = F.linear(o.transpose(1, 2).contiguous().view(b, t, d), p["wo"], p.get("bo"))
    return {"out": out, "k": ks, "v": vs, "lam": lam, "lse": attention_lse(qs, ks) if with_lse else None}


# ------------------------------------------------------------ L3 chunk recall --
# The reference describes the L3 tier (mka/config/memory_hierarchy.py:1-10,
# "DRAM (vectorized hash, chunk recall)"; lines 30-34, l3_recall_top_r "top-R
# chunks per query") and implements no recall, so nothing here is pinned to the
# reference: this restates the recall of mka_b200.l3 / l3_recall.cu (block-mean
# queries, dot-product scores, top-R with the lower index first on ties,
# softmax weights, one weighted sum per query block) so that the kernels can be
# checked against it.
def l3_block_mean(x: Tensor, block_len: int) -> Tensor:
    """bf16-rounded means of block_len-token blocks of x [B, T, D] -> [B * nq, D] (fp32 values)."""
    b, t, d = x.shape
    nq = (t + block_len - 1) // block_len
    out = torch.empty(b, nq, d, dtype=torch.float64)
    xd = x.double()
    for j in range(nq):
        out[:, j] = xd[:, j * block_len:min((j + 1) * block_len, t)].mean(1)
    return out.float().bfloat16().float().reshape(b * nq, d)


def l3_topr(scores: Tensor, top_r: int, scale: float) -> Tuple[Tensor, Tensor]:
    """Per row: the top_r best columns (score descending, the lower index first on
    ties) and softmax(scale * score) over them."""
    m, n = scores.shape
    idx = torch.empty(m, top_r, dtype=torch.int64)
    w = torch.empty(m, top_r, dtype=torch.float32)
    cols = torch.arange(n)
    for i in range(m):
        s = scores[i].double()
        order = sorted(range(n), key=lambda c: (-s[c].item(), c))[:top_r]
        idx[i] = torch.tensor(order)
        sel = s[cols[order]]
        e = torch.exp((sel - sel.max()) * scale)
        w[i] = (e / e.sum()).float()
    return idx, w


def l3_chunk_recall(x: Tensor, keys: Tensor, values: Tensor, top_r: int, block_len: int,
                    scale: Optional[float] = None, q: Optional[Tensor] = None):
    """R [B, T, D], idx, w and the scores for x [B, T, D] and a chunk bank keys /
    values [n_chunks, D]; q (the block summaries) may be given, e.g. the GPU's
    own, so that a ranking comparison does not hinge on a bf16 rounding."""
    b, t, d = x.shape
    q = l3_block_mean(x, block_len) if q is None else q.float()
    scores = q.double() @ keys.double().t()
    idx, w = l3_topr(scores, top_r, d ** -0.5 if scale is None else scale)
    vecs = (w.double().unsqueeze(-1) * values.double()[idx]).sum(1)  # [B * nq, D]
    nq = (t + block_len - 1) // block_len
    rows = torch.arange(t) // block_len
    r = vecs.view(b, nq, d)[:, rows]
    return r.float(), idx, w, scores
