"""Tensor-level FastMKA ops on B200, each one call into libfastmka_b200.so.

Every op launches on the current torch CUDA stream of its inputs' device, takes
bf16 CUDA tensors (the reference-compatible wrappers at the bottom also accept
fp16/fp32 and convert), allocates its outputs with torch, and raises
FastMKAError / RuntimeError on bad input. There is no CPU path: calling an op
with CPU tensors raises.

Reference op API mirrored here: mka/cuda/ops.py (fastmka_attn :73-77,
fused_route_mka_attn :47-70, has_fastmka_cuda :25-26, has_fused_route_mka_cuda
:43-44).
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch

from . import _lib

HEAD_DIM = 128
ACT_SILU = 0
ACT_GELU = 1
# bits of the device status word (FMKA_STATUS_* in include/fastmka_b200.h)
STATUS_WAIT_TIMEOUT = 1
STATUS_LOOKBACK_TIMEOUT = 2
STATUS_BAD_LAUNCH = 4
STATUS_PEER_TIMEOUT = 8


# ------------------------------------------------------------------ helpers --
def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("FastMKA B200 ops need CUDA tensors (there is no CPU fallback)")


def _check_bf16(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and t.dtype != torch.bfloat16:
            raise RuntimeError(f"expected a bfloat16 tensor, got {t.dtype}")


def _f32(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    if t is None:
        return None
    return t.detach().to(torch.float32).contiguous()


class _Workspace:
    """Grow-only per-(device, stream) scratch buffer; reuse is stream-ordered."""

    def __init__(self) -> None:
        self._bufs: dict[tuple[int, int], torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int) -> Optional[torch.Tensor]:
        if nbytes <= 0:
            return None
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        return buf


_WS = _Workspace()


def device_status(clear: bool = True) -> int:
    """Returns (and by default clears) the device status word of the current device."""
    st = _lib.c_uint32(0)
    _lib.call("fmka_device_status", _lib.ctypes.byref(st), int(clear), torch.cuda.current_stream().cuda_stream)
    return int(st.value)


# -------------------------------------------------------------------- GEMMs --
def gemm(a: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None,
         out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[M, N] = a[M, K] @ w[N, K]^T (+ bias), bf16 with fp32 accumulation."""
    _check_cuda(a, w)
    _check_bf16(a, w)
    if a.dim() != 2 or w.dim() != 2 or a.shape[1] != w.shape[1]:
        raise RuntimeError("gemm: expected a [M, K] and w [N, K]")
    if a.stride(1) != 1 or w.stride(1) != 1:
        raise RuntimeError("gemm: inner dimension must be contiguous")
    M, K = a.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    b32 = _f32(bias)
    _lib.call("fmka_gemm_bf16", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), _ptr(b32),
              out.data_ptr(), out.stride(0), M, N, K, _stream(a))
    return out


def gemm_kblocked(a_blocks: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[M, N] = A[M, K] @ w[N, K]^T where A is given as blocks a_blocks[j] = A[:, j*kb:(j+1)*kb]
    (a_blocks: [K / kb, M, kb], e.g. an all-gathered attention output), read in place."""
    _check_cuda(a_blocks, w)
    _check_bf16(a_blocks, w)
    if a_blocks.dim() != 3 or a_blocks.stride(2) != 1:
        raise RuntimeError("gemm_kblocked: a_blocks must be [nblk, M, kb] with a contiguous last dimension")
    nblk, M, kb = a_blocks.shape
    K = nblk * kb
    if w.shape[1] != K:
        raise RuntimeError("gemm_kblocked: w must be [N, nblk * kb]")
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a_blocks.device)
    b32 = _f32(bias)
    _lib.call("fmka_gemm_bf16_kblocked", a_blocks.data_ptr(), kb, a_blocks.stride(0), a_blocks.stride(1),
              w.data_ptr(), w.stride(0), _ptr(b32), out.data_ptr(), out.stride(0), M, N, K, _stream(a_blocks))
    return out


def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """[2I, K] weight for gemm_swiglu from gate_proj / up_proj weights [I, K]:
    blocks of 128 gate rows followed by the matching 128 up rows. Also works
    on biases ([I] -> [2I])."""
    if w_gate.shape != w_up.shape or w_gate.shape[0] % 128:
        raise RuntimeError("interleave_gate_up: gate and up must match, with a multiple of 128 rows")
    I = w_gate.shape[0]
    rest = tuple(w_gate.shape[1:])
    return torch.stack([w_gate.reshape(I // 128, 128, *rest), w_up.reshape(I // 128, 128, *rest)], 1).reshape(
        2 * I, *rest).contiguous()


def gemm_swiglu(x: torch.Tensor, w_gu: torch.Tensor, bias_gu: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[M, I] = silu(x w_gate^T + b_gate) * (x w_up^T + b_up) in one GEMM, with
    w_gu (and bias_gu) from interleave_gate_up."""
    _check_cuda(x, w_gu)
    _check_bf16(x, w_gu)
    if x.dim() != 2 or w_gu.dim() != 2 or x.shape[1] != w_gu.shape[1] or w_gu.shape[0] % 256:
        raise RuntimeError("gemm_swiglu: expected x [M, K] and w_gu [2I, K] with I a multiple of 128")
    if x.stride(1) != 1 or w_gu.stride(1) != 1:
        raise RuntimeError("gemm_swiglu: inner dimension must be contiguous")
    M, K = x.shape
    I = w_gu.shape[0] // 2
    if out is None:
        out = torch.empty((M, I), dtype=torch.bfloat16, device=x.device)
    b32 = _f32(bias_gu)
    _lib.call("fmka_gemm_bf16_swiglu", x.data_ptr(), x.stride(0), w_gu.data_ptr(), w_gu.stride(0), _ptr(b32),
              out.data_ptr(), out.stride(0), M, I, K, _stream(x))
    return out


def gemm_kblocked_scatter(a_blocks: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor],
                          dst_ptrs: Sequence[int], row0: int, ldc: int) -> None:
    """gemm_kblocked whose output row m goes to row row0 + m of every buffer in
    dst_ptrs (device addresses of bf16 [*, ldc] buffers, local or peer-mapped;
    at most 8). Nothing is returned: the rows land in the destinations."""
    _check_cuda(a_blocks, w)
    _check_bf16(a_blocks, w)
    if a_blocks.dim() != 3 or a_blocks.stride(2) != 1:
        raise RuntimeError("gemm_kblocked_scatter: a_blocks must be [nblk, M, kb] with a contiguous last dimension")
    nblk, M, kb = a_blocks.shape
    K = nblk * kb
    if w.shape[1] != K:
        raise RuntimeError("gemm_kblocked_scatter: w must be [N, nblk * kb]")
    N = w.shape[0]
    n = len(dst_ptrs)
    arr = (_lib.ctypes.c_void_p * max(n, 1))(*dst_ptrs)
    b32 = _f32(bias)
    _lib.call("fmka_gemm_bf16_kblocked_scatter", a_blocks.data_ptr(), kb, a_blocks.stride(0), a_blocks.stride(1),
              w.data_ptr(), w.stride(0), _ptr(b32), arr, n, int(row0), int(ldc), M, N, K, _stream(a_blocks))


def qr_proj(x2d: torch.Tensor, w_qr: torch.Tensor, bias_qr: Optional[torch.Tensor], B: int, T: int,
            num_heads: int, router_hidden: int, w2: Optional[torch.Tensor], levels: int, act: int,
            rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
            q_out: Optional[torch.Tensor] = None, t_offset: int = 0) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Q projection (head-split, optional RoPE) fused with the router's first layer.

    Returns q [B, Hq, T, 128] and router logits [B*T, L] (fp32, without the
    router's output bias), or None for the logits when router_hidden == 0.
    """
    _check_cuda(x2d, w_qr)
    _check_bf16(x2d, w_qr)
    D = x2d.shape[1]
    if q_out is None:
        q_out = torch.empty((B, num_heads, T, HEAD_DIM), dtype=torch.bfloat16, device=x2d.device)
    logits = None
    if router_hidden > 0:
        logits = torch.zeros((B * T, levels), dtype=torch.float32, device=x2d.device)
    cos, sin, rsb, rst = _rope_args(rope, B, T)
    w2c = _f32(w2)
    _lib.call("fmka_qr_proj", x2d.data_ptr(), x2d.stride(0), w_qr.data_ptr(), w_qr.stride(0), _ptr(bias_qr),
              B, T, D, num_heads, router_hidden, q_out.data_ptr(), q_out.stride(0), q_out.stride(1),
              q_out.stride(2), t_offset, _ptr(cos), _ptr(sin), rsb, rst, _ptr(w2c), levels, act, _ptr(logits),
              _stream(x2d))
    return q_out, logits


def kv_proj(h2d: torch.Tensor, w_kv: torch.Tensor, bias_kv: Optional[torch.Tensor], B: int, T: int,
            num_kv_heads: int, rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
            k_out: Optional[torch.Tensor] = None, v_out: Optional[torch.Tensor] = None,
            t_offset: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """K/V projection of the fused memory, written head-split ([B, Hkv, Tcap, 128])."""
    _check_cuda(h2d, w_kv)
    _check_bf16(h2d, w_kv)
    D = h2d.shape[1]
    if k_out is None:
        k_out = torch.empty((B, num_kv_heads, T, HEAD_DIM), dtype=torch.bfloat16, device=h2d.device)
    if v_out is None:
        v_out = torch.empty_like(k_out)
    if k_out.stride() != v_out.stride():
        raise RuntimeError("kv_proj: k and v outputs must share strides")
    cos, sin, rsb, rst = _rope_args(rope, B, T)
    _lib.call("fmka_kv_proj", h2d.data_ptr(), h2d.stride(0), w_kv.data_ptr(), w_kv.stride(0), _ptr(bias_kv),
              B, T, D, num_kv_heads, k_out.data_ptr(), v_out.data_ptr(), k_out.stride(0), k_out.stride(1),
              k_out.stride(2), t_offset, _ptr(cos), _ptr(sin), rsb, rst, _stream(h2d))
    return k_out, v_out


def _rope_args(rope, B: int, T: int):
    """Normalises (cos, sin) of shape [T, 128], [1|B, T, 128] or [1|B, 1, T, 128] to fp32."""
    if rope is None:
        return None, None, 0, 0
    cos, sin = rope
    out = []
    for t in (cos, sin):
        t = t.detach()
        if t.dim() == 4:
            t = t[:, 0]
        if t.dim() == 2:
            t = t.unsqueeze(0)
        if t.shape[-1] != HEAD_DIM or t.shape[-2] != T or t.shape[0] not in (1, B):
            raise RuntimeError(f"rope cos/sin must be [1|B, T, 128], got {tuple(t.shape)}")
        out.append(t.to(torch.float32).contiguous())
    cos, sin = out
    sb = 0 if cos.shape[0] == 1 else cos.stride(0)
    return cos, sin, sb, cos.stride(1)


# ----------------------------------------------------------------- stage 1 --
def route_ema_blend(x: torch.Tensor, beta: float, logits: Optional[torch.Tensor] = None,
                    b2: Optional[torch.Tensor] = None, gate: Optional[torch.Tensor] = None,
                    levels: int = 2, l3: Optional[torch.Tensor] = None,
                    want_lam: bool = True, ema_state: Optional[torch.Tensor] = None,
                    ema_out: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """H = lam0 * x + lam1 * EMA(x) (+ lam2 * L3) with lam = softmax(logits + b2) (or `gate`).

    x [B, T, D] bf16 (token rows contiguous in D); l3 [B, T3, D] bf16 or None.
    ema_state: fp32 [B, D] EMA state before token 0 (None: zero, the
    reference's restart on every call); ema_out: fp32 [B, D] buffer that
    receives the state after token T-1. Returns H [B, T, D] bf16 and lam
    [B, T, L] fp32.
    """
    _check_cuda(x, logits, gate, l3, ema_state, ema_out)
    for name, t in (("ema_state", ema_state), ("ema_out", ema_out)):
        if t is not None and (t.dtype != torch.float32 or tuple(t.shape) != (x.shape[0], x.shape[2])
                              or not t.is_contiguous()):
            raise RuntimeError(f"route_ema_blend: {name} must be a contiguous fp32 [B, D] tensor")
    if ema_state is not None and ema_out is not None and ema_state.data_ptr() == ema_out.data_ptr():
        raise RuntimeError("route_ema_blend: ema_state and ema_out must be different buffers")
    _check_bf16(x, l3)
    B, T, D = x.shape
    if x.stride(2) != 1:
        x = x.contiguous()
    h = torch.empty((B, T, D), dtype=torch.bfloat16, device=x.device)
    lam = torch.empty((B, T, levels), dtype=torch.float32, device=x.device) if want_lam else None
    l3_sb = l3_st = 0
    T3 = 0
    if levels == 3:
        if l3 is None:
            raise RuntimeError("route_ema_blend: three levels need an L3 memory")
        if l3.stride(2) != 1:
            l3 = l3.contiguous()
        T3 = l3.shape[1]
        l3_sb, l3_st = l3.stride(0), (l3.stride(1) if T3 > 1 else 0)
    ws_bytes = _lib.load().fmka_route_ema_blend_workspace_size(B, T, D)
    ws = _WS.get(x.device, ws_bytes)
    b2c = _f32(b2)
    logits_c = None if logits is None else logits.contiguous()
    gate_c = None if gate is None else gate.to(torch.float32).contiguous()
    if ema_state is None and ema_out is None:
        _lib.call("fmka_route_ema_blend", x.data_ptr(), x.stride(0), x.stride(1), _ptr(logits_c), _ptr(b2c),
                  _ptr(gate_c), levels, _ptr(l3), l3_sb, l3_st, T3, float(beta), B, T, D, h.data_ptr(),
                  h.stride(0), h.stride(1), _ptr(lam), _ptr(ws), ws_bytes, _stream(x))
    else:
        _lib.call("fmka_route_ema_blend_state", x.data_ptr(), x.stride(0), x.stride(1), _ptr(logits_c), _ptr(b2c),
                  _ptr(gate_c), levels, _ptr(l3), l3_sb, l3_st, T3, float(beta), B, T, D, h.data_ptr(),
                  h.stride(0), h.stride(1), _ptr(lam), _ptr(ema_state), _ptr(ema_out), _ptr(ws), ws_bytes,
                  _stream(x))
    return h, lam


def route_ema_blend_kv(y: torch.Tensor, beta: float, logits: torch.Tensor, b2: Optional[torch.Tensor], B: int,
                       T: int, num_kv_heads: int, bias: Optional[torch.Tensor] = None,
                       rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                       k_out: Optional[torch.Tensor] = None, v_out: Optional[torch.Tensor] = None,
                       t_offset: int = 0, want_lam: bool = True, ema_state: Optional[torch.Tensor] = None,
                       ema_out: Optional[torch.Tensor] = None, y3: Optional[torch.Tensor] = None):
    """K/V of the route blend from y = x [Wk ; Wv]^T ([B*T, 2*Hkv*128] bf16).

    K = lam0 * yk + lam1 * EMA(yk) + bk (then RoPE), V likewise: the reference's
    k/v projection of lam0 * x + lam1 * EMA(x), in the commuted order (the EMA
    runs along tokens, the projection along channels). Written head-split into
    k_out / v_out ([B, Hkv, Tcap, 128]) at token slots [t_offset, t_offset + T).
    ema_state / ema_out: fp32 [B, 2*Hkv*128] states of EMA(y). y3: the third
    level projected, l3 [Wk ; Wv]^T ([B, T3, 2*Hkv*128] bf16; token t uses row
    min(t, T3 - 1)); logits then hold 3 levels. Returns (k_out, v_out, lam
    [B, T, L] fp32 or None).
    """
    _check_cuda(y, logits, ema_state, ema_out, y3)
    _check_bf16(y, y3)
    L = 3 if y3 is not None else 2
    y3_sb = y3_st = 0
    T3 = 0
    if y3 is not None:
        if y3.dim() != 3 or y3.shape[0] != B or y3.shape[2] != 2 * num_kv_heads * HEAD_DIM or y3.stride(2) != 1:
            raise RuntimeError("route_ema_blend_kv: y3 must be [B, T3, 2*Hkv*128] with contiguous rows")
        T3 = y3.shape[1]
        y3_sb, y3_st = y3.stride(0), (y3.stride(1) if T3 > 1 else 0)
    N = 2 * num_kv_heads * HEAD_DIM
    if y.dim() != 2 or y.shape[0] != B * T or y.shape[1] != N or y.stride(1) != 1:
        raise RuntimeError(f"route_ema_blend_kv: y must be [B*T, {N}] with contiguous rows")
    for name, t in (("ema_state", ema_state), ("ema_out", ema_out)):
        if t is not None and (t.dtype != torch.float32 or tuple(t.shape) != (B, N) or not t.is_contiguous()):
            raise RuntimeError(f"route_ema_blend_kv: {name} must be a contiguous fp32 [B, {N}] tensor")
    if ema_state is not None and ema_out is not None and ema_state.data_ptr() == ema_out.data_ptr():
        raise RuntimeError("route_ema_blend_kv: ema_state and ema_out must be different buffers")
    if k_out is None:
        k_out = torch.empty((B, num_kv_heads, T, HEAD_DIM), dtype=torch.bfloat16, device=y.device)
    if v_out is None:
        v_out = torch.empty_like(k_out)
    if k_out.stride() != v_out.stride():
        raise RuntimeError("route_ema_blend_kv: k and v outputs must share strides")
    lam = torch.empty((B, T, L), dtype=torch.float32, device=y.device) if want_lam else None
    cos, sin, rsb, rst = _rope_args(rope, B, T)
    ws_bytes = _lib.load().fmka_route_ema_blend_kv_workspace_size(B, T, num_kv_heads)
    ws = _WS.get(y.device, ws_bytes)
    _lib.call("fmka_route_ema_blend_kv", y.data_ptr(), T * y.stride(0), y.stride(0), _ptr(logits.contiguous()),
              _ptr(_f32(b2)), _ptr(y3), y3_sb, y3_st, T3, float(beta), B, T, num_kv_heads, _ptr(_f32(bias)), k_out.data_ptr(), v_out.data_ptr(),
              k_out.stride(0), k_out.stride(1), k_out.stride(2), t_offset, _ptr(cos), _ptr(sin), rsb, rst,
              _ptr(lam), _ptr(ema_state), _ptr(ema_out), _ptr(ws), ws_bytes, _stream(y))
    return k_out, v_out, lam


def causal_prefix_ema(x: torch.Tensor, beta: float = 0.9, state: Optional[torch.Tensor] = None,
                      state_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """L2[t] = beta * L2[t-1] + (1 - beta) * x[t] with L2[-1] = 0 (session_memory.py:6-22),
    or L2[-1] = `state` (fp32 [B, D]) to continue an earlier call; `state_out`
    (fp32 [B, D]) receives L2[T-1].

    Runs the stage-1 kernel with the gate fixed to (0, 1), so H == EMA(x).
    """
    B, T, _ = x.shape
    gate = torch.zeros((B * T, 2), dtype=torch.float32, device=x.device)
    gate[:, 1] = 1.0
    h, _ = route_ema_blend(x, beta, gate=gate, levels=2, want_lam=False, ema_state=state, ema_out=state_out)
    return h


# --------------------------------------------------------------- attention --
def attn_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                 scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                 want_lse: bool = True) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Causal (bottom-right aligned) GQA attention on tcgen05.

    q [B, Hq, Tq, 128], k/v [B, Hkv, Tk, 128] (any strides with contiguous head
    dim). Returns o [B, Tq, Hq, 128] (or into `out`, any [B, Tq, Hq, 128]-indexable
    strided view) and lse [B, Hq, Tq] fp32.
    """
    _check_cuda(q, k, v)
    _check_bf16(q, k, v)
    B, Hq, Tq, Dh = q.shape
    _, Hkv, Tk, _ = k.shape
    if k.stride() != v.stride() or k.shape != v.shape:
        raise RuntimeError("attn_prefill: k and v must have the same shape and strides")
    if scale is None:
        scale = 1.0 / math.sqrt(Dh)
    if out is None:
        out = torch.empty((B, Tq, Hq, Dh), dtype=torch.bfloat16, device=q.device)
    lse = torch.empty((B, Hq, Tq), dtype=torch.float32, device=q.device) if want_lse else None
    _lib.call("fmka_attn_fwd_prefill", q.data_ptr(), q.stride(0), q.stride(1), q.stride(2), k.data_ptr(),
              v.data_ptr(), k.stride(0), k.stride(1), k.stride(2), out.data_ptr(), out.stride(0), out.stride(1),
              out.stride(2), _ptr(lse), lse.stride(0) if lse is not None else 0,
              lse.stride(1) if lse is not None else 0, B, Hq, Hkv, Tq, Tk, Dh, int(causal), float(scale),
              _stream(q))
    return out, lse


def attn_prefill_scatter(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, dst_ptrs: Sequence[int],
                         rows_per_dst: int, o_strides: Tuple[int, int, int], causal: bool = True,
                         scale: Optional[float] = None) -> None:
    """attn_prefill with the output rows split over several buffers: query rows
    [j * rows_per_dst, (j + 1) * rows_per_dst) go to dst_ptrs[j] (device
    addresses, local or peer-mapped; at most 8), indexed [b, t, h, :] with
    element strides o_strides = (sb, st, sh). No LSE."""
    _check_cuda(q, k, v)
    _check_bf16(q, k, v)
    B, Hq, Tq, Dh = q.shape
    _, Hkv, Tk, _ = k.shape
    if k.stride() != v.stride() or k.shape != v.shape:
        raise RuntimeError("attn_prefill_scatter: k and v must have the same shape and strides")
    if scale is None:
        scale = 1.0 / math.sqrt(Dh)
    n = len(dst_ptrs)
    arr = (_lib.ctypes.c_void_p * max(n, 1))(*dst_ptrs)
    sb, st, sh = o_strides
    _lib.call("fmka_attn_fwd_prefill_scatter", q.data_ptr(), q.stride(0), q.stride(1), q.stride(2), k.data_ptr(),
              v.data_ptr(), k.stride(0), k.stride(1), k.stride(2), arr, n, int(rows_per_dst), int(sb), int(st),
              int(sh), B, Hq, Hkv, Tq, Tk, Dh, int(causal), float(scale), _stream(q))


def attn_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float] = None,
                num_splits: int = 0, out: Optional[torch.Tensor] = None,
                want_lse: bool = True) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Single-token decode attention over Tk cached keys (split along the keys).

    q [B, Hq, 1, 128] or [B, Hq, 128]; k/v [B, Hkv, Tk, 128] (strided views of a
    larger cache are fine). Returns o [B, 1, Hq, 128] and lse [B, Hq].
    """
    _check_cuda(q, k, v)
    _check_bf16(q, k, v)
    if q.dim() == 4:
        if q.shape[2] != 1:
            raise RuntimeError("attn_decode: one query token per sequence")
        q3 = q[:, :, 0]
    else:
        q3 = q
    B, Hq, Dh = q3.shape
    _, Hkv, Tk, _ = k.shape
    if k.stride() != v.stride() or k.shape != v.shape:
        raise RuntimeError("attn_decode: k and v must have the same shape and strides")
    if q3.stride(2) != 1:
        q3 = q3.contiguous()
    if scale is None:
        scale = 1.0 / math.sqrt(Dh)
    if out is None:
        out = torch.empty((B, 1, Hq, Dh), dtype=torch.bfloat16, device=q.device)
    lse = torch.empty((B, Hq), dtype=torch.float32, device=q.device) if want_lse else None
    lib = _lib.load()
    ws_bytes = lib.fmka_attn_decode_workspace_size(B, Hq, Hkv, Tk, num_splits)
    ws = _WS.get(q.device, ws_bytes)
    _lib.call("fmka_attn_decode_splitkv", q3.data_ptr(), q3.stride(0), q3.stride(1), k.data_ptr(), v.data_ptr(),
              k.stride(0), k.stride(1), k.stride(2), out.data_ptr(), out.stride(0), out.stride(2), _ptr(lse),
              lse.stride(0) if lse is not None else 0, B, Hq, Hkv, Tk, Dh, float(scale), num_splits, _ptr(ws),
              ws_bytes, _stream(q))
    return out, lse


# ----------------------------------------------------- decoder-layer norm --
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """RMSNorm over the last dimension as transformers' LlamaRMSNorm computes it
    for bf16 input: bf16(w * bf16(x * rsqrt(mean(x^2) + eps))), one pass."""
    _check_cuda(x, weight)
    _check_bf16(x, weight)
    D = x.shape[-1]
    if weight.shape != (D,) or not weight.is_contiguous():
        raise RuntimeError("rmsnorm: weight must be a contiguous [D] tensor")
    x2 = x.reshape(-1, D)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    y2 = out.view(-1, D)
    _lib.call("fmka_rmsnorm_bf16", x2.data_ptr(), x2.stride(0), weight.data_ptr(), float(eps), y2.data_ptr(),
              y2.stride(0), x2.shape[0], D, _stream(x))
    return out


def silu_mul(g: torch.Tensor, u: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16(bf16(silu(g)) * u), the SiLU product of a gated MLP, in one pass
    (out may be g)."""
    _check_cuda(g, u)
    _check_bf16(g, u)
    if g.shape != u.shape or not g.is_contiguous() or not u.is_contiguous():
        raise RuntimeError("silu_mul: g and u must be contiguous tensors of the same shape")
    if out is None:
        out = torch.empty_like(g)
    elif out.shape != g.shape or not out.is_contiguous() or out.dtype != torch.bfloat16:
        raise RuntimeError("silu_mul: out must be a contiguous bf16 tensor of g's shape")
    _lib.call("fmka_silu_mul_bf16", g.data_ptr(), u.data_ptr(), out.data_ptr(), g.numel(), _stream(g))
    return out


# ------------------------------------------------------------ L3 recall --
def gemm_f32out(a: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[M, N] = a[M, K] @ w[N, K]^T in fp32 (bf16 operands, tcgen05)."""
    _check_cuda(a, w)
    _check_bf16(a, w)
    if a.dim() != 2 or w.dim() != 2 or a.shape[1] != w.shape[1]:
        raise RuntimeError("gemm_f32out: expected a [M, K] and w [N, K]")
    if a.stride(1) != 1 or w.stride(1) != 1:
        raise RuntimeError("gemm_f32out: inner dimension must be contiguous")
    M, K = a.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, (N + 7) // 8 * 8), dtype=torch.float32, device=a.device)[:, :N]
    _lib.call("fmka_gemm_bf16_f32out", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(),
              out.stride(0), M, N, K, _stream(a))
    return out


def l3_block_mean(x: torch.Tensor, block_len: int) -> torch.Tensor:
    """Block summaries q[b * nq + j] = bf16(mean of x[b, j*L:(j+1)*L]) of x [B, T, D]
    (nq = ceil(T / L), the last block partial): the queries of the L3 recall."""
    _check_cuda(x)
    _check_bf16(x)
    if x.dim() != 3 or x.stride(2) != 1:
        raise RuntimeError("l3_block_mean: x must be [B, T, D] with contiguous channels")
    B, T, D = x.shape
    nq = (T + block_len - 1) // block_len
    q = torch.empty((B * nq, D), dtype=torch.bfloat16, device=x.device)
    _lib.call("fmka_l3_block_mean_bf16", x.data_ptr(), x.stride(0), x.stride(1), B, T, D, block_len,
              q.data_ptr(), q.stride(0), _stream(x))
    return q


def l3_topr(scores: torch.Tensor, top_r: int, scale: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """The top_r best columns of every row of scores [M, N] (fp32; ties: the lower
    index first) and softmax(scale * score) over them: idx int32 [M, R], w fp32 [M, R]."""
    _check_cuda(scores)
    if scores.dtype != torch.float32 or scores.dim() != 2 or scores.stride(1) != 1:
        raise RuntimeError("l3_topr: scores must be fp32 [M, N] with contiguous rows")
    M, N = scores.shape
    idx = torch.empty((M, top_r), dtype=torch.int32, device=scores.device)
    w = torch.empty((M, top_r), dtype=torch.float32, device=scores.device)
    _lib.call("fmka_l3_topr_f32", scores.data_ptr(), scores.stride(0), M, N, top_r, float(scale),
              idx.data_ptr(), w.data_ptr(), _stream(scores))
    return idx, w


def l3_recall_gather(idx: torch.Tensor, w: torch.Tensor, values: torch.Tensor, B: int, T: int, block_len: int,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """R[b, t] = sum_r w[b * nq + t // L, r] * values[idx[.., r]] for every token: [B, T, D] bf16."""
    _check_cuda(idx, w, values)
    _check_bf16(values)
    if idx.dtype != torch.int32 or w.dtype != torch.float32 or idx.shape != w.shape or not idx.is_contiguous() \
            or not w.is_contiguous():
        raise RuntimeError("l3_recall_gather: idx int32 and w fp32 of the same contiguous shape [M, R]")
    if values.dim() != 2 or values.stride(1) != 1:
        raise RuntimeError("l3_recall_gather: values must be [n_chunks, D] with contiguous channels")
    n_chunks, D = values.shape
    if out is None:
        out = torch.empty((B, T, D), dtype=torch.bfloat16, device=values.device)
    _lib.call("fmka_l3_recall_gather_bf16", idx.data_ptr(), w.data_ptr(), idx.shape[1], values.data_ptr(),
              values.stride(0), n_chunks, D, B, T, block_len, out.data_ptr(), out.stride(0), out.stride(1),
              _stream(values))
    return out


def l3_chunk_recall(x: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, top_r: int, block_len: int = 64,
                    scale: Optional[float] = None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The L3 memory R [B, T, D] recalled for x [B, T, D] from a chunk bank (keys,
    values [n_chunks, D] bf16): block summaries of x score every key, each block
    takes its top_r chunks and softmax(scale * score) weights (scale defaults to
    1/sqrt(D)), and every token of the block receives their weighted sum.
    Returns (R, idx [B * nq, top_r] int32, w [B * nq, top_r] fp32)."""
    B, T, D = x.shape
    if keys.shape != values.shape or keys.shape[1] != D:
        raise RuntimeError("l3_chunk_recall: keys and values must both be [n_chunks, D]")
    q = l3_block_mean(x, block_len)
    scores = gemm_f32out(q, keys)
    idx, w = l3_topr(scores, top_r, D ** -0.5 if scale is None else scale)
    return l3_recall_gather(idx, w, values, B, T, block_len), idx, w


# ---------------------------------------- reference-compatible op wrappers --
def has_fastmka_cuda() -> bool:
    """True when the library loads and a CUDA device is visible (mka/cuda/ops.py:25-26)."""
    try:
        _lib.load()
    except Exception:
        return False
    return torch.cuda.is_available()


def has_fused_route_mka_cuda() -> bool:
    """Same probe for the fused route op (mka/cuda/ops.py:43-44)."""
    return has_fastmka_cuda()


def _to_bf16(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)


def fastmka_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True) -> torch.Tensor:
    """Drop-in for mka.cuda.ops.fastmka_attn (ops.py:73-77): causal attention with
    offset Tk - Tq, output [B, H, Tq, D] in q's dtype. Adds GQA and bf16; D == 128.
    As in the reference kernel (fastmka_attn.cu:95,126-127), with causal and
    Tq > Tk the first Tq - Tk queries see no key and their rows are zero."""
    _check_cuda(q, k, v)
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise RuntimeError("q/k/v must be 4D")
    if q.size(0) != k.size(0) or k.shape != v.shape or q.size(3) != k.size(3):
        raise RuntimeError("B/H mismatch or head dim mismatch")
    if q.size(1) % k.size(1) != 0:
        raise RuntimeError("B/H mismatch")
    if q.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise RuntimeError(f"unsupported dtype {q.dtype}")
    qb, kb, vb = _to_bf16(q), _to_bf16(k), _to_bf16(v)
    B, H, Tq, D = q.shape
    Tk = k.size(2)
    out = torch.empty((B, H, Tq, D), dtype=torch.bfloat16, device=q.device)
    blind = Tq - Tk if causal and Tq > Tk else 0  # queries before the first key
    if blind:
        out[:, :, :blind].zero_()
        qb, out_seen = qb[:, :, blind:], out[:, :, blind:]
    else:
        out_seen = out
    if qb.size(2) == 1 and causal:
        attn_decode(qb, kb, vb, out=out_seen.permute(0, 2, 1, 3), want_lse=False)
    else:
        attn_prefill(qb, kb, vb, causal=causal, out=out_seen.permute(0, 2, 1, 3), want_lse=False)
    return out if q.dtype == torch.bfloat16 else out.to(q.dtype)


def fused_route_mka_attn(q: torch.Tensor, l1: torch.Tensor, l2: torch.Tensor, l3: torch.Tensor,
                         lam: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor) -> torch.Tensor:
    """Drop-in for mka.cuda.ops.fused_route_mka_attn (ops.py:47-70): fused = sum_l lam_l * l_l,
    k = fused wk^T, v = fused wv^T, causal attention with q. MHA (H * Dh == D), no cache."""
    _check_cuda(q, l1, l2, l3, lam, wk, wv)
    if q.dim() != 4:
        raise RuntimeError("q must be [B,H,T,Dh]")
    if l1.dim() != 3 or l2.dim() != 3 or l3.dim() != 3:
        raise RuntimeError("l1/l2/l3 must be [B,T,D]")
    if lam.dim() != 3:
        raise RuntimeError("lam must be [B,T,L]")
    if wk.dim() != 2 or wv.dim() != 2:
        raise RuntimeError("wk/wv must be [D,D]")
    B, H, T, Dh = q.shape
    D = l1.shape[2]
    L = lam.shape[2]
    if l1.shape != l2.shape or l1.shape != l3.shape:
        raise RuntimeError("l1/l2/l3 shapes must match")
    if l1.shape[0] != B or l1.shape[1] != T:
        raise RuntimeError("l1 batch/seq must match q")
    if lam.shape[0] != B or lam.shape[1] != T:
        raise RuntimeError("lam batch/seq must match q")
    if L not in (2, 3):
        raise RuntimeError("lam last dim must be 2 or 3")
    if H * Dh != D or wk.shape != (D, D) or wv.shape != (D, D):
        raise RuntimeError("expected H*Dh == D (hidden_size) and wk/wv [D,D]")
    l1b, l2b, l3b = (_to_bf16(t).contiguous() for t in (l1, l2, l3))
    gate = lam.reshape(B * T, L).to(torch.float32).contiguous()
    h = torch.empty((B, T, D), dtype=torch.bfloat16, device=q.device)
    _lib.call("fmka_route_blend", l1b.data_ptr(), l1b.stride(0), l1b.stride(1), l2b.data_ptr(), l2b.stride(0),
              l2b.stride(1), l3b.data_ptr() if L == 3 else None, l3b.stride(0), l3b.stride(1), T, gate.data_ptr(), L,
              B, T, D, h.data_ptr(), h.stride(0), h.stride(1), _stream(q))
    w_kv = torch.cat([_to_bf16(wk), _to_bf16(wv)], 0).contiguous()
    k, v = kv_proj(h.reshape(B * T, D), w_kv, None, B, T, H)
    out = torch.empty((B, H, T, Dh), dtype=torch.bfloat16, device=q.device)
    attn_prefill(_to_bf16(q), k, v, causal=True, out=out.permute(0, 2, 1, 3), want_lse=False)
    return out if q.dtype == torch.bfloat16 else out.to(q.dtype)
