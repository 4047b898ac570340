"""FastMKA layer partitioned over the GPUs of one box by (sequence x kv head).

The reference has no distributed code inside the layer (DDP / HF tensor
parallel live in its scripts, scripts/train_hf_patch.py:97-129). Here the unit
of work is one (sequence, kv head) pair: a kv head, its G = Hq / Hkv query
heads, and the fused memory of that sequence.

  * world <= batch: every rank owns whole sequences (batch / world of them)
    and runs the unsharded layer on them; no collective at all.
  * world > batch: the ranks of a sequence group (world / batch ranks per
    sequence) split the kv heads. Each rank computes the router for its
    sequence - it needs all of q, so its first layer is not split - and Q, K,
    V (stage 1 in the projected space of its own kv heads) and causal
    attention for its own heads. Then the group exchanges data in one of two
    ways (`transport`):
      "peer" (default): the sequence's T rows are split into one block per
        rank. The attention kernel stores each row block of its output
        straight into the owning rank's gather buffer (peer memory over
        NVLink); after a flag barrier each rank runs o_proj on its own row
        block only - a 1/gs share of the o_proj FLOPs - and the GEMM's
        epilogue stores every output row into all ranks' output buffers;
        a second barrier completes the step. Two kernels carry both
        exchanges; no collective library call and no replicated o_proj.
      "nccl": one NCCL all-gather of the attention output feeds o_proj,
        which reads the gathered [ranks, B*T, heads*128] buffer in place
        (fmka_gemm_bf16_kblocked) and runs whole on every rank.
    Either way every rank ends with the full layer output of its sequence.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.nn as nn

from . import ops
from .layers.forward import fastmka_forward, project_l3
from .layers.prepared import PreparedWeights
from .peer import PeerRegion, bf16_view, exchange_plan

HEAD_DIM = ops.HEAD_DIM


@dataclass(frozen=True)
class RankPlan:
    rank: int
    batch: Tuple[int, int]     # [b0, b1) sequences this rank works on
    kv_heads: Tuple[int, int]  # [h0, h1) kv heads this rank computes
    group: Tuple[int, ...]     # ranks that share these sequences (all-gather group)


def plan_units(batch: int, num_kv_heads: int, world_size: int) -> List[RankPlan]:
    """Assigns the batch x num_kv_heads (sequence, kv head) units to ranks."""
    if world_size < 1 or batch < 1 or num_kv_heads < 1:
        raise ValueError("batch, num_kv_heads and world_size must be positive")
    plans = []
    if world_size <= batch:
        if batch % world_size:
            raise ValueError(f"batch {batch} does not split over {world_size} ranks")
        per = batch // world_size
        for r in range(world_size):
            plans.append(RankPlan(r, (r * per, (r + 1) * per), (0, num_kv_heads), (r,)))
        return plans
    if world_size % batch:
        raise ValueError(f"{world_size} ranks do not split into groups over {batch} sequences")
    gs = world_size // batch
    if num_kv_heads % gs:
        raise ValueError(f"{num_kv_heads} kv heads do not split over {gs} ranks")
    hpr = num_kv_heads // gs
    for r in range(world_size):
        b, j = divmod(r, gs)
        plans.append(RankPlan(r, (b, b + 1), (j * hpr, (j + 1) * hpr), tuple(range(b * gs, (b + 1) * gs))))
    return plans


def shard_weights(W: PreparedWeights, num_heads: int, num_kv_heads: int, kv_heads: Tuple[int, int]) -> PreparedWeights:
    """The prepared weights restricted to kv heads [h0, h1) and their query heads;
    the router rows (the folded first layer) and o_proj stay whole."""
    h0, h1 = kv_heads
    g = num_heads // num_kv_heads
    q0, q1 = h0 * g * HEAD_DIM, h1 * g * HEAD_DIM
    nq = num_heads * HEAD_DIM
    nk = num_kv_heads * HEAD_DIM
    k0, k1 = h0 * HEAD_DIM, h1 * HEAD_DIM
    w_qr = torch.cat([W.w_qr[q0:q1], W.w_qr[nq:]], 0).contiguous()
    b_qr = torch.cat([W.b_qr[q0:q1], W.b_qr[nq:]], 0).contiguous() if W.b_qr is not None else None
    w_kv = torch.cat([W.w_kv[k0:k1], W.w_kv[nk + k0:nk + k1]], 0).contiguous()
    b_kv = torch.cat([W.b_kv[k0:k1], W.b_kv[nk + k0:nk + k1]], 0).contiguous() if W.b_kv is not None else None
    return PreparedWeights(key=W.key + (kv_heads,), w_qr=w_qr, b_qr=b_qr, w2=W.w2, b2=W.b2,
                           router_hidden=W.router_hidden, levels=W.levels, act=W.act, w_kv=w_kv, b_kv=b_kv,
                           w_o=W.w_o, b_o=W.b_o)


class HeadShardedFastMKA(nn.Module):
    """Runs one FastMKA attention layer (an HFFastMKAAttention or FastMKAAttention)
    on this rank's share of a batch, per `plan_units`.

    `groups` maps each sequence group (tuple of ranks) to its torch.distributed
    process group (NCCL); create them on every rank in the same order with
    `make_groups` before the first forward.

    With transport "peer" the returned output is a view of this layer's shared
    output buffer: it stays valid until the next forward of this module (copy
    it to keep it longer). The peer exchange needs T divisible by the group
    size; other lengths take the NCCL all-gather. Call `close()` on every rank
    before the process group is destroyed.

    A peer barrier that waits longer than its 2 s limit (a rank of the group
    never arrived) returns with FMKA_STATUS_PEER_TIMEOUT set in the device
    status word, and the step's output is then incomplete. With
    `check_peer_status` (the default) every peer-exchange forward reads the
    status word once at its end (one stream synchronisation) and raises
    PeerExchangeError; a caller that polls `ops.device_status()` itself can turn
    the check off to keep the stream asynchronous.
    """

    def __init__(self, layer: nn.Module, batch: int, rank: int, world_size: int, groups: Optional[dict] = None,
                 transport: str = "peer", check_peer_status: bool = True):
        super().__init__()
        if transport not in ("peer", "nccl"):
            raise ValueError("transport must be 'peer' or 'nccl'")
        self.transport = transport
        self.check_peer_status = check_peer_status
        self._region: Optional[PeerRegion] = None
        self._region_key = None
        self.layer = layer
        self.num_heads = getattr(layer, "num_heads", None) or layer.cfg.num_heads
        self.num_kv_heads = getattr(layer, "num_key_value_heads", None) or self.num_heads
        self.beta = getattr(layer, "ema_beta", None)
        if self.beta is None:
            self.beta = layer.cfg.ema_beta
        self.use_l3 = getattr(layer, "use_l3", None)
        if self.use_l3 is None:
            self.use_l3 = layer.cfg.use_l3
        self.plan = plan_units(batch, self.num_kv_heads, world_size)[rank]
        self.groups = groups or {}
        self._w: Optional[PreparedWeights] = None
        self._w_key = None

    def _weights(self, device) -> PreparedWeights:
        W = self.layer.prepared(device)
        if self._w is None or self._w_key != W.key:
            h0, h1 = self.plan.kv_heads
            if (h0, h1) == (0, self.num_kv_heads):
                self._w = W
            else:
                self._w = shard_weights(W, self.num_heads, self.num_kv_heads, self.plan.kv_heads)
            self._w_key = W.key
        return self._w

    def forward(self, x: torch.Tensor, rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                l3_memory: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x: [b1 - b0, T, D], this rank's sequences. Returns the layer output for them."""
        import torch.distributed as dist

        W = self._weights(x.device)
        h0, h1 = self.plan.kv_heads
        g = self.num_heads // self.num_kv_heads
        hq_r, hkv_r = (h1 - h0) * g, h1 - h0
        with torch.no_grad():
            if len(self.plan.group) == 1:
                return fastmka_forward(x, W, self.num_heads, self.num_kv_heads, self.beta, self.use_l3,
                                       l3_memory=l3_memory, rope=rope)["out"]
            B, T, D = x.shape
            gs = len(self.plan.group)
            if self.transport == "peer" and B == 1 and T % gs == 0:
                return self._forward_peer(x, W, hq_r, hkv_r, l3_memory, rope)
            r = fastmka_forward_heads(x, W, hq_r, hkv_r, self.beta, self.use_l3, l3_memory, rope)
            o = r.view(B * T, hq_r * HEAD_DIM)
            flat = torch.empty((gs * B * T, hq_r * HEAD_DIM), dtype=torch.bfloat16, device=x.device)
            dist.all_gather_into_tensor(flat, o, group=self.groups[self.plan.group])
            gathered = flat.view(gs, B * T, hq_r * HEAD_DIM)  # group rank j's heads in block j
            return ops.gemm_kblocked(gathered, W.w_o, W.b_o).view(B, T, D)

    def _peer_region(self, nbytes: int, key, device) -> PeerRegion:
        if self._region is None or self._region_key != key:
            if self._region is not None:
                self._region.close()
            gs = len(self.plan.group)
            idx = self.plan.group.index(self.plan.rank)
            self._region = PeerRegion(self.groups[self.plan.group], idx, gs, nbytes, device)
            self._region_key = key
        return self._region

    def _forward_peer(self, x, W, hq_r, hkv_r, l3_memory, rope) -> torch.Tensor:
        _, T, D = x.shape
        gs = len(self.plan.group)
        width = hq_r * HEAD_DIM
        pl = exchange_plan(gs, self.plan.group.index(self.plan.rank), T, D, width)
        reg = self._peer_region(pl.nbytes, (T, D, width, str(x.device)), x.device)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        q, k, v = heads_qkv(x, W, hq_r, hkv_r, self.beta, self.use_l3, l3_memory, rope)
        # row block j of this rank's attention output -> block `me` of rank j's gather area
        ops.attn_prefill_scatter(q, k, v, [p + pl.attn_dst_off for p in reg.ptrs], pl.rows,
                                 (pl.rows * width, width, HEAD_DIM))
        reg.barrier(stream)  # every rank's rows of this block have landed here
        gathered = bf16_view(reg.local + pl.gather_off, (gs, pl.rows, width), x.device)
        # o_proj on this rank's rows, each written into every rank's output
        ops.gemm_kblocked_scatter(gathered, W.w_o, W.b_o, [p + pl.out_off for p in reg.ptrs], pl.gemm_row0, D)
        reg.barrier(stream)  # every rank's o_proj rows have landed here
        if self.check_peer_status:
            raise_on_peer_timeout()
        return bf16_view(reg.local + pl.out_off, (T, D), x.device).view(1, T, D)

    def close(self) -> None:
        """Releases the peer buffers (collective over the sequence group)."""
        if self._region is not None:
            self._region.close()
            self._region = None
            self._region_key = None


class PeerExchangeError(RuntimeError):
    """A cross-GPU barrier of the peer exchange ran out of time."""


def raise_on_peer_timeout() -> None:
    """Reads the device status word (without clearing it) and raises
    PeerExchangeError when a peer barrier has timed out since it was last cleared."""
    if ops.device_status(clear=False) & ops.STATUS_PEER_TIMEOUT:
        raise PeerExchangeError("head-sharded FastMKA: a peer barrier ran out of time (a rank of the sequence "
                                "group did not arrive within 2 s); this step's layer output is incomplete")


def fastmka_forward_heads(x: torch.Tensor, W: PreparedWeights, hq: int, hkv: int, beta: float, use_l3: bool,
                          l3_memory: Optional[torch.Tensor], rope) -> torch.Tensor:
    """Stages 1-4 of the layer for a subset of heads (W restricted by shard_weights):
    returns the attention output [B, T, hq, 128]."""
    q, k, v = heads_qkv(x, W, hq, hkv, beta, use_l3, l3_memory, rope)
    o, _ = ops.attn_prefill(q, k, v, causal=True, want_lse=False)
    return o


def heads_qkv(x: torch.Tensor, W: PreparedWeights, hq: int, hkv: int, beta: float, use_l3: bool,
              l3_memory: Optional[torch.Tensor], rope):
    """Stages 1-3 for a subset of heads: q [B, hq, T, 128] and k, v [B, hkv, T, 128]."""
    B, T, D = x.shape
    xb = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
    xb = xb.contiguous()
    L = 3 if use_l3 else 2
    q, logits = ops.qr_proj(xb.view(B * T, D), W.w_qr, W.b_qr, B, T, hq, W.router_hidden, W.w2, L, W.act, rope=rope)
    # this rank's K/V only: the projection first, then the gate / EMA / blend
    # scan over this rank's 2*hkv*128 channels (no stage replicated over d_model)
    y = ops.gemm(xb.view(B * T, D), W.w_kv)
    y3 = project_l3(l3_memory, W, B, D, hkv, x.device) if use_l3 else None
    k, v, _ = ops.route_ema_blend_kv(y, beta, logits, W.b2, B, T, hkv, bias=W.b_kv, rope=rope, want_lam=False, y3=y3)
    return q, k, v


def make_groups(batch: int, num_kv_heads: int, world_size: int) -> dict:
    """Creates the NCCL subgroups of every sequence group (collective: call on all ranks)."""
    import torch.distributed as dist

    groups = {}
    seen = []
    for p in plan_units(batch, num_kv_heads, world_size):
        if len(p.group) > 1 and p.group not in seen:
            seen.append(p.group)
    for grp in seen:
        groups[grp] = dist.new_group(list(grp))
    return groups
