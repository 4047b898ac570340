"""A Llama-architecture transformers model with every self_attn patched to
FastMKA, run over the GPUs of one box by sequence and kv head.

The reference runs the patched model on one device (mka/hf/patch.py:30-48 wraps
each self_attn; its distributed code is DDP / tensor parallel in
scripts/train_hf_patch.py:97-129). Here one process per GPU holds the whole
model (same weights on every rank) and the forward of one long sequence is
split so that no rank repeats another's work:

  residual stream   rank r keeps rows [r T/W, (r+1) T/W) of the hidden states
                    between layers (sequence parallel): embeddings, the
                    RMSNorms, the residual adds and the MLP run on those rows
  router            per token, so each rank computes the gate logits of its own
                    rows (the router's first layer is folded through q_proj,
                    as in the one-GPU layer) and the logits are all-gathered
  attention         rank r owns kv heads [r Hkv/W, (r+1) Hkv/W) and their
                    query heads over the whole sequence: the normed hidden
                    states are all-gathered (NCCL), then q, y = x [Wk ; Wv]^T,
                    y3 = L3 [Wk ; Wv]^T, the gate / EMA / blend scan and the
                    causal attention run for those heads only
  exchange          the attention kernel stores row block j of its output
                    straight into rank j's gather area (peer memory, no NCCL);
                    after a flag barrier rank r runs o_proj on its own rows
                    over all heads, which gives its residual rows directly

Per layer that is one all-gather of the normed hidden states (T x D bf16), one
of the gate logits (T x L fp32) and the row exchange inside the attention
kernel. The logits of the last position (the only ones the prefill needs) come
out on the last rank.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.nn as nn

from .. import ops
from ..layers.prepared import PreparedWeights
from ..peer import PeerRegion, bf16_view
from ..sharded import raise_on_peer_timeout, shard_weights
from .attention import HFFastMKAAttention
from .patch import _iter_layers

HEAD_DIM = ops.HEAD_DIM
_FLAGS = 1024  # bytes before the gather area in each peer region


class SequenceHeadShardedLlama:
    """Runs `model` (a LlamaForCausalLM-style model whose self_attn modules are
    HFFastMKAAttention, e.g. after apply_hf_attention_patch) over `world` ranks.

    Collective: construct, call and `close()` on every rank in the same order,
    with the default process group initialised (NCCL). Needs the kv heads and
    the sequence length to split evenly over the ranks.

    With `check_peer_status` (the default) each forward ends by reading the
    device status word once and raises PeerExchangeError if one of its peer
    barriers ran out of time (a rank never arrived, so some rows are missing);
    pass False to keep the stream asynchronous and poll `ops.device_status()`.
    """

    def __init__(self, model: nn.Module, rank: int, world: int, group=None, check_peer_status: bool = True):
        self.check_peer_status = check_peer_status
        self.model = model
        self.rank, self.world, self.group = rank, world, group
        self.layers = list(_iter_layers(model))
        att = self.layers[0].self_attn
        if not isinstance(att, HFFastMKAAttention):
            raise ValueError("patch the model's self_attn with FastMKA first (apply_hf_attention_patch)")
        self.num_heads, self.num_kv_heads = att.num_heads, att.num_key_value_heads
        if self.num_kv_heads % world:
            raise ValueError(f"{self.num_kv_heads} kv heads do not split over {world} ranks")
        hpr = self.num_kv_heads // world
        self.kv_heads = (rank * hpr, (rank + 1) * hpr)
        self.hkv = hpr
        self.hq = hpr * (self.num_heads // self.num_kv_heads)
        self._w: List[Optional[PreparedWeights]] = [None] * len(self.layers)
        self._keys: List[Optional[tuple]] = [None] * len(self.layers)
        self._regions: List[PeerRegion] = []
        self._region_key = None

    # ---------------------------------------------------------------- setup --
    def _weights(self, i: int, device) -> PreparedWeights:
        W = self.layers[i].self_attn.prepared(device)
        if self._keys[i] != W.key:
            self._w[i] = shard_weights(W, self.num_heads, self.num_kv_heads, self.kv_heads)
            self._keys[i] = W.key
        return self._w[i]

    def _gather_regions(self, rows: int, width: int, device) -> List[PeerRegion]:
        """Two gather areas [world, rows, width] (alternating by layer), each
        mapped into every rank."""
        key = (rows, width, str(device))
        if self._region_key != key:
            self.close_regions()
            nbytes = _FLAGS + self.world * rows * width * 2
            grp = self.group if self.group is not None else _world_group()
            self._regions = [PeerRegion(grp, self.rank, self.world, nbytes, device) for _ in range(2)]
            self._region_key = key
        return self._regions

    # -------------------------------------------------------------- forward --
    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, l3_memory: Optional[torch.Tensor] = None,
                return_hidden: bool = False):
        """input_ids [1, T] (the same on every rank); l3_memory [1, T3, D] (the
        same on every rank) for models patched with use_l3. Returns the logits
        of the last position [1, 1, vocab] on the last rank, None elsewhere;
        with return_hidden also this rank's rows of the final normed hidden
        states ([1, T / world, D]) as a second value."""
        import torch.distributed as dist

        m = self.model
        inner = m.model
        device = input_ids.device
        B, T = input_ids.shape
        if B != 1:
            raise NotImplementedError("the sequence-sharded forward runs one sequence at a time")
        W_ = self.world
        if T % W_:
            raise ValueError(f"{T} tokens do not split into {W_} row blocks")
        rows = T // W_
        r0 = self.rank * rows
        width = self.hq * HEAD_DIM
        att0 = self.layers[0].self_attn
        D = att0.hidden_size
        use_l3 = att0.use_l3
        if use_l3 and l3_memory is not None and l3_memory.shape[0] != 1:
            raise ValueError("l3_memory must be [1, T3, D]")
        regions = self._gather_regions(rows, width, device)
        stream = torch.cuda.current_stream(device).cuda_stream
        grp = self.group

        h = inner.embed_tokens(input_ids[:, r0:r0 + rows])  # [1, rows, D] this rank's rows
        pos = torch.arange(T, device=device).unsqueeze(0)
        cos, sin = inner.rotary_emb(h, pos)  # [1, T, 128]
        rope = (cos, sin)
        x_full = torch.empty((T, D), dtype=torch.bfloat16, device=device)
        l3b = None
        if use_l3 and l3_memory is not None:
            l3b = l3_memory[0].to(torch.bfloat16).contiguous()
        for i, layer in enumerate(self.layers):
            att = layer.self_attn
            Wl = self._weights(i, device)
            L = Wl.levels
            nq = self.hq * HEAD_DIM
            xs = layer.input_layernorm(h).to(torch.bfloat16).reshape(rows, D).contiguous()
            # gate logits of this rank's rows (the q columns computed with them are not needed)
            _, lg_local = ops.qr_proj(xs, Wl.w_qr, Wl.b_qr, 1, rows, self.hq, Wl.router_hidden, Wl.w2, L, Wl.act)
            lg = torch.empty((T, L), dtype=torch.float32, device=device)
            dist.all_gather_into_tensor(x_full, xs, group=grp)
            dist.all_gather_into_tensor(lg, lg_local, group=grp)
            # this rank's heads over the whole sequence
            q, _ = ops.qr_proj(x_full, Wl.w_qr[:nq], Wl.b_qr[:nq] if Wl.b_qr is not None else None, 1, T, self.hq,
                               0, None, L, Wl.act, rope=rope)
            y = ops.gemm(x_full, Wl.w_kv)
            y3 = None
            if use_l3:
                if l3b is None:
                    y3 = torch.zeros((1, 1, 2 * self.hkv * HEAD_DIM), dtype=torch.bfloat16, device=device)
                else:
                    y3 = ops.gemm(l3b, Wl.w_kv).view(1, l3b.shape[0], -1)
            k, v, _ = ops.route_ema_blend_kv(y, att.ema_beta, lg, Wl.b2, 1, T, self.hkv, bias=Wl.b_kv, rope=rope,
                                             want_lam=False, y3=y3)
            reg = regions[i & 1]
            # row block j of the attention output -> block `rank` of rank j's gather area
            ops.attn_prefill_scatter(q, k, v, [p + _FLAGS + self.rank * rows * width * 2 for p in reg.ptrs], rows,
                                     (rows * width, width, HEAD_DIM))
            reg.barrier(stream)  # every rank's block of this rank's rows has landed
            gathered = bf16_view(reg.local + _FLAGS, (W_, rows, width), device)
            o = ops.gemm_kblocked(gathered, Wl.w_o, Wl.b_o).view(1, rows, D)
            h = h + o.to(h.dtype)
            h = h + layer.mlp(layer.post_attention_layernorm(h))
        if self.check_peer_status:
            raise_on_peer_timeout()
        logits = m.lm_head(inner.norm(h[:, -1:])) if self.rank == W_ - 1 else None
        if return_hidden:
            return logits, inner.norm(h)
        return logits

    __call__ = forward

    def close_regions(self) -> None:
        for r in self._regions:
            r.close()
        self._regions = []
        self._region_key = None

    def close(self) -> None:
        """Releases the peer regions (collective over the ranks)."""
        self.close_regions()


def _world_group():
    import torch.distributed as dist

    return dist.group.WORLD
