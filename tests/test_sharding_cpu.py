"""Host-side logic of the (sequence x kv head) partition, on the CPU:
the unit plan, the per-rank weight slices, and - with two gloo ranks - the
all-gather layout that o_proj reads block by block."""
import os

import pytest
import torch
import torch.multiprocessing as mp
import torch.nn as nn

from mka_b200.layers.prepared import prepare
from mka_b200.sharded import plan_units, shard_weights


@pytest.mark.parametrize("batch,hkv,world", [(4, 4, 1), (4, 4, 2), (4, 4, 4), (2, 4, 8), (1, 8, 8), (2, 4, 4),
                                             (1, 4, 2), (8, 8, 8)])
def test_plan_covers_every_unit_once(batch, hkv, world):
    plans = plan_units(batch, hkv, world)
    assert [p.rank for p in plans] == list(range(world))
    seen = set()
    for p in plans:
        for b in range(*p.batch):
            for h in range(*p.kv_heads):
                assert (b, h) not in seen
                seen.add((b, h))
        assert p.rank in p.group
        # every rank of a group works on the same sequences
        assert all(plans[r].batch == p.batch for r in p.group)
    assert seen == {(b, h) for b in range(batch) for h in range(hkv)}
    # whole sequences per rank need no collective
    if world <= batch:
        assert all(len(p.group) == 1 for p in plans)


@pytest.mark.parametrize("batch,hkv,world", [(3, 4, 2), (2, 3, 4), (2, 4, 3)])
def test_plan_rejects_uneven_splits(batch, hkv, world):
    with pytest.raises(ValueError):
        plan_units(batch, hkv, world)


def test_shard_weights_slices_heads_and_keeps_router_and_o_proj():
    torch.manual_seed(0)
    D, H, HKV, R = 512, 4, 2, 64
    q, k, v, o = (nn.Linear(D, n * 128, bias=b) for n, b in ((H, True), (HKV, True), (HKV, True), (H, False)))
    o = nn.Linear(H * 128, D, bias=False)
    router = nn.Sequential(nn.Linear(D, R), nn.SiLU(), nn.Linear(R, 2))
    W = prepare(q, k, v, o, router, torch.device("cpu"))
    parts = [shard_weights(W, H, HKV, (h, h + 1)) for h in range(HKV)]
    # query rows of the shards concatenate to the full query rows; router rows are whole in each
    assert torch.equal(torch.cat([p.w_qr[:2 * 128] for p in parts]), W.w_qr[:H * 128])
    for p in parts:
        assert torch.equal(p.w_qr[2 * 128:], W.w_qr[H * 128:])
        assert p.w_o is W.w_o and p.w2 is W.w2
    assert torch.equal(torch.cat([p.w_kv[:128] for p in parts]), W.w_kv[:HKV * 128])
    assert torch.equal(torch.cat([p.w_kv[128:] for p in parts]), W.w_kv[HKV * 128:])
    assert torch.equal(torch.cat([p.b_kv[:128] for p in parts]), W.b_kv[:HKV * 128])


def _gather_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        M, H, D = 24, 4, 96
        o_full = torch.randn(M, H * 128)       # attention output of all heads, [B*T, Hq*128]
        wo = torch.randn(D, H * 128) / 30
        hpr = H // world
        mine = o_full[:, rank * hpr * 128:(rank + 1) * hpr * 128].contiguous()
        flat = torch.empty(world * M, hpr * 128)  # rank j's block at rows [j*M, (j+1)*M)
        dist.all_gather_into_tensor(flat, mine)
        gathered = flat.view(world, M, hpr * 128)
        # o_proj read block by block, as fmka_gemm_bf16_kblocked does: A[m, k] = blocks[k // kb][m][k % kb]
        kb = hpr * 128
        out = sum(gathered[j] @ wo[:, j * kb:(j + 1) * kb].t() for j in range(world))
        q.put((rank, (out - o_full @ wo.t()).abs().max().item()))
    finally:
        dist.destroy_process_group()


def test_gloo_all_gather_layout_matches_blocked_o_proj():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 2
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=60) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, err in res:
        assert err < 1e-3
