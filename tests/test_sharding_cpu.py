"""Host-side logic of the (sequence x kv head) partition, on the CPU:
the unit plan, the per-rank weight slices, with two gloo ranks the all-gather
layout that o_proj reads block by block, and the peer exchange: the byte plan
of the shared regions (emulated for 2, 4 and 8 ranks) and, with two gloo ranks
and a stand-in for the library, the handle exchange, barrier epochs and
teardown order of PeerRegion."""
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


@pytest.mark.parametrize("gs,T,hq_r,D", [(2, 64, 2, 96), (4, 96, 1, 64), (8, 64, 1, 128)])
def test_peer_exchange_plan_rebuilds_o_proj(gs, T, hq_r, D):
    """Emulates the peer exchange of the head-sharded layer on the CPU with one
    byte region per rank: every rank stores its attention row blocks where the
    plan says (as fmka_attn_fwd_prefill_scatter does), runs o_proj on its own
    gather area and stores its output rows into every region (as
    fmka_gemm_bf16_kblocked_scatter does). Every region must then hold the
    unsharded o_proj output of the whole sequence."""
    from mka_b200.peer import exchange_plan

    torch.manual_seed(gs * 100 + T)
    width = hq_r * 128
    o_full = torch.randn(T, gs * width).bfloat16()      # all heads' attention output
    wo = (torch.randn(D, gs * width) / 40).bfloat16()
    plans = [exchange_plan(gs, r, T, D, width) for r in range(gs)]
    assert len({(p.gather_off, p.out_off, p.nbytes) for p in plans}) == 1  # same layout on every rank
    pl0 = plans[0]
    assert pl0.gather_off % 1024 == 0 and pl0.out_off % 1024 == 0 and pl0.gather_off >= 8 * 4
    regions = [torch.zeros(pl0.nbytes, dtype=torch.uint8) for _ in range(gs)]

    def bf16_at(reg, off, n):
        return reg[off:off + 2 * n].view(torch.bfloat16)

    for r, pl in enumerate(plans):  # attention epilogue of rank r
        o_r = o_full[:, r * width:(r + 1) * width]
        for j in range(gs):
            blk = o_r[j * pl.rows:(j + 1) * pl.rows].contiguous().view(-1)
            bf16_at(regions[j], pl.attn_dst_off, blk.numel()).copy_(blk)
    for r, pl in enumerate(plans):  # o_proj of rank r, scattered to every region
        gathered = bf16_at(regions[r], pl.gather_off, gs * pl.rows * width).view(gs, pl.rows, width)
        rows = sum(gathered[j].float() @ wo[:, j * width:(j + 1) * width].float().t() for j in range(gs))
        for j in range(gs):
            out_j = bf16_at(regions[j], pl.out_off, T * D).view(T, D)
            out_j[pl.gemm_row0:pl.gemm_row0 + pl.rows] = rows.bfloat16()
    ref = (o_full.float() @ wo.float().t()).bfloat16()
    for j in range(gs):
        out_j = bf16_at(regions[j], pl0.out_off, T * D).view(T, D)
        assert ((out_j.float() - ref.float()).abs().max() / ref.float().abs().max()).item() < 1e-2
        assert bool((regions[j][:pl0.gather_off] == 0).all())  # flags area untouched by data


def test_peer_exchange_plan_rejects_ragged_rows():
    from mka_b200.peer import exchange_plan

    with pytest.raises(ValueError):
        exchange_plan(4, 0, 102, 64, 128)


class _FakePeerLib:
    """Stands in for the library's fmka_peer_* calls: allocations are fake
    addresses, a handle carries (rank, address), an import maps it to a
    distinct address; every call is recorded."""

    def __init__(self, rank):
        self.rank = rank
        self.calls = []

    def call(self, name, *args):
        import ctypes

        self.calls.append(name)
        if name == "fmka_peer_alloc":
            args[1]._obj.value = 0x100000 * (self.rank + 1)
        elif name == "fmka_peer_export":
            args[1][:16] = (int(self.rank).to_bytes(8, "little") + int(args[0]).to_bytes(8, "little"))
        elif name == "fmka_peer_import":
            raw = bytes(args[0])
            owner, addr = int.from_bytes(raw[:8], "little"), int.from_bytes(raw[8:16], "little")
            args[1]._obj.value = 0x7000000 + 0x1000 * self.rank + addr + owner
        elif name == "fmka_peer_barrier":
            arr, idx, n, epoch = args[0], args[1], args[2], args[3]
            self.calls[-1] = (name, [arr[i] for i in range(n)], idx, n, epoch)


def _region_worker(rank, world, port, q):
    import torch.distributed as dist

    from mka_b200 import peer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fake = _FakePeerLib(rank)
        peer._lib = fake  # this process only
        reg = peer.PeerRegion(dist.group.WORLD, rank, world, 4096, torch.device("cpu"))
        reg.barrier(0)
        reg.barrier(0)
        ptrs = list(reg.ptrs)
        reg.close()
        q.put((rank, ptrs, fake.calls))
    finally:
        dist.destroy_process_group()


def test_gloo_peer_region_maps_every_rank_once():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 2
    port = 29600 + os.getpid() % 300
    procs = [ctx.Process(target=_region_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=60) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ptrs, calls in res:
        own = 0x100000 * (rank + 1)
        other = 1 - rank
        assert ptrs[rank] == own
        assert ptrs[other] == 0x7000000 + 0x1000 * rank + 0x100000 * (other + 1) + other
        barriers = [c for c in calls if isinstance(c, tuple)]
        assert [b[4] for b in barriers] == [1, 2]  # epochs grow by one from 1
        assert all(b[1] == ptrs and b[2] == rank and b[3] == world for b in barriers)
        names = [c if isinstance(c, str) else c[0] for c in calls]
        assert names.index("fmka_peer_close") < names.index("fmka_peer_free")
        assert names.count("fmka_peer_import") == 1 and names.count("fmka_peer_close") == 1
