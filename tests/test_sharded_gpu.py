"""Head-sharded FastMKA layer on 2 GPUs: every rank's output for its sequences
matches the unsharded layer run on the same sequences, with the exchange done
by NCCL or by the kernels' own stores into peer memory (three forwards in a
row for the latter, so that the barriers and the reused buffers are exercised).
Skipped with fewer than 2 GPUs."""
import math
import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, batch, transport, heads, q):
    import torch.distributed as dist
    import torch.nn as nn

    from mka_b200 import ops
    from mka_b200.layers.forward import fastmka_forward
    from mka_b200.sharded import HeadShardedFastMKA, make_groups

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    try:
        from tests.test_parity_gpu import _hf_like_layer

        # the router is folded through q_proj, so d_model = query heads x 128
        layer = _hf_like_layer(seed=3, D=heads[0] * 128, H=heads[0], HKV=heads[1])
        D, T = heads[0] * 128, 640
        g = torch.Generator(device="cuda").manual_seed(17)
        x_all = (torch.randn(batch, T, D, generator=g, device="cuda") / math.sqrt(D)).bfloat16()
        pos = torch.arange(T, device="cuda").float()
        inv = 1.0 / (10000 ** (torch.arange(0, 128, 2, device="cuda").float() / 128))
        ang = torch.cat([pos[:, None] * inv, pos[:, None] * inv], -1)
        rope = (ang.cos()[None], ang.sin()[None])
        groups = make_groups(batch, layer.num_key_value_heads, world)
        sh = HeadShardedFastMKA(layer, batch, rank, world, groups, transport=transport)
        b0, b1 = sh.plan.batch
        xs = x_all[b0:b1].contiguous()
        ref = fastmka_forward(xs, layer.prepared(torch.device("cuda")), layer.num_heads,
                              layer.num_key_value_heads, layer.ema_beta, False, rope=rope)["out"]
        errs = []
        for i in range(3):
            # a different input each time, so that a stale buffer would show
            xi = xs if i != 1 else (xs * 0.5).contiguous()
            out = sh(xi, rope=rope).clone()
            torch.cuda.synchronize()
            r = ref if i != 1 else fastmka_forward(xi, layer.prepared(torch.device("cuda")), layer.num_heads,
                                                    layer.num_key_value_heads, layer.ema_beta, False,
                                                    rope=rope)["out"]
            errs.append(((out.float() - r.float()).abs().max() / r.float().abs().max()).item())
        sh.close()
        q.put((rank, max(errs), len(sh.plan.group), ops.device_status()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,batch,transport,heads", [(2, 1, "peer", (4, 2)), (2, 1, "nccl", (4, 2)),
                                                        (2, 2, "peer", (4, 2)), (4, 1, "peer", (8, 4)),
                                                        (4, 2, "peer", (4, 2))])
def test_head_sharded_layer_matches_unsharded(world, batch, transport, heads):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29100 + 8 * world + 2 * batch + (transport == "peer") + os.getpid() % 500
    procs = [ctx.Process(target=_worker, args=(r, world, port, batch, transport, heads, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, gsize, status in res:
        assert status == 0
        assert gsize == max(world // batch, 1)
        assert err < 2e-2
