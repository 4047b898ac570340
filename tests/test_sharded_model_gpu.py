"""The Llama-architecture model with every self_attn patched to FastMKA, run
over 2 and 4 GPUs by sequence and kv head (mka_b200.hf.sharded_llama), against
the same model run whole on one GPU (the reference's usage: the patched
transformers model, mka/hf/patch.py:30-48): each rank's rows of the final
hidden states and the last position's logits. Three levels with a per-position
L3 memory. Skipped with fewer GPUs than ranks."""
import datetime
import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _worker(rank, world, port, heads, q):
    import torch.distributed as dist
    from transformers import LlamaConfig, LlamaForCausalLM

    from mka_b200 import ops
    from mka_b200.hf.patch import HFPatchConfig, apply_hf_attention_patch
    from mka_b200.hf.sharded_llama import SequenceHeadShardedLlama

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        H, HKV = heads
        D, T = H * 128, 512
        cfg = LlamaConfig(vocab_size=256, hidden_size=D, intermediate_size=2 * D, num_hidden_layers=2,
                          num_attention_heads=H, num_key_value_heads=HKV, max_position_embeddings=4096,
                          rope_theta=500000.0, attn_implementation="sdpa")
        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            with torch.device(dev):
                torch.manual_seed(5)
                model = LlamaForCausalLM(cfg).eval()
                apply_hf_attention_patch(model, HFPatchConfig(use_l3=True, verbose=False))
        finally:
            torch.set_default_dtype(prev)
        g = torch.Generator(device=dev).manual_seed(6)
        ids = torch.randint(0, 256, (1, T), generator=g, device=dev)
        l3 = (torch.randn(1, T, D, generator=g, device=dev) * 0.5).bfloat16()
        with torch.no_grad():
            ref_h = model.model(ids, use_cache=False, l3_memory=l3).last_hidden_state
            ref_logits = model(ids, use_cache=False, logits_to_keep=1, l3_memory=l3).logits
        sh = SequenceHeadShardedLlama(model, rank, world)
        errs = []
        for _ in range(2):  # twice: the gather areas and barrier epochs are reused
            logits, hid = sh(ids, l3_memory=l3, return_hidden=True)
            torch.cuda.synchronize()
            rows = T // world
            r = ref_h[:, rank * rows:(rank + 1) * rows].float()
            errs.append(((hid.float() - r).abs().max() / r.abs().max()).item())
            if logits is not None:
                errs.append(((logits.float() - ref_logits.float()).abs().max() / ref_logits.float().abs().max()).item())
        sh.close()
        q.put((rank, max(errs), ops.device_status()))
    except Exception:
        import traceback

        q.put((rank, "error", traceback.format_exc()))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,heads", [(2, (4, 2)), (4, (8, 4))])
def test_sequence_head_sharded_llama_matches_one_gpu(world, heads):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29300 + 10 * world + os.getpid() % 500
    procs = [ctx.Process(target=_worker, args=(r, world, port, heads, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = [q.get(timeout=300) for _ in range(world)]
        errors = [r for r in res if r[1] == "error"]
        assert not errors, errors[0][2]
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    finally:
        for p in procs:  # a rank that failed must not keep its GPU for the next test
            if p.is_alive():
                p.kill()
                p.join(timeout=30)
    for rank, err, status in res:
        assert status == 0
        assert err < TOL, (rank, err)
