"""FastMKA attention-layer benchmark on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (one step = one forward of a FastMKA attention layer):
  prefill  Qwen-7B-like layer: batch 4 per GPU, seq 8192, d_model 3584, 28 query /
           4 kv heads (GQA), head_dim 128, q/k/v bias, RoPE (theta 1e6), L1+L2
           routing (EMA decay 0.9), router 3584 -> 512 -> 2 (SiLU), bf16,
           X ~ N(0,1)/sqrt(3584), weights N(0, 0.02), seeded
Also reported in the same line:
  decode   Llama-3-8B-like layer: batch 64, one new token per sequence against a
           32768-long cached fused K/V (in-place cache), d_model 4096, 32/8 heads,
           router 4096 -> 2048 -> 2, cache ~ N(0,1)*0.1, X ~ N(0,1)

value   = prefill tokens/s of the whole job (all ranks), inputs resident in HBM
e2e     = the same through the module API with the input copied from pinned host
          memory and the layer output copied back, every step
roofline: the attention kernel (tensor-bound, algorithmic FLOPs 4*B*Hq*Dh*T(T+1)/2)
          timed with CUDA events inside the timed steps against the measured
          burst bf16 peak (a ~2 ms kernel inside a ms-scale step, not a
          seconds-long loop); decode: the split-KV kernel's K/V bytes against the
          measured HBM copy bandwidth. Kernel times also appear in SM cycles
          (ms x the median SM clock sampled during the run)
Multi-GPU (torchrun): weak scaling by batch: every rank runs its own 4 sequences
(units = (sequence, kv head) pairs, whole sequences per rank), no collective in
the data path; the step time is the max over ranks.
--impl reference: the reference's CPU algorithm (the CPU oracle restating
FastLM/MKA's FastMKA forward op for op) on the host cores, one whole 8192-token
sequence of the prefill configuration per step (tokens/s of a sequence does not
depend on the batch on the CPU, which runs the sequences one after another).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch
import torch.nn as nn

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PREFILL = dict(B=4, T=8192, D=3584, H=28, HKV=4, R=512, L=2, theta=1.0e6, bias=True)
DECODE = dict(B=64, TK=32768, D=4096, H=32, HKV=8, R=2048, L=2, theta=5.0e5, bias=False)
LONG = dict(B=2, T=32768, D=3584, H=28, HKV=4, R=512, L=3, theta=1.0e6, bias=True)
CPU_SEQ_T = PREFILL["T"]  # the CPU arms run one whole prefill sequence per step


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return {"hbm": float(m["hbm_gbs"]), "bf16": float(m["bf16_tflops"]),
                "bf16_sust": float(m["bf16_tflops_sustained"]), "src": "measured"}
    except Exception:
        return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sust": 1400.0, "src": "fallback"}


class _Rotary:
    """Stands in for an HF rotary module: makes the wrapper apply RoPE."""

    def __init__(self, theta):
        self.theta = theta

    def cos_sin(self, positions, device):
        inv = 1.0 / (self.theta ** (torch.arange(0, 128, 2, device=device, dtype=torch.float32) / 128))
        ang = positions.to(torch.float32)[:, None] * inv[None]
        ang = torch.cat([ang, ang], -1)
        return ang.cos()[None], ang.sin()[None]  # [1, T, 128]


class _AttnHolder(nn.Module):
    """A Qwen2/Llama-style attention module (q/k/v/o_proj) to wrap."""

    def __init__(self, d, h, hkv, bias, theta):
        super().__init__()
        self.hidden_size, self.num_heads, self.num_key_value_heads = d, h, hkv
        self.q_proj = nn.Linear(d, h * 128, bias=bias)
        self.k_proj = nn.Linear(d, hkv * 128, bias=bias)
        self.v_proj = nn.Linear(d, hkv * 128, bias=bias)
        self.o_proj = nn.Linear(h * 128, d, bias=False)
        self.rotary_emb = _Rotary(theta)


def build_layer(cfg, device, seed=0):
    from mka_b200 import HFFastMKAAttention

    torch.manual_seed(seed)
    holder = _AttnHolder(cfg["D"], cfg["H"], cfg["HKV"], cfg["bias"], cfg["theta"])
    layer = HFFastMKAAttention(holder, use_l3=cfg["L"] == 3, ema_beta=0.9)
    layer.router = nn.Sequential(nn.Linear(cfg["D"], cfg["R"]), nn.SiLU(), nn.Linear(cfg["R"], cfg["L"]))
    g = torch.Generator(device=device).manual_seed(seed)
    layer = layer.to(device=device, dtype=torch.bfloat16)
    with torch.no_grad():
        for m in layer.modules():
            if isinstance(m, nn.Linear):
                m.weight.copy_(torch.randn(m.weight.shape, generator=g, device=device) * 0.02)
                if m.bias is not None:
                    m.bias.copy_(torch.randn(m.bias.shape, generator=g, device=device) * 0.02)
    return layer.eval()


class ClockSampler:
    """nvidia-smi SM clocks and throttle reasons sampled during a timed region."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, device_index):
        self.idx = device_index
        self.proc = None
        out_dir = os.environ.get("FMKA_BENCH_CLOCKS_DIR") or tempfile.gettempdir()
        self.path = os.path.join(out_dir, f"fmka_clocks_rank{device_index}_{os.getpid()}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        loaded = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1:
        import datetime

        import torch.distributed as dist

        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
        return dist, dist.get_rank(), ws, local
    return None, 0, 1, 0


def _barrier(dist):
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


def _max_over_ranks(dist, v):
    if dist is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _timed(dist, fn, steps):
    _barrier(dist)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    _barrier(dist)
    return _max_over_ranks(dist, a.elapsed_time(b) / steps)


def _stage_times(fn, steps):
    """Average duration (ms) of each forward stage over `steps` instrumented calls.

    A spin kernel queued ahead of each call (outside every measured interval)
    lets the host enqueue the whole forward before the GPU reaches it, so the
    stages run back to back and each event pair times the device, not a wait
    for the host's next launch."""
    acc = {}
    for _ in range(steps):
        timers = []
        torch.cuda._sleep(int(5e7))
        fn(timers)
        torch.cuda.synchronize()
        for name, s, e in timers:
            acc.setdefault(name, []).append(s.elapsed_time(e))
    return {k: sum(v) / len(v) for k, v in acc.items()}


def _attention_beside_sdpa(r, flops, reps=5):
    """This package's attention kernel and torch's SDPA (the reference's default
    prefill path, mka/layers/fastmka.py:134,157) on the layer's own q/k/v, each
    timed over `reps` launches queued behind a spin kernel."""
    from mka_b200 import ops

    q, k, v = r["q"], r["k"], r["v"]
    runs = {"attn_prefill": lambda: ops.attn_prefill(q, k, v, want_lse=False),
            "sdpa": lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True,
                                                                              enable_gqa=True)}
    out = {}
    for name, fn in runs.items():
        fn()
        torch.cuda.synchronize()
        torch.cuda._sleep(int(2e8))
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(e) / reps
        out[name] = {"ms": round(ms, 4), "tflops": round(flops / (ms * 1e-3) / 1e12, 1)}
    return out


def _traffic(name):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary (profiles/)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(name)
    except Exception:
        return None


def _e2e_pipelined(dist, layer, x, pe, steps):
    """Average ms per step of host->device input, forward, device->host output.

    Each step's sequences are pipelined as separate units through the public
    layer call: the upload of unit u+1 and the download of unit u-1 overlap the
    forward of unit u on three streams, so only one sequence's upload and one
    sequence's download are not hidden. Device-timed on the compute stream,
    which waits for the last download before the end event."""
    comp = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    B = x.shape[0]
    g = torch.Generator().manual_seed(7)
    x_host = [x.cpu().pin_memory(), (x.cpu() + 0.01 * torch.randn(x.shape, generator=g).to(x.dtype)).pin_memory()]
    out_host = [torch.empty(x.shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    nbuf = 3
    x_dev = [torch.empty_like(x[:1]) for _ in range(nbuf)]
    ev_up = [torch.cuda.Event() for _ in range(nbuf)]
    ev_comp = [torch.cuda.Event() for _ in range(nbuf)]

    def unit_src(u):
        return x_host[(u // B) % 2][u % B: u % B + 1]

    def run(n_steps):
        n = n_steps * B
        with torch.cuda.stream(up):
            x_dev[0].copy_(unit_src(0), non_blocking=True)
            ev_up[0].record(up)
        last_down = torch.cuda.Event()
        for u in range(n):
            bu = u % nbuf
            if u + 1 < n:
                nb = (u + 1) % nbuf
                with torch.cuda.stream(up):
                    if u + 1 >= nbuf:
                        up.wait_event(ev_comp[nb])  # the unit that last used this buffer has been read
                    x_dev[nb].copy_(unit_src(u + 1), non_blocking=True)
                    ev_up[nb].record(up)
            comp.wait_event(ev_up[bu])
            out, _, _ = layer(x_dev[bu], position_embeddings=pe)
            ev_comp[bu].record(comp)
            with torch.cuda.stream(down):
                down.wait_event(ev_comp[bu])
                out_host[(u // B) % 2][u % B: u % B + 1].copy_(out, non_blocking=True)
                out.record_stream(down)
                last_down.record(down)
        comp.wait_event(last_down)

    run(2)
    _barrier(dist)
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(comp)
    run(steps)
    e.record(comp)
    _barrier(dist)
    return _max_over_ranks(dist, a.elapsed_time(e) / steps)


# ------------------------------------------------------------------ prefill --
def bench_prefill(args, dist, rank, world, device, peaks):
    from mka_b200.layers.forward import fastmka_forward

    c = PREFILL
    B, T, D = c["B"], c["T"], c["D"]
    layer = build_layer(c, device)
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    x = (torch.randn(B, T, D, generator=g, device=device) / math.sqrt(D)).to(torch.bfloat16)
    cos, sin = layer.rotary_emb.cos_sin(torch.arange(T, device=device), device)
    pe = (cos, sin)

    def step():
        layer(x, position_embeddings=pe)

    for _ in range(args.warmup):
        step()
    ms = _timed(dist, step, args.steps)

    # per-kernel times inside the same kind of step (instrumented)
    W = layer.prepared(device)
    st = _stage_times(lambda timers: fastmka_forward(x, W, c["H"], c["HKV"], 0.9, False, rope=pe, timers=timers),
                      max(3, min(args.steps, 10)))
    attn_ms = st.get("attention", float("nan"))
    flops = 4.0 * B * c["H"] * 128 * T * (T + 1) / 2
    achieved = flops / (attn_ms * 1e-3) / 1e12
    sdpa = _attention_beside_sdpa(fastmka_forward(x, W, c["H"], c["HKV"], 0.9, False, rope=pe), flops)

    # end to end through the module with host buffers: every step uploads its
    # input from pinned host memory and downloads the layer output, pipelined
    # per sequence on three streams (the upload of the next sequence and the
    # download of the previous one overlap the forward of the current one)
    e2e_ms = _e2e_pipelined(dist, layer, x, pe, args.steps)
    tokens = B * T * world
    return {
        "ms": ms, "tok_s": tokens / (ms * 1e-3), "e2e_tok_s": tokens / (e2e_ms * 1e-3), "e2e_ms": e2e_ms,
        "h2d": x.numel() * 2, "d2h": x.numel() * 2, "stages_ms": st,
        "attention_beside_sdpa": sdpa,
        "roofline": {"bound": "tensor", "kernel": "attn_prefill", "achieved": round(achieved, 1),
                     "peak": peaks["bf16"], "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16"], 4),
                     "peak_kind": f"{peaks['src']} burst bf16 (a ~2 ms kernel inside a ms-scale step)",
                     "algorithmic_tflop_per_launch": flops / 1e12, "launch_ms": attn_ms,
                     "traffic": _traffic("attn_prefill")},
        "layer": layer, "x": x, "pe": pe,
    }


# ------------------------------------------------------------------- decode --
def bench_decode(args, dist, rank, world, device, peaks):
    from mka_b200 import StaticKVCache
    from mka_b200.layers.forward import fastmka_forward

    c = DECODE
    B, TK, D = c["B"], c["TK"], c["D"]
    layer = build_layer(c, device, seed=1)
    cap = TK + 8
    cache = StaticKVCache(B, c["HKV"], cap, 1, device=device)
    g = torch.Generator(device=device).manual_seed(2000 + rank)
    for t in (cache.k[0], cache.v[0]):
        t.normal_(0.0, 0.1, generator=g)
    cache._index(layer)
    x = torch.randn(B, 1, D, generator=g, device=device).to(torch.bfloat16)
    cos, sin = layer.rotary_emb.cos_sin(torch.tensor([TK], device=device), device)
    pe = (cos, sin)

    def step():
        cache.lengths[0] = TK
        layer(x, position_embeddings=pe, past_key_value=cache)

    for _ in range(args.warmup):
        step()
    ms = _timed(dist, step, args.steps)
    W = layer.prepared(device)
    kc, vc = cache.k[0], cache.v[0]
    st = _stage_times(lambda timers: fastmka_forward(x, W, c["H"], c["HKV"], 0.9, False, rope=pe, kv_out=(kc, vc),
                                                     past_len=TK, timers=timers), max(3, min(args.steps, 10)))
    attn_ms = st.get("attention", float("nan"))
    kv_bytes = 2.0 * B * c["HKV"] * (TK + 1) * 128 * 2
    achieved = kv_bytes / (attn_ms * 1e-3) / 1e9
    return {
        "ms": ms, "tok_s": B * world / (ms * 1e-3), "stages_ms": st,
        "roofline": {"bound": "hbm", "kernel": "attn_decode", "achieved": round(achieved, 1), "peak": peaks["hbm"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm"], 4), "peak_kind": f"{peaks['src']} HBM copy",
                     "algorithmic_gb_per_launch": kv_bytes / 1e9, "launch_ms": attn_ms,
                     "traffic": _traffic("attn_decode")},
    }


# ------------------------------------------------------------ long context --
def bench_long_context(args, dist, rank, world, device, peaks):
    """The Qwen-7B-like layer with L3 retrieved memory at batch 2, seq 32768 (fixed
    total work): whole sequences per rank up to 2 GPUs, then kv heads split inside
    each sequence's group; the group exchanges attention rows and o_proj rows by
    the kernels' own stores into peer memory (`--exchange nccl`: an NCCL
    all-gather before a replicated o_proj)."""
    from mka_b200.sharded import HeadShardedFastMKA, make_groups

    c = LONG
    B, T, D = c["B"], c["T"], c["D"]
    layer = build_layer(c, device, seed=2)
    groups = make_groups(B, c["HKV"], world) if dist is not None else {}
    # the step stays asynchronous; the status word (peer timeouts included) is read once after the
    # timed steps and reported as device_status
    sh = HeadShardedFastMKA(layer, B, rank, world, groups, transport=args.exchange, check_peer_status=False)
    b0, b1 = sh.plan.batch
    g = torch.Generator(device=device).manual_seed(3000)
    x = (torch.randn(B, T, D, generator=g, device=device) / math.sqrt(D)).to(torch.bfloat16)[b0:b1].contiguous()
    r = (torch.randn(B, T, D, generator=g, device=device) * 0.5).to(torch.bfloat16)[b0:b1].contiguous()
    cos, sin = layer.rotary_emb.cos_sin(torch.arange(T, device=device), device)
    pe = (cos, sin)

    def step():
        sh(x, rope=pe, l3_memory=r)

    for _ in range(max(2, args.warmup)):
        step()
    steps = max(3, min(args.steps, 10))
    ms = _timed(dist, step, steps)
    from mka_b200 import ops

    xk = None
    if sh._region is not None:
        # the fused o_proj + all-gather kernel alone, on every rank at once:
        # this rank's rows of o_proj, stored into every rank's output
        from mka_b200.peer import bf16_view, exchange_plan

        gs = len(sh.plan.group)
        W = sh._weights(device)
        K = W.w_o.shape[1]
        pl = exchange_plan(gs, sh._region.index, T, D, K // gs)
        gathered = bf16_view(sh._region.local + pl.gather_off, (gs, pl.rows, K // gs), device)
        dsts = [p + pl.out_off for p in sh._region.ptrs]

        def xstep():
            ops.gemm_kblocked_scatter(gathered, W.w_o, W.b_o, dsts, pl.gemm_row0, D)

        xstep()
        xms = _timed(dist, xstep, steps)
        xflops = 2.0 * pl.rows * D * K
        xbytes = (gs - 1) * pl.rows * D * 2
        target = max(xflops / (peaks["bf16"] * 1e12), xbytes / 770e9) * 1e3
        xk = {"kernel": "gemm_pair_kernel<scatter>: this rank's o_proj rows stored into every rank's output",
              "ms": xms, "rows": pl.rows, "flops": xflops, "nvlink_bytes_out": xbytes,
              "target_ms": round(target, 4), "frac": round(target / xms, 4),
              "target_basis": "max(FLOPs / measured bf16 burst, bytes out over NVLink / 770 GB/s measured "
                              "peer copy)"}
    # this rank's attention kernel alone: its query heads over its sequences

    h0, h1 = sh.plan.kv_heads
    hq = (h1 - h0) * (c["H"] // c["HKV"])
    q = torch.randn(b1 - b0, hq, T, 128, generator=g, device=device, dtype=torch.bfloat16)
    k = torch.randn(b1 - b0, h1 - h0, T, 128, generator=g, device=device, dtype=torch.bfloat16)
    v = torch.randn_like(k)
    for _ in range(2):
        ops.attn_prefill(q, k, v, want_lse=False)
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        ops.attn_prefill(q, k, v, want_lse=False)
    e.record()
    torch.cuda.synchronize()
    attn_ms = a.elapsed_time(e) / steps
    flops = 4.0 * (b1 - b0) * hq * 128 * T * (T + 1) / 2
    achieved = flops / (attn_ms * 1e-3) / 1e12
    gsz = len(sh.plan.group)
    sh.close()
    del q, k, v
    recall = _l3_recall_line(x, steps, peaks, device, g)
    exchange = ("none" if gsz == 1 else "peer stores from the attention and o_proj epilogues"
                if args.exchange == "peer" else "NCCL all-gather, o_proj on every rank")
    return {"metric": "FastMKA prefill tokens/s, long context with L3 (fixed total work)",
            "value": B * T / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms, "scaling": "strong",
            "config": {"batch": B, "seq_len": T, "d_model": D, "heads": f"{c['H']}/{c['HKV']}", "levels": 3,
                       "router": f"{D}->{c['R']}->3", "partition": f"sequences x kv heads, group size "
                                                                  f"{gsz}", "exchange": exchange},
            "exchange_kernel": xk, "l3_recall": recall,
            "roofline": {"bound": "tensor", "kernel": "attn_prefill (this rank's heads, T=32768)",
                         "achieved": round(achieved, 1), "peak": peaks["bf16"], "unit": "TFLOP/s",
                         "frac": round(achieved / peaks["bf16"], 4), "peak_kind": f"{peaks['src']} burst bf16",
                         "launch_ms": attn_ms}}


def _l3_recall_line(x, steps, peaks, device, g, n_chunks=8192, top_r=8, block_len=64):
    """The L3 chunk recall that produces R (mka_b200.l3) for this rank's sequences:
    a bank of n_chunks seeded N(0, 0.5) chunk keys and values (standing in for the
    chunk means of an earlier 512k-token context), the top-8 chunks of every
    64-token block. Timed on its own: the layer step above takes its R as given,
    as the reference's layers do."""
    from mka_b200.l3 import L3ChunkStore

    Bl, T, D = x.shape
    keys = (torch.randn(n_chunks, D, generator=g, device=device) * 0.5).to(torch.bfloat16)
    vals = (torch.randn(n_chunks, D, generator=g, device=device) * 0.5).to(torch.bfloat16)
    store = L3ChunkStore(keys, vals)
    for _ in range(2):
        store.recall(x, top_r, block_len)
    torch.cuda.synchronize()
    torch.cuda._sleep(int(2e8))
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        store.recall(x, top_r, block_len)
    e.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(e) / steps
    hbm = 2 * Bl * T * D * 2  # x read for the block means + R written
    return {"ms": ms, "bank_chunks": n_chunks, "top_r": top_r, "block_len": block_len, "rows": Bl * T,
            "hbm_bytes": hbm, "achieved_gbs": round(hbm / (ms * 1e-3) / 1e9, 1),
            "frac_of_hbm": round(hbm / (ms * 1e-3) / 1e9 / peaks["hbm"], 4),
            "kernels": "block means, scores GEMM (fp32 out), top-R, weighted gather"}


# -------------------------------------------------------------- CPU (oracle) --
def _oracle_params(layer):
    f = lambda t: None if t is None else t.detach().float().cpu()  # noqa: E731
    return {"wq": f(layer.q_proj.weight), "bq": f(layer.q_proj.bias), "wk": f(layer.k_proj.weight),
            "bk": f(layer.k_proj.bias), "wv": f(layer.v_proj.weight), "bv": f(layer.v_proj.bias),
            "wo": f(layer.o_proj.weight), "r1w": f(layer.router[0].weight), "r1b": f(layer.router[0].bias),
            "r2w": f(layer.router[2].weight), "r2b": f(layer.router[2].bias)}


def cpu_reference_step(p, x_cpu, cos, sin):
    """One forward of the reference algorithm on the CPU (out, k/v, gate; the
    reference computes no log-sum-exp, so neither does the timed step)."""
    from oracle import fastmka_oracle as orc

    with torch.no_grad():
        orc.hf_fastmka_forward(x_cpu, p, PREFILL["H"], PREFILL["HKV"], False, 0.9, "silu", cos=cos, sin=sin,
                               with_lse=False)


def cpu_sample_inputs(seed=0, t=None):
    """One whole prefill sequence on the CPU: x [1, T, D] fp32 (T = CPU_SEQ_T by
    default) and its RoPE tables."""
    c = PREFILL
    t = t or CPU_SEQ_T
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(1, t, c["D"], generator=g) / math.sqrt(c["D"])
    rot = _Rotary(c["theta"])
    cos, sin = rot.cos_sin(torch.arange(t), "cpu")
    return x, cos[:, None], sin[:, None]


def cpu_params_random(seed=0):
    c = PREFILL
    g = torch.Generator().manual_seed(seed)
    D, H, HKV, R = c["D"], c["H"], c["HKV"], c["R"]
    r = lambda *s: torch.randn(*s, generator=g) * 0.02  # noqa: E731
    return {"wq": r(H * 128, D), "bq": r(H * 128), "wk": r(HKV * 128, D), "bk": r(HKV * 128), "wv": r(HKV * 128, D),
            "bv": r(HKV * 128), "wo": r(D, H * 128), "r1w": r(R, D), "r1b": r(R), "r2w": r(2, R), "r2b": r(2)}


def measure_cpu(p, steps=1, warmup=1):
    torch.set_num_threads(os.cpu_count() or 1)
    x, cos, sin = cpu_sample_inputs()
    for _ in range(warmup):
        cpu_reference_step(p, x, cos, sin)
    t0 = time.perf_counter()
    for _ in range(steps):
        cpu_reference_step(p, x, cos, sin)
    dt = (time.perf_counter() - t0) / steps
    return {"value": CPU_SEQ_T / dt, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"reference FastMKA forward (CPU oracle, fp32) on one whole sequence of the prefill "
                      f"config (batch 1, seq {CPU_SEQ_T}); {dt:.2f} s per sequence after {warmup} warm-up"}


def run_reference(args):
    dist, rank, world, _ = (None, int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), 0)
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    p = cpu_params_random()
    x, cos, sin = cpu_sample_inputs()
    for _ in range(args.warmup):
        cpu_reference_step(p, x, cos, sin)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_reference_step(p, x, cos, sin)
    dt = (time.perf_counter() - t0) / args.steps
    v = CPU_SEQ_T / dt
    cores = torch.get_num_threads()
    sample = (f"reference FastMKA forward (CPU oracle restating FastLM/MKA op for op, fp32, {cores} threads) on "
              f"one whole sequence per step: batch 1, seq {CPU_SEQ_T} of the prefill config")
    line = {"metric": "FastMKA prefill tokens/s (Qwen-7B-like layer, B200)", "value": v, "unit": "tokens/s",
            "impl": "reference", "n_gpus": 0, "host_threads": cores, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": _ref_config(cores),
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_kernel_only(args):
    """`--only KERNEL`: launches one kernel of the layer alone (warmup + steps
    launches) on synthetic inputs of the configured shapes, with the batch
    overridable by --batch: the small-case command for ncu captures."""
    from mka_b200 import ops

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    c, d = PREFILL, DECODE
    n = args.warmup + args.steps
    if args.only in ("attn_prefill", "route_ema_blend", "route_ema_blend_h", "qr_proj", "kv_gemm", "kv_proj",
                     "o_proj"):
        B = args.batch or c["B"]
        T, D = args.seq or c["T"], c["D"]
        if args.only == "attn_prefill":
            q = torch.randn(B, c["H"], T, 128, generator=g, device=dev, dtype=torch.bfloat16)
            k = torch.randn(B, c["HKV"], T, 128, generator=g, device=dev, dtype=torch.bfloat16)
            v = torch.randn(B, c["HKV"], T, 128, generator=g, device=dev, dtype=torch.bfloat16)
            fn = lambda: ops.attn_prefill(q, k, v)  # noqa: E731
        elif args.only == "route_ema_blend_h":  # the blend-first stage 1 over d_model (op API)
            x = torch.randn(B, T, D, generator=g, device=dev, dtype=torch.bfloat16)
            lg = torch.randn(B * T, c["L"], generator=g, device=dev)
            fn = lambda: ops.route_ema_blend(x, 0.9, logits=lg, b2=None, levels=c["L"])  # noqa: E731
        else:
            layer = build_layer(c, dev)
            W = layer.prepared(dev)
            x = (torch.randn(B * T, D, generator=g, device=dev) / math.sqrt(D)).to(torch.bfloat16)
            cos, sin = layer.rotary_emb.cos_sin(torch.arange(T, device=dev), dev)
            if args.only == "route_ema_blend":  # the layer's stage 1: on y = x [Wk ; Wv]^T, K/V out
                y = (torch.randn(B * T, 2 * c["HKV"] * 128, generator=g, device=dev) * 0.05).to(torch.bfloat16)
                lg = torch.randn(B * T, c["L"], generator=g, device=dev)
                fn = lambda: ops.route_ema_blend_kv(y, 0.9, lg, W.b2, B, T, c["HKV"], bias=W.b_kv,  # noqa: E731
                                                    rope=(cos, sin))
            elif args.only == "kv_gemm":  # the layer's K/V GEMM: y = x [Wk ; Wv]^T
                fn = lambda: ops.gemm(x, W.w_kv)  # noqa: E731
            elif args.only == "qr_proj":
                fn = lambda: ops.qr_proj(x, W.w_qr, W.b_qr, B, T, c["H"], W.router_hidden, W.w2, c["L"], W.act,  # noqa
                                         rope=(cos, sin))
            elif args.only == "kv_proj":  # the blend-first K/V projection (op API)
                fn = lambda: ops.kv_proj(x, W.w_kv, W.b_kv, B, T, c["HKV"], rope=(cos, sin))  # noqa: E731
            else:
                fn = lambda: ops.gemm(x, W.w_o, W.b_o)  # noqa: E731
    elif args.only in ("o_proj_scatter", "o_proj_blocked"):
        # o_proj of one rank of a head-sharded group of G ranks (--batch G, default 4) at
        # the long-context size: T/G rows of the gathered attention output [G, T/G, Hq*128/G].
        # o_proj_scatter writes every row into G local buffers standing in for the group's
        # output areas; o_proj_blocked is the plain blocked GEMM on the same operands.
        G = args.batch or 4
        cl = LONG
        rows, width = cl["T"] // G, cl["H"] * 128 // G
        a = torch.randn(G, rows, width, generator=g, device=dev).to(torch.bfloat16)
        w = (torch.randn(cl["D"], G * width, generator=g, device=dev) / 60).to(torch.bfloat16)
        if args.only == "o_proj_scatter":
            outs = [torch.empty(cl["T"], cl["D"], device=dev, dtype=torch.bfloat16) for _ in range(G)]
            ptrs = [o.data_ptr() for o in outs]
            fn = lambda: ops.gemm_kblocked_scatter(a, w, None, ptrs, 0, cl["D"])  # noqa: E731
        else:
            fn = lambda: ops.gemm_kblocked(a, w)  # noqa: E731
    elif args.only == "l3_recall":
        # the L3 chunk recall at the long-context size (per batch row --batch, default 2):
        # a bank of 8192 seeded chunks, the top-8 chunks of every 64-token block
        from mka_b200.l3 import L3ChunkStore

        cl = LONG
        B = args.batch or cl["B"]
        T = args.seq or cl["T"]
        x = torch.randn(B, T, cl["D"], generator=g, device=dev).mul_(0.5).to(torch.bfloat16)
        keys = torch.randn(8192, cl["D"], generator=g, device=dev).mul_(0.5).to(torch.bfloat16)
        vals = torch.randn(8192, cl["D"], generator=g, device=dev).mul_(0.5).to(torch.bfloat16)
        store = L3ChunkStore(keys, vals)
        fn = lambda: store.recall(x, top_r=8, block_len=64)  # noqa: E731
    elif args.only == "attn_decode":
        B = args.batch or d["B"]
        q = torch.randn(B, d["H"], 1, 128, generator=g, device=dev, dtype=torch.bfloat16)
        k = torch.randn(B, d["HKV"], d["TK"], 128, generator=g, device=dev, dtype=torch.bfloat16).mul_(0.1)
        v = torch.randn(B, d["HKV"], d["TK"], 128, generator=g, device=dev, dtype=torch.bfloat16).mul_(0.1)
        fn = lambda: ops.attn_decode(q, k, v)  # noqa: E731
    else:
        raise SystemExit(f"unknown kernel {args.only}")
    for _ in range(args.warmup):
        fn()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # a spin kernel ahead of the timed launches lets the host queue them all first, so the
    # events time the device, not the Python wrappers' host overhead (outside the timed region)
    torch.cuda.synchronize()
    torch.cuda._sleep(int(2e8))
    e0.record()
    for _ in range(args.steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(args.steps, 1)
    line = {"only": args.only, "launches": n, "ms_per_launch": ms, "device_status": ops.device_status()}
    if args.only == "attn_prefill":
        flops = 4.0 * B * c["H"] * 128 * T * (T + 1) / 2
        line.update(batch=B, seq=T, tflops=round(flops / (ms * 1e-3) / 1e12, 1))
        # the reference's default prefill path is torch SDPA (mka/layers/fastmka.py:134,157): the same
        # q/k/v through torch.nn.functional.scaled_dot_product_attention (causal, GQA), timed the same way
        sdpa = lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True,  # noqa: E731
                                                                         enable_gqa=True)
        for _ in range(args.warmup):
            sdpa()
        torch.cuda.synchronize()
        torch.cuda._sleep(int(2e8))
        e0.record()
        for _ in range(args.steps):
            sdpa()
        e1.record()
        torch.cuda.synchronize()
        sms = e0.elapsed_time(e1) / max(args.steps, 1)
        line.update(sdpa_ms=sms, sdpa_tflops=round(flops / (sms * 1e-3) / 1e12, 1))
    print(json.dumps(line))


def _ref_config(threads):
    """What the CPU arm runs: one whole sequence of the prefill layer per step."""
    c = PREFILL
    return {"workload": f"FastMKA attention layer prefill, Qwen-7B-like: batch 1 (one whole sequence of the "
                        f"prefill configuration per step), seq {CPU_SEQ_T}, d_model {c['D']}, {c['H']}/{c['HKV']} "
                        f"heads, head_dim 128, L1+L2, router {c['D']}->{c['R']}->2, RoPE",
            "global_batch": 1, "seq_len": CPU_SEQ_T, "parallelism": f"host CPU, {threads} threads",
            "l2": "not applicable (CPU)"}


def _config(args):
    c = PREFILL
    return {"workload": f"FastMKA attention layer prefill, Qwen-7B-like: batch {c['B']} per GPU, seq {c['T']}, "
                        f"d_model {c['D']}, {c['H']}/{c['HKV']} heads, head_dim 128, L1+L2, router "
                        f"{c['D']}->{c['R']}->2, RoPE",
            "global_batch": c["B"] * args.gpus, "seq_len": c["T"], "parallelism": f"dp{args.gpus} (batch x kv-head units, whole sequences per rank)",
            "l2": "inputs larger than L2 (X 235 MB per GPU; decode cache 8.6 GB)"}


# -------------------------------------------------------------- full model --
MODEL = dict(name="Llama-3-8B", vocab=128256, D=4096, FFN=14336, layers=32, H=32, HKV=8, theta=5e5, T=65536, B=1)


def bench_model(args, device):
    """The whole Llama-3-8B architecture from transformers (random bf16 weights,
    N(0, 0.02)) with every self_attn replaced by the FastMKA module through the
    reference's patch API with three levels (L1 + L2 + L3; the L3 memory is one
    seeded N(0, 0.5) [1, 65536, 4096] tensor passed with the model call, which
    transformers forwards to every self_attn), every MLP's SiLU product by the
    one-pass kernel (--model-mlp silu_mul; "fused" takes the SwiGLU GEMM,
    "transformers" leaves the MLP alone) and every RMSNorm by the one-pass
    kernel (--model-norm); one prefill forward of a 65536-token sequence
    per step (logits of the last position only). Also times one patched
    self_attn alone at that length, the part of each layer this package
    replaces."""
    from transformers import LlamaConfig, LlamaForCausalLM

    from mka_b200.hf.mlp import apply_mlp_fusion
    from mka_b200.hf.norm import apply_norm_fusion
    from mka_b200.hf.patch import HFPatchConfig, apply_hf_attention_patch

    c = MODEL
    cfg = LlamaConfig(vocab_size=c["vocab"], hidden_size=c["D"], intermediate_size=c["FFN"],
                      num_hidden_layers=c["layers"], num_attention_heads=c["H"], num_key_value_heads=c["HKV"],
                      max_position_embeddings=131072, rope_theta=c["theta"], attn_implementation="sdpa")
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(device):
            torch.manual_seed(5)
            model = LlamaForCausalLM(cfg).eval()
            patched = apply_hf_attention_patch(model, HFPatchConfig(use_l3=True, verbose=False))
            fused_mlp = (apply_mlp_fusion(model, mode="swiglu" if args.model_mlp == "fused" else "silu_mul")
                         if args.model_mlp != "transformers" else 0)
            fused_norms = apply_norm_fusion(model) if args.model_norm == "fused" else 0
    finally:
        torch.set_default_dtype(prev)
    g = torch.Generator(device=device).manual_seed(6)
    ids = torch.randint(0, c["vocab"], (c["B"], c["T"]), generator=g, device=device)
    l3 = (torch.randn(c["B"], c["T"], c["D"], generator=g, device=device) * 0.5).to(torch.bfloat16)

    def step():
        with torch.no_grad():
            model(ids, use_cache=False, logits_to_keep=1, l3_memory=l3)

    step()  # warm-up: first call also folds and caches each layer's weights
    steps = max(1, min(args.steps, 3))
    ms = _timed(None, step, steps)

    x = (torch.randn(c["B"], c["T"], c["D"], generator=g, device=device) * 0.5).to(torch.bfloat16)
    pos = torch.arange(c["T"], device=device).unsqueeze(0)
    pe = model.model.rotary_emb(x, pos)
    attn = model.model.layers[0].self_attn

    def attn_step():
        with torch.no_grad():
            attn(hidden_states=x, position_embeddings=pe, l3_memory=l3)

    attn_step()
    attn_ms = _timed(None, attn_step, steps)
    tokens = c["B"] * c["T"]
    attn_flops = 4.0 * c["B"] * c["H"] * 128 * c["T"] * (c["T"] + 1) / 2
    out = {
        "metric": "Llama-3-8B prefill tokens/s, every self_attn patched with FastMKA (transformers model)",
        "value": tokens / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
        "patched_layers": patched, "fused_mlp_layers": fused_mlp, "fused_norms": fused_norms,
        "fastmka_self_attn_ms_per_layer": attn_ms,
        "fastmka_self_attn_share": round(attn_ms * c["layers"] / ms, 4),
        "attention_tflops_per_layer": attn_flops / 1e12,
        "config": {"model": c["name"], "layers": c["layers"], "d_model": c["D"], "ffn": c["FFN"],
                   "heads": f"{c['H']}/{c['HKV']}", "vocab": c["vocab"], "rope_theta": c["theta"],
                   "batch": c["B"], "seq_len": c["T"], "logits": "last position",
                   "levels": "L1 + L2 + L3 (L3: seeded N(0, 0.5) memory [1, 65536, 4096], the same for every layer)",
                   "mlp": {"fused": "gate/up GEMM with the SiLU-product epilogue, then down_proj (FusedSwiGLUMLP)",
                           "silu_mul": "transformers' cuBLAS GEMMs, one-pass SiLU product (SiLUMulMLP)",
                           "transformers": "transformers LlamaMLP (cuBLAS GEMMs + elementwise)"}[args.model_mlp],
                   "norms": ("one-pass RMSNorm kernel (FusedRMSNorm)" if fused_norms
                             else "transformers LlamaRMSNorm (elementwise kernels)")},
        "data": "synthetic token ids U[0, vocab), random N(0, 0.02) bf16 weights",
    }
    del model
    torch.cuda.empty_cache()
    return out


def bench_model_sharded(args, dist, rank, world, device):
    """The same full-model prefill over `world` GPUs of the box: every rank
    holds the whole model; the sequence's residual rows, RMSNorms and MLP are
    split by rows and the attention by kv heads (mka_b200.hf.sharded_llama):
    one NCCL all-gather of the normed hidden states and one of the gate logits
    per layer, and the attention output exchanged by the attention kernel's own
    stores into peer memory. One 65536-token sequence per step (fixed total
    work), device-timed, max over ranks."""
    from transformers import LlamaConfig, LlamaForCausalLM

    from mka_b200.hf.norm import apply_norm_fusion
    from mka_b200.hf.patch import HFPatchConfig, apply_hf_attention_patch
    from mka_b200.hf.sharded_llama import SequenceHeadShardedLlama

    c = MODEL
    cfg = LlamaConfig(vocab_size=c["vocab"], hidden_size=c["D"], intermediate_size=c["FFN"],
                      num_hidden_layers=c["layers"], num_attention_heads=c["H"], num_key_value_heads=c["HKV"],
                      max_position_embeddings=131072, rope_theta=c["theta"], attn_implementation="sdpa")
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(device):
            torch.manual_seed(5)
            model = LlamaForCausalLM(cfg).eval()
            patched = apply_hf_attention_patch(model, HFPatchConfig(use_l3=True, verbose=False))
            fused_norms = apply_norm_fusion(model) if args.model_norm == "fused" else 0
    finally:
        torch.set_default_dtype(prev)
    g = torch.Generator(device=device).manual_seed(6)
    ids = torch.randint(0, c["vocab"], (c["B"], c["T"]), generator=g, device=device)
    l3 = (torch.randn(c["B"], c["T"], c["D"], generator=g, device=device) * 0.5).to(torch.bfloat16)
    # the stream stays asynchronous; the status word is read once at the end of the run
    sh = SequenceHeadShardedLlama(model, rank, world, check_peer_status=False)

    def step():
        sh(ids, l3_memory=l3)

    step()  # warm-up: folds and shards each layer's weights, maps the peer regions
    steps = max(1, min(args.steps, 3))
    ms = _timed(dist, step, steps)
    sh.close()
    tokens = c["B"] * c["T"]
    out = {
        "metric": "Llama-3-8B prefill tokens/s, every self_attn patched with FastMKA, one sequence over the box",
        "value": tokens / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps, "n_gpus": world,
        "scaling": "strong", "patched_layers": patched, "fused_norms": fused_norms,
        "config": {"model": c["name"], "layers": c["layers"], "d_model": c["D"], "ffn": c["FFN"],
                   "heads": f"{c['H']}/{c['HKV']}", "vocab": c["vocab"], "rope_theta": c["theta"],
                   "batch": c["B"], "seq_len": c["T"], "logits": "last position",
                   "levels": "L1 + L2 + L3 (L3: seeded N(0, 0.5) memory [1, 65536, 4096], the same for every layer)",
                   "partition": f"rows {c['T'] // world} per rank (embeddings, RMSNorm, MLP, o_proj), "
                                f"{c['HKV'] // world} kv head(s) per rank (q/k/v, scan, attention)",
                   "collectives": "per layer: NCCL all-gather of the normed hidden states and of the gate logits; "
                                  "attention rows exchanged by peer stores from the attention kernel"},
        "data": "synthetic token ids U[0, vocab), random N(0, 0.02) bf16 weights",
    }
    del model, sh
    torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-long", action="store_true", help="skip the long-context (L3, seq 32768) measurement")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="how a head-sharded sequence group exchanges rows (long context, N > 2)")
    ap.add_argument("--model-mlp", choices=["fused", "silu_mul", "transformers"], default="silu_mul",
                    help="the full-model line's MLP: transformers' GEMMs with the one-pass SiLU product (default), "
                         "transformers' own, or the fused SwiGLU GEMM")
    ap.add_argument("--model-norm", choices=["fused", "transformers"], default="fused",
                    help="the full-model line's RMSNorms: the one-pass kernel (default) or transformers' own")
    ap.add_argument("--no-model", action="store_true",
                    help="skip the full Llama-3-8B model measurement (one GPU only)")
    ap.add_argument("--only", default=None,
                    help="run one kernel alone (attn_prefill, attn_decode, route_ema_blend, route_ema_blend_h, "
                         "qr_proj, kv_gemm, kv_proj, o_proj, o_proj_scatter, o_proj_blocked, l3_recall)")
    ap.add_argument("--batch", type=int, default=0, help="batch override for --only")
    ap.add_argument("--seq", type=int, default=0, help="sequence-length override for --only (prefill kernels)")
    args = ap.parse_args()
    if args.only:
        run_kernel_only(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    dist, rank, world, local = _dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    peaks = _peaks()
    from mka_b200 import ops

    sampler = ClockSampler(local)
    sampler.start()
    pre = bench_prefill(args, dist, rank, world, device, peaks)
    dec = None if args.no_decode else bench_decode(args, dist, rank, world, device, peaks)
    lc = None
    if not args.no_long:
        try:
            from mka_b200.sharded import plan_units

            plan_units(LONG["B"], LONG["HKV"], world)  # raises for world sizes the units do not split over
            lc = bench_long_context(args, dist, rank, world, device, peaks)
        except ValueError as e:
            lc = {"skipped": str(e)}
    clocks = sampler.stop()
    mhz = clocks["sm_mhz"] if clocks else None

    def mcycles(ms):  # kernel time in millions of SM cycles at the run's median clock
        return None if mhz is None or ms is None else round(ms * mhz * 1e-3, 4)
    model = None
    if not args.no_model:
        if world == 1:
            try:
                model = bench_model(args, device)
            except Exception as e:  # a secondary line must not take the headline line down with it
                model = {"error": f"{type(e).__name__}: {e}"[:400]}
                torch.cuda.empty_cache()
        elif MODEL["HKV"] % world == 0:
            try:
                model = bench_model_sharded(args, dist, rank, world, device)
            except Exception as e:  # a secondary line must not take the headline line down with it
                model = {"error": f"{type(e).__name__}: {e}"[:400]}
                torch.cuda.empty_cache()
        else:
            model = {"skipped": f"{MODEL['HKV']} kv heads do not split over {world} GPUs"}
    status = ops.device_status()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = measure_cpu(_oracle_params(pre["layer"]))
    launches_per_step = 5
    if rank == 0:
        line = {
            "metric": "FastMKA prefill tokens/s (Qwen-7B-like layer, B200)",
            "value": pre["tok_s"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": pre["ms"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1)/sqrt(d) input, N(0,0.02) weights)",
            "config": _config(args),
            "e2e": {"value": pre["e2e_tok_s"], "unit": "tokens/s", "h2d_bytes_per_step": pre["h2d"],
                    "d2h_bytes_per_step": pre["d2h"], "ms_per_step": pre["e2e_ms"],
                    "pipeline": "per sequence: upload of sequence u+1 and download of u-1 overlap the forward of u (3 streams)"},
            "roofline": dict(pre["roofline"], launch_mcycles=mcycles(pre["roofline"]["launch_ms"])),
            "attention_beside_sdpa": pre["attention_beside_sdpa"],
            "cpu_baseline": cpu,
            "gpu_launches": launches_per_step * args.steps,
            "stages_ms": {k: round(v, 4) for k, v in pre["stages_ms"].items()},
            "stages_mcycles": {k: mcycles(v) for k, v in pre["stages_ms"].items()},
            "clocks": clocks,
            "device_status": status,
        }
        if dec is not None:
            d = DECODE
            line["decode"] = {
                "metric": "FastMKA decode tokens/s (Llama-3-8B-like layer, batch 64, 32768 cached)",
                "value": dec["tok_s"], "unit": "tokens/s", "ms_per_step": dec["ms"], "roofline": dec["roofline"],
                "stages_ms": {k: round(v, 4) for k, v in dec["stages_ms"].items()},
                "stages_mcycles": {k: mcycles(v) for k, v in dec["stages_ms"].items()},
                "config": {"batch_per_gpu": d["B"], "cache_len": d["TK"], "d_model": d["D"],
                           "heads": f"{d['H']}/{d['HKV']}"},
                "gpu_launches": launches_per_step * args.steps,
            }
        if lc is not None:
            if "roofline" in lc:
                lc["roofline"]["launch_mcycles"] = mcycles(lc["roofline"]["launch_ms"])
            line["long_context"] = lc
        if model is not None:
            line["model"] = model
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
