"""CPU-only checks of the host side: the C-ABI library loads and exports every
entry point include/fastmka_b200.h declares (no compute is launched), argument
errors come back as status codes with messages, the Python layers keep the
reference's API, and weight preparation is exact."""
import ctypes
import os
import re

import pytest
import torch
import torch.nn as nn

from tests import golden_io

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fastmka_b200.h")


def _header_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"FMKA_API\s+[\w\s\*]+?\b(fmka_\w+)\s*\(", src)))


def test_library_exports_every_header_symbol():
    from mka_b200 import _lib

    lib = _lib.load()
    names = _header_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.exported_symbols())
    assert b"sm_100a" in lib.fmka_version()


def test_argument_errors_are_status_codes():
    from mka_b200 import _lib

    lib = _lib.load()
    rc = lib.fmka_gemm_bf16(None, 0, None, 0, None, None, 0, 1, 1, 1, None)
    assert rc == 1  # FMKA_ERR_INVALID_ARGUMENT
    code, msg = _lib.last_error()
    assert code == 1 and "null" in msg
    rc = lib.fmka_attn_fwd_prefill(None, 0, 0, 0, None, None, 0, 0, 0, None, 0, 0, 0, None, 0, 0,
                                   1, 1, 1, 1, 1, 128, 1, 1.0, None)
    assert rc == 1
    with pytest.raises(_lib.FastMKAError, match="null"):
        _lib.call("fmka_route_ema_blend", None, 0, 0, None, None, None, 2, None, 0, 0, 0, 0.9, 1, 1, 8, None, 0, 0,
                  None, None, 0, None)


def test_argument_errors_of_the_newer_entry_points():
    """Checked on the host before any device work, so they run without a GPU:
    rows that would overlap, the SwiGLU channel rule, scatter destination
    counts and coverage, and the barrier's rank / group size."""
    from mka_b200 import _lib

    lib = _lib.load()
    P = ctypes.c_void_p
    a, w, c = P(1 << 12), P(1 << 13), P(1 << 14)  # aligned addresses; nothing is launched
    rc = lib.fmka_gemm_bf16(a, 64, w, 64, None, c, 32, 128, 64, 64, None)  # ldc 32 < N 64
    assert rc == 1 and "row stride" in _lib.last_error()[1]
    rc = lib.fmka_gemm_bf16_swiglu(a, 64, w, 64, None, c, 192, 128, 192, 64, None)  # I = 192
    assert rc == 1 and "multiple of 128" in _lib.last_error()[1]
    rc = lib.fmka_gemm_bf16_swiglu(a, 64, w, 64, None, c, 64, 128, 128, 64, None)  # ldc 64 < I 128
    assert rc == 1 and "row stride" in _lib.last_error()[1]
    dsts = (P * 9)(*([c] * 9))
    rc = lib.fmka_gemm_bf16_kblocked_scatter(a, 64, 128 * 64, 64, w, 128, None, dsts, 9, 0, 128, 128, 128, 128, None)
    assert rc == 1 and "1 to 8" in _lib.last_error()[1]
    rc = lib.fmka_attn_fwd_prefill_scatter(a, 0, 0, 128, w, w, 0, 0, 128, dsts, 2, 100, 0, 256, 128,
                                           1, 2, 1, 300, 300, 128, 1, 0.1, None)  # 2 x 100 rows < 300
    assert rc == 1 and "cover" in _lib.last_error()[1]
    flags = (P * 2)(c, c)
    assert lib.fmka_peer_barrier(flags, 2, 2, 1, None) == 1  # rank outside the group
    assert lib.fmka_peer_barrier(flags, 0, 9, 1, None) == 1  # more than 8 ranks
    assert lib.fmka_peer_alloc(0, ctypes.byref(P())) == 1
    # L3 chunk recall
    rc = lib.fmka_l3_topr_f32(c, 64, 10, 64, 33, 1.0, a, w, None)  # R > 32
    assert rc == 2 and "1..32" in _lib.last_error()[1]
    rc = lib.fmka_l3_topr_f32(c, 64, 10, 4, 8, 1.0, a, w, None)  # R > N
    assert rc == 1 and "exceeds" in _lib.last_error()[1]
    rc = lib.fmka_l3_topr_f32(c, 32, 10, 64, 4, 1.0, a, w, None)  # row stride < N
    assert rc == 1 and "row stride" in _lib.last_error()[1]
    rc = lib.fmka_l3_block_mean_bf16(a, 0, 100, 1, 16, 100, 4, c, 100, None)  # D = 100 not a multiple of 8
    assert rc == 1 and "multiples of 8" in _lib.last_error()[1]
    rc = lib.fmka_l3_recall_gather_bf16(a, w, 0, c, 64, 10, 64, 1, 16, 4, c, 64, 64, None)  # R = 0
    assert rc == 2 and "1..32" in _lib.last_error()[1]
    rc = lib.fmka_gemm_bf16_f32out(a, 64, w, 64, None, 64, 128, 64, 64, None)
    assert rc == 1 and "null" in _lib.last_error()[1]


def test_l3_store_validates_its_bank():
    """Host checks of the L3 chunk bank (no device work)."""
    from mka_b200.l3 import L3ChunkStore

    with pytest.raises(ValueError, match="bf16 CUDA"):
        L3ChunkStore(torch.zeros(8, 64, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="n_chunks, D"):
        L3ChunkStore(torch.zeros(8, 64), torch.zeros(8, 32))


def test_workspace_sizes():
    from mka_b200 import _lib

    lib = _lib.load()
    # route/EMA: ticket + flags (256-aligned) + two fp32 [records, 256] arrays, one
    # record per (batch row, 256-channel slice, 64-token chunk)
    B, T, D = 4, 8192, 3584
    nrec = B * ((D + 255) // 256) * ((T + 63) // 64)
    flag_bytes = ((nrec * 4 + 256 + 255) // 256) * 256
    assert lib.fmka_route_ema_blend_workspace_size(B, T, D) == flag_bytes + 2 * nrec * 256 * 4
    assert lib.fmka_route_ema_blend_workspace_size(0, 1, 1) == 0
    # decode with one split needs no workspace; more splits need (Dh + 1) floats per (b, h, split)
    assert lib.fmka_attn_decode_workspace_size(2, 8, 8, 64, 1) == 0
    assert lib.fmka_attn_decode_workspace_size(2, 8, 8, 4096, 4) == 2 * 8 * 4 * 129 * 4


def test_ops_refuse_cpu_tensors():
    from mka_b200 import ops

    q = torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.attn_prefill(q, q, q)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.causal_prefix_ema(torch.zeros(1, 4, 8, dtype=torch.bfloat16))
    # the reference's op API (mka/cuda/ops.py): same probes, same RuntimeError on CPU inputs
    from mka_b200 import cuda as mka_cuda

    assert mka_cuda.has_fastmka_cuda() == torch.cuda.is_available()
    assert mka_cuda.has_fused_route_mka_cuda() == torch.cuda.is_available()
    with pytest.raises(RuntimeError):
        mka_cuda.fastmka_attn(q, q, q)
    x = torch.zeros(1, 128, 128)
    with pytest.raises(RuntimeError):
        mka_cuda.fused_route_mka_attn(q, x, x, x, torch.zeros(1, 128, 2), torch.zeros(128, 128), torch.zeros(128, 128))


def test_fastmka_module_matches_reference_parameters():
    """Same parameter names and shapes as the reference module (golden state_dict)."""
    from mka_b200 import FastMKAAttention, FastMKAConfig

    c = golden_io.load("fastmka_mha_l3_pad")
    ref = golden_io.params(c)
    m = FastMKAAttention(FastMKAConfig(hidden_size=256, num_heads=2, use_l3=True))
    ours = {k: tuple(v.shape) for k, v in m.state_dict().items()}
    assert ours == {k: tuple(v.shape) for k, v in ref.items()}
    m.load_state_dict(ref)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.zeros(1, 4, 256))


def test_hf_wrapper_reads_config_and_patch_walks_layers():
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaAttention

    from mka_b200 import HFFastMKAAttention, HFPatchConfig, apply_hf_attention_patch, parse_patch_config

    cfg = LlamaConfig(hidden_size=512, num_attention_heads=4, num_key_value_heads=1, intermediate_size=64,
                      vocab_size=16)

    class Layer(nn.Module):
        def __init__(self):
            super().__init__()
            self.self_attn = LlamaAttention(cfg, layer_idx=0)

    class Inner(nn.Module):
        def __init__(self):
            super().__init__()
            self.layers = nn.ModuleList([Layer(), Layer(), nn.Module()])

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.model = Inner()

    model = Model()
    pc = parse_patch_config({"use_l3": True, "ema_beta": 0.8, "verbose": False})
    assert pc == HFPatchConfig(use_l3=True, ema_beta=0.8, verbose=False)
    assert apply_hf_attention_patch(model, pc) == 2
    w = model.model.layers[0].self_attn
    assert isinstance(w, HFFastMKAAttention)
    assert (w.hidden_size, w.num_heads, w.num_key_value_heads, w.head_dim) == (512, 4, 1, 128)
    assert w.router[2].out_features == 3 and w.router[0].out_features == 256
    assert apply_hf_attention_patch(model, HFPatchConfig(mode="off")) == 0
    with pytest.raises(ValueError):
        apply_hf_attention_patch(nn.Linear(2, 2), HFPatchConfig(verbose=False))


def test_prepared_weights_fold_router_through_q():
    """router(q) == W2 act((W1 Wq) x + (W1 bq + b1)) + b2 exactly in fp32."""
    from mka_b200.layers.prepared import prepare

    torch.manual_seed(0)
    D, R = 256, 64
    wq, wk, wv, wo = (nn.Linear(D, D, bias=b) for b in (True, True, True, False))
    router = nn.Sequential(nn.Linear(D, R), nn.GELU(), nn.Linear(R, 3))
    W = prepare(wq, wk, wv, wo, router, torch.device("cpu"))
    assert W.act == 1 and W.levels == 3 and W.router_hidden == R
    x = torch.randn(5, D)
    folded = x @ W.w_qr.float()[D:].t() + W.b_qr[D:]
    direct = router[0](wq(x))
    assert (folded - direct).abs().max().item() < 0.05  # bf16 rounding of the stacked weight
    W2 = prepare(wq, wk, wv, wo, router, torch.device("cpu"), W)
    assert W2 is W  # unchanged parameters reuse the prepared copy
    with torch.no_grad():
        wq.weight.add_(1.0)
    assert prepare(wq, wk, wv, wo, router, torch.device("cpu"), W) is not W
    router[1] = nn.Tanh()
    with pytest.raises(NotImplementedError):
        prepare(wq, wk, wv, wo, router, torch.device("cpu"))


def test_static_kv_cache_bookkeeping():
    """Host logic of the in-place decode cache (buffers on the CPU here): one
    slot per attention module in call order, lengths, the capacity and layer
    limits, prefix loading, and the EMA state ping-pong of carry_ema."""
    from mka_b200 import StaticKVCache

    c = StaticKVCache(batch=2, num_kv_heads=1, capacity=8, num_layers=2, device="cpu", carry_ema=True)
    a, b, extra = nn.Linear(1, 1), nn.Linear(1, 1), nn.Linear(1, 1)
    ka, _ = c.layer(a)
    kb, _ = c.layer(b)
    assert ka.data_ptr() != kb.data_ptr() and c.layer(a)[0].data_ptr() == ka.data_ptr()
    with pytest.raises(RuntimeError):
        c.layer(extra)  # more attention modules than layers
    c.advance(a, 5)
    assert c.length(a) == 5 and c.length(b) == 0
    with pytest.raises(RuntimeError):
        c.advance(a, 4)  # 9 > capacity 8
    assert c.length(a) == 5
    k = torch.randn(2, 1, 3, 128).bfloat16()
    c.load_prefix(1, k, -k)
    assert c.length(b) == 3 and torch.equal(c.k[1][:, :, :3], k) and torch.equal(c.v[1][:, :, :3], -k)
    s_in, s_out = c.ema_buffers(a, 256, "cpu")
    assert s_in.shape == (2, 256) and s_in.dtype == torch.float32 and not s_in.any()
    s_out.fill_(1.0)
    c.commit_ema(a)
    s_in2, s_out2 = c.ema_buffers(a, 256, "cpu")
    assert s_in2.data_ptr() == s_out.data_ptr() and s_out2.data_ptr() == s_in.data_ptr()
    assert bool((s_in2 == 1.0).all())


def test_peer_timeout_in_status_word_raises(monkeypatch):
    """A peer barrier that ran out of time leaves FMKA_STATUS_PEER_TIMEOUT in the
    device status word; the head-sharded layer's check turns it into an error
    (the status read is replaced by a fake, so no GPU is needed)."""
    from mka_b200 import ops, sharded

    seen = []

    def fake_status(clear=True):
        seen.append(clear)
        return fake_status.word

    monkeypatch.setattr(ops, "device_status", fake_status)
    fake_status.word = 0
    sharded.raise_on_peer_timeout()
    fake_status.word = ops.STATUS_LOOKBACK_TIMEOUT  # other bits are not this check's business
    sharded.raise_on_peer_timeout()
    fake_status.word = ops.STATUS_PEER_TIMEOUT | ops.STATUS_WAIT_TIMEOUT
    with pytest.raises(sharded.PeerExchangeError, match="peer barrier"):
        sharded.raise_on_peer_timeout()
    assert seen == [False, False, False]  # the word is left for the caller's own poll
