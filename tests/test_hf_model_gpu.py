"""A transformers LlamaForCausalLM with the FastMKA self_attn patch installed,
run the way transformers >= 4.48 runs it (decoder layers unpack two values,
K/V go through a DynamicCache, RoPE comes in as position_embeddings), against
the same model whose attention is the oracle in fp32 on the CPU.

Reference behaviour: mka/hf/patch.py:30-48 (the patch), mka/hf/attention.py:82-199
(the wrapped forward). Both models hold the same bf16-rounded weights; the
patched one runs on cuda:0 in bf16.
"""
import copy

import pytest
import torch
import torch.nn as nn

transformers = pytest.importorskip("transformers")
from transformers import DynamicCache, LlamaConfig, LlamaForCausalLM  # noqa: E402

from mka_b200.hf.attention import HFFastMKAAttention, _is_hf_cache  # noqa: E402
from mka_b200.hf.patch import HFPatchConfig, _two_value_attention_api, apply_hf_attention_patch  # noqa: E402
from oracle import fastmka_oracle as O  # noqa: E402


class OracleAttention(nn.Module):
    """The reference HF FastMKA attention in fp32 on the CPU, with the weights of
    a patched module, speaking the transformers >= 4.48 self_attn protocol."""

    def __init__(self, patched: HFFastMKAAttention, layer_idx: int):
        super().__init__()
        f = lambda t: None if t is None else t.detach().float().cpu().clone()  # noqa: E731
        self.p = {"wq": f(patched.q_proj.weight), "bq": f(patched.q_proj.bias),
                  "wk": f(patched.k_proj.weight), "bk": f(patched.k_proj.bias),
                  "wv": f(patched.v_proj.weight), "bv": f(patched.v_proj.bias),
                  "wo": f(patched.o_proj.weight), "bo": f(patched.o_proj.bias),
                  "r1w": f(patched.router[0].weight), "r1b": f(patched.router[0].bias),
                  "r2w": f(patched.router[2].weight), "r2b": f(patched.router[2].bias)}
        self.p = {k: v for k, v in self.p.items() if v is not None}
        self.nh, self.nkv, self.beta = patched.num_heads, patched.num_key_value_heads, patched.ema_beta
        self.idx = layer_idx

    def forward(self, hidden_states, position_embeddings=None, attention_mask=None, past_key_values=None, **kw):
        assert attention_mask is None
        cos, sin = position_embeddings
        past = None
        if past_key_values is not None and past_key_values.get_seq_length(self.idx) > 0:
            lay = past_key_values.layers[self.idx]
            past = (lay.keys, lay.values)
        r = O.hf_fastmka_forward(hidden_states.float(), self.p, self.nh, self.nkv, False, self.beta, "silu",
                                 past=past, cos=cos.float().unsqueeze(1), sin=sin.float().unsqueeze(1))
        if past_key_values is not None:
            t = hidden_states.shape[1]
            past_key_values.update(r["k"][:, :, -t:], r["v"][:, :, -t:], self.idx)
        return r["out"], None


def _tiny_llama(seed=0):
    cfg = LlamaConfig(vocab_size=128, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=2, num_key_value_heads=1, max_position_embeddings=1024,
                      rope_theta=500000.0, attn_implementation="sdpa")
    torch.manual_seed(seed)
    return LlamaForCausalLM(cfg).eval()


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm()).item()


def test_patch_picks_transformers_protocol():
    """Host logic only: the patch installs two-value modules on transformers
    >= 4.48, leaves the reference's three-value form otherwise, and the Cache
    detection accepts transformers caches but not tuples."""
    model = _tiny_llama()
    n = apply_hf_attention_patch(model, HFPatchConfig(verbose=False))
    assert n == 2
    for layer in model.model.layers:
        assert isinstance(layer.self_attn, HFFastMKAAttention)
        assert layer.self_attn.return_present == (not _two_value_attention_api())
        assert layer.self_attn.layer_idx is not None
    assert _is_hf_cache(DynamicCache())
    assert not _is_hf_cache((torch.zeros(1), torch.zeros(1)))
    assert not _is_hf_cache(None)
    assert apply_hf_attention_patch(_tiny_llama(), HFPatchConfig(enabled=False, verbose=False)) == 0


@pytest.mark.gpu
def test_patched_llama_prefill_and_cached_decode():
    if not _two_value_attention_api():
        pytest.skip("needs the transformers >= 4.48 self_attn protocol")
    model = _tiny_llama().to(torch.bfloat16)
    assert apply_hf_attention_patch(model, HFPatchConfig(verbose=False)) == 2
    with torch.no_grad():  # bf16-round the new router weights too, then copy for the oracle
        for layer in model.model.layers:
            for prm in layer.self_attn.router.parameters():
                prm.copy_(prm.to(torch.bfloat16))
    ref = copy.deepcopy(model).float()
    for i, (lr, lm) in enumerate(zip(ref.model.layers, model.model.layers)):
        lr.self_attn = OracleAttention(lm.self_attn, i)
    model = model.to("cuda")

    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 128, (2, 96), generator=g)
    with torch.no_grad():
        out = model(ids.cuda(), use_cache=True)
        ref_out = ref(ids, use_cache=True)
        assert isinstance(out.past_key_values, DynamicCache)
        assert out.past_key_values.get_seq_length() == 96
        # bf16 weights, activations, P and O against fp32 throughout: relative
        # Frobenius error of the logits
        assert _rel(out.logits, ref_out.logits) < 3e-2
        pkv, rkv = out.past_key_values, ref_out.past_key_values
        for step in range(2):
            tok = torch.randint(0, 128, (2, 1), generator=g)
            o = model(tok.cuda(), past_key_values=pkv, use_cache=True)
            r = ref(tok, past_key_values=rkv, use_cache=True)
            assert o.past_key_values.get_seq_length() == 97 + step
            assert _rel(o.logits, r.logits) < 3e-2, step
            pkv, rkv = o.past_key_values, r.past_key_values
        k_gpu = pkv.layers[1].keys.float().cpu()
        k_ref = rkv.layers[1].keys
        assert k_gpu.shape == k_ref.shape == (2, 1, 98, 128)
        assert _rel(k_gpu, k_ref) < 3e-2


def test_mlp_fusion_walks_layers_and_keeps_parameter_names():
    """Host logic only: every gated SiLU MLP is replaced, the state_dict keys
    and tensors are unchanged, and a second call changes nothing."""
    from mka_b200.hf.mlp import FusedSwiGLUMLP, apply_mlp_fusion

    model = _tiny_llama()
    keys = {k: v.clone() for k, v in model.state_dict().items()}
    assert apply_mlp_fusion(model) == 2
    assert all(isinstance(layer.mlp, FusedSwiGLUMLP) for layer in model.model.layers)
    after = model.state_dict()
    assert set(after) == set(keys)
    assert all(torch.equal(after[k], keys[k]) for k in keys)
    assert apply_mlp_fusion(model) == 0


def test_silu_mul_mlp_walk_keeps_parameter_names():
    """Host logic of mode="silu_mul": bf16 gated SiLU MLPs are replaced by
    SiLUMulMLP with the same state_dict; an fp32 model is left alone."""
    from mka_b200.hf.mlp import SiLUMulMLP, apply_mlp_fusion

    model = _tiny_llama()
    assert apply_mlp_fusion(model, mode="silu_mul") == 0  # fp32 weights: not replaced
    model = model.to(torch.bfloat16)
    keys = {k: v.clone() for k, v in model.state_dict().items()}
    assert apply_mlp_fusion(model, mode="silu_mul") == 2
    assert all(isinstance(layer.mlp, SiLUMulMLP) for layer in model.model.layers)
    after = model.state_dict()
    assert set(after) == set(keys)
    assert all(torch.equal(after[k], keys[k]) for k in keys)
    assert apply_mlp_fusion(model, mode="silu_mul") == 0
    assert apply_mlp_fusion(model) == 0
    with pytest.raises(ValueError):
        apply_mlp_fusion(model, mode="gelu")


@pytest.mark.gpu
def test_silu_mul_mlp_matches_transformers_mlp():
    """SiLUMulMLP against transformers' LlamaMLP (same GEMMs, same roundings)
    and against an fp32 SwiGLU MLP; a patched model with it against the same
    model with transformers' MLP."""
    from mka_b200.hf.mlp import SiLUMulMLP, apply_mlp_fusion

    model = _tiny_llama().to(torch.bfloat16)
    assert apply_hf_attention_patch(model, HFPatchConfig(verbose=False)) == 2
    model = model.to("cuda")
    fused = copy.deepcopy(model)
    assert apply_mlp_fusion(fused, mode="silu_mul") == 2
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(2, 96, 256, generator=g) * 0.5).bfloat16().cuda()
    with torch.no_grad():
        mlp = model.model.layers[0].mlp
        sm = SiLUMulMLP(mlp)
        f32 = lambda lin: lin.weight.detach().float().cpu()  # noqa: E731
        xf = x.float().cpu()
        ref = torch.nn.functional.silu(xf @ f32(mlp.gate_proj).T) * (xf @ f32(mlp.up_proj).T)
        ref = ref @ f32(mlp.down_proj).T
        assert _rel(sm(x), ref) < 2e-2
        assert _rel(sm(x), mlp(x)) < 1e-2
        ids = torch.randint(0, 128, (2, 96), generator=g).cuda()
        a = model(ids).logits
        b = fused(ids).logits
    assert _rel(b, a) < 1e-2


@pytest.mark.gpu
def test_fused_mlp_matches_transformers_mlp():
    """The fused MLP of one layer against an fp32 SwiGLU MLP on the CPU, and a
    patched LlamaForCausalLM with the fused MLP against the same model with
    transformers' MLP (both bf16 on the GPU, self_attn patched in both)."""
    from mka_b200.hf.mlp import FusedSwiGLUMLP, apply_mlp_fusion

    model = _tiny_llama().to(torch.bfloat16)
    assert apply_hf_attention_patch(model, HFPatchConfig(verbose=False)) == 2
    model = model.to("cuda")
    fused = copy.deepcopy(model)
    assert apply_mlp_fusion(fused) == 2
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(2, 96, 256, generator=g) * 0.5).bfloat16().cuda()
    with torch.no_grad():
        mlp = model.model.layers[0].mlp
        fm = FusedSwiGLUMLP(mlp)
        # an fp32 SwiGLU MLP with the same (bf16) weights on the CPU: down(silu(gate x) * up x)
        f32 = lambda lin: lin.weight.detach().float().cpu()  # noqa: E731
        xf = x.float().cpu()
        ref = torch.nn.functional.silu(xf @ f32(mlp.gate_proj).T) * (xf @ f32(mlp.up_proj).T)
        ref = ref @ f32(mlp.down_proj).T
        assert _rel(fm(x), ref) < 2e-2
        assert _rel(fm(x), mlp(x)) < 2e-2
        ids = torch.randint(0, 128, (2, 96), generator=g).cuda()
        a = model(ids).logits
        b = fused(ids).logits
    assert _rel(b, a) < 2e-2


def test_l3_memory_reaches_every_patched_layer(monkeypatch):
    """Host logic only: an L3 memory passed with the model call (the three-level
    full-model configuration) arrives at every patched self_attn's
    forward_with_lse, unchanged, next to the model's own RoPE tables."""
    if not _two_value_attention_api():
        pytest.skip("needs the transformers >= 4.48 self_attn protocol")
    model = _tiny_llama()
    assert apply_hf_attention_patch(model, HFPatchConfig(use_l3=True, verbose=False)) == 2
    seen = []

    def fake(self, hidden_states, attention_mask=None, position_ids=None, past_key_value=None,
             output_attentions=False, use_cache=False, cache_position=None, position_embeddings=None,
             l3_memory=None, **kw):
        seen.append((self.layer_idx, l3_memory, position_embeddings is not None))
        return hidden_states, None, None, None, None

    monkeypatch.setattr(HFFastMKAAttention, "forward_with_lse", fake)
    r = torch.randn(1, 12, 256)
    with torch.no_grad():
        model(torch.randint(0, 128, (1, 12)), use_cache=False, logits_to_keep=1, l3_memory=r)
    assert [s[0] for s in seen] == [0, 1]
    assert all(s[1] is r and s[2] for s in seen)
    assert all(layer.self_attn.use_l3 for layer in model.model.layers)


def test_norm_fusion_walks_modules_and_keeps_parameter_names():
    """Host logic only: every RMSNorm of a bf16 Llama (two per decoder layer and
    the final one) is replaced, the state_dict is unchanged, a second call
    changes nothing, fp32 models are left alone, and the fused module refuses
    CPU input (it has no CPU path)."""
    from mka_b200.hf.norm import FusedRMSNorm, apply_norm_fusion

    model = _tiny_llama()
    assert apply_norm_fusion(model) == 0  # fp32 weights: not installed
    model = model.to(torch.bfloat16)
    keys = {k: v.clone() for k, v in model.state_dict().items()}
    assert apply_norm_fusion(model) == 2 * 2 + 1
    assert isinstance(model.model.norm, FusedRMSNorm)
    assert all(isinstance(layer.input_layernorm, FusedRMSNorm) for layer in model.model.layers)
    after = model.state_dict()
    assert set(after) == set(keys) and all(torch.equal(after[k], keys[k]) for k in keys)
    assert apply_norm_fusion(model) == 0
    with pytest.raises(RuntimeError, match="CUDA"):
        model.model.norm(torch.zeros(2, 256, dtype=torch.bfloat16))
