"""GPU checks of the L3 chunk recall (mka_b200.l3, l3_recall.cu) against the
oracle's restatement. The reference describes the tier and implements none
(mka/config/memory_hierarchy.py:1-10,30-34), so these pin the package's own
algorithm: block-mean queries, fp32 dot-product scores, top-R with the lower
chunk index first on ties, softmax weights, one weighted sum per query block.

Tolerances: block means within one bf16 step; scores to 1e-4 relative (fp32
accumulation against fp64); chunk indices exact wherever the oracle's scores
leave a margin at the R-th place; weights 1e-4; R to 1e-2 relative (bf16 out).
"""
import math

import pytest
import torch

from oracle import fastmka_oracle as orc

pytestmark = pytest.mark.gpu


def _bf(*shape, gen, scale=1.0):
    return (torch.randn(*shape, generator=gen) * scale).bfloat16()


@pytest.fixture(scope="module")
def ops():
    from mka_b200 import ops as o
    return o


@pytest.mark.parametrize("M,N,K", [(7, 100, 64), (300, 4096, 512), (1024, 1000, 3584)])
def test_gemm_f32out(ops, M, N, K):
    g = torch.Generator().manual_seed(M + N)
    a, w = _bf(M, K, gen=g), _bf(N, K, gen=g)
    out = ops.gemm_f32out(a.cuda(), w.cuda())
    assert out.dtype == torch.float32 and out.shape == (M, N)
    ref = a.double() @ w.double().t()
    assert ((out.cpu().double() - ref).abs().max() / ref.abs().max()).item() < 1e-4


@pytest.mark.parametrize("B,T,D,L", [(1, 64, 256, 64), (2, 700, 512, 64), (3, 33, 136, 16), (1, 5, 3584, 64)])
def test_block_mean(ops, B, T, D, L):
    g = torch.Generator().manual_seed(T + D)
    x = _bf(B, T, D, gen=g)
    q = ops.l3_block_mean(x.cuda(), L).cpu().float()
    ref = orc.l3_block_mean(x.float(), L)
    assert q.shape == ref.shape
    assert ((q - ref).abs() <= ref.abs() * 2 ** -7 + 1e-6).all()


@pytest.mark.parametrize("M,N,R", [(1, 37, 1), (13, 1000, 5), (300, 4096, 8), (64, 2000, 16), (20, 300, 32),
                                   (9, 8, 8)])
def test_topr_matches_oracle(ops, M, N, R):
    g = torch.Generator().manual_seed(M * N + R)
    s = torch.randn(M, N, generator=g)
    idx, w = ops.l3_topr(s.cuda(), R, 0.7)
    ridx, rw = orc.l3_topr(s, R, 0.7)
    assert torch.equal(idx.cpu().long(), ridx)
    assert (w.cpu() - rw).abs().max().item() < 1e-5


def test_topr_ties_take_the_lower_index(ops):
    g = torch.Generator().manual_seed(3)
    s = (torch.randn(40, 700, generator=g) * 4).round() / 4  # many equal scores
    idx, w = ops.l3_topr(s.cuda(), 12, 1.0)
    ridx, rw = orc.l3_topr(s, 12, 1.0)
    assert torch.equal(idx.cpu().long(), ridx)
    assert (w.cpu() - rw).abs().max().item() < 1e-5


@pytest.mark.parametrize("B,T,D,N,R,L", [(2, 700, 512, 3000, 8, 64), (1, 256, 3584, 512, 4, 64),
                                         (3, 100, 256, 64, 16, 32)])
def test_recall_matches_oracle(ops, B, T, D, N, R, L):
    g = torch.Generator().manual_seed(B * T + N)
    x = _bf(B, T, D, gen=g)
    keys = _bf(N, D, gen=g)
    vals = _bf(N, D, gen=g)
    out, idx, w = ops.l3_chunk_recall(x.cuda(), keys.cuda(), vals.cuda(), R, L)
    q = ops.l3_block_mean(x.cuda(), L).cpu().float()
    r_ref, idx_ref, w_ref, scores = orc.l3_chunk_recall(x.float(), keys.float(), vals.float(), R, L, q=q)
    idx = idx.cpu().long()
    # rows whose R-th and (R+1)-th scores are too close to rank reliably in fp32 are left out
    srt = scores.sort(dim=1, descending=True).values
    margin = (srt[:, R - 1] - srt[:, R]).abs() if N > R else torch.full((scores.shape[0],), 1.0, dtype=torch.float64)
    ok = margin > 1e-4 * srt[:, 0].abs().clamp_min(1.0)
    assert ok.float().mean().item() > 0.9
    assert torch.equal(idx[ok], idx_ref[ok])
    assert (w.cpu()[ok] - w_ref[ok]).abs().max().item() < 1e-4
    nq = (T + L - 1) // L
    rows_ok = ok.view(B, nq)[:, torch.arange(T) // L]
    err = (out.cpu().float() - r_ref).abs()[rows_ok]
    assert err.max().item() <= 1e-2 * r_ref.abs().max().item()
    assert out.shape == (B, T, D) and out.dtype == torch.bfloat16


def test_store_from_history_feeds_the_attention(ops):
    """A bank made from earlier hidden states recalls R for the current ones, and
    the patched HF attention with use_l3 takes it as l3_memory, matching the
    oracle's forward with the same R."""
    from mka_b200.l3 import L3ChunkStore
    from tests.test_parity_gpu import _check_gqa_layer, _gqa_l3_layer

    g = torch.Generator().manual_seed(11)
    hist = _bf(1, 2048, 512, gen=g, scale=0.5)
    store = L3ChunkStore.from_history(hist.cuda(), 64)
    assert store.n_chunks == 32
    x = _bf(2, 300, 512, gen=g, scale=0.5)
    r = store.recall(x.cuda(), top_r=4, block_len=32)
    r_same, _, _ = ops.l3_chunk_recall(x.cuda(), store.keys, store.values, 4, 32)
    assert torch.equal(r, r_same)
    assert r.shape == (2, 300, 512) and torch.isfinite(r.float()).all()
    layer, p = _gqa_l3_layer(512, 4, 2, 256, 3, seed=27, w_std=0.05)
    _check_gqa_layer(layer, p, x.float(), 4, 2, l3=r.cpu().float())


def test_store_append_keeps_chunk_order(ops):
    """Two banks appended: the chunks of the second follow those of the first, and
    the recall over the joined bank is the recall over its keys and values."""
    from mka_b200.l3 import L3ChunkStore

    g = torch.Generator().manual_seed(13)
    k1, v1 = _bf(40, 256, gen=g).cuda(), _bf(40, 256, gen=g).cuda()
    k2, v2 = _bf(25, 256, gen=g).cuda(), _bf(25, 256, gen=g).cuda()
    joined = L3ChunkStore(k1, v1).append(L3ChunkStore(k2, v2))
    assert joined.n_chunks == 65
    assert torch.equal(joined.keys[40:], k2) and torch.equal(joined.values[:40], v1)
    x = _bf(1, 130, 256, gen=g).cuda()
    r, idx, w = joined.recall_with_indices(x, top_r=6, block_len=64)
    r2, idx2, w2 = ops.l3_chunk_recall(x, torch.cat([k1, k2]), torch.cat([v1, v2]), 6, 64)
    assert torch.equal(r, r2) and torch.equal(idx, idx2)
    with pytest.raises(ValueError):
        joined.recall(x, top_r=33)
