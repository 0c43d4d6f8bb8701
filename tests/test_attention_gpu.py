"""Decode attention over the paged K/V cache (wk_attention_decode, the kernel
the engine's decode steps launch) against the oracle's restatement of the
reference's rounding points, and the cluster kernel (one cluster of CTAs per
(row, KV head), partial results exchanged through distributed shared memory)
against the one-CTA kernel.

Pages are shuffled in the block table, the newest page of every sequence
holds NaN past the sequence end (stale cache bytes that must not reach the
output), and the shapes cover head_dim 64 and 128, 1 to 8 query heads per KV
head, contexts from 1 token to 4096, and enough (row, KV head) pairs that the
clusters run in several waves.
"""
import numpy as np
import pytest

import wukong_b200 as wk
from oracle import oracle as orc
from tests.gpu_util import alloc, down, free, up

pytestmark = pytest.mark.gpu


def _case(rows, H, Hk, D, positions, max_len, act, seed):
    rng = np.random.default_rng(seed)
    max_pages = (max_len + 63) // 64
    npool = rows * max_pages + 3
    perm = rng.permutation(npool)[: rows * max_pages].reshape(rows, max_pages).astype(np.int32)
    kpool = orc.round_act(rng.standard_normal((npool, Hk, 64, D)).astype(np.float32), act)
    vpool = orc.round_act(rng.standard_normal((npool, Hk, 64, D)).astype(np.float32), act)
    for r, p in enumerate(positions):
        last = perm[r, p // 64]
        kpool[last, :, p % 64 + 1:, :] = np.nan
        vpool[last, :, p % 64 + 1:, :] = np.nan
    q = orc.round_act(rng.standard_normal((rows, H * D)).astype(np.float32), act)
    return q, kpool, vpool, perm


def _bits(x, act):
    if act == wk.F16:
        return x.astype(np.float16)
    u = x.astype(np.float32).view(np.uint32)
    return (u >> 16).astype(np.uint16)


def _from(raw, act):
    if act == wk.F16:
        return raw.astype(np.float32)
    return (raw.astype(np.uint32) << 16).view(np.float32)


def _run(dev, q, kpool, vpool, perm, positions, H, Hk, D, max_len, act):
    rows = q.shape[0]
    seq = np.arange(rows, dtype=np.int32)
    pos = np.asarray(positions, np.int32)
    pq, pk, pv, pb, ps, pp = up(_bits(q, act)), up(_bits(kpool, act)), up(_bits(vpool, act)), up(perm), up(seq), \
        up(pos)
    po = alloc(2 * rows * H * D)
    wk.check(dev.wk_attention_decode(po, pq, pk, pv, pb, perm.shape[1], ps, pp, rows, max_len, H, Hk, D, act))
    raw = down(po, (rows, H * D), np.float16 if act == wk.F16 else np.uint16)
    free(pq, pk, pv, pb, ps, pp, po)
    return _from(raw, act)


CASES = [
    # rows, H, Hk, D, positions, max_len, act
    (1, 32, 8, 64, [383], 512, wk.F16),            # Llama-3.2-1B decode, 384-token context
    (1, 32, 8, 64, [0], 512, wk.F16),              # a one-token context
    (2, 32, 8, 64, [64, 127], 130, wk.F16),        # crossing / ending a page; max_len not a page multiple
    (1, 32, 8, 128, [2047], 2048, wk.F16),         # Llama-3.1-8B at 2048 (16 CTAs per pair)
    (1, 4, 1, 128, [2047], 2048, wk.F16),          # its tensor-parallel slice over 8 ranks
    (2, 64, 8, 128, [4095, 3000], 4096, wk.F16),   # Llama-3.1-70B widths (8 query heads per KV head)
    (32, 32, 8, 64, list(range(100, 1024, 29))[:32], 1024, wk.F16),  # 256 pairs: clusters in waves
    (3, 16, 2, 128, [5, 700, 1999], 2048, wk.BF16),
]


@pytest.mark.parametrize("rows,H,Hk,D,positions,max_len,act", CASES)
def test_decode_attention_vs_oracle(dev, monkeypatch, rows, H, Hk, D, positions, max_len, act):
    q, kpool, vpool, perm = _case(rows, H, Hk, D, positions, max_len, act, seed=rows * 7 + D + H)
    want = orc.decode_attention(q, kpool, vpool, perm, np.arange(rows), positions, H, Hk, D, act)
    monkeypatch.delenv("WUKONG_CLUSTER_ATTN", raising=False)
    monkeypatch.delenv("WUKONG_SPLIT_ATTN", raising=False)
    got = _run(dev, q, kpool, vpool, perm, positions, H, Hk, D, max_len, act)
    monkeypatch.setenv("WUKONG_CLUSTER_ATTN", "0")
    one = _run(dev, q, kpool, vpool, perm, positions, H, Hk, D, max_len, act)
    assert np.isfinite(got).all() and np.isfinite(one).all()
    tol = 1e-3 if act == wk.F16 else 1e-2  # normwise relative error; bf16: one bf16 rounding step
    for name, x in (("cluster", got), ("one CTA", one)):
        nw = float(np.linalg.norm(x - want) / np.linalg.norm(want))
        mx = float(np.abs(x - want).max())
        print(f"{name}: normwise {nw:.2e}, max |diff| {mx:.2e}")
        assert nw <= tol and mx <= 10 * tol, (name, nw, mx)
    # the two kernels differ only in the fp32 order of the softmax sum and of P.V
    same = float(np.mean(got == one))
    print(f"cluster vs one CTA: {same:.4f} of the outputs identical, max |diff| {np.abs(got - one).max():.2e}")
    assert np.abs(got - one).max() <= 4 * tol
    assert same >= 0.9
