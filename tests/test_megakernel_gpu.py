"""The persistent decode kernel (one cooperative launch per decode step, grid
barriers between phases) against the graph of per-op kernels.

Both paths run the same arithmetic unit for unit (same tile / chunk split over
warps, same dequantised mma.sync products, same RMSNorm, RoPE, attention and
argmax rounding points), so free-running greedy decoding must produce the
same tokens, step for step.  Shapes cover head_dim 64 and 128, batches 1..8,
a vocabulary that is not a multiple of the 16-row tile, and positions that
cross a KV page boundary.
"""
import ctypes

import numpy as np
import pytest

import wukong_b200 as wk
from tests.gpu_util import alloc, down, free, up
from tests.model_util import DeviceModel, build_engine, make_weights

pytestmark = pytest.mark.gpu


def _decode(monkeypatch, mk, dm, w, cfg, B, ctx, ids, steps):
    monkeypatch.setenv("WUKONG_MEGAKERNEL", mk)
    # the persistent kernel runs one CTA per (row, kv head); so does the reference path here
    monkeypatch.setenv("WUKONG_SPLIT_ATTN", "0")
    L = wk.lib()
    m = build_engine(dm, w, cfg, wk.Q8_0, wk.Q8_0, wk.F16, max_batch=B, ctx=ctx)
    pids, ptok = up(ids), alloc(4 * B)
    wk.check(L.wk_model_prefill(m, pids, B, ids.shape[1], ptok))
    toks = [down(ptok, B, np.int32).tolist()]
    for _ in range(steps):
        wk.check(L.wk_model_decode_step(m))
        toks.append(down(L.wk_model_tokens(m), B, np.int32).tolist())
    launches = L.wk_model_step_launches(m)
    L.wk_model_destroy(m)
    free(pids, ptok)
    return toks, launches


@pytest.mark.parametrize("D,B,F,V", [(64, 1, 1024, 2000), (64, 3, 1024, 2000), (64, 8, 1024, 2000),
                                     (128, 2, 1024, 3000), (64, 2, 8192, 65600)])
def test_persistent_decode_equals_graph_path(dev, monkeypatch, D, B, F, V):
    """V = 65600 (4100 tiles) reaches the warp-tile mode of the logits layer
    (>= 4096 tiles by default); the other layers split tiles over a CTA."""
    H, Hk = 8, 2
    cfg = dict(L=2, d=H * D, H=H, Hk=Hk, D=D, F=F, V=V, eps=1e-5, theta=500000.0)
    ctx, n, steps = 96, 40, 30  # positions 40..70 cross the 64-token page
    w = make_weights(cfg, wk.Q8_0, wk.Q8_0, wk.F16, seed=17 + D + B, ctx=ctx)
    dm = DeviceModel(w)
    ids = np.random.default_rng(B).integers(0, cfg["V"], size=(B, n)).astype(np.int32)
    ref, ref_launches = _decode(monkeypatch, "0", dm, w, cfg, B, ctx, ids, steps)
    got, launches = _decode(monkeypatch, "1", dm, w, cfg, B, ctx, ids, steps)
    dm.free()
    assert ref_launches > 1
    assert launches == 1, "the persistent kernel did not run"
    assert got == ref
