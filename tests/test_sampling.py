"""Sampling beyond argmax (temperature, top-k, top-p): the CPU restatement of
the rule (oracle/) against an independent numpy statement and against its
own limits, and the CUDA sampler against the restatement on the same logits.
The reference has no sampling (cuda.cu:988 leaves it as a TODO); the rule is
the library's own (include/wukong_ext.h, wk_model_set_sampling)."""
import ctypes

import numpy as np
import pytest

import wukong_b200 as wk
from oracle import oracle as orc


def _mix64(z):
    M = (1 << 64) - 1
    z &= M
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
    return z ^ (z >> 31)


def _numpy_sample(x, temperature, top_k, top_p, seed, step, row):
    V = x.size
    K = min(top_k if 0 < top_k < 256 else 256, V)
    order = sorted(range(V), key=lambda i: (-float(x[i]), i))[:K]
    e = np.exp((x[order].astype(np.float64) - float(x[order[0]])) / temperature)
    c = np.cumsum(e)
    m = K
    if 0 < top_p < 1:
        m = int(np.argmax(c >= top_p * c[-1])) + 1
    h = _mix64(seed + 0x9E3779B97F4A7C15 * (step * 65536 + row + 1))
    u = (h >> 40) / 16777216.0 * c[m - 1]
    pick = next((i for i in range(m) if c[i] > u), m - 1)
    return order[pick], float(np.min(np.abs(c[:m] - u)) / c[m - 1])


def test_sampler_restatement_matches_numpy():
    rng = np.random.default_rng(0)
    x = rng.normal(0, 2, size=(24, 3000)).astype(np.float16).astype(np.float32)
    for (t, k, p) in [(1.0, 0, 1.0), (0.7, 40, 0.9), (1.3, 5, 0.0), (0.5, 300, 0.5)]:
        got, ud = orc.sample(x, t, k, p, 1234, 77)
        for r in range(x.shape[0]):
            want, dist = _numpy_sample(x[r], t, k, p, 1234, 77, r)
            if got[r] != want:
                assert dist < 1e-5, (t, k, p, r, got[r], want, dist)


def test_sampler_limits():
    x = np.zeros((3, 100), np.float32)
    x[0, 7] = x[0, 3] = 5.0       # tie: the smaller index first
    x[1, 42] = 1.0
    x[2, :] = np.linspace(0, 1, 100)
    got, _ = orc.sample(x, 1.0, 1, 1.0, 9, 0)  # top-k 1: the (smallest-index) maximum
    assert got.tolist() == [3, 42, 99]
    got, _ = orc.sample(x, 1.0, 0, 1e-6, 9, 0)  # a tiny top-p keeps one candidate
    assert got.tolist() == [3, 42, 99]


def test_sampler_distribution():
    """Over many steps the draws follow softmax(l / T) of the kept candidates."""
    l = np.array([2.0, 1.0, 0.5, 0.0, -1.0, -3.0], np.float32)
    T, n = 0.8, 20000
    x = np.tile(l, (n, 1))
    got, _ = orc.sample(x, T, 0, 1.0, 5, np.zeros(n, np.int64))  # rows differ by their row index
    p = np.exp(l / T) / np.exp(l / T).sum()
    freq = np.bincount(got, minlength=l.size) / n
    assert np.abs(freq - p).max() < 0.015, (freq, p)
    # top-p 0.6 keeps the shortest prefix reaching 60 %: here the two best
    got, _ = orc.sample(x, T, 0, 0.6, 5, np.zeros(n, np.int64))
    assert set(np.unique(got)) <= {0, 1}


@pytest.mark.gpu
@pytest.mark.parametrize("t,k,p", [(1.0, 0, 1.0), (0.7, 40, 0.9), (1.5, 8, 0.0), (0.3, 256, 0.95), (1.0, 1, 1.0)])
def test_cuda_sampler_matches_restatement(dev, t, k, p):
    """wk_sample_logits on fp16 logits rows of the Llama-3 vocabulary: the same
    token as the restatement, except where u lies within 1e-5 of a prefix-sum
    boundary (expf of the two sides may differ in the last bit)."""
    from tests.gpu_util import alloc, down, free, up
    rows, V = 6, 128256
    x = (np.random.default_rng(int(t * 10) + k).normal(0, 3, size=(rows, V))).astype(np.float16)
    px, pt = up(x), alloc(4 * rows)
    wk.check(dev.wk_sample_logits(pt, px, rows, V, wk.F16, t, k, p, 4321, 17))
    got = down(pt, rows, np.int32)
    want, ud = orc.sample(x.astype(np.float32), t, k, p, 4321, 17)
    free(px, pt)
    for r in range(rows):
        if got[r] != want[r]:
            assert ud[r, 1] < 1e-5, (r, got[r], want[r], ud[r])


@pytest.mark.gpu
def test_engine_sampling_vs_oracle(dev):
    """The engine with sampling on (prefill + decode steps feeding the drawn
    token back on the device) against the oracle run on the engine's tokens:
    the same draw wherever the oracle's u is not within 1e-2 of a prefix-sum
    boundary (the two sides' logits differ by fp32 summation order, which moves
    the prefix sums by up to ~1e-2); the engine's draw equals the rule applied
    to the engine's own logits; the same seed reproduces the tokens, another
    seed changes them."""
    from tests.gpu_util import alloc, down, free, up
    from tests.model_util import LLAMA_1B, DeviceModel, build_engine, make_weights, oracle_model
    cfg = dict(LLAMA_1B, L=2)
    n, steps, ctx = 24, 12, 48
    T, K, P, SEED = 0.9, 50, 0.95, 11
    w = make_weights(cfg, wk.Q8_0, wk.Q8_0, wk.F16, seed=31, ctx=ctx)
    dm = DeviceModel(w)
    ids = np.random.default_rng(2).integers(0, cfg["V"], size=(1, n)).astype(np.int32)

    def run(seed):
        m = build_engine(dm, w, cfg, wk.Q8_0, wk.Q8_0, wk.F16, max_batch=1, ctx=ctx)
        wk.check(dev.wk_model_set_sampling(m, T, K, P, seed))
        pids, ptok = up(ids), alloc(4)
        wk.check(dev.wk_model_prefill(m, pids, 1, n, ptok))
        toks = [int(down(ptok, 1, np.int32)[0])]
        lg = [down(dev.wk_model_logits(m), (1, cfg["V"]), np.float16).astype(np.float32)]
        for _ in range(steps):
            wk.check(dev.wk_model_decode_step(m))
            toks.append(int(down(dev.wk_model_tokens(m), 1, np.int32)[0]))
            lg.append(down(dev.wk_model_logits(m), (1, cfg["V"]), np.float16).astype(np.float32))
        dev.wk_model_destroy(m)
        free(pids, ptok)
        return toks, lg

    (a, la), (b, _), (c, _) = run(SEED), run(SEED), run(SEED + 1)
    assert a == b
    assert a != c
    # the draw inside the engine is the sampling rule applied to the engine's own logits
    for s, (tok, lg) in enumerate(zip(a, la)):
        want, ud = orc.sample(lg, T, K, P, SEED, n - 1 + s)
        if tok != want[0]:
            assert ud[0, 1] < 1e-5, (s, tok, want[0], ud[0])
    # against the oracle's logits for the same inputs: every drawn token is among
    # the oracle's best K (+ a margin for order changes at the K-th place), and
    # the draw is the same wherever u is far from a prefix-sum boundary
    om = oracle_model(w, cfg, wk.Q8_0, wk.Q8_0, wk.F16, ctx)
    om.reset(1)
    _, logits, _ = om.forward(ids)
    for s, tok in enumerate(a):
        want, ud = orc.sample(logits, T, K, P, SEED, n - 1 + s)
        assert tok in np.argsort(-logits[0], kind="stable")[:K + 5], (s, tok)
        if ud[0, 1] > 1e-2:
            assert tok == want[0], (s, tok, want[0], ud[0])
        _, logits, _ = om.forward(np.array([[tok]], np.int32))
    dm.free()
