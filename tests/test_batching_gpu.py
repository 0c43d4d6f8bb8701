"""Continuous batching: sequences of different lengths join and leave the
decode batch (wk_model_add_seqs / wk_model_remove_seq) while it runs; every
sequence's tokens must be those of the oracle running that sequence alone
(teacher-forced with the engine's own tokens; a different token is allowed
only at an fp16 near-tie of the oracle's logits, and is counted)."""
import ctypes

import numpy as np
import pytest

import wukong_b200 as wk
from tests.gpu_util import down, free, up
from tests.model_util import LLAMA_1B, DeviceModel, build_engine, make_weights, oracle_model

pytestmark = pytest.mark.gpu


def near_tie(logits, a, b):
    return abs(float(logits[a]) - float(logits[b])) <= 2 * 2.0 ** -10 * float(np.abs(logits).max())


class Tracker:
    """One oracle per sequence, fed the engine's tokens."""

    def __init__(self, w, cfg, ctx):
        self.w, self.cfg, self.ctx = w, cfg, ctx
        self.seq = {}  # slot -> (oracle, expected next token, logits)
        self.ties = 0
        self.checked = 0

    def add(self, slot, prompt, first):
        om = oracle_model(self.w, self.cfg, wk.Q8_0, wk.Q8_0, wk.F16, self.ctx)
        om.reset(1)
        tok, logits, _ = om.forward(prompt.reshape(1, -1))
        self.check(int(tok[0]), logits[0], first)
        self.seq[slot] = [om, first]

    def check(self, want, logits, got):
        self.checked += 1
        if got != want:
            assert near_tie(logits, got, want), (got, want)
            self.ties += 1

    def step(self, slot, got):
        om, last = self.seq[slot]
        tok, logits, _ = om.forward(np.array([[last]], np.int32))
        self.check(int(tok[0]), logits[0], got)
        self.seq[slot][1] = got


def test_sequences_join_and_leave_the_decode_batch(dev):
    cfg = dict(LLAMA_1B, L=2)
    ctx, maxb = 80, 4
    w = make_weights(cfg, wk.Q8_0, wk.Q8_0, wk.F16, seed=77, ctx=ctx)
    dm = DeviceModel(w)
    m = build_engine(dm, w, cfg, wk.Q8_0, wk.Q8_0, wk.F16, max_batch=maxb, ctx=ctx)
    L = wk.lib()
    rng = np.random.default_rng(12)
    tr = Tracker(w, cfg, ctx)

    def rows():
        slots = np.zeros(maxb, np.int32)
        n = L.wk_model_rows(m, slots.ctypes.data_as(ctypes.c_void_p))
        return slots[:n].tolist()

    def add(lens):
        prompts = [rng.integers(0, cfg["V"], size=n).astype(np.int32) for n in lens]
        ids = up(np.concatenate(prompts))
        hl = np.array(lens, np.int32)
        slots = np.zeros(len(lens), np.int32)
        b0 = len(rows())
        wk.check(L.wk_model_add_seqs(m, ids, hl.ctypes.data_as(ctypes.c_void_p), len(lens),
                                     slots.ctypes.data_as(ctypes.c_void_p)))
        toks = down(L.wk_model_tokens(m), b0 + len(lens), np.int32)
        for i, sl in enumerate(slots.tolist()):
            tr.add(sl, prompts[i], int(toks[b0 + i]))
        free(ids)
        return slots.tolist()

    def steps(k):
        for _ in range(k):
            wk.check(L.wk_model_decode_step(m))
            r = rows()
            toks = down(L.wk_model_tokens(m), len(r), np.int32)
            for i, sl in enumerate(r):
                tr.step(sl, int(toks[i]))

    assert add([20, 7]) == [0, 1]
    steps(5)
    assert add([13]) == [2]
    steps(4)
    wk.check(L.wk_model_remove_seq(m, 0))
    del tr.seq[0]
    assert sorted(rows()) == [1, 2]
    steps(3)
    assert add([9, 30]) == [0, 3]  # the freed slot is reused
    steps(4)
    assert L.wk_model_remove_seq(m, 0) == 0 and L.wk_model_remove_seq(m, 0) != 0  # twice is an error
    steps(2)
    L.wk_model_destroy(m)
    dm.free()
    print(f"continuous batching: {tr.checked} tokens checked, {tr.ties} near-ties")
    assert tr.ties <= 1 + tr.checked // 20
