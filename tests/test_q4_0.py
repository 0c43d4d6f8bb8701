"""GGUF Q4_0 weights (one of the dtype-table types the reference lists but
does not implement, cuda.cu:5-42 / :1006-1012): the oracle's restatement of
ggml's published Q4_0 rule pinned by a hand-computed block, and the library's
dequantise, embedding, decode GEMV and engine against it."""
import ctypes

import numpy as np
import pytest

import wukong_b200 as wk
from oracle import oracle as orc


def test_q4_0_known_block():
    """x_i = (i - 16) / 8: the largest magnitude is x_0 = -2, so d = -2 / -8 =
    0.25 and nibble_i = min(15, (int)(4 x_i + 8.5)); byte i holds x_i low and
    x_{i+16} high."""
    x = ((np.arange(32) - 16) / 8.0).astype(np.float32)
    blk = orc.quantize_q4_0(x, 1, 32)
    assert blk[:2].view(np.float16)[0] == np.float16(0.25)
    nib = [min(15, int(4 * v + 8.5)) for v in x]
    assert blk[2:].tolist() == [nib[i] | (nib[i + 16] << 4) for i in range(16)]
    deq = orc.dequant_q4_0(blk, 1, 32)[0]
    assert deq.tolist() == [(n - 8) * 0.25 for n in nib]
    # every value within half a step of its input, except the clamped top
    assert np.all(np.abs(deq[:31] - x[:31]) <= 0.125)


def test_q4_0_generator_quantises_its_normals():
    rows, cols = 4, 256
    q = orc.gen_q4_0(rows, cols, 7, 0.02)
    deq = orc.dequant_q4_0(q, rows, cols)
    ref = orc.gen_normal(rows * cols, 7, 0.02)  # the same counter-based samples
    assert q.size == rows * cols // 32 * 18
    d = np.abs(q.reshape(-1, 18)[:, :2].copy().view(np.float16).astype(np.float32)).repeat(32)
    # half a step, or one step for the value clamped at nibble 15, plus the fp16 rounding of d
    assert np.all(np.abs(deq.ravel() - ref) <= d * 1.01 + 1e-6)


@pytest.mark.gpu
def test_q4_0_device_generator_and_dequantise_bit_exact(dev):
    from tests.gpu_util import alloc, down, free
    rows, cols = 300, 2048
    p = alloc(rows * cols // 32 * 18)
    wk.check(dev.wk_fill_random_q4_0(p, rows, cols, 123, 0.02))
    got = down(p, rows * cols // 32 * 18, np.uint8)
    want = orc.gen_q4_0(rows, cols, 123, 0.02)
    bad = np.flatnonzero(got != want)
    assert bad.size == 0, (bad.size, bad[:8].tolist(), got[bad[:8]].tolist(), want[bad[:8]].tolist())
    o = alloc(4 * rows * cols)
    dev.cuda_dequantize(o, p, rows, cols, wk.Q4_0)
    assert np.array_equal(down(o, (rows, cols), np.float32), orc.dequant_q4_0(want, rows, cols))
    free(p, o)


@pytest.mark.gpu
@pytest.mark.parametrize("N,K,M", [(8192, 2048, 1), (3072, 2048, 3), (2048, 8192, 8), (4096, 4096, 37), (1000, 2080, 2)])
def test_q4_0_matmul_vs_oracle(dev, N, K, M):
    """cuda_matmul with Q4_0 weights: the decode GEMV (TMA tiles of 8 blocks
    when a row is a multiple of 16 bytes, K % 256 == 0; plain copies
    otherwise), 8-row passes above 8 rows."""
    from tests.gpu_util import alloc, down, free, h16, rel_err, up
    w = orc.gen_q4_0(N, K, 5 + M, 0.02)
    x = orc.gen_normal(M * K, 9, 1.0).reshape(M, K)
    pw, px, po = up(w), up(h16(x)), alloc(2 * M * N)
    dev.cuda_matmul(po, px, pw, None, M, K, N, wk.Q4_0)
    got = down(po, (M, N), np.float16).astype(np.float32)
    want = orc.matmul(h16(x).astype(np.float32), w, None, M, K, N, wk.Q4_0, wk.F16)
    free(pw, px, po)
    assert rel_err(got, want) <= 1e-3


@pytest.mark.gpu
def test_q4_0_embedding(dev):
    from tests.gpu_util import alloc, down, free, up
    V, d = 1000, 512
    tab = orc.gen_q4_0(V, d, 44, 1.0)
    ids = np.array([0, 999, 17, 17, 500], np.int32)
    pt, pi, po = up(tab), up(ids), alloc(2 * ids.size * d)
    dev.cuda_embedding(po, pi, pt, 1, ids.size, d, wk.Q4_0)
    got = down(po, (ids.size, d), np.float16).astype(np.float32)
    free(pt, pi, po)
    assert np.array_equal(got, orc.embedding(ids, tab, d, wk.Q4_0))


@pytest.mark.gpu
def test_q4_0_engine_decode_vs_oracle(dev):
    """A 2-layer Llama-3.2-1B-width model with Q4_0 linear and output weights:
    prefill on 8-row GEMV passes, decode steps on the Q4_0 GEMV,
    teacher-forced against the oracle (near-ties reported as in the Q8_0 tests)."""
    from tests.model_util import LLAMA_1B, DeviceModel, build_engine, make_weights, oracle_model
    from tests.test_parity_gpu import teacher_forced
    cfg = dict(LLAMA_1B, L=2)
    ctx = 40
    w = make_weights(cfg, wk.Q4_0, wk.Q4_0, wk.F16, seed=404, ctx=ctx)
    dm = DeviceModel(w)
    m = build_engine(dm, w, cfg, wk.Q4_0, wk.Q4_0, wk.F16, max_batch=2, ctx=ctx)
    om = oracle_model(w, cfg, wk.Q4_0, wk.Q4_0, wk.F16, ctx)
    om.reset(2)
    ids = np.random.default_rng(4).integers(0, cfg["V"], size=(2, 20)).astype(np.int32)
    ties = teacher_forced(m, om, ids, 8)
    dev.wk_model_destroy(m)
    dm.free()
    assert len(ties) <= 2
