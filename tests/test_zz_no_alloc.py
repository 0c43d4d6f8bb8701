"""wk_predict_noalloc: cuda_predict without device allocation.

Some hosts cannot call cudaMalloc when they predict: a serving process that has
given all free HBM to its own KV-cache pool, or a latency-critical loop in
which cudaMalloc / cudaFree would synchronise the device.  wk_predict_noalloc
runs the same fused logits + argmax kernel as cuda_predict with its scratch in
a fixed array inside the library, so its token ids must equal cuda_predict's
exactly.  Two calls in a row, with different shapes, weight types and pass
counts, check that the leftover contents of the shared array do not leak from
one call into the next.

This file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

import wukong_b200 as wk
from oracle import oracle as orc
from tests.gpu_util import alloc, bf16_bits, down, free, h16, up

pytestmark = pytest.mark.gpu
F32, F16, Q8_0, BF16 = wk.F32, wk.F16, wk.Q8_0, wk.BF16
EPS = 1e-5
MAX_BATCH = 64


def _case(wtype, B, Tn, d, V, seed):
    if wtype == Q8_0:
        w = orc.gen_q8_0(V, d, seed)
    else:
        g = orc.gen_normal(V * d, seed, 0.02)
        w = h16(g) if wtype == F16 else bf16_bits(g)
    nw = (1.0 + orc.gen_normal(d, seed + 1, 0.1)).astype(np.float32)
    x = orc.gen_normal(B * Tn * d, seed + 2, 1.0)
    xd = bf16_bits(x) if wtype == BF16 else h16(x)
    return dict(wtype=wtype, B=B, Tn=Tn, d=d, V=V, p=[up(w), up(nw), up(xd)])


def _noalloc(dev, c, out):
    pw, pn, px = c["p"]
    rc = dev.wk_predict_noalloc(out, px, pn, pw, c["B"], c["Tn"], c["d"], c["V"], EPS, c["wtype"])
    assert rc == 0, dev.wk_last_error().decode()


def _existing(dev, c, out):
    pw, pn, px = c["p"]
    dev.cuda_predict(out, px, pn, pw, c["B"], c["Tn"], c["d"], c["V"], EPS, c["wtype"])


def test_noalloc_predict_matches_cuda_predict(dev):
    """Token ids equal cuda_predict's (same kernel, exact) on two calls in a row."""
    first = _case(Q8_0, B=5, Tn=3, d=2048, V=128256, seed=501)    # one 5-row pass
    second = _case(F16, B=19, Tn=2, d=1024, V=32000, seed=601)    # three passes, the last ragged
    o1, o2, r1, r2 = alloc(4 * first["B"]), alloc(4 * second["B"]), alloc(4 * first["B"]), alloc(4 * second["B"])
    _noalloc(dev, first, o1)
    _noalloc(dev, second, o2)
    _existing(dev, first, r1)
    _existing(dev, second, r2)
    got1, got2 = down(o1, first["B"], np.int32), down(o2, second["B"], np.int32)
    assert got1.tolist() == down(r1, first["B"], np.int32).tolist()
    assert got2.tolist() == down(r2, second["B"], np.int32).tolist()
    assert (got1 >= 0).all() and (got1 < first["V"]).all()
    assert (got2 >= 0).all() and (got2 < second["V"]).all()
    # the first shape again, after the second left its partials in the array
    _noalloc(dev, first, o1)
    assert down(o1, first["B"], np.int32).tolist() == got1.tolist()
    free(o1, o2, r1, r2, *first["p"], *second["p"])


def test_noalloc_predict_full_batch_bf16(dev):
    """The largest batch the static scratch holds (64 sequences, 8 passes)."""
    c = _case(BF16, B=MAX_BATCH, Tn=1, d=512, V=4096, seed=701)
    o, r = alloc(4 * MAX_BATCH), alloc(4 * MAX_BATCH)
    _noalloc(dev, c, o)
    _existing(dev, c, r)
    assert down(o, MAX_BATCH, np.int32).tolist() == down(r, MAX_BATCH, np.int32).tolist()
    free(o, r, *c["p"])


def test_noalloc_predict_rejects_sizes_beyond_its_scratch(dev):
    """Oversized or unsupported calls return -1 with a message and launch nothing."""
    p = alloc(4096)
    for args, words in [((MAX_BATCH + 1, 1, 512, 100, Q8_0), "batch 65"),
                        ((0, 1, 512, 100, Q8_0), "batch 0"),
                        ((1, 1, 32800, 100, Q8_0), "col 32800"),
                        ((1, 1, 500, 100, Q8_0), "col 500"),
                        ((1, 1, 512, 100, F32), "dtype 0")]:
        B, Tn, d, V, wt = args
        assert dev.wk_predict_noalloc(p, p, p, p, B, Tn, d, V, EPS, wt) == -1
        assert words in dev.wk_last_error().decode()
    free(p)


def _driver_memory():
    """(free device bytes, bytes in use in the device's default stream-ordered
    pool) through the CUDA driver, on the context the library made current."""
    cu = ctypes.CDLL("libcuda.so.1")
    free_b, total_b = ctypes.c_size_t(), ctypes.c_size_t()
    assert cu.cuMemGetInfo_v2(ctypes.byref(free_b), ctypes.byref(total_b)) == 0
    pool, used = ctypes.c_void_p(), ctypes.c_uint64()
    assert cu.cuDeviceGetDefaultMemPool(ctypes.byref(pool), 0) == 0
    CU_MEMPOOL_ATTR_USED_MEM_CURRENT = 7
    assert cu.cuMemPoolGetAttribute(pool, CU_MEMPOOL_ATTR_USED_MEM_CURRENT, ctypes.byref(used)) == 0
    return free_b.value, used.value


def test_noalloc_predict_allocates_nothing(dev):
    """After one call of each shape (which may load the kernels' code onto the
    device), further calls of both shapes leave the device's free memory and
    the default stream-ordered pool's usage unchanged."""
    first = _case(Q8_0, B=3, Tn=2, d=2048, V=32000, seed=801)     # one pass
    second = _case(F16, B=40, Tn=1, d=1024, V=8192, seed=901)     # five passes
    o1, o2 = alloc(4 * first["B"]), alloc(4 * second["B"])
    _noalloc(dev, first, o1)
    _noalloc(dev, second, o2)
    assert dev.wk_device_error(0) == 0  # synchronises the library stream
    before = _driver_memory()
    for _ in range(3):
        _noalloc(dev, first, o1)
        _noalloc(dev, second, o2)
    got = down(o2, second["B"], np.int32)  # synchronises
    assert _driver_memory() == before
    assert (got >= 0).all() and (got < second["V"]).all()
    free(o1, o2, *first["p"], *second["p"])
