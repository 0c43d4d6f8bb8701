"""Failure detection of the tensor-parallel exchange, on one GPU and without a
GPU fault.

The exchange kernels wait (bounded) for the flag every peer publishes in its
own buffer.  wk_tp_exchange_selftest runs it on one GPU with the peers
emulated by local buffers: published, the exchange completes and its sum is
checked; unpublished (a lost rank), every CTA's wait runs out after
WUKONG_WAIT_LIMIT_MS, records code 40 in the device error word and returns, so
the context stays usable.  The host then learns of it (the reference ends the
process on errors, wukong.h:173-188): cuda_to_host ends the process with the
code, the engine refuses to launch further steps, and after wk_device_error(1)
the library works again.
"""
import json
import os
import subprocess
import sys

import pytest

import wukong_b200 as wk

pytestmark = pytest.mark.gpu

SCRIPT = r"""
import ctypes, json, os, sys, time
import numpy as np
sys.path.insert(0, sys.argv[1])
mode = sys.argv[2]
import wukong_b200 as wk
L = wk.lib()
L.cuda_init(0)
res = {"published": L.wk_tp_exchange_selftest(2, 1), "published4": L.wk_tp_exchange_selftest(4, 1)}
t0 = time.time()
res["lost"] = L.wk_tp_exchange_selftest(2, 0)
res["seconds"] = time.time() - t0
res["error_word"] = L.wk_device_error(0)
if mode == "abort":
    print(json.dumps(res), flush=True)
    buf = L.cuda_malloc(4)
    out = np.zeros(1, np.int32)
    L.cuda_to_host(out.ctypes.data_as(ctypes.c_void_p), buf, 4)  # ends the process
    print("cuda_to_host returned", flush=True)
    sys.exit(0)
# engine: refused while the error word is set, works again once it is cleared
from tests.gpu_util import alloc, up
from tests.model_util import DeviceModel, build_engine, make_weights
cfg = dict(L=1, d=256, H=8, Hk=2, D=32, F=512, V=1024, eps=1e-5, theta=500000.0)
w = make_weights(cfg, wk.Q8_0, wk.Q8_0, wk.F16, seed=3, ctx=32)
dm = DeviceModel(w)
m = build_engine(dm, w, cfg, wk.Q8_0, wk.Q8_0, wk.F16, max_batch=1, ctx=32)
ids = up(np.arange(1, 9, dtype=np.int32).reshape(1, 8))
tok = alloc(4)
res["refused"] = L.wk_model_prefill(m, ids, 1, 8, tok)
res["refused_msg"] = L.wk_last_error().decode()
res["cleared"] = L.wk_device_error(1)
res["after_clear"] = L.wk_model_prefill(m, ids, 1, 8, tok)
res["step"] = L.wk_model_decode_step(m)
res["error_word_end"] = L.wk_device_error(0)
L.wk_model_destroy(m)
dm.free()
L.cuda_fini()
print(json.dumps(res), flush=True)
"""


def _run(mode):
    env = dict(os.environ, WUKONG_WAIT_LIMIT_MS="50")
    return subprocess.run([sys.executable, "-c", SCRIPT, wk.ROOT, mode], capture_output=True, text=True, env=env,
                          timeout=300)


def _res(r):
    return json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][0])


def test_lost_peer_wait_runs_out_and_ends_the_process_at_cuda_to_host():
    r = _run("abort")
    res = _res(r)
    assert res["published"] == 0 and res["published4"] == 0, res
    assert res["lost"] == 40 and res["error_word"] == 40, res
    # every CTA gave up after the 50 ms limit, not after the default second
    assert 0.04 <= res["seconds"] < 0.9, res
    assert r.returncode != 0
    assert "cuda_to_host returned" not in r.stdout
    assert "code 40" in r.stderr, r.stderr[-2000:]


def test_engine_refuses_steps_until_the_error_is_cleared():
    r = _run("engine")
    assert r.returncode == 0, r.stderr[-2000:]
    res = _res(r)
    assert res["lost"] == 40
    assert res["refused"] == -1 and "code 40" in res["refused_msg"], res
    assert res["cleared"] == 40
    assert res["after_clear"] == 0 and res["step"] == 0 and res["error_word_end"] == 0, res


@pytest.mark.parametrize("world,N,K,M", [(2, 4096, 512, 1), (8, 4096, 1792, 3), (4, 2048, 2048, 8), (2, 8192, 256, 2)])
def test_fused_exchange_gemv_matches_its_partial_sums(dev, world, N, K, M):
    """The o / down GEMV of tensor-parallel decode with its all-reduce +
    residual epilogue, on one GPU with the other ranks emulated (their tiles
    already published): x = T(x + T(sum over ranks)) element for element."""
    assert dev.wk_device_error(1) == 0
    rc = dev.wk_tp_gemv_selftest(world, N, K, M)
    assert rc == 0, dev.wk_last_error().decode()
