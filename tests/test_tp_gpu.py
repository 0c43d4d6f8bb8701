"""Tensor-parallel engine on 2 GPUs against the single-GPU engine.

Two child processes (one per GPU) shard a small Q8_0 Llama with
wukong_b200.tp, join one NCCL communicator through wk_tp_init and run prefill
(tcgen05 GEMM path, 48 rows) and greedy decode steps (GEMV path) with the
row-parallel partial sums, the fp32 all-reduce and the vocabulary-parallel
argmax exchange.  Their tokens must equal those of the unsharded engine on the
same weights.  A second test shards one layer at Llama-3.1-8B widths (head_dim
128, d 4096, FFN 14336, vocabulary 128256) and checks the ranks' tokens
against the CPU oracle, teacher-forced.  Skipped on a box with fewer than 2
GPUs.
"""
import ctypes
import os

import numpy as np
import pytest

import wukong_b200 as wk

pytestmark = pytest.mark.gpu
CFG = dict(L=2, d=512, H=8, Hk=4, D=64, F=1024, V=4096, eps=1e-5, theta=500000.0)
B, P, STEPS, CTX = 2, 24, 8, 64


def _model():
    from tests.model_util import make_weights
    return make_weights(CFG, wk.Q8_0, wk.Q8_0, wk.F16, seed=515, ctx=CTX)


def _run(engine_cfg, layers, w, tp):
    """Prefill + STEPS greedy steps; returns the tokens of each call."""
    from tests.gpu_util import down, up
    from wukong_b200.engine import Engine
    L = wk.lib()
    ptrs = [up(w["token_embd"]), up(w["output_norm"]), up(w["output"]), up(w["freqs"])]
    eng = Engine(engine_cfg, layers, ptrs[0], ptrs[1], ptrs[2], ptrs[3], CTX, max_batch=B, tp=tp)
    prompt = np.random.default_rng(3).integers(0, CFG["V"], size=(B, P)).astype(np.int32)
    dp = up(prompt)
    toks = []
    eng.prefill(dp, B, P)
    toks.append(down(eng.tokens_ptr(), B, np.int32).tolist())
    for _ in range(STEPS):
        eng.step()
        toks.append(down(eng.tokens_ptr(), B, np.int32).tolist())
    eng.destroy()
    for p in ptrs + [dp]:
        L.cuda_free(p)
    return toks


def _worker(rank, world, uid, q, p2p):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["WUKONG_TP_P2P"] = p2p
    try:
        from tests.gpu_util import up
        from wukong_b200 import tp
        L = wk.lib()
        L.cuda_init(rank)
        wk.check(L.wk_tp_init(rank, world, uid))
        w = _model()
        layers = []
        for lw in w["layers"]:
            s = tp.shard_layer(lw, CFG, wk.Q8_0, rank, world)
            layers.append({k: up(v) for k, v in s.items()})
        wo = dict(w, output=tp.shard_output(w["output"], CFG, wk.Q8_0, rank, world))
        toks = _run(tp.local_config(CFG, world), layers, wo, tp=True)
        used = L.wk_tp_p2p()
        L.wk_tp_fini()
        q.put((rank, (toks, used)))
    except Exception as e:  # reported to the parent
        q.put((rank, f"{type(e).__name__}: {e}"))


@pytest.mark.parametrize("p2p", ["1", "0"])
def test_tp2_engine_matches_single_gpu(dev, p2p):
    """p2p=1: partials exchanged through peer memory in one fused launch;
    p2p=0: NCCL all-reduce and all-gather."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("tensor parallelism needs 2 GPUs")
    import torch.multiprocessing as mp
    from tests.gpu_util import up
    uid = ctypes.create_string_buffer(128)
    wk.check(dev.wk_tp_unique_id(uid))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, uid.raw, q, p2p)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        # poll, so that a child that dies without reporting fails the test at once
        import queue
        import time
        t0 = time.time()
        while len(got) < len(procs) and time.time() - t0 < 240:
            try:
                r, v = q.get(timeout=2)
                got[r] = v
            except queue.Empty:
                dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
                if dead and q.empty():
                    break
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    # the unsharded engine on the same weights, in this process (cuda:0)
    w = _model()
    from tests.model_util import fused_for_oracle
    layers = [{k: up(v) for k, v in lw.items()} for lw in fused_for_oracle(w)["layers"]]
    ref = _run(CFG, layers, w, tp=False)
    assert set(got) == {0, 1}, f"ranks reported {sorted(got)}; exit codes {[p.exitcode for p in procs]}"
    assert isinstance(got[0], tuple), got[0]
    assert isinstance(got[1], tuple), got[1]
    (t0, used0), (t1, used1) = got[0], got[1]
    assert used0 == used1 == int(p2p)
    assert t0 == t1
    assert t0 == ref


# ------------------------------------------------------------------ 8B widths vs the oracle
CFG8 = dict(L=1, d=4096, H=32, Hk=8, D=128, F=14336, V=128256, eps=1e-5, theta=500000.0)
B8, P8, STEPS8, CTX8 = 2, 40, 6, 64


def _model8():
    from tests.model_util import make_weights
    return make_weights(CFG8, wk.Q8_0, wk.Q8_0, wk.F16, seed=8080, ctx=CTX8)


def _worker8(rank, world, uid, q, prompt, forced):
    """Prefill, then one decode step per oracle token (teacher forcing)."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        from tests.gpu_util import down, up
        from wukong_b200 import tp
        from wukong_b200.engine import Engine
        L = wk.lib()
        L.cuda_init(rank)
        wk.check(L.wk_tp_init(rank, world, uid))
        w = _model8()
        layers = []
        for lw in w["layers"]:
            s = tp.shard_layer(lw, CFG8, wk.Q8_0, rank, world)
            layers.append({k: up(v) for k, v in s.items()})
        out = up(tp.shard_output(w["output"], CFG8, wk.Q8_0, rank, world))
        ptrs = [up(w["token_embd"]), up(w["output_norm"]), up(w["freqs"])]
        eng = Engine(tp.local_config(CFG8, world), layers, ptrs[0], ptrs[1], out, ptrs[2], CTX8, max_batch=B8,
                     tp=True)
        dp = up(prompt)
        eng.prefill(dp, B8, P8)
        toks = [down(eng.tokens_ptr(), B8, np.int32).tolist()]
        for f in forced:
            fa = np.ascontiguousarray(f, np.int32)
            L.cuda_to_device(L.wk_model_next_ids(eng.m), fa.ctypes.data_as(ctypes.c_void_p), 4 * B8)
            eng.step()
            toks.append(down(eng.tokens_ptr(), B8, np.int32).tolist())
        eng.destroy()
        L.wk_tp_fini()
        q.put((rank, toks))
    except Exception as e:  # reported to the parent
        q.put((rank, f"{type(e).__name__}: {e}"))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_8b_widths_vs_oracle(dev, world):
    """One Llama-3.1-8B-width layer sharded over 2, 4 or 8 ranks (one per GPU;
    skipped when the box has fewer), teacher-forced against the oracle."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import queue
    import time
    import torch.multiprocessing as mp
    from tests.model_util import oracle_model
    w = _model8()
    prompt = np.random.default_rng(88).integers(0, CFG8["V"], size=(B8, P8)).astype(np.int32)
    om = oracle_model(w, CFG8, wk.Q8_0, wk.Q8_0, wk.F16, CTX8)
    om.reset(B8)
    tok, logits, _ = om.forward(prompt)
    ref, lgs = [tok.tolist()], [logits]
    for _ in range(STEPS8):
        tok, logits, _ = om.forward(tok.reshape(B8, 1))
        ref.append(tok.tolist())
        lgs.append(logits)
    uid = ctypes.create_string_buffer(128)
    wk.check(dev.wk_tp_unique_id(uid))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker8, args=(r, world, uid.raw, q, prompt, ref[:-1])) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        t0 = time.time()
        while len(got) < world and time.time() - t0 < 300:
            try:
                r, v = q.get(timeout=2)
                got[r] = v
            except queue.Empty:
                if any(p.exitcode not in (None, 0) for p in procs) and q.empty():
                    break
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert set(got) == set(range(world)), f"ranks reported {sorted(got)}; exit codes {[p.exitcode for p in procs]}"
    assert isinstance(got[0], list), got[0]
    assert all(got[r] == got[0] for r in range(world))
    ties = []
    for s, (g, r, lg) in enumerate(zip(got[0], ref, lgs)):
        for b in range(B8):
            if g[b] != r[b]:
                scale = float(np.abs(lg[b]).max())
                mg = abs(float(lg[b][g[b]]) - float(lg[b][r[b]]))
                assert mg <= 2 * 2.0 ** -10 * scale, (s, b, g[b], r[b], mg)
                ties.append((s, b, mg))
    assert len(ties) <= 1, ties
