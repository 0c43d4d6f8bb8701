"""Tensor-parallel decomposition on the CPU: two gloo ranks shard a small
Q8_0 Llama layer with wukong_b200.tp, compute their shares with the oracle and
exchange them the way the GPU engine does (fp32 all-reduce of the o / down
partials, all-gather of one logits winner per row); the result must equal the
single-rank oracle.  This covers the host logic of the N > 1 path (byte-level
sharding of GGUF rows / K-blocks, the rounding order after the all-reduce, the
winner exchange in the reference argmax's tie order) without a GPU.
"""
import os
import socket

import numpy as np
import pytest

CFG = dict(L=1, d=256, H=4, Hk=2, D=64, F=512, V=1000, eps=1e-5, theta=500000.0)
B = 3
PACK = 8  # half logits: 16-byte loads of 8 values (cuda.cu:480-531)


def _brev5(v):
    return int(f"{v:05b}"[::-1], 2)


def logits_key(idx, pack=PACK):
    """Order key of element idx in the reference argmax (smaller wins a tie)."""
    p = idx // pack
    tid, j, e = p & 255, p >> 8, idx - p * pack
    return (_brev5(tid >> 5) << 58) | (_brev5(tid & 31) << 53) | (j << 8) | e


def winner(row, col0, n_total, pack=PACK):
    """(value, key) of the best element of a logits shard starting at column col0."""
    lim = n_total // pack * pack
    best = (-np.inf, None)
    for i, v in enumerate(row):
        g = col0 + i
        if g >= lim:
            continue
        k = logits_key(g, pack)
        if best[1] is None or v > best[0] or (v == best[0] and k < best[1]):
            best = (float(v), k)
    return best


def _index_of(key, pack=PACK):
    bw, bl = (key >> 58) & 31, (key >> 53) & 31
    tid = (_brev5(bw) << 5) | _brev5(bl)
    j = (key >> 8) & ((1 << 45) - 1)
    return ((j << 8) + tid) * pack + (key & 255)


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from oracle import oracle as orc
        from tests.model_util import make_weights
        from wukong_b200 import tp
        Q8, F16, F32 = orc.Q8_0, orc.F16, orc.F32
        d, H, Hk, D, F, V = CFG["d"], CFG["H"], CFG["Hk"], CFG["D"], CFG["F"], CFG["V"] * 2
        cfg = dict(CFG, V=V)
        tp.check_divisible(cfg, world, Q8)
        w = make_weights(cfg, Q8, Q8, F16, seed=31, ctx=64)
        lw = w["layers"][0]
        s = tp.shard_layer(lw, cfg, Q8, rank, world)
        h, hk, f, v = H // world, Hk // world, F // world, V // world

        def rnd16(a):
            return a.astype(np.float16).astype(np.float32)

        x = rnd16(orc.gen_normal(B * d, 5, 1.0).reshape(B, d))
        xn = orc.rmsnorm(x, lw["attn_norm"], B, d, CFG["eps"], F16)
        # column-parallel q|k|v: this rank's rows of the full product, exactly
        W = (H + 2 * Hk) * D
        full = orc.matmul(xn, np.concatenate([lw["q"], lw["k"], lw["v"]]), None, B, d, W, Q8, F32)
        loc = orc.matmul(xn, s["qkv"], None, B, d, (h + 2 * hk) * D, Q8, F32)
        rows = np.r_[rank * h * D:(rank + 1) * h * D, H * D + rank * hk * D:H * D + (rank + 1) * hk * D,
                     (H + Hk) * D + rank * hk * D:(H + Hk) * D + (rank + 1) * hk * D]
        assert np.array_equal(loc, full[:, rows]), "qkv shard"
        # row-parallel o: fp32 partials, all-reduce, one rounding (as one GEMM up to the sum order)
        att = rnd16(orc.gen_normal(B * H * D, 6, 1.0).reshape(B, H * D))
        part = orc.matmul(np.ascontiguousarray(att[:, rank * h * D:(rank + 1) * h * D]), s["o"], None, B, h * D, d,
                          Q8, F32)
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t)
        y = rnd16(t.numpy())
        ref = orc.matmul(att, lw["o"], None, B, H * D, d, Q8, F16)
        assert np.abs(y - ref).max() <= 1e-3 * np.abs(ref).max(), "o all-reduce"
        # FFN: local SwiGLU on the shard's up/gate rows, row-parallel down
        hf = orc.swiglu(orc.matmul(xn, np.concatenate([lw["up"], lw["gate"]]), None, B, d, 2 * F, Q8, F16), B, F, F16)
        hl = orc.swiglu(orc.matmul(xn, s["fc"], None, B, d, 2 * f, Q8, F16), B, f, F16)
        assert np.array_equal(hl, hf[:, rank * f:(rank + 1) * f]), "fc shard + swiglu"
        part = orc.matmul(hl, s["down"], None, B, f, d, Q8, F32)
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t)
        y = rnd16(t.numpy())
        ref = orc.matmul(hf, lw["down"], None, B, F, d, Q8, F16)
        assert np.abs(y - ref).max() <= 1e-3 * np.abs(ref).max(), "down all-reduce"
        # vocabulary-parallel logits + winner exchange == argmax of the whole row
        out_s = tp.shard_output(w["output"], cfg, Q8, rank, world)
        lg_full = orc.matmul(xn, w["output"], None, B, d, V, Q8, F16)
        lg = orc.matmul(xn, out_s, None, B, d, v, Q8, F16)
        assert np.array_equal(lg, lg_full[:, rank * v:(rank + 1) * v]), "output shard"
        mine = [winner(lg[b], rank * v, V) for b in range(B)]
        allw = [None] * world
        dist.all_gather_object(allw, mine)
        toks = []
        for b in range(B):
            best = None
            for r in range(world):
                val, key = allw[r][b]
                if key is None:
                    continue
                if best is None or val > best[0] or (val == best[0] and key < best[1]):
                    best = (val, key)
            toks.append(_index_of(best[1]))
        assert toks == orc.argmax(lg_full, B, V, PACK).tolist(), "winner exchange"
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q.put((rank, f"{type(e).__name__}: {e}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tp_decomposition_two_gloo_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results


def test_shard_bytes_and_errors():
    """K-slices of Q8_0 rows keep whole 34-byte blocks; uneven splits are refused."""
    from oracle import oracle as orc
    from wukong_b200 import tp
    w = orc.gen_q8_0(4, 128, 3)
    left = tp.col_slice(w, 4, 128, orc.Q8_0, 0, 64).reshape(4, 2 * 34)
    right = tp.col_slice(w, 4, 128, orc.Q8_0, 64, 128).reshape(4, 2 * 34)
    assert np.array_equal(np.concatenate([left, right], axis=1).reshape(-1), w)
    with pytest.raises(ValueError):
        tp.col_slice(w, 4, 128, orc.Q8_0, 0, 48)
    with pytest.raises(ValueError):
        tp.check_divisible(dict(CFG, V=1001), 2, orc.Q8_0)
