"""Per-launch timeline of the engine's decode step (diagnostic).

Loads libwukong_timeline.so (``python -m wukong_b200.build --timeline``), runs
greedy decode on a synthetic Llama model and prints, per kind of launch, where
its time goes (means over CTAs and launches, in microseconds):

  gap     end of the previous recorded launch's last CTA -> first CTA past its
          griddepcontrol.wait (the dependency hand-over)
  active  first CTA past the wait -> last CTA done
  tail    first CTA done -> last CTA done
  head    first CTA started -> first CTA past the wait (prefetch time it had)
  phases  per CTA, from the first wait return: GEMV p0 activations staged,
          p1 first weight unit landed, p2 first unit consumed, p3 first tile
          stored, p4 all tiles, p5 attention run by the q|k|v GEMV; decode
          attention p0 q staged, p1 scores, p2 softmax, p3 P.V; split-K
          attention scores p0 own scores, p1 row staged (last CTA), p2
          normaliser; P.V p0 P, p1 partial, p2 combined (last CTA);
          end = the CTA's last stamp.  N / K columns: the GEMV's shape;
          attention pages and query heads per KV head (split: pages, splits)

Usage: python -m wukong_b200.timeline [--model 1b|8b|70b] [--steps N] [--prompt P] [--batch B]
           [--shard N]  (rank 0's slice of an N-way split on this GPU alone, no exchanges)
       python -m torch.distributed.run --nproc-per-node N -m wukong_b200.timeline --model 8b
           (tensor-parallel over N GPUs; all-reduce+resid p5: first tile published)
"""
import argparse
import ctypes
import os
import sys

import numpy as np

SLOTS, BLOCKS, STAMPS = 1024, 320, 9
KINDS = {0: "store", 1: "resid", 2: "qkv", 3: "swiglu", 4: "logits", 5: "partial", 6: "all-reduce+resid",
         100: "attention",
         101: "attention scores (split)", 102: "attention P.V (split)", 103: "attention (split, one launch)",
         104: "attention (cluster)"}


def record(model="1b", steps=12, prompt=None, batch=1, shard=1):
    """Under torch.distributed.run with more than one rank the model is
    tensor-parallel over the ranks (one per GPU); every rank records its own
    launches.  shard > 1 (one process): rank 0's slice of a model split over
    `shard` ranks, run on this GPU alone without the exchanges (the per-rank
    compute of tensor-parallel decode)."""
    import wukong_b200 as wk
    wk.LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libwukong_timeline.so")
    from wukong_b200.engine import LLAMA, Engine, SyntheticLlama
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    L = wk.lib()
    L.cuda_init(int(os.environ.get("LOCAL_RANK", "0")))
    if world > 1:
        import torch
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        torch.distributed.init_process_group("gloo")
        idbuf = ctypes.create_string_buffer(128)
        if rank == 0:
            wk.check(L.wk_tp_unique_id(idbuf))
        t = torch.frombuffer(bytearray(idbuf.raw), dtype=torch.uint8)
        torch.distributed.broadcast(t, 0)
        wk.check(L.wk_tp_init(rank, world, bytes(t.numpy())))
    cfg = dict(LLAMA[model])
    P = prompt or {"1b": 128, "8b": 2048, "70b": 4096}[model]
    sm = SyntheticLlama(cfg, P + steps + 16, seed=1234, tp_rank=rank, tp_world=world if world > 1 else shard)
    eng = Engine.from_synthetic(sm, max_batch=batch, tp=world > 1)
    # token ids within the engine's vocabulary (a one-process shard has the rank's slice of it)
    vocab = cfg["V"] if world > 1 else sm.local["V"]
    ids = np.random.default_rng(7).integers(0, vocab, size=(batch, P)).astype(np.int32)
    d = L.cuda_malloc(ids.nbytes)
    L.cuda_to_device(d, ids.ctypes.data_as(ctypes.c_void_p), ids.nbytes)
    eng.prefill(d, batch, P)
    for _ in range(3):
        eng.step()
    wk.check(L.wk_timeline_init(SLOTS, BLOCKS))
    for _ in range(steps):
        eng.step()
    info = np.zeros((SLOTS, 4), np.int32)
    stamps = np.zeros((SLOTS, BLOCKS, STAMPS), np.uint64)
    n = L.wk_timeline_read(info.ctypes.data_as(ctypes.c_void_p), stamps.ctypes.data_as(ctypes.c_void_p))
    if n < 0:
        raise RuntimeError(L.wk_last_error().decode())
    res = L.wk_timeline_resolution_ns()
    lps = eng.launches_per_step()
    eng.destroy()
    L.cuda_free(d)
    if world > 1:
        L.wk_tp_fini()
    return info, stamps.astype(np.int64), n, res, lps


def summarize(info, stamps, n):
    """Per kind of launch (kind, N, K): [gap, active, tail, head, p0..p5, end] in ns."""
    n = min(n, SLOTS)
    ev = []
    for s in range(n):
        kind, N, K, grid = (int(v) for v in info[s])
        g = min(grid, BLOCKS)
        t = stamps[s, :g]
        if grid == 0 or (t[:, 2] == 0).any():
            continue
        ev.append(dict(kind=kind, N=N, K=K, grid=grid, t=t))
    ev.sort(key=lambda e: e["t"][:, 1].min())
    rows = {}
    for i in range(1, len(ev)):
        e, p = ev[i], ev[i - 1]
        t = e["t"]
        t1 = t[:, 1].min()
        ph = np.where(t[:, 3:] > 0, t[:, 3:] - t1, np.nan).astype(float)
        cnt = np.isfinite(ph).sum(0)
        phm = np.where(cnt > 0, np.nansum(np.nan_to_num(ph, nan=0.0), 0) / np.maximum(cnt, 1), np.nan)
        key = (KINDS.get(e["kind"], str(e["kind"])), e["N"], e["K"])
        r = rows.setdefault(key, dict(n=0, grid=e["grid"], v=[]))
        r["n"] += 1
        r["v"].append(np.concatenate([
            [t1 - p["t"][:, 2].max(), t[:, 2].max() - t1, t[:, 2].max() - t[:, 2].min(), t1 - t[:, 0].min()],
            phm, [(t[:, 2] - t1).mean()]]))
    span = ev[-1]["t"][:, 2].max() - ev[0]["t"][:, 1].min() if ev else 0
    return rows, span / 1e3, len(ev)


def _mean(vs):
    a = np.array(vs, dtype=float)
    cnt = np.isfinite(a).sum(0)
    return np.where(cnt > 0, np.nansum(np.nan_to_num(a, nan=0.0), 0) / np.maximum(cnt, 1), np.nan)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", default="1b", choices=["1b", "8b", "70b"])
    ap.add_argument("--steps", type=int, default=12)
    ap.add_argument("--prompt", type=int, default=None)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--shard", type=int, default=1,
                    help="one process: rank 0's slice of the model split over this many ranks, no exchanges")
    a = ap.parse_args(argv)
    info, stamps, n, res, lps = record(a.model, a.steps, a.prompt, a.batch, a.shard)
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    rows, span_us, nev = summarize(info, stamps, n)
    print(f"model {a.model}" + (f" (rank 0 of {a.shard}, no exchanges)" if a.shard > 1 else "") +
          f", batch {a.batch}: {nev} GEMV / attention launches recorded over {span_us:.1f} us ({a.steps} decode "
          f"steps of {lps} launches; %globaltimer step {res} ns)")
    print("| launch | N | K | CTAs | count | gap | active | tail | head | p0 | p1 | p2 | p3 | p4 | p5 | end |")
    print("|---|---|---|---|---|---|---|---|---|---|---|---|---|---|---|---|")
    tot = 0.0
    for key, r in sorted(rows.items(), key=lambda kv: -_mean(kv[1]["v"])[:2].sum() * kv[1]["n"]):
        m = _mean(r["v"]) / 1e3
        cells = " | ".join("%.2f" % x if np.isfinite(x) else "" for x in m)
        print(f"| {key[0]} | {key[1]} | {key[2]} | {r['grid']} | {r['n']} | {cells} |")
        tot += (m[0] + m[1]) * r["n"] / a.steps
    print(f"per step: gaps + active of the recorded launches = {tot:.1f} us")
    return 0


if __name__ == "__main__":
    sys.exit(main())
