"""Benchmark: greedy decode tokens/s of Llama-3.2-1B with Q8_0 weights on B200.

Workload (default): Llama-3.2-1B architecture (16 layers, d 2048, 32/8 heads,
head_dim 64, SwiGLU 8192, vocab 128256, RoPE theta 500000, RMSNorm eps 1e-5),
random-init weights: linear layers and output.weight Q8_0 (w ~ N(0, 0.02)
quantised GGUF-style), token_embd F16, norms 1.0; batch 1 (--batch), a
128-token uniform-random prompt, then greedy decode.  A step is one decode step
(one token per sequence).  Weights per step (1.31 GB) exceed the 126 MB L2, so
no flush is needed between steps.

Arms
  (default)            the native engine (wukong_ext.h): CUDA-graph decode step,
                       inputs resident in HBM -> `value`; `e2e` runs the
                       reference's Go call sequence (llama.go Predict per step)
                       through the cuda.h ABI with host buffers and the prefix
                       cache on.
  --impl reference     the reference's CPU path: the reference has none (its
                       only Runner is CUDA, llm/array.go:123-135), so this times
                       the C++ CPU restatement of its semantics (oracle/) on all
                       host cores.
  --impl reference-gpu (extra) the reference's own cuda.cu built for sm_100a,
                       driven by the same Go-loop host mirror (full re-prefill
                       per step, as llm/model.go does).

Multi-GPU: the 1B decode does not shard; --gpus N runs N independent replicas
(one process per GPU under torchrun), value = tokens/s summed over ranks with
the max time over ranks.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# the e2e arm drives the ABI like the Go runtime; its incremental mode must be
# chosen before cuda_init reads it
os.environ.setdefault("WUKONG_PREFIX_CACHE", "1")

METRIC = "decode tokens/sec (batch 1, Q8_0)"
CFG_1B = dict(L=16, d=2048, H=32, Hk=8, D=64, F=8192, V=128256, eps=1e-5, theta=500000.0)
PROMPT = 128


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return j["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def step_bytes(cfg, ctx_avg, batch):
    """Algorithmic HBM bytes of one decode step: every weight once (Q8_0 =
    34/32 bytes per element) plus the K/V rows read by attention."""
    d, H, Hk, D, F, V, L = cfg["d"], cfg["H"], cfg["Hk"], cfg["D"], cfg["F"], cfg["V"], cfg["L"]
    per_layer = ((H + 2 * Hk) * D * d + d * d + 2 * F * d + d * F) * 34 // 32
    logits = V * d * 34 // 32
    kv = batch * ctx_avg * L * 2 * Hk * D * 2
    return L * per_layer + logits + kv


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, gpu):
        self.gpu = gpu
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out" if os.path.isdir(os.path.join(ROOT, "gpurun_out")) else "_work",
                                 f"clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()
            self.f.close()

    def summary(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        rows = []
        for line in open(self.path):
            p = [s.strip() for s in line.split(",")]
            if len(p) >= 8 and p[1].isdigit():
                rows.append(p)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(int(r[1]) for r in rows), "sm_max_mhz": int(rows[0][2]),
                "reasons": reasons, "samples": len(rows)}


def make_model_host(cfg, seed):
    from oracle import oracle as orc
    from tests.model_util import make_weights
    return make_weights(cfg, 8, 8, 1, seed=seed, ctx=PROMPT + 512 + 64)


# ------------------------------------------------------------------ our arm
def run_ours(args, rank, world):
    import torch
    import wukong_b200 as wk
    from tests.model_util import DeviceModel, build_engine, host_mirror

    torch.cuda.set_device(rank % max(1, torch.cuda.device_count()))
    L = wk.lib()
    L.cuda_init(rank % max(1, torch.cuda.device_count()))
    cfg = dict(CFG_1B)
    B, K, W = args.batch, args.steps, args.warmup
    ctx = PROMPT + W + K + 8
    w = make_model_host(cfg, seed=1234)
    dm = DeviceModel(w)
    m = build_engine(dm, w, cfg, 8, 8, 1, max_batch=B, ctx=ctx)
    prompt = np.random.default_rng(7).integers(0, cfg["V"], size=(B, PROMPT)).astype(np.int32)
    d_prompt = L.cuda_malloc(prompt.nbytes)
    L.cuda_to_device(d_prompt, prompt.ctypes.data_as(ctypes.c_void_p), prompt.nbytes)
    wk.check(L.wk_model_prefill(m, d_prompt, B, PROMPT, None))
    stream = torch.cuda.ExternalStream(L.wk_stream())
    for _ in range(W):
        wk.check(L.wk_model_decode_step(m))
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(rank) as clk:
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(K):
            L.wk_model_decode_step(m)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    launches = L.wk_model_step_launches(m)
    ctx_avg = PROMPT + W + K // 2
    sb = step_bytes(cfg, ctx_avg, B)
    res = dict(ms=ms, launches=launches, clocks=clk.summary(), step_bytes=sb)

    # dominant kernel: the Q8_0 dequant-GEMV at the FFN up|gate shape (16384 x 2048),
    # timed alone over 8 rotating weight copies (> L2) with CUDA events
    res["gemv"] = time_gemv(L, stream, N=16384, K=2048, M=B)
    res["gemv_op"] = time_gemv(L, stream, N=8192, K=2048, M=B)

    # e2e: the Go call sequence through cuda.h (host ids in, host token out), prefix cache on
    if not args.no_e2e:
        res["e2e"] = run_e2e(L, dm, cfg, B, K, W, prompt)
    L.wk_model_destroy(m)
    dm.free()
    return res


def time_gemv(L, stream, N, K, M, copies=8, reps=20):
    import torch
    rb = N * (K // 32) * 34
    ws = [L.cuda_malloc(rb) for _ in range(copies)]
    for i, p in enumerate(ws):
        L.wk_fill_random_q8_0(p, N, K, 77 + i, 0.02)
    x = L.cuda_malloc(2 * M * K)
    L.wk_fill_random_f16(x, M * K, 5, 1.0)
    o = L.cuda_malloc(2 * M * N)
    for i in range(3):
        L.wk_gemv(o, x, ws[i % copies], M, K, N, 8)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    n = reps * copies
    for i in range(n):
        L.wk_gemv(o, x, ws[i % copies], M, K, N, 8)
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000 / n
    for p in ws + [x, o]:
        L.cuda_free(p)
    byts = rb + 2 * M * K + 2 * M * N
    return dict(N=N, K=K, M=M, us=us, bytes=byts, gbs=byts / us / 1e3)


def run_e2e(L, dm, cfg, B, K, W, prompt):
    import torch
    from tests.model_util import host_mirror
    ctx = PROMPT + W + K + 8
    h, _ = host_mirror(dm, cfg, 8, 8, 1, ctx)
    seqs = [list(prompt[b]) for b in range(B)]
    buf = np.zeros((B, ctx), np.int32)
    out = np.zeros(B, np.int32)

    def step():
        n = len(seqs[0])
        for b in range(B):
            buf[b, :n] = seqs[b]
        ids = np.ascontiguousarray(buf[:, :n])
        rc = L.wk_host_llama_predict(h, ids.ctypes.data_as(ctypes.c_void_p), B, n, out.ctypes.data_as(ctypes.c_void_p))
        assert rc == 0
        for b in range(B):
            seqs[b].append(int(out[b]))
        return n

    for _ in range(W + 1):  # the first call is the prompt prefill
        step()
    t0 = time.perf_counter()
    h2d = 0
    for _ in range(K):
        h2d += 4 * B * step()
    dt = time.perf_counter() - t0
    L.wk_host_llama_destroy(h)
    return dict(value=B * K / dt, unit="tokens/s", h2d_bytes_per_step=h2d // K, d2h_bytes_per_step=4 * B,
                path="cuda.h ABI, llama.go call sequence, WUKONG_PREFIX_CACHE=1")


# ------------------------------------------------------------------ CPU baseline
def run_cpu(cfg, B, steps, budget_s=25.0):
    """The oracle port (C++ restatement of the reference semantics) on the host
    cores: prefill the 128-token prompt, then time greedy decode steps until the
    step budget or the time budget is used."""
    from oracle import oracle as orc
    from tests.model_util import oracle_model
    orc.set_threads(os.cpu_count() or 1)
    w = make_model_host(cfg, seed=1234)
    om = oracle_model(w, cfg, 8, 8, 1, PROMPT + steps + 16)
    om.reset(B)
    prompt = np.random.default_rng(7).integers(0, cfg["V"], size=(B, PROMPT)).astype(np.int32)
    tok, _, _ = om.forward(prompt)
    t0 = time.perf_counter()
    n = 0
    while n < steps and (time.perf_counter() - t0) < budget_s:
        tok, _, _ = om.forward(tok.reshape(B, 1))
        n += 1
    dt = time.perf_counter() - t0
    return dict(value=B * n / dt, unit="tokens/s", cores=orc.num_threads(), kind="port",
                sample=f"{n} decode steps after a {PROMPT}-token prefill, batch {B}, Llama-3.2-1B Q8_0")


def run_reference_gpu(args):
    """The reference's own cuda.cu (oracle/_ref) through the Go-loop host mirror."""
    import wukong_b200 as wk
    from oracle import oracle as orc
    from tests.model_util import DeviceModel, host_mirror
    ref = ctypes.CDLL(orc.REF_LIB_PATH, mode=ctypes.RTLD_LOCAL)
    ref.cuda_init.argtypes = [ctypes.c_int]
    ref.cuda_init(0)
    L = wk.lib()
    L.cuda_init(0)
    cfg = dict(CFG_1B)
    B, K, W = args.batch, args.steps, args.warmup
    ctx = PROMPT + W + K + 8
    w = make_model_host(cfg, seed=1234)
    dm = DeviceModel(w)
    L.cuda_to_host(ctypes.byref(ctypes.c_int()), dm.freqs, 4)  # weights resident
    h, _ = host_mirror(dm, cfg, 8, 8, 1, ctx, lib_handle=ref._handle)
    prompt = np.random.default_rng(7).integers(0, cfg["V"], size=(B, PROMPT)).astype(np.int32)
    seqs = [list(prompt[b]) for b in range(B)]
    out = np.zeros(B, np.int32)

    def step():
        ids = np.ascontiguousarray(np.array(seqs, np.int32))
        assert L.wk_host_llama_predict(h, ids.ctypes.data_as(ctypes.c_void_p), B, ids.shape[1],
                                       out.ctypes.data_as(ctypes.c_void_p)) == 0
        for b in range(B):
            seqs[b].append(int(out[b]))

    for _ in range(W + 1):
        step()
    t0 = time.perf_counter()
    for _ in range(K):
        step()
    dt = time.perf_counter() - t0
    return B * K / dt


# ------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    cfg = dict(CFG_1B)
    config = {"workload": f"Llama-3.2-1B Q8_0 greedy decode, batch {args.batch}, {PROMPT}-token prompt",
              "batch": args.batch, "prompt": PROMPT, "decode_steps": args.steps, "weights": "Q8_0 (output Q8_0), "
              "token_embd F16, norms 1.0, w ~ N(0, 0.02)", "l2": "per-step weights 1.31 GB > 126 MB L2, no flush",
              "parallelism": f"replicas x{world}" if world > 1 else "single GPU"}

    if args.impl == "reference":
        if rank != 0:
            return
        cpu = run_cpu(cfg, args.batch, args.warmup + args.steps, budget_s=150.0)
        line = {"impl": "reference", "metric": METRIC, "value": cpu["value"], "unit": "tokens/s", "n_gpus": 1,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "int8 x f16 -> f32",
                "data": "synthetic", "config": config,
                "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": cpu["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "note": "the reference has no CPU compute path (llm/array.go:123-135); this is the C++ restatement "
                        "of its semantics in oracle/ on all host cores"}
        print(json.dumps(line))
        return

    if args.impl == "reference-gpu":
        v = run_reference_gpu(args)
        print(json.dumps({"impl": "reference-gpu", "metric": METRIC, "value": v, "unit": "tokens/s",
                          "config": config, "path": "reference cuda.cu (sm_100a) via the llama.go call sequence, "
                          "full re-prefill per step"}))
        return

    if world > 1:
        import torch
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", rank % torch.cuda.device_count()))
    res = run_ours(args, rank, world)
    if world > 1:
        import torch
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    hbm, src = peaks()
    K = args.steps
    value = world * args.batch * K / (res["ms"] / 1e3)
    g = res["gemv"]
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": args.warmup,
        "ms_per_step": res["ms"] / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 x f16 -> f32", "data": "synthetic", "config": config,
        "gpu_launches": res["launches"] * K,
        "roofline": {"bound": "hbm", "kernel": f"gemv_kernel<Q8_0> {g['N']}x{g['K']} M={g['M']}",
                     "achieved": g["gbs"], "peak": hbm, "unit": "GB/s", "frac": g["gbs"] / hbm,
                     "peak_source": src, "traffic": None,
                     "step": {"bytes": res["step_bytes"], "achieved": res["step_bytes"] / (res["ms"] / K) / 1e6,
                              "frac": res["step_bytes"] / (res["ms"] / K) / 1e6 / hbm}},
        "op_gemv_8192x2048": res["gemv_op"],
        "clocks": res["clocks"],
    }
    if "e2e" in res:
        line["e2e"] = res["e2e"]
    if not args.no_cpu and world == 1:
        cpu = run_cpu(cfg, args.batch, 64)
        line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps(line))


if __name__ == "__main__":
    main()
