"""Benchmark: greedy decode tokens/s of Llama-3 with Q8_0 weights on B200.

Workload (default, --model 1b): Llama-3.2-1B architecture (16 layers, d 2048,
32/8 heads, head_dim 64, SwiGLU 8192, vocab 128256, RoPE theta 500000, RMSNorm
eps 1e-5), random-init weights generated on the device: linear layers and
output.weight Q8_0 (w ~ N(0, 0.02) quantised GGUF-style), token_embd F16,
norms 1.0; batch 1 (--batch), a 128-token uniform-random prompt, then greedy
decode.  A step is one decode step (one token per sequence).  The weights read
per step (1.31 GB) exceed the 126 MB L2, so no flush is needed between steps.
--model 8b / 70b: Llama-3.1-8B / -70B shapes with a 2048 / 4096-token prompt.

Arms
  (default)          the native engine (wukong_ext.h): CUDA-graph decode step,
                     inputs resident in HBM -> `value`.  `e2e`: for 1b, the
                     reference's Go call sequence (llama.go Predict per step)
                     through the cuda.h ABI with host ids in and the host token
                     out, prefix cache on; for tensor-parallel runs, the engine
                     with the step's ids copied from pinned host memory and the
                     tokens read back every step.
  --impl reference   the reference's CPU path: the reference has none (its only
                     Runner is CUDA, llm/array.go:123-135), so this times the C++
                     CPU restatement of its semantics (oracle/) on all host cores.
  --op NxKxM,...     the single Q8_0 dequant-matmul op through cuda_matmul.

Multi-GPU: 1b does not shard (replicas: --gpus N runs N independent copies,
one process per GPU, value = tokens/s summed over ranks, weak scaling); 8b and
70b are tensor-parallel over the N GPUs (one model, value = its tokens/s,
strong scaling).  Times are the max over ranks of CUDA-event durations.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# the e2e arm drives the ABI like the Go runtime; its incremental mode must be
# chosen before cuda_init reads it
os.environ.setdefault("WUKONG_PREFIX_CACHE", "1")

METRIC = "decode tokens/sec (batch 1, Q8_0)"
PROMPTS = {"1b": 128, "8b": 2048, "70b": 4096}
NAMES = {"1b": "Llama-3.2-1B", "8b": "Llama-3.1-8B", "70b": "Llama-3.1-70B"}
SEED = 1234


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return j["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def profiled_traffic(name):
    """DRAM bytes per launch of a kernel from its committed ncu summary
    (a `traffic_bytes_per_launch: N` line in profiles/<name>.md), or None."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            return int(line.split(":", 1)[1].strip().split()[0])
    return None


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, gpu):
        self.gpu = gpu
        self.proc = None
        out = os.path.join(ROOT, "gpurun_out")
        self.path = os.path.join(out if os.path.isdir(out) else tempfile.gettempdir(), f"clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
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


def kv_bytes(cfg, ctx_avg, batch, world):
    """K/V rows read by attention per step on one rank (fp16)."""
    return batch * ctx_avg * cfg["L"] * 2 * (cfg["Hk"] // world) * cfg["D"] * 2


# ------------------------------------------------------------------ our arm
def run_ours(args, rank, world, local_rank):
    import torch
    import wukong_b200 as wk
    from wukong_b200.engine import LLAMA, Engine, HostLlama, SyntheticLlama

    torch.cuda.set_device(local_rank)
    L = wk.lib()
    L.cuda_init(local_rank)
    cfg = dict(LLAMA[args.model])
    tpw = world if args.model != "1b" else 1
    if tpw > 1:
        idbuf = ctypes.create_string_buffer(128)
        if rank == 0:
            wk.check(L.wk_tp_unique_id(idbuf))
        t = torch.frombuffer(bytearray(idbuf.raw), dtype=torch.uint8).cuda()
        torch.distributed.broadcast(t, 0)
        wk.check(L.wk_tp_init(rank, world, bytes(t.cpu().numpy())))
    B, K, W, P = args.batch, args.steps, args.warmup, args.prompt
    e2e_abi = not args.no_e2e and tpw == 1
    # the engine e2e leg (tensor-parallel runs) continues decoding after the timed steps
    ctx = P + W + K + 8 + (W + K if (not args.no_e2e and not e2e_abi) else 0)
    wt = wk.F16 if args.wtype == "f16" else wk.Q8_0
    sm = SyntheticLlama(cfg, ctx, wtype=wt, out_type=wt, seed=SEED, unfused=e2e_abi, tp_rank=rank if tpw > 1 else 0,
                        tp_world=tpw)
    eng = Engine.from_synthetic(sm, max_batch=B, tp=tpw > 1)
    prompt = np.random.default_rng(7).integers(0, cfg["V"], size=(B, P)).astype(np.int32)
    d_prompt = L.cuda_malloc(prompt.nbytes)
    L.cuda_to_device(d_prompt, prompt.ctypes.data_as(ctypes.c_void_p), prompt.nbytes)
    eng.prefill(d_prompt, B, P)
    stream = torch.cuda.ExternalStream(L.wk_stream())
    for _ in range(W):
        eng.step()
    torch.cuda.synchronize()
    # Every timed block decodes the same K steps: the sequences are rolled back
    # to the block's start (wk_model_truncate) and get the same input ids again.
    pos0 = L.wk_model_position(eng.m)
    ids0 = np.zeros(B, np.int32)
    L.cuda_to_host(ids0.ctypes.data_as(ctypes.c_void_p), L.wk_model_next_ids(eng.m), 4 * B)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def block():
        wk.check(L.wk_model_truncate(eng.m, pos0))
        L.cuda_to_device(L.wk_model_next_ids(eng.m), ids0.ctypes.data_as(ctypes.c_void_p), 4 * B)
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(K):
            L.wk_model_decode_step(eng.m)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    def max_over_ranks(vals):
        if world == 1:
            return list(vals)
        t = torch.tensor(vals, device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return t.tolist()

    # enough identical blocks for the clock sampler to see seconds of load
    first = max_over_ranks([block()])[0]
    R = int(min(args.max_blocks, max(args.min_blocks, -(-args.timed_seconds * 1e3 // first))))
    with Clocks(local_rank) as clk:
        times = [block() for _ in range(R)]
    times = max_over_ranks(times)
    ms = statistics.median(times)
    res = dict(ms=ms, blocks=R, block_ms_min=min(times), block_ms_max=max(times), launches=eng.launches_per_step(),
               clocks=clk.summary(), tp=tpw, step_bytes=sm.weight_bytes_per_step() + kv_bytes(cfg, pos0 + K // 2, B, tpw))

    # dominant kernel: the Q8_0 dequant-GEMV at the FFN up|gate shape of the
    # model (per rank), timed alone over 8 rotating weight copies (> L2)
    if rank == 0:
        res["gemv"] = time_gemv(L, stream, N=2 * sm.local["F"], K=cfg["d"], M=min(B, 8), wtype=wt)
        res["gemv_op"] = time_gemv(L, stream, N=8192, K=2048, M=min(B, 8), wtype=wt)

    if not args.no_e2e:
        if e2e_abi:
            res["e2e"] = run_e2e_abi(L, sm, B, K, W, prompt)
        else:
            res["e2e"] = run_e2e_engine(L, eng, B, K, W, world)
    eng.destroy()
    sm.free()
    L.cuda_free(d_prompt)
    if tpw > 1:
        L.wk_tp_fini()
    return res


def time_gemv(L, stream, N, K, M, copies=8, reps=20, wtype=8):
    import torch
    rb = N * (K // 32) * 34 if wtype == 8 else N * K * 2
    ws = [L.cuda_malloc(rb) for _ in range(copies)]
    for i, p in enumerate(ws):
        if wtype == 8:
            L.wk_fill_random_q8_0(p, N, K, 77 + i, 0.02)
        else:
            L.wk_fill_random_f16(p, N * K, 77 + i, 0.02)
    x = L.cuda_malloc(2 * M * K)
    L.wk_fill_random_f16(x, M * K, 5, 1.0)
    o = L.cuda_malloc(2 * M * N)
    for i in range(3):
        L.wk_gemv(o, x, ws[i % copies], M, K, N, wtype)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    n = reps * copies
    for i in range(n):
        L.wk_gemv(o, x, ws[i % copies], M, K, N, wtype)
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000 / n
    for p in ws + [x, o]:
        L.cuda_free(p)
    byts = rb + 2 * M * K + 2 * M * N
    return dict(N=N, K=K, M=M, us=us, bytes=byts, gbs=byts / us / 1e3)


def run_e2e_abi(L, sm, B, K, W, prompt):
    """The reference's Go call sequence through cuda.h (host ids in, host token
    out every step), with the prefix cache on."""
    from wukong_b200.engine import HostLlama
    h = HostLlama(sm)
    ctx = sm.ctx
    seqs = [list(prompt[b]) for b in range(B)]
    buf = np.zeros((B, ctx), np.int32)
    out = np.zeros(B, np.int32)

    def step():
        n = len(seqs[0])
        for b in range(B):
            buf[b, :n] = seqs[b]
        h.predict(buf[:, :n], out)
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
    h.destroy()
    return dict(value=B * K / dt, unit="tokens/s", h2d_bytes_per_step=h2d // K, d2h_bytes_per_step=4 * B,
                path="cuda.h ABI, llama.go call sequence, WUKONG_PREFIX_CACHE=1")


def run_e2e_engine(L, eng, B, K, W, world):
    """The engine with host I/O every step: the step's ids are copied from
    pinned host memory, the step runs, its tokens are read back."""
    import torch
    import wukong_b200 as wk
    ids = torch.zeros(B, dtype=torch.int32).pin_memory()
    toks = torch.zeros(B, dtype=torch.int32).pin_memory()
    nxt = L.wk_model_next_ids(eng.m)
    cur = L.wk_model_tokens(eng.m)

    def step():
        L.cuda_to_device(nxt, ctypes.c_void_p(ids.data_ptr()), 4 * B)
        wk.check(L.wk_model_decode_step(eng.m))
        L.cuda_to_host(ctypes.c_void_p(toks.data_ptr()), cur, 4 * B)
        ids.copy_(toks)

    L.cuda_to_host(ctypes.c_void_p(toks.data_ptr()), cur, 4 * B)
    ids.copy_(toks)
    for _ in range(W):
        step()
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        step()
    dt = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([dt], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        dt = float(t.item())
    return dict(value=B * K / dt, unit="tokens/s", h2d_bytes_per_step=4 * B, d2h_bytes_per_step=4 * B,
                path="wukong_ext.h engine, ids from pinned host memory and tokens back every step")


def run_op(spec, copies=8, reps=20):
    """The single Q8_0 dequant-matmul op: W [N, K] Q8_0 (8 rotating copies, >
    L2 for the default shapes), X [M, K] fp16, out [M, N] fp16, through
    cuda_matmul (GEMV for M <= 8, tcgen05 GEMM for M >= 16)."""
    import torch
    import wukong_b200 as wk
    L = wk.lib()
    L.cuda_init(0)
    stream = torch.cuda.ExternalStream(L.wk_stream())
    hbm, src = peaks()
    for item in spec.split(","):
        N, K, M = (int(v) for v in item.lower().split("x"))
        rb = N * (K // 32) * 34
        ws = [L.cuda_malloc(rb) for _ in range(copies)]
        for i, p in enumerate(ws):
            L.wk_fill_random_q8_0(p, N, K, 77 + i, 0.02)
        x = L.cuda_malloc(2 * M * K)
        L.wk_fill_random_f16(x, M * K, 5, 1.0)
        o = L.cuda_malloc(2 * M * N)
        for i in range(3):
            L.cuda_matmul(o, x, ws[i % copies], None, M, K, N, 8)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = reps * copies
        e0.record(stream)
        for i in range(n):
            L.cuda_matmul(o, x, ws[i % copies], None, M, K, N, 8)
        e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000 / n
        byts = rb + 2 * M * K + 2 * M * N
        print(json.dumps({"op": "cuda_matmul Q8_0", "N": N, "K": K, "M": M, "us": us, "bytes": byts,
                          "gbs": byts / us / 1e3, "hbm_frac": byts / us / 1e3 / hbm, "peak_source": src,
                          "tflops": 2.0 * M * N * K / us / 1e6}))
        for p in ws + [x, o]:
            L.cuda_free(p)
    L.cuda_fini()


def prefill_flops(cfg, B, T):
    """Dense FLOPs of one prefill: every linear layer on all B T rows, causal
    attention (q.k and p.v over the keys at or before each row), logits of the
    last row of each sequence."""
    d, H, Hk, D, F, V, L = (cfg[k] for k in ("d", "H", "Hk", "D", "F", "V", "L"))
    linear = L * ((H + 2 * Hk) * D * d + d * H * D + 2 * F * d + d * F)
    attn = L * H * D * 2 * 2 * (T * (T + 1) // 2)
    return 2.0 * linear * B * T + attn * B + 2.0 * V * d * B


def run_prefill(args):
    """Prefill throughput: wk_model_prefill of B prompts of T tokens (the
    tcgen05 GEMMs with fused dequantisation and epilogues, the flash-style
    prefill attention, the logits of the last rows), inputs resident in HBM;
    tokens/s and the fraction of the measured sustained bf16 tensor peak."""
    import torch
    import wukong_b200 as wk
    from wukong_b200.engine import LLAMA, Engine, SyntheticLlama
    L = wk.lib()
    L.cuda_init(0)
    stream = torch.cuda.ExternalStream(L.wk_stream())
    cfg = dict(LLAMA[args.model])
    wt = wk.F16 if args.wtype == "f16" else wk.Q8_0
    B, T = args.batch, args.prompt
    sm = SyntheticLlama(cfg, T + 8, wtype=wt, out_type=wt, seed=SEED)
    eng = Engine.from_synthetic(sm, max_batch=B)
    prompt = np.random.default_rng(7).integers(0, cfg["V"], size=(B, T)).astype(np.int32)
    d_prompt = L.cuda_malloc(prompt.nbytes)
    L.cuda_to_device(d_prompt, prompt.ctypes.data_as(ctypes.c_void_p), prompt.nbytes)
    for _ in range(args.warmup):
        eng.prefill(d_prompt, B, T)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    with Clocks(0) as clk:
        for _ in range(args.steps):
            torch.cuda.synchronize()
            e0.record(stream)
            eng.prefill(d_prompt, B, T)
            e1.record(stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
    ms = statistics.median(times)
    flops = prefill_flops(cfg, B, T)
    pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {"bf16_tflops_sustained": 1400.0}
    tf = flops / (ms / 1e3) / 1e12
    line = {"metric": "prefill tokens/sec", "value": B * T / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "dtype": "f16 x f16 -> f32" if wt == wk.F16 else "int8 x f16 -> f32", "data": "synthetic",
            "config": {"workload": f"{NAMES[args.model]} {args.wtype.upper()} prefill, batch {B}, {T}-token prompt",
                       "model": NAMES[args.model], "batch": B, "prompt": T,
                       "timing": "median of single prefills (CUDA events), weights read per prefill exceed L2"},
            "roofline": {"bound": "tensor", "achieved": tf, "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                         "frac": tf / pk["bf16_tflops_sustained"], "flops_per_step": flops,
                         "peak_source": "measured sustained bf16 (cuBLAS) of MEASURED_PEAKS.json"},
            "gpu_launches": None, "clocks": clk.summary()}
    print(json.dumps(line))
    eng.destroy()
    sm.free()
    L.cuda_free(d_prompt)
    L.cuda_fini()


# ------------------------------------------------------------------ CPU baseline
def run_cpu(model, B, P, steps, budget_s=25.0, wtype=8):
    """The oracle port (C++ restatement of the reference semantics) on the host
    cores, on the same synthetic model (the oracle's generator is bit-identical
    to the device one): prefill the prompt, then time greedy decode steps until
    the step budget or the time budget is used."""
    from oracle import oracle as orc
    from tests.model_util import make_weights, oracle_model
    from wukong_b200.engine import LLAMA
    cfg = dict(LLAMA[model])
    orc.set_threads(os.cpu_count() or 1)
    # 8B: a 128-token prompt instead of 2048 keeps the CPU prefill to seconds;
    # a decode step there is bound by the 8 GB of weights, not by the context
    P_full, P = P, (P if model == "1b" else min(P, 128))
    w = make_weights(cfg, wtype, wtype, 1, seed=SEED, ctx=P + steps + 16)
    om = oracle_model(w, cfg, wtype, wtype, 1, P + steps + 16)
    om.reset(B)
    prompt = np.random.default_rng(7).integers(0, cfg["V"], size=(B, P)).astype(np.int32)
    tok, _, _ = om.forward(prompt)
    t0 = time.perf_counter()
    n = 0
    while n < steps and (time.perf_counter() - t0) < budget_s:
        tok, _, _ = om.forward(tok.reshape(B, 1))
        n += 1
    dt = time.perf_counter() - t0
    return dict(value=B * n / dt, unit="tokens/s", cores=orc.num_threads(), kind="port",
                sample=f"{n} decode steps after a {P}-token prefill, batch {B}, {NAMES[model]} "
                       f"{'Q8_0' if wtype == 8 else 'F16'}"
                       + ("" if P == P_full else f" (the GPU arm's prompt is {P_full} tokens)"))


# ------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--model", default=None, choices=["1b", "8b", "70b"],
                    help="default: 1b on one plain process; 8b (tensor-parallel over the ranks) under "
                         "torch.distributed.run, at every world size including 1")
    ap.add_argument("--min-blocks", type=int, default=20, help="timed blocks of --steps steps (at least)")
    ap.add_argument("--max-blocks", type=int, default=400)
    ap.add_argument("--timed-seconds", type=float, default=3.0,
                    help="blocks are added until about this much decode time is timed")
    ap.add_argument("--prompt", type=int, default=None, help="prompt tokens (default 128 / 2048 / 4096)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default="decode", choices=["decode", "prefill"],
                    help="prefill: time wk_model_prefill of --batch prompts of --prompt tokens (one JSON line)")
    ap.add_argument("--wtype", default="q8_0", choices=["q8_0", "f16"], help="linear and output weights")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--op", default=None, metavar="NxKxM[,...]",
                    help="time only the Q8_0 dequant-matmul op at these shapes (one JSON line each), "
                         "e.g. 8192x2048x1,8192x2048x16,8192x2048x128")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.model is None:
        # the multi-GPU curve is tensor-parallel Llama-3.1-8B decode at every N
        # (N = 1 included when launched by torch.distributed.run); one plain
        # process measures the single-GPU headline, Llama-3.2-1B
        launched = "TORCHELASTIC_RUN_ID" in os.environ or "LOCAL_WORLD_SIZE" in os.environ
        args.model = "8b" if (launched or world > 1 or args.gpus > 1) else "1b"
    if args.prompt is None:
        args.prompt = PROMPTS[args.model]
    dtype_str = "int8 x f16 -> f32" if args.wtype == "q8_0" else "f16 x f16 -> f32"
    metric = METRIC if (args.batch == 1 and args.wtype == "q8_0") else \
        f"decode tokens/sec (batch {args.batch}, {args.wtype.upper()})"
    tp = args.model != "1b" and world > 1
    if tp:
        par = f"tp{world}"
    elif world > 1:
        par = f"replicas x{world}"
    else:
        par = "single GPU"
    config = {"workload": f"{NAMES[args.model]} {args.wtype.upper()} greedy decode, batch {args.batch}, "
                          f"{args.prompt}-token prompt",
              "model": NAMES[args.model], "batch": args.batch, "prompt": args.prompt, "decode_steps": args.steps,
              "weights": f"{args.wtype.upper()} linear layers and output.weight, token_embd F16, norms 1.0, "
                         "w ~ N(0, 0.02), "
                         "generated on the device",
              "l2": "weights read per step exceed the 126 MB L2, no flush", "parallelism": par,
              "timing": f"median of identical timed blocks of {args.steps} decode steps, each from the same "
                        "position with the same ids (max over ranks per block)"}

    if args.op:
        run_op(args.op)
        return
    if args.mode == "prefill":
        run_prefill(args)
        return

    if args.impl == "reference":
        if rank != 0:
            return
        if args.model == "70b":
            print(json.dumps({"impl": "reference", "unavailable": "the 70B CPU restatement needs about 80 GB of "
                              "host memory for its weights; no CPU run at this size"}))
            return
        cpu = run_cpu(args.model, args.batch, args.prompt, args.warmup + args.steps, budget_s=150.0,
                      wtype=8 if args.wtype == "q8_0" else 1)
        line = {"impl": "reference", "metric": metric, "value": cpu["value"], "unit": "tokens/s", "n_gpus": 1,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": dtype_str,
                "data": "synthetic", "config": config,
                "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": cpu["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "note": "the reference has no CPU compute path (llm/array.go:123-135); this is the C++ restatement "
                        "of its semantics in oracle/ on all host cores"}
        print(json.dumps(line))
        return

    if world > 1:
        import datetime
        import torch
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                             timeout=datetime.timedelta(seconds=300))
    res = run_ours(args, rank, world, local_rank)
    if world > 1:
        import torch
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    hbm, src = peaks()
    K = args.steps
    value = (1 if tp else world) * args.batch * K / (res["ms"] / 1e3)
    g = res["gemv"]
    gname = f"gemv_{args.wtype}_{g['N']}x{g['K']}_m{g['M']}"
    step_gbs = res["step_bytes"] / (res["ms"] / K) / 1e6
    line = {
        "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": args.warmup,
        "ms_per_step": res["ms"] / K, "timed_blocks": res["blocks"],
        "block_ms": {"median": res["ms"], "min": res["block_ms_min"], "max": res["block_ms_max"]},
        "higher_is_better": True, "scaling": "strong" if tp else "weak",
        "vs_baseline": None, "dtype": dtype_str, "data": "synthetic", "config": config,
        "gpu_launches": res["launches"] * K,
        "roofline": {"bound": "hbm", "kernel": f"gemv_kernel<{args.wtype.upper()}> {g['N']}x{g['K']} M={g['M']}",
                     "achieved": g["gbs"], "peak": hbm, "unit": "GB/s", "frac": g["gbs"] / hbm,
                     "peak_source": src, "traffic": profiled_traffic(gname),
                     "step": {"bytes_per_gpu": res["step_bytes"], "achieved": step_gbs, "frac": step_gbs / hbm}},
        "op_gemv_8192x2048": res["gemv_op"],
        "clocks": res["clocks"],
    }
    if "e2e" in res:
        line["e2e"] = res["e2e"]
    if not args.no_cpu and world == 1 and args.model in ("1b", "8b"):
        cpu = run_cpu(args.model, args.batch, args.prompt, 64, wtype=8 if args.wtype == "q8_0" else 1)
        line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps(line))


if __name__ == "__main__":
    main()
