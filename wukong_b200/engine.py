"""Python front of the native decode engine (include/wukong_ext.h) and of the
C++ mirror of the reference's Go host loop (include/wukong_host.h), with
synthetic device-resident weights.

Synthetic weights are generated on the device by the library
(wk_fill_random_q8_0 / wk_fill_random_f16: Irwin-Hall(4) normal samples of a
counter-based hash, quantised GGUF-style), in the layout of a GGUF file after
llama.go's fusion (llm/llama.go:80-112).  The seeds follow one scheme per
tensor so that a host generator with the same scheme reproduces the bytes.
"""
import ctypes

import numpy as np

import wukong_b200 as wk

LLAMA = {
    "1b": dict(L=16, d=2048, H=32, Hk=8, D=64, F=8192, V=128256, eps=1e-5, theta=500000.0),
    "8b": dict(L=32, d=4096, H=32, Hk=8, D=128, F=14336, V=128256, eps=1e-5, theta=500000.0),
    "70b": dict(L=80, d=8192, H=64, Hk=8, D=128, F=28672, V=128256, eps=1e-5, theta=500000.0),
}

# per-tensor seed offsets: layer l uses seed + 100 * l + offset
SEED_Q, SEED_K, SEED_V, SEED_O, SEED_UP, SEED_GATE, SEED_DOWN = 1, 2, 3, 4, 5, 6, 7
SEED_EMBD, SEED_OUT = 90001, 90002


def wbytes(rows, cols, wtype):
    if wtype == wk.Q8_0:
        return rows * (cols // 32) * 34
    if wtype == wk.F32:
        return rows * cols * 4
    return rows * cols * 2


class DeviceBuffers:
    """cuda_malloc'ed buffers freed together."""

    def __init__(self):
        self.ptrs = []

    def alloc(self, nbytes):
        p = wk.lib().cuda_malloc(max(int(nbytes), 16))
        if not p:
            raise MemoryError(f"cuda_malloc({nbytes}) failed")
        self.ptrs.append(p)
        return p

    def free(self):
        for p in self.ptrs:
            wk.lib().cuda_free(p)
        self.ptrs = []


def fill(ptr, rows, cols, wtype, seed, std=0.02):
    L = wk.lib()
    if wtype == wk.Q8_0:
        wk.check(L.wk_fill_random_q8_0(ptr, rows, cols, seed, std))
    elif wtype == wk.F16:
        wk.check(L.wk_fill_random_f16(ptr, rows * cols, seed, std))
    else:
        raise ValueError(f"synthetic weights for dtype {wtype} are not generated on the device")


def make_freqs(D, ctx, theta):
    """RoPE table of llama.go:54-67, built by the library's host code."""
    out = np.empty((ctx, D), np.float32)
    wk.lib().wk_host_make_freqs(out.ctypes.data_as(ctypes.c_void_p), None, D, ctx, theta)
    return out


class SyntheticLlama:
    """Random-init Llama-3 weights on the current device.

    unfused=True also keeps q, k, v, up, gate as separate tensors (the form the
    reference's Go loader hands to llama.go's Setup, used by HostLlama).  With
    tp_world > 1 every tensor is this rank's shard (wukong_b200.tp layout) with
    its own seeds, sized for the per-rank counts."""

    def __init__(self, cfg, ctx, wtype=wk.Q8_0, out_type=wk.Q8_0, embd_type=wk.F16, seed=1234, unfused=False,
                 tp_rank=0, tp_world=1):
        self.cfg, self.ctx = dict(cfg), ctx
        self.wtype, self.out_type, self.embd_type = wtype, out_type, embd_type
        self.buf = DeviceBuffers()
        L = wk.lib()
        d, D = cfg["d"], cfg["D"]
        H, Hk, F, V = (cfg[k] // tp_world for k in ("H", "Hk", "F", "V"))
        self.local = dict(cfg, H=H, Hk=Hk, F=F, V=V)
        sh = 7919 * tp_rank
        ones = self.buf.alloc(4 * d)
        wk.check(L.wk_fill_const_f32(ones, d, 1.0))
        self.layers = []
        for l in range(cfg["L"]):
            s = seed + 100 * l + sh
            qkv = self.buf.alloc(wbytes((H + 2 * Hk) * D, d, wtype))
            fill(qkv, H * D, d, wtype, s + SEED_Q)
            fill(qkv + wbytes(H * D, d, wtype), Hk * D, d, wtype, s + SEED_K)
            fill(qkv + wbytes((H + Hk) * D, d, wtype), Hk * D, d, wtype, s + SEED_V)
            fc = self.buf.alloc(wbytes(2 * F, d, wtype))
            fill(fc, F, d, wtype, s + SEED_UP)
            fill(fc + wbytes(F, d, wtype), F, d, wtype, s + SEED_GATE)
            o = self.buf.alloc(wbytes(d, H * D, wtype))
            fill(o, d, H * D, wtype, s + SEED_O)
            down = self.buf.alloc(wbytes(d, F, wtype))
            fill(down, d, F, wtype, s + SEED_DOWN)
            lw = dict(attn_norm=ones, ffn_norm=ones, qkv=qkv, fc=fc, o=o, down=down)
            if unfused:
                # separate tensors with the same bytes (the Go loader's view)
                for name, rows, seed_off in (("q", H * D, SEED_Q), ("k", Hk * D, SEED_K), ("v", Hk * D, SEED_V),
                                             ("up", F, SEED_UP), ("gate", F, SEED_GATE)):
                    p = self.buf.alloc(wbytes(rows, d, wtype))
                    fill(p, rows, d, wtype, s + seed_off)
                    lw[name] = p
            self.layers.append(lw)
        self.token_embd = self.buf.alloc(wbytes(cfg["V"], d, embd_type))
        fill(self.token_embd, cfg["V"], d, embd_type, seed + SEED_EMBD, 1.0)
        self.output = self.buf.alloc(wbytes(V, d, out_type))
        fill(self.output, V, d, out_type, seed + SEED_OUT + sh)
        self.output_norm = ones
        fr = make_freqs(D, ctx, cfg["theta"])
        self.freqs = self.buf.alloc(fr.nbytes)
        L.cuda_to_device(self.freqs, fr.ctypes.data_as(ctypes.c_void_p), fr.nbytes)

    def weight_bytes_per_step(self):
        c, wt = self.local, self.wtype
        d, D = c["d"], c["D"]
        per = (wbytes((c["H"] + 2 * c["Hk"]) * D, d, wt) + wbytes(d, c["H"] * D, wt) + wbytes(2 * c["F"], d, wt) +
               wbytes(d, c["F"], wt))
        return c["L"] * per + wbytes(c["V"], d, self.out_type)

    def free(self):
        self.buf.free()


class Engine:
    """wk_model over device weights (a dict per layer with attn_norm, qkv, o,
    ffn_norm, fc, down, and token_embd / output_norm / output / freqs)."""

    def __init__(self, cfg, layers, token_embd, output_norm, output, freqs, ctx, max_batch, wtype=wk.Q8_0,
                 out_type=wk.Q8_0, embd_type=wk.F16, tp=False):
        L = wk.lib()
        c = wk.WKConfig(cfg["L"], cfg["d"], cfg["H"], cfg["Hk"], cfg["D"], cfg["F"], cfg["V"], cfg["eps"], wtype,
                        out_type, embd_type)
        self.m = L.wk_model_create(ctypes.byref(c))
        if not self.m:
            raise RuntimeError(L.wk_last_error().decode())
        if tp:
            wk.check(L.wk_model_set_tp(self.m, 1))
        for i, lw in enumerate(layers):
            wk.check(L.wk_model_set_layer(self.m, i, lw["attn_norm"], lw["qkv"], lw["o"], lw["ffn_norm"], lw["fc"],
                                          lw["down"]))
        wk.check(L.wk_model_set_head(self.m, token_embd, output_norm, output, freqs, ctx))
        wk.check(L.wk_model_alloc_cache(self.m, max_batch, ctx))

    @classmethod
    def from_synthetic(cls, sm, max_batch, tp=False):
        return cls(sm.local, sm.layers, sm.token_embd, sm.output_norm, sm.output, sm.freqs, sm.ctx, max_batch,
                   sm.wtype, sm.out_type, sm.embd_type, tp=tp)

    def prefill(self, d_ids, batch, n, d_tokens_out=None):
        wk.check(wk.lib().wk_model_prefill(self.m, d_ids, batch, n, d_tokens_out))

    def step(self):
        wk.check(wk.lib().wk_model_decode_step(self.m))

    def tokens_ptr(self):
        return wk.lib().wk_model_tokens(self.m)

    def launches_per_step(self):
        return wk.lib().wk_model_step_launches(self.m)

    def destroy(self):
        if self.m:
            wk.lib().wk_model_destroy(self.m)
            self.m = None


class HostLlama:
    """wk_host_llama: llama.go's Setup / Predict and model.go's greedy loop in
    C++ above a table of cuda.h entry points (this library by default)."""

    def __init__(self, sm, lib_handle=None):
        L = wk.lib()
        cfg = sm.cfg
        self.table = ctypes.create_string_buffer(wk.WK_ABI_SIZE)
        rc = L.wk_abi_bind(self.table, lib_handle if lib_handle is not None else L._handle)
        if rc != 0:
            raise RuntimeError(L.wk_host_last_error().decode())
        hc = wk.WKHostConfig(cfg["L"], cfg["d"], cfg["H"], cfg["Hk"], cfg["D"], cfg["F"], cfg["V"], sm.ctx,
                             cfg["eps"], cfg["theta"], sm.wtype, sm.out_type, sm.embd_type)
        self.h = L.wk_host_llama_create(self.table, ctypes.byref(hc))
        layers = (wk.WKHostLayer * cfg["L"])()
        for i, lw in enumerate(sm.layers):
            for k in ("attn_norm", "q", "k", "v", "o", "ffn_norm", "up", "gate", "down"):
                setattr(layers[i], k, lw[k])
        rc = L.wk_host_llama_setup(self.h, layers, sm.token_embd, sm.output_norm, sm.output, None)
        if rc != 0:
            raise RuntimeError(L.wk_host_last_error().decode())

    def predict(self, ids, out):
        """ids: int32 [batch, n] host array; out: int32 [batch] host array."""
        ids = np.ascontiguousarray(ids, np.int32)
        rc = wk.lib().wk_host_llama_predict(self.h, ids.ctypes.data_as(ctypes.c_void_p), ids.shape[0], ids.shape[1],
                                            out.ctypes.data_as(ctypes.c_void_p))
        if rc != 0:
            raise RuntimeError(wk.lib().wk_host_last_error().decode())

    def destroy(self):
        if self.h:
            wk.lib().wk_host_llama_destroy(self.h)
            self.h = None
