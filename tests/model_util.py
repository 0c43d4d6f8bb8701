"""Synthetic Llama-3 models for the model-level GPU tests and the benchmark:
weights are generated on the host by the oracle's counter-based generator
(bit-identical to the library's device generator), so the CPU oracle and the
GPU see the same bytes."""
import ctypes

import numpy as np

import wukong_b200 as wk
from oracle import oracle as orc
from tests.gpu_util import up

LLAMA_1B = dict(L=16, d=2048, H=32, Hk=8, D=64, F=8192, V=128256, eps=1e-5, theta=500000.0)


def make_weights(cfg, wtype, out_type, embd_type, seed, ctx):
    """Unfused GGUF-layout weights (q, k, v, up, gate separate, as in the file)."""
    d, H, Hk, D, F, V = cfg["d"], cfg["H"], cfg["Hk"], cfg["D"], cfg["F"], cfg["V"]

    def W(rows, cols, s, wt=wtype, std=0.02):
        if wt == wk.Q8_0:
            return orc.gen_q8_0(rows, cols, s, std)
        if wt == wk.Q4_0:
            return orc.gen_q4_0(rows, cols, s, std)
        return orc.gen_f16(rows * cols, s, std)

    layers = []
    for l in range(cfg["L"]):
        s = seed + 100 * l
        layers.append(dict(attn_norm=np.ones(d, np.float32), ffn_norm=np.ones(d, np.float32),
                           q=W(H * D, d, s + 1), k=W(Hk * D, d, s + 2), v=W(Hk * D, d, s + 3), o=W(d, d, s + 4),
                           up=W(F, d, s + 5), gate=W(F, d, s + 6), down=W(d, F, s + 7)))
    return dict(layers=layers, token_embd=W(V, d, seed + 90001, embd_type, 1.0), output=W(V, d, seed + 90002, out_type),
                output_norm=np.ones(d, np.float32), freqs=orc.make_freqs(D, ctx, cfg["theta"]))


def fused_for_oracle(w):
    """llama.go:80-112 fusion (row concatenation of raw bytes) for the oracle."""
    layers = [dict(attn_norm=l["attn_norm"], ffn_norm=l["ffn_norm"], o=l["o"], down=l["down"],
                   qkv=np.concatenate([l["q"], l["k"], l["v"]]), fc=np.concatenate([l["up"], l["gate"]]))
              for l in w["layers"]]
    return dict(layers=layers, token_embd=w["token_embd"], output=w["output"], output_norm=w["output_norm"],
                freqs=w["freqs"])


def oracle_model(w, cfg, wtype, out_type, embd_type, ctx):
    c = dict(L=cfg["L"], d=cfg["d"], H=cfg["H"], Hk=cfg["Hk"], D=cfg["D"], F=cfg["F"], V=cfg["V"], eps=cfg["eps"],
             wtype=wtype, out_type=out_type, embd_type=embd_type)
    return orc.Llama(fused_for_oracle(w), c, ctx)


class DeviceModel:
    """Weights uploaded once; used by the engine and the host mirror."""

    def __init__(self, w):
        self.ptrs = []
        self.layers = []
        for l in w["layers"]:
            self.layers.append({k: self._up(v) for k, v in l.items()})
        self.token_embd = self._up(w["token_embd"])
        self.output = self._up(w["output"])
        self.output_norm = self._up(w["output_norm"])
        self.freqs = self._up(w["freqs"])
        self.fused = []

    def _up(self, a):
        p = up(a)
        self.ptrs.append(p)
        return p

    def free(self):
        for p in self.ptrs + self.fused:
            wk.lib().cuda_free(p)
        self.ptrs, self.fused = [], []


def build_engine(dm, w, cfg, wtype, out_type, embd_type, max_batch, ctx):
    L = wk.lib()
    c = wk.WKConfig(cfg["L"], cfg["d"], cfg["H"], cfg["Hk"], cfg["D"], cfg["F"], cfg["V"], cfg["eps"], wtype, out_type,
                    embd_type)
    m = L.wk_model_create(ctypes.byref(c))
    assert m, L.wk_last_error()
    fw = fused_for_oracle(w)
    for i, l in enumerate(fw["layers"]):
        qkv, fc = up(l["qkv"]), up(l["fc"])
        dm.fused += [qkv, fc]
        wk.check(L.wk_model_set_layer(m, i, dm.layers[i]["attn_norm"], qkv, dm.layers[i]["o"],
                                      dm.layers[i]["ffn_norm"], fc, dm.layers[i]["down"]))
    wk.check(L.wk_model_set_head(m, dm.token_embd, dm.output_norm, dm.output, dm.freqs, ctx))
    wk.check(L.wk_model_alloc_cache(m, max_batch, ctx))
    return m


def host_mirror(dm, cfg, wtype, out_type, embd_type, ctx, lib_handle=None, abi_lib=None):
    """wk_host_llama bound to a cuda.h library (default: this one)."""
    L = wk.lib()
    table = ctypes.create_string_buffer(wk.WK_ABI_SIZE)
    handle = lib_handle if lib_handle is not None else L._handle
    rc = L.wk_abi_bind(table, handle)
    assert rc == 0, L.wk_host_last_error()
    hc = wk.WKHostConfig(cfg["L"], cfg["d"], cfg["H"], cfg["Hk"], cfg["D"], cfg["F"], cfg["V"], ctx, cfg["eps"],
                         cfg["theta"], wtype, out_type, embd_type)
    h = L.wk_host_llama_create(table, ctypes.byref(hc))
    layers = (wk.WKHostLayer * cfg["L"])()
    for i, l in enumerate(dm.layers):
        for k in ("attn_norm", "q", "k", "v", "o", "ffn_norm", "up", "gate", "down"):
            setattr(layers[i], k, l[k])
    rc = L.wk_host_llama_setup(h, layers, dm.token_embd, dm.output_norm, dm.output, None)
    assert rc == 0, L.wk_host_last_error()
    return h, table
