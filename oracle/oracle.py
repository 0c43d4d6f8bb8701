"""ctypes front-end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module.  It wraps ``oracle/liboracle.so`` (a C++ restatement of the
reference's cuda.cu semantics, see oracle.cpp) with numpy-facing helpers.

Activations cross this boundary as float32 arrays whose values lie on the grid
of the activation type (F32 / F16 / BF16); ``to_act``/``from_act`` convert raw
fp16/bf16 buffers.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libwukong_ref.so")

F32, F16, Q4_0, Q8_0, BF16 = 0, 1, 2, 8, 30


def build():
    subprocess.check_call(["make", "-s", "-C", HERE])


def _load():
    if not os.path.exists(LIB_PATH):
        build()
    lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_LOCAL)
    P, I, F, L = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
    sig = {
        "orc_round": (F, [I, F]),
        "orc_dequant_q8_0": (None, [P, P, I, I, I]),
        "orc_matmul": (None, [P, P, P, P, I, I, I, I, I]),
        "orc_rmsnorm": (None, [P, P, P, I, I, F, I]),
        "orc_rope_qkv": (None, [P, P, I, I, I, I, I, I, I]),
        "orc_rope": (None, [P, P, I, I, I, I, I]),
        "orc_swiglu": (None, [P, P, I, I, I]),
        "orc_add": (None, [P, P, P, L, I]),
        "orc_div": (None, [P, P, P, L]),
        "orc_softmax": (None, [P, P, I, I]),
        "orc_gqa_sdpa": (None, [P, P, I, I, I, I, I, I]),
        "orc_get_row": (None, [P, P, I, I, I, I]),
        "orc_argmax": (None, [P, P, I, I, I]),
        "orc_sample": (None, [P, P, P, I, I, F, I, F, ctypes.c_uint64, P]),
        "orc_gen_q4_0": (None, [P, I, I, ctypes.c_uint64, F]),
        "orc_quantize_q4_0": (None, [P, P, I, I]),
        "orc_dequant_q4_0": (None, [P, P, I, I, I]),
        "orc_embedding": (None, [P, P, P, I, I, I]),
        "orc_gqa_layer": (None, [P, P, P, P, P, I, I, I, I, I, I, F, I, I, P, P, I]),
        "orc_ffn_layer": (None, [P, P, P, P, I, I, I, I, F, I, I]),
        "orc_classify": (None, [P, P, P, P, I, I, I, I, F, I, I]),
        "orc_gen_normal": (None, [P, L, ctypes.c_uint64, F]),
        "orc_gen_q8_0": (None, [P, I, I, ctypes.c_uint64, F]),
        "orc_gen_f16": (None, [P, L, ctypes.c_uint64, F]),
        "orc_quantize_q8_0": (None, [P, P, I, I]),
        "orc_make_freqs": (None, [P, P, I, I, F]),
        "orc_num_threads": (I, []),
        "orc_set_threads": (None, [I]),
        "orc_set_f32_tf32": (None, [I]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def act_of(wtype):
    """Activation type the reference uses for a weight dtype (cuda.cu:1324-1338)."""
    return {F32: F32, BF16: BF16}.get(wtype, F16)


def round_act(x, act):
    x = _f32(x).copy()
    if act == F16:
        return x.astype(np.float16).astype(np.float32)
    if act == BF16:
        u = x.view(np.uint32).astype(np.uint64)
        u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
        return u.astype(np.uint32).view(np.float32)
    return x


# ---------------------------------------------------------------- ops
def dequant_q8_0(blocks, rows, cols, out_half=False):
    out = np.empty((rows, cols), np.float32)
    lib().orc_dequant_q8_0(_p(out), _p(np.ascontiguousarray(blocks, np.uint8)), rows, cols, int(out_half))
    return out


def matmul(x, w, bias, M, K, N, wtype, act):
    out = np.empty((M, N), np.float32)
    lib().orc_matmul(_p(out), _p(_f32(x)), _p(np.ascontiguousarray(w)),
                     _p(None if bias is None else _f32(bias)), M, K, N, wtype, act)
    return out


def rmsnorm(x, w, rows, C, eps, act):
    out = np.empty((rows, C), np.float32)
    lib().orc_rmsnorm(_p(out), _p(_f32(x)), _p(_f32(w)), rows, C, eps, act)
    return out


def rope_qkv(qkv, freqs, batch, row, NH, kvNH, HS, act, pos0=0):
    q = _f32(qkv).copy()
    lib().orc_rope_qkv(_p(q), _p(_f32(freqs)), batch, row, pos0, NH, kvNH, HS, act)
    return q


def rope(x, freqs, batch, row, NH, HS, act):
    q = _f32(x).copy()
    lib().orc_rope(_p(q), _p(_f32(freqs)), batch, row, NH, HS, act)
    return q


def swiglu(inp, rows, C, act):
    out = np.empty((rows, C), np.float32)
    lib().orc_swiglu(_p(out), _p(_f32(inp)), rows, C, act)
    return out


def add(a, b, act):
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    lib().orc_add(_p(out), _p(a), _p(b), a.size, act)
    return out


def div(a, b):
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    lib().orc_div(_p(out), _p(a), _p(b), a.size)
    return out


def softmax(x, rows, cols):
    out = np.empty((rows, cols), np.float32)
    lib().orc_softmax(_p(out), _p(_f32(x)), rows, cols)
    return out


def gqa_sdpa(qkv, batch, row, NH, kvNH, HS, act):
    out = np.empty((batch, row, NH * HS), np.float32)
    lib().orc_gqa_sdpa(_p(out), _p(_f32(qkv)), batch, row, NH, kvNH, HS, act)
    return out


def decode_attention(q, kpool, vpool, block_table, seq, pos, NH, kvNH, HS, act):
    """Attention of the newest token of each sequence over its cached keys,
    with the rounding points of cuda.cu:767-852 and the softmax of :673-765:
    s_j = T(q . k_j), e_j = exp(s_j / sqrt(HS) - max), sum of the unrounded
    e_j, P_j = T(T(e_j) * (1 / sum)), o = T(sum_j P_j v_j).  q: [rows, NH * HS];
    kpool / vpool: [pages, kvNH, 64, HS] (values on the grid of `act`);
    block_table: [seqs, max_pages].  Products and sums in float64 before each
    rounding point."""
    rows = q.shape[0]
    G = NH // kvNH
    scale = np.float32(1.0 / np.sqrt(np.float32(HS)))
    out = np.zeros((rows, NH * HS), np.float32)
    for r in range(rows):
        L = int(pos[r]) + 1
        pages = block_table[seq[r], :(L + 63) // 64]
        K = kpool[pages].transpose(1, 0, 2, 3).reshape(kvNH, -1, HS)[:, :L].astype(np.float64)
        V = vpool[pages].transpose(1, 0, 2, 3).reshape(kvNH, -1, HS)[:, :L].astype(np.float64)
        for h in range(kvNH):
            qg = q[r, h * G * HS:(h + 1) * G * HS].reshape(G, HS).astype(np.float64)
            s = round_act((qg @ K[h].T).astype(np.float32), act)
            x = s * scale
            e = np.exp((x - x.max(axis=1, keepdims=True)).astype(np.float64)).astype(np.float32)
            tot = e.astype(np.float64).sum(axis=1, keepdims=True).astype(np.float32)
            P = round_act(round_act(e, act) * (np.float32(1.0) / tot), act)
            out[r, h * G * HS:(h + 1) * G * HS] = round_act((P.astype(np.float64) @ V[h]).astype(np.float32),
                                                           act).ravel()
    return out


def get_row(x, batch, row, col, idx):
    out = np.empty((batch, col), np.float32)
    lib().orc_get_row(_p(out), _p(_f32(x)), batch, row, col, idx)
    return out


def argmax(x, rows, cols, pack):
    out = np.empty(rows, np.int32)
    lib().orc_argmax(_p(out), _p(_f32(x)), rows, cols, pack)
    return out


def sample(logits, temperature, top_k, top_p, seed, steps):
    """Tokens drawn per row (the library's sampling rule, restated); also
    returns per row (u / c_m, distance of u to the nearest prefix-sum boundary
    relative to c_m)."""
    x = _f32(logits)
    rows, V = x.shape
    out = np.empty(rows, np.int32)
    u = np.empty((rows, 2), np.float32)
    st = np.ascontiguousarray(np.broadcast_to(np.asarray(steps, np.int64), (rows,)))
    lib().orc_sample(_p(out), _p(u), _p(x), rows, V, temperature, top_k, top_p, seed, _p(st))
    return out, u


def embedding(ids, table, col, dtype):
    ids = np.ascontiguousarray(ids, np.int32)
    out = np.empty((ids.size, col), np.float32)
    lib().orc_embedding(_p(out), _p(ids), _p(np.ascontiguousarray(table)), ids.size, col, dtype)
    return out


def gen_q8_0(rows, cols, seed, std=0.02):
    out = np.empty(rows * cols // 32 * 34, np.uint8)
    lib().orc_gen_q8_0(_p(out), rows, cols, seed, std)
    return out


def gen_q4_0(rows, cols, seed, std=0.02):
    out = np.empty(rows * cols // 32 * 18, np.uint8)
    lib().orc_gen_q4_0(_p(out), rows, cols, seed, std)
    return out


def quantize_q4_0(x, rows, cols):
    out = np.empty(rows * cols // 32 * 18, np.uint8)
    lib().orc_quantize_q4_0(_p(out), _p(_f32(x)), rows, cols)
    return out


def dequant_q4_0(blocks, rows, cols, out_half=False):
    out = np.empty((rows, cols), np.float32)
    lib().orc_dequant_q4_0(_p(out), _p(np.ascontiguousarray(blocks, np.uint8)), rows, cols, int(out_half))
    return out


def gen_f16(n, seed, std=0.02):
    out = np.empty(n, np.uint16)
    lib().orc_gen_f16(_p(out), n, seed, std)
    return out


def gen_normal(n, seed, std=1.0):
    out = np.empty(n, np.float32)
    lib().orc_gen_normal(_p(out), n, seed, std)
    return out


def quantize_q8_0(x, rows, cols):
    out = np.empty(rows * cols // 32 * 34, np.uint8)
    lib().orc_quantize_q8_0(_p(out), _p(_f32(x)), rows, cols)
    return out


def make_freqs(HS, ctx, theta, factor=None):
    out = np.empty((ctx, HS), np.float32)
    lib().orc_make_freqs(_p(out), _p(None if factor is None else _f32(factor)), HS, ctx, theta)
    return out


def set_threads(n):
    lib().orc_set_threads(int(n))


def num_threads():
    return lib().orc_num_threads()


# ---------------------------------------------------------------- model
class Llama:
    """Llama-3 forward restated from llama.go:117-154 with the layer drivers of
    cuda.cu:902-990; keeps a KV cache so that decode steps compute only the new
    rows (per-row results equal the reference's full recompute)."""

    def __init__(self, w, cfg, max_ctx):
        self.w, self.cfg = w, cfg
        L, Hk, D = cfg["L"], cfg["Hk"], cfg["D"]
        self.act = act_of(cfg["wtype"])
        self.cap = max_ctx
        self.B = None
        self.kc = self.vc = None
        self.pos = 0

    def reset(self, B):
        c = self.cfg
        self.B = B
        self.kc = [np.zeros((B, c["Hk"], self.cap, c["D"]), np.float32) for _ in range(c["L"])]
        self.vc = [np.zeros((B, c["Hk"], self.cap, c["D"]), np.float32) for _ in range(c["L"])]
        self.pos = 0

    def forward(self, ids):
        """ids: [B, n] new tokens at positions pos..pos+n-1.  Returns (tokens, logits)."""
        c, w = self.cfg, self.w
        ids = np.ascontiguousarray(ids, np.int32)
        B, n = ids.shape
        d = c["d"]
        x = embedding(ids.reshape(-1), w["token_embd"], d, c["embd_type"])
        x = round_act(x, self.act).reshape(B, n, d)
        for l in range(c["L"]):
            lw = w["layers"][l]
            lib().orc_gqa_layer(_p(x), _p(w["freqs"]), _p(lw["attn_norm"]), _p(lw["qkv"]), _p(lw["o"]),
                                B, n, self.pos, c["H"], c["Hk"], c["D"], c["eps"], c["wtype"], self.act,
                                _p(self.kc[l]), _p(self.vc[l]), self.cap)
            lib().orc_ffn_layer(_p(x), _p(lw["ffn_norm"]), _p(lw["fc"]), _p(lw["down"]),
                                B, n, d, c["F"], c["eps"], c["wtype"], self.act)
        self.pos += n
        logits = np.empty((B, c["V"]), np.float32)
        lib().orc_classify(_p(logits), _p(x), _p(w["output_norm"]), _p(w["output"]), B, n, d, c["V"],
                           c["eps"], c["out_type"], self.act)
        pack = 4 if self.act == F32 else 8
        return argmax(logits, B, c["V"], pack), logits, x
