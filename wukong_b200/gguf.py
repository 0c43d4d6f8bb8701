"""GGUF files: read a Llama-3 checkpoint straight into one rank's engine
weights (the host side of the reference's loader, llm/parser.go:146-201 and
:529-546, and of its tensor fusion, llm/llama.go:69-115).

The reference maps the whole file, copies every tensor to the device with one
cudaMemcpyAsync each and then concatenates q|k|v and up|gate on the device
(cuda_cat).  Here each rank reads only the bytes of its own shard from the
mapping -- rows of q/k/v/up/gate, whole Q8_0 blocks of o/down columns,
vocabulary rows of output.weight (the wukong_b200.tp split) -- assembles the
fused q|k|v and up|gate rows on the host, and copies each resulting tensor to
the device with one host-to-device copy (no device-side concatenation, and no
rank ever copies another rank's bytes).

Format (GGUF version 3, little endian): magic "GGUF", u32 version, u64 tensor
count, u64 metadata count; metadata (string key, u32 type, value); tensor
infos (string name, u32 n_dims, u64 dims innermost first, u32 ggml type, u64
offset into the data section); the data section starts at the next multiple
of general.alignment (default 32).  Strings are u64 length + bytes.
"""
import ctypes
import mmap
import struct

import numpy as np

from wukong_b200 import tp

# metadata value types (GGUF)
U8, I8, U16, I16, U32, I32, F32T, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32T: "<f", BOOL: "<?", U64: "<Q",
           I64: "<q", F64: "<d"}
# ggml tensor types: (elements per block, bytes per block)
BLOCK = {0: (1, 4), 1: (1, 2), 2: (32, 18), 8: (32, 34), 30: (1, 2)}
DEFAULT_ALIGNMENT = 32


class GGUFFile:
    """A memory-mapped GGUF file: metadata, tensor infos and raw tensor bytes."""

    def __init__(self, path):
        self.path = path
        self._f = open(path, "rb")
        self.mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self.pos = 0
        magic = self._read(4)
        if magic != b"GGUF":
            raise ValueError(f"invalid magic number: expected 'GGUF', got {magic!r}")
        version, n_tensors, n_kv = struct.unpack("<IQQ", self._read(20))
        if version != 3:
            raise ValueError(f"unsupported version: expected 3, got {version}")
        self.kv = {}
        for _ in range(n_kv):
            key = self._string()
            (vt,) = struct.unpack("<I", self._read(4))
            self.kv[key] = self._value(vt)
        self.tensors = {}
        for _ in range(n_tensors):
            name = self._string()
            (nd,) = struct.unpack("<I", self._read(4))
            dims = list(struct.unpack(f"<{nd}Q", self._read(8 * nd)))
            ttype, off = struct.unpack("<IQ", self._read(12))
            # dims are stored innermost first; [rows, cols] as the reference reverses them (parser.go:433)
            self.tensors[name] = dict(dims=dims[::-1], type=ttype, offset=off)
        align = int(self.kv.get("general.alignment", DEFAULT_ALIGNMENT))
        self.data = (self.pos + align - 1) // align * align

    def _read(self, n):
        b = self.mm[self.pos:self.pos + n]
        if len(b) != n:
            raise ValueError("truncated GGUF file")
        self.pos += n
        return b

    def _string(self):
        (n,) = struct.unpack("<Q", self._read(8))
        return self._read(n).decode("utf-8")

    def _value(self, vt):
        if vt in _SCALAR:
            fmt = _SCALAR[vt]
            return struct.unpack(fmt, self._read(struct.calcsize(fmt)))[0]
        if vt == STRING:
            return self._string()
        if vt == ARRAY:
            et, n = struct.unpack("<IQ", self._read(12))
            return [self._value(et) for _ in range(n)]
        raise ValueError(f"unknown metadata type {vt}")

    def nbytes(self, name):
        t = self.tensors[name]
        n = int(np.prod(t["dims"]))
        per, size = BLOCK[t["type"]]
        return n // per * size

    def raw(self, name):
        """The tensor's bytes as a read-only uint8 array over the mapping."""
        t = self.tensors[name]
        start = self.data + t["offset"]
        return np.frombuffer(self.mm, np.uint8, self.nbytes(name), start)

    def close(self):
        # arrays returned by raw() keep the mapping alive; it is released with the last of them
        try:
            self.mm.close()
        except BufferError:
            pass
        self._f.close()


def write_gguf(path, kv, tensors, alignment=DEFAULT_ALIGNMENT):
    """Write a GGUF v3 file.  kv: {key: (type, value)}; tensors: {name: (ggml
    type, [rows, cols] or [n], raw bytes)} in order."""
    def s(x):
        b = x.encode("utf-8")
        return struct.pack("<Q", len(b)) + b

    def val(vt, v):
        if vt in _SCALAR:
            return struct.pack(_SCALAR[vt], v)
        if vt == STRING:
            return s(v)
        if vt == ARRAY:
            et, items = v
            return struct.pack("<IQ", et, len(items)) + b"".join(val(et, i) for i in items)
        raise ValueError(vt)

    kv = dict(kv)
    kv.setdefault("general.alignment", (U32, alignment))
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv))
    for k, (vt, v) in kv.items():
        head += s(k) + struct.pack("<I", vt) + val(vt, v)
    blobs = {name: bytes(np.ascontiguousarray(data).view(np.uint8)) for name, (tt, dims, data) in tensors.items()}
    offs, off = [], 0
    for name in tensors:
        offs.append(off)
        off += (len(blobs[name]) + alignment - 1) // alignment * alignment
    for (name, (tt, dims, data)), o in zip(tensors.items(), offs):
        head += s(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims[::-1])
        head += struct.pack("<IQ", tt, o)
    pad = (len(head) + alignment - 1) // alignment * alignment - len(head)
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        for name in tensors:
            b = blobs[name]
            f.write(b + b"\0" * ((len(b) + alignment - 1) // alignment * alignment - len(b)))


def llama_config(g):
    """Llama-3 shapes from the metadata (llama.* keys) and the tensor shapes."""
    arch = g.kv.get("general.architecture", "llama")
    L = int(g.kv[f"{arch}.block_count"])
    d = int(g.kv[f"{arch}.embedding_length"])
    H = int(g.kv[f"{arch}.attention.head_count"])
    Hk = int(g.kv.get(f"{arch}.attention.head_count_kv", H))
    F = int(g.kv[f"{arch}.feed_forward_length"])
    V = g.tensors["token_embd.weight"]["dims"][0]
    return dict(L=L, d=d, H=H, Hk=Hk, D=d // H, F=F, V=V, eps=float(g.kv.get(f"{arch}.attention.layer_norm_rms_epsilon",
                                                                               1e-5)),
                theta=float(g.kv.get(f"{arch}.rope.freq_base", 500000.0)))


def shard_host(g, cfg, rank=0, world=1):
    """One rank's weights read from the mapping (host arrays): per layer
    attn_norm, qkv (fused), o, ffn_norm, fc (fused), down; and token_embd,
    output_norm, output (output.weight, or the embeddings when absent as in
    llama.go:75-78), plus the dtypes."""
    wt = g.tensors["blk.0.attn_q.weight"]["type"]
    out_name = "output.weight" if "output.weight" in g.tensors else "token_embd.weight"
    out_type = g.tensors[out_name]["type"]
    if world > 1:
        tp.check_divisible(cfg, world, wt)
    layers = []
    for l in range(cfg["L"]):
        b = f"blk.{l}."
        raw = {k: g.raw(b + n + ".weight") for k, n in (("q", "attn_q"), ("k", "attn_k"), ("v", "attn_v"),
                                                          ("o", "attn_output"), ("up", "ffn_up"),
                                                          ("gate", "ffn_gate"), ("down", "ffn_down"))}
        raw["attn_norm"] = g.raw(b + "attn_norm.weight").view(np.float32)
        raw["ffn_norm"] = g.raw(b + "ffn_norm.weight").view(np.float32)
        if world > 1:
            layers.append(tp.shard_layer(raw, cfg, wt, rank, world))
        else:
            layers.append(dict(attn_norm=raw["attn_norm"], ffn_norm=raw["ffn_norm"], o=raw["o"], down=raw["down"],
                               qkv=np.concatenate([raw["q"], raw["k"], raw["v"]]),
                               fc=np.concatenate([raw["up"], raw["gate"]])))
    out = g.raw(out_name)
    if world > 1:
        out = tp.shard_output(out, cfg, out_type, rank, world)
    return dict(layers=layers, token_embd=g.raw("token_embd.weight"), output=out,
                output_norm=g.raw("output_norm.weight").view(np.float32),
                wtype=wt, out_type=out_type, embd_type=g.tensors["token_embd.weight"]["type"])


def load_to_device(g, cfg, rank=0, world=1):
    """shard_host(), then one host-to-device copy (cuda_to_device) per tensor.
    Returns (device pointers in shard_host's layout, list of all pointers)."""
    import wukong_b200 as wk
    L = wk.lib()
    h = shard_host(g, cfg, rank, world)
    ptrs = []

    def up(a):
        a = np.ascontiguousarray(a)
        p = L.cuda_malloc(max(a.nbytes, 16))
        ptrs.append(p)
        L.cuda_to_device(p, a.ctypes.data_as(ctypes.c_void_p), a.nbytes)
        return p

    dev = dict(layers=[{k: up(v) for k, v in lw.items()} for lw in h["layers"]],
               token_embd=up(h["token_embd"]), output=up(h["output"]), output_norm=up(h["output_norm"]),
               wtype=h["wtype"], out_type=h["out_type"], embd_type=h["embd_type"])
    return dev, ptrs
