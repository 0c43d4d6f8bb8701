"""Tensor-parallel sharding of GGUF weights (host side of include/wukong_ext.h's
TP engine).

Megatron-style split of a Llama-3 layer across `world` ranks of one node, on
raw GGUF bytes (no dequantisation, so every rank streams exactly the bytes the
single-GPU path would):

* q|k|v (fused as in llm/llama.go:80-112): rank r keeps q heads
  [r*H/world, (r+1)*H/world) and k, v heads [r*Hk/world, (r+1)*Hk/world)
  -- column-parallel, attention stays local;
* o [d, H*D]: the K-columns of those q heads -- row-parallel, fp32 partials;
* up|gate: up rows [r*F/world, ...) then the same gate rows -- column-parallel,
  SwiGLU stays local;
* down [d, F]: the K-columns r*F/world.. -- row-parallel;
* output [V, d]: vocabulary rows r*V/world.. -- logits and a winner exchange.

Q8_0 rows are [K/32 blocks of 34 bytes]; a K-slice is a slice of whole blocks,
so K/world must be a multiple of 32 for Q8_0 (16 for 16-bit types).
"""
import numpy as np

F32, F16, Q8_0, BF16 = 0, 1, 8, 30


def _as_rows(w, rows, cols, wtype):
    """Raw weight bytes as [rows, blocks, block_bytes] (Q8_0) or [rows, cols]."""
    if wtype == Q8_0:
        return np.asarray(w).view(np.uint8).reshape(rows, cols // 32, 34)
    if wtype in (F16, BF16):
        return np.asarray(w).view(np.uint16).reshape(rows, cols)
    return np.asarray(w).view(np.float32).reshape(rows, cols)


def row_slice(w, rows, cols, wtype, r0, r1):
    """Rows [r0, r1) of a [rows, cols] weight, in its storage type."""
    return np.ascontiguousarray(_as_rows(w, rows, cols, wtype)[r0:r1]).reshape(-1)


def col_slice(w, rows, cols, wtype, c0, c1):
    """Columns (the K dimension) [c0, c1) of a [rows, cols] weight."""
    if wtype == Q8_0:
        if c0 % 32 or c1 % 32:
            raise ValueError(f"Q8_0 K-slice [{c0}, {c1}) must start and end on 32-element blocks")
        return np.ascontiguousarray(_as_rows(w, rows, cols, wtype)[:, c0 // 32:c1 // 32]).reshape(-1)
    return np.ascontiguousarray(_as_rows(w, rows, cols, wtype)[:, c0:c1]).reshape(-1)


def check_divisible(cfg, world, wtype):
    """Raise unless the model splits evenly over `world` ranks."""
    H, Hk, F, V, D = cfg["H"], cfg["Hk"], cfg["F"], cfg["V"], cfg["D"]
    for name, n in (("n_heads", H), ("n_kv_heads", Hk), ("ffn", F), ("vocab", V)):
        if n % world:
            raise ValueError(f"{name}={n} is not divisible by the tensor-parallel degree {world}")
    blk = 32 if wtype == Q8_0 else 16
    for name, k in (("o K-slice", H // world * D), ("down K-slice", F // world)):
        if k % blk:
            raise ValueError(f"{name} of {k} columns is not a multiple of {blk}")


def local_config(cfg, world):
    """Per-rank counts of a sharded model (d_model, head_dim, layers unchanged)."""
    c = dict(cfg)
    c["H"], c["Hk"], c["F"], c["V"] = cfg["H"] // world, cfg["Hk"] // world, cfg["F"] // world, cfg["V"] // world
    return c


def shard_layer(layer, cfg, wtype, rank, world):
    """One rank's share of a layer given its unfused GGUF tensors (q, k, v, o,
    up, gate, down, attn_norm, ffn_norm); returns the fused qkv / fc shards the
    engine takes plus o / down K-slices and the (whole) norms."""
    d, H, Hk, D, F = cfg["d"], cfg["H"], cfg["Hk"], cfg["D"], cfg["F"]
    h, hk, f = H // world, Hk // world, F // world
    q = row_slice(layer["q"], H * D, d, wtype, rank * h * D, (rank + 1) * h * D)
    k = row_slice(layer["k"], Hk * D, d, wtype, rank * hk * D, (rank + 1) * hk * D)
    v = row_slice(layer["v"], Hk * D, d, wtype, rank * hk * D, (rank + 1) * hk * D)
    up = row_slice(layer["up"], F, d, wtype, rank * f, (rank + 1) * f)
    gate = row_slice(layer["gate"], F, d, wtype, rank * f, (rank + 1) * f)
    return dict(attn_norm=layer["attn_norm"], ffn_norm=layer["ffn_norm"],
                qkv=np.concatenate([q, k, v]), fc=np.concatenate([up, gate]),
                o=col_slice(layer["o"], d, H * D, wtype, rank * h * D, (rank + 1) * h * D),
                down=col_slice(layer["down"], d, F, wtype, rank * f, (rank + 1) * f))


def shard_output(output, cfg, out_type, rank, world):
    """Vocabulary rows of output.weight for one rank."""
    V, d = cfg["V"], cfg["d"]
    v = V // world
    return row_slice(output, V, d, out_type, rank * v, (rank + 1) * v)
