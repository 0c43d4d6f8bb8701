"""GGUF load path (llm/parser.go:146-201, :529-546 of the reference): a GGUF v3
file written here is parsed back (metadata, tensor infos, bytes), each rank's
shard is read straight from the mapping and equals wukong_b200.tp's split of
the same tensors, and a model loaded from the file decodes the same tokens as
the same weights loaded from memory."""
import ctypes
import os

import numpy as np
import pytest

import wukong_b200 as wk
from wukong_b200 import gguf, tp
from tests.model_util import fused_for_oracle, make_weights

CFG = dict(L=2, d=256, H=8, Hk=4, D=32, F=512, V=1024, eps=1e-5, theta=500000.0)


def _write(path, cfg, w, wt=wk.Q8_0, with_output=True):
    kv = {"general.architecture": (gguf.STRING, "llama"), "llama.block_count": (gguf.U32, cfg["L"]),
          "llama.embedding_length": (gguf.U32, cfg["d"]), "llama.attention.head_count": (gguf.U32, cfg["H"]),
          "llama.attention.head_count_kv": (gguf.U32, cfg["Hk"]), "llama.feed_forward_length": (gguf.U32, cfg["F"]),
          "llama.rope.freq_base": (gguf.F32T, cfg["theta"]),
          "llama.attention.layer_norm_rms_epsilon": (gguf.F32T, cfg["eps"]),
          "tokenizer.ggml.tokens": (gguf.ARRAY, (gguf.STRING, ["a", "b", "<|end|>"]))}
    d, H, Hk, D, F, V = (cfg[k] for k in ("d", "H", "Hk", "D", "F", "V"))
    t = {"token_embd.weight": (wk.F16, [V, d], w["token_embd"])}
    for l, lw in enumerate(w["layers"]):
        b = f"blk.{l}."
        t[b + "attn_norm.weight"] = (wk.F32, [d], lw["attn_norm"])
        t[b + "attn_q.weight"] = (wt, [H * D, d], lw["q"])
        t[b + "attn_k.weight"] = (wt, [Hk * D, d], lw["k"])
        t[b + "attn_v.weight"] = (wt, [Hk * D, d], lw["v"])
        t[b + "attn_output.weight"] = (wt, [d, H * D], lw["o"])
        t[b + "ffn_norm.weight"] = (wk.F32, [d], lw["ffn_norm"])
        t[b + "ffn_up.weight"] = (wt, [F, d], lw["up"])
        t[b + "ffn_gate.weight"] = (wt, [F, d], lw["gate"])
        t[b + "ffn_down.weight"] = (wt, [d, F], lw["down"])
    t["output_norm.weight"] = (wk.F32, [d], w["output_norm"])
    if with_output:
        t["output.weight"] = (wt, [V, d], w["output"])
    gguf.write_gguf(path, kv, t)


def test_gguf_round_trip(tmp_path):
    w = make_weights(CFG, wk.Q8_0, wk.Q8_0, wk.F16, seed=3, ctx=16)
    p = str(tmp_path / "m.gguf")
    _write(p, CFG, w)
    g = gguf.GGUFFile(p)
    assert g.kv["llama.block_count"] == 2 and g.kv["tokenizer.ggml.tokens"] == ["a", "b", "<|end|>"]
    assert abs(g.kv["llama.rope.freq_base"] - 500000.0) < 1e-3
    assert g.tensors["blk.1.ffn_down.weight"]["dims"] == [CFG["d"], CFG["F"]]
    assert g.data % 32 == 0
    assert np.array_equal(g.raw("blk.1.attn_k.weight"), w["layers"][1]["k"])
    assert np.array_equal(g.raw("token_embd.weight").view(np.uint16), w["token_embd"])
    cfg = gguf.llama_config(g)
    assert {k: cfg[k] for k in ("L", "d", "H", "Hk", "D", "F", "V")} == {k: CFG[k] for k in ("L", "d", "H", "Hk", "D",
                                                                                              "F", "V")}
    g.close()


def test_gguf_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUG" + b"\0" * 60)
    with pytest.raises(ValueError, match="magic"):
        gguf.GGUFFile(str(p))
    p.write_bytes(b"GGUF" + (2).to_bytes(4, "little") + b"\0" * 60)
    with pytest.raises(ValueError, match="version"):
        gguf.GGUFFile(str(p))


@pytest.mark.parametrize("world", [1, 2, 4])
def test_gguf_shards_equal_the_tp_split(tmp_path, world):
    w = make_weights(CFG, wk.Q8_0, wk.Q8_0, wk.F16, seed=5, ctx=16)
    p = str(tmp_path / "m.gguf")
    _write(p, CFG, w)
    g = gguf.GGUFFile(p)
    for rank in range(world):
        h = gguf.shard_host(g, CFG, rank, world)
        for l, lw in enumerate(w["layers"]):
            want = tp.shard_layer(lw, CFG, wk.Q8_0, rank, world) if world > 1 else fused_for_oracle(w)["layers"][l]
            for k in ("qkv", "o", "fc", "down", "attn_norm", "ffn_norm"):
                assert np.array_equal(np.asarray(h["layers"][l][k]).view(np.uint8),
                                      np.asarray(want[k]).view(np.uint8)), (rank, l, k)
        want_out = tp.shard_output(w["output"], CFG, wk.Q8_0, rank, world) if world > 1 else w["output"]
        assert np.array_equal(h["output"], want_out)
    g.close()


def test_gguf_tied_output_uses_the_embeddings(tmp_path):
    """Without output.weight the logits use token_embd (llama.go:75-78)."""
    w = make_weights(CFG, wk.F16, wk.F16, wk.F16, seed=6, ctx=16)
    p = str(tmp_path / "m.gguf")
    _write(p, CFG, w, wt=wk.F16, with_output=False)
    g = gguf.GGUFFile(p)
    h = gguf.shard_host(g, CFG)
    assert h["out_type"] == wk.F16 and np.array_equal(h["output"], np.asarray(w["token_embd"]).view(np.uint8))
    g.close()


@pytest.mark.gpu
def test_model_from_gguf_decodes_like_the_same_weights(dev, tmp_path):
    from tests.gpu_util import down, free, up
    from wukong_b200.engine import Engine, make_freqs
    w = make_weights(CFG, wk.Q8_0, wk.Q8_0, wk.F16, seed=8, ctx=40)
    p = str(tmp_path / "m.gguf")
    _write(p, CFG, w)
    g = gguf.GGUFFile(p)
    dv, ptrs = gguf.load_to_device(g, CFG)
    fr = up(make_freqs(CFG["D"], 40, CFG["theta"]))

    def run(layers, embd, onorm, out):
        e = Engine(CFG, layers, embd, onorm, out, fr, 40, max_batch=2)
        ids = up(np.random.default_rng(1).integers(0, CFG["V"], size=(2, 9)).astype(np.int32))
        e.prefill(ids, 2, 9)
        toks = [down(e.tokens_ptr(), 2, np.int32).tolist()]
        for _ in range(5):
            e.step()
            toks.append(down(e.tokens_ptr(), 2, np.int32).tolist())
        e.destroy()
        free(ids)
        return toks

    got = run(dv["layers"], dv["token_embd"], dv["output_norm"], dv["output"])
    fw = fused_for_oracle(w)
    mem = [{k: up(v) for k, v in lw.items()} for lw in fw["layers"]]
    extra = [up(w["token_embd"]), up(w["output_norm"]), up(w["output"])]
    want = run(mem, *extra)
    free(fr, *ptrs, *extra, *[v for lw in mem for v in lw.values()])
    g.close()
    assert got == want
