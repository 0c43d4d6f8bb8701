"""GPU parity of every C ABI entry point: the reference's own known-answer
vectors (test_cuda.cu / array_test.go, replayed through the same calls) and the
CPU oracle on seeded random inputs.

Tolerances: the reference's 1e-5 absolute for its fp32 vectors; for fp16/bf16
paths a normwise relative error <= 1e-3 with fp32 accumulation (the bar stated
for matmul, attention and logits), and Q8_0 dequantisation bit-exact.
"""
import ctypes

import numpy as np
import pytest

import wukong_b200 as wk
from oracle import oracle as orc
from tests.gpu_util import alloc, bf16_bits, bf16_to_f32, down, free, h16, rel_err, up

pytestmark = pytest.mark.gpu
F32, F16, Q8_0, BF16 = wk.F32, wk.F16, wk.Q8_0, wk.BF16
KAT_TOL = 1e-5  # test_cuda.cu:9
REL = 1e-3
REL_BF16 = 1e-2  # bf16 keeps 8 mantissa bits: one rounding step is 2^-8 relative


def tol(act):
    return REL_BF16 if act == BF16 else REL


def close(a, b, tol=KAT_TOL):
    # expected values are the reference's float32 literals: compare in float32 terms
    np.testing.assert_allclose(np.asarray(a, np.float32).astype(np.float64).ravel(),
                               np.asarray(b, np.float32).astype(np.float64).ravel(), rtol=0, atol=tol)


def f32(v):
    return np.asarray(v, np.float32)


# ----------------------------------------------------------------- reference KATs
def test_kat_matmul(dev, kat):
    t = kat["test_cuda.cu/cuda_matmul"]
    x, w, b = up(f32(t["inp"])), up(f32(t["weight"])), up(f32(t["bias"]))
    o = alloc(4 * 16)
    dev.cuda_matmul(o, x, w, b, 4, 3, 4, F32)
    close(down(o, 16, np.float32), t["res"])
    dev.cuda_matmul(o, x, w, None, 4, 3, 4, F32)
    close(down(o, 16, np.float32), t["res_nob"])
    free(x, w, b, o)


def test_kat_softmax(dev, kat):
    t = kat["test_cuda.cu/cuda_softmax"]
    x = up(f32(t["inp"]))
    o = alloc(24)
    dev.cuda_softmax(o, x, 2, 3)
    close(down(o, 6, np.float32), t["res"])
    free(x, o)


@pytest.mark.parametrize("name,batch,row,NH,kvNH,HS", [
    ("cuda_mh_sdpa", 2, 4, 1, 1, 2), ("cuda_gq_sdpa", 2, 2, 4, 2, 2), ("cuda_mq_sdpa", 2, 2, 2, 1, 8)])
def test_kat_sdpa(dev, kat, name, batch, row, NH, kvNH, HS):
    t = kat["test_cuda.cu/" + name]
    x = up(f32(t["inp"]))
    n = batch * row * NH * HS
    o = alloc(4 * n)
    if name == "cuda_mh_sdpa":
        dev.cuda_mh_sdpa(o, x, batch, row, NH, HS)
    elif name == "cuda_gq_sdpa":
        dev.cuda_gq_sdpa(o, x, batch, row, NH, kvNH, HS)
    else:
        dev.cuda_mq_sdpa(o, x, batch, row, NH, HS)
    close(down(o, n, np.float32), t["res"])
    # the input is left untouched
    close(down(x, len(t["inp"]), np.float32), t["inp"], 0)
    free(x, o)


def test_kat_rmsnorm_swiglu(dev, kat):
    t = kat["test_cuda.cu/cuda_rmsnorm"]
    x, w = up(f32(t["inp"])), up(f32(t["weight"]))
    o = alloc(64)
    dev.cuda_rmsnorm(o, x, w, 4, 4, 1e-5)
    close(down(o, 16, np.float32), t["res"])
    free(x, w, o)
    t = kat["test_cuda.cu/cuda_swiglu"]
    x, w = up(f32(t["inp"])), up(f32(t["weights_fc"]))
    fc, o = alloc(4 * 32), alloc(4 * 16)
    dev.cuda_matmul(fc, x, w, None, 4, 4, 8, F32)
    dev.cuda_swiglu(o, fc, 2, 2, 4)
    close(down(o, 16, np.float32), t["res"])
    # in place, as feed_forward does (cuda.cu:939)
    dev.cuda_swiglu(fc, fc, 2, 2, 4)
    close(down(fc, 16, np.float32), t["res"])
    free(x, w, fc, o)


def test_kat_rope_qkv(dev, kat):
    t = kat["test_cuda.cu/cuda_rope_qkv"]
    f1 = up(f32(t["fc_res"]))
    q = up(f32(t["qkv"]))
    dev.cuda_rope_qkv(q, q, f1, 1, 2, 2, 1, 2)
    close(down(q, 16, np.float32), t["res"])
    f2 = up(f32(t["fc_res2"]))
    q2 = up(f32(t["qkv2"]))
    dev.cuda_rope_qkv(q2, q2, f2, 1, 2, 1, 1, 4)
    close(down(q2, 24, np.float32), t["res2"])
    free(f1, q, f2, q2)


def test_rope_matches_oracle(dev):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 5, 3, 8)).astype(np.float32)
    f = orc.make_freqs(8, 5, 10000.0)
    px, pf = up(x), up(f)
    o = alloc(x.nbytes)
    dev.cuda_rope(o, px, pf, 2, 5, 3, 8)
    close(down(o, x.shape, np.float32), orc.rope(x, f, 2, 5, 3, 8, F32), 1e-6)
    free(px, pf, o)


def test_kat_embedding(dev, kat):
    t = kat["test_cuda.cu/cuda_embedding"]
    ids, e = up(np.array(t["inp"], np.int32)), up(f32(t["embd"]))
    o = alloc(4 * 32)
    dev.cuda_embedding(o, ids, e, 2, 4, 4, F32)
    close(down(o, 32, np.float32), t["expected"])
    free(ids, e, o)
    g = kat["array_test.go/TestTensorEmbedding"]
    table = up(np.array(g["data"], np.uint8))
    ids = up(np.array([2, 1], np.int32))
    o = alloc(2 * 64)
    dev.cuda_embedding(o, ids, table, 1, 2, 32, Q8_0)
    assert down(o, 64, np.int16).tolist() == g["expected"]
    free(table, ids, o)


def test_kat_cat_div_add_get_row(dev, kat):
    t = kat["test_cuda.cu/cuda_cat"]
    a, b = up(f32(t["a"])), up(f32(t["b"]))
    o = alloc(36)
    dev.cuda_cat(o, a, b, 2, 1, 3, F32)
    close(down(o, 9, np.float32), t["expected"], 0)
    free(a, b, o)
    t = kat["test_cuda.cu/cuda_div"]
    a, b = up(f32(t["a"])), up(f32(t["b"]))
    o = alloc(24)
    dev.cuda_div(o, a, b, 2, 3)
    close(down(o, 6, np.float32), t["expected"], 0)
    free(a, b, o)
    t = kat["test_cuda.cu/cuda_add"]
    a, b = up(f32(t["a"])), up(f32(t["b"]))
    o = alloc(32)
    dev.cuda_add(o, a, b, 2, 4)
    close(down(o, 8, np.float32), t["expected"], 0)
    free(a, b, o)
    t = kat["test_cuda.cu/cuda_get_row"]
    x = up(f32(t["inp"]))
    o = alloc(32)
    for idx, key in ((0, "res0"), (1, "res1"), (2, "res2"), (-1, "res2")):
        dev.cuda_get_row(o, x, 2, 3, 4, idx)
        close(down(o, 8, np.float32), t[key], 0)
    free(x, o)


def test_kat_dequantize_bit_exact(dev, kat):
    t = kat["test_cuda.cu/cuda_dequantize"]
    x = up(np.array(t["inp"], np.uint8))
    o = alloc(4 * 128)
    dev.cuda_dequantize(o, x, 2, 64, Q8_0)
    got = down(o, (2, 64), np.float32)
    close(got, t["expected"])
    assert np.array_equal(got, orc.dequant_q8_0(np.array(t["inp"], np.uint8), 2, 64))
    free(x, o)


def test_dequantize_large_bit_exact(dev):
    """Q8_0 -> fp32 over a 8192 x 2048 weight (array_test.go:618 benchmarks the 128256 x 8192 case)."""
    rows, cols = 8192, 2048
    blocks = orc.gen_q8_0(rows, cols, seed=11)
    x = up(blocks)
    o = alloc(4 * rows * cols)
    dev.cuda_dequantize(o, x, rows, cols, Q8_0)
    assert np.array_equal(down(o, (rows, cols), np.float32), orc.dequant_q8_0(blocks, rows, cols))
    free(x, o)


def test_device_weight_generators_match_the_oracle(dev):
    """The benchmark's weights come from the device generators: Q8_0 blocks and
    F16 values bit-identical to the oracle's host generators."""
    rows, cols = 300, 2048
    nb = rows * cols // 32 * 34
    p = alloc(nb)
    wk.check(dev.wk_fill_random_q8_0(p, rows, cols, 123, 0.02))
    got, want = down(p, nb, np.uint8), orc.gen_q8_0(rows, cols, 123, 0.02)
    bad = np.flatnonzero(got != want)
    assert bad.size == 0, (bad.size, bad[:8].tolist(), got[bad[:8]].tolist(), want[bad[:8]].tolist())
    f = alloc(2 * rows * cols)
    wk.check(dev.wk_fill_random_f16(f, rows * cols, 77, 0.02))
    assert np.array_equal(down(f, rows * cols, np.uint16), orc.gen_f16(rows * cols, 77, 0.02))
    free(p, f)


def test_kat_repeat_qkv(dev, kat):
    t = kat["test_cuda.cu/cuda_repeat_qkv"]
    x = up(f32(t["inp"]))
    o = alloc(4 * 96)
    dev.cuda_repeat_qkv(o, x, 2, 2, 4, 2, 2)
    close(down(o, 96, np.float32), t["res"], 0)
    free(x, o)


def test_kat_group_query_attention(dev, kat):
    t = kat["test_cuda.cu/cuda_group_query_attention"]
    e = up(f32(t["embeds"]))
    fr, nw, qkv, ow = up(f32(t["freqs"])), up(f32(t["norm_weight"])), up(f32(t["qkv_weight"])), up(f32(t["out_weight"]))
    dev.cuda_group_query_attention(e, e, fr, nw, qkv, ow, 2, 2, 2, 1, 4, 1e-5, F32)
    close(down(e, 32, np.float32), t["res"])
    free(e, fr, nw, qkv, ow)


def test_kat_feed_forward(dev, kat):
    t = kat["test_cuda.cu/cuda_feed_forward"]
    a = up(f32(t["attn"]))
    nw, fc, ow = up(f32(t["norm_weight"])), up(f32(t["fc_weight"])), up(f32(t["out_weight"]))
    dev.cuda_feed_forward(a, a, nw, fc, ow, 2, 2, 4, 8, 1e-5, F32)
    close(down(a, 16, np.float32), t["expected"])
    free(a, nw, fc, ow)


def test_kat_classify_argmax_predict(dev, kat):
    t = kat["test_cuda.cu/cuda_classify"]
    ff, nw, ow = up(f32(t["ff"])), up(f32(t["norm_weight"])), up(f32(t["out_weight"]))
    o = alloc(4 * 32)
    dev.cuda_classify(o, ff, nw, ow, 2, 4, 4, 16, 1e-5, F32)
    close(down(o, 32, np.float32), t["expected"])
    dev.cuda_predict(o, ff, nw, ow, 2, 4, 4, 16, 1e-5, F32)
    assert down(o, 2, np.int32).tolist() == [int(v) for v in kat["test_cuda.cu/cuda_predict"]["expected"]]
    free(ff, nw, ow, o)
    t = kat["test_cuda.cu/cuda_argmax"]
    x = up(f32(t["inp"]))
    o = alloc(8)
    dev.cuda_argmax(o, x, 2, 48)
    assert down(o, 2, np.int32).tolist() == t["expected"]
    free(x, o)


def test_kat_go_end_to_end(dev, kat):
    """array_test.go:656-845 through the Tensor mirror of array.go.  The Go vectors
    carry TF32 linear layers (cuBLASLt FAST_TF32); this library's F32 path is exact
    fp32, so the residual is compared at 1e-3 and against the exact oracle at 1e-5."""
    from wukong_b200 import tensor as T
    g = kat["array_test.go/TestEndToEndInference"]
    B, Tn, d, NH, kvNH, HS, F, V = 2, 4, 8, 2, 1, 4, 16, 16
    mk = lambda k, shape: T.make_tensor(shape, f32(g[k]))
    emb = mk("embedding", [V, d])
    ids = T.make_tensor([B, Tn], np.array(g["ids"], np.int32))
    x = emb.embedding(ids)
    x.group_query_attention(mk("freqs", [Tn, HS]), mk("attn_norm", [d]), mk("qkv_weight", [(NH + 2 * kvNH) * HS, d]),
                            mk("attn_out", [d, d]), NH, kvNH, 1e-5)
    x.feed_forward(mk("ff_norm", [d]), mk("ff_weight", [2 * F, d]), mk("ff_out", [d, F]), F, 1e-5)
    got = x.to_host()
    close(got, g["ff_expected"], 1e-3)
    # exact-fp32 oracle
    xo = orc.embedding(np.array(g["ids"]), f32(g["embedding"]), d, F32).reshape(B, Tn, d).copy()
    kc = np.zeros((B, kvNH, Tn, HS), np.float32)
    vc = np.zeros_like(kc)
    L, p = orc.lib(), orc._p
    L.orc_gqa_layer(p(xo), p(f32(g["freqs"])), p(f32(g["attn_norm"])), p(f32(g["qkv_weight"])), p(f32(g["attn_out"])),
                    B, Tn, 0, NH, kvNH, HS, 1e-5, F32, F32, p(kc), p(vc), Tn)
    L.orc_ffn_layer(p(xo), p(f32(g["ff_norm"])), p(f32(g["ff_weight"])), p(f32(g["ff_out"])), B, Tn, d, F, 1e-5, F32, F32)
    close(got, xo, 1e-5)
    assert x.predict(mk("ff_norm", [d]), mk("classifier", [V, d]), V, 1e-5).tolist() == g["expected"]


# ----------------------------------------------------------------- random parity vs oracle
def _weights(wtype, N, K, seed):
    if wtype == Q8_0:
        return orc.gen_q8_0(N, K, seed)
    w = orc.gen_normal(N * K, seed, 0.02)
    return h16(w) if wtype == F16 else bf16_bits(w)


def _acts(act, M, K, seed, std=1.0):
    x = orc.gen_normal(M * K, seed, std).reshape(M, K)
    if act == F16:
        return h16(x), h16(x).astype(np.float32)
    return bf16_bits(x), bf16_to_f32(bf16_bits(x))


def _from_dev(raw, act):
    return raw.astype(np.float32) if act == F16 else bf16_to_f32(raw)


@pytest.mark.parametrize("wtype", [Q8_0, F16, BF16])
@pytest.mark.parametrize("M,N,K", [(1, 8192, 2048), (16, 8192, 2048), (128, 8192, 2048), (5, 2048, 8192),
                                   (3, 97, 256), (8, 70, 160), (2, 48, 4096), (512, 2048, 2048),
                                   (1100, 1024, 4096), (2048, 640, 1024), (32, 2048, 8192), (48, 3072, 2048)])
def test_matmul_vs_oracle(dev, wtype, M, N, K):
    """BASELINE op: W [8192 x 2048] (Q8_0: scale max|w|/127, q = round(w/scale)),
    X [M x 2048] ~ N(0, 1), M in {1, 16, 128}; plus ragged and unaligned shapes,
    prefill-sized blocks (128- and 256-token tiles of the tcgen05 GEMM) and
    batched-decode blocks whose few output tiles split K over the SMs."""
    if wtype == Q8_0 and K % 32:
        pytest.skip("Q8_0 needs K % 32 == 0")
    act = BF16 if wtype == BF16 else F16
    w = _weights(wtype, N, K, seed=100 + M)
    xd, xf = _acts(act, M, K, seed=200 + K)
    pw, px = up(w), up(xd)
    po = alloc(2 * M * N)
    dev.cuda_matmul(po, px, pw, None, M, K, N, wtype)
    got = _from_dev(down(po, (M, N), np.uint16 if act == BF16 else np.float16), act)
    ref = orc.matmul(xf, w, None, M, K, N, wtype, act)
    assert rel_err(got, ref) <= tol(act)
    free(pw, px, po)


def test_matmul_f16_bias(dev):
    M, N, K = 3, 40, 64
    w = _weights(F16, N, K, 5)
    xd, xf = _acts(F16, M, K, 6)
    b = h16(orc.gen_normal(N, 7, 0.5))
    pw, px, pb = up(w), up(xd), up(b)
    po = alloc(2 * M * N)
    dev.cuda_matmul(po, px, pw, pb, M, K, N, F16)
    ref = orc.matmul(xf, w, b.astype(np.float32), M, K, N, F16, F16)
    assert rel_err(down(po, (M, N), np.float16), ref) <= REL
    free(pw, px, pb, po)


def _layer_weights(wtype, d, H, Hk, D, F, seed):
    W = (H + 2 * Hk) * D
    return dict(attn_norm=(1.0 + orc.gen_normal(d, seed + 1, 0.1)).astype(np.float32),
                ffn_norm=(1.0 + orc.gen_normal(d, seed + 2, 0.1)).astype(np.float32),
                qkv=_weights(wtype, W, d, seed + 3), o=_weights(wtype, d, d, seed + 4),
                fc=_weights(wtype, 2 * F, d, seed + 5), down=_weights(wtype, d, F, seed + 6))


@pytest.mark.parametrize("wtype", [Q8_0, F16, BF16])
@pytest.mark.parametrize("B,Tn", [(1, 1), (2, 5), (1, 37)])
def test_layers_vs_oracle(dev, wtype, B, Tn):
    """cuda_group_query_attention + cuda_feed_forward at Llama-3.2-1B widths."""
    d, H, Hk, D, F = 2048, 32, 8, 64, 8192
    act = BF16 if wtype == BF16 else F16
    lw = _layer_weights(wtype, d, H, Hk, D, F, seed=40)
    freqs = orc.make_freqs(D, 64, 500000.0)
    xd, xf = _acts(act, B * Tn, d, seed=41, std=1.0)
    p = {k: up(v) for k, v in lw.items()}
    pf, px = up(freqs), up(xd)
    dev.cuda_group_query_attention(px, px, pf, p["attn_norm"], p["qkv"], p["o"], B, Tn, H, Hk, D, 1e-5, wtype)
    x_attn = _from_dev(down(px, (B * Tn, d), np.uint16 if act == BF16 else np.float16), act)
    dev.cuda_feed_forward(px, px, p["ffn_norm"], p["fc"], p["down"], B, Tn, d, F, 1e-5, wtype)
    x_ffn = _from_dev(down(px, (B * Tn, d), np.uint16 if act == BF16 else np.float16), act)
    # oracle
    xo = xf.reshape(B, Tn, d).copy()
    kc = np.zeros((B, Hk, Tn, D), np.float32)
    vc = np.zeros_like(kc)
    L, pp = orc.lib(), orc._p
    L.orc_gqa_layer(pp(xo), pp(freqs), pp(lw["attn_norm"]), pp(lw["qkv"]), pp(lw["o"]), B, Tn, 0, H, Hk, D, 1e-5,
                    wtype, act, pp(kc), pp(vc), Tn)
    # the update (x - x0) is what the sublayer computed; compare it normwise
    assert rel_err(x_attn - xf, xo.reshape(B * Tn, d) - xf) <= 2 * tol(act)
    assert rel_err(x_attn, xo.reshape(B * Tn, d)) <= tol(act)
    x1 = xo.copy()
    L.orc_ffn_layer(pp(x1), pp(lw["ffn_norm"]), pp(lw["fc"]), pp(lw["down"]), B, Tn, d, F, 1e-5, wtype, act)
    # start the FFN oracle from the GPU's attention output to isolate the FFN
    x2 = x_attn.reshape(B, Tn, d).copy()
    L.orc_ffn_layer(pp(x2), pp(lw["ffn_norm"]), pp(lw["fc"]), pp(lw["down"]), B, Tn, d, F, 1e-5, wtype, act)
    assert rel_err(x_ffn, x2.reshape(B * Tn, d)) <= tol(act)
    assert rel_err(x_ffn, x1.reshape(B * Tn, d)) <= 2 * tol(act)
    free(pf, px, *p.values())


@pytest.mark.parametrize("d,H,Hk,D,B,Tn,wtype", [(2048, 32, 8, 64, 1, 512, Q8_0), (2048, 32, 8, 64, 2, 300, F16),
                                                   (4096, 32, 8, 128, 1, 2048, Q8_0), (1024, 8, 8, 128, 1, 130, BF16),
                                                   (1024, 16, 2, 64, 1, 200, Q8_0)])
def test_prefill_attention_sublayer_vs_oracle(dev, d, H, Hk, D, B, Tn, wtype):
    """The attention sublayer over a long prompt (the flash-style prefill
    kernel): Llama-3.2-1B widths at 512 and 300 tokens, Llama-3.1-8B widths
    (head_dim 128) at 2048, and 1 and 8 query heads per KV head."""
    act = BF16 if wtype == BF16 else F16
    W = (H + 2 * Hk) * D
    lw = dict(attn_norm=np.ones(d, np.float32), qkv=_weights(wtype, W, d, 90), o=_weights(wtype, d, H * D, 91))
    freqs = orc.make_freqs(D, Tn, 500000.0)
    xd, xf = _acts(act, B * Tn, d, seed=92, std=1.0)
    p = {k: up(v) for k, v in lw.items()}
    pf, px = up(freqs), up(xd)
    dev.cuda_group_query_attention(px, px, pf, p["attn_norm"], p["qkv"], p["o"], B, Tn, H, Hk, D, 1e-5, wtype)
    x_attn = _from_dev(down(px, (B * Tn, d), np.uint16 if act == BF16 else np.float16), act)
    xo = xf.reshape(B, Tn, d).copy()
    kc = np.zeros((B, Hk, Tn, D), np.float32)
    vc = np.zeros_like(kc)
    L, pp = orc.lib(), orc._p
    L.orc_gqa_layer(pp(xo), pp(freqs), pp(lw["attn_norm"]), pp(lw["qkv"]), pp(lw["o"]), B, Tn, 0, H, Hk, D, 1e-5,
                    wtype, act, pp(kc), pp(vc), Tn)
    upd, ref = x_attn - xf, xo.reshape(B * Tn, d) - xf
    nw = float(np.linalg.norm(upd - ref) / np.linalg.norm(ref))
    print(f"prefill attention {B}x{Tn} d {d} H {H}/{Hk} D {D}: normwise rel-err of the update {nw:.2e}")
    assert rel_err(upd, ref) <= 2 * tol(act)
    assert nw <= tol(act)
    free(pf, px, *p.values())


@pytest.mark.parametrize("wtype", [Q8_0, F16])
def test_classify_predict_vocab_vs_oracle(dev, wtype):
    """Logits over the 128256 vocabulary and the fused argmax (reference tie order)."""
    B, Tn, d, V = 3, 4, 2048, 128256
    act = F16
    w = _weights(wtype, V, d, seed=77)
    nw = (1.0 + orc.gen_normal(d, 78, 0.1)).astype(np.float32)
    xd, xf = _acts(act, B * Tn, d, seed=79)
    pw, pn, px = up(w), up(nw), up(xd)
    pl, pt = alloc(2 * B * V), alloc(4 * B)
    dev.cuda_classify(pl, px, pn, pw, B, Tn, d, V, 1e-5, wtype)
    logits = down(pl, (B, V), np.float16).astype(np.float32)
    ref = np.empty((B, V), np.float32)
    orc.lib().orc_classify(orc._p(ref), orc._p(xf), orc._p(nw), orc._p(w), B, Tn, d, V, 1e-5, wtype, act)
    assert rel_err(logits, ref) <= REL
    dev.cuda_predict(pt, px, pn, pw, B, Tn, d, V, 1e-5, wtype)
    toks = down(pt, B, np.int32)
    # exact: the fused argmax equals the reference-order argmax of the GPU's own logits
    assert toks.tolist() == orc.argmax(logits, B, V, 8).tolist()
    free(pw, pn, px, pl, pt)


def test_argmax_tie_order_gpu(dev):
    """Exact ties resolve like the reference kernel (cuda.cu:480-531)."""
    x = np.zeros((3, 16384), np.float32)
    x[0, 8 * 4 + 3] = 5.0
    x[0, 16 * 4 + 1] = 5.0
    x[1, 3 * 4 + 2] = 1.0
    x[1, (3 + 256) * 4] = 1.0
    x[2, :] = -np.inf
    px = up(x)
    po = alloc(12)
    dev.cuda_argmax(po, px, 3, 16384)
    assert down(po, 3, np.int32).tolist() == orc.argmax(x, 3, 16384, 4).tolist()
    free(px, po)
