"""CPU-only checks of the drop-in boundary: the library loads, exports every
declared entry point, the static archive links with the reference's cgo line,
and the host-side logic (no device calls) matches the reference's Go code."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import wukong_b200 as wk
from wukong_b200 import tensor as T
from oracle import oracle as orc

ROOT = wk.ROOT


def _declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b(\w+)\s*\([^;{]*\)\s*;", text)
    return sorted({n for n in names if n.startswith(("cuda_", "wk_"))})


@pytest.mark.parametrize("header", ["wukong.h", "wukong_ext.h", "wukong_host.h"])
def test_library_exports_every_declared_symbol(header):
    L = wk.lib()
    names = _declared(header)
    assert names, header
    for n in names:
        assert hasattr(L, n), f"{n} declared in {header} but not exported"


def test_abi_has_the_27_reference_entry_points():
    # cuda.h:1-28 of the reference declares exactly these names
    expected = {"cuda_init", "cuda_fini", "cuda_malloc", "cuda_to_host", "cuda_to_device", "cuda_free",
                "cuda_matmul", "cuda_softmax", "cuda_mh_sdpa", "cuda_gq_sdpa", "cuda_mq_sdpa", "cuda_rmsnorm",
                "cuda_swiglu", "cuda_rope_qkv", "cuda_rope", "cuda_embedding", "cuda_cat", "cuda_div",
                "cuda_dequantize", "cuda_add", "cuda_group_query_attention", "cuda_repeat_qkv",
                "cuda_feed_forward", "cuda_get_row", "cuda_classify", "cuda_argmax", "cuda_predict"}
    assert set(_declared("wukong.h")) == expected
    assert set(wk.ABI) == expected


def test_static_archive_links_with_the_cgo_line(tmp_path):
    """llm/array.go:4 links ./build/libwukong.a -lcublasLt -lcudart -lm -lcublas with a C
    compiler: the archive must not need libstdc++ or any other library."""
    archive = os.path.join(ROOT, "build", "libwukong.a")
    assert os.path.exists(archive)
    names = _declared("wukong.h")
    src = tmp_path / "probe.c"
    src.write_text('#include "wukong.h"\n#include <stdio.h>\nint main(void){void *f[]={' +
                   ",".join(f"(void*){n}" for n in names) + '};printf("%d\\n",(int)(sizeof f/sizeof *f));return 0;}\n')
    exe = tmp_path / "probe"
    r = subprocess.run(["gcc", "-I" + os.path.join(ROOT, "include"), str(src), archive, "-L/usr/local/cuda/lib64",
                        "-lcublasLt", "-lcudart", "-lm", "-lcublas", "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.stdout.strip() == str(len(names))


def test_host_freqs_match_llama_go():
    """wk_host_make_freqs restates llama.go:54-67; the oracle restates the same."""
    HS, ctx = 64, 300
    factor = (1.0 + np.arange(HS // 2, dtype=np.float32) / 7).astype(np.float32)
    got = np.empty((ctx, HS), np.float32)
    wk.lib().wk_host_make_freqs(got.ctypes.data_as(ctypes.c_void_p), factor.ctypes.data_as(ctypes.c_void_p), HS,
                                ctx, 500000.0)
    ref = orc.make_freqs(HS, ctx, 500000.0, factor)
    assert np.array_equal(got, ref)


def test_tensor_shape_errors_match_array_go():
    """cudaRunner's argument checks (array.go:632-757) fire before any device call."""
    a = T.Tensor([2, 3], wk.F32)
    b = T.Tensor([2, 2], wk.F32)
    with pytest.raises(ValueError, match="array shapes do not match"):
        a.matmul(b)
    with pytest.raises(ValueError, match="arrays must have at least 2 dimensions"):
        a.matmul(T.Tensor([2, 2, 2], wk.F32))
    with pytest.raises(ValueError, match="bias shape does not match"):
        a.matmul(T.Tensor([2, 3], wk.F32), T.Tensor([3], wk.F32))
    with pytest.raises(ValueError, match="index must be an int32 integer"):
        T.Tensor([4, 4], wk.F32).embedding(T.Tensor([2], 27))
    with pytest.raises(ValueError, match="embedding must be 2D"):
        T.Tensor([2, 2, 2], wk.F32).embedding(T.Tensor([2], wk.I32))
    with pytest.raises(ValueError, match="arrays must have the same dtype"):
        T.Tensor([3, 2], wk.I32).cat(T.Tensor([2, 3], wk.F32))
    with pytest.raises(ValueError, match="Tensor dtype must be Q8_0"):
        T.Tensor([2, 32], wk.F32).dequantize()
    with pytest.raises(ValueError, match="is not aligned to 32"):
        T.make_tensor_from([2, 12], np.zeros(8, np.uint8), wk.Q8_0)
    with pytest.raises(ValueError, match="does not match shape length"):
        T.make_tensor([2, 2], np.zeros(3, np.float32))
    t = T.Tensor([4, 3], wk.F32)
    t.dptr = 4096
    for s, e in ((3, 1), (1, 5), (-5, 2), (1, -5)):
        with pytest.raises(IndexError):
            t.row_slice(s, e)
    v = t.row_slice(-3, -1)
    assert v.shape == [2, 3] and v.dptr == 4096 + 12 and not v.owner
    t.dptr = None


def test_tensor_sizes_match_array_go():
    # TestTensorSize / TestTensorElemSize (array_test.go:29-62)
    assert T.Tensor([2, 3], wk.F32).size() == 24
    assert T.Tensor([2, 3], 25).size() == 12
    assert T.Tensor([4, 64], wk.Q8_0).size() == 4 * 2 * 34


def test_reference_library_builds_where_sources_exist():
    """oracle/_ref holds the reference's own cuda.cu compiled for sm_100a (test
    infrastructure, used by the GPU parity tests)."""
    if not os.path.exists(orc.REF_LIB_PATH):
        subprocess.check_call(["make", "-s", "-C", os.path.dirname(orc.LIB_PATH), "ref-if-present"])
    if not os.path.exists(orc.REF_LIB_PATH):
        pytest.skip("reference sources not mounted and no prebuilt oracle/_ref")
    L = ctypes.CDLL(orc.REF_LIB_PATH, mode=ctypes.RTLD_LOCAL)
    for n in wk.ABI:
        if n != "cuda_rope":  # declared by the reference's cuda.h but never defined
            assert hasattr(L, n), n
