"""Host-side Tensor mirroring the reference's Go ``Tensor`` / ``cudaRunner``
(llm/array.go:116-778) on top of the C ABI.

Same method names (snake_case), argument meaning, shape checks and error
messages as the Go code, so that the tests read like array_test.go.  Output
buffers are allocated with cuda_malloc and released with cuda_free, as the Go
runner does (array.go:573-620).
"""
import ctypes

import numpy as np

from . import BF16, F16, F32, I32, Q8_0, lib

# llm/array.go:73-110 (block size, type size); the dtypes this path uses
DTYPE_INFO = {F32: ("F32", 1, 4), F16: ("F16", 1, 2), Q8_0: ("GGML_TYPE_Q8_0", 32, 34), BF16: ("BF16", 1, 2),
              24: ("Int8", 1, 1), 25: ("Int16", 1, 2), I32: ("Int32", 1, 4), 27: ("Int64", 1, 8), 28: ("F64", 1, 8)}
_NP = {np.dtype(np.float32): F32, np.dtype(np.float16): F16, np.dtype(np.int32): I32, np.dtype(np.int8): 24,
       np.dtype(np.int16): 25, np.dtype(np.int64): 27, np.dtype(np.float64): 28}
_HOST = {F32: np.float32, F16: np.int16, I32: np.int32, 24: np.int8, 25: np.int16, 27: np.int64, 28: np.float64,
         BF16: np.int16}


class Tensor:
    def __init__(self, shape, dtype):
        self.shape = list(shape)
        self.dtype = dtype
        self.dptr = None
        self.owner = True

    # ---- shape helpers (array.go:146-197)
    def len(self):
        n = 1
        for v in self.shape:
            n *= v
        return n

    def dim(self, i):
        return self.shape[i]

    def ndims(self):
        return len(self.shape)

    def size(self):
        name, bs, ts = DTYPE_INFO[self.dtype]
        if self.shape[-1] % bs:
            raise ValueError(f"Shape {self.shape} is not aligned to {bs}")
        return self.len() // bs * ts

    # ---- memory (array.go:573-620)
    def to_device(self, host):
        host = np.ascontiguousarray(host)
        if self.dptr is None:
            self.dptr = lib().cuda_malloc(self.size())
        lib().cuda_to_device(self.dptr, host.ctypes.data_as(ctypes.c_void_p), self.size())

    def to_host(self):
        dst = np.empty(self.size(), np.uint8)
        lib().cuda_to_host(dst.ctypes.data_as(ctypes.c_void_p), self.dptr, self.size())
        if self.dtype not in _HOST:
            raise ValueError(f"unsupported dtype {self.dtype}")
        return dst.view(_HOST[self.dtype]).copy()

    def device_free(self):
        if self.dptr is not None and self.owner:
            lib().cuda_free(self.dptr)
        self.dptr = None

    def __del__(self):
        try:
            self.device_free()
        except Exception:
            pass

    # ---- ops (array.go:622-778)
    def softmax(self):
        col = self.dim(-1)
        row = self.len() // col
        out = _new(self.shape, self.dtype)
        lib().cuda_softmax(out.dptr, self.dptr, row, col)
        return out

    def matmul(self, b, bias=None):
        if self.ndims() < 2 or b.ndims() != 2:
            raise ValueError("arrays must have at least 2 dimensions")
        if self.dim(-1) != b.dim(-1):
            raise ValueError("array shapes do not match")
        if bias is not None and bias.len() != b.dim(-2):
            raise ValueError("bias shape does not match")
        column = self.dim(-1)
        row = self.len() // column
        oc = b.dim(-2)
        shape = self.shape[:-1] + [oc]
        out = _new(shape, self.dtype)
        lib().cuda_matmul(out.dptr, self.dptr, b.dptr, None if bias is None else bias.dptr, row, column, oc, b.dtype)
        return out

    def embedding(self, ids):
        if ids.dtype != I32:
            raise ValueError("index must be an int32 integer")
        if ids.ndims() > 2:
            raise ValueError("index must be 1D or 2D")
        if self.ndims() != 2:
            raise ValueError("embedding must be 2D")
        col = self.dim(1)
        row = ids.dim(-1)
        batch = ids.dim(0) if ids.ndims() == 2 else 1
        dtype = self.dtype if self.dtype in (F32, F16, BF16) else F16
        out = _new([batch, row, col], dtype)
        lib().cuda_embedding(out.dptr, ids.dptr, self.dptr, batch, row, col, self.dtype)
        return out

    def cat(self, b):
        if self.dtype != b.dtype:
            raise ValueError("arrays must have the same dtype")
        if self.ndims() != 2 or b.ndims() != 2:
            raise ValueError("arrays must have 2 dimensions")
        if self.dim(-1) != b.dim(-1):
            raise ValueError("array shapes do not match")
        out = _new([self.dim(0) + b.dim(0), self.dim(1)], self.dtype)
        lib().cuda_cat(out.dptr, self.dptr, b.dptr, self.dim(0), b.dim(0), self.dim(1), self.dtype)
        return out

    def dequantize(self):
        if self.dtype != Q8_0:
            raise ValueError("Tensor dtype must be Q8_0")
        col = self.dim(-1)
        row = self.len() // col
        out = _new(self.shape, F32)
        lib().cuda_dequantize(out.dptr, self.dptr, row, col, self.dtype)
        return out

    def group_query_attention(self, freqs, norm_weight, qkv_weight, out_weight, NH, kvNH, eps):
        col = self.dim(-1)
        HS = col // NH
        row = self.dim(-2)
        if freqs.dim(0) != row or freqs.dim(1) != HS:
            raise ValueError(f"bad freqs shape {freqs.shape}")
        if norm_weight.ndims() != 1 or norm_weight.dim(0) != col:
            raise ValueError(f"bad norm_weight shape {norm_weight.shape}")
        if qkv_weight.dim(0) != (NH + 2 * kvNH) * HS or qkv_weight.dim(1) != col:
            raise ValueError(f"bad qkv_weight shape {qkv_weight.shape}")
        if out_weight.dim(0) != col or out_weight.dim(1) != col:
            raise ValueError(f"bad out_weight shape {out_weight.shape}")
        batch = self.dim(0) if self.ndims() == 3 else 1
        lib().cuda_group_query_attention(self.dptr, self.dptr, freqs.dptr, norm_weight.dptr, qkv_weight.dptr,
                                         out_weight.dptr, batch, row, NH, kvNH, HS, eps, out_weight.dtype)

    def feed_forward(self, norm_weight, fc_weight, out_weight, ffl, eps):
        col = self.dim(-1)
        row = self.dim(-2)
        if norm_weight.ndims() != 1 or norm_weight.dim(0) != col:
            raise ValueError(f"bad norm_weight shape {norm_weight.shape}")
        if fc_weight.dim(0) != 2 * ffl or fc_weight.dim(1) != col:
            raise ValueError(f"bad fc_weight shape {fc_weight.shape}")
        if out_weight.dim(0) != col or out_weight.dim(1) != ffl:
            raise ValueError(f"bad out_weight shape {out_weight.shape}")
        batch = self.dim(0) if self.ndims() == 3 else 1
        lib().cuda_feed_forward(self.dptr, self.dptr, norm_weight.dptr, fc_weight.dptr, out_weight.dptr, batch, row,
                                col, ffl, eps, out_weight.dtype)

    def predict(self, norm_weight, out_weight, vocab_size, eps):
        col = self.dim(-1)
        row = self.dim(-2)
        batch = self.dim(0) if self.ndims() == 3 else 1
        tids = np.zeros(batch, np.int32)
        d_out = lib().cuda_malloc(4 * batch)
        lib().cuda_predict(d_out, self.dptr, norm_weight.dptr, out_weight.dptr, batch, row, col, vocab_size, eps,
                           out_weight.dtype)
        lib().cuda_to_host(tids.ctypes.data_as(ctypes.c_void_p), d_out, 4 * batch)
        lib().cuda_free(d_out)
        return tids

    def row_slice(self, start, end):
        """Non-owning view of rows [start, end) (array.go:457-477)."""
        if self.ndims() != 2:
            raise ValueError("only 2D tensor is supported")
        if start < 0:
            start += self.dim(0)
        if end < 0:
            end += self.dim(0)
        if start < 0 or start >= self.dim(0) or end < 0 or end > self.dim(0):
            raise IndexError(f"slice index out of range: {start}, {end}")
        if start >= end:
            raise IndexError(f"invalid slice range: {start}, {end}")
        t = Tensor([end - start, self.dim(1)], self.dtype)
        _, bs, ts = DTYPE_INFO[self.dtype]
        t.dptr = self.dptr + start * self.dim(1) * ts // bs
        t.owner = False
        return t


def _new(shape, dtype):
    t = Tensor(shape, dtype)
    t.dptr = lib().cuda_malloc(t.size())
    return t


def make_tensor(shape, data):
    """MakeTensorErr (array.go:280-294): dtype from the numpy element type."""
    data = np.ascontiguousarray(data)
    if data.size != int(np.prod(shape)):
        raise ValueError(f"data length {data.size} does not match shape length {int(np.prod(shape))}")
    if data.dtype not in _NP:
        raise ValueError(f"unsupported type {data.dtype}")
    t = Tensor(shape, _NP[data.dtype])
    t.to_device(data)
    return t


def make_tensor_from(shape, raw, dtype):
    """MakeTensorFrom (array.go:222-239): raw bytes of a given GGML dtype."""
    if not shape or int(np.prod(shape)) <= 0:
        raise ValueError(f"bad shape: {shape}")
    if dtype not in DTYPE_INFO:
        raise ValueError(f"bad dtype: {dtype}")
    if shape[-1] % DTYPE_INFO[dtype][1]:
        raise ValueError(f"shape {shape} is not aligned to {DTYPE_INFO[dtype][1]}")
    t = Tensor(shape, dtype)
    t.to_device(np.frombuffer(np.ascontiguousarray(raw).tobytes(), np.uint8))
    return t
