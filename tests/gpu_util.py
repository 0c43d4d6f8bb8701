"""Device buffer helpers for the GPU tests (through the library's own C ABI)."""
import ctypes

import numpy as np

import wukong_b200 as wk


def up(arr):
    a = np.ascontiguousarray(arr)
    p = wk.lib().cuda_malloc(max(a.nbytes, 4))
    wk.lib().cuda_to_device(p, a.ctypes.data_as(ctypes.c_void_p), a.nbytes)
    return p


def down(p, shape, dtype):
    out = np.empty(shape, dtype)
    wk.lib().cuda_to_host(out.ctypes.data_as(ctypes.c_void_p), p, out.nbytes)
    return out


def alloc(nbytes):
    return wk.lib().cuda_malloc(max(int(nbytes), 4))


def free(*ps):
    for p in ps:
        wk.lib().cuda_free(p)


def h16(x):
    """float32 values -> fp16 storage."""
    return np.asarray(x, np.float32).astype(np.float16)


def bf16_bits(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_to_f32(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))
