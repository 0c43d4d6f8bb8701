"""wukong_b200 -- B200-native (sm_100a) hot path of the wukong LLM engine.

The product is the shared library ``libwukong.so`` (and the static archive
``build/libwukong.a``) exporting the reference's C ABI (``include/wukong.h``,
a drop-in for liuy/wukong's cuda.h) plus a native decode engine
(``include/wukong_ext.h``).  This package loads it through ctypes; there is no
fallback implementation: importing fails loudly when the library is missing.

    import wukong_b200 as wk
    wk.lib().cuda_init(0)
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libwukong.so")
ROOT = os.path.dirname(HERE)

F32, F16, Q4_0, Q8_0, BF16, I32 = 0, 1, 2, 8, 30, 26

_P, _I, _F, _S = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
_U64, _L = ctypes.c_uint64, ctypes.c_long

# name -> (restype, argtypes); the 27 entry points of cuda.h plus the wk_* API
ABI = {
    "cuda_init": (None, [_I]),
    "cuda_fini": (None, []),
    "cuda_malloc": (_P, [_S]),
    "cuda_to_host": (None, [_P, _P, _S]),
    "cuda_to_device": (None, [_P, _P, _S]),
    "cuda_free": (None, [_P]),
    "cuda_matmul": (None, [_P, _P, _P, _P, _I, _I, _I, _I]),
    "cuda_softmax": (None, [_P, _P, _I, _I]),
    "cuda_mh_sdpa": (None, [_P, _P, _I, _I, _I, _I]),
    "cuda_gq_sdpa": (None, [_P, _P, _I, _I, _I, _I, _I]),
    "cuda_mq_sdpa": (None, [_P, _P, _I, _I, _I, _I]),
    "cuda_rmsnorm": (None, [_P, _P, _P, _I, _I, _F]),
    "cuda_swiglu": (None, [_P, _P, _I, _I, _I]),
    "cuda_rope_qkv": (None, [_P, _P, _P, _I, _I, _I, _I, _I]),
    "cuda_rope": (None, [_P, _P, _P, _I, _I, _I, _I]),
    "cuda_embedding": (None, [_P, _P, _P, _I, _I, _I, _I]),
    "cuda_cat": (None, [_P, _P, _P, _I, _I, _I, _I]),
    "cuda_div": (None, [_P, _P, _P, _I, _I]),
    "cuda_dequantize": (None, [_P, _P, _I, _I, _I]),
    "cuda_add": (None, [_P, _P, _P, _I, _I]),
    "cuda_group_query_attention": (None, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _I]),
    "cuda_repeat_qkv": (None, [_P, _P, _I, _I, _I, _I, _I]),
    "cuda_feed_forward": (None, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _I]),
    "cuda_get_row": (None, [_P, _P, _I, _I, _I, _I]),
    "cuda_classify": (None, [_P, _P, _P, _P, _I, _I, _I, _I, _F, _I]),
    "cuda_argmax": (None, [_P, _P, _I, _I]),
    "cuda_predict": (None, [_P, _P, _P, _P, _I, _I, _I, _I, _F, _I]),
}
EXT = {
    "wk_last_error": (ctypes.c_char_p, []),
    "wk_stream": (_P, []),
    "wk_model_create": (_P, [_P]),
    "wk_model_destroy": (None, [_P]),
    "wk_model_set_layer": (_I, [_P, _I, _P, _P, _P, _P, _P, _P]),
    "wk_model_set_head": (_I, [_P, _P, _P, _P, _P, _I]),
    "wk_model_alloc_cache": (_I, [_P, _I, _I]),
    "wk_model_prefill": (_I, [_P, _P, _I, _I, _P]),
    "wk_model_decode_step": (_I, [_P]),
    "wk_model_tokens": (_P, [_P]),
    "wk_model_logits": (_P, [_P]),
    "wk_model_next_ids": (_P, [_P]),
    "wk_model_step_launches": (_I, [_P]),
    "wk_model_position": (_I, [_P]),
    "wk_model_truncate": (_I, [_P, _I]),
    "wk_model_add_seqs": (_I, [_P, _P, _P, _I, _P]),
    "wk_model_remove_seq": (_I, [_P, _I]),
    "wk_model_rows": (_I, [_P, _P]),
    "wk_model_set_sampling": (_I, [_P, _F, _I, _F, _U64]),
    "wk_sample_logits": (_I, [_P, _P, _I, _I, _I, _F, _I, _F, _U64, ctypes.c_longlong]),
    "wk_attention_decode": (_I, [_P, _P, _P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _I]),
    "wk_fill_random_q8_0": (_I, [_P, _L, _I, _U64, _F]),
    "wk_fill_random_q4_0": (_I, [_P, _L, _I, _U64, _F]),
    "wk_fill_random_f16": (_I, [_P, _L, _U64, _F]),
    "wk_fill_const_f32": (_I, [_P, _L, _F]),
    "wk_gemv": (_I, [_P, _P, _P, _I, _I, _I, _I]),
    "wk_predict_noalloc": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _F, _I]),
    "wk_timeline_init": (_I, [_I, _I]),
    "wk_timeline_read": (_I, [_P, _P]),
    "wk_timeline_resolution_ns": (ctypes.c_longlong, []),
    "wk_tp_unique_id": (_I, [_P]),
    "wk_tp_init": (_I, [_I, _I, _P]),
    "wk_tp_fini": (None, []),
    "wk_tp_rank": (_I, []),
    "wk_tp_world": (_I, []),
    "wk_tp_p2p": (_I, []),
    "wk_model_set_tp": (_I, [_P, _I]),
    "wk_tp_exchange_selftest": (_I, [_I, _I]),
    "wk_tp_gemv_selftest": (_I, [_I, _I, _I, _I]),
    "wk_device_error": (_I, [_I]),
}


HOST = {
    "wk_host_last_error": (ctypes.c_char_p, []),
    "wk_abi_bind": (_I, [_P, _P]),
    "wk_host_make_freqs": (None, [_P, _P, _I, _I, _F]),
    "wk_host_llama_create": (_P, [_P, _P]),
    "wk_host_llama_destroy": (None, [_P]),
    "wk_host_llama_setup": (_I, [_P, _P, _P, _P, _P, _P]),
    "wk_host_llama_predict": (_I, [_P, _P, _I, _I, _P]),
    "wk_host_llama_generate": (_I, [_P, _P, _I, _I, _P]),
}


class WKHostConfig(ctypes.Structure):
    _fields_ = [("n_layers", _I), ("d_model", _I), ("n_heads", _I), ("n_kv_heads", _I), ("head_dim", _I),
                ("ffn", _I), ("vocab", _I), ("ctx", _I), ("eps", _F), ("rope_theta", _F), ("wtype", _I),
                ("out_wtype", _I), ("embd_wtype", _I)]


class WKHostLayer(ctypes.Structure):
    _fields_ = [(n, _P) for n in ("attn_norm", "q", "k", "v", "o", "ffn_norm", "up", "gate", "down")]


# wk_abi: 11 function pointers (include/wukong_host.h)
WK_ABI_SIZE = 11 * ctypes.sizeof(ctypes.c_void_p)


class WKConfig(ctypes.Structure):
    _fields_ = [("n_layers", _I), ("d_model", _I), ("n_heads", _I), ("n_kv_heads", _I), ("head_dim", _I),
                ("ffn", _I), ("vocab", _I), ("eps", _F), ("wtype", _I), ("out_wtype", _I), ("embd_wtype", _I)]


_lib = None


def lib():
    """The loaded C library (ctypes.CDLL); raises if the build is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m wukong_b200.build` "
                              "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_LOCAL)
        for table in (ABI, EXT, HOST):
            for name, (res, args) in table.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
        _lib = L
    return _lib


def check(rc):
    if rc != 0:
        raise RuntimeError(lib().wk_last_error().decode())
    return rc
