"""ctypes binding of liblightx2v_cuda.so (the C ABI in include/lightx2v_cuda.h).

This is the binding a host language adds to call the library; a Rust crate
declares the same functions in an `extern "C"` block. There is no fallback:
if the shared library is missing, importing the backend raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "liblightx2v_cuda.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)

OK = 0
ERR_INVALID = 1
ERR_CUDA = 2
ERR_OOM = 3
ERR_UNSUPPORTED = 4
ERR_NO_DEVICE = 5
ERR_DEVICE = 6
STATUS_NAMES = {0: "OK", 1: "INVALID", 2: "CUDA", 3: "OOM", 4: "UNSUPPORTED", 5: "NO_DEVICE",
                6: "DEVICE"}

ACT_NONE = 0
ACT_GELU_TANH = 1
BF16 = 0
F32 = 1
W_BF16, W_Q8, W_Q4, W_FP8, W_NVFP4 = 0, 1, 2, 3, 4

_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_st = ctypes.c_int
_pp = ctypes.POINTER(ctypes.c_void_p)

# name -> (restype, argtypes); mirrors include/lightx2v_cuda.h one to one.
SIGNATURES = {
    "lx2v_init": (_st, [ctypes.c_int, _pp]),
    "lx2v_free_ctx": (None, [_vp]),
    "lx2v_last_error": (ctypes.c_char_p, [_vp]),
    "lx2v_name": (_st, [_vp, ctypes.c_char_p, _sz]),
    "lx2v_sync": (_st, [_vp]),
    "lx2v_stream": (_vp, [_vp]),
    "lx2v_buf_alloc": (_st, [_vp, _sz, ctypes.c_int, _pp]),
    "lx2v_buf_upload_f32": (_st, [_vp, _vp, _sz, ctypes.c_int, _pp]),
    "lx2v_buf_write_f32": (_st, [_vp, _vp, _vp, _sz]),
    "lx2v_buf_download_f32": (_st, [_vp, _vp, _vp, _sz]),
    "lx2v_buf_download_f32_async": (_st, [_vp, _vp, _vp, _sz]),
    "lx2v_buf_len": (_st, [_vp, _vp, ctypes.POINTER(_sz)]),
    "lx2v_buf_info": (_st, [_vp, _vp, ctypes.POINTER(ctypes.c_int), _pp]),
    "lx2v_buf_copy": (_st, [_vp, _vp, _sz, _vp, _sz, _sz]),
    "lx2v_buf_free": (None, [_vp, _vp]),
    "lx2v_weight_f32": (_st, [_vp, _vp, _sz, _sz, _pp]),
    "lx2v_weight_q8": (_st, [_vp, _vp, _vp, _sz, _sz, _sz, _pp]),
    "lx2v_weight_q4": (_st, [_vp, _vp, _vp, _vp, _sz, _sz, _sz, _pp]),
    "lx2v_weight_fp8": (_st, [_vp, _vp, _vp, _sz, _sz, _sz, _pp]),
    "lx2v_sparse_prepare": (_st, [_vp, _vp, _vp, _sz, _sz, _sz, _sz, _sz, ctypes.c_float, _pp]),
    "lx2v_sparse_free": (None, [_vp, _vp]),
    "lx2v_sparse_attention": (_st, [_vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "lx2v_weight_nvfp4": (_st, [_vp, _vp, _vp, ctypes.c_float, _sz, _sz, _pp]),
    "lx2v_weight_free": (None, [_vp, _vp]),
    "lx2v_weight_info": (_st, [_vp, _vp, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(_sz),
                               ctypes.POINTER(_sz), ctypes.POINTER(_sz)]),
    "lx2v_weight_dequant_f32": (_st, [_vp, _vp, _vp]),
    "lx2v_linear": (_st, [_vp, _vp, _sz, _sz, _vp, _vp, ctypes.c_int, _vp, _sz]),
    "lx2v_linear_noalloc": (_st, [_vp, _vp, _sz, _sz, _vp, _vp, ctypes.c_int, _vp, _sz]),
    "lx2v_linear_gate_residual": (_st, [_vp, _vp, _sz, _sz, _vp, _vp, ctypes.c_int, _vp, _sz,
                                        _vp, _sz]),
    "lx2v_gate_residual": (_st, [_vp, _vp, _vp, _sz, _sz, _vp, _sz]),
    "lx2v_attention": (_st, [_vp, _vp, _vp, _vp, _sz, _sz, _sz, _sz, _vp]),
    "lx2v_causal_attention": (_st, [_vp, _vp, _vp, _vp, _sz, _sz, _sz, _sz, _vp, _vp]),
    "lx2v_causal_attention_temporal": (_st, [_vp, _vp, _vp, _vp, _sz, _sz, _sz, _sz, _vp, _vp, _vp]),
    "lx2v_layer_norm": (_st, [_vp, _vp, _sz, _sz, ctypes.c_int, _vp, _vp, _sz, _sz, _vp, ctypes.c_float, _vp]),
    "lx2v_residual_norm": (_st, [_vp, _vp, _vp, _sz, _sz, _vp, ctypes.c_long, ctypes.c_int, _vp, _vp, _sz, _sz,
                                 ctypes.c_float, _vp]),
    "lx2v_head_split": (_st, [_vp, _vp, _sz, _sz, _sz, _sz, _sz, _vp, _vp, _vp, ctypes.c_float, _vp]),
    "lx2v_row_sumsq": (_st, [_vp, _vp, _sz, _sz, _sz, _sz, _vp]),
    "lx2v_head_split_rms": (_st, [_vp, _vp, _sz, _sz, _sz, _sz, _sz, _vp, _vp, _sz, _vp, _vp, ctypes.c_float,
                                  _vp]),
    "lx2v_patchify": (_st, [_vp, _vp, _sz, _sz, _sz, _sz, _sz, _vp]),
    "lx2v_unpatchify": (_st, [_vp, _vp, _sz, _sz, _sz, _sz, _sz, _vp]),
    "lx2v_dmd_step": (_st, [_vp, _vp, _vp, _vp, ctypes.c_float, ctypes.c_float, _sz]),
    "lx2v_kv_cache_new": (_st, [_vp, _sz, _sz, _sz, _pp]),
    "lx2v_kv_cache_free": (None, [_vp, _vp]),
    "lx2v_kv_cache_append": (_st, [_vp, _vp, _vp, _vp, _sz, _vp]),
    "lx2v_kv_cache_put": (_st, [_vp, _vp, _vp, _vp, _sz, _vp]),
    "lx2v_kv_cache_len": (_st, [_vp, _vp, ctypes.POINTER(_sz)]),
    "lx2v_kv_cache_temporal": (_st, [_vp, _vp, _vp, _sz]),
    "lx2v_kv_cache_kv": (_st, [_vp, _vp, _vp, _vp]),
    "lx2v_kv_cache_memrope_update": (_st, [_vp, _vp, _sz, _sz, _sz, ctypes.c_float, ctypes.c_float, _sz]),
    "lx2v_kv_cache_attention": (_st, [_vp, _vp, _sz, _vp, _vp, _vp]),
    "lx2v_profile_json": (_st, [_vp, ctypes.c_char_p, _sz, ctypes.POINTER(_sz)]),
    "lx2v_profile_reset": (_st, [_vp]),
    "lx2v_set_linear_path": (_st, [_vp, ctypes.c_int]),
    "lx2v_set_token_tile": (_st, [_vp, ctypes.c_int]),
    "lx2v_set_split_mode": (_st, [_vp, ctypes.c_int]),
    "lx2v_set_wait_limit_ns": (_st, [_vp, ctypes.c_uint64]),
    "lx2v_launch_count": (_st, [_vp, ctypes.POINTER(ctypes.c_uint64)]),
    "lx2v_comm_unique_id": (_st, [_vp, _sz]),
    "lx2v_comm_init": (_st, [_vp, _vp, ctypes.c_int, ctypes.c_int]),
    "lx2v_all_reduce_sum": (_st, [_vp, _vp, _sz]),
    "lx2v_buf_ipc_handle": (_st, [_vp, _vp, _vp, _sz]),
    "lx2v_buf_open_ipc": (_st, [_vp, _vp, _sz, ctypes.c_int, _pp]),
    "lx2v_peers_create": (_st, [_vp, ctypes.c_int, ctypes.c_int, _pp, _pp]),
    "lx2v_peers_free": (None, [_vp]),
    "lx2v_peers_barrier": (_st, [_vp, _vp]),
    "lx2v_row_sumsq_peers": (_st, [_vp, _vp, _vp, _sz, _sz, _sz, _sz, _pp]),
    "lx2v_head_split_rms_parts": (_st, [_vp, _vp, _sz, _sz, _sz, _sz, _sz, _vp, _vp, _sz, _sz, _vp, _vp,
                                        ctypes.c_float, _vp]),
    "lx2v_tp_reduce_norm": (_st, [_vp, _vp, _pp, _vp, _sz, _sz, _sz, _vp, ctypes.c_long, ctypes.c_int, _vp, _vp,
                                  _vp, _sz, _sz, ctypes.c_float, _pp]),
}

COMM_ID_BYTES = 128
IPC_HANDLE_BYTES = 64

_lib = None


class LibraryMissing(RuntimeError):
    pass


def load(path: str | None = None):
    """Load the shared library and declare every entry point."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise LibraryMissing(
            f"{p} is missing: build it with `make -C lightx2v-rs_b200/csrc` "
            "(or __graft_entry__.build()); there is no CPU fallback")
    lib = ctypes.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


class Lx2vError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"lx2v status {STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status
