"""ctypes binding of the C ABI declared in include/m1moe_cuda.h.

The shared library is the product: there is no Python or CPU fallback.  If
libm1moe_cuda.so is missing, importing the ops raises immediately.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libm1moe_cuda.so"

M1MOE_OK = 0
STATUS_NAMES = {
    0: "OK", 1: "INVALID_ARG", 2: "OUT_OF_MEMORY", 3: "CUDA", 4: "NOT_LOADED", 5: "DEVICE",
    6: "UNSUPPORTED",
}
DTYPE_F32 = 0
DTYPE_BF16 = 1


class M1MoECudaError(RuntimeError):
    """A C-ABI call returned a non-zero m1moe_status."""

    def __init__(self, status: int, func: str, message: str):
        self.status = status
        super().__init__(f"{func}: M1MOE_ERR_{STATUS_NAMES.get(status, status)}: {message}")


class Cfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "hidden_dim", "intermediate_dim", "num_experts", "top_k", "group_size", "num_layers",
        "norm_topk_prob", "max_batch", "device", "expert_begin", "expert_count")]


class DenseCfg(ctypes.Structure):
    _fields_ = [("hidden_dim", ctypes.c_int32), ("num_heads", ctypes.c_int32),
                ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("num_layers", ctypes.c_int32), ("vocab_size", ctypes.c_int32),
                ("qk_norm", ctypes.c_int32), ("rms_norm_eps", ctypes.c_float),
                ("rope_theta", ctypes.c_float), ("max_batch", ctypes.c_int32),
                ("max_seq", ctypes.c_int32), ("device", ctypes.c_int32)]


# m1moe_dense_tensor
W_EMBED, W_FINAL_NORM, W_LM_HEAD, W_INPUT_NORM, W_POST_NORM = 0, 1, 2, 3, 4
W_Q, W_K, W_V, W_O, W_Q_NORM, W_K_NORM = 5, 6, 7, 8, 9, 10

_lib = None

# (name, restype, argtypes) for every entry point in include/m1moe_cuda.h.
_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_SIGS = [
    ("m1moe_cuda_abi_version", ctypes.c_int32, []),
    ("m1moe_cuda_last_error", ctypes.c_char_p, []),
    ("m1moe_cuda_expert_bytes", ctypes.c_size_t, [_i32, _i32, _i32]),
    ("m1moe_cuda_create", ctypes.c_int, [ctypes.POINTER(Cfg), ctypes.POINTER(_vp)]),
    ("m1moe_cuda_destroy", ctypes.c_int, [_vp]),
    ("m1moe_cuda_load_expert_layer", ctypes.c_int, [_vp, _i32, _vp, ctypes.c_size_t]),
    ("m1moe_cuda_load_expert_layer_device", ctypes.c_int, [_vp, _i32, _vp, ctypes.c_size_t, _vp]),
    ("m1moe_cuda_load_router", ctypes.c_int, [_vp, _i32, _vp, ctypes.c_size_t]),
    ("m1moe_cuda_load_expert_files", ctypes.c_int, [_vp, ctypes.c_char_p, _i32]),
    ("m1moe_cuda_matvec4", ctypes.c_int,
     [_vp, _vp, _vp, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32, _vp]),
    ("m1moe_cuda_matvec4_strided", ctypes.c_int,
     [_vp, _vp, _vp, ctypes.c_int64, _i32, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32, _vp]),
    ("m1moe_cuda_unpack4", ctypes.c_int, [_vp, _vp, _i32, _i32, _vp]),
    ("m1moe_cuda_router_topk", ctypes.c_int, [_vp, _i32, _vp, _i32, _i32, _vp, _vp, _vp, _vp]),
    ("m1moe_cuda_router_topk_noalloc", ctypes.c_int,
     [_vp, _i32, _i32, _i32, _i32, _vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp]),
    ("m1moe_cuda_moe_layer", ctypes.c_int,
     [_vp, _i32, _vp, _i32, _vp, _i32, _vp, _i32, _i32, _vp, _vp, _vp]),
    ("m1moe_cuda_moe_prefill", ctypes.c_int,
     [_vp, _i32, _vp, _i32, _vp, _i32, _vp, _i32, _i32, _vp, _vp, _vp]),
    ("m1moe_cuda_ep_region", ctypes.c_int, [_vp, _i32, _i32, _vp]),
    ("m1moe_cuda_ep_connect", ctypes.c_int, [_vp, _i32, _vp]),
    ("m1moe_cuda_ep_connect_local", ctypes.c_int, [_vp, _i32, _vp]),
    ("m1moe_cuda_set_wait_limit", ctypes.c_int, [_vp, ctypes.c_uint32]),
    ("m1moe_cuda_moe_layer_ep", ctypes.c_int,
     [_vp, _i32, _vp, _i32, _vp, _i32, _vp, _i32, _vp, _vp, _vp]),
    ("m1moe_cuda_moe_layer_host", ctypes.c_int, [_vp, _i32, _vp, _vp, _vp, _i32, _vp, _vp]),
    ("m1moe_cuda_synchronize", ctypes.c_int, [_vp]),
    ("m1moe_cuda_launch_count", ctypes.c_int64, []),
    ("m1moe_cuda_set_trace", ctypes.c_int, [_vp, _vp]),
    ("m1moe_cuda_dense_create", ctypes.c_int, [ctypes.POINTER(DenseCfg), ctypes.POINTER(_vp)]),
    ("m1moe_cuda_dense_destroy", ctypes.c_int, [_vp]),
    ("m1moe_cuda_dense_load", ctypes.c_int, [_vp, _i32, _i32, _vp, ctypes.c_size_t]),
    ("m1moe_cuda_dense_load_device", ctypes.c_int, [_vp, _i32, _i32, _vp, ctypes.c_size_t, _vp]),
    ("m1moe_cuda_dense_kv_cache", ctypes.c_int,
     [_vp, _i32, ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
    ("m1moe_cuda_dense_set_position", ctypes.c_int, [_vp, _i32]),
    ("m1moe_cuda_dense_get_position", ctypes.c_int, [_vp, ctypes.POINTER(_i32)]),
    ("m1moe_cuda_dense_reset", ctypes.c_int, [_vp]),
    ("m1moe_cuda_dense_synchronize", ctypes.c_int, [_vp]),
    ("m1moe_cuda_dense_gemv", ctypes.c_int,
     [_vp, _i32, _i32, _vp, _i32, _vp, ctypes.c_float, _vp, _vp, _i32, _vp]),
    ("m1moe_cuda_dense_rmsnorm", ctypes.c_int,
     [_vp, _i32, _vp, ctypes.c_float, _vp, _i32, _i32, _vp]),
    ("m1moe_cuda_dense_attention", ctypes.c_int, [_vp, _i32, _vp, _i32, _vp, _vp]),
    ("m1moe_cuda_dense_lm_head", ctypes.c_int, [_vp, _vp, _i32, _vp, _vp, _vp]),
    ("m1moe_cuda_decode_step", ctypes.c_int, [_vp, _vp, _vp, _i32, _vp, _vp, _vp]),
    ("m1moe_cuda_prefill_step", ctypes.c_int, [_vp, _vp, _vp, _i32, _vp, _vp, _vp]),
]


def lib() -> ctypes.CDLL:
    """Load libm1moe_cuda.so (once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m m1moe_b200.build` "
                "(m1moe_b200 has no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, res, args in _SIGS:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, func: str) -> None:
    if status != M1MOE_OK:
        msg = lib().m1moe_cuda_last_error()
        raise M1MoECudaError(status, func, msg.decode() if msg else "")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
