"""m1moe_b200 — B200 (sm_100a) int4 group-quantised MoE expert FFN.

A from-scratch CUDA implementation of M1MoE's hot path (the 4-bit expert FFN:
router softmax/top-K, SwiGLU gate/up/down dequant-matvecs, weighted combine)
behind the C ABI in include/m1moe_cuda.h.  This package is the Python host
side of that ABI; the computation lives in _lib/libm1moe_cuda.so.
"""
from . import _lib
from .spec import MIXTRAL_8X7B, OLMOE_1B_7B, ModelSpec, expert_bytes, expert_offsets

__all__ = ["ModelSpec", "OLMOE_1B_7B", "MIXTRAL_8X7B", "expert_bytes", "expert_offsets",
           "MoEBlock", "matvec4", "matvec4_strided", "unpack4", "M1MoECudaError", "library"]

M1MoECudaError = _lib.M1MoECudaError


def library():
    """The loaded libm1moe_cuda.so (ctypes.CDLL); raises if it has not been built."""
    return _lib.lib()


def __getattr__(name):
    # torch-facing modules load lazily so that `import m1moe_b200` stays cheap.
    if name == "MoEBlock":
        from .moe_block import MoEBlock
        return MoEBlock
    if name in ("matvec4", "matvec4_strided", "unpack4"):
        from . import expert_ffn
        return getattr(expert_ffn, name)
    raise AttributeError(name)
