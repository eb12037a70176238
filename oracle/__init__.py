"""CPU oracle for M1MoE's int4 expert FFN — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this package, and only as the checker or the timed CPU baseline; the product
package (m1moe_b200) never imports it.

It wraps m1moe_oracle.c (a C restatement of Shaders.metal:11-14, 39-92,
138-149, 360-376 and InferenceEngine.swift:79-97, 490-519) through ctypes.
Parity pin: the format and dequant rule are checked against fixtures that the
reference's own quantiser/extractor produced (tests/golden/make_golden.py);
the Metal/Swift arithmetic cannot execute here, so the kernel-order restatement
is pinned by source semantics only.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "m1moe_oracle.c"
LIB = HERE / "liboracle_m1moe.so"
# x86-64-v3 (AVX2+FMA) rather than -march=native: the library is built in one
# container and may run on another host.
CFLAGS = ["-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fPIC", "-shared", "-pthread",
          "-std=c11"]

_lib = None


def build(force: bool = False) -> Path:
    if force or not LIB.exists() or LIB.stat().st_mtime < max(
            SRC.stat().st_mtime, (HERE / "m1moe_oracle.h").stat().st_mtime):
        tmp = LIB.with_suffix(".so.tmp")
        subprocess.run(["gcc", *CFLAGS, str(SRC), "-o", str(tmp), "-lm"], check=True)
        os.replace(tmp, LIB)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = ctypes.CDLL(str(LIB))
        u8p = ctypes.POINTER(ctypes.c_uint8)
        u16p = ctypes.POINTER(ctypes.c_uint16)
        u32p = ctypes.POINTER(ctypes.c_uint32)
        f32p = ctypes.POINTER(ctypes.c_float)
        i32p = ctypes.POINTER(ctypes.c_int32)
        c_int = ctypes.c_int
        L.orc_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_bf16_to_f32.restype = ctypes.c_float
        L.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        L.orc_f32_to_bf16.restype = ctypes.c_uint16
        L.orc_expert_bytes.argtypes = [c_int, c_int, c_int]
        L.orc_expert_bytes.restype = ctypes.c_size_t
        L.orc_expert_offsets.argtypes = [c_int, c_int, c_int, ctypes.POINTER(ctypes.c_size_t)]
        L.orc_matvec4bit.argtypes = [u32p, u16p, u16p, f32p, f32p, c_int, c_int, c_int]
        L.orc_matvec4bit_mt.argtypes = [u32p, u16p, u16p, f32p, f32p, c_int, c_int, c_int, c_int]
        L.orc_matvec4bit_rows.argtypes = [u32p, u16p, u16p, f32p, f32p, c_int, c_int, c_int,
                                          c_int, c_int]
        L.orc_swiglu.argtypes = [f32p, f32p, f32p, c_int]
        L.orc_moe_combine.argtypes = [f32p, f32p, f32p, f32p, c_int, c_int]
        L.orc_router_scores.argtypes = [u16p, f32p, c_int, c_int, f32p]
        L.orc_select_topk.argtypes = [f32p, c_int, c_int, c_int, i32p, f32p]
        L.orc_expert_forward.argtypes = [u8p, f32p, c_int, c_int, c_int, f32p, f32p]
        L.orc_moe_layer.argtypes = [u8p, u16p, f32p, f32p, f32p, c_int, c_int, c_int, c_int,
                                    c_int, c_int, c_int, i32p, f32p, c_int]
        L.orc_moe_layer.restype = c_int
        _lib = L
    return _lib


def _p(a: np.ndarray, ct):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.POINTER(ct))


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def expert_bytes(h: int, inter: int, gs: int) -> int:
    return int(lib().orc_expert_bytes(h, inter, gs))


def expert_offsets(h: int, inter: int, gs: int) -> list[int]:
    arr = (ctypes.c_size_t * 9)()
    lib().orc_expert_offsets(h, inter, gs, arr)
    return list(arr)


def matvec4bit(W: np.ndarray, S: np.ndarray, B: np.ndarray, x: np.ndarray, gs: int,
               nthreads: int = 1) -> np.ndarray:
    """Shaders.metal:39-92 on the CPU. W uint32[out][in/8], S/B uint16[out][in/gs], x f32[in]."""
    W = np.ascontiguousarray(W, dtype=np.uint32)
    S = np.ascontiguousarray(S, dtype=np.uint16)
    B = np.ascontiguousarray(B, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.float32)
    out_dim, in_dim = W.shape[0], W.shape[1] * 8
    assert x.shape == (in_dim,)
    y = np.empty(out_dim, dtype=np.float32)
    lib().orc_matvec4bit_mt(_p(W, ctypes.c_uint32), _p(S, ctypes.c_uint16),
                            _p(B, ctypes.c_uint16), _p(x, ctypes.c_float),
                            _p(y, ctypes.c_float), out_dim, in_dim, gs, nthreads)
    return y


def matvec4bit_plain(W: np.ndarray, S: np.ndarray, B: np.ndarray, x: np.ndarray,
                     gs: int) -> np.ndarray:
    """The literal lane-by-lane restatement of Shaders.metal:39-92 (lanes outermost,
    single thread); matvec4bit() runs the lane-vectorised form, bit-identical."""
    W = np.ascontiguousarray(W, dtype=np.uint32)
    S = np.ascontiguousarray(S, dtype=np.uint16)
    B = np.ascontiguousarray(B, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.float32)
    out_dim, in_dim = W.shape[0], W.shape[1] * 8
    y = np.empty(out_dim, dtype=np.float32)
    lib().orc_matvec4bit_rows(_p(W, ctypes.c_uint32), _p(S, ctypes.c_uint16),
                              _p(B, ctypes.c_uint16), _p(x, ctypes.c_float),
                              _p(y, ctypes.c_float), out_dim, in_dim, gs, 0, out_dim)
    return y


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    gate = np.ascontiguousarray(gate, dtype=np.float32)
    up = np.ascontiguousarray(up, dtype=np.float32)
    act = np.empty_like(gate)
    lib().orc_swiglu(_p(gate, ctypes.c_float), _p(up, ctypes.c_float), _p(act, ctypes.c_float),
                     gate.size)
    return act


def router_scores(router_bf16: np.ndarray, x: np.ndarray) -> np.ndarray:
    router_bf16 = np.ascontiguousarray(router_bf16, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.float32)
    E, h = router_bf16.shape
    s = np.empty(E, dtype=np.float32)
    lib().orc_router_scores(_p(router_bf16, ctypes.c_uint16), _p(x, ctypes.c_float), E, h,
                            _p(s, ctypes.c_float))
    return s


def select_topk(scores: np.ndarray, K: int, norm: bool):
    scores = np.ascontiguousarray(scores, dtype=np.float32)
    idx = np.empty(K, dtype=np.int32)
    w = np.empty(K, dtype=np.float32)
    lib().orc_select_topk(_p(scores, ctypes.c_float), scores.size, K, int(norm),
                          _p(idx, ctypes.c_int32), _p(w, ctypes.c_float))
    return idx, w


def expert_forward(block: np.ndarray, x: np.ndarray, h: int, inter: int, gs: int) -> np.ndarray:
    block = np.ascontiguousarray(block, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(h, dtype=np.float32)
    scratch = np.empty(3 * inter, dtype=np.float32)
    lib().orc_expert_forward(_p(block, ctypes.c_uint8), _p(x, ctypes.c_float), h, inter, gs,
                             _p(y, ctypes.c_float), _p(scratch, ctypes.c_float))
    return y


def moe_layer(table: np.ndarray, router_bf16: np.ndarray, x: np.ndarray, residual, *, h: int,
              inter: int, E: int, K: int, gs: int, norm: bool, nthreads: int = 1):
    """MoE part of InferenceEngine.runLayer (:240-266) for B tokens.

    table: uint8 image of one layer_NN.bin; x, residual: f32 [B][h] (residual may be None).
    Returns (out f32[B][h], idx int32[B][K], w f32[B][K]).
    """
    table = np.ascontiguousarray(table, dtype=np.uint8)
    router_bf16 = np.ascontiguousarray(router_bf16, dtype=np.uint16)
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    B = x.shape[0]
    res = (np.zeros_like(x) if residual is None
           else np.ascontiguousarray(np.atleast_2d(residual), dtype=np.float32))
    out = np.empty((B, h), dtype=np.float32)
    idx = np.empty((B, K), dtype=np.int32)
    w = np.empty((B, K), dtype=np.float32)
    rc = lib().orc_moe_layer(_p(table, ctypes.c_uint8), _p(router_bf16, ctypes.c_uint16),
                             _p(x, ctypes.c_float), _p(res, ctypes.c_float),
                             _p(out, ctypes.c_float), B, h, inter, E, K, gs, int(norm),
                             _p(idx, ctypes.c_int32), _p(w, ctypes.c_float), nthreads)
    if rc != 0:
        raise RuntimeError(f"orc_moe_layer failed ({rc})")
    return out, idx, w
