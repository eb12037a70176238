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
        L.orc_rmsnorm.argtypes = [f32p, u16p, ctypes.c_float, f32p, c_int]
        L.orc_matvec_bf16.argtypes = [u16p, f32p, f32p, c_int, c_int, c_int]
        L.orc_head_rmsnorm.argtypes = [f32p, c_int, c_int, u16p, ctypes.c_float]
        L.orc_rope.argtypes = [f32p, c_int, c_int, ctypes.c_float, c_int]
        L.orc_attention.argtypes = [f32p, u16p, u16p, c_int, c_int, c_int, c_int, c_int, f32p]
        L.orc_argmax.argtypes = [f32p, c_int]
        L.orc_argmax.restype = c_int
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


# ------------------------------------------------------------------ dense ----
def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _u16(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint16)


def rmsnorm(x: np.ndarray, w_bf16: np.ndarray, eps: float) -> np.ndarray:
    """Shaders.metal:97-134 for one vector."""
    x, w = _f32(x), _u16(w_bf16)
    y = np.empty_like(x)
    lib().orc_rmsnorm(_p(x, ctypes.c_float), _p(w, ctypes.c_uint16), eps, _p(y, ctypes.c_float), x.size)
    return y


def matvec_bf16(W_bf16: np.ndarray, x: np.ndarray, nthreads: int = 1) -> np.ndarray:
    """Shaders.metal:328-353: bf16 W [out][in] times f32 x."""
    W, x = _u16(W_bf16), _f32(x)
    y = np.empty(W.shape[0], dtype=np.float32)
    lib().orc_matvec_bf16(_p(W, ctypes.c_uint16), _p(x, ctypes.c_float), _p(y, ctypes.c_float),
                          W.shape[0], W.shape[1], nthreads)
    return y


def head_rmsnorm(buf: np.ndarray, num_heads: int, head_dim: int, w_bf16: np.ndarray,
                 eps: float) -> np.ndarray:
    b, w = _f32(buf).copy(), _u16(w_bf16)
    lib().orc_head_rmsnorm(_p(b, ctypes.c_float), num_heads, head_dim, _p(w, ctypes.c_uint16), eps)
    return b


def rope(buf: np.ndarray, num_heads: int, head_dim: int, theta: float, pos: int) -> np.ndarray:
    b = _f32(buf).copy()
    lib().orc_rope(_p(b, ctypes.c_float), num_heads, head_dim, theta, pos)
    return b


def attention(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, num_heads: int, num_kv_heads: int,
              head_dim: int, seq_len: int) -> np.ndarray:
    """Shaders.metal:209-313 for one sequence; kc/vc bf16 [nkv][max_seq][hd]."""
    q, kc, vc = _f32(q), _u16(kc), _u16(vc)
    out = np.empty(num_heads * head_dim, dtype=np.float32)
    lib().orc_attention(_p(q, ctypes.c_float), _p(kc, ctypes.c_uint16), _p(vc, ctypes.c_uint16),
                        num_heads, num_kv_heads, head_dim, kc.shape[1], seq_len,
                        _p(out, ctypes.c_float))
    return out


def argmax(logits: np.ndarray) -> int:
    lg = _f32(logits)
    return int(lib().orc_argmax(_p(lg, ctypes.c_float), lg.size))


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round to nearest even (the cache store's rounding)."""
    u = _f32(a).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def decode_step(dense: dict, moe: dict, kv: list, tokens, pos: int, nthreads: int = 1):
    """InferenceEngine.forward (:124-156) at temperature 0 for a batch of
    sequences at one position, composed from the restatements above and
    moe_layer (runLayer, :167-267).

    dense: cfg keys h, nh, nkv, hd, layers, vocab, eps, theta, qk_norm and the
    bf16 tensors embed, final_norm, lm_head, and per layer (lists) in_norm,
    post_norm, wq, wk, wv, wo, qn, kn.  moe: tables (layer images), routers,
    inter, E, K, gs, norm.  kv: per layer (k, v) bf16 arrays
    [batch][nkv][max_seq][hd], updated in place at `pos` (k and v rounded to
    bf16 as the B200 cache stores them; the reference keeps f32 rows).
    Returns (next tokens, logits [batch][vocab])."""
    h, nh, nkv, hd = dense["h"], dense["nh"], dense["nkv"], dense["hd"]
    eps, theta = dense["eps"], dense["theta"]
    toks, all_logits = [], []
    for b, tok in enumerate(tokens):
        residual = bf16_to_f32(dense["embed"][tok]).astype(np.float32)
        for L in range(dense["layers"]):
            xn = rmsnorm(residual, dense["in_norm"][L], eps)
            q = matvec_bf16(dense["wq"][L], xn, nthreads)
            k = matvec_bf16(dense["wk"][L], xn, nthreads)
            v = matvec_bf16(dense["wv"][L], xn, nthreads)
            if dense["qk_norm"]:
                q = head_rmsnorm(q, nh, hd, dense["qn"][L], eps)
                k = head_rmsnorm(k, nkv, hd, dense["kn"][L], eps)
            q = rope(q, nh, hd, theta, pos)
            k = rope(k, nkv, hd, theta, pos)
            kc, vc = kv[L]
            kc[b, :, pos, :] = f32_to_bf16_bits(k).reshape(nkv, hd)
            vc[b, :, pos, :] = f32_to_bf16_bits(v).reshape(nkv, hd)
            att = attention(q, kc[b], vc[b], nh, nkv, hd, pos + 1)
            o = matvec_bf16(dense["wo"][L], att, nthreads)
            residual = (residual + o).astype(np.float32)  # residualAdd
            h_mid = rmsnorm(residual, dense["post_norm"][L], eps)
            out, _, _ = moe_layer(moe["tables"][L], moe["routers"][L], h_mid[None, :],
                                  residual[None, :], h=h, inter=moe["inter"], E=moe["E"],
                                  K=moe["K"], gs=moe["gs"], norm=moe["norm"], nthreads=nthreads)
            residual = out[0]
        xn = rmsnorm(residual, dense["final_norm"], eps)
        logits = matvec_bf16(dense["lm_head"], xn, nthreads)
        toks.append(argmax(logits))
        all_logits.append(logits)
    return np.array(toks, dtype=np.int32), np.stack(all_logits)
