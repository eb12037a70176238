"""DenseModel — the non-expert half of a decode step, and the whole step.

Host-side mirror of the rest of the reference's InferenceEngine
(Sources/M1MoE/InferenceEngine.swift): `load` takes the WeightStore tensors
(model_weights.bin, WeightStore.swift:47-126) by their m1moe_dense_tensor
name; `gemv`, `rmsnorm`, `attention` and `lm_head` are the encoders and CPU
steps of runLayer and forward (:167-238, :140-155, :298-399, :521-555);
`step` is forward() at temperature 0 for a batch of sequences, with the MoE
block of an MoEBlock.  All work happens in libm1moe_cuda.so through the C ABI;
torch supplies device buffers and streams only.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .expert_ffn import _check_cuda, _stream, dtype_code

_TENSORS = {"embed": _lib.W_EMBED, "final_norm": _lib.W_FINAL_NORM, "lm_head": _lib.W_LM_HEAD,
            "in_norm": _lib.W_INPUT_NORM, "post_norm": _lib.W_POST_NORM, "wq": _lib.W_Q,
            "wk": _lib.W_K, "wv": _lib.W_V, "wo": _lib.W_O, "qn": _lib.W_Q_NORM, "kn": _lib.W_K_NORM}
PER_LAYER = ("in_norm", "post_norm", "wq", "wk", "wv", "wo", "qn", "kn")


class DenseModel:
    def __init__(self, *, hidden_dim: int, num_heads: int, num_kv_heads: int, num_layers: int,
                 vocab_size: int, qk_norm: bool, rms_norm_eps: float = 1e-5,
                 rope_theta: float = 10000.0, head_dim: int = 128, max_batch: int = 1,
                 max_seq: int = 4096, device: int = 0):
        self.cfg = _lib.DenseCfg(hidden_dim, num_heads, num_kv_heads, head_dim, num_layers,
                                 vocab_size, int(qk_norm), rms_norm_eps, rope_theta, max_batch,
                                 max_seq, device)
        self.hidden_dim, self.num_heads, self.num_kv_heads = hidden_dim, num_heads, num_kv_heads
        self.head_dim, self.num_layers, self.vocab_size = head_dim, num_layers, vocab_size
        self.max_batch, self.max_seq, self.device = max_batch, max_seq, device
        self.qk_norm = qk_norm
        h = ctypes.c_void_p()
        _lib.call("m1moe_cuda_dense_create", ctypes.byref(self.cfg), ctypes.byref(h))
        self._ctx = h

    # ------------------------------------------------------------ lifetime --
    def close(self) -> None:
        if getattr(self, "_ctx", None):
            _lib.call("m1moe_cuda_dense_destroy", self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ------------------------------------------------------------- loading --
    def load(self, name: str, data, layer: int = 0) -> None:
        """One bf16 tensor (numpy uint16 bit patterns, or a CUDA tensor of 2-byte elements)."""
        t = _TENSORS[name]
        if isinstance(data, torch.Tensor) and data.is_cuda:
            _check_cuda(data)
            _lib.call("m1moe_cuda_dense_load_device", self._ctx, t, layer, data.data_ptr(),
                      data.numel(), _stream())
            return
        if isinstance(data, torch.Tensor):
            data = data.view(torch.int16).numpy().view(np.uint16)
        a = np.ascontiguousarray(data, dtype=np.uint16)
        _lib.call("m1moe_cuda_dense_load", self._ctx, t, layer, a.ctypes.data, a.size)

    def load_all(self, weights: dict) -> None:
        """weights: the tensors by name; per-layer ones as lists."""
        for name, v in weights.items():
            if name not in _TENSORS or (name in ("qn", "kn") and not self.qk_norm):
                continue
            if name in PER_LAYER:
                for L, w in enumerate(v):
                    self.load(name, w, L)
            else:
                self.load(name, v)

    def kv_cache(self, layer: int):
        """(k, v) of one layer as torch bf16 views [max_batch][nkv][max_seq][hd]."""
        k, v = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.call("m1moe_cuda_dense_kv_cache", self._ctx, layer, ctypes.byref(k), ctypes.byref(v))
        shape = (self.max_batch, self.num_kv_heads, self.max_seq, self.head_dim)
        n = int(np.prod(shape))
        out = []
        for ptr in (k.value, v.value):
            out.append(_from_ptr(ptr, n, self.device).view(shape))
        return tuple(out)

    def set_position(self, pos: int) -> None:
        _lib.call("m1moe_cuda_dense_set_position", self._ctx, pos)

    def position(self) -> int:
        v = ctypes.c_int32()
        _lib.call("m1moe_cuda_dense_get_position", self._ctx, ctypes.byref(v))
        return v.value

    def reset(self) -> None:
        _lib.call("m1moe_cuda_dense_reset", self._ctx)

    def synchronize(self) -> None:
        _lib.call("m1moe_cuda_dense_synchronize", self._ctx)

    # ------------------------------------------------------------- compute --
    def attention(self, layer: int, qkv: torch.Tensor, *, out: torch.Tensor | None = None,
                  stream=None) -> torch.Tensor:
        B = qkv.shape[0]
        if out is None:
            out = torch.empty((B, self.num_heads * self.head_dim), dtype=torch.float32,
                              device=qkv.device)
        _check_cuda(qkv, out)
        _lib.call("m1moe_cuda_dense_attention", self._ctx, layer, qkv.data_ptr(), B, out.data_ptr(),
                  _stream(stream))
        return out

    def lm_head(self, x: torch.Tensor, *, logits: bool = True, stream=None):
        B = x.shape[0]
        tok = torch.empty((B,), dtype=torch.int32, device=x.device)
        lg = torch.empty((B, self.vocab_size), dtype=torch.float32, device=x.device) if logits else None
        _check_cuda(x)
        _lib.call("m1moe_cuda_dense_lm_head", self._ctx, x.data_ptr(), B, tok.data_ptr(),
                  lg.data_ptr() if lg is not None else 0, _stream(stream))
        return tok, lg

    def prefill(self, moe, tokens: torch.Tensor, *, logits: torch.Tensor | None = None, stream=None):
        """Token-parallel prefill of the prompt tokens [T] (int32, CUDA) into
        sequence slot 0 at the current position: returns the greedy next token
        [1] (and fills `logits` [vocab] if given); the position advances by T."""
        T = tokens.shape[0]
        nxt = torch.empty((1,), dtype=torch.int32, device=tokens.device)
        _check_cuda(tokens)
        _lib.call("m1moe_cuda_prefill_step", self._ctx, moe._ctx, tokens.data_ptr(), T, nxt.data_ptr(),
                  logits.data_ptr() if logits is not None else 0, _stream(stream))
        return nxt

    def step(self, moe, tokens: torch.Tensor, *, next_tokens: torch.Tensor | None = None,
             logits: torch.Tensor | None = None, stream=None):
        """One decode step for tokens [B] (int32, CUDA): returns the next tokens
        (and fills `logits` [B][vocab] if given); the position advances by one."""
        B = tokens.shape[0]
        if next_tokens is None:
            next_tokens = torch.empty((B,), dtype=torch.int32, device=tokens.device)
        _check_cuda(tokens, next_tokens)
        _lib.call("m1moe_cuda_decode_step", self._ctx, moe._ctx, tokens.data_ptr(), B,
                  next_tokens.data_ptr(), logits.data_ptr() if logits is not None else 0,
                  _stream(stream))
        return next_tokens


def _from_ptr(ptr: int, n: int, device: int) -> torch.Tensor:
    """A torch bf16 view of n elements of device memory that the library owns
    (valid while its context lives), through __cuda_array_interface__."""
    class _Arr:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "<i2", "data": (ptr, False),
                                    "version": 3}
    return torch.as_tensor(_Arr(), device=f"cuda:{device}").view(torch.bfloat16)


def gemv(w: torch.Tensor, x: torch.Tensor, *, norm_w: torch.Tensor | None = None, eps: float = 1e-5,
         residual: torch.Tensor | None = None, out: torch.Tensor | None = None, stream=None):
    """y = W . (rmsnorm(x) * norm_w or x) (+ residual), bf16 W [rows][K], x [B][K]."""
    x2 = x.unsqueeze(0) if x.dim() == 1 else x
    B, K = x2.shape
    rows = w.shape[0]
    if out is None:
        out = torch.empty((B, rows), dtype=torch.float32, device=x.device)
    _check_cuda(w, x2, out)
    _lib.call("m1moe_cuda_dense_gemv", w.data_ptr(), rows, K, x2.data_ptr(), dtype_code(x2.dtype),
              norm_w.data_ptr() if norm_w is not None else 0, eps,
              residual.data_ptr() if residual is not None else 0, out.data_ptr(), B, _stream(stream))
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-5, *, out=None, stream=None):
    x2 = x.unsqueeze(0) if x.dim() == 1 else x
    B, D = x2.shape
    if out is None:
        out = torch.empty((B, D), dtype=torch.float32, device=x.device)
    _check_cuda(x2, w, out)
    _lib.call("m1moe_cuda_dense_rmsnorm", x2.data_ptr(), dtype_code(x2.dtype), w.data_ptr(), eps,
              out.data_ptr(), D, B, _stream(stream))
    return out
