"""Stateless int4 expert-FFN operators on torch CUDA tensors.

Thin wrappers over the C ABI (include/m1moe_cuda.h).  torch supplies device
memory and the current stream; every computation runs in libm1moe_cuda.so.

  matvec4          encode4BitMV + matvec4bit (InferenceEngine.swift:446-465,
                   Shaders.metal:39-92), batch 1..8 tokens
  matvec4_strided  the same over many matrices a fixed stride apart
  unpack4          the nibble unpack of Shaders.metal:73-74, for bit-exact checks
"""
from __future__ import annotations

import torch

from . import _lib

_DT = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DT[t]
    except KeyError:
        raise TypeError(f"activations must be float32 or bfloat16, got {t}") from None


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _check_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise ValueError("m1moe_b200 operators take CUDA tensors")
        if not t.is_contiguous():
            raise ValueError("m1moe_b200 operators take contiguous tensors")


def matvec4(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, x: torch.Tensor, *,
            group_size: int = 64, out: torch.Tensor | None = None,
            out_dtype: torch.dtype = torch.float32, stream=None) -> torch.Tensor:
    """y[t] = dequant(W) @ x[t].  w int32/uint32 [out][in/8]; scales/biases bf16/int16
    [out][in/gs]; x [in] or [batch][in] (f32 or bf16)."""
    x2 = x.unsqueeze(0) if x.dim() == 1 else x
    out_dim, in_dim = w.shape[0], w.shape[1] * 8
    if x2.shape[-1] != in_dim:
        raise ValueError(f"x has {x2.shape[-1]} columns, W has {in_dim}")
    if out is None:
        out = torch.empty((x2.shape[0], out_dim), dtype=out_dtype, device=w.device)
    _check_cuda(w, scales, biases, x2, out)
    _lib.call("m1moe_cuda_matvec4", w.data_ptr(), scales.data_ptr(), biases.data_ptr(),
              x2.data_ptr(), dtype_code(x2.dtype), out.data_ptr(), dtype_code(out.dtype), out_dim,
              in_dim, group_size, x2.shape[0], _stream(stream))
    return out.squeeze(0) if x.dim() == 1 else out


def matvec4_strided(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                    mat_stride_bytes: int, num_mats: int, out_dim: int, in_dim: int,
                    x: torch.Tensor, *, group_size: int = 64, out: torch.Tensor | None = None,
                    out_dtype: torch.dtype = torch.float32, stream=None) -> torch.Tensor:
    """y[m][t] for num_mats matrices whose W/S/B start mat_stride_bytes apart.
    w/scales/biases are tensors whose data_ptr is the first matrix's W/S/B."""
    x2 = x.unsqueeze(0) if x.dim() == 1 else x
    if out is None:
        out = torch.empty((num_mats, x2.shape[0], out_dim), dtype=out_dtype, device=x.device)
    _check_cuda(x2, out)
    _lib.call("m1moe_cuda_matvec4_strided", w.data_ptr(), scales.data_ptr(), biases.data_ptr(),
              mat_stride_bytes, num_mats, x2.data_ptr(), dtype_code(x2.dtype), out.data_ptr(),
              dtype_code(out.dtype), out_dim, in_dim, group_size, x2.shape[0], _stream(stream))
    return out


def unpack4(w: torch.Tensor, stream=None) -> torch.Tensor:
    """uint8 q[rows][cols] from packed uint32 W[rows][cols/8]."""
    rows, cols = w.shape[0], w.shape[1] * 8
    q = torch.empty((rows, cols), dtype=torch.uint8, device=w.device)
    _check_cuda(w, q)
    _lib.call("m1moe_cuda_unpack4", w.data_ptr(), q.data_ptr(), rows, cols, _stream(stream))
    return q
