"""MoEBlock — the HBM-resident MoE block of every layer of one model.

Host-side mirror of the MoE part of the reference's InferenceEngine
(Sources/M1MoE/InferenceEngine.swift): the per-layer expert table replaces
the expert fds + per-token pread (:62-97, :271-280), `load_router` replaces the
router preconvert (:99-113), `route` is computeRouterScores + selectTopK
(:490-519), and `forward` is runLayer's router -> experts -> moeCombine
sequence (:240-266).  All work happens in libm1moe_cuda.so through the C ABI;
torch supplies device buffers and streams only.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .expert_ffn import _check_cuda, _stream, dtype_code
from .spec import ModelSpec


class MoEBlock:
    def __init__(self, *, hidden_dim: int, intermediate_dim: int, num_experts: int, top_k: int,
                 group_size: int = 64, num_layers: int = 1, norm_topk_prob: bool = False,
                 max_batch: int = 1, device: int = 0, expert_begin: int = 0,
                 expert_count: int = 0):
        self.cfg = _lib.Cfg(hidden_dim, intermediate_dim, num_experts, top_k, group_size,
                            num_layers, int(norm_topk_prob), max_batch, device, expert_begin,
                            expert_count)
        self.hidden_dim, self.intermediate_dim = hidden_dim, intermediate_dim
        self.num_experts, self.top_k, self.group_size = num_experts, top_k, group_size
        self.num_layers, self.max_batch, self.device = num_layers, max_batch, device
        self.expert_begin = expert_begin
        self.expert_count = expert_count or num_experts
        self.expert_bytes = int(_lib.lib().m1moe_cuda_expert_bytes(hidden_dim, intermediate_dim,
                                                                    group_size))
        h = ctypes.c_void_p()
        _lib.call("m1moe_cuda_create", ctypes.byref(self.cfg), ctypes.byref(h))
        self._ctx = h

    @classmethod
    def from_spec(cls, spec: ModelSpec, **kw) -> "MoEBlock":
        return cls(hidden_dim=spec.hidden_dim, intermediate_dim=spec.moe.intermediate_dim,
                   num_experts=spec.moe.num_experts, top_k=spec.moe.top_k,
                   group_size=spec.quantization.group_size, num_layers=spec.num_layers,
                   norm_topk_prob=spec.moe.norm_topk_prob, **kw)

    # ------------------------------------------------------------ lifetime --
    def close(self) -> None:
        if getattr(self, "_ctx", None):
            _lib.call("m1moe_cuda_destroy", self._ctx)
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
    def load_expert_layer(self, layer: int, data) -> None:
        """data: the bytes of packed_experts/layer_NN.bin (numpy uint8, bytes) or a CUDA
        uint8 tensor holding the same image."""
        if isinstance(data, torch.Tensor):
            if not data.is_cuda:
                data = data.numpy()
            else:
                _check_cuda(data)
                _lib.call("m1moe_cuda_load_expert_layer_device", self._ctx, layer,
                          data.data_ptr(), data.numel() * data.element_size(), _stream())
                return
        buf = np.ascontiguousarray(np.frombuffer(data, dtype=np.uint8)
                                   if isinstance(data, (bytes, bytearray, memoryview)) else data)
        _lib.call("m1moe_cuda_load_expert_layer", self._ctx, layer,
                  buf.ctypes.data, buf.nbytes)

    def load_expert_files(self, packed_experts_dir, io_threads: int = 4) -> None:
        """Cold start: every packed_experts/layer_NN.bin of the converted model
        directory, read by `io_threads` native threads while earlier chunks are
        copied and repacked (m1moe_cuda_load_expert_files).  Raises
        M1MoECudaError (INVALID_ARG) naming a missing or wrong-sized file."""
        _lib.call("m1moe_cuda_load_expert_files", self._ctx, str(packed_experts_dir).encode(),
                  io_threads)

    def load_router(self, layer: int, router_bf16) -> None:
        """router_bf16: bf16 bit patterns [num_experts][hidden_dim] (numpy uint16)."""
        if isinstance(router_bf16, torch.Tensor):
            router_bf16 = router_bf16.detach().cpu().view(torch.int16).numpy().view(np.uint16)
        r = np.ascontiguousarray(router_bf16, dtype=np.uint16)
        _lib.call("m1moe_cuda_load_router", self._ctx, layer, r.ctypes.data, r.size)

    # ------------------------------------------------------------- compute --
    def route(self, layer: int, x: torch.Tensor, stream=None):
        """Top-K experts, their weights and the softmax scores for x [B][h]."""
        x2 = x.unsqueeze(0) if x.dim() == 1 else x
        B = x2.shape[0]
        idx = torch.empty((B, self.top_k), dtype=torch.int32, device=x.device)
        w = torch.empty((B, self.top_k), dtype=torch.float32, device=x.device)
        scores = torch.empty((B, self.num_experts), dtype=torch.float32, device=x.device)
        _check_cuda(x2)
        _lib.call("m1moe_cuda_router_topk", self._ctx, layer, x2.data_ptr(), dtype_code(x2.dtype),
                  B, idx.data_ptr(), w.data_ptr(), scores.data_ptr(), _stream(stream))
        return idx, w, scores

    def forward(self, layer: int, x: torch.Tensor, residual: torch.Tensor | None = None, *,
                out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.float32,
                return_topk: bool = False, stream=None):
        """out[t] = residual[t] + sum_k w[t][k] * Expert_{idx[t][k]}(x[t]) for x [B][h]."""
        x2 = x.unsqueeze(0) if x.dim() == 1 else x
        B = x2.shape[0]
        if out is None:
            out = torch.empty((B, self.hidden_dim), dtype=out_dtype, device=x.device)
        _check_cuda(x2, out)
        res_ptr, res_dt = 0, 0
        if residual is not None:
            r2 = residual.unsqueeze(0) if residual.dim() == 1 else residual
            _check_cuda(r2)
            res_ptr, res_dt = r2.data_ptr(), dtype_code(r2.dtype)
        idx = w = None
        if return_topk:
            idx = torch.empty((B, self.top_k), dtype=torch.int32, device=x.device)
            w = torch.empty((B, self.top_k), dtype=torch.float32, device=x.device)
        _lib.call("m1moe_cuda_moe_layer", self._ctx, layer, x2.data_ptr(), dtype_code(x2.dtype),
                  res_ptr, res_dt, out.data_ptr(), dtype_code(out.dtype), B,
                  idx.data_ptr() if idx is not None else 0,
                  w.data_ptr() if w is not None else 0, _stream(stream))
        out_v = out.squeeze(0) if x.dim() == 1 else out
        return (out_v, idx, w) if return_topk else out_v

    def prefill(self, layer: int, x: torch.Tensor, residual: torch.Tensor | None = None, *,
                out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.float32,
                return_topk: bool = False, stream=None):
        """forward() for many tokens x [T][h] at once: grouped GEMMs on the tensor
        cores (m1moe_cuda_moe_prefill); the same result within the FFN tolerance."""
        x2 = x.unsqueeze(0) if x.dim() == 1 else x
        T = x2.shape[0]
        if out is None:
            out = torch.empty((T, self.hidden_dim), dtype=out_dtype, device=x.device)
        _check_cuda(x2, out)
        res_ptr, res_dt = 0, 0
        if residual is not None:
            r2 = residual.unsqueeze(0) if residual.dim() == 1 else residual
            _check_cuda(r2)
            res_ptr, res_dt = r2.data_ptr(), dtype_code(r2.dtype)
        idx = w = None
        if return_topk:
            idx = torch.empty((T, self.top_k), dtype=torch.int32, device=x.device)
            w = torch.empty((T, self.top_k), dtype=torch.float32, device=x.device)
        _lib.call("m1moe_cuda_moe_prefill", self._ctx, layer, x2.data_ptr(), dtype_code(x2.dtype),
                  res_ptr, res_dt, out.data_ptr(), dtype_code(out.dtype), T,
                  idx.data_ptr() if idx is not None else 0,
                  w.data_ptr() if w is not None else 0, _stream(stream))
        out_v = out.squeeze(0) if x.dim() == 1 else out
        return (out_v, idx, w) if return_topk else out_v

    def forward_host(self, layer: int, x: np.ndarray, residual: np.ndarray | None = None):
        """Synchronous host-buffer call with the reference's f32 buffers.
        Returns (out f32[B][h], idx int32[B][K], w f32[B][K])."""
        x2 = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
        B = x2.shape[0]
        out = np.empty_like(x2)
        idx = np.empty((B, self.top_k), dtype=np.int32)
        w = np.empty((B, self.top_k), dtype=np.float32)
        res = None if residual is None else np.ascontiguousarray(np.atleast_2d(residual),
                                                                 dtype=np.float32)
        _lib.call("m1moe_cuda_moe_layer_host", self._ctx, layer, x2.ctypes.data,
                  res.ctypes.data if res is not None else 0, out.ctypes.data, B,
                  idx.ctypes.data, w.ctypes.data)
        return out, idx, w

    def synchronize(self) -> None:
        _lib.call("m1moe_cuda_synchronize", self._ctx)
