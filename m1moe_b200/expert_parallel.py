"""Expert parallelism for the MoE block across ranks (one process per GPU).

Experts are independent, so a layer's E experts are split into contiguous
equal shards, one per rank (expert_begin/expert_count of m1moe_cuda_cfg).
Every rank owns `tokens_per_rank` decode tokens.  One step, per layer:

  1. all-gather every rank's tokens (the hidden state is small: h floats);
  2. each rank applies its local experts to every gathered token routed to
     them (m1moe_cuda_moe_layer with the shard's context), adding the
     residual only for the tokens it owns, so the residual enters once;
  3. reduce-scatter the partial sums back to the tokens' owners.

EPStep does this with torch.distributed collectives (NCCL over NVLink on GPUs,
gloo on CPU for the tests); the buffers are preallocated so that a step can be
captured in a CUDA graph, and the local computation is a callable, which lets
the CPU tests substitute a reference computation for the CUDA kernel.
EPFused does the same exchange inside the MoE kernel over NVLink peer memory
(m1moe_cuda_moe_layer_ep: each CTA pushes its slice of the rank's tokens into
every rank's exchange region, the last CTA sends each rank its tokens' partial
sums and adds those it receives), so a layer is one launch per GPU with no
collective library call.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def shard(num_experts: int, world: int, rank: int) -> tuple[int, int]:
    """(expert_begin, expert_count) of `rank`: contiguous, equal shards."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not shard evenly over {world} ranks")
    n = num_experts // world
    return rank * n, n


# local(x_all [W*b, h] f32, residual_all [W*b, h] f32, out_all [W*b, h] f32) -> None
LocalFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], None]


class EPStep:
    """One expert-parallel MoE step for `tokens_per_rank` tokens on every rank.

    `local` writes this rank's partial sums for all gathered tokens into its
    third argument.  Call with this rank's token state `own` [b, h] (f32); the
    result [b, h] is the full MoE output (residual included) of those tokens.
    """

    def __init__(self, local: LocalFn, tokens_per_rank: int, hidden: int, *,
                 device: torch.device | str = "cpu", group=None):
        self.local = local
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        b, W = tokens_per_rank, self.world
        self.b = b
        self.x_all = torch.zeros((W * b, hidden), dtype=torch.float32, device=device)
        self.res_all = torch.zeros((W * b, hidden), dtype=torch.float32, device=device)
        self.part = torch.zeros((W * b, hidden), dtype=torch.float32, device=device)
        self.out = torch.zeros((b, hidden), dtype=torch.float32, device=device)

    def __call__(self, own: torch.Tensor) -> torch.Tensor:
        dist.all_gather_into_tensor(self.x_all, own, group=self.group)
        lo = self.rank * self.b
        self.res_all[lo:lo + self.b].copy_(own)  # other rows stay zero: residual enters once
        self.local(self.x_all, self.res_all, self.part)
        dist.reduce_scatter_tensor(self.out, self.part, group=self.group)
        return self.out


class EPFused:
    """Expert-parallel MoE steps in one kernel per layer over NVLink peer memory
    (m1moe_cuda_moe_layer_ep): no collective library on the data path.

    `blk` is this rank's MoEBlock, created with expert_begin/expert_count of its
    shard and max_batch >= world * tokens_per_rank.  The constructor exchanges
    the ranks' CUDA IPC handles over `group` (a host-side all_gather) and maps
    every peer's exchange region.  Call with this rank's tokens `own`
    [tokens_per_rank, h] for a layer; the result is those tokens' full output.
    """

    def __init__(self, blk, tokens_per_rank: int, *, group=None):
        import ctypes

        from . import _lib
        self.blk = blk
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.b = tokens_per_rank
        handle = (ctypes.c_uint8 * 64)()
        _lib.call("m1moe_cuda_ep_region", blk._ctx, self.world, tokens_per_rank,
                  ctypes.addressof(handle))
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        allh = (ctypes.c_uint8 * (64 * self.world)).from_buffer_copy(b"".join(handles))
        _lib.call("m1moe_cuda_ep_connect", blk._ctx, self.rank, ctypes.addressof(allh))

    def __call__(self, layer: int, own: torch.Tensor, residual: torch.Tensor | None = None, *,
                 out: torch.Tensor | None = None, idx: torch.Tensor | None = None,
                 w: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        from . import _lib
        from .expert_ffn import _stream, dtype_code
        if out is None:
            out = torch.empty((self.b, own.shape[-1]), dtype=torch.float32, device=own.device)
        res_ptr, res_dt = (0, 0) if residual is None else (residual.data_ptr(), dtype_code(residual.dtype))
        _lib.call("m1moe_cuda_moe_layer_ep", self.blk._ctx, layer, own.data_ptr(), dtype_code(own.dtype),
                  res_ptr, res_dt, out.data_ptr(), dtype_code(out.dtype),
                  idx.data_ptr() if idx is not None else 0, w.data_ptr() if w is not None else 0,
                  _stream(stream))
        return out
