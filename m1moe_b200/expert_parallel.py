"""Expert parallelism for the MoE block across ranks (one process per GPU).

Experts are independent, so a layer's E experts are split into contiguous
equal shards, one per rank (expert_begin/expert_count of m1moe_cuda_cfg).
Every rank owns `tokens_per_rank` decode tokens.  One step, per layer:

  1. all-gather every rank's tokens (the hidden state is small: h floats);
  2. each rank applies its local experts to every gathered token routed to
     them (m1moe_cuda_moe_layer with the shard's context), adding the
     residual only for the tokens it owns, so the residual enters once;
  3. reduce-scatter the partial sums back to the tokens' owners.

The collectives are torch.distributed calls (NCCL over NVLink on GPUs, gloo on
CPU for the tests); the buffers are preallocated so that a step can be
captured in a CUDA graph.  The local computation is a callable, which lets the
CPU tests substitute a reference computation for the CUDA kernel.
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
