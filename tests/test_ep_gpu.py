"""Expert parallelism over NVLink peer memory (m1moe_cuda_moe_layer_ep), 2 GPUs.

Two processes, one per GPU, each holding half of the experts; every rank owns
two tokens.  Each call gathers all ranks' tokens inside the kernel, applies
the local experts and returns each rank its own tokens' full output.  The
result must equal the single-context MoE block (all experts) on the same
tokens within the FFN tolerance, over several calls in a row (the exchange
slots alternate between calls), with the residual added once.  Skipped when
fewer than two GPUs are visible.
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
H, I, E, K, B = 512, 256, 8, 2, 2  # B tokens per rank


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from conftest import rel_max_err
    from m1moe_b200 import MoEBlock, synth
    from m1moe_b200.expert_parallel import EPFused, shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        layers = 2
        imgs = [synth.layer_image(40 + L, E, H, I, 64) for L in range(layers)]
        routers = [synth.router_weights(50 + L, E, H) for L in range(layers)]
        e0, ne = shard(E, world, rank)
        kw = dict(hidden_dim=H, intermediate_dim=I, num_experts=E, top_k=K, num_layers=layers,
                  norm_topk_prob=True, max_batch=world * B, device=rank)
        part = MoEBlock(expert_begin=e0, expert_count=ne, **kw)
        full = MoEBlock(**kw)
        for L in range(layers):
            for blk in (part, full):
                blk.load_expert_layer(L, imgs[L])
                blk.load_router(L, routers[L])
        ep = EPFused(part, B)
        errs = []
        for call in range(5):
            L = call % layers
            xall = torch.from_numpy(synth.bf16_to_f32(synth.hidden_states(60 + call, world * B, H))).cuda()
            own = xall[rank * B:(rank + 1) * B].contiguous()
            res = own * 0.5
            got = ep(L, own, res)
            ref = full.forward(L, own, res)
            torch.cuda.synchronize()
            part.synchronize()
            errs.append(rel_max_err(got.cpu().numpy(), ref.cpu().numpy()))
        q.put((rank, max(errs)))
        dist.barrier()
        part.close()
        full.close()
    except Exception as exc:  # reported to the parent
        q.put((rank, f"{type(exc).__name__}: {exc}"))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_expert_parallel_matches_single_context():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish")
    res = {}
    while not q.empty():
        r, v = q.get()
        res[r] = v
    assert sorted(res) == [0, 1], res
    for r, v in res.items():
        assert isinstance(v, float) and v < 1e-3, (r, v)
