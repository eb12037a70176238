"""Expert-parallel step on CPU: two gloo ranks, the oracle standing in for the
CUDA kernel (each rank applies only its shard of the experts).

Checks that gather -> local shard -> reduce-scatter reproduces the single-rank
MoE output for every rank's tokens (residual added once), and that a rank that
never joins makes its peer's collective end with an error instead of a hang
(short process-group timeout), as the multi-GPU bench relies on.
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

H, I, E, K, GS, B = 128, 64, 4, 2, 64, 2  # B tokens per rank


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model():
    from m1moe_b200 import synth
    table = synth.layer_image(77, E, H, I, GS)
    router = synth.router_weights(78, E, H)
    return table, router


def _oracle_partial(table, router, x_all, res_all, e0, ne, norm):
    """This shard's partial sums: residual rows + sum over local routed experts."""
    import oracle
    eb = oracle.expert_bytes(H, I, GS)
    out = res_all.copy()
    for t in range(x_all.shape[0]):
        idx, w = oracle.select_topk(oracle.router_scores(router, x_all[t]), K, norm)
        for k in range(K):
            e = int(idx[k])
            if e0 <= e < e0 + ne:
                y = oracle.expert_forward(table[e * eb:(e + 1) * eb], x_all[t], H, I, GS)
                out[t] += np.float32(w[k]) * y
    return out


def _worker(rank, world, port, norm, mode, q):
    import torch.distributed as dist

    from m1moe_b200.expert_parallel import EPStep, shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=5))
        if mode == "drop" and rank == 1:
            q.put((rank, "left"))
            return  # never takes part in the step
        table, router = _model()
        e0, ne = shard(E, world, rank)

        def local(x_all, res_all, out_all):
            out_all.copy_(torch.from_numpy(_oracle_partial(
                table, router, x_all.numpy(), res_all.numpy(), e0, ne, norm)))

        from m1moe_b200 import synth
        own = torch.from_numpy(synth.bf16_to_f32(synth.hidden_states(90 + rank, B, H)))
        step = EPStep(local, B, H)
        try:
            got = step(own).numpy().copy()
        except Exception as exc:  # the peer never joined
            q.put((rank, f"error: {type(exc).__name__}"))
            return
        full = _oracle_partial(table, router, own.numpy(), own.numpy(), 0, E, norm)
        q.put((rank, float(np.max(np.abs(got - full)) / np.max(np.abs(full)))))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(mode, norm=False, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, norm, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    out = {}
    while not q.empty():
        r, v = q.get()
        out[r] = v
    return out


@pytest.mark.parametrize("norm", [False, True])
def test_expert_parallel_step_matches_single_rank(norm):
    res = _run("full", norm)
    assert sorted(res) == [0, 1], res
    for r, err in res.items():
        assert isinstance(err, float) and err < 1e-5, (r, err)


def test_rank_that_never_joins_ends_peer_with_error():
    res = _run("drop")
    assert res.get(1) == "left"
    assert isinstance(res.get(0), str) and res[0].startswith("error"), res


def test_shard_ranges():
    from m1moe_b200.expert_parallel import shard
    assert [shard(8, 4, r) for r in range(4)] == [(0, 2), (2, 2), (4, 2), (6, 2)]
    assert shard(64, 8, 7) == (56, 8)
    with pytest.raises(ValueError):
        shard(8, 3, 0)
