"""Small, self-contained GPU cases for profiling the library's kernels.

    python profile_cases.py layer olmoe 1     # k_moe_layer, OLMoE shapes, batch 1
    python profile_cases.py layer mixtral 1   # k_moe_layer, Mixtral shapes
    python profile_cases.py matvec 1          # k_matvec4_ring over 2048 matrices
    python profile_cases.py prefill mixtral 512  # k_prefill_gemm, 512 tokens
    python profile_cases.py decode olmoe 1    # whole decode steps, config-2 shapes, 2 layers
    python profile_cases.py prefill_step olmoe 512   # token-parallel prompt prefill, 2 layers
    python profile_cases.py trace olmoe 1     # k_moe_layer phase trace summary (no profiler)
    torchrun --nproc-per-node 2 profile_cases.py trace_ep olmoe   # the expert-parallel kernel's trace

Each case builds synthetic weights (m1moe_b200.synth), runs the kernel a few
times and exits 0; the device footprint stays at a few GB so that a profiler
capture of one launch ends quickly.  Intended for `ncu -k ... -s ... -c 1`.
"""
from __future__ import annotations

import os
import sys


def layer_case(workload: str, batch: int) -> None:
    import torch

    from m1moe_b200 import MoEBlock, _lib, synth

    if workload == "olmoe":
        h, inter, e, k, norm, layers = 2048, 1024, 64, 8, False, 4
    elif workload == "mixtral":
        h, inter, e, k, norm, layers = 4096, 14336, 8, 2, True, 2
    else:
        raise SystemExit(f"unknown workload {workload!r}")
    torch.cuda.set_device(0)
    blk = MoEBlock(hidden_dim=h, intermediate_dim=inter, num_experts=e, top_k=k,
                   num_layers=layers, max_batch=8, norm_topk_prob=norm)
    for layer in range(layers):
        img = synth.layer_image_device(e, h, inter, 64, seed=layer, device="cuda")
        blk.load_expert_layer(layer, img)
        del img
        blk.load_router(layer, synth.router_weights(100 + layer, e, h))
    x = torch.randn(batch, h, device="cuda")
    out = torch.empty(batch, h, device="cuda")
    idx = torch.zeros(batch, k, dtype=torch.int32, device="cuda")
    for _ in range(2):
        for layer in range(layers):
            _lib.call("m1moe_cuda_moe_layer", blk._ctx, layer, x.data_ptr(), 0, x.data_ptr(), 0,
                      out.data_ptr(), 0, batch, idx.data_ptr(), 0, 0)
    torch.cuda.synchronize()
    blk.synchronize()
    blk.close()
    print("ok")


def matvec_case(batch: int) -> None:
    import torch

    from m1moe_b200 import _lib

    out, inn, gs, nm = 1024, 2048, 64, 2048  # 2048 OLMoE gate matrices, 2.4 GB
    wbytes, sbytes = out * inn // 2, out * (inn // gs) * 2
    stride = wbytes + 2 * sbytes
    torch.cuda.set_device(0)
    buf = torch.randint(0, 2**31 - 1, (nm * stride // 4,), dtype=torch.int32, device="cuda")
    x = torch.randn(8, inn, device="cuda").to(torch.bfloat16)
    y = torch.empty(nm * 8 * out, dtype=torch.bfloat16, device="cuda")
    base = buf.data_ptr()
    for _ in range(3):
        _lib.call("m1moe_cuda_matvec4_strided", base, base + wbytes, base + wbytes + sbytes, stride,
                  nm, x.data_ptr(), 1, y.data_ptr(), 1, out, inn, gs, batch, 0)
    torch.cuda.synchronize()
    print("ok")


def prefill_case(workload: str, tokens: int) -> None:
    import torch

    from m1moe_b200 import MoEBlock, synth

    if workload == "olmoe":
        h, inter, e, k, norm = 2048, 1024, 64, 8, False
    elif workload == "mixtral":
        h, inter, e, k, norm = 4096, 14336, 8, 2, True
    else:
        raise SystemExit(f"unknown workload {workload!r}")
    torch.cuda.set_device(0)
    blk = MoEBlock(hidden_dim=h, intermediate_dim=inter, num_experts=e, top_k=k, num_layers=1,
                   max_batch=8, norm_topk_prob=norm)
    img = synth.layer_image_device(e, h, inter, 64, seed=0, device="cuda")
    blk.load_expert_layer(0, img)
    del img
    blk.load_router(0, synth.router_weights(100, e, h))
    x = torch.randn(tokens, h, device="cuda").to(torch.bfloat16)
    out = torch.empty(tokens, h, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        blk.prefill(0, x, None, out=out)
    torch.cuda.synchronize()
    blk.synchronize()
    blk.close()
    print("ok")


def decode_case(workload: str, batch: int, layers: int = 2, steps: int = 4) -> None:
    """Whole decode steps (m1moe_cuda_decode_step) at config 2 or 4 shapes with
    `layers` layers, the KV cache at the full context: for a launch list of
    every kernel of a step."""
    import torch

    from m1moe_b200 import MoEBlock, synth
    from m1moe_b200.dense import DenseModel

    if workload == "olmoe":
        h, nh, nkv, V, qk, th, E, K, I, norm, ctx = 2048, 16, 16, 50304, True, 1e4, 64, 8, 1024, False, 2048
    elif workload == "mixtral":
        h, nh, nkv, V, qk, th, E, K, I, norm, ctx = 4096, 32, 8, 32000, False, 1e6, 8, 2, 14336, True, 4096
    else:
        raise SystemExit(f"unknown workload {workload!r}")
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    dm = DenseModel(hidden_dim=h, num_heads=nh, num_kv_heads=nkv, num_layers=layers, vocab_size=V,
                    qk_norm=qk, rope_theta=th, max_batch=batch, max_seq=ctx + steps + 1)
    dm.load_all(synth.dense_weights_device(1, h=h, nh=nh, nkv=nkv, hd=128, layers=layers, vocab=V,
                                           qk_norm=qk, device=dev))
    blk = MoEBlock(hidden_dim=h, intermediate_dim=I, num_experts=E, top_k=K, num_layers=layers,
                   max_batch=batch, norm_topk_prob=norm)
    for layer in range(layers):
        img = synth.layer_image_device(E, h, I, 64, seed=layer, device=dev)
        blk.load_expert_layer(layer, img)
        del img
        blk.load_router(layer, synth.router_weights(100 + layer, E, h))
        k, v = dm.kv_cache(layer)
        k.normal_()
        v.normal_()
    dm.set_position(ctx)
    tok = torch.arange(batch, dtype=torch.int32, device=dev)
    for _ in range(steps):
        tok = dm.step(blk, tok).clone()
    torch.cuda.synchronize()
    dm.synchronize()
    blk.synchronize()
    dm.close()
    blk.close()
    print("ok")


def prefill_step_case(workload: str, tokens: int, layers: int = 2) -> None:
    """A prompt of `tokens` tokens through m1moe_cuda_prefill_step (token-parallel
    dense prefill) at config 2 or 4 shapes with `layers` layers, twice: for a
    launch list of every kernel of the call."""
    import torch

    from m1moe_b200 import MoEBlock, synth
    from m1moe_b200.dense import DenseModel

    if workload == "olmoe":
        h, nh, nkv, V, qk, th, E, K, I, norm = 2048, 16, 16, 50304, True, 1e4, 64, 8, 1024, False
    else:
        h, nh, nkv, V, qk, th, E, K, I, norm = 4096, 32, 8, 32000, False, 1e6, 8, 2, 14336, True
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    dm = DenseModel(hidden_dim=h, num_heads=nh, num_kv_heads=nkv, num_layers=layers, vocab_size=V,
                    qk_norm=qk, rope_theta=th, max_batch=1, max_seq=tokens + 1)
    dm.load_all(synth.dense_weights_device(1, h=h, nh=nh, nkv=nkv, hd=128, layers=layers, vocab=V,
                                           qk_norm=qk, device=dev))
    blk = MoEBlock(hidden_dim=h, intermediate_dim=I, num_experts=E, top_k=K, num_layers=layers,
                   max_batch=8, norm_topk_prob=norm)
    for layer in range(layers):
        img = synth.layer_image_device(E, h, I, 64, seed=layer, device=dev)
        blk.load_expert_layer(layer, img)
        del img
        blk.load_router(layer, synth.router_weights(100 + layer, E, h))
    prompt = torch.randint(0, V, (tokens,), dtype=torch.int32, device=dev)
    for _ in range(2):
        dm.set_position(0)
        dm.prefill(blk, prompt)
    torch.cuda.synchronize()
    dm.synchronize()
    blk.synchronize()
    dm.close()
    blk.close()
    print("ok")


def trace_case(workload: str, batch: int, layers: int = 4, calls: int = 20) -> None:
    """Phase trace of k_moe_layer (m1moe_cuda_set_trace) over `calls` calls of
    `layers` distinct layers, launched back to back; prints, per phase event,
    the median over CTAs and calls of its time after the call's first CTA
    start (us), and the spread of the end event."""
    import numpy as np
    import torch

    from m1moe_b200 import MoEBlock, _lib, synth

    if workload == "olmoe":
        h, inter, e, k, norm = 2048, 1024, 64, 8, False
    elif workload == "mixtral":
        h, inter, e, k, norm = 4096, 14336, 8, 2, True
    else:
        raise SystemExit(f"unknown workload {workload!r}")
    torch.cuda.set_device(0)
    blk = MoEBlock(hidden_dim=h, intermediate_dim=inter, num_experts=e, top_k=k,
                   num_layers=layers, max_batch=8, norm_topk_prob=norm)
    for layer in range(layers):
        img = synth.layer_image_device(e, h, inter, 64, seed=layer, device="cuda")
        blk.load_expert_layer(layer, img)
        del img
        blk.load_router(layer, synth.router_weights(100 + layer, e, h))
    x = torch.randn(batch, h, device="cuda")
    out = torch.empty(batch, h, device="cuda")
    trace = torch.zeros((160, 32), dtype=torch.int64, device="cuda")
    names = dict(TRACE_NAMES)  # events a call did not record are left out
    rows = {ev: [] for ev in names}
    spread = {ev: [] for ev in names}
    tiles = []
    for it in range(calls + 3):
        for layer in range(layers):
            rec = it >= 3 and layer == layers - 1
            _lib.call("m1moe_cuda_set_trace", blk._ctx, trace.data_ptr() if rec else 0)
            _lib.call("m1moe_cuda_moe_layer", blk._ctx, layer, x.data_ptr(), 0, x.data_ptr(), 0,
                      out.data_ptr(), 0, batch, 0, 0, 0)
            if rec:
                torch.cuda.synchronize()
                t = trace.cpu().numpy().astype(np.int64)
                G = min(148, 160)
                ns0, ns1 = t[:G, 20], t[:G, 21]
                c0, c1 = t[:G, 0], t[:G, 10]
                # cycles -> ns per CTA from its own start/end pair
                scale = (ns1 - ns0) / np.maximum(c1 - c0, 1)
                t0 = ns0.min()
                for ev in names:
                    vals = ns0 + (t[:G, ev] - c0) * scale - t0
                    ok = t[:G, ev] != 0
                    if ok.any():
                        rows[ev].append(np.median(vals[ok]) / 1e3)
                        spread[ev].append((np.percentile(vals[ok], 10) / 1e3, np.percentile(vals[ok], 90) / 1e3))
                tiles.append(t[:G, 15].copy())
                trace.zero_()
    _lib.call("m1moe_cuda_set_trace", blk._ctx, 0)
    blk.synchronize()
    print(f"k_moe_layer phase trace: {workload}, batch {batch}, median over CTAs and {calls} calls")
    print("| event | us after the first CTA's start (median CTA) | 10th / 90th percentile CTA |")
    print("|---|---|---|")
    order = sorted((float(np.median(v)), ev) for ev, v in rows.items() if v)
    for med, ev in order:
        lo = float(np.median([a for a, _ in spread[ev]]))
        hi = float(np.median([b for _, b in spread[ev]]))
        print(f"| {names[ev]} | {med:.2f} | {lo:.2f} / {hi:.2f} |")
    tt = np.concatenate(tiles)
    ntg, ntd = tt & 0xFFFFFFFF, tt >> 32
    print(f"\ntiles per CTA: gate/up {np.median(ntg):.0f} (max {ntg.max()}), down {np.median(ntd):.0f} (max {ntd.max()})")
    blk.close()


TRACE_NAMES = {0: "start", 1: "out rows init", 2: "logits published", 12: "all logits seen",
               13: "ranks counted", 3: "top-K ranked", 19: "producer saw routing",
               16: "geometry", 11: "first tile issued", 4: "consumers released",
               5: "first tile landed", 9: "all tiles issued", 17: "gate/up done",
               6: "activations quantised", 18: "first down item", 22: "first down tile",
               23: "last down tile", 7: "epochs seen", 8: "down items done", 10: "end",
               24: "ep: own tokens pushed", 25: "ep: every rank's tokens seen",
               26: "ep: every CTA's sums seen", 27: "ep: slices sent", 28: "ep: peers' slices seen"}


def trace_ep_case(workload: str, layers: int = 2, calls: int = 20) -> None:
    """Phase trace of the expert-parallel layer kernel (m1moe_cuda_moe_layer_ep)
    on every rank of a torchrun job, one token per rank; rank 0 prints, per
    event, the median over CTAs and calls of its time after the call's first
    CTA start on that rank (us), and each rank's median call span."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from m1moe_b200 import MoEBlock, _lib, synth
    from m1moe_b200.expert_parallel import EPFused, shard

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo")
    if workload == "olmoe":
        h, inter, e, k, norm = 2048, 1024, 64, 8, False
    else:
        h, inter, e, k, norm = 4096, 14336, 8, 2, True
    e0, ne = shard(e, world, rank)
    blk = MoEBlock(hidden_dim=h, intermediate_dim=inter, num_experts=e, top_k=k, num_layers=layers,
                   max_batch=8, norm_topk_prob=norm, device=rank, expert_begin=e0, expert_count=ne)
    for layer in range(layers):
        img = synth.layer_image_device(e, h, inter, 64, seed=layer, device="cuda")
        blk.load_expert_layer(layer, img)
        del img
        blk.load_router(layer, synth.router_weights(100 + layer, e, h))
    ep = EPFused(blk, 1)
    x = torch.randn(1, h, device="cuda")
    trace = torch.zeros((160, 32), dtype=torch.int64, device="cuda")
    rows = {ev: [] for ev in TRACE_NAMES}
    spans = []
    for it in range(calls + 3):
        for layer in range(layers):
            rec = it >= 3 and layer == layers - 1
            _lib.call("m1moe_cuda_set_trace", blk._ctx, trace.data_ptr() if rec else 0)
            ep(layer, x, x, out=x)
            if rec:
                torch.cuda.synchronize()
                t = trace.cpu().numpy().astype(np.int64)
                G = 148
                ns0, ns1 = t[:G, 20], t[:G, 21]
                c0, c1 = t[:G, 0], t[:G, 10]
                scale = (ns1 - ns0) / np.maximum(c1 - c0, 1)
                t0 = ns0.min()
                for ev in TRACE_NAMES:
                    vals = ns0 + (t[:G, ev] - c0) * scale - t0
                    ok = t[:G, ev] != 0
                    if ok.any():
                        rows[ev].append(np.median(vals[ok]) / 1e3)
                spans.append((ns1.max() - t0) / 1e3)
                trace.zero_()
    _lib.call("m1moe_cuda_set_trace", blk._ctx, 0)
    blk.synchronize()
    med = {ev: float(np.median(v)) for ev, v in rows.items() if v}
    allspans = [None] * world
    dist.all_gather_object(allspans, float(np.median(spans)))
    if rank == 0:
        print(f"expert-parallel k_moe_layer trace: {workload}, {world} ranks, 1 token per rank, "
              f"rank 0, median over CTAs and {calls} calls")
        print("| event | us after the call's first CTA start |")
        print("|---|---|")
        for ev in sorted(med, key=med.get):
            print(f"| {TRACE_NAMES[ev]} | {med[ev]:.2f} |")
        print("\nmedian call span (first CTA start to last CTA end) per rank, us: " +
              ", ".join(f"{v:.1f}" for v in allspans))
    dist.barrier()
    blk.close()
    dist.destroy_process_group()


def main(argv: list[str]) -> None:
    if len(argv) >= 1 and argv[0] == "layer":
        layer_case(argv[1] if len(argv) > 1 else "olmoe", int(argv[2]) if len(argv) > 2 else 1)
    elif len(argv) >= 1 and argv[0] == "prefill":
        prefill_case(argv[1] if len(argv) > 1 else "mixtral", int(argv[2]) if len(argv) > 2 else 512)
    elif len(argv) >= 1 and argv[0] == "decode":
        decode_case(argv[1] if len(argv) > 1 else "olmoe", int(argv[2]) if len(argv) > 2 else 1)
    elif len(argv) >= 1 and argv[0] == "prefill_step":
        prefill_step_case(argv[1] if len(argv) > 1 else "olmoe", int(argv[2]) if len(argv) > 2 else 512)
    elif len(argv) >= 1 and argv[0] == "trace_ep":
        trace_ep_case(argv[1] if len(argv) > 1 else "olmoe")
    elif len(argv) >= 1 and argv[0] == "trace":
        trace_case(argv[1] if len(argv) > 1 else "olmoe", int(argv[2]) if len(argv) > 2 else 1)
    elif len(argv) >= 1 and argv[0] == "matvec":
        matvec_case(int(argv[1]) if len(argv) > 1 else 1)
    else:
        raise SystemExit(__doc__)


if __name__ == "__main__":
    main(sys.argv[1:])
