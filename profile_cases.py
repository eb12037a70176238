"""Small, self-contained GPU cases for profiling the library's kernels.

    python profile_cases.py layer olmoe 1     # k_moe_layer, OLMoE shapes, batch 1
    python profile_cases.py layer mixtral 1   # k_moe_layer, Mixtral shapes
    python profile_cases.py matvec 1          # k_matvec4_ring over 2048 matrices
    python profile_cases.py prefill mixtral 512  # k_prefill_gemm, 512 tokens

Each case builds synthetic weights (m1moe_b200.synth), runs the kernel a few
times and exits 0; the device footprint stays at a few GB so that a profiler
capture of one launch ends quickly.  Intended for `ncu -k ... -s ... -c 1`.
"""
from __future__ import annotations

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


def main(argv: list[str]) -> None:
    if len(argv) >= 1 and argv[0] == "layer":
        layer_case(argv[1] if len(argv) > 1 else "olmoe", int(argv[2]) if len(argv) > 2 else 1)
    elif len(argv) >= 1 and argv[0] == "prefill":
        prefill_case(argv[1] if len(argv) > 1 else "mixtral", int(argv[2]) if len(argv) > 2 else 512)
    elif len(argv) >= 1 and argv[0] == "matvec":
        matvec_case(int(argv[1]) if len(argv) > 1 else 1)
    else:
        raise SystemExit(__doc__)


if __name__ == "__main__":
    main(sys.argv[1:])
