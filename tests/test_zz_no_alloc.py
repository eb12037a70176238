"""The allocation-free router top-K against the context-based one (GPU).

m1moe_cuda_router_topk_noalloc serves callers that may not call cudaMalloc:
runtimes that hand out all GPU memory themselves, plugins that must not grow
the process's device footprint, code running where allocation is not allowed.
Its scratch is a fixed array inside the library, so it takes the router and x
from the caller instead of a context.  This file checks, over the C ABI, that
two calls in a row give the same experts, weights and scores as
m1moe_cuda_router_topk (experts identical, weights and scores within the
routing tolerance of the other GPU tests), and that sizes beyond the fixed
scratch are refused.  It is named to be collected last.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from m1moe_b200 import MoEBlock, _lib, synth

pytestmark = pytest.mark.gpu
W_TOL = 1e-5  # relative, as the routing checks in test_moe_gpu.py


def _dev_bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()


def _noalloc(router_dev, E, h, K, norm, x, B):
    idx = torch.full((B, K), -1, dtype=torch.int32, device="cuda")
    w = torch.zeros((B, K), dtype=torch.float32, device="cuda")
    scores = torch.zeros((B, E), dtype=torch.float32, device="cuda")
    status = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    xdt = _lib.DTYPE_BF16 if x.dtype == torch.bfloat16 else _lib.DTYPE_F32
    _lib.call("m1moe_cuda_router_topk_noalloc", router_dev.data_ptr(), E, h, K, int(norm),
              x.data_ptr(), xdt, B, idx.data_ptr(), w.data_ptr(), scores.data_ptr(),
              status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return idx.cpu().numpy(), w.cpu().numpy(), scores.cpu().numpy()


@pytest.mark.parametrize("E,K,h,norm,B", [(64, 8, 2048, False, 3), (8, 2, 4096, True, 8)])
def test_noalloc_router_matches_context_router(E, K, h, norm, B):
    router = synth.router_weights(31 + E, E, h)
    blk = MoEBlock(hidden_dim=h, intermediate_dim=64, num_experts=E, top_k=K,
                   norm_topk_prob=norm, max_batch=8)
    blk.load_router(0, router)
    router_dev = _dev_bf16(router)
    for call in range(2):  # two calls in a row share (and reuse) the scratch
        xb = synth.hidden_states(100 + 10 * call + E, B, h)
        x = _dev_bf16(xb).view(torch.bfloat16) if call == 0 else \
            torch.from_numpy(synth.bf16_to_f32(xb)).cuda()
        ref_idx, ref_w, ref_s = (t.cpu().numpy() for t in blk.route(0, x))
        idx, w, s = _noalloc(router_dev, E, h, K, norm, x, B)
        assert np.array_equal(idx, ref_idx), call
        assert np.all(np.abs(w - ref_w) <= W_TOL * np.abs(ref_w) + 1e-7), call
        assert np.all(np.abs(s - ref_s) <= W_TOL * np.abs(ref_s) + 1e-7), call
    blk.synchronize()
    blk.close()


def test_noalloc_router_rejects_sizes_beyond_its_scratch():
    h = 256
    router_dev = _dev_bf16(synth.router_weights(5, 8, h))
    x = torch.zeros((9, h), dtype=torch.float32, device="cuda")
    with pytest.raises(_lib.M1MoECudaError, match="batch 9"):
        _lib.call("m1moe_cuda_router_topk_noalloc", router_dev.data_ptr(), 8, h, 2, 0,
                  x.data_ptr(), _lib.DTYPE_F32, 9, 0, 0, 0, 0, 0)
    with pytest.raises(_lib.M1MoECudaError, match="num_experts 300"):
        _lib.call("m1moe_cuda_router_topk_noalloc", router_dev.data_ptr(), 300, h, 2, 0,
                  x.data_ptr(), _lib.DTYPE_F32, 1, 0, 0, 0, 0, 0)
