"""The allocation-free router top-K against the context-based one and the oracle (GPU).

m1moe_cuda_router_topk_noalloc serves callers that may not call cudaMalloc:
runtimes that hand out all GPU memory themselves, plugins that must not grow
the process's device footprint, code running where allocation is not allowed.
Its scratch is a fixed array inside the library, so it takes the router and x
from the caller instead of a context.  This file checks, over the C ABI, that
two calls in a row give bit-identical experts, weights and scores to
m1moe_cuda_router_topk (both run the same kernel variant for a batch), that
those agree with the CPU oracle (experts identical where the logit gaps
exceed 1e-5, weights within 1e-5 relative), that a NULL status word and sizes
beyond the fixed scratch are refused, and that a hidden size far beyond the
model shapes still routes.  It is named to be collected last.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from m1moe_b200 import MoEBlock, _lib, synth

pytestmark = pytest.mark.gpu
W_TOL = 1e-5  # relative, as the routing checks in test_moe_gpu.py
GAP = 1e-5


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


def _check_vs_oracle(idx, w, scores, router, x_f32, K, norm, tol=W_TOL):
    """Experts equal to the oracle's wherever the K-th and (K+1)-th scores are
    more than GAP apart (and in order where neighbours are), weights and
    scores within `tol` relative."""
    import oracle
    oracle.build()
    checked = 0
    for t in range(idx.shape[0]):
        ref_s = oracle.router_scores(router, x_f32[t])
        ref_i, ref_w = oracle.select_topk(ref_s, K, norm)
        assert np.all(np.abs(scores[t] - ref_s) <= tol * np.abs(ref_s) + 1e-7), t
        srt = np.sort(ref_s)[::-1]
        if K < len(ref_s) and srt[K - 1] - srt[K] <= GAP:
            continue
        checked += 1
        assert set(idx[t].tolist()) == set(ref_i.tolist()), t
        for k in range(K):
            if k == 0 or srt[k - 1] - srt[k] > GAP:
                assert idx[t][k] == ref_i[k], (t, k)
        wd, rd = dict(zip(idx[t].tolist(), w[t].tolist())), dict(zip(ref_i.tolist(), ref_w.tolist()))
        assert all(abs(wd[e] - rd[e]) <= tol * abs(rd[e]) + 1e-7 for e in rd), t
    assert checked >= max(1, (9 * idx.shape[0]) // 10), checked


# (E, K, h, norm, B): the slot-path batches (3, 8), the row-group batches 1 and
# 2 at h 2048, and batch 2 at h 4096, which takes the slot path in both entry points
@pytest.mark.parametrize("E,K,h,norm,B", [(64, 8, 2048, False, 3), (8, 2, 4096, True, 8),
                                          (64, 8, 2048, False, 1), (64, 8, 2048, False, 2),
                                          (8, 2, 4096, True, 2)])
def test_noalloc_router_matches_context_router(E, K, h, norm, B):
    router = synth.router_weights(31 + E, E, h)
    blk = MoEBlock(hidden_dim=h, intermediate_dim=64, num_experts=E, top_k=K,
                   norm_topk_prob=norm, max_batch=8)
    blk.load_router(0, router)
    router_dev = _dev_bf16(router)
    for call in range(2):  # two calls in a row share (and reuse) the scratch
        xb = synth.hidden_states(100 + 10 * call + E + B, B, h)
        x = _dev_bf16(xb).view(torch.bfloat16) if call == 0 else \
            torch.from_numpy(synth.bf16_to_f32(xb)).cuda()
        ref_idx, ref_w, ref_s = (t.cpu().numpy() for t in blk.route(0, x))
        idx, w, s = _noalloc(router_dev, E, h, K, norm, x, B)
        assert np.array_equal(idx, ref_idx), call
        assert np.array_equal(w, ref_w), call
        assert np.array_equal(s, ref_s), call
        _check_vs_oracle(idx, w, s, router, synth.bf16_to_f32(xb), K, norm)
    blk.synchronize()
    blk.close()


def test_noalloc_router_wide_hidden():
    """Routing stages nothing that grows with the hidden size, so a 32768-wide
    router (beyond any model shape here) routes as well.  A logit here sums 16x
    more terms than at h 2048, in another order than the oracle's, so scores
    and weights are held to 1e-4 relative (experts still exactly)."""
    E, K, h, B = 16, 4, 32768, 4
    router = synth.router_weights(77, E, h)
    xb = synth.hidden_states(78, B, h)
    x = torch.from_numpy(synth.bf16_to_f32(xb)).cuda()
    idx, w, s = _noalloc(_dev_bf16(router), E, h, K, True, x, B)
    _check_vs_oracle(idx, w, s, router, synth.bf16_to_f32(xb), K, True, tol=1e-4)


def test_noalloc_router_rejects_null_status_and_sizes_beyond_its_scratch():
    h = 256
    router_dev = _dev_bf16(synth.router_weights(5, 8, h))
    x = torch.zeros((9, h), dtype=torch.float32, device="cuda")
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.M1MoECudaError, match="batch 9"):
        _lib.call("m1moe_cuda_router_topk_noalloc", router_dev.data_ptr(), 8, h, 2, 0,
                  x.data_ptr(), _lib.DTYPE_F32, 9, 0, 0, 0, status.data_ptr(), 0)
    with pytest.raises(_lib.M1MoECudaError, match="num_experts 300"):
        _lib.call("m1moe_cuda_router_topk_noalloc", router_dev.data_ptr(), 300, h, 2, 0,
                  x.data_ptr(), _lib.DTYPE_F32, 1, 0, 0, 0, status.data_ptr(), 0)
    with pytest.raises(_lib.M1MoECudaError, match="d_status is NULL"):
        _lib.call("m1moe_cuda_router_topk_noalloc", router_dev.data_ptr(), 8, h, 2, 0,
                  x.data_ptr(), _lib.DTYPE_F32, 1, 0, 0, 0, 0, 0)
