"""Tensor-core prefill of the MoE block (m1moe_cuda_moe_prefill) vs the CPU oracle.

The reference has no batched MoE path (it runs runLayer per token), so the
oracle is the same per-token restatement as for the decode kernel.  Bars as
in test_moe_gpu.py: expert indices equal wherever the K-th and (K+1)-th
scores differ by more than 1e-5, weights within 1e-5 relative, outputs
max |out - ref| <= 1e-3 * ||ref||_2, on at least 90 % of the tokens (a
token whose expert set differs from the oracle's at a near-tie is skipped).
The weights (q*s + b, one rounding), tokens and SwiGLU activations enter the
tensor cores as fp16 with fp32 accumulation; that error is inside the output
bar, which is checked here without the residual, on the expert sum alone.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_max_err
from m1moe_b200 import synth
from test_moe_gpu import GAP, TOL, _bf16_dev, _block, _check_routing

pytestmark = pytest.mark.gpu


def _prefill_case(oracle_lib, img, router, *, h, I, E, K, norm, T, seed, xdt=torch.bfloat16,
                  odt=torch.float32, with_res=False, shard=None):
    blk = _block([img], [router], h=h, I=I, E=E, K=K, norm=norm, max_batch=8,
                 **(shard or {}))
    xb = synth.hidden_states(seed + 1, T, h)
    rb = synth.hidden_states(seed + 2, T, h)
    xf, rf = synth.bf16_to_f32(xb), synth.bf16_to_f32(rb)
    out, idx, w = blk.prefill(0, _bf16_dev(xb, xdt), _bf16_dev(rb, torch.float32) if with_res else None,
                              out_dtype=odt, return_topk=True)
    out = out.float().cpu().numpy()
    idx, w = idx.cpu().numpy(), w.cpu().numpy()
    blk.synchronize()  # raises if a bounded device wait gave up
    blk.close()
    return out, idx, w, xf, rf


def _check_against_oracle(oracle_lib, img, router, out, idx, w, xf, rf, *, h, I, E, K, norm):
    ref, ridx, rw = oracle_lib.moe_layer(img, router, xf, rf, h=h, inter=I, E=E, K=K, gs=64,
                                         norm=norm, nthreads=8)
    _check_routing(idx, w, ridx, rw, xf, router, K)
    checked = 0
    for t in range(out.shape[0]):
        if set(idx[t].tolist()) == set(ridx[t].tolist()):
            assert rel_max_err(out[t], ref[t]) < TOL, t
            checked += 1
    assert checked >= 0.9 * out.shape[0]


@pytest.mark.parametrize("T", [1, 40, 300])
def test_prefill_on_reference_extracted_layer(golden, oracle_lib, T):
    """mixtral_tiny (h 128, I 128, 4 experts, top-2 renormalised); 300 tokens
    put more than one 256-token tile on some experts."""
    from golden.make_golden import router_weights
    g = golden("mixtral_tiny")
    L, E, h, I, gs, seed = (int(v) for v in g["meta"])
    router = router_weights(seed, L, E, h)[0]
    out, idx, w, xf, _ = _prefill_case(oracle_lib, g["layer_00"], router, h=h, I=I, E=E, K=2,
                                       norm=True, T=T, seed=7 * T)
    _check_against_oracle(oracle_lib, g["layer_00"], router, out, idx, w, xf, None, h=h, I=I, E=E,
                          K=2, norm=True)


def test_prefill_olmoe_shape(oracle_lib):
    """Config 1's layer shape (h 2048, 64 experts, top-8, I 1024) for 48 tokens."""
    h, I, E, K = 2048, 1024, 64, 8
    img = synth.layer_image_device(E, h, I, 64, seed=3, device="cuda").cpu().numpy()
    router = synth.router_weights(4, E, h)
    out, idx, w, xf, _ = _prefill_case(oracle_lib, img, router, h=h, I=I, E=E, K=K, norm=False,
                                       T=48, seed=5)
    _check_against_oracle(oracle_lib, img, router, out, idx, w, xf, None, h=h, I=I, E=E, K=K,
                          norm=False)


def test_prefill_mixtral_shape(oracle_lib):
    """Config 3's layer shape (h 4096, 8 experts, top-2 renormalised, I 14336)."""
    h, I, E, K = 4096, 14336, 8, 2
    img = synth.layer_image_device(E, h, I, 64, seed=13, device="cuda").cpu().numpy()
    router = synth.router_weights(14, E, h)
    out, idx, w, xf, _ = _prefill_case(oracle_lib, img, router, h=h, I=I, E=E, K=K, norm=True,
                                       T=24, seed=15)
    _check_against_oracle(oracle_lib, img, router, out, idx, w, xf, None, h=h, I=I, E=E, K=K,
                          norm=True)


def test_prefill_mixtral_512_tokens(oracle_lib):
    """The benchmarked prefill case (bench.py's `prefill`): Mixtral's layer shape
    over 512 tokens, so every expert's token tiles are full-sized (~128 tokens
    each).  A seeded sample of 48 tokens is checked against the oracle, with
    the same bars and the same >= 90 % floor."""
    h, I, E, K, T = 4096, 14336, 8, 2, 512
    img = synth.layer_image_device(E, h, I, 64, seed=23, device="cuda").cpu().numpy()
    router = synth.router_weights(24, E, h)
    out, idx, w, xf, _ = _prefill_case(oracle_lib, img, router, h=h, I=I, E=E, K=K, norm=True,
                                       T=T, seed=25)
    # every expert got a full-sized share of the 1024 (token, expert) pairs
    counts = np.bincount(idx.ravel(), minlength=E)
    assert counts.min() >= 32, counts
    pick = np.sort(np.random.default_rng(26).choice(T, size=48, replace=False))
    _check_against_oracle(oracle_lib, img, router, out[pick], idx[pick], w[pick], xf[pick], None,
                          h=h, I=I, E=E, K=K, norm=True)


@pytest.mark.parametrize("xdt,odt", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16)])
def test_prefill_dtypes_with_residual(golden, oracle_lib, xdt, odt):
    from golden.make_golden import router_weights
    g = golden("mixtral_tiny")
    L, E, h, I, gs, seed = (int(v) for v in g["meta"])
    router = router_weights(seed, L, E, h)[0]
    out, idx, w, xf, rf = _prefill_case(oracle_lib, g["layer_00"], router, h=h, I=I, E=E, K=2,
                                        norm=True, T=33, seed=3, xdt=xdt, odt=odt, with_res=True)
    ref, ridx, rw = oracle_lib.moe_layer(g["layer_00"], router, xf, rf, h=h, inter=I, E=E, K=2,
                                         gs=64, norm=True, nthreads=8)
    tol = TOL if odt == torch.float32 else 4e-3  # bf16 output rounding (<= 2^-9 max|y|)
    for t in range(33):
        if set(idx[t].tolist()) == set(ridx[t].tolist()):
            assert rel_max_err(out[t], ref[t]) < tol, t


def test_prefill_matches_decode_path(golden):
    """The tensor-core path and the decode kernel agree token by token."""
    from golden.make_golden import router_weights
    g = golden("mixtral_tiny")
    L, E, h, I, gs, seed = (int(v) for v in g["meta"])
    router = router_weights(seed, L, E, h)[0]
    blk = _block([g["layer_00"]], [router], h=h, I=I, E=E, K=2, norm=True, max_batch=8)
    x = _bf16_dev(synth.hidden_states(21, 16, h))
    r = _bf16_dev(synth.hidden_states(22, 16, h), torch.float32)
    pre, pidx, pw = blk.prefill(0, x, r, return_topk=True)
    dec = torch.cat([blk.forward(0, x[i:i + 8], r[i:i + 8]) for i in (0, 8)])
    didx = torch.cat([blk.route(0, x[i:i + 8])[0] for i in (0, 8)])
    blk.synchronize()
    assert torch.equal(pidx.cpu(), didx.cpu())
    assert rel_max_err(pre.cpu().numpy() - r.cpu().numpy(), dec.cpu().numpy() - r.cpu().numpy()) < TOL
    blk.close()


def test_prefill_expert_shards_sum_to_full(golden):
    """Expert-parallel shards: the partial outputs (residual in one shard) sum
    to the single-context output."""
    from golden.make_golden import router_weights
    g = golden("mixtral_tiny")
    L, E, h, I, gs, seed = (int(v) for v in g["meta"])
    router = router_weights(seed, L, E, h)[0]
    x = _bf16_dev(synth.hidden_states(31, 50, h))
    r = _bf16_dev(synth.hidden_states(32, 50, h), torch.float32)
    full = _block([g["layer_00"]], [router], h=h, I=I, E=E, K=2, norm=True)
    s0 = _block([g["layer_00"]], [router], h=h, I=I, E=E, K=2, norm=True, expert_begin=0,
                expert_count=2)
    s1 = _block([g["layer_00"]], [router], h=h, I=I, E=E, K=2, norm=True, expert_begin=2,
                expert_count=2)
    y = full.prefill(0, x, r).cpu().numpy()
    y0 = s0.prefill(0, x, r).cpu().numpy()
    y1 = s1.prefill(0, x, None).cpu().numpy()
    for b in (full, s0, s1):
        b.synchronize()
        b.close()
    assert rel_max_err(y0 + y1, y) < 1e-5


def test_prefill_unsupported_shape_is_an_error(golden):
    """intermediate_dim 64 (olmoe_tiny) is not a multiple of the 128-row MMA."""
    from golden.make_golden import router_weights
    from m1moe_b200 import M1MoECudaError
    g = golden("olmoe_tiny")
    L, E, h, I, gs, seed = (int(v) for v in g["meta"])
    blk = _block([g["layer_00"]], [router_weights(seed, L, E, h)[0]], h=h, I=I, E=E, K=2,
                 norm=False)
    with pytest.raises(M1MoECudaError, match="UNSUPPORTED"):
        blk.prefill(0, torch.zeros((4, h), device="cuda"))
    blk.close()


def test_prefill_large_magnitudes_and_range_error(golden, oracle_lib):
    """Tokens enter the tensor cores as fp16.  Inputs 100x larger than the
    synthetic N(0,1) (within fp16 range, and so are the SwiGLU activations
    here) keep the parity bar, fp16's relative precision being scale-free.
    A token value beyond fp16's range (1e5 > 65504) is not turned into an
    infinity: the call reports it (M1MOE_ERR_DEVICE from synchronize, the
    error word's range bit), and the context works again afterwards."""
    from golden.make_golden import router_weights
    from m1moe_b200._lib import M1MoECudaError
    g = golden("mixtral_tiny")
    L, E, h, I, gs, seed = (int(v) for v in g["meta"])
    router = router_weights(seed, L, E, h)[0]
    img = g["layer_00"]
    blk = _block([img], [router], h=h, I=I, E=E, K=2, norm=True, max_batch=8)
    T = 40
    xf = (synth.bf16_to_f32(synth.hidden_states(91, T, h)) * 100.0).astype(np.float32)
    out, idx, w = blk.prefill(0, torch.from_numpy(xf).cuda(), return_topk=True)
    blk.synchronize()
    _check_against_oracle(oracle_lib, img, router, out.cpu().numpy(), idx.cpu().numpy(),
                          w.cpu().numpy(), xf, None, h=h, I=I, E=E, K=2, norm=True)
    bad = xf.copy()
    bad[3, 17] = 1.0e5
    blk.prefill(0, torch.from_numpy(bad).cuda())
    with pytest.raises(M1MoECudaError) as ei:
        blk.synchronize()
    assert "0x4" in str(ei.value) or "range" in str(ei.value)
    out2, idx2, w2 = blk.prefill(0, torch.from_numpy(xf).cuda(), return_topk=True)
    blk.synchronize()
    assert torch.equal(idx2, idx) and rel_max_err(out2.cpu().numpy(), out.cpu().numpy()) < 1e-6
    blk.close()
