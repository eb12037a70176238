"""Failure paths on the GPU, made without faulting it (GPU).

Every device-side wait in the library is bounded: a wait that runs out sets
the context's error word and the kernel unwinds, so the context's next
synchronize reports M1MOE_ERR_DEVICE and nothing hangs.  These tests make
such waits run out on purpose with flags that nothing sets, and check the
other error words the kernels raise on bad inputs:

  * an expert-parallel rank whose peer never calls: two contexts on one GPU
    are joined as ranks 0 and 1 (m1moe_cuda_ep_connect_local) and only rank
    0 is called, with a short wait limit -- its kernel waits for rank 1's
    tokens, gives up, and the call reports M1MOE_ERR_DEVICE within seconds;
    contexts made afterwards work (only one kernel runs at a time: nothing
    here waits on another running kernel);
  * the dense step given a token id beyond the vocabulary, or run past the
    end of its KV cache, reports M1MOE_ERR_DEVICE (the id is read as 0, the
    position as 0, nothing outside the buffers is touched);
  * the tensor-core prefill given a value beyond the fp16 range of its
    operands reports M1MOE_ERR_DEVICE instead of returning infinities.
"""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

from conftest import rel_max_err
from m1moe_b200 import M1MoECudaError, MoEBlock, _lib, synth
from m1moe_b200.dense import DenseModel

pytestmark = pytest.mark.gpu
H, I, E, K = 512, 256, 8, 2


def _block(**kw):
    blk = MoEBlock(hidden_dim=H, intermediate_dim=I, num_experts=E, top_k=K, num_layers=1,
                   norm_topk_prob=True, max_batch=2, **kw)
    blk.load_expert_layer(0, synth.layer_image(40, E, H, I, 64))
    blk.load_router(0, synth.router_weights(50, E, H))
    return blk


def test_expert_parallel_peer_that_never_calls_times_out(oracle_lib):
    r0 = _block(expert_begin=0, expert_count=4)
    r1 = _block(expert_begin=4, expert_count=4)
    handle = (ctypes.c_uint8 * 64)()
    for blk in (r0, r1):
        _lib.call("m1moe_cuda_ep_region", blk._ctx, 2, 1, ctypes.addressof(handle))
    ctxs = (ctypes.c_void_p * 2)(r0._ctx.value, r1._ctx.value)
    _lib.call("m1moe_cuda_ep_connect_local", r0._ctx, 0, ctxs)
    _lib.call("m1moe_cuda_ep_connect_local", r1._ctx, 1, ctxs)
    _lib.call("m1moe_cuda_set_wait_limit", r0._ctx, 4096)
    x = torch.from_numpy(synth.bf16_to_f32(synth.hidden_states(1, 1, H))).cuda()
    out = torch.empty_like(x)
    t0 = time.perf_counter()
    # rank 0 alone: rank 1's tokens never arrive
    _lib.call("m1moe_cuda_moe_layer_ep", r0._ctx, 0, x.data_ptr(), 0, x.data_ptr(), 0,
              out.data_ptr(), 0, 0, 0, torch.cuda.current_stream().cuda_stream)
    with pytest.raises(M1MoECudaError, match="DEVICE"):
        r0.synchronize()
    assert time.perf_counter() - t0 < 30.0
    r0.close()
    r1.close()
    # fresh contexts on the same GPU work
    blk = _block()
    xb = synth.hidden_states(2, 2, H)
    y = blk.forward(0, torch.from_numpy(synth.bf16_to_f32(xb)).cuda()).cpu().numpy()
    blk.synchronize()
    img = synth.layer_image(40, E, H, I, 64)
    ref, _, _ = oracle_lib.moe_layer(img, synth.router_weights(50, E, H), synth.bf16_to_f32(xb),
                                     None, h=H, inter=I, E=E, K=K, gs=64, norm=True)
    assert rel_max_err(y, ref) < 1e-3
    blk.close()


def _tiny_decode(max_seq=8, B=1):
    dm = DenseModel(hidden_dim=256, num_heads=2, num_kv_heads=2, num_layers=1, vocab_size=100,
                    qk_norm=False, max_batch=B, max_seq=max_seq)
    dm.load_all(synth.dense_weights(3, h=256, nh=2, nkv=2, hd=128, layers=1, vocab=100,
                                    qk_norm=False))
    blk = MoEBlock(hidden_dim=256, intermediate_dim=128, num_experts=4, top_k=2, num_layers=1,
                   max_batch=B)
    blk.load_expert_layer(0, synth.layer_image(4, 4, 256, 128, 64))
    blk.load_router(0, synth.router_weights(5, 4, 256))
    return dm, blk


def test_decode_step_token_id_out_of_range():
    dm, blk = _tiny_decode()
    dm.step(blk, torch.tensor([100], dtype=torch.int32, device="cuda"))
    with pytest.raises(M1MoECudaError, match="DEVICE"):
        dm.synchronize()
    dm.reset()
    tok = dm.step(blk, torch.tensor([7], dtype=torch.int32, device="cuda"))
    dm.synchronize()  # the error word was cleared; a good step reports nothing
    assert 0 <= int(tok.item()) < 100
    dm.close()
    blk.close()


def test_decode_step_past_the_kv_cache():
    dm, blk = _tiny_decode(max_seq=4)
    dm.set_position(3)
    tok = torch.tensor([1], dtype=torch.int32, device="cuda")
    tok = dm.step(blk, tok).clone()  # position 3, the last slot
    dm.synchronize()
    assert dm.position() == 4
    dm.step(blk, tok)  # position 4 is past the end
    with pytest.raises(M1MoECudaError, match="DEVICE"):
        dm.synchronize()
    dm.close()
    blk.close()


def test_prefill_value_beyond_fp16_range():
    blk = MoEBlock(hidden_dim=512, intermediate_dim=256, num_experts=E, top_k=K, num_layers=1,
                   norm_topk_prob=True, max_batch=8)
    blk.load_expert_layer(0, synth.layer_image(40, E, 512, 256, 64))
    blk.load_router(0, synth.router_weights(50, E, 512))
    x = torch.from_numpy(synth.bf16_to_f32(synth.hidden_states(9, 16, 512))).cuda()
    x[3, 17] = 1.0e6  # beyond 65504: the token operand cannot be fp16
    blk.prefill(0, x)
    with pytest.raises(M1MoECudaError, match="DEVICE"):
        blk.synchronize()
    # the same call without the outlier is clean
    x[3, 17] = 0.5
    blk.prefill(0, x)
    blk.synchronize()
    blk.close()
