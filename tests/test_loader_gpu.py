"""Native cold-start loader (m1moe_cuda_load_expert_files) on the GPU.

The converted model directory is written from the reference converter's
fixtures and from synthetic OLMoE-shaped layers; loading it through the
native loader (io threads, pinned ring, overlapped copies and repacks) must
give the same table as loading the same bytes through
m1moe_cuda_load_expert_layer: the MoE outputs of both contexts agree and the
routing is identical, for whole models and for expert shards.  A missing or
wrong-sized file fails the call with INVALID_ARG naming the file.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_max_err
from m1moe_b200 import M1MoECudaError, MoEBlock, checkpoint, synth
from test_checkpoint_cpu import write_model_dir

pytestmark = pytest.mark.gpu


def _pair(h, I, E, K, layers, norm, **shard):
    kw = dict(hidden_dim=h, intermediate_dim=I, num_experts=E, top_k=K, num_layers=layers,
              norm_topk_prob=norm, max_batch=8, **shard)
    return MoEBlock(**kw), MoEBlock(**kw)


def _same_outputs(a, b, layers, h, B=8, seed=3):
    x = torch.from_numpy(synth.bf16_to_f32(synth.hidden_states(seed, B, h))).cuda()
    for L in range(layers):
        ya, ia, _ = a.forward(L, x, x, return_topk=True)
        yb, ib, _ = b.forward(L, x, x, return_topk=True)
        a.synchronize()
        b.synchronize()
        assert torch.equal(ia, ib), L
        assert rel_max_err(ya.cpu().numpy(), yb.cpu().numpy()) < 1e-6, L


@pytest.mark.parametrize("name", ["olmoe_tiny", "mixtral_tiny"])
@pytest.mark.parametrize("threads", [1, 4])
def test_native_loader_matches_byte_loader(golden, tmp_path, name, threads):
    from golden.make_golden import router_weights
    g = golden(name)
    sp = write_model_dir(g, tmp_path, name)
    L, E, h, I, gs, seed = (int(v) for v in g["meta"])
    routers = router_weights(seed, L, E, h)
    a, b = _pair(h, I, E, 2, L, name.startswith("mixtral"))
    checkpoint.load_model_dir(a, sp, tmp_path, io_threads=threads)
    for layer in range(L):
        b.load_expert_layer(layer, g[f"layer_{layer:02d}"])
        b.load_router(layer, routers[layer])
    _same_outputs(a, b, L, h)
    a.close()
    b.close()


@pytest.mark.parametrize("shard", [dict(expert_begin=0, expert_count=32),
                                   dict(expert_begin=48, expert_count=16)])
def test_native_loader_olmoe_shape_and_shards(tmp_path, shard):
    """Two OLMoE-shaped layers (226 MB files: several 32 MB chunks and staging
    groups per layer), whole and as expert shards."""
    h, I, E, K, L = 2048, 1024, 64, 8, 2
    d = tmp_path / "packed_experts"
    d.mkdir()
    imgs = []
    for layer in range(L):
        img = synth.layer_image_device(E, h, I, 64, seed=70 + layer, device="cuda").cpu().numpy()
        img.tofile(d / f"layer_{layer:02d}.bin")
        imgs.append(img)
    routers = [synth.router_weights(80 + layer, E, h) for layer in range(L)]
    for kw in (dict(), shard):
        a, b = _pair(h, I, E, K, L, False, **kw)
        a.load_expert_files(d, io_threads=3)
        for layer in range(L):
            a.load_router(layer, routers[layer])
            b.load_expert_layer(layer, imgs[layer])
            b.load_router(layer, routers[layer])
        _same_outputs(a, b, L, h)
        a.close()
        b.close()


def test_native_loader_rejects_bad_files(golden, tmp_path):
    g = golden("olmoe_tiny")
    sp = write_model_dir(g, tmp_path, "olmoe_tiny")
    L, E, h, I, gs, seed = (int(v) for v in g["meta"])
    d = tmp_path / "packed_experts"
    blk = MoEBlock(hidden_dim=h, intermediate_dim=I, num_experts=E, top_k=2, num_layers=L)
    p = d / "layer_01.bin"
    good = p.read_bytes()
    p.write_bytes(good[:-64])
    with pytest.raises(M1MoECudaError, match=r"INVALID_ARG.*layer_01\.bin: \d+ bytes, expected"):
        blk.load_expert_files(d)
    p.write_bytes(good + b"\0" * 64)
    with pytest.raises(M1MoECudaError, match=r"layer_01\.bin: \d+ bytes, expected"):
        blk.load_expert_files(d)
    p.unlink()
    with pytest.raises(M1MoECudaError, match=r"layer_01\.bin: cannot open"):
        blk.load_expert_files(d)
    # nothing was marked loaded: the layer call still reports it
    with pytest.raises(M1MoECudaError, match="NOT_LOADED"):
        blk.forward(0, torch.zeros((1, h), device="cuda"))
    blk.close()
