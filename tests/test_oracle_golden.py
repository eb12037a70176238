"""Pin the CPU oracle (and the host-side format code) to the reference's fixtures.

The fixtures in tests/golden were produced by the reference's own converter
(scripts/extract_olmoe.py, scripts/extract_mixtral.py) — see make_golden.py.
CPU only.
"""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import rel_max_err
from m1moe_b200 import spec, synth
from m1moe_b200.checkpoint import WeightStore


def test_bf16_known_answers(golden, oracle_lib):
    g = golden("quant_cases")
    L = oracle_lib.lib()
    for v, want, back in zip(g["bf16_in"], g["bf16_out"], g["bf16_back"]):
        assert L.orc_f32_to_bf16(float(v)) == int(want)
        assert np.float32(L.orc_bf16_to_f32(int(want))).view(np.uint32) == back.view(np.uint32)
    assert np.array_equal(synth.f32_to_bf16(g["bf16_in"]), g["bf16_out"])
    assert np.array_equal(synth.bf16_to_f32(g["bf16_out"]).view(np.uint32),
                          g["bf16_back"].view(np.uint32))


def test_expert_bytes(golden, oracle_lib):
    g = golden("quant_cases")
    for (h, i, gs), want in zip(g["expert_bytes_dims"], g["expert_bytes"]):
        assert oracle_lib.expert_bytes(int(h), int(i), int(gs)) == want
        assert spec.expert_bytes(int(h), int(i), int(gs)) == want
    # The shipped configs' documented block sizes (docs/LIMITS.md:31, ModelSpec.swift:36-52).
    assert spec.OLMOE_1B_7B.expert_bytes_4bit == 3_538_944
    assert spec.MIXTRAL_8X7B.expert_bytes_4bit == 99_090_432
    offs = oracle_lib.expert_offsets(2048, 1024, 64)
    o = spec.expert_offsets(2048, 1024, 64)
    assert offs == [o[k] for k in ("gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b",
                                   "down_w", "down_s", "down_b")]


def test_nibble_pack_matches_reference(golden):
    """Our pack/unpack reproduces the reference quantiser's word layout bit for bit."""
    g = golden("quant_cases")
    for i in range(4):
        p = g[f"packed{i}"]
        q = synth.unpack_nibbles(p)
        assert q.max() <= 15
        assert np.array_equal(synth.pack_nibbles(q), p)
    # hand-built words: 0x76543210 -> 0..7, 0xFEDCBA98 -> 8..15
    w = np.array([[0x76543210, 0xFEDCBA98]], dtype=np.uint32)
    assert synth.unpack_nibbles(w).tolist() == [list(range(16))]


def test_dequant_rule_matches_reference_quantiser(golden):
    """dequant(q, scale, bias) = q*scale + bias reproduces the quantised weights."""
    g = golden("quant_cases")
    for i in range(4):
        w, p, s, b = g[f"w{i}"], g[f"packed{i}"], g[f"scales{i}"], g[f"biases{i}"]
        deq = synth.dequant(p, s, b, 64)
        sf = np.repeat(synth.bf16_to_f32(s), 64, axis=1).astype(np.float64)
        bf = np.repeat(synth.bf16_to_f32(b), 64, axis=1).astype(np.float64)
        # half a step of rounding, plus the bf16 rounding of scale (x15) and bias
        bound = 0.5 * sf + 16 * sf * 2.0 ** -8 + np.abs(bf) * 2.0 ** -8 + 1e-7
        # all-zero groups quantise with scale 1 -> exact zeros
        assert np.all(np.abs(deq - w) <= bound)


@pytest.mark.parametrize("case", range(4))
def test_oracle_matvec_vs_reference_golden(golden, oracle_lib, case):
    g = golden("quant_cases")
    y = oracle_lib.matvec4bit(g[f"packed{case}"], g[f"scales{case}"], g[f"biases{case}"],
                              g[f"x{case}"], 64)
    assert rel_max_err(y, g[f"y{case}"]) < 1e-5


def test_oracle_matvec_threads_identical(oracle_lib):
    rng = np.random.default_rng(3)
    W, S, B, _ = synth.quant_matrix(rng, 256, 512, 64)
    x = synth.bf16_to_f32(synth.hidden_states(5, 1, 512))[0]
    y1 = oracle_lib.matvec4bit(W, S, B, x, 64, nthreads=1)
    y4 = oracle_lib.matvec4bit(W, S, B, x, 64, nthreads=4)
    assert np.array_equal(y1, y4)


@pytest.mark.parametrize("out_dim,in_dim,gs", [(64, 512, 64), (37, 4096 + 512, 64),
                                               (16, 8 * 72, 32), (8, 14336, 64)])
def test_oracle_lane_vectorised_matvec_bit_identical(oracle_lib, out_dim, in_dim, gs):
    """The lane-innermost matvec (used for the timed baseline and the large checks)
    gives the same bits as the literal lanes-outermost restatement, including a
    ragged last block of 64 words."""
    rng = np.random.default_rng(out_dim + in_dim)
    W, S, B, _ = synth.quant_matrix(rng, out_dim, in_dim, gs)
    x = rng.normal(0.0, 1.0, size=in_dim).astype(np.float32)
    y_plain = oracle_lib.matvec4bit_plain(W, S, B, x, gs)
    for nt in (1, 3):
        y = oracle_lib.matvec4bit(W, S, B, x, gs, nthreads=nt)
        assert np.array_equal(y.view(np.uint32), y_plain.view(np.uint32)), nt


@pytest.mark.parametrize("name", ["olmoe_tiny", "mixtral_tiny"])
def test_layer_file_layout(golden, tmp_path, name):
    """The reference extractor's layer_NN.bin splits at our offsets into blocks whose
    dequantised projections reproduce the synthetic source weights."""
    from golden.make_golden import source_expert_weights, router_weights

    g = golden(name)
    L, E, h, I, gs, seed = (int(v) for v in g["meta"])
    src = source_expert_weights(seed, L, E, h, I)
    eb = spec.expert_bytes(h, I, gs)
    for l in range(L):
        img = g[f"layer_{l:02d}"]
        assert img.size == E * eb
        for e in range(E):
            parts = synth.split_block(img[e * eb:(e + 1) * eb], h, I, gs)
            for proj in ("gate", "up", "down"):
                w = synth.bf16_to_f32(src[(l, e, proj)]).astype(np.float64)
                deq = synth.dequant(parts[f"{proj}_w"], parts[f"{proj}_s"], parts[f"{proj}_b"], gs)
                sf = np.repeat(synth.bf16_to_f32(parts[f"{proj}_s"]), gs, axis=1)
                assert np.all(np.abs(deq - w) <= 0.57 * sf + 1e-6), (l, e, proj)
    # router tensors read back through the manifest
    mdir = tmp_path / "m"
    mdir.mkdir()
    (mdir / "model_weights.json").write_bytes(g["manifest_json"].tobytes())
    (mdir / "model_weights.bin").write_bytes(g["model_weights_bin"].tobytes())
    store = WeightStore(mdir)
    arch = "olmoe" if name.startswith("olmoe") else "mixtral"
    sp = spec.ModelSpec("t", arch, h, 1, L, 1e-5, spec.MoESpec(E, 2, I, False), spec.QuantSpec(4, gs))
    for l, r in enumerate(router_weights(seed, L, E, h)):
        assert np.array_equal(store.tensor(sp.router_key(l)), r)
    store.close()
    assert json.loads(g["manifest_json"].tobytes())  # well-formed


def _f64_moe(img, router, x, res, h, I, E, K, gs, norm):
    """Float64 restatement of the MoE block from the reference's definitions."""
    eb = spec.expert_bytes(h, I, gs)
    logits = synth.bf16_to_f32(router).astype(np.float64) @ x
    p = np.exp(logits - logits.max())
    p /= p.sum()
    order = sorted(range(E), key=lambda e: (-p[e], e))[:K]
    w = p[order]
    if norm:
        w = w / w.sum()
    out = res.astype(np.float64).copy()
    for k, e in enumerate(order):
        parts = synth.split_block(img[e * eb:(e + 1) * eb], h, I, gs)
        g = synth.dequant(parts["gate_w"], parts["gate_s"], parts["gate_b"], gs) @ x
        u = synth.dequant(parts["up_w"], parts["up_s"], parts["up_b"], gs) @ x
        a = g / (1 + np.exp(-g)) * u
        out += w[k] * (synth.dequant(parts["down_w"], parts["down_s"], parts["down_b"], gs) @ a)
    return out, np.array(order), w, p


@pytest.mark.parametrize("name,K,norm", [("olmoe_tiny", 2, False), ("mixtral_tiny", 2, True)])
def test_oracle_moe_layer_vs_f64(golden, oracle_lib, name, K, norm):
    from golden.make_golden import router_weights

    g = golden(name)
    L, E, h, I, gs, seed = (int(v) for v in g["meta"])
    routers = router_weights(seed, L, E, h)
    x = synth.bf16_to_f32(synth.hidden_states(11, 3, h))
    res = synth.bf16_to_f32(synth.hidden_states(12, 3, h))
    out, idx, w = oracle_lib.moe_layer(g["layer_00"], routers[0], x, res, h=h, inter=I, E=E, K=K,
                                       gs=gs, norm=norm)
    for t in range(3):
        ref, order, wr, p = _f64_moe(g["layer_00"], routers[0], x[t].astype(np.float64), res[t],
                                     h, I, E, K, gs, norm)
        assert list(idx[t]) == list(order)
        assert np.allclose(w[t], wr, rtol=1e-5, atol=1e-7)
        assert rel_max_err(out[t], ref) < 1e-5


def test_oracle_topk_ties_and_renorm(oracle_lib):
    s = np.array([0.1, 0.3, 0.3, 0.2, 0.1], dtype=np.float32)
    idx, w = oracle_lib.select_topk(s, 3, False)
    assert idx.tolist() == [1, 2, 3]
    idx, w = oracle_lib.select_topk(s, 2, True)
    assert idx.tolist() == [1, 2] and np.allclose(w, [0.5, 0.5])
