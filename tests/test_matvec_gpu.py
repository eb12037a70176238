"""CUDA int4 matvec / unpack vs the CPU oracle and the reference's fixtures.

Tolerance (the parity bar): max |y - y_ref| <= 1e-3 * ||y_ref||_2 with fp32
accumulation; nibble unpacking bit-exact.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_max_err
from m1moe_b200 import synth

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _dev(a: np.ndarray) -> torch.Tensor:
    a = np.ascontiguousarray(a)
    view = {np.dtype(np.uint32): np.int32, np.dtype(np.uint16): np.int16}.get(a.dtype, a.dtype)
    return torch.from_numpy(a.view(view)).cuda()


def _x_dev(x_bf16: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(x_bf16).view(np.int16)).cuda().view(torch.bfloat16)
    return t if dtype == torch.bfloat16 else t.float()


@pytest.mark.parametrize("case", range(4))
def test_matvec_vs_reference_golden(golden, case):
    from m1moe_b200 import matvec4
    g = golden("quant_cases")
    x = torch.from_numpy(g[f"x{case}"]).cuda()
    y = matvec4(_dev(g[f"packed{case}"]), _dev(g[f"scales{case}"]), _dev(g[f"biases{case}"]), x)
    torch.cuda.synchronize()
    assert rel_max_err(y.cpu().numpy(), g[f"y{case}"]) < TOL


def test_unpack_bit_exact_vs_reference_quantiser(golden):
    from m1moe_b200 import unpack4
    g = golden("quant_cases")
    for i in range(4):
        p = g[f"packed{i}"]
        q = unpack4(_dev(p)).cpu().numpy()
        assert np.array_equal(q, synth.unpack_nibbles(p))
    w = np.array([[0x76543210, 0xFEDCBA98]], dtype=np.uint32)
    assert unpack4(_dev(w)).cpu().numpy().tolist() == [list(range(16))]


@pytest.mark.parametrize("out_dim,in_dim", [(1024, 2048), (2048, 1024), (64, 64), (40, 192),
                                            (7, 1088), (4096, 14336)])
@pytest.mark.parametrize("batch", [1, 3, 8])
def test_matvec_vs_oracle(oracle_lib, out_dim, in_dim, batch):
    from m1moe_b200 import matvec4
    rng = np.random.default_rng(out_dim * 7 + in_dim + batch)
    W, S, B, _ = synth.quant_matrix(rng, out_dim, in_dim, 64)
    xb = synth.hidden_states(batch + 100, batch, in_dim)
    xf = synth.bf16_to_f32(xb)
    refs = [oracle_lib.matvec4bit(W, S, B, xf[t], 64, nthreads=8) for t in range(batch)]
    for xdt in (torch.bfloat16, torch.float32):
        for ydt in (torch.float32, torch.bfloat16):
            y = matvec4(_dev(W), _dev(S), _dev(B), _x_dev(xb, xdt), out_dtype=ydt)
            yc = y.float().cpu().numpy()
            for t in range(batch):
                if ydt == torch.bfloat16:
                    # bf16 output: the arithmetic bar plus the output's own rounding
                    # (half an ulp, 2^-9 relative, of each element).
                    bound = TOL * np.linalg.norm(refs[t]) + 2.0 ** -8 * np.abs(refs[t])
                    assert np.all(np.abs(yc[t] - refs[t]) <= bound), (xdt, ydt, t)
                else:
                    assert rel_max_err(yc[t], refs[t]) < TOL, (xdt, ydt, t)


def test_matvec_group_size_128(oracle_lib):
    from m1moe_b200 import matvec4
    rng = np.random.default_rng(9)
    W, S, B, _ = synth.quant_matrix(rng, 256, 1024, 128)
    xf = synth.bf16_to_f32(synth.hidden_states(1, 1, 1024))[0]
    y = matvec4(_dev(W), _dev(S), _dev(B), torch.from_numpy(xf).cuda(), group_size=128)
    assert rel_max_err(y.cpu().numpy(), oracle_lib.matvec4bit(W, S, B, xf, 128)) < TOL


def test_matvec_strided_over_expert_table(oracle_lib):
    """All experts' gate projections of one layer image in one launch."""
    from m1moe_b200 import matvec4_strided, spec
    h, I, E = 512, 256, 6
    img = synth.layer_image(5, E, h, I, 64)
    o = spec.expert_offsets(h, I, 64)
    eb = spec.expert_bytes(h, I, 64)
    d = torch.from_numpy(img).cuda()
    xb = synth.hidden_states(3, 2, h)
    xf = synth.bf16_to_f32(xb)
    y = matvec4_strided(d[o["gate_w"]:], d[o["gate_s"]:], d[o["gate_b"]:], eb, E, I, h,
                        _x_dev(xb, torch.bfloat16))
    yc = y.cpu().numpy()
    for e in range(E):
        parts = synth.split_block(img[e * eb:(e + 1) * eb], h, I, 64)
        for t in range(2):
            ref = oracle_lib.matvec4bit(parts["gate_w"], parts["gate_s"], parts["gate_b"], xf[t], 64)
            assert rel_max_err(yc[e, t], ref) < TOL


@pytest.mark.parametrize("batch", [1, 8])
def test_matvec_strided_stream_of_experts(oracle_lib, batch):
    """OLMoE-shaped gate projections of 16 experts in one launch: enough row
    tiles for the bulk-copy ring kernel (one CTA per SM, producer warp)."""
    from m1moe_b200 import matvec4_strided, spec
    h, I, E = 2048, 1024, 16
    img = synth.layer_image(11, E, h, I, 64)
    o = spec.expert_offsets(h, I, 64)
    eb = spec.expert_bytes(h, I, 64)
    d = torch.from_numpy(img).cuda()
    xb = synth.hidden_states(13, batch, h)
    xf = synth.bf16_to_f32(xb)
    y = matvec4_strided(d[o["gate_w"]:], d[o["gate_s"]:], d[o["gate_b"]:], eb, E, I, h,
                        _x_dev(xb, torch.bfloat16))
    yc = y.cpu().numpy()
    for e in range(E):
        parts = synth.split_block(img[e * eb:(e + 1) * eb], h, I, 64)
        for t in range(batch):
            ref = oracle_lib.matvec4bit(parts["gate_w"], parts["gate_s"], parts["gate_b"], xf[t], 64,
                                        nthreads=8)
            assert rel_max_err(yc[e, t], ref) < TOL, (e, t)


@pytest.mark.parametrize("out_dim", [1028, 1020])
def test_matvec_stream_ragged_tiles(oracle_lib, out_dim):
    """A stream of 12 matrices whose row count the ring's 36-row tiles do not
    divide (1028 = 28 x 36 + 20, 1020 = 28 x 36 + 12: a short tail tile per
    matrix): every row of every matrix."""
    from m1moe_b200 import matvec4_strided
    in_dim, M = 2048, 12
    rng = np.random.default_rng(out_dim)
    mats = [synth.quant_matrix(rng, out_dim, in_dim, 64)[:3] for _ in range(M)]
    wb, sb = out_dim * in_dim // 2, out_dim * (in_dim // 64) * 2
    stride = wb + 2 * sb
    blob = np.concatenate([np.concatenate([W.view(np.uint8).ravel(), S.view(np.uint8).ravel(),
                                           B.view(np.uint8).ravel()]) for W, S, B in mats])
    d = torch.from_numpy(blob).cuda()
    xb = synth.hidden_states(7, 1, in_dim)
    xf = synth.bf16_to_f32(xb)
    y = matvec4_strided(d, d[wb:], d[wb + sb:], stride, M, out_dim, in_dim, _x_dev(xb, torch.bfloat16))
    yc = y.cpu().numpy()
    for m, (W, S, B) in enumerate(mats):
        ref = oracle_lib.matvec4bit(W, S, B, xf[0], 64, nthreads=8)
        assert rel_max_err(yc[m, 0], ref) < TOL, m


def test_matvec_rejects_bad_shapes():
    from m1moe_b200 import M1MoECudaError, matvec4
    w = torch.zeros((4, 12), dtype=torch.int32, device="cuda")  # in_dim 96: not % 64
    s = torch.zeros((4, 2), dtype=torch.int16, device="cuda")
    x = torch.zeros(96, device="cuda")
    with pytest.raises(M1MoECudaError, match="INVALID_ARG"):
        matvec4(w, s, s, x)
    w = torch.zeros((4, 16), dtype=torch.int32, device="cuda")
    x = torch.zeros(128, device="cuda")
    with pytest.raises(M1MoECudaError, match="UNSUPPORTED"):
        matvec4(w, s, s, x, group_size=16)
