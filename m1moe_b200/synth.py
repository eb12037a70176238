"""Seeded synthetic weights and activations with the benchmark's distributions.

Real checkpoints are not available, so every run uses synthetic data of the
reference's format and the BASELINE shapes:
  q ~ U{0..15} packed 8 per uint32 (nibble b of word w = column 8w+b),
  scale ~ U(0.005, 0.02) -> bf16, bias = -8*scale + N(0, 1e-3) -> bf16,
  router ~ N(0, 0.02) -> bf16, hidden ~ N(0, 1) -> bf16.
Host (numpy) generators feed parity tests and the CPU oracle; device (torch)
generators fill multi-GB expert tables for the benchmark without host traffic.
"""
from __future__ import annotations

import numpy as np

from .spec import expert_bytes, expert_offsets


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round to nearest even, the reference's rule (scripts/extract_olmoe.py:104-111)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def pack_nibbles(q: np.ndarray) -> np.ndarray:
    """uint8 q[rows][cols] (values 0..15) -> uint32[rows][cols/8], low nibble first."""
    rows, cols = q.shape
    g = q.reshape(rows, cols // 8, 8).astype(np.uint32)
    return np.bitwise_or.reduce(g << (4 * np.arange(8, dtype=np.uint32)), axis=2).astype(np.uint32)


def unpack_nibbles(w: np.ndarray) -> np.ndarray:
    rows, words = w.shape
    sh = (4 * np.arange(8, dtype=np.uint32))
    return ((w[:, :, None] >> sh) & 0xF).astype(np.uint8).reshape(rows, words * 8)


def quant_matrix(rng: np.random.Generator, rows: int, cols: int, gs: int):
    """One projection (W uint32[rows][cols/8], S, B uint16[rows][cols/gs]) and its q."""
    q = rng.integers(0, 16, size=(rows, cols), dtype=np.uint8)
    ng = cols // gs
    scale = f32_to_bf16(rng.uniform(0.005, 0.02, size=(rows, ng)).astype(np.float32))
    bias = f32_to_bf16((-8.0 * bf16_to_f32(scale)
                        + rng.normal(0.0, 1e-3, size=(rows, ng))).astype(np.float32))
    return pack_nibbles(q), scale, bias, q


def dequant(W: np.ndarray, S: np.ndarray, B: np.ndarray, gs: int) -> np.ndarray:
    """w = q*scale + bias in float64 (the reference's dequant rule)."""
    q = unpack_nibbles(W).astype(np.float64)
    s = np.repeat(bf16_to_f32(S).astype(np.float64), gs, axis=1)
    b = np.repeat(bf16_to_f32(B).astype(np.float64), gs, axis=1)
    return q * s + b


def expert_block(rng: np.random.Generator, hidden: int, inter: int, gs: int) -> np.ndarray:
    """One expert block [gateW|gateS|gateB|upW|upS|upB|downW|downS|downB] as uint8."""
    parts = []
    for rows, cols in ((inter, hidden), (inter, hidden), (hidden, inter)):
        W, S, B, _ = quant_matrix(rng, rows, cols, gs)
        parts += [W.view(np.uint8).ravel(), S.view(np.uint8).ravel(), B.view(np.uint8).ravel()]
    blk = np.concatenate(parts)
    assert blk.size == expert_bytes(hidden, inter, gs)
    return blk


def layer_image(seed: int, num_experts: int, hidden: int, inter: int, gs: int) -> np.ndarray:
    """One packed_experts/layer_NN.bin image (num_experts blocks) as uint8.

    Packed words are drawn as uniform random bytes (equivalent to q ~ U{0..15}
    per nibble, and much faster for multi-hundred-MB images)."""
    rng = np.random.default_rng(seed)
    eb = expert_bytes(hidden, inter, gs)
    img = np.empty((num_experts, eb), dtype=np.uint8)
    o = expert_offsets(hidden, inter, gs)
    for name, rows, cols in (("gate", inter, hidden), ("up", inter, hidden), ("down", hidden, inter)):
        nw, ng = rows * cols // 2, rows * (cols // gs)
        w0, s0, b0 = o[f"{name}_w"], o[f"{name}_s"], o[f"{name}_b"]
        img[:, w0:w0 + nw] = rng.integers(0, 256, size=(num_experts, nw), dtype=np.uint8)
        scale = f32_to_bf16(rng.uniform(0.005, 0.02, size=(num_experts, ng)).astype(np.float32))
        bias = f32_to_bf16((-8.0 * bf16_to_f32(scale)
                            + rng.normal(0.0, 1e-3, size=(num_experts, ng))).astype(np.float32))
        img[:, s0:s0 + 2 * ng] = scale.view(np.uint8).reshape(num_experts, 2 * ng)
        img[:, b0:b0 + 2 * ng] = bias.view(np.uint8).reshape(num_experts, 2 * ng)
    return img.reshape(-1)


def split_block(block: np.ndarray, hidden: int, inter: int, gs: int) -> dict[str, np.ndarray]:
    """Views of one expert block's nine arrays with their logical shapes."""
    o = expert_offsets(hidden, inter, gs)
    shapes = {"gate": (inter, hidden), "up": (inter, hidden), "down": (hidden, inter)}
    out = {}
    for name, (rows, cols) in shapes.items():
        w0, s0, b0 = o[f"{name}_w"], o[f"{name}_s"], o[f"{name}_b"]
        nw, ns = rows * cols // 2, rows * (cols // gs) * 2
        out[f"{name}_w"] = block[w0:w0 + nw].view(np.uint32).reshape(rows, cols // 8)
        out[f"{name}_s"] = block[s0:s0 + ns].view(np.uint16).reshape(rows, cols // gs)
        out[f"{name}_b"] = block[b0:b0 + ns].view(np.uint16).reshape(rows, cols // gs)
    return out


def router_weights(seed: int, num_experts: int, hidden: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return f32_to_bf16(rng.normal(0.0, 0.02, size=(num_experts, hidden)).astype(np.float32))


def hidden_states(seed: int, batch: int, hidden: int) -> np.ndarray:
    """bf16 bit patterns [batch][hidden] ~ N(0, 1)."""
    rng = np.random.default_rng(seed)
    return f32_to_bf16(rng.normal(0.0, 1.0, size=(batch, hidden)).astype(np.float32))


# ---------------------------------------------------------------- device ----

def layer_image_device(num_experts: int, hidden: int, inter: int, gs: int, *, seed: int,
                       device):
    """A layer image generated directly in HBM (torch uint8 tensor).

    Same distributions as layer_image(); the random stream differs (torch's
    generator), which does not matter for throughput runs.
    """
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    eb = expert_bytes(hidden, inter, gs)
    img = torch.empty((num_experts, eb), dtype=torch.uint8, device=device)
    o = expert_offsets(hidden, inter, gs)
    for name, rows, cols in (("gate", inter, hidden), ("up", inter, hidden), ("down", hidden, inter)):
        nw, ns = rows * cols // 2, rows * (cols // gs) * 2
        w0, s0, b0 = o[f"{name}_w"], o[f"{name}_s"], o[f"{name}_b"]
        img[:, w0:w0 + nw] = torch.randint(0, 256, (num_experts, nw), dtype=torch.uint8,
                                           generator=g, device=device)
        scale = (torch.rand((num_experts, ns // 2), generator=g, device=device) * 0.015 + 0.005
                 ).to(torch.bfloat16)
        bias = (-8.0 * scale.float() + 1e-3 * torch.randn((num_experts, ns // 2), generator=g,
                                                          device=device)).to(torch.bfloat16)
        img[:, s0:s0 + ns] = scale.view(torch.uint8).view(num_experts, ns)
        img[:, b0:b0 + ns] = bias.view(torch.uint8).view(num_experts, ns)
    return img.view(-1)


# ------------------------------------------------------------------ dense ----

def dense_weights(seed: int, *, h: int, nh: int, nkv: int, hd: int, layers: int, vocab: int,
                  qk_norm: bool) -> dict:
    """Non-expert weights of a decoder (bf16 bit patterns): projections,
    embedding and LM head ~ N(0, 0.02); norm weights 1 + N(0, 0.02)."""
    rng = np.random.default_rng(seed)

    def mat(rows, cols, std=0.02):
        return f32_to_bf16(rng.normal(0.0, std, size=(rows, cols)).astype(np.float32))

    def norm(n):
        return f32_to_bf16((1.0 + rng.normal(0.0, 0.02, size=n)).astype(np.float32))

    qd, kvd = nh * hd, nkv * hd
    w = {"embed": mat(vocab, h), "lm_head": mat(vocab, h), "final_norm": norm(h),
         "in_norm": [], "post_norm": [], "wq": [], "wk": [], "wv": [], "wo": [], "qn": [], "kn": []}
    for _ in range(layers):
        w["in_norm"].append(norm(h))
        w["post_norm"].append(norm(h))
        w["wq"].append(mat(qd, h))
        w["wk"].append(mat(kvd, h))
        w["wv"].append(mat(kvd, h))
        w["wo"].append(mat(h, qd))
        if qk_norm:
            w["qn"].append(norm(qd))
            w["kn"].append(norm(kvd))
    return w


def dense_weights_device(seed: int, *, h: int, nh: int, nkv: int, hd: int, layers: int, vocab: int,
                         qk_norm: bool, device) -> dict:
    """The same distributions generated in HBM (torch bf16 tensors), for
    multi-GB benchmark models; the random stream differs from dense_weights."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def mat(rows, cols, std=0.02):
        return (torch.randn((rows, cols), generator=g, device=device) * std).to(torch.bfloat16)

    def norm(n):
        return (1.0 + 0.02 * torch.randn((n,), generator=g, device=device)).to(torch.bfloat16)

    qd, kvd = nh * hd, nkv * hd
    w = {"embed": mat(vocab, h), "lm_head": mat(vocab, h), "final_norm": norm(h),
         "in_norm": [], "post_norm": [], "wq": [], "wk": [], "wv": [], "wo": [], "qn": [], "kn": []}
    for _ in range(layers):
        w["in_norm"].append(norm(h))
        w["post_norm"].append(norm(h))
        w["wq"].append(mat(qd, h))
        w["wk"].append(mat(kvd, h))
        w["wv"].append(mat(kvd, h))
        w["wo"].append(mat(h, qd))
        if qk_norm:
            w["qn"].append(norm(qd))
            w["kn"].append(norm(kvd))
    return w
