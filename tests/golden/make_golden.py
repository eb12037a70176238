"""Generate the golden fixtures in tests/golden/ from the REFERENCE's own code.

    python tests/golden/make_golden.py --reference <path to an M1MoE checkout>

M1MoE ships no tests, fixtures or golden vectors.  Its only code that runs
outside Apple hardware is the Python converter (scripts/extract_olmoe.py and
scripts/extract_mixtral.py: safetensors reader, f32_to_bf16, quantize_4bit,
expert_bytes, extract).  This script imports those modules from the given
checkout and runs them on seeded synthetic inputs:

  * quant_cases.npz   quantize_4bit outputs (both copies, which must agree) on
                      seeded matrices including constant and all-zero groups,
                      f32_to_bf16 / bf16_to_f32 known answers, expert_bytes for
                      the shipped and test shapes, and float64 golden matvecs
                      y = dequant(W) @ x computed from the quantiser's outputs
                      with the reference's own bf16_to_f32.
  * olmoe_tiny.npz,   a synthetic OLMoE- / Mixtral-named safetensors checkpoint
    mixtral_tiny.npz  run end to end through the reference's extract(): the
                      resulting packed_experts/layer_NN.bin bytes, the router
                      tensors read back through model_weights.json, and the
                      seeds that regenerate the source weights.

The tests then check the CPU oracle and the CUDA path against these files.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import struct
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# Shapes of the end-to-end extraction fixtures.
OLMOE_TINY = dict(hidden=128, inter=64, experts=4, layers=2, seed=1234)
MIXTRAL_TINY = dict(hidden=128, inter=128, experts=4, layers=1, seed=4321)


def _load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _bf16(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def source_expert_weights(seed: int, layers: int, experts: int, hidden: int, inter: int):
    """Seeded bf16 source weights {(L, E, proj): uint16 array}, proj in gate/up/down.

    Expert 0 of layer 0 carries the quantiser's edge cases: its gate row 0
    has an all-zero first group (scale 0 -> 1 branch) and row 1 a constant
    first group; its up row 0 spans a wide range with an outlier."""
    rng = np.random.default_rng(seed)
    out = {}
    for L in range(layers):
        for E in range(experts):
            for proj, (r, c) in (("gate", (inter, hidden)), ("up", (inter, hidden)),
                                 ("down", (hidden, inter))):
                w = rng.normal(0.0, 0.02, size=(r, c)).astype(np.float32)
                if L == 0 and E == 0 and proj == "gate":
                    w[0, :64] = 0.0
                    w[1, :64] = 0.5
                if L == 0 and E == 0 and proj == "up":
                    w[0, 5] = 3.0
                out[(L, E, proj)] = _bf16(w)
    return out


def router_weights(seed: int, layers: int, experts: int, hidden: int):
    rng = np.random.default_rng(seed + 1)
    return [_bf16(rng.normal(0.0, 0.02, size=(experts, hidden)).astype(np.float32))
            for _ in range(layers)]


def write_safetensors(path: Path, tensors: dict[str, np.ndarray]) -> None:
    """Minimal safetensors writer (8-byte header length, JSON header, raw data)."""
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        dt = {np.dtype(np.uint16): "BF16", np.dtype(np.float32): "F32"}[arr.dtype]
        raw = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)


def run_extract(mod, arch: str, cfg: dict, workdir: Path) -> dict:
    L, E, h, I, seed = cfg["layers"], cfg["experts"], cfg["hidden"], cfg["inter"], cfg["seed"]
    src = source_expert_weights(seed, L, E, h, I)
    routers = router_weights(seed, L, E, h)
    tensors = {}
    for l in range(L):
        if arch == "olmoe":
            tensors[f"model.layers.{l}.mlp.gate.weight"] = routers[l]
            for e in range(E):
                for proj in ("gate", "up", "down"):
                    tensors[f"model.layers.{l}.mlp.experts.{e}.{proj}_proj.weight"] = src[(l, e, proj)]
        else:
            tensors[f"model.layers.{l}.block_sparse_moe.gate.weight"] = routers[l]
            for e in range(E):
                for proj, w in (("gate", "w1"), ("up", "w3"), ("down", "w2")):
                    tensors[f"model.layers.{l}.block_sparse_moe.experts.{e}.{w}"] = src[(l, e, proj)]
        tensors[f"model.layers.{l}.post_attention_layernorm.weight"] = np.ones(h, np.float32)
    model_dir, out_dir = workdir / f"{arch}_src", workdir / f"{arch}_out"
    model_dir.mkdir()
    write_safetensors(model_dir / "model-00001-of-00001.safetensors", tensors)
    mod.extract(str(model_dir), str(out_dir), group_size=64, verbose=False)
    manifest = json.loads((out_dir / "model_weights.json").read_text())
    wbin = (out_dir / "model_weights.bin").read_bytes()
    res = {"manifest_json": np.frombuffer(json.dumps(manifest, sort_keys=True).encode(), np.uint8),
           "model_weights_bin": np.frombuffer(wbin, np.uint8),
           "meta": np.array([L, E, h, I, 64, seed], dtype=np.int64)}
    for l in range(L):
        res[f"layer_{l:02d}"] = np.frombuffer(
            (out_dir / "packed_experts" / f"layer_{l:02d}.bin").read_bytes(), np.uint8)
    return res


def quant_cases(eo, em) -> dict:
    rng = np.random.default_rng(7)
    out = {}
    shapes = [(8, 128), (16, 256), (3, 64), (32, 1024)]
    for i, (r, c) in enumerate(shapes):
        w = rng.normal(0.0, 0.05, size=(r, c)).astype(np.float32)
        if i == 0:
            w[0, :64] = 0.0           # scale == 0 -> 1
            w[1, 64:] = -1.25         # constant group
            w[2, 3] = 40.0            # outlier
            w[3, :] = np.linspace(-1, 1, c, dtype=np.float32)
        p, s, b = eo.quantize_4bit(w, 64)
        p2, s2, b2 = em.quantize_4bit(w, 64)
        assert np.array_equal(p, p2) and np.array_equal(s, s2) and np.array_equal(b, b2), \
            "the two quantize_4bit copies disagree"
        x = eo.bf16_to_f32(_bf16(rng.normal(0.0, 1.0, size=c).astype(np.float32)))
        # dequant with the reference's own bf16_to_f32 (w = q*scale + bias), float64 matvec
        q = ((p[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 0xF).reshape(r, c)
        sf = np.repeat(eo.bf16_to_f32(s).astype(np.float64), 64, axis=1)
        bf = np.repeat(eo.bf16_to_f32(b).astype(np.float64), 64, axis=1)
        y = (q.astype(np.float64) * sf + bf) @ x.astype(np.float64)
        out.update({f"w{i}": w, f"packed{i}": p, f"scales{i}": s, f"biases{i}": b,
                    f"x{i}": x, f"y{i}": y})
    v = np.array([0.0, -0.0, 1.0, -1.0, 1.00390625, 1.005859375, 1.0029296875, 3.14159265,
                  -2.71828182, 1e-30, 65504.0, 3.3895314e38, 0.1, 1.0 / 3.0, -7.5e-5],
                 dtype=np.float32)
    out["bf16_in"] = v
    out["bf16_out"] = eo.f32_to_bf16(v)
    out["bf16_back"] = eo.bf16_to_f32(out["bf16_out"])
    dims = [(2048, 1024, 64), (4096, 14336, 64), (128, 64, 64), (128, 128, 64), (256, 512, 128)]
    out["expert_bytes_dims"] = np.array(dims, dtype=np.int64)
    out["expert_bytes"] = np.array([eo.expert_bytes(*d) for d in dims], dtype=np.int64)
    assert all(em.expert_bytes(*d) == eo.expert_bytes(*d) for d in dims)
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", required=True, type=Path,
                    help="root of an M1MoE checkout (contains scripts/extract_olmoe.py)")
    args = ap.parse_args()
    eo = _load(args.reference / "scripts" / "extract_olmoe.py", "ref_extract_olmoe")
    em = _load(args.reference / "scripts" / "extract_mixtral.py", "ref_extract_mixtral")
    np.savez_compressed(HERE / "quant_cases.npz", **quant_cases(eo, em))
    with tempfile.TemporaryDirectory() as td:
        td = Path(td)
        np.savez_compressed(HERE / "olmoe_tiny.npz", **run_extract(eo, "olmoe", OLMOE_TINY, td))
        np.savez_compressed(HERE / "mixtral_tiny.npz",
                            **run_extract(em, "mixtral", MIXTRAL_TINY, td))
    for f in sorted(HERE.glob("*.npz")):
        print(f"{f.name}: {f.stat().st_size} bytes")


if __name__ == "__main__":
    sys.exit(main())
