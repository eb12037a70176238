"""Readers for the reference's converted-model directory (cold start).

Layout written by scripts/extract_olmoe.py:10-18 / extract_mixtral.py:10-18:
  model_weights.bin   flat non-expert tensors, 4-byte aligned
  model_weights.json  manifest {name: {offset, shape, dtype}} (dtype "bf16"/"f32")
  packed_experts/layer_NN.bin   num_experts expert blocks back to back

WeightStore (Sources/M1MoE/WeightStore.swift:15-30, 47-76, 90-126) mmaps the
first two; InferenceEngine re-reads the layer files with pread on every token
(:62-77, :271-280).  Here the layer files are read once, in parallel threads
(the shape of ExpertCache.prefetch, ExpertCache.swift:126-196), and copied
into the HBM expert table through pinned staging by the C ABI.
"""
from __future__ import annotations

import json
import mmap
from pathlib import Path

import numpy as np

from .spec import ModelSpec

_NP_DTYPE = {"bf16": np.uint16, "f32": np.float32}


class WeightStore:
    """Read-only view of model_weights.bin through its JSON manifest."""

    def __init__(self, model_dir: str | Path):
        d = Path(model_dir)
        self.manifest = json.loads((d / "model_weights.json").read_text())
        self._f = open(d / "model_weights.bin", "rb")
        size = (d / "model_weights.bin").stat().st_size
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ) if size else None
        self._buf = np.frombuffer(self._mm, dtype=np.uint8) if self._mm else np.empty(0, np.uint8)

    def tensor(self, name: str) -> np.ndarray:
        """The named tensor (bf16 as uint16 bit patterns).  KeyError if absent."""
        info = self.manifest[name]
        dt = np.dtype(_NP_DTYPE[info["dtype"]])
        n = int(np.prod(info["shape"])) if info["shape"] else 1
        off = int(info["offset"])
        return self._buf[off:off + n * dt.itemsize].view(dt).reshape(info["shape"])

    def close(self) -> None:
        self._buf = None
        if self._mm is not None:
            self._mm.close()
        self._f.close()


def layer_path(model_dir: str | Path, layer: int) -> Path:
    return Path(model_dir) / "packed_experts" / f"layer_{layer:02d}.bin"


def read_layer(model_dir: str | Path, layer: int, spec: ModelSpec) -> np.ndarray:
    """The bytes of layer_NN.bin, checked against num_experts * expertBytes4Bit
    (the size check of extract_olmoe.py:340-344)."""
    p = layer_path(model_dir, layer)
    want = spec.moe.num_experts * spec.expert_bytes_4bit
    data = np.fromfile(p, dtype=np.uint8)
    if data.size != want:
        raise ValueError(f"{p}: {data.size} bytes, expected {want}")
    return data


def check_layer_files(model_dir: str | Path, spec: ModelSpec) -> None:
    """Every layer file exists with the size the converter guarantees
    (extract_olmoe.py:340-344), before anything is copied."""
    want = spec.moe.num_experts * spec.expert_bytes_4bit
    for L in range(spec.num_layers):
        p = layer_path(model_dir, L)
        if not p.exists():
            raise FileNotFoundError(f"{p}: missing")
        if p.stat().st_size != want:
            raise ValueError(f"{p}: {p.stat().st_size} bytes, expected {want}")


def load_model_dir(block, spec: ModelSpec, model_dir: str | Path, io_threads: int = 4) -> None:
    """Cold start: fill `block` (a MoEBlock) with every layer's experts and router.

    The expert files go through the library's native loader
    (MoEBlock.load_expert_files: io_threads threads read 32 MB chunks into
    pinned buffers while earlier chunks are copied and repacked on the GPU,
    the concurrent-read shape of ExpertCache.prefetch,
    ExpertCache.swift:126-196); the routers come from model_weights.bin.
    Unlike the reference, which keeps going with zeroed weights after a short
    read (InferenceEngine.swift:274-279), a missing or wrong-sized file raises
    before anything is copied."""
    check_layer_files(model_dir, spec)
    store = WeightStore(model_dir)
    try:
        block.load_expert_files(Path(model_dir) / "packed_experts", io_threads=io_threads)
        for L in range(spec.num_layers):
            block.load_router(L, store.tensor(spec.router_key(L)))
    finally:
        store.close()
