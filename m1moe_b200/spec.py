"""Model configuration: the reference's ModelSpec JSON schema, read unchanged.

Mirrors Sources/M1MoE/ModelSpec.swift:11-158 (snake_case JSON keys decoded with
.convertFromSnakeCase, :56-61), including the derived expertBytes4Bit
(:36-52) and the expert block byte offsets of InferenceEngine.swift:79-97.
Only the fields the MoE hot path reads are typed; the rest stay available in
`raw`.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path


@dataclass(frozen=True)
class MoESpec:
    num_experts: int
    top_k: int
    intermediate_dim: int
    norm_topk_prob: bool


@dataclass(frozen=True)
class QuantSpec:
    bits: int
    group_size: int


@dataclass(frozen=True)
class ModelSpec:
    name: str
    architecture: str
    hidden_dim: int
    vocab_size: int
    num_layers: int
    rms_norm_eps: float
    moe: MoESpec
    quantization: QuantSpec
    model_dir: str | None = None
    raw: dict = field(default_factory=dict, compare=False, repr=False)

    @staticmethod
    def load(path: str | Path) -> "ModelSpec":
        return ModelSpec.from_dict(json.loads(Path(path).read_text()))

    @staticmethod
    def from_dict(d: dict) -> "ModelSpec":
        m, q = d["moe"], d["quantization"]
        if int(q["bits"]) != 4:
            raise ValueError(f"only 4-bit expert quantisation exists in this format, got {q['bits']}")
        return ModelSpec(
            name=d["name"], architecture=d["architecture"], hidden_dim=int(d["hidden_dim"]),
            vocab_size=int(d["vocab_size"]), num_layers=int(d["num_layers"]),
            rms_norm_eps=float(d["rms_norm_eps"]),
            moe=MoESpec(int(m["num_experts"]), int(m["top_k"]), int(m["intermediate_dim"]),
                        bool(m["norm_topk_prob"])),
            quantization=QuantSpec(int(q["bits"]), int(q["group_size"])),
            model_dir=d.get("model_dir"), raw=d)

    @property
    def expert_bytes_4bit(self) -> int:
        """ModelSpec.expertBytes4Bit (ModelSpec.swift:36-52)."""
        return expert_bytes(self.hidden_dim, self.moe.intermediate_dim, self.quantization.group_size)

    def router_key(self, layer: int) -> str:
        """Router tensor name in model_weights.json (InferenceEngine.swift:593-598)."""
        if self.architecture == "mixtral":
            return f"model.layers.{layer}.block_sparse_moe.gate.weight"
        return f"model.layers.{layer}.mlp.gate.weight"


def expert_bytes(hidden: int, inter: int, gs: int) -> int:
    gw, gsb = inter * (hidden // 8) * 4, inter * (hidden // gs) * 2
    dw, dsb = hidden * (inter // 8) * 4, hidden * (inter // gs) * 2
    return (gw + 2 * gsb) * 2 + dw + 2 * dsb


def expert_offsets(hidden: int, inter: int, gs: int) -> dict[str, int]:
    """Byte offsets inside one expert block (InferenceEngine.swift:79-97)."""
    gw, gsb = inter * (hidden // 8) * 4, inter * (hidden // gs) * 2
    dw, dsb = hidden * (inter // 8) * 4, hidden * (inter // gs) * 2
    o = {"gate_w": 0}
    o["gate_s"] = o["gate_w"] + gw
    o["gate_b"] = o["gate_s"] + gsb
    o["up_w"] = o["gate_b"] + gsb
    o["up_s"] = o["up_w"] + gw
    o["up_b"] = o["up_s"] + gsb
    o["down_w"] = o["up_b"] + gsb
    o["down_s"] = o["down_w"] + dw
    o["down_b"] = o["down_s"] + dsb
    return o


# The reference's two shipped configs (configs/olmoe-1b-7b.json,
# configs/mixtral-8x7b.json), restated for the fields the hot path uses.
OLMOE_1B_7B = ModelSpec("OLMoE-1B-7B-0924", "olmoe", 2048, 50304, 16, 1e-5,
                        MoESpec(64, 8, 1024, False), QuantSpec(4, 64))
MIXTRAL_8X7B = ModelSpec("Mixtral-8x7B-Instruct-v0.1", "mixtral", 4096, 32000, 32, 1e-5,
                         MoESpec(8, 2, 14336, False), QuantSpec(4, 64))
