"""The converted-model directory loader's host logic (CPU only).

A model directory is written from the fixtures the reference's converter
produced (tests/golden, make_golden.py): model_weights.{json,bin} and
packed_experts/layer_NN.bin.  load_model_dir must check every layer file's
size first -- the converter's own check, scripts/extract_olmoe.py:340-344 --
and raise naming a missing or wrong-sized file before anything is copied,
then hand the experts directory to the block's native loader and the routers
from the manifest to load_router.
"""
from __future__ import annotations

import numpy as np
import pytest

from m1moe_b200 import checkpoint, spec


def write_model_dir(g, root, name):
    L, E, h, I, gs, seed = (int(v) for v in g["meta"])
    (root / "packed_experts").mkdir(parents=True)
    (root / "model_weights.json").write_bytes(g["manifest_json"].tobytes())
    (root / "model_weights.bin").write_bytes(g["model_weights_bin"].tobytes())
    for layer in range(L):
        g[f"layer_{layer:02d}"].tofile(root / "packed_experts" / f"layer_{layer:02d}.bin")
    arch = "olmoe" if name.startswith("olmoe") else "mixtral"
    return spec.ModelSpec("t", arch, h, 1, L, 1e-5, spec.MoESpec(E, 2, I, False),
                          spec.QuantSpec(4, gs))


class FakeBlock:
    def __init__(self):
        self.calls = []

    def load_expert_files(self, path, io_threads=4):
        self.calls.append(("files", str(path), io_threads))

    def load_router(self, layer, r):
        self.calls.append(("router", layer, np.array(r)))


@pytest.mark.parametrize("name", ["olmoe_tiny", "mixtral_tiny"])
def test_load_model_dir_calls(golden, tmp_path, name):
    from golden.make_golden import router_weights
    g = golden(name)
    sp = write_model_dir(g, tmp_path, name)
    blk = FakeBlock()
    checkpoint.load_model_dir(blk, sp, tmp_path, io_threads=3)
    assert blk.calls[0] == ("files", str(tmp_path / "packed_experts"), 3)
    routers = router_weights(int(g["meta"][5]), sp.num_layers, sp.moe.num_experts, sp.hidden_dim)
    got = [c for c in blk.calls if c[0] == "router"]
    assert [c[1] for c in got] == list(range(sp.num_layers))
    for c, r in zip(got, routers):
        assert np.array_equal(c[2], r)


def test_truncated_layer_file_raises_before_any_copy(golden, tmp_path):
    g = golden("olmoe_tiny")
    sp = write_model_dir(g, tmp_path, "olmoe_tiny")
    p = tmp_path / "packed_experts" / "layer_01.bin"
    p.write_bytes(p.read_bytes()[:-16])
    blk = FakeBlock()
    with pytest.raises(ValueError, match="layer_01.bin: .* bytes, expected"):
        checkpoint.load_model_dir(blk, sp, tmp_path)
    assert blk.calls == []
    with pytest.raises(ValueError, match="expected"):
        checkpoint.read_layer(tmp_path, 1, sp)


def test_missing_layer_file_raises(golden, tmp_path):
    g = golden("mixtral_tiny")
    sp = write_model_dir(g, tmp_path, "mixtral_tiny")
    (tmp_path / "packed_experts" / "layer_00.bin").unlink()
    with pytest.raises(FileNotFoundError, match="layer_00.bin"):
        checkpoint.load_model_dir(FakeBlock(), sp, tmp_path)


def test_read_layer_returns_the_file_bytes(golden, tmp_path):
    g = golden("olmoe_tiny")
    sp = write_model_dir(g, tmp_path, "olmoe_tiny")
    for layer in range(sp.num_layers):
        assert np.array_equal(checkpoint.read_layer(tmp_path, layer, sp), g[f"layer_{layer:02d}"])
