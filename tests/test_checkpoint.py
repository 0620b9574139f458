"""The int8 checkpoint's file layer on CPU: write -> read round trip, and the validation
that refuses files which do not describe a consistent set of Llama projections."""

from __future__ import annotations

import pytest
import torch

from llm_serving_engine_b200.checkpoint import FORMAT, read_int8_checkpoint, write_int8_checkpoint

H, I, SIZES, LAYERS = 64, 96, (64, 32, 32), 2


def _tensors(seed: int = 0) -> tuple[dict[str, torch.Tensor], dict[str, str]]:
    g = torch.Generator().manual_seed(seed)
    shapes = {"self_attn.qkv_proj": (sum(SIZES), H), "self_attn.o_proj": (H, SIZES[0]),
              "mlp.gate_up_proj": (2 * I, H), "mlp.down_proj": (H, I)}
    t = {}
    for i in range(LAYERS):
        for p, (n, k) in shapes.items():
            t[f"model.layers.{i}.{p}.qweight"] = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
            t[f"model.layers.{i}.{p}.scale"] = torch.rand(n, generator=g) * 1e-3
    meta = {"num_layers": str(LAYERS), "qkv_sizes": ",".join(map(str, SIZES)), "intermediate_size": str(I)}
    return t, meta


def test_round_trip_is_bit_exact(tmp_path):
    t, meta = _tensors()
    path = str(tmp_path / "ckpt.safetensors")
    write_int8_checkpoint(path, t, meta)
    back, m2 = read_int8_checkpoint(path)
    assert m2["format"] == FORMAT and m2["num_layers"] == str(LAYERS)
    assert set(back) == set(t)
    for k in t:
        assert back[k].dtype == t[k].dtype and torch.equal(back[k], t[k]), k


@pytest.mark.parametrize("breakage", ["missing", "dtype", "rows", "chain", "meta"])
def test_inconsistent_checkpoints_are_refused(tmp_path, breakage):
    t, meta = _tensors(1)
    if breakage == "missing":
        del t["model.layers.1.mlp.down_proj.scale"]
    elif breakage == "dtype":
        t["model.layers.0.self_attn.o_proj.qweight"] = t["model.layers.0.self_attn.o_proj.qweight"].float()
    elif breakage == "rows":
        meta["intermediate_size"] = str(I + 8)
    elif breakage == "chain":
        t["model.layers.0.mlp.down_proj.qweight"] = torch.zeros(H, I + 8, dtype=torch.int8)
    elif breakage == "meta":
        meta["qkv_sizes"] = "64,32"
    with pytest.raises(ValueError):
        write_int8_checkpoint(str(tmp_path / "bad.safetensors"), t, meta)


def test_foreign_file_is_refused(tmp_path):
    from safetensors.torch import save_file

    path = str(tmp_path / "other.safetensors")
    save_file({"w": torch.zeros(2, 2)}, path, metadata={"format": "pt"})
    with pytest.raises(ValueError):
        read_int8_checkpoint(path)
