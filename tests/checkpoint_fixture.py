"""A synthetic step-0 QAD checkpoint for the loader tests: HiF4-grid bf16 weights with
the compact metadata the oracle fits from their source (the layout of
qad_checkpoint.py:43-48, hif4.py:68-79), in two safetensors shards with an index and a
qad_init.json receipt."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from oracle import hif4 as oh

LINEARS = {"layers.0.q_proj": (256, 512), "layers.0.o_proj": (512, 256)}  # name -> (out, in)


def grid_weight(n: int, k: int, seed: int) -> tuple[np.ndarray, dict[str, np.ndarray]]:
    """A source weight's HiF4 grid values and the metadata fitted from the source."""
    src = (np.random.default_rng(seed).standard_normal((n, k)) * 0.02).astype(np.float32)
    src = oh.bf16_round(src)
    compact = oh.fit_compact(src.reshape(n, k // 64, 64), "123")
    return oh.fake_quantize(src, "123"), compact


def write_checkpoint(root: Path, *, levels: str = "123", corrupt_lv2: bool = False) -> dict[str, np.ndarray]:
    """Writes the checkpoint under ``root``; returns the grid weights by module name."""
    from safetensors.torch import save_file

    root.mkdir(parents=True, exist_ok=True)
    weights, shards = {}, [{}, {}]
    for i, (name, (n, k)) in enumerate(LINEARS.items()):
        w, c = grid_weight(n, k, seed=i)
        weights[name] = w
        g = k // 64
        lv2 = c["lv2"].copy()
        if corrupt_lv2 and i == 0:
            lv2[0, 0, 0] ^= 1  # one sub-block exponent flipped: its 8 values leave the grid
        shard = shards[i]
        shard[f"{name}.weight"] = torch.from_numpy(w).to(torch.bfloat16)
        shard[f"{name}.weight_hif4_scale"] = torch.from_numpy(c["scale"].reshape(n, g, 1, 1, 1).copy())
        shard[f"{name}.weight_hif4_reciprocal"] = torch.from_numpy(c["reciprocal"].reshape(n, g, 1, 1, 1).copy())
        shard[f"{name}.weight_hif4_scale_lv2_exponent"] = torch.from_numpy(lv2.reshape(n, g, 8, 1, 1).copy())
        shard[f"{name}.weight_hif4_scale_lv3_exponent"] = torch.from_numpy(c["lv3"].reshape(n, g, 8, 2, 1).copy())
    shards[1]["norm.weight"] = torch.ones(512, dtype=torch.bfloat16)  # a tensor that is not quantized
    weight_map = {}
    for j, shard in enumerate(shards):
        fname = f"model-{j + 1:05d}-of-00002.safetensors"
        save_file(shard, str(root / fname))
        weight_map.update({key: fname for key in shard})
    (root / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
    (root / "qad_init.json").write_text(json.dumps({"hif4_scale_levels": levels, "hif4_act_scale_levels": levels}))
    return weights
