"""HiSQ per-linear input rotation: derivation of signs and permutation (host side).

Mirrors ``derive_hisq_rotation`` (``src/faquant/hisq_rotation.py:23-47``) and the
Qwen variant tables it is called with (``derive_qwen_hisq_rotation
hisq_rotation.py:170-212``, ``restrict_hisq_rotation :156-167``,
``hisq_rotation_source :125-150``). The derivation is offline, once per layer:
the layer key ``f"{seed}::{name}"`` is hashed with SHA-256, its first eight bytes
(little endian) modulo ``2^31 - 1`` seed torch's CPU generator, and the generator
draws ``randint(0, 2, (n,))`` for the signs and then ``randperm(n)`` for the
permutation. The generator must be torch's, on the host, for the signs and
permutation to equal the ones the reference folded into its weights; the
device kernels only consume the resulting ``int8`` signs and ``int64``
permutation.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HiSQRotation:
    signs: torch.Tensor  # int8 [n], +-1
    permutation: torch.Tensor  # int64 [n]
    block_size: int
    layer_seed: int


def _layer_seed(name: str, seed: int) -> int:
    digest = hashlib.sha256(f"{seed}::{name}".encode("utf-8")).digest()
    return int.from_bytes(digest[:8], "little") % (2**31 - 1)


def derive_hisq_rotation(
    layer_name: str,
    in_features: int,
    *,
    seed: int = 17,
    block_size: int = 1024,
    device: torch.device | str = "cpu",
) -> HiSQRotation:
    """Signs, permutation and block size of one linear's ``diag(s) P H_block`` rotation."""
    if block_size <= 0 or block_size & (block_size - 1):
        raise ValueError("HiSQ rotation block_size must be a positive power of two")
    if in_features % block_size:
        raise ValueError(f"in_features={in_features} is not divisible by block_size={block_size}")
    layer_seed = _layer_seed(layer_name, seed)
    generator = torch.Generator(device="cpu").manual_seed(layer_seed)
    signs = torch.randint(0, 2, (in_features,), generator=generator, dtype=torch.int64)
    signs = (signs * 2 - 1).to(device=device, dtype=torch.int8)
    permutation = torch.randperm(in_features, generator=generator, dtype=torch.int64).to(device=device)
    return HiSQRotation(signs, permutation, block_size, layer_seed)


def restrict_hisq_rotation(rotation: HiSQRotation, construction: str) -> HiSQRotation:
    """``full`` keeps everything, ``signs`` drops the permutation, ``plain`` the signs too."""
    if construction == "full":
        return rotation
    if construction not in ("signs", "plain"):
        raise ValueError(f"unknown HiSQ construction {construction!r}")
    identity = torch.arange(rotation.permutation.numel(), device=rotation.permutation.device)
    signs = rotation.signs if construction == "signs" else torch.ones_like(rotation.signs)
    return HiSQRotation(signs, identity, rotation.block_size, rotation.layer_seed)


def hisq_rotation_source(layer_name: str, sharing: str, *, seed: int, global_seed: int) -> tuple[str, int]:
    """Key and seed a projection's rotation is derived from under a sharing mode."""
    if sharing not in ("linear", "norm", "global"):
        raise ValueError(f"unknown HiSQ rotation sharing {sharing!r}")
    parent, _, projection = layer_name.rpartition(".")
    if sharing == "linear" or projection in ("o_proj", "down_proj"):
        return layer_name, seed
    if sharing == "global":
        return "global_residual", global_seed
    if projection in ("q_proj", "k_proj", "v_proj"):
        norm = "input_layernorm"
    elif projection in ("gate_proj", "up_proj"):
        norm = "post_attention_layernorm"
    else:
        raise ValueError(f"{layer_name} reads no RMSNorm a rotation could be keyed by")
    return f"{parent.rpartition('.')[0]}.{norm}", seed
