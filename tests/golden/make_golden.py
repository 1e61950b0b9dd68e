"""Generate the golden fixtures in this directory from the reference itself.

Run in a checkout that has the reference FAQUANT sources available (set
``FAQUANT_REFERENCE_SRC`` to its ``src`` directory)::

    FAQUANT_REFERENCE_SRC=/path/to/FAQUANT-Public/src python tests/golden/make_golden.py

Every fixture is produced by calling the reference's own functions on seeded
inputs (torch CPU generator). Inputs that are cheap to regenerate are not
stored: the fixture keeps the seed and a SHA-256 of the input bytes, and the
tests regenerate the input with the same torch generator and check the hash.

Fixtures (all ``.npz``):

- ``hif4_golden``: the upstream GCC-HiFloat golden vector of the reference test
  ``tests/test_quantization.py:51-74``, read from that file as text, checked
  against ``faquant.hif4.fake_quantize_hif4`` and stored with its outputs;
- ``hif4_random``: ``fake_quantize_hif4`` and ``fit_hif4_compact_parameters``
  for the three level variants on rows with outliers, zero blocks, tiny and huge
  values and a ragged tail;
- ``rotation``: ``derive_hisq_rotation`` for the BASELINE configurations;
- ``linear_*``: ``FakeQuantLinear`` forwards (``rbh_r64``-style block 64 and HiSQ
  block 1024; three-level and, in a child process, two-level scales);
- ``attention_*``: ``simulated_flash_attention_forward`` with HiF4 operands;
- ``qk_prep``: the post-RoPE Q/K transform of ``qwen3._attention_forward``;
- ``gptq``: a GPTQ HiF4 weight with its compact metadata; ``gptq_cases``: two larger
  layers at the deployed GPTQ settings (full Hessian, and block-diagonal);
- ``config1_attention``: BASELINE config 1's attention in full (B=1, 32/8 heads,
  S=2048, causal, post-RoPE Hadamard, HiF4 Q/K/P/V, P-Reordering) through
  ``simulated_flash_attention_forward``: sampled query rows of the output, the sum over
  head_dim of every (query, head) and the simulator's geometry counters;
- ``config1_linear`` (two-level, in a child process): BASELINE config 1's QuantLinear in
  full (X [2048, 4096] with 8 outlier channels, W [4096, 4096], ``rbh_r64`` reader
  rotation, RTN): the weight grid's SHA-256, sampled output rows and every row's sum;
- ``c2_projection``: a config-2 projection (q_proj, HiSQ1024 seed 17, three-level) on
  512 tokens, the same quantities.

``wan_triton.npz`` comes from ``make_triton_golden.py`` instead: the reference's Triton
kernel needs a GPU, so that script runs on a GPU box.

Every sampled fixture stores rows picked at the start, the middle and the end of the
tensor plus a regular stride, and a per-row sum of the whole tensor, so a test compares
all rows through their sums and the sampled rows value by value.
"""

from __future__ import annotations

import ast
import json
import math
import os
import re
import subprocess
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
if not os.environ.get("FAQUANT_REFERENCE_SRC"):
    raise SystemExit("set FAQUANT_REFERENCE_SRC to the reference checkout's src directory")
REF_SRC = Path(os.environ["FAQUANT_REFERENCE_SRC"])
sys.path.insert(0, str(REF_SRC))
sys.path.insert(0, str(HERE))

from inputs import (  # noqa: E402
    ATTENTION_CASES,
    LINEAR_CASES,
    attention_inputs,
    c2_projection_inputs,
    config1_linear_inputs,
    linear_inputs,
    outlier_rows,
    sha,
    special_rows,
)


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def save(name: str, **arrays) -> None:
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(f"wrote {name}.npz ({(HERE / f'{name}.npz').stat().st_size} bytes)")


# ---------------------------------------------------------------- fixtures
def make_hif4_golden() -> None:
    from faquant.quantization import fake_quantize

    text = (REF_SRC.parent / "tests" / "test_quantization.py").read_text()
    match = re.search(r"expected_values = (\[.*?\])", text, re.S)
    expected = [float(v) for v in ast.literal_eval(match.group(1))]
    x32 = torch.linspace(-17.25, 18.75, 70, dtype=torch.float32)
    out32 = fake_quantize(x32, quant_format="hif4", bits=4, group_size=64)
    xb = x32.to(torch.bfloat16)
    outb = fake_quantize(xb, quant_format="hif4", bits=4, group_size=64)
    exp32 = torch.tensor(expected, dtype=torch.float32)
    expb_list = list(expected)
    expb_list[2] = -17.5  # the reference test's bf16 adjustment (test_quantization.py:68-69)
    expb = torch.tensor(expb_list, dtype=torch.bfloat16)
    assert torch.equal(out32, exp32) and torch.equal(out32.view(torch.int32), exp32.view(torch.int32))
    assert torch.equal(outb.view(torch.int16), expb.view(torch.int16))
    save(
        "hif4_golden",
        x_f32=x32.numpy(),
        x_bf16=bits(xb),
        upstream_f32=exp32.numpy(),
        upstream_bf16=bits(expb),
        ref_f32=out32.numpy(),
        ref_bf16=bits(outb),
    )


def make_hif4_random() -> None:
    from faquant.hif4 import _group_for_hif4, fake_quantize_hif4, fit_hif4_compact_parameters

    rnd = outlier_rows(8, 320, seed=11, outliers=6)
    spec = special_rows()
    arrays = {"random_x": rnd.numpy(), "special_x": spec.numpy()}
    for name, x in (("random", rnd), ("special", spec)):
        for levels in ("123", "12", "13"):
            arrays[f"{name}_f32_{levels}"] = fake_quantize_hif4(x, levels=levels).numpy()
            xb = x.to(torch.bfloat16)
            arrays[f"{name}_bf16_{levels}"] = bits(fake_quantize_hif4(xb, levels=levels))
            grouped, _ = _group_for_hif4(x, what="fixture")
            compact = fit_hif4_compact_parameters(grouped, levels=levels)
            arrays[f"{name}_scale_{levels}"] = compact.scale.reshape(x.shape[0], -1).numpy()
            arrays[f"{name}_rec_{levels}"] = compact.reciprocal.reshape(x.shape[0], -1).numpy()
            arrays[f"{name}_lv2_{levels}"] = compact.scale_lv2_exponent.reshape(x.shape[0], -1, 8).numpy()
            arrays[f"{name}_lv3_{levels}"] = compact.scale_lv3_exponent.reshape(x.shape[0], -1, 16).numpy()
    save("hif4_random", **arrays)


ROTATIONS = [
    # (name, in_features, seed, block)
    ("global_residual", 4096, 0, 64),  # config 1: rbh_r64 reader rotation
    ("model.layers.0.self_attn.q_proj", 4096, 17, 1024),  # config 2: HiSQ1024 per linear
    ("model.layers.0.self_attn.k_proj", 4096, 17, 1024),
    ("model.layers.0.self_attn.v_proj", 4096, 17, 1024),
    ("model.layers.0.self_attn.o_proj", 4096, 17, 1024),
    ("model.layers.0.mlp.gate_proj", 4096, 17, 1024),
    ("model.layers.0.mlp.up_proj", 4096, 17, 1024),
    ("model.layers.0.mlp.down_proj", 12288, 17, 1024),
    ("model.layers.0.input_layernorm", 5120, 17, 64),  # rbhn_r64-style reader (Wan width)
]


def make_rotation() -> None:
    from faquant.hisq_rotation import derive_hisq_rotation

    arrays = {}
    meta = []
    for i, (name, n, seed, block) in enumerate(ROTATIONS):
        rot = derive_hisq_rotation(name, n, seed=seed, block_size=block)
        meta.append({"name": name, "in_features": n, "seed": seed, "block": block,
                     "layer_seed": rot.layer_seed, "signs_sha": sha(rot.signs), "perm_sha": sha(rot.permutation)})
        if i == 0:
            arrays["c1_signs"] = rot.signs.numpy()
            arrays["c1_perm"] = rot.permutation.numpy().astype(np.int32)
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    save("rotation", **arrays)


def make_linear(levels: str) -> None:
    """Must run in a process whose FAQUANT_HIF4_SCALE_LEVELS equals ``levels``."""
    from faquant.hif4 import HIF4_ACT_SCALE_LEVELS, HIF4_SCALE_LEVELS
    from faquant.hisq_rotation import derive_hisq_rotation
    from faquant.quantization import FakeQuantLinear, fake_quantize
    from faquant.rotation import chunked_block_hadamard_transform

    assert HIF4_SCALE_LEVELS == levels and HIF4_ACT_SCALE_LEVELS == levels
    arrays = {}
    for tag, rows, fin, fout, block, seed, rname, rseed in LINEAR_CASES:
        x, w, b = linear_inputs(rows, fin, fout, seed)
        lin = torch.nn.Linear(fin, fout, bias=True)
        with torch.no_grad():
            lin.weight.copy_(w)
            lin.bias.copy_(b)
        lin = lin.to(torch.bfloat16)
        kwargs = {}
        if rname is not None:
            rot = derive_hisq_rotation(rname, fin, seed=rseed, block_size=block)
            kwargs = dict(input_rotation_signs=rot.signs, input_rotation_permutation=rot.permutation,
                          input_rotation_block_size=block)
            arrays[f"{tag}_rot_sha"] = np.array(sha(rot.signs) + sha(rot.permutation))
        mod = FakeQuantLinear(lin, quant_format="hif4", bits=4, weight_group_size=64,
                              activation_group_size=64, symmetric=True, clip_ratio=1.0, **kwargs)
        with torch.no_grad():
            y = mod(x)
            # the activation operand F.linear sees, recomputed with the reference's own functions
            if rname is not None:
                work = x.float() * rot.signs.float()
                work = work.index_select(-1, rot.permutation)
                work = chunked_block_hadamard_transform(work, block_size=block, chunk_rows=256).to(x.dtype)
            else:
                work = x
            xq = fake_quantize(work, quant_format="hif4", bits=4, group_size=64)
        arrays[f"{tag}_in_sha"] = np.array(sha(x) + sha(w) + sha(b))
        arrays[f"{tag}_wq"] = bits(mod.weight.detach())
        arrays[f"{tag}_xq"] = bits(xq)
        arrays[f"{tag}_y"] = bits(y)
        arrays[f"{tag}_block"] = np.array(-1 if block is None else block)
    save(f"linear_{levels}", **arrays)


def _sim_module(causal: bool, normalizer: str, qk: bool, pv: bool) -> SimpleNamespace:
    from faquant.simulated_flash_attention import new_simulated_attention_stats

    return SimpleNamespace(
        is_causal=causal,
        training=False,
        faquant_attention_query_chunk_size=256,
        faquant_attention_key_chunk_size=128,
        faquant_qk_matmul_quant=qk,
        faquant_pv_matmul_quant=pv,
        faquant_pv_normalizer_mode=normalizer,
        faquant_matmul_quant_kwargs={"quant_format": "hif4", "bits": 4, "group_size": 64,
                                     "symmetric": True, "clip_ratio": 1.0},
        faquant_simulated_attention_stats=new_simulated_attention_stats(),
    )


def make_attention() -> None:
    from faquant.simulated_flash_attention import simulated_flash_attention_forward

    arrays = {}
    for tag, b, h, kv, sq, sk, causal, normalizer, qk, pv, seed in ATTENTION_CASES:
        q, k, v = attention_inputs(b, h, kv, sq, sk, seed)
        module = _sim_module(causal, normalizer, qk, pv)
        with torch.no_grad():
            out, _ = simulated_flash_attention_forward(module, q, k, v, None, scaling=128**-0.5)
        arrays[f"{tag}_in_sha"] = np.array(sha(q) + sha(k) + sha(v))
        arrays[f"{tag}_out"] = bits(out)
        arrays[f"{tag}_stats"] = np.frombuffer(json.dumps(module.faquant_simulated_attention_stats).encode(), np.uint8)
    save("attention", **arrays)


def make_qk_prep() -> None:
    from faquant.rotation import hadamard_transform

    g = torch.Generator().manual_seed(41)
    q = (torch.randn(1, 4, 33, 128, generator=g) * 3).to(torch.bfloat16)
    k = (torch.randn(1, 2, 33, 128, generator=g) * 3).to(torch.bfloat16)
    scale = torch.exp(torch.empty(128).uniform_(math.log(0.5), math.log(2.0), generator=g))
    offset = torch.randn(2, 128, generator=g) * 0.5
    # qwen3._attention_forward (qwen3.py:101-130): one fp32 excursion, one bf16 cast
    qf, kf = q.float(), k.float()
    kf = kf - offset[:, None, :]
    qf = qf * scale
    kf = kf / scale
    qf, kf = hadamard_transform(qf), hadamard_transform(kf)
    save("qk_prep", q=bits(q), k=bits(k), scale=scale.numpy(), offset=offset.numpy(),
         q_out=bits(qf.to(torch.bfloat16)), k_out=bits(kf.to(torch.bfloat16)))


def make_gptq() -> None:
    from faquant.gptq import GPTQ

    torch.manual_seed(51)
    lin = torch.nn.Linear(256, 48, bias=False)
    with torch.no_grad():
        lin.weight.normal_(0.0, 0.02)
    gptq = GPTQ(lin)
    g = torch.Generator().manual_seed(52)
    gptq.add_batch(torch.randn(512, 256, generator=g))
    gptq.quantize(quant_format="hif4", bits=4, group_size=64, damp=0.01, block_size=128,
                  capture_hif4_metadata=True)
    meta = lin.faquant_hif4_qat_parameters
    save("gptq", w=bits(lin.weight.detach().to(torch.bfloat16)),
         scale=meta.scale.reshape(48, 4).numpy(), rec=meta.reciprocal.reshape(48, 4).numpy(),
         lv2=meta.scale_lv2_exponent.reshape(48, 4, 8).numpy(),
         lv3=meta.scale_lv3_exponent.reshape(48, 4, 16).numpy())


def sample_rows(n: int, edge: int, stride: int) -> np.ndarray:
    """Rows at the start, the middle and the end of an n-row tensor plus every stride-th."""
    mid = n // 2 - edge // 2
    rows = set(range(edge)) | set(range(mid, mid + edge)) | set(range(n - edge, n)) | set(range(0, n, stride))
    return np.array(sorted(rows), dtype=np.int64)


def make_config1_attention() -> None:
    from faquant.rotation import hadamard_transform
    from faquant.simulated_flash_attention import simulated_flash_attention_forward

    b, h, kv, s, d = 1, 32, 8, 2048, 128
    q, k, v = attention_inputs(b, h, kv, s, s, seed=0)
    # qwen3._attention_forward (qwen3.py:113-130): fp32 Hadamard over head_dim, one bf16 cast
    qh = hadamard_transform(q.float()).to(torch.bfloat16)
    kh = hadamard_transform(k.float()).to(torch.bfloat16)
    module = _sim_module(True, "quantized_same", True, True)
    with torch.no_grad():
        out, _ = simulated_flash_attention_forward(module, qh, kh, v, None, scaling=d**-0.5)
    rows = sample_rows(s, 64, 32)
    save("config1_attention", in_sha=np.array(sha(q) + sha(k) + sha(v)), rows=rows,
         out_rows=bits(out[0, rows]), head_sums=out[0].float().sum(dim=-1).numpy(),
         stats=np.frombuffer(json.dumps(module.faquant_simulated_attention_stats).encode(), np.uint8))


def _linear_fixture(name: str, x: torch.Tensor, w: torch.Tensor, rot, block: int, levels: str) -> None:
    from faquant.hif4 import HIF4_ACT_SCALE_LEVELS, HIF4_SCALE_LEVELS
    from faquant.quantization import FakeQuantLinear

    assert HIF4_SCALE_LEVELS == levels and HIF4_ACT_SCALE_LEVELS == levels
    lin = torch.nn.Linear(w.shape[1], w.shape[0], bias=False).to(torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(w)
    mod = FakeQuantLinear(lin, quant_format="hif4", bits=4, weight_group_size=64, activation_group_size=64,
                          symmetric=True, clip_ratio=1.0, input_rotation_signs=rot.signs,
                          input_rotation_permutation=rot.permutation, input_rotation_block_size=block)
    with torch.no_grad():
        y = mod(x)
    rows = sample_rows(x.shape[0], 16, max(1, x.shape[0] // 32))
    save(name, in_sha=np.array(sha(x) + sha(w)), rot_sha=np.array(sha(rot.signs) + sha(rot.permutation)),
         wq_sha=np.array(sha(mod.weight.detach())), rows=rows, y_rows=bits(y[rows]),
         row_sums=y.double().sum(dim=1).numpy(), levels=np.array(levels))


def make_config1_linear(levels: str) -> None:
    """Must run in a process whose FAQUANT_HIF4_SCALE_LEVELS equals ``levels`` (12)."""
    from faquant.hisq_rotation import derive_hisq_rotation

    x, w = config1_linear_inputs()
    rot = derive_hisq_rotation("global_residual", 4096, seed=0, block_size=64)
    _linear_fixture("config1_linear", x, w, rot, 64, levels)


def make_c2_projection(levels: str) -> None:
    from faquant.hisq_rotation import derive_hisq_rotation

    x, w = c2_projection_inputs()
    rot = derive_hisq_rotation("model.layers.0.self_attn.q_proj", 4096, seed=17, block_size=1024)
    _linear_fixture("c2_projection", x, w, rot, 1024, levels)


def make_gptq_cases() -> None:
    """GPTQ at the deployed settings (gptq.py:324-593, GPTQ_SETTINGS of
    workflows/wan22_gptq.py:58) on two larger layers: the full-Hessian solver (256 x 1024,
    block 128, 4096 calibration rows with 1 % outlier channels) and the block-diagonal
    one (128 x 512, 64-column Hessian blocks). Stores the bf16 result and the metadata."""
    from faquant.gptq import GPTQ

    arrays = {}
    for tag, n, k, hblock, seed in (("full", 256, 1024, None, 61), ("blockdiag", 128, 512, 64, 62)):
        torch.manual_seed(seed)
        lin = torch.nn.Linear(k, n, bias=False)
        with torch.no_grad():
            lin.weight.normal_(0.0, 0.02)
        gp = GPTQ(lin, hessian_block_size=hblock)
        gp.add_batch(outlier_rows(4096, k, seed=seed + 1, outliers=max(1, k // 100)))
        gp.quantize(quant_format="hif4", bits=4, group_size=64, damp=0.01, block_size=128,
                    capture_hif4_metadata=True)
        meta = lin.faquant_hif4_qat_parameters
        g = k // 64
        arrays[f"{tag}_w"] = bits(lin.weight.detach().to(torch.bfloat16))
        arrays[f"{tag}_scale"] = meta.scale.reshape(n, g).numpy()
        arrays[f"{tag}_lv2"] = meta.scale_lv2_exponent.reshape(n, g, 8).numpy()
        arrays[f"{tag}_lv3"] = meta.scale_lv3_exponent.reshape(n, g, 16).numpy()
    save("gptq_cases", **arrays)


def main() -> None:
    if len(sys.argv) > 1 and sys.argv[1] == "--linear":
        make_linear(sys.argv[2])
        return
    if len(sys.argv) > 1 and sys.argv[1] == "--config1-linear":
        make_config1_linear(sys.argv[2])
        return
    if len(sys.argv) > 1 and sys.argv[1] == "--gptq":
        torch.set_num_threads(min(8, os.cpu_count() or 1))
        make_gptq_cases()
        return
    if len(sys.argv) > 1 and sys.argv[1] == "--baseline-sizes":
        # the BASELINE-size fixtures alone (the others are unchanged by them)
        torch.set_num_threads(min(8, os.cpu_count() or 1))
        make_config1_attention()
        make_c2_projection("123")
        env = dict(os.environ, FAQUANT_HIF4_SCALE_LEVELS="12")
        env.pop("FAQUANT_HIF4_ACT_SCALE_LEVELS", None)
        subprocess.run([sys.executable, __file__, "--config1-linear", "12"], check=True, env=env)
        return
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    make_hif4_golden()
    make_hif4_random()
    make_rotation()
    make_attention()
    make_qk_prep()
    make_gptq()
    make_gptq_cases()
    for levels in ("123", "12"):
        env = dict(os.environ, FAQUANT_HIF4_SCALE_LEVELS=levels)
        env.pop("FAQUANT_HIF4_ACT_SCALE_LEVELS", None)
        subprocess.run([sys.executable, __file__, "--linear", levels], check=True, env=env)
    make_config1_attention()
    make_c2_projection("123")
    env = dict(os.environ, FAQUANT_HIF4_SCALE_LEVELS="12")
    env.pop("FAQUANT_HIF4_ACT_SCALE_LEVELS", None)
    subprocess.run([sys.executable, __file__, "--config1-linear", "12"], check=True, env=env)


if __name__ == "__main__":
    main()
