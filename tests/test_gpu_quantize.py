"""GPU parity of K1 (rotation + HiF4 quantization), K2 (weight packing) and the
dequantizer against the oracle and the reference fixtures: bit-exact."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from inputs import LINEAR_CASES, linear_inputs, outlier_rows, sha, special_rows
from oracle import hif4 as oh
from oracle import linear as olin

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ops():
    from faquant_b200 import ops

    return ops


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy().view(np.uint32)


def _oracle_bits(x: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    if dtype == torch.bfloat16:
        return oh.f32_to_bf16_bits(x)
    return np.asarray(x, np.float32).view(np.uint32)


def test_golden_vector_bit_exact() -> None:
    ops = _ops()
    g = load_golden("hif4_golden")
    x32 = torch.from_numpy(g["x_f32"]).to(DEV)
    q32, _, _ = ops.hif4_quantize(x32, levels="123")
    assert np.array_equal(_bits(q32), g["upstream_f32"].view(np.uint32))
    xb = torch.from_numpy(g["x_bf16"].view(np.int16)).view(torch.bfloat16).to(DEV)
    qb, _, _ = ops.hif4_quantize(xb, levels="123")
    assert np.array_equal(_bits(qb), g["upstream_bf16"])


@pytest.mark.parametrize("name", ["random", "special"])
@pytest.mark.parametrize("levels", ["123", "12", "13"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_reference_fixtures_and_codes(name: str, levels: str, dtype: torch.dtype) -> None:
    ops = _ops()
    g = load_golden("hif4_random")
    x = torch.from_numpy(g[f"{name}_x"]).to(dtype)
    qdq, codes, meta = ops.hif4_quantize(x.to(DEV), levels=levels, want_codes=True)
    ref = g[f"{name}_{'f32' if dtype == torch.float32 else 'bf16'}_{levels}"]
    assert np.array_equal(_bits(qdq), ref.view(np.uint32) if dtype == torch.float32 else ref)
    xo = x.float().numpy()
    ocodes, ometa = oh.hif4_encode(xo, levels)
    assert np.array_equal(codes.cpu().numpy(), ocodes)
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), ometa)
    back = ops.hif4_dequantize(codes, meta, x.shape[1], dtype=torch.float32)
    assert np.array_equal(_bits(back), oh.fake_quantize(xo, levels).view(np.uint32))


BLOCKS = [1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024]


@pytest.mark.parametrize("block", BLOCKS)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("kind", ["ragged", "aligned"])
def test_rotation_blocks_bit_exact(block: int, dtype: torch.dtype, kind: str) -> None:
    """Every block size through both kernels: rows with a ragged 64-tail (staged path)
    and rows of whole 64-blocks (the double-buffered bf16 path)."""
    ops = _ops()
    if kind == "aligned":
        k = 3072 if block <= 1024 and 3072 % block == 0 else 2048
    else:
        k = 2048 if block >= 64 else 64 * 5 + block
    k = k - k % block
    rng = np.random.default_rng(block)
    x = torch.from_numpy(rng.standard_normal((37, k)).astype(np.float32) * 3).to(dtype)
    x[:, rng.integers(0, k, 3)] *= 25
    signs = torch.from_numpy(rng.choice([-1, 1], k).astype(np.int8))
    perm = torch.from_numpy(rng.permutation(k).astype(np.int64))
    for levels in ("123", "12"):
        qdq, codes, meta = ops.hif4_quantize(x.to(DEV), levels=levels, signs=signs.to(DEV), permutation=perm.to(DEV),
                                             rot_block=block, want_codes=True)
        odt = "bf16" if dtype == torch.bfloat16 else "f32"
        expect = olin.quantize_activations(x.float().numpy(), levels=levels, dtype=odt, signs=signs.numpy(),
                                           permutation=perm.numpy(), block=block)
        assert np.array_equal(_bits(qdq), _oracle_bits(expect, dtype)), (block, levels)


@pytest.mark.parametrize("k,block", [(5120, 1024), (8192, 256), (12288, 1024), (16384, 512)])
def test_rotation_wide_rows_bit_exact(k: int, block: int) -> None:
    """The bf16 rotation kernel runs one warp per 1024 channels, so K = 5120 ... 16384
    launch its wider CTA classes; 333 rows give every CTA (one per SM at the widest) two
    or three rows, so both row buffers are refilled while other warps still work."""
    ops = _ops()
    rng = np.random.default_rng(k + block)
    x = torch.from_numpy(rng.standard_normal((333, k)).astype(np.float32) * 2).to(torch.bfloat16)
    x[:, rng.integers(0, k, 5)] *= 30
    x[3, :100] = 0.0
    signs = torch.from_numpy(rng.choice([-1, 1], k).astype(np.int8))
    perm = torch.from_numpy(rng.permutation(k).astype(np.int64))
    qdq, codes, meta = ops.hif4_quantize(x.to(DEV), levels="123", signs=signs.to(DEV), permutation=perm.to(DEV),
                                         rot_block=block, want_codes=True)
    rotated = olin.rotate_input(x.float().numpy(), signs.numpy(), perm.numpy(), block, "bf16")
    assert np.array_equal(_bits(qdq), oh.f32_to_bf16_bits(oh.fake_quantize(rotated, "123")))
    ocodes, ometa = oh.hif4_encode(rotated, "123")
    assert np.array_equal(codes.cpu().numpy(), ocodes)
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), ometa)


@pytest.mark.parametrize("k,block,rows", [(4096, 1024, 1), (4096, 64, 5), (12288, 1024, 3), (5120, 512, 16)])
def test_rotation_few_rows_bit_exact(k: int, block: int, rows: int) -> None:
    """A few rows (a decode step's activations: fewer rows than CTAs, each CTA building
    the whole permutation map for a row or two) give the bits of the oracle, codes and meta
    included."""
    ops = _ops()
    rng = np.random.default_rng(7 * k + rows)
    x = torch.from_numpy(rng.standard_normal((rows, k)).astype(np.float32) * 2).to(torch.bfloat16)
    x[:, rng.integers(0, k, 3)] *= 30
    signs = torch.from_numpy(rng.choice([-1, 1], k).astype(np.int8))
    perm = torch.from_numpy(rng.permutation(k).astype(np.int64))
    qdq, codes, meta = ops.hif4_quantize(x.to(DEV), levels="123", signs=signs.to(DEV), permutation=perm.to(DEV),
                                         rot_block=block, want_codes=True)
    rotated = olin.rotate_input(x.float().numpy(), signs.numpy(), perm.numpy(), block, "bf16")
    assert np.array_equal(_bits(qdq), oh.f32_to_bf16_bits(oh.fake_quantize(rotated, "123")))
    ocodes, ometa = oh.hif4_encode(rotated, "123")
    assert np.array_equal(codes.cpu().numpy(), ocodes)
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), ometa)


@pytest.mark.parametrize("block", [8, 16, 32, 64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_signs_only_rotation_streaming_bit_exact(block: int, dtype: torch.dtype) -> None:
    """Signs without a permutation (the "signs" construction of row-parallel shards): the
    streaming kernel, with and without an input scale, codes and meta included."""
    ops = _ops()
    rng = np.random.default_rng(100 + block)
    k = 25600 if block <= 256 and 25600 % block == 0 else 4096
    x = torch.from_numpy(rng.standard_normal((23, k)).astype(np.float32) * 2).to(dtype)
    x[:, rng.integers(0, k, 5)] *= 30
    signs = rng.choice([-1, 1], k).astype(np.int8)
    scale = torch.from_numpy(rng.uniform(0.5, 2.0, k).astype(np.float32)).to(dtype)
    odt = "bf16" if dtype == torch.bfloat16 else "f32"
    for levels, use_scale in (("123", False), ("12", True)):
        qdq, codes, meta = ops.hif4_quantize(x.to(DEV), levels=levels, signs=torch.from_numpy(signs).to(DEV),
                                             rot_block=block, want_codes=True,
                                             input_scale=scale.to(DEV) if use_scale else None)
        expect = olin.quantize_activations(x.float().numpy(), levels=levels, dtype=odt, signs=signs, block=block,
                                           input_scale=scale.float().numpy() if use_scale else None)
        assert np.array_equal(_bits(qdq), _oracle_bits(expect, dtype)), (block, levels)
        xs = x.float().numpy()
        if use_scale:
            xs = olin.round_to(xs * scale.float().numpy(), odt)
        ocodes, ometa = oh.hif4_encode(olin.rotate_input(xs, signs, np.arange(k), block, odt), levels)
        assert np.array_equal(codes.cpu().numpy(), ocodes) and np.array_equal(meta.cpu().numpy().view(np.uint32), ometa)


@pytest.mark.parametrize("levels", ["123", "12"])
@pytest.mark.parametrize("case", LINEAR_CASES, ids=[c[0] for c in LINEAR_CASES])
def test_linear_fixture_activations_bit_exact(levels: str, case) -> None:
    from faquant_b200.hisq_rotation import derive_hisq_rotation

    ops = _ops()
    g = load_golden(f"linear_{levels}")
    tag, rows, fin, fout, block, seed, rname, rseed = case
    x, w, b = linear_inputs(rows, fin, fout, seed)
    assert str(g[f"{tag}_in_sha"]) == sha(x) + sha(w) + sha(b)
    kwargs = {}
    if rname is not None:
        rot = derive_hisq_rotation(rname, fin, seed=rseed, block_size=block)
        kwargs = dict(signs=rot.signs.to(DEV), permutation=rot.permutation.to(DEV), rot_block=block)
    qdq, _, _ = ops.hif4_quantize(x.to(DEV), levels=levels, **kwargs)
    assert np.array_equal(_bits(qdq), g[f"{tag}_xq"])
    wq, _, _ = ops.hif4_quantize(w.to(DEV), levels=levels)
    assert np.array_equal(_bits(wq), g[f"{tag}_wq"])


def test_config1_activation_path_full_size() -> None:
    """X [2048, 4096] with outliers, rbh_r64 rotation, two-level scale."""
    from faquant_b200.hisq_rotation import derive_hisq_rotation

    ops = _ops()
    x = outlier_rows(2048, 4096, seed=0, outliers=8).to(torch.bfloat16)
    rot = derive_hisq_rotation("global_residual", 4096, seed=0, block_size=64)
    qdq, codes, meta = ops.hif4_quantize(x.to(DEV), levels="12", signs=rot.signs.to(DEV),
                                         permutation=rot.permutation.to(DEV), rot_block=64, want_codes=True)
    rotated = olin.rotate_input(x.float().numpy(), rot.signs.numpy(), rot.permutation.numpy(), 64, "bf16")
    expect = oh.fake_quantize(rotated, "12")
    assert np.array_equal(_bits(qdq), oh.f32_to_bf16_bits(expect))
    ocodes, ometa = oh.hif4_encode(rotated, "12")
    assert np.array_equal(codes.cpu().numpy(), ocodes)
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), ometa)


@pytest.mark.parametrize("levels", ["123", "12", "13"])
def test_scale_sweep_every_bf16_block_maximum(levels: str) -> None:
    """One 64-block per positive finite bf16 value v (subnormals to the largest), holding
    +-v and values below it: every E6M2 scale, reciprocal and lv2/lv3 decision the bf16
    grid can reach, both clamp ends included, bit-exact -- directly, and through the
    rotated bf16 path for the blocks whose 1024-point Hadamard cannot overflow."""
    ops = _ops()
    rng = np.random.default_rng(77)
    v = (np.arange(1, 0x7F80, dtype=np.uint32) << 16).view(np.float32)
    n = v.size
    blocks = rng.uniform(-1, 1, (n, 64)).astype(np.float32) * v[:, None]
    blocks[np.arange(n), rng.integers(0, 64, n)] = v * rng.choice([-1, 1], n).astype(np.float32)
    blocks = np.concatenate([blocks, np.zeros((-n % 16, 64), np.float32)])
    x = oh.bf16_round(blocks).reshape(-1, 1024)
    qdq, codes, meta = ops.hif4_quantize(torch.from_numpy(x).to(torch.bfloat16).to(DEV), levels=levels,
                                         want_codes=True)
    ocodes, ometa = oh.hif4_encode(x, levels)
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), ometa)
    assert np.array_equal(codes.cpu().numpy(), ocodes)
    assert np.array_equal(_bits(qdq), oh.f32_to_bf16_bits(oh.fake_quantize(x, levels)))
    q32, _, _ = ops.hif4_quantize(torch.from_numpy(x).to(DEV), levels=levels)
    assert np.array_equal(_bits(q32), oh.fake_quantize(x, levels).view(np.uint32))
    safe = x[np.abs(x).max(axis=1) < 1e30]
    signs = rng.choice([-1, 1], 1024).astype(np.int8)
    rq, _, _ = ops.hif4_quantize(torch.from_numpy(safe).to(torch.bfloat16).to(DEV), levels=levels,
                                 signs=torch.from_numpy(signs).to(DEV), rot_block=1024)
    expect = olin.quantize_activations(safe, levels=levels, dtype="bf16", signs=signs, block=1024)
    assert np.array_equal(_bits(rq), oh.f32_to_bf16_bits(expect))


def test_input_scale_strided_rows_and_empty() -> None:
    ops = _ops()
    rng = np.random.default_rng(5)
    base = torch.from_numpy(rng.standard_normal((20, 320)).astype(np.float32)).to(torch.bfloat16)
    x = base[:, :256]  # row stride 320 > k
    scale = torch.from_numpy(rng.uniform(0.5, 2.0, 256).astype(np.float32)).to(torch.bfloat16)
    signs = torch.from_numpy(rng.choice([-1, 1], 256).astype(np.int8))
    qdq, _, _ = ops.hif4_quantize(x.to(DEV), levels="123", input_scale=scale.to(DEV), signs=signs.to(DEV),
                                  rot_block=64)
    expect = olin.quantize_activations(x.float().numpy(), levels="123", input_scale=scale.float().numpy(),
                                       signs=signs.numpy(), block=64)
    assert np.array_equal(_bits(qdq), oh.f32_to_bf16_bits(expect))
    empty, _, _ = ops.hif4_quantize(torch.zeros(0, 64, device=DEV, dtype=torch.bfloat16))
    assert empty.shape == (0, 64)
    with pytest.raises(ValueError):
        ops.hif4_quantize(torch.zeros(3, 0, device=DEV))


def test_pack_rtn_and_gptq_weights() -> None:
    ops = _ops()
    g = load_golden("linear_123")
    tag, rows, fin, fout, block, seed, rname, rseed = LINEAR_CASES[0]
    _, w_src, _ = linear_inputs(rows, fin, fout, seed)
    wq = torch.from_numpy(g[f"{tag}_wq"].view(np.int16)).view(torch.bfloat16).to(DEV)
    # RTN: pack from the source weight; the packed form decodes to the reference's RTN weight
    codes, meta, changed = ops.hif4_pack_weight(w_src.to(DEV), levels="123")
    assert torch.equal(ops.hif4_dequantize(codes, meta, fin), wq)
    assert changed == int((w_src.to(DEV) != wq).sum())
    # GPTQ weight with its recorded metadata (gptq.py:562-570): exact, nothing changed
    gp = load_golden("gptq")
    w = torch.from_numpy(gp["w"].view(np.int16)).view(torch.bfloat16).to(DEV)
    scale, lv2, lv3 = (torch.from_numpy(gp[n]) for n in ("scale", "lv2", "lv3"))
    codes, meta, bad = ops.hif4_pack_weight(w, scale=scale, lv2=lv2, lv3=lv3)
    assert bad == 0
    assert torch.equal(ops.hif4_dequantize(codes, meta, w.shape[1]), w)
    # a weight off its recorded grid is reported
    off = w.clone()
    off[0, 0] = off[0, 0] * 1.01 + 1e-3
    _, _, bad = ops.hif4_pack_weight(off, scale=scale, lv2=lv2, lv3=lv3)
    assert bad >= 1
