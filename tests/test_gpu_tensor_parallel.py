"""GPU tests of the tensor-parallel prefill (configs 4 and 5 in their sharded form).

* Sharding is exact where it should be: column-parallel shards reproduce the unsharded
  projection bit for bit, and the shard-local quantized inputs of a row-parallel
  projection are, concatenated, bit-identical to the unsharded quantized input; only
  the partial-sum order differs (tolerance on the outputs).
* A small Qwen3 prefill and a small Wan2.2 block at TP 1, stage by stage: each stage's
  GPU output against the oracle (rotation + HiF4 quantization, HiF4 attention, fp32
  matmuls) applied to that stage's own GPU input. 4-bit quantization is discontinuous:
  a last-bit difference before a K1 can re-code a whole 64-block, so two implementations
  are only comparable one stage at a time (an end-to-end comparison through several
  quantized stages measures that amplification, not the kernels).
* With two or more GPUs, TP 2 over NCCL against TP 1 on the first layer.
"""

from __future__ import annotations

import dataclasses

import os
import socket

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import hif4 as oh
from oracle import linear as olin

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rel(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _bf16(x: np.ndarray) -> np.ndarray:
    return oh.bf16_round(np.asarray(x, np.float32))


def _qwen_cfg():
    from faquant_b200.tensor_parallel import Qwen3TPConfig

    return Qwen3TPConfig(hidden=512, layers=2, heads=8, kv_heads=2, head_dim=128, ffn=1024, vocab=1000,
                         bf16_layers=(1,), column_block=512)


def _wan_cfg():
    from faquant_b200.tensor_parallel import WanBlockConfig

    return WanBlockConfig(dim=512, heads=4, head_dim=128, ffn=1024, grid=(2, 6, 16))


def _qwen_full_width_cfg():
    """One Qwen3-32B layer at its full width (hidden 5120, 64/8 heads,
    FFN 25600); one layer and a small vocabulary keep the oracle's host work in seconds."""
    from faquant_b200.tensor_parallel import Qwen3TPConfig

    return Qwen3TPConfig(layers=1, vocab=1000, bf16_layers=())


def _wan_full_width_cfg():
    """A Wan2.2-A14B block at its full width (dim 5120, 40 heads, FFN
    13824) on a 1 x 4 x 64 latent grid (256 tokens)."""
    from faquant_b200.tensor_parallel import WanBlockConfig

    return WanBlockConfig(grid=(1, 4, 64))


QWEN_CASES = [("small", _qwen_cfg, 2, 192), ("config5_full_width", _qwen_full_width_cfg, 1, 256)]
WAN_CASES = [("small", _wan_cfg), ("config4_full_width", _wan_full_width_cfg)]


def test_shards_reproduce_the_unsharded_projection() -> None:
    from faquant_b200.tensor_parallel import TPGroup, TPHiF4Linear, column_rotation, random_weight, row_rotation

    x = torch.randn(300, 1024, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).to(DEV)
    w = random_weight((768, 1024), 5, DEV)
    rot = column_rotation("model.layers.0.self_attn.q_proj", 1024, seed=17, block=1024)
    y = TPHiF4Linear(w, rotation=rot, quantize=True)(x)
    cols = [TPHiF4Linear(w[r * 384:(r + 1) * 384], rotation=rot, quantize=True)(x) for r in range(2)]
    assert torch.equal(torch.cat(cols, dim=1), y)

    w2 = random_weight((512, 1024), 6, DEV)
    full = TPHiF4Linear(w2, rotation=row_rotation("m.o_proj", 1024, TPGroup(0, 1), seed=17), quantize=True)
    parts = [TPHiF4Linear(w2[:, r * 512:(r + 1) * 512], quantize=True,
                          rotation=row_rotation("m.o_proj", 1024, TPGroup(r, 2), seed=17)) for r in range(2)]
    xs = [x[:, r * 512:(r + 1) * 512] for r in range(2)]
    assert torch.equal(torch.cat([p.quantize_input(s) for p, s in zip(parts, xs)], dim=1), full.quantize_input(x))
    y1 = full(x).float()
    p0, p1 = parts[0](xs[0]), parts[1](xs[1])
    y2 = (p0 + p1).float()  # what the bf16 all-reduce adds
    # each partial and their sum round to bf16 once (<= 2^-9 relative each), the full
    # product once; the fp32 sums differ only in order
    bound = 2.0**-8 * (p0.float().abs() + p1.float().abs() + y1.abs()) + 1e-4 * y1.abs().max()
    assert torch.all((y2 - y1).abs() <= bound)


def _oracle_linear(h: np.ndarray, lin, quantize: bool) -> np.ndarray:
    """bf16(Xq @ Wq^T + b) with the oracle's rotation + HiF4 quantization of the input."""
    w = lin.weight.float().cpu().numpy()
    if quantize:
        r = lin.rotation
        h = olin.quantize_activations(
            h, levels=lin.levels, dtype="bf16",
            signs=None if r.signs is None else r.signs.cpu().numpy(),
            permutation=None if r.permutation is None else r.permutation.cpu().numpy(),
            block=r.block if r.signs is not None else None)
    y = h @ w.T
    if lin.bias is not None:
        y = y + lin.bias.float().cpu().numpy()
    return _bf16(y)


ATT_REL_FRO = 5e-3  # HiF4 attention kernel vs the oracle on identical operands
ATT_MAX_ABS = 6e-2


def _close_linear(got: np.ndarray, ref: np.ndarray) -> None:
    """bf16 output of a GEMM vs the fp32 oracle product rounded to bf16: the two fp32 sums
    differ only in order, so the bf16 results differ by at most an ulp or so."""
    assert np.all(np.abs(got - ref) <= 2.0**-7 * np.abs(ref) + 1e-3 * np.abs(ref).max())


def _close_attention(got: np.ndarray, ref: np.ndarray) -> None:
    err = got - ref
    assert _rel(got, ref) <= ATT_REL_FRO and float(np.abs(err).max()) <= ATT_MAX_ABS


def _traced(module):
    trace = {}

    def hook(stage, index, t):
        trace[(stage, index)] = t.detach().float().cpu()

    module.trace = hook
    return trace


def _within_ulp(got: np.ndarray, ref: np.ndarray) -> None:
    assert np.all(np.abs(got - ref) <= 2.0**-7 * np.abs(ref) + 1e-30)


def _mostly_equal(got: np.ndarray, ref: np.ndarray) -> None:
    """HiF4 operands after a reduction (RMSNorm) whose sum order differs from torch's: a
    one-ulp difference before K4 can move one 64-block's scale, so most -- not all --
    values agree."""
    assert np.mean(got == ref) >= 0.995 and _rel(got, ref) <= 2e-2


@pytest.mark.parametrize("case", QWEN_CASES, ids=[c[0] for c in QWEN_CASES])
def test_qwen3_prefill_stages_match_the_oracle(case) -> None:
    """Every stage of a prefill against the reference's torch glue and the oracle, each
    applied to that stage's own GPU input: the RMSNorms, the W4A4 projections (K1 +
    GEMM), the fused q/k norm + RoPE + Hadamard + HiF4 (K4), the HiF4 attention (K5),
    SwiGLU and the logits. Two shapes: a 2-layer model (one HiF4 layer, one bf16 layer)
    at a small width, and one Qwen3-32B layer at its full width."""
    from faquant_b200.tensor_parallel import (Qwen3TPPrefill, TPGroup, apply_rope, default_input_ids, rms_norm,
                                              rope_tables)

    _, make_cfg, batch, seq = case
    model = Qwen3TPPrefill(make_cfg(), TPGroup(), DEV)
    cfg, d = model.cfg, model.cfg.head_dim
    tr = _traced(model)
    ids = default_input_ids(batch, seq, cfg.vocab, DEV, seed=3)
    logits = model(ids).cpu().numpy()
    b, s = ids.shape
    cos, sin = rope_tables(s, d, cfg.rope_theta, torch.device("cpu"))
    bf = lambda t: t.to(torch.bfloat16)  # noqa: E731
    for i, L in enumerate(model.layers):
        quant = i not in cfg.bf16_layers
        _within_ulp(tr[("input_norm", i)].numpy(), rms_norm(bf(tr[("x", i)]), L.input_norm.cpu(), cfg.eps).float().numpy())
        qkv = tr[("qkv", i)]
        _close_linear(qkv.numpy(), _oracle_linear(tr[("input_norm", i)].numpy(), L.qkv, quant))
        nq, nk = L.heads * d, L.kv_heads * d
        for name, cols, heads, w in (("qd", slice(0, nq), L.heads, L.q_norm), ("kd", slice(nq, nq + nk), L.kv_heads,
                                                                               L.k_norm)):
            r = apply_rope(rms_norm(bf(qkv[:, cols]).view(b, s, heads, d), w.cpu(), cfg.eps), cos, sin)
            r = r.transpose(1, 2).float().numpy()
            _mostly_equal(tr[(name, i)].numpy(), oh.fake_quantize(oatt.qk_pretransform(r, r)[0], cfg.levels))
        v = qkv[:, nq + nk:].reshape(b, s, L.kv_heads, d).transpose(1, 2).numpy()
        assert np.array_equal(tr[("vd", i)].numpy(), oh.fake_quantize(v, cfg.levels))
        att = oatt.attention(tr[("qd", i)].numpy(), tr[("kd", i)].numpy(), tr[("vd", i)].numpy(), causal=True,
                             scale=d**-0.5, normalizer="quantized_same", operands_quantized=True)
        _close_attention(tr[("attention", i)].numpy(), att)
        _close_linear(tr[("o", i)].numpy(), _oracle_linear(tr[("attention", i)].reshape(b * s, nq).numpy(), L.o, quant))
        _within_ulp(tr[("post_norm", i)].numpy(),
                    rms_norm(bf(tr[("x_mid", i)]), L.post_norm.cpu(), cfg.eps).float().numpy())
        gu = tr[("gate_up", i)]
        _close_linear(gu.numpy(), _oracle_linear(tr[("post_norm", i)].numpy(), L.gate_up, quant))
        act = torch.nn.functional.silu(bf(gu[:, :L.ffn])) * bf(gu[:, L.ffn:])
        _within_ulp(tr[("act", i)].numpy(), act.float().numpy())
        _close_linear(tr[("down", i)].numpy(), _oracle_linear(tr[("act", i)].numpy(), L.down, quant))
    final = bf(tr[("final", len(model.layers))])
    ref = torch.nn.functional.linear(rms_norm(final, model.final_norm.cpu(), cfg.eps), model.lm_head.cpu())
    assert logits.shape == (batch, cfg.vocab) and _rel(logits, ref.float().numpy()) <= 1e-2


def test_residual_adds_in_the_gemm_epilogue_are_the_same_bits() -> None:
    """The o_proj / down_proj (Wan: o / ffn.2) residual adds run in the GEMM epilogue unless
    a trace hook needs the projections' own outputs; the fused forwards give the same bits
    as the separate bf16 adds."""
    from faquant_b200.tensor_parallel import Qwen3TPPrefill, TPGroup, WanBlockTP, default_input_ids

    # hidden 1024 also takes the RMSNorms into the qkv / gate_up input quantization
    # (faq_hif4_quantize_rms_norm needs k % 1024 == 0); hidden 512 keeps them separate
    for cfg in (_qwen_cfg(), dataclasses.replace(_qwen_cfg(), hidden=1024, column_block=1024)):
        model = Qwen3TPPrefill(cfg, TPGroup(), DEV)
        ids = default_input_ids(2, 192, model.cfg.vocab, DEV, seed=4)
        fused = model(ids)
        model.fuse_residual = False
        assert torch.equal(fused, model(ids)), cfg.hidden
    # dim 1024 also takes the LayerNorms into the qkv / ffn.0 input quantization
    for cfg in (_wan_cfg(), dataclasses.replace(_wan_cfg(), dim=1024, heads=8)):
        block = WanBlockTP(cfg, TPGroup(), DEV)
        x = torch.randn(block.cfg.seq, block.cfg.dim, generator=torch.Generator().manual_seed(5))
        x = x.to(torch.bfloat16).to(DEV)
        fused = block(x)
        block.fuse_residual = False
        assert torch.equal(fused, block(x)), cfg.dim


@pytest.mark.parametrize("case", WAN_CASES, ids=[c[0] for c in WAN_CASES])
def test_wan_block_stages_match_the_oracle(case) -> None:
    """Every stage of a Wan2.2 block at TP 1 against the reference's torch glue and the
    oracle: the LayerNorms, the W4A4 projections, the fused q/k RMSNorm over all heads +
    3-D RoPE (fp64) + Hadamard + HiF4 (K4), V's HiF4, the attention and the GELU; at a
    small width and at the full Wan2.2-A14B width."""
    from faquant_b200.tensor_parallel import TPGroup, WanBlockTP, apply_rope3d, wan_qk_norm

    block = WanBlockTP(case[1](), TPGroup(), DEV)
    cfg, d, hl = block.cfg, block.cfg.head_dim, block.h_local
    tr = _traced(block)
    x = torch.randn(cfg.seq, cfg.dim, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    y = block(x.to(DEV)).float().cpu().numpy()
    assert np.isfinite(y).all()
    seq, n = cfg.seq, hl * d
    bf = lambda t: t.to(torch.bfloat16)  # noqa: E731

    def layer_norm(t):
        return torch.nn.functional.layer_norm(bf(t).float(), (cfg.dim,), eps=cfg.eps).to(torch.bfloat16).float()

    _within_ulp(tr[("norm1", 0)].numpy(), layer_norm(x).numpy())
    qkv = tr[("qkv", 0)]
    _close_linear(qkv.numpy(), _oracle_linear(tr[("norm1", 0)].numpy(), block.qkv, True))
    cos, sin = block.cos.cpu(), block.sin.cpu()
    for name, lo, w in (("qd", 0, block.norm_q), ("kd", n, block.norm_k)):
        r = apply_rope3d(wan_qk_norm(qkv[:, lo:lo + n], w.cpu(), cfg.dim, cfg.eps).view(seq, hl, d), cos, sin)
        r = r.transpose(0, 1)[None].numpy()
        _mostly_equal(tr[(name, 0)].numpy(), oh.fake_quantize(oatt.qk_pretransform(r, r)[0], cfg.levels))
    v = qkv[:, 2 * n:].view(seq, hl, d).transpose(0, 1)[None].numpy()
    assert np.array_equal(tr[("vd", 0)].numpy(), oh.fake_quantize(v, cfg.levels))
    att = oatt.attention(tr[("qd", 0)].numpy(), tr[("kd", 0)].numpy(), tr[("vd", 0)].numpy(), causal=False,
                         scale=d**-0.5, normalizer="quantized_same", operands_quantized=True)
    _close_attention(tr[("attention", 0)].numpy(), att)
    _close_linear(tr[("o", 0)].numpy(), _oracle_linear(tr[("attention", 0)].reshape(seq, n).numpy(), block.o, True))
    _within_ulp(tr[("norm2", 0)].numpy(), layer_norm(tr[("x_mid", 0)]).numpy())
    _close_linear(tr[("ffn0", 0)].numpy(), _oracle_linear(tr[("norm2", 0)].numpy(), block.ffn0, True))
    act = bf(torch.nn.functional.gelu(tr[("ffn0", 0)], approximate="tanh")).float().numpy()
    got = tr[("act", 0)].numpy()
    # one bf16 ulp; the far negative tail, where 1 + tanh cancels, to an absolute 1e-5
    assert np.all(np.abs(got - act) <= 2.0**-7 * np.abs(act) + 1e-5)
    _close_linear(tr[("ffn2", 0)].numpy(), _oracle_linear(tr[("act", 0)].numpy(), block.ffn2, True))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_rank(rank: int, world: int, port: int, results) -> None:
    import torch.distributed as dist

    from faquant_b200.tensor_parallel import Qwen3TPPrefill, TPGroup, WanBlockTP, default_input_ids

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        tp = TPGroup(rank, world)
        model = Qwen3TPPrefill(_qwen_cfg(), tp, dev)
        tq = _traced(model)
        model(default_input_ids(2, 192, model.cfg.vocab, dev, seed=3))
        block = WanBlockTP(_wan_cfg(), tp, dev)
        tw = _traced(block)
        x = torch.randn(block.cfg.seq, block.cfg.dim, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
        block(x.to(dev))
        mine = {("qwen",) + k: v.numpy() for k, v in tq.items() if k[1] == 0 and k[0] in ("qkv", "attention", "o")}
        mine.update({("wan",) + k: v.numpy() for k, v in tw.items() if k[0] in ("qkv", "qd", "kd", "attention", "o")})
        # a row-parallel projection large enough for the chunked, overlapped all-reduce:
        # with two ranks each element sums two values, so it equals one whole all-reduce
        from faquant_b200.tensor_parallel import TPHiF4Linear, random_weight, row_rotation

        w = random_weight((768, 2048), 41, dev)[:, rank * 1024:(rank + 1) * 1024]
        lin = TPHiF4Linear(w, rotation=row_rotation("chunked.o_proj", 2048, tp, seed=17), quantize=True, reduce=tp)
        xr = torch.randn(5000, 2048, generator=torch.Generator().manual_seed(42)).to(torch.bfloat16)
        xr = xr[:, rank * 1024:(rank + 1) * 1024].contiguous().to(dev)
        chunked = lin(xr)
        lin.overlap_min_rows = 1 << 30
        mine["chunked_equal"] = bool(torch.equal(chunked, lin(xr)))
        # sequence parallel (norm + K1 on the row shard, packed codes all-gathered, outputs
        # reduce-scattered) against the all-reduce path: with two ranks every sum is of two
        # values, so the same bits. Width 1024 takes the fused-norm packed path; layer 1 of
        # the Qwen3 model is a bf16 layer (its normalized rows are gathered as bf16)
        from faquant_b200.tensor_parallel import Qwen3TPConfig, WanBlockConfig

        qc = Qwen3TPConfig(hidden=1024, layers=2, heads=8, kv_heads=2, head_dim=128, ffn=2048, vocab=1000,
                           bf16_layers=(1,), column_block=1024)
        m = Qwen3TPPrefill(qc, tp, dev)
        ids = default_input_ids(2, 256, qc.vocab, dev, seed=5)
        assert m.seq_layout(2, 256) is not None
        sp = m(ids)
        m.sequence_parallel = False
        mine["qwen_sp_equal"] = bool(torch.equal(sp, m(ids)))
        wc = WanBlockConfig(dim=1024, heads=8, head_dim=128, ffn=2048, grid=(2, 6, 16))
        wb = WanBlockTP(wc, tp, dev)
        wb.sp_chunks = 4  # the chunked collectives (the Qwen3 model runs the default single chunk)
        xw = torch.randn(wc.seq, wc.dim, generator=torch.Generator().manual_seed(19)).to(torch.bfloat16).to(dev)
        assert wb.seq_layout(wc.seq).chunks == 4 and m.seq_layout(2, 256).chunks == 1
        sp = wb(xw)
        wb.sequence_parallel = False
        mine["wan_sp_equal"] = bool(torch.equal(sp, wb(xw)))
        results[rank] = mine  # one assignment: a managed dict hands out copies of its values
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp2_over_nccl_matches_tp1() -> None:
    """TP 2 over NCCL against TP 1, first layer: the column-parallel projections and the
    attention of each rank are bit-identical slices of the TP 1 results (same quantized
    inputs, same kernels); the row-parallel o_proj after the all-reduce differs only by
    the order of its partial sums. (Later stages re-quantize those last-bit differences,
    so they are checked against the oracle stage by stage instead.) The sequence-parallel
    forwards of both models equal their all-reduce forwards bit for bit at TP 2."""
    import torch.multiprocessing as mp

    from faquant_b200.tensor_parallel import Qwen3TPPrefill, TPGroup, WanBlockTP, default_input_ids

    results = mp.Manager().dict()
    mp.spawn(_tp_rank, args=(2, _free_port(), results), nprocs=2, join=True)
    model = Qwen3TPPrefill(_qwen_cfg(), TPGroup(), DEV)
    tq = _traced(model)
    model(default_input_ids(2, 192, model.cfg.vocab, DEV, seed=3))
    block = WanBlockTP(_wan_cfg(), TPGroup(), DEV)
    tw = _traced(block)
    x = torch.randn(block.cfg.seq, block.cfg.dim, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    block(x.to(DEV))
    assert results[0]["chunked_equal"] and results[1]["chunked_equal"]
    for key in ("qwen_sp_equal", "wan_sp_equal"):
        assert results[0][key] and results[1][key], key
    for tag, tr, hq, hkv in (("qwen", tq, 8, 2), ("wan", tw, 4, 4)):
        d = 128
        qkv1 = tr[("qkv", 0)].numpy()
        att1 = tr[("attention", 0)].numpy()
        for r in range(2):
            got = results[r]
            nq, nk = hq // 2 * d, hkv // 2 * d
            q1 = qkv1[:, r * nq:(r + 1) * nq]
            k1 = qkv1[:, hq * d + r * nk:hq * d + (r + 1) * nk]
            v1 = qkv1[:, hq * d + hkv * d + r * nk:hq * d + hkv * d + (r + 1) * nk]
            assert np.array_equal(got[(tag, "qkv", 0)], np.concatenate([q1, k1, v1], axis=1)), (tag, r)
            if tag == "wan":  # the norm over all heads adds the gathered per-head sums in one fixed order
                for op in ("qd", "kd"):
                    assert np.array_equal(got[(tag, op, 0)], tr[(op, 0)].numpy()[:, r * hq // 2:(r + 1) * hq // 2])
            assert np.array_equal(got[(tag, "attention", 0)], att1[..., r * hq // 2:(r + 1) * hq // 2, :]), (tag, r)
            o1 = tr[("o", 0)].numpy()
            assert np.all(np.abs(got[(tag, "o", 0)] - o1) <= 2.0**-6 * np.abs(o1) + 2e-3 * np.abs(o1).max()), (tag, r)
