"""Host logic of the tensor-parallel prefill (no GPU): shard plans, shard-local rotations,
and the column/row-parallel algebra over a real 2-rank ``gloo`` process group."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from faquant_b200.hisq_rotation import derive_hisq_rotation, restrict_hisq_rotation
from faquant_b200.tensor_parallel import (HIF4_GROUP, Qwen3TPConfig, SeqLayout, TPGroup, WanBlockConfig,
                                          column_rotation, qwen3_shard_slices, random_weight, row_rotation,
                                          seq_layout, sp_gather_rows, sp_reduce_scatter_rows)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_qwen3_32b_and_wan_shards_are_even_and_group_aligned(world: int) -> None:
    cfg = Qwen3TPConfig()
    seen_ffn, seen_q = [], []
    for rank in range(world):
        sl = qwen3_shard_slices(cfg, TPGroup(rank, world))
        for key in ("q_rows", "kv_rows", "ffn"):
            assert sl[key].start % HIF4_GROUP == 0 and (sl[key].stop - sl[key].start) % HIF4_GROUP == 0
        assert (sl["q_rows"].stop - sl["q_rows"].start) == cfg.heads // world * cfg.head_dim
        seen_ffn.append(sl["ffn"])
        seen_q.append(sl["q_rows"])
    assert seen_ffn[0].start == 0 and seen_ffn[-1].stop == cfg.ffn
    assert all(a.stop == b.start for a, b in zip(seen_ffn, seen_ffn[1:]))
    assert seen_q[-1].stop == cfg.heads * cfg.head_dim
    wan = WanBlockConfig()
    start, size = TPGroup(world - 1, world).shard(wan.ffn, HIF4_GROUP)
    assert start + size == wan.ffn and size % HIF4_GROUP == 0
    assert wan.heads % world == 0


def test_uneven_shards_are_refused() -> None:
    with pytest.raises(ValueError):
        TPGroup(0, 3).shard(25600, 64)
    with pytest.raises(ValueError):
        qwen3_shard_slices(Qwen3TPConfig(kv_heads=8), TPGroup(0, 16))


def test_row_rotations_are_the_shards_of_the_signs_construction() -> None:
    k, world = 8192, 4
    full = restrict_hisq_rotation(derive_hisq_rotation("model.layers.3.self_attn.o_proj", k, seed=17, block_size=64),
                                  "signs")
    parts = [row_rotation("model.layers.3.self_attn.o_proj", k, TPGroup(r, world), seed=17) for r in range(world)]
    assert all(p.permutation is None and p.block == 64 for p in parts)
    assert torch.equal(torch.cat([p.signs for p in parts]), full.signs)
    assert torch.equal(full.permutation, torch.arange(k))


def test_column_rotation_is_shared_per_norm() -> None:
    a = column_rotation("model.layers.5.self_attn.q_proj", 5120, seed=17, block=1024)
    b = column_rotation("model.layers.5.self_attn.v_proj", 5120, seed=17, block=1024)
    c = column_rotation("model.layers.5.mlp.up_proj", 5120, seed=17, block=1024)
    ref = derive_hisq_rotation("model.layers.5.input_layernorm", 5120, seed=17, block_size=1024)
    assert torch.equal(a.signs, b.signs) and torch.equal(a.permutation, b.permutation)
    assert torch.equal(a.signs, ref.signs) and torch.equal(a.permutation, ref.permutation)
    assert not torch.equal(a.permutation, c.permutation)


@pytest.mark.parametrize("rows,world", [(32768, 1), (32768, 2), (32768, 8), (75600, 2), (75600, 4), (75600, 8),
                                        (48, 2), (96, 3)])
def test_sequence_parallel_layout_partitions_the_rows(rows: int, world: int) -> None:
    """Every row belongs to exactly one rank's shard; ``locate`` inverts ``owned``; chunks are
    whole and as many as allowed (at most 4) for the BASELINE token counts."""
    lays = [seq_layout(rows, TPGroup(r, world)) for r in range(world)]
    assert all(lay is not None for lay in lays)
    owned = torch.cat([lay.owned() for lay in lays])
    assert torch.equal(owned.sort().values, torch.arange(rows))
    for r, lay in enumerate(lays):
        assert lay.shard_rows * world == rows and lay.chunks * lay.chunk_rows == rows
        for i, row in enumerate(lay.owned().tolist()):
            assert lay.locate(row) == (r, i)
    assert lays[0].chunks == (3 if (rows, world) == (75600, 8) else 4)
    assert seq_layout(75601, TPGroup(0, 2)) is None


def _sp_rank_main(rank: int, world: int, port: int, results) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tp = TPGroup(rank, world)
        lay = SeqLayout(48, world, rank, 3)
        g = torch.Generator().manual_seed(7)
        full = torch.randn(48, 5, generator=g)
        parts = [torch.randn(48, 5, generator=g) for _ in range(world)]  # every rank's partial output
        shard = full[lay.owned()]
        # the all-gather of the shards rebuilds the rows in order
        ok_ag = torch.equal(sp_gather_rows(tp, lay, shard), full)
        # the reduce-scatter of the partials gives this rank's rows of their sum
        red = sp_reduce_scatter_rows(tp, lay, parts[rank])
        ok_rs = torch.allclose(red, sum(parts)[lay.owned()], atol=1e-6)
        results[rank] = bool(ok_ag and ok_rs)
    finally:
        dist.destroy_process_group()


def test_sequence_parallel_collectives_over_gloo() -> None:
    world = 2
    results = mp.Manager().dict()
    mp.spawn(_sp_rank_main, args=(world, _free_port(), results), nprocs=world, join=True)
    assert dict(results) == {0: True, 1: True}


def _sp_packed_rank_main(rank: int, world: int, port: int, results) -> None:
    import numpy as np

    from oracle import hif4 as oh

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tp = TPGroup(rank, world)
        rows, k = 96, 256
        lay = seq_layout(rows, tp, max_chunks=3)
        g = torch.Generator().manual_seed(23)
        x = (torch.randn(rows, k, generator=g) * 3).to(torch.bfloat16).float().numpy()
        x[5, :64] = 0.0  # a zero block
        mine = x[lay.owned().numpy()]
        # this rank packs its own rows only (what the fused-norm K1 writes on the shard)
        codes, meta = oh.hif4_encode(mine)
        full_codes = sp_gather_rows(tp, lay, torch.from_numpy(codes))
        full_meta = sp_gather_rows(tp, lay, torch.from_numpy(meta.view(np.int32)))
        got = oh.hif4_decode(full_codes.numpy(), full_meta.numpy().view(np.uint32), k)
        results[rank] = bool(np.array_equal(got, oh.fake_quantize(x)) and lay.chunks == 3)
    finally:
        dist.destroy_process_group()


def test_sequence_parallel_packed_code_gather_matches_the_oracle_over_gloo() -> None:
    """The sequence-parallel all-gather of packed HiF4 codes and meta words (uint8 and
    int32, chunked row layout): every rank packs only its own rows, and the gathered bytes
    decode to the oracle's QDQ of all rows in row order."""
    world = 2
    results = mp.Manager().dict()
    mp.spawn(_sp_packed_rank_main, args=(world, _free_port(), results), nprocs=world, join=True)
    assert dict(results) == {0: True, 1: True}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, results) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = Qwen3TPConfig(hidden=256, heads=8, kv_heads=2, head_dim=32, ffn=512)
        tp = TPGroup(rank, world)
        sl = qwen3_shard_slices(cfg, tp)
        cpu = torch.device("cpu")
        x = torch.randn(16, cfg.hidden, generator=torch.Generator().manual_seed(3))
        wq = random_weight((cfg.heads * cfg.head_dim, cfg.hidden), 11, cpu).float()
        wo = random_weight((cfg.hidden, cfg.heads * cfg.head_dim), 12, cpu).float()
        wd = random_weight((cfg.hidden, cfg.ffn), 13, cpu).float()
        a = torch.randn(16, cfg.heads * cfg.head_dim, generator=torch.Generator().manual_seed(4))
        h = torch.randn(16, cfg.ffn, generator=torch.Generator().manual_seed(5))
        # column-parallel: this rank's output columns of the full product
        q_part = x @ wq[sl["q_rows"]].T
        ok_col = torch.allclose(q_part, (x @ wq.T)[:, sl["q_rows"]], atol=1e-5)
        # row-parallel: partial sums over this rank's input columns, summed by the all-reduce
        o = tp.all_reduce_(a[:, sl["o_cols"]] @ wo[:, sl["o_cols"]].T)
        d = tp.all_reduce_(h[:, sl["ffn"]] @ wd[:, sl["ffn"]].T)
        ok_row = torch.allclose(o, a @ wo.T, atol=1e-4) and torch.allclose(d, h @ wd.T, atol=1e-4)
        results[rank] = bool(ok_col and ok_row)
    finally:
        dist.destroy_process_group()


def test_column_and_row_parallel_algebra_over_gloo() -> None:
    world = 2
    results = mp.Manager().dict()
    mp.spawn(_rank_main, args=(world, _free_port(), results), nprocs=world, join=True)
    assert dict(results) == {0: True, 1: True}
