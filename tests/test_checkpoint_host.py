"""Host side of the step-0 QAD checkpoint loader (faquant_b200.checkpoint): the shard
reader splits the HiF4 metadata leaves off by module, and the receipt checks of
qad_checkpoint.py:295-313 refuse other level variants and trained checkpoints."""

from __future__ import annotations

import pytest

from checkpoint_fixture import LINEARS, write_checkpoint


def test_reader_splits_metadata_by_module(tmp_path) -> None:
    from faquant_b200.checkpoint import read_checkpoint

    write_checkpoint(tmp_path)
    state, metadata = read_checkpoint(tmp_path)
    assert set(state) == {f"{name}.weight" for name in LINEARS} | {"norm.weight"}
    assert set(metadata) == set(LINEARS)
    for name, (n, k) in LINEARS.items():
        m = metadata[name]
        assert set(m) == {"scale", "reciprocal", "scale_lv2_exponent", "scale_lv3_exponent"}
        assert tuple(m["scale"].shape) == (n, k // 64, 1, 1, 1)
        assert tuple(m["scale_lv3_exponent"].shape) == (n, k // 64, 8, 2, 1)


def test_receipt_refuses_other_levels_and_trained_checkpoints(tmp_path) -> None:
    from faquant_b200.checkpoint import check_receipt

    write_checkpoint(tmp_path / "a", levels="12")
    with pytest.raises(ValueError, match="scale levels"):
        check_receipt(tmp_path / "a", weight_levels="123")
    check_receipt(tmp_path / "a", weight_levels="12")
    write_checkpoint(tmp_path / "b")
    (tmp_path / "b" / "training_receipt.json").write_text("{}")
    with pytest.raises(ValueError, match="step-0"):
        check_receipt(tmp_path / "b")
