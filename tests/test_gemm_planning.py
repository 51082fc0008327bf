"""Host-side GEMM planning that runs without a GPU: the split-K choice."""

from __future__ import annotations

import math

import pytest

from mini_nccl_b200.ops.kernels import NUM_SMS, _splits_for


def _kblock_time(m: int, n: int, k: int, s: int) -> int:
    """k-blocks the busiest SM runs with split factor s (whole waves of units)."""
    bn = 256 if n >= 256 else 128
    tiles = math.ceil(m / 128) * math.ceil(n / bn)
    kb = math.ceil(k / 64)
    per = math.ceil(kb / s)
    s_eff = math.ceil(kb / per)
    return math.ceil(tiles * s_eff / NUM_SMS) * per


@pytest.mark.parametrize("m,n", [(2304, 768), (3072, 768), (768, 3072), (768, 768)])
def test_weight_gradient_splits_fill_whole_waves(m: int, n: int) -> None:
    # GPT-124M weight gradients: K = 16 x 1024 tokens, few output tiles
    k = 16384
    s = _splits_for(m, n, k)
    bn = 256 if n >= 256 else 128
    ideal = math.ceil(m / 128) * math.ceil(n / bn) * math.ceil(k / 64) / NUM_SMS
    assert s > 1
    assert _kblock_time(m, n, k, s) <= 1.15 * ideal, (s, _kblock_time(m, n, k, s), ideal)


def test_qkv_weight_gradient_avoids_a_nearly_empty_second_wave() -> None:
    # 54 tiles x 3 splits = 162 units: a second wave of 14; the model moves off 3
    assert _splits_for(2304, 768, 16384) != 3
    assert _kblock_time(2304, 768, 16384, _splits_for(2304, 768, 16384)) < _kblock_time(2304, 768, 16384, 3)


@pytest.mark.parametrize("m,n,k", [(16384, 2304, 768), (16384, 768, 3072), (16384, 768, 2304),
                                   (16384, 768, 50304), (50304, 768, 16384), (2304, 768, 512)])
def test_no_split_when_the_grid_is_full_or_k_is_short(m: int, n: int, k: int) -> None:
    # a full grid stays unsplit even with a ragged last wave: the LM head's data
    # gradient (16384 x 768 x 50304) measured slower in 5 splits than in one
    assert _splits_for(m, n, k) == 1


def test_split_never_leaves_units_shorter_than_four_k_blocks() -> None:
    for k in (1024, 2048, 4096, 16384, 65536):
        s = _splits_for(128, 128, k)
        assert math.ceil(math.ceil(k / 64) / s) >= 4
