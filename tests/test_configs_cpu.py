"""Tile choices on the host: the untuned heuristic and the committed B200 table give
tilings that a B200 kernel exists for (no GPU needed)."""

from __future__ import annotations

import json

import pytest

from int8_linear.kernel import TUNED_PATH, Config, default_config


@pytest.mark.parametrize("m", [1, 2, 3, 16, 17, 64, 256, 257, 4096])
@pytest.mark.parametrize("k,n", [(2048, 4096), (1024, 2048), (6144, 2048), (14336, 4096), (512, 2048),
                                 (4096, 28672), (2048, 12288)])
def test_default_config_is_a_valid_tiling(m, k, n):
    default_config(m, n, k).check()


def test_small_batches_default_to_cuda_core_tiles():
    cfg = default_config(1, 4096, 2048)
    assert (cfg.bm, cfg.bn, cfg.split) == (1, 0, 5)
    assert default_config(3, 4096, 2048).bm == 4                   # the smallest token count >= M
    assert default_config(4, 28672, 4096).split == 5               # up to 4 tokens on any weight
    assert default_config(8, 4096, 2048).split == 5                # 8 tokens on weights <= 16 MB
    assert default_config(8, 12288, 2048).swapped                  # 8 tokens on a 25 MB weight
    assert default_config(9, 4096, 2048).swapped                   # beyond 8 tokens: tensor cores


def test_choose_config_fits_a_cuda_core_bucket_to_the_batch(monkeypatch):
    from int8_linear import kernel

    monkeypatch.setattr(kernel.torch.cuda, "current_device", lambda: 0)
    monkeypatch.setattr(kernel, "tuned_config", lambda m, n, k: Config(4, 0, split=5))
    monkeypatch.setattr(kernel, "_chosen", {})
    assert kernel.choose_config(3, 4096, 2048).bm == 4
    assert kernel.choose_config(5, 4096, 2048) == Config(8, 0, split=5)       # bumped to 8 tokens
    assert kernel.choose_config(12, 4096, 2048) == Config(16, 0, split=5)      # up to 16 tokens
    assert kernel.choose_config(20, 4096, 2048) == default_config(20, 4096, 2048)


def test_tuned_table_entries_are_valid_tilings():
    tables = json.loads(TUNED_PATH.read_text())
    count = 0
    for shapes in tables.values():
        for shape, buckets in shapes.items():
            k, n = (int(x) for x in shape.split("x"))
            for m, entry in buckets.items():
                cfg = Config(**entry["config"])
                cfg.check()
                if cfg.split == 3 and not cfg.swapped:
                    # narrow tiles (<= 16 tokens) take 256 weight rows; above 16 tokens the
                    # same split is the 128-token tile with the weight on the MMA's N side
                    assert cfg.bm == 128 and (cfg.bn == 256 or int(m) > 16), (shape, m)
                assert entry.get("graph_us", entry.get("stand_in_us", 0)) > 0
                count += 1
    assert count > 0


def test_tuner_weight_pools_cover_twice_the_l2():
    from int8_linear.tune import COPIES, L2_BYTES, pool_size

    for nbytes in (4096 * 2048, 2048 * 2048, 12288 * 2048, 28672 * 4096, 1 << 30):
        n = pool_size(nbytes)
        assert n >= COPIES and n * nbytes >= 2 * L2_BYTES, nbytes


@pytest.mark.parametrize("m", [1, 2, 4, 16, 17, 64, 256, 1024, 4096])
@pytest.mark.parametrize("k,n", [(2048, 4096), (6144, 2048), (4096, 28672)])
def test_tuner_candidates_are_valid_and_narrow_only_for_small_batches(m, k, n):
    """Split 3 without swap_ab: narrow 128 x 256 tiles up to 16 tokens, 128-token tiles
    with cluster split-K from 17 to 512 tokens, never for prefill batches."""
    from int8_linear.tune import candidates

    cands = candidates(m, n, k, 148)
    assert cands and len({c.name for c in cands}) == len(cands)
    for c in cands:
        c.check()
        if c.split == 3 and not c.swapped:
            assert (m <= 16 and c.bn == 256) or 16 < m <= 512, c.name


def test_fused_activation_tiling_is_the_swap_tile_with_direct_loads():
    from int8_linear.kernel import fused_act_config

    assert fused_act_config(Config(16, 128, split=3, cluster=4)) == Config(16, 128, split=3, cluster=4, act=2)
    assert fused_act_config(Config(32, 128, act=2)) == Config(32, 128, act=2)
    assert fused_act_config(Config(128, 256, split=3, cluster=8)) is None   # narrow: no direct loads
    assert fused_act_config(Config(128, 256)) is None


def test_fused_activation_entry_validates_before_touching_a_gpu():
    import torch

    from int8_linear import NotSupported, w8a8_mm_quant_act

    w = torch.zeros((64, 32), dtype=torch.int8)
    sb = torch.ones(1)
    with pytest.raises(NotSupported, match="bf16/fp16"):
        w8a8_mm_quant_act(torch.zeros((2, 64)), w, sb)                     # fp32 activation
    with pytest.raises(ValueError, match="cannot multiply"):
        w8a8_mm_quant_act(torch.zeros((2, 48), dtype=torch.bfloat16), w, sb)


def test_cuda_core_tiles_are_valid_configs():
    from int8_linear import Config, NotSupported

    cfg = Config(4, 0, split=5, ctas=100)
    cfg.check()
    assert not cfg.swapped and cfg.name == "gemv m4 s0 c100"
    t = cfg.as_tile()
    assert (t.swap_ab, t.tok_tile, t.w_tile, t.split, t.ctas) == (0, 4, 0, 5, 100)
    for bad in (Config(3, 0, split=5), Config(32, 0, split=5), Config(8, 128, split=5)):
        with pytest.raises(NotSupported):
            bad.check()
    # cluster split-K now takes the wider token tiles too
    Config(128, 128, swap_ab=True, split=3, cluster=4).check()
    Config(256, 128, split=3, cluster=2).check()
