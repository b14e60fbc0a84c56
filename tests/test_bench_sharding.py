"""Host logic of the bench's sequence sharding (no GPU): the batch of every rank."""

from types import SimpleNamespace

import numpy as np
import pytest

import bench


@pytest.mark.parametrize("world", [2, 4, 8])
def test_balanced_share_partitions_the_global_draw(world):
    args = SimpleNamespace(batch=256, min_len=512, max_len=16384)
    shares = [bench.balanced_share(args, r, world) for r in range(world)]
    assert all(len(s) == args.batch for s in shares)
    glob = np.random.default_rng(bench.SEED).integers(args.min_len, args.max_len + 1,
                                                      size=args.batch * world)
    assert np.array_equal(np.sort(np.concatenate(shares)), np.sort(glob))
    sums = np.array([s.sum() for s in shares], np.float64)
    assert sums.max() / sums.min() < 1.001


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_config2_snake_deal_partitions_the_64_sequences(world):
    lengths = np.random.default_rng(2).integers(1024, 32 * 1024 + 1, size=64)
    shares = [bench.snake_deal(lengths, r, world) for r in range(world)]
    assert sorted(np.concatenate(shares).tolist()) == list(range(64))
    assert all(len(s) == 64 // world for s in shares)
    sums = np.array([lengths[s].sum() for s in shares], np.float64)
    assert sums.max() / sums.min() < 1.05


def test_split_floor_only_where_the_wave_rule_splits_long_sequences_finely():
    """bf16 attention splits grow to 128 pages while half a wave of CTAs remains, then
    double while a wave remains and a sequence still spans three splits: config 2's long
    sequences take 256-page splits on 1, 2 and 4 GPUs and 128 on 8 (on B200 the fastest
    size or within noise of it at each share); the config-3 batch and a batch of short
    sequences keep their split."""
    from shellsmith_b200 import paged

    lengths = np.random.default_rng(2).integers(1024, 32 * 1024 + 1, size=64)
    picks = {}
    for world in (1, 2, 4, 8):
        share = lengths[bench.snake_deal(lengths, 0, world)]
        pages = -(-(share + 3) // 16)
        args = (int(pages.max()), None, int(pages.sum()) * 2, 148)
        kw = dict(waves=3, cap=1024, rows=2 * len(share))
        picks[world] = (paged.split_plan(*args, **kw)[0],
                        paged.split_plan(*args, **kw, min_pages=128)[0])
    assert picks == {1: (256, 256), 2: (256, 256), 4: (256, 256), 8: (128, 128)}
    ctx = np.random.default_rng(3).integers(512, 16385, size=256)
    pages = -(-ctx // 16)
    assert paged.split_plan(int(pages.max()), None, int(pages.sum()) * 2, 148, waves=3,
                            cap=1024, rows=512, min_pages=128)[0] == 1024
    assert paged.split_plan(64, None, 8 * 64 * 2, 148, waves=3, cap=1024, rows=16,
                            min_pages=128)[0] == 16


def test_split_plan_follows_the_device_sm_count():
    """The adaptive split is planned for the SM count it is given: a part with fewer SMs
    reaches the wave target with larger splits, and no count means no adaptive plan."""
    import pytest

    from shellsmith_b200 import paged
    from shellsmith_b200.engine import HybridConfig

    ctx = np.random.default_rng(3).integers(512, 16385, size=64)
    pages = -(-ctx // 16)
    args = (int(pages.max()), None, int(pages.sum()) * 2)
    kw = dict(waves=3, cap=1024, rows=128)
    picks = {sms: paged.split_plan(*args, sms, **kw)[0] for sms in (74, 132, 148, 296)}
    assert picks[74] >= picks[132] >= picks[148] >= picks[296]
    assert picks[74] > picks[296]
    avg = args[2] / kw["rows"]   # pages of an average sequence (per head group)
    for sms, pps in picks.items():
        # the largest split that still fills 3 waves, or a longer one that fills a wave
        # while an average sequence still spans three splits
        ctas = lambda p: args[2] / p + kw["rows"] / 2  # noqa: E731
        assert pps == 16 or ctas(pps) >= 3 * sms or (ctas(pps) >= sms and avg / pps >= 3)
        assert pps == 1024 or ctas(2 * pps) < 3 * sms
    with pytest.raises(ValueError, match="SM count"):
        paged.split_plan(*args, **kw)
    assert paged.split_plan(100, 16) == (16, 7)          # an explicit size needs no count
    assert HybridConfig().sms is None and HybridConfig(sms=132).sms == 132


def test_strong_share_partitions_the_one_gpu_draw():
    """config3_strong: the 1-GPU draw of 256 sequences split over N ranks, 256/N each,
    disjoint and complete, with nearly equal context sums."""
    from types import SimpleNamespace

    args = SimpleNamespace(batch=256, min_len=512, max_len=16384)
    draw = np.random.default_rng(bench.SEED).integers(512, 16385, size=256)
    for world in (1, 2, 4, 8):
        shares = [bench.strong_share(args, r, world) for r in range(world)]
        assert all(len(s) == 256 // world for s in shares)
        assert sorted(np.concatenate(shares).tolist()) == sorted(draw.tolist())
        sums = np.array([s.sum() for s in shares], float)
        assert sums.max() / sums.min() < 1.05
    assert np.array_equal(np.sort(bench.strong_share(args, 0, 1)), np.sort(draw))
