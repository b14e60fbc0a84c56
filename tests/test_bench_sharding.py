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
