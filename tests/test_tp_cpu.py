"""Host-side layout of tensor-parallel decoding: vocab shards of the vocab-parallel sampler and the rank
groups of a TP x DP rollout."""

import pytest

from vlmrl.parallel.tp import tp_partition, vocab_shard


@pytest.mark.parametrize("V,W", [(151936, 2), (151936, 8), (1024, 2), (1000, 4), (151936, 3)])
def test_vocab_shards_are_whole_tiles_that_cover_the_vocabulary(V, W):
    shards = [vocab_shard(V, W, r) for r in range(W)]
    assert shards[0][0] == 0 and shards[-1][1] == V
    for (a0, a1), (b0, b1) in zip(shards, shards[1:]):
        assert a1 == b0                       # contiguous, no gap or overlap
    for v0, v1 in shards[:-1]:
        assert v0 % 128 == 0 and (v1 - v0) % 128 == 0 and v1 > v0
    sizes = [v1 - v0 for v0, v1 in shards]
    assert max(sizes) - min(sizes) <= 128 * W  # balanced to within a tile per rank


def test_tp_partition_groups_consecutive_ranks():
    assert tp_partition(8, 2) == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert tp_partition(4, 4) == [[0, 1, 2, 3]]
    with pytest.raises(ValueError):
        tp_partition(6, 4)
