"""Host-side split policy (kv_cache.auto_partition): which batches take the
balanced split when the caller leaves the choice to the library."""

from cloverinfer_b200 import _lib
from cloverinfer_b200.kv_cache import auto_partition


def test_uniform_contexts_keep_fixed_partitions():
    assert auto_partition([32768] * 8, 1) == 0


def test_ragged_single_token_batches_take_the_balanced_split():
    assert auto_partition([1024, 4096, 2000, 3000], 1) == _lib.PARTITION_BALANCED


def test_multitoken_sharded_empty_and_huge_batches_keep_fixed_partitions():
    ragged = [16, 16384, 300, 5000]
    assert auto_partition(ragged, 4) == 0
    assert auto_partition(ragged, 1, sharded=True) == 0
    assert auto_partition([], 1) == 0
    assert auto_partition([0, 0], 1) == 0
    assert auto_partition([1] * 1024 + [4000], 1) == 0
