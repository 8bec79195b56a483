"""Host-side scheduling logic that needs no GPU."""

import pytest

from saeflow_b200.ops import _chunk_plan


@pytest.mark.parametrize("M,C", [(16384, 4096), (16384, 2048), (1500, 64), (1500, 1000), (1500, 5000),
                                 (5000, 4096), (10, 4), (3, 1), (100, 1), (1, 4096), (12288, 4096),
                                 (16384, 8192), (9000, 8192), (262144, 16384)])
def test_forward_host_chunk_plan(M, C):
    plan = _chunk_plan(M, C)
    assert sum(plan) == M and min(plan) >= 1 and max(plan) <= C
    if M > C:
        # the copies nothing overlaps move C/16 rows, and every chunk's copy hides behind a
        # neighbour of at least half its size (growing towards the middle, shrinking after it)
        assert plan[0] == plan[-1] == max(1, C // 16)
        assert all(b <= 2 * a for a, b in zip(plan, plan[1:]))
        assert all(a <= 2 * b for a, b in zip(plan, plan[1:]))
