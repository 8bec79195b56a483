"""Host-side scheduling logic that needs no GPU."""

import pytest

from saeflow_b200.ops import _chunk_plan


@pytest.mark.parametrize("M,C", [(16384, 4096), (16384, 2048), (1500, 64), (1500, 1000), (1500, 5000),
                                 (5000, 4096), (10, 4), (3, 1), (100, 1), (1, 4096), (12288, 4096),
                                 (16384, 8192), (9000, 8192), (262144, 16384)])
def test_forward_host_chunk_plan(M, C):
    for stream in (True, False):
        plan = _chunk_plan(M, C, stream)
        assert sum(plan) == M and min(plan) >= 1 and max(plan) <= C
        if M > C and (stream or M > 3 * C):
            # small chunks at both ends (the copies nothing overlaps), and no chunk more than
            # 2.5x its neighbour, so its copy hides behind the neighbour's compute
            assert plan[0] == plan[-1] <= max(1, C // 4)
            assert all(b <= 2.5 * a and a <= 2.5 * b for a, b in zip(plan, plan[1:]))
    if M > 3 * C:
        assert _chunk_plan(M, C, True)[0] == max(1, C // 16)
        assert _chunk_plan(M, C, False)[:2] == [max(1, C // 4), max(1, C // 2)]
