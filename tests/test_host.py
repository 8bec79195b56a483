"""Host-side scheduling logic that needs no GPU."""

import pytest

from saeflow_b200.ops import SMALL_SPLIT_ROWS, _chunk_plan


@pytest.mark.parametrize("M,C", [(16384, 4096), (16384, 2048), (1500, 64), (1500, 1000), (1500, 5000),
                                 (5000, 4096), (10, 4), (3, 1), (100, 1), (1, 4096), (12288, 4096),
                                 (16384, 8192), (9000, 8192), (262144, 16384), (4096, 8192), (2047, 8192),
                                 (2048, 2048), (8192, 8192)])
def test_forward_host_chunk_plan(M, C):
    plan = _chunk_plan(M, C)
    assert sum(plan) == M and min(plan) >= 1 and max(plan) <= C
    if M > 3 * C:
        # quarter and half chunks at both ends shorten the copies nothing overlaps
        ramp = [max(1, C // 4), max(1, C // 2)]
        assert plan[:2] == ramp and plan[-2:] == ramp[::-1]
    if SMALL_SPLIT_ROWS <= M <= C:
        # a batch of one chunk still overlaps its copies: quarter, half, quarter
        assert plan == [M // 4, M - 2 * (M // 4), M // 4]
    if M < SMALL_SPLIT_ROWS and M <= C:
        assert plan == [M]
