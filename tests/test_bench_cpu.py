"""Host-side logic of bench.py that needs no GPU: the end-to-end pipeline
chunks cover every (batch, kv-head) unit of the rank exactly once, each chunk
is one batch element's contiguous kv-head range, and the first and last
chunks are a single kv head when the ranges allow it."""
import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402
from ssa_b200.sharding import GroupSlice, group_slices  # noqa: E402


def _units(spans):
    return [(b, g) for b, g0, g1 in spans for g in range(g0, g1)]


@pytest.mark.parametrize("B,n_kv,world", [(4, 8, 1), (4, 8, 2), (4, 8, 4), (4, 8, 8), (8, 1, 1), (2, 8, 1),
                                          (16, 8, 1), (1, 16, 1), (4, 8, 3)])
def test_e2e_spans_cover_each_unit_once(B, n_kv, world):
    for rank in range(world):
        slices = group_slices(B, n_kv, world, rank) if world > 1 else [GroupSlice(0, B, 0, n_kv)]
        want = [(b, g) for s in slices for b in range(s.b0, s.b1) for g in range(s.g0, s.g1)]
        spans = bench.e2e_spans(slices, 8)
        assert sorted(_units(spans)) == sorted(want)
        assert _units(spans) == want  # in order: the pipeline walks the units batch-major
        assert all(g1 > g0 for _, g0, g1 in spans)
        if want and len(want) > 1:
            assert spans[0][2] - spans[0][1] == 1 and spans[-1][2] - spans[-1][1] == 1


def test_e2e_spans_c2_single_gpu_plan():
    spans = bench.e2e_spans([GroupSlice(0, 4, 0, 8)], 8)
    assert [g1 - g0 for _, g0, g1 in spans] == [1, 3, 4, 4, 4, 4, 4, 4, 3, 1]
