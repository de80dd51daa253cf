"""CPU: token chunk boundaries of the host pipeline (cernels_b200.pipeline.HostPipeline)."""

import pytest

from cernels_b200.pipeline import HostPipeline


@pytest.mark.parametrize("T", [1, 2, 5, 7, 100, 4096, 16384])
@pytest.mark.parametrize("chunks", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("taper", [False, True])
def test_chunks_cover_every_token_once(T, chunks, taper):
    b = HostPipeline.chunk_bounds(T, chunks, taper)
    assert b[0] == 0 and b[-1] == T
    assert all(y > x for x, y in zip(b[:-1], b[1:]))  # no empty chunk
    assert len(b) - 1 == min(chunks, T)


def test_tapered_chunks_are_half_size_at_both_ends():
    b = HostPipeline.chunk_bounds(16384, 4, True)
    sizes = [y - x for x, y in zip(b[:-1], b[1:])]
    assert abs(sizes[0] * 2 - sizes[1]) <= 2 and abs(sizes[-1] * 2 - sizes[-2]) <= 2
