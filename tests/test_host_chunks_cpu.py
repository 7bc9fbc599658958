"""Token chunks of the host-pipelined forward (localai_b200.moe.chunk_bounds):
they tile [0, T) without empty chunks, and with three or more chunks the first
and last are about half the size of the others (their PCIe copies overlap no
computation)."""
import pytest

from localai_b200.moe import chunk_bounds


@pytest.mark.parametrize('T', [1, 2, 3, 5, 10, 301, 2048, 16384])
@pytest.mark.parametrize('chunks', [1, 2, 3, 4, 6, 8, 64])
def test_chunk_bounds_tile_the_tokens(T, chunks):
    b = chunk_bounds(T, chunks)
    assert b[0] == 0 and b[-1] == T
    sizes = [b[i + 1] - b[i] for i in range(len(b) - 1)]
    assert all(sz > 0 for sz in sizes)
    assert len(sizes) <= max(1, min(chunks, T))
    if chunks >= 3 and T >= 64 * chunks:
        mid = sizes[1:-1]
        for end in (sizes[0], sizes[-1]):
            assert abs(2 * end - sum(mid) / len(mid)) <= 2
