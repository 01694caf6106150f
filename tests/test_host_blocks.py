"""Row blocks of the host-buffer forward (host logic, CPU)."""
import pytest

from gsa_gdn_benchmarkstudy_b200.gsa import host_row_block_bounds


@pytest.mark.parametrize("T,chunks", [(16384, None), (65536, None), (4096, None), (1024, None),
                                      (300, 3), (4096, 4), (16384, 7), (129, 5), (128, 1)])
def test_blocks_cover_the_sequence_on_tile_edges(T, chunks):
    b = host_row_block_bounds(T, chunks)
    assert b[0] == 0 and b[-1] == T and b == sorted(set(b))
    assert all(e % 128 == 0 for e in b[1:-1])          # inner edges on query tiles
    sizes = [e - s for s, e in zip(b[:-1], b[1:])]
    assert all(n > 0 for n in sizes)


def test_default_counts_and_half_size_ends():
    b = host_row_block_bounds(16384)
    sizes = [e - s for s, e in zip(b[:-1], b[1:])]
    assert sizes == [2048, 4096, 4096, 4096, 2048]     # 5 blocks, half-size first and last
    assert len(host_row_block_bounds(4096)) - 1 == 2    # at least 2048 rows per block
    assert len(host_row_block_bounds(1024)) - 1 == 1
    assert len(host_row_block_bounds(4096, 4)) - 1 == 4  # an explicit count is honoured


def test_graphed_default_counts():
    """Replayed from a CUDA graph: up to 9 blocks, one per 1024 rows."""
    b = host_row_block_bounds(16384, graphed=True)
    sizes = [e - s for s, e in zip(b[:-1], b[1:])]
    assert len(sizes) == 9 and sizes[0] == sizes[-1] == 1024 and set(sizes[1:-1]) == {2048}
    assert len(host_row_block_bounds(4096, graphed=True)) - 1 == 4
    assert len(host_row_block_bounds(65536, graphed=True)) - 1 == 9
    assert len(host_row_block_bounds(1500, graphed=True)) - 1 == 1
    assert host_row_block_bounds(4096, 2, graphed=True) == host_row_block_bounds(4096, 2)
