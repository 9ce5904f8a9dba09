"""ep_sort_rows_kernel's index arithmetic (litemind_b200/csrc/router.cu), restated on the CPU.

The expert-parallel receive buffer holds chunks of local experts one after another, each
chunk source-major (or, in the fixed-block exchange, one block of `src_stride` rows per
source).  The kernel's block (source r, local expert e of the chunk) sums the
(source, expert) counts before its group -- in receive order and in expert-major order
-- and copies its rows, 16 at a time over row blocks y, y + gridDim.y, ...  Every
received row must land exactly once in the expert-major buffer, with row_src pointing
back at it, whatever the chunking and however small the grid's y extent.
"""
import numpy as np
import pytest

K_SORT_ROWS = 16


def receive_layout(counts: np.ndarray, chunks: int, src_stride: int):
    """Receive position of every (source, expert, j) row: the exchange's layout."""
    N, El = counts.shape
    pos = {}
    if src_stride > 0:
        for r in range(N):
            p = r * src_stride
            for e in range(El):
                for j in range(counts[r, e]):
                    pos[(r, e, j)] = p
                    p += 1
        return pos
    p = 0
    for k in range(chunks):
        lo, hi = k * El // chunks, (k + 1) * El // chunks
        for r in range(N):
            for e in range(lo, hi):
                for j in range(counts[r, e]):
                    pos[(r, e, j)] = p
                    p += 1
    return pos


def sort_launch(counts, src_stride, e_lo, e_hi, grid_y_cap, x_sorted, row_src):
    """One launch of ep_sort_rows_kernel over chunk [e_lo, e_hi)."""
    N, El = counts.shape
    ne = e_hi - e_lo
    max_group = int(counts[:, e_lo:e_hi].max()) if counts.size else 0
    if max_group <= 0:
        return
    grid_y = min((max_group + K_SORT_ROWS - 1) // K_SORT_ROWS, grid_y_cap)
    for bx in range(N * ne):
        r = bx // ne
        e = e_lo + (bx - r * ne)
        src = dst = 0
        for i in range(N * El):  # the first warp's sums (order does not matter)
            rr, ee = divmod(i, El)
            c = int(counts[rr, ee])
            before = (rr == r and ee < e) if src_stride > 0 else (
                ee < e_lo or (ee < e_hi and (rr < r or (rr == r and ee < e))))
            if before:
                src += c
            if ee < e or (ee == e and rr < r):
                dst += c
        s_src = (r * src_stride if src_stride > 0 else 0) + src
        cnt = int(counts[r, e])
        for by in range(grid_y):
            j0 = by * K_SORT_ROWS
            while j0 < cnt:
                rows = min(K_SORT_ROWS, cnt - j0)
                for j in range(rows):
                    assert x_sorted[dst + j0 + j] == -1, "a row written twice"
                    x_sorted[dst + j0 + j] = s_src + j0 + j
                    row_src[dst + j0 + j] = s_src + j0 + j
                j0 += grid_y * K_SORT_ROWS


@pytest.mark.parametrize("N,El,chunks,fixed,grid_y_cap", [(1, 64, 2, False, 65535), (2, 4, 4, False, 65535),
                                                          (8, 8, 2, False, 65535), (4, 8, 3, False, 2),
                                                          (2, 4, 1, True, 65535), (8, 8, 1, True, 1),
                                                          (3, 5, 1, False, 1)])
def test_sorted_rows_are_expert_major_and_map_back(N, El, chunks, fixed, grid_y_cap):
    rng = np.random.default_rng(N * 100 + El)
    counts = rng.integers(0, 70, size=(N, El))
    counts[0, 0] = 0  # an empty group
    src_stride = int(counts.sum(axis=1).max()) + 3 if fixed else 0
    pos = receive_layout(counts, chunks, src_stride)
    total = int(counts.sum())
    x_sorted = np.full(total, -1, np.int64)  # each entry: the receive position copied there
    row_src = np.full(total, -1, np.int64)
    for k in range(chunks):
        sort_launch(counts, src_stride, k * El // chunks, (k + 1) * El // chunks, grid_y_cap, x_sorted, row_src)
    # Expert-major order: expert 0's rows from source 0, 1, ..., then expert 1's, ...
    expected = [pos[(r, e, j)] for e in range(El) for r in range(N) for j in range(counts[r, e])]
    np.testing.assert_array_equal(x_sorted, expected)
    np.testing.assert_array_equal(row_src, x_sorted)
