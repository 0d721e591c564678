"""CPU model of the stream-K decode kernel's schedule (gemv_sk_kernel in csrc/gemm_small_sk.cuh).

The kernel gives CTA c the chunk range [c*U/G, (c+1)*U/G) of the U = n_blocks * k_blocks
(row block, k-chunk) units, row-block-major; its 16 compute warps form NG = 16 / WPC groups of
WPC warps (WPC = 1 for M <= 8, 4 above), group q takes the CTA's chunks i = q (mod NG), and at
every row-block change and at the end each of the group's WPC warps adds its partial sums of the
row block (covering the chunks it processed) into the fp32 sums.  This model replays that
bookkeeping: every unit is processed exactly once, and the flushes of every row block together
cover each of its k_blocks chunks with all WPC warps (128 / WPC rows each) exactly once, so the
sums the finalize kernel converts are complete (gemv_sk_finalize_kernel).
"""

import itertools

import pytest


def replay(n_blocks, k_blocks, grid, wpc):
    ng = 16 // wpc
    U = n_blocks * k_blocks
    seen = [0] * U
    events = []  # (row block, chunks) flushes, in an arbitrary but complete order
    for c in range(grid):
        u0, u1 = U * c // grid, U * (c + 1) // grid
        for q in range(ng):
            seg_rb, seg_n = -1, 0
            for i in range(q, u1 - u0, ng):
                u = u0 + i
                rb = u // k_blocks
                if rb != seg_rb:
                    if seg_rb >= 0:
                        events += [(seg_rb, seg_n)] * wpc  # the group's warps
                    seg_rb, seg_n = rb, 0
                seen[u] += 1
                seg_n += 1
            if seg_rb >= 0:
                events += [(seg_rb, seg_n)] * wpc
    return seen, events


@pytest.mark.parametrize("n_blocks,k_blocks,grid", [
    (80, 128, 148), (64, 128, 148), (448, 128, 148), (64, 448, 148),  # decode shapes (N/128, K/64)
    (1, 1, 1), (1, 3, 1), (3, 5, 7), (2, 2, 148), (7, 13, 5), (5, 1, 3),
])
@pytest.mark.parametrize("wpc", [1, 2, 4])
def test_every_unit_once_and_every_row_block_fully_flushed(n_blocks, k_blocks, grid, wpc):
    grid = min(grid, n_blocks * k_blocks)
    seen, events = replay(n_blocks, k_blocks, grid, wpc)
    assert all(s == 1 for s in seen)
    count = [0] * n_blocks
    for rb, n in events:
        count[rb] += n
    assert count == [wpc * k_blocks] * n_blocks


def test_shares_differ_by_at_most_one_chunk():
    for nb, kb, g in itertools.product((64, 80, 448), (128, 448), (148, 147)):
        U = nb * kb
        sizes = [U * (c + 1) // g - U * c // g for c in range(g)]
        assert max(sizes) - min(sizes) <= 1
