"""The fused decode kernel's work split, restated on the CPU (no GPU needed).

moe_decode_kernel (litemind_b200/csrc/decode_fused.cu) relies on three pieces of index
arithmetic that no GPU test can exercise exhaustively:

* ListWalk (decode_fused.cu:110-128): a list of `tiles` tiles of `nkb` k-blocks each is
  cut into gridDim.x equal ranges of k-block iterations; a CTA walks its range as units
  (tile, kb0, kb1).  Every k-block must belong to exactly one unit.
* Split gate/up tiles (decode_fused.cu:899-924, 932-949): a tile whose k-blocks several
  CTAs share is completed by the CTA holding k-block 0.  Every other share must be the
  first unit of its CTA's range (each CTA has one partial-sum slot), and the completer
  finds those CTAs as blockIdx.x + 1 .. c_hi, skipping empty ranges, with
  c_hi = ceil((j0 + nkb) * G / iters) - 1; it waits until they have added nkb - kb1
  k-blocks to the tile's ticket.
* Staged router-logit tasks in gather mode (decode_fused.cu:208-220, the producer's
  copies and the epilogue's rounds): CTA b takes expert block b % n_eb and token groups
  b / n_eb + r * cta_per_eb for rounds r < rounds <= 2; every (token group, expert) pair
  must be computed exactly once, and the staged bytes must fit the free ring.

These tests restate that arithmetic in Python and check those properties over list sizes
from one tile to thousands, the grid sizes of a B200 (148 CTAs) and of smaller parts, and
every batch the fused kernel takes.
"""
import itertools

import pytest

# Ring geometry of moe_decode_kernel<32, 2> (gather mode), decode_fused.cu:58-91.
K_ATILE = 128 * 64 * 2
K_BTILE_32 = 32 * 64 * 2
K_DYN_BUDGET = 206 * 1024
K_STAGING_32 = 32 * 64 * 2
K_STAGES_32 = min(12, (K_DYN_BUDGET - 1024 - K_STAGING_32 - 1024) // (K_ATILE + K_BTILE_32))
K_EPI_WARPS = 8
K_LOGIT_TOKENS = 8


def walk(tiles: int, nkb: int, grid: int, cta: int):
    """ListWalk::init + next: CTA `cta`'s units (tile, kb0, kb1)."""
    iters = tiles * nkb
    it, end = iters * cta // grid, iters * (cta + 1) // grid
    units = []
    while it < end:
        t = it // nkb
        kb0 = it - t * nkb
        left = end - it
        kb1 = kb0 + left if left < nkb - kb0 else nkb
        units.append((t, kb0, kb1))
        it += kb1 - kb0
    return units


# V2-Lite lists: gate/up has 22 weight blocks of 32 k-blocks, down 16 of 22; tile counts
# of one to a few thousand (2 shared experts + up to 64 routed, 1-8 column tiles each).
LISTS = list(itertools.product([1, 2, 3, 5, 8, 22, 44, 176, 500, 1408, 1584, 2904], [1, 4, 22, 32]))
GRIDS = [1, 2, 7, 132, 148]


@pytest.mark.parametrize("grid", GRIDS)
def test_stream_k_ranges_cover_every_k_block_once(grid):
    for tiles, nkb in LISTS:
        seen = {}
        for cta in range(grid):
            for t, kb0, kb1 in walk(tiles, nkb, grid, cta):
                assert 0 <= t < tiles and 0 <= kb0 < kb1 <= nkb
                for kb in range(kb0, kb1):
                    assert (t, kb) not in seen, (tiles, nkb, grid, t, kb)
                    seen[(t, kb)] = cta
        assert len(seen) == tiles * nkb, (tiles, nkb, grid)


@pytest.mark.parametrize("grid", GRIDS)
def test_split_tiles_have_one_completer_and_its_partners(grid):
    for tiles, nkb in LISTS:
        iters = tiles * nkb
        shares = {}
        for cta in range(grid):
            units = walk(tiles, nkb, grid, cta)
            for i, (t, kb0, kb1) in enumerate(units):
                shares.setdefault(t, []).append((cta, kb0, kb1))
                if kb0 > 0:
                    # A share another CTA completes: the first unit of this CTA's range,
                    # so its one partial-sum slot suffices.
                    assert i == 0, (tiles, nkb, grid, cta)
        for t, lst in shares.items():
            owners = [(c, k1) for c, k0, k1 in lst if k0 == 0]
            assert len(owners) == 1
            owner, own_kb1 = owners[0]
            if own_kb1 == nkb:
                assert len(lst) == 1  # a whole tile has no other shares
                continue
            j0 = t * nkb
            c_hi = ((j0 + nkb) * grid + iters - 1) // iters - 1
            partners = [c for c in range(owner + 1, c_hi + 1) if iters * (c + 1) // grid != iters * c // grid]
            assert partners == sorted(c for c, k0, _ in lst if k0 > 0), (tiles, nkb, grid, t)
            # The ticket the completer waits for: the partners' k-blocks.
            assert sum(k1 - k0 for _, k0, k1 in lst if k0 > 0) == nkb - own_kb1


def staged_tasks(T: int, E: int, H: int, grid: int):
    """The staged-logit decision and each CTA's (token group, expert) tasks, or None."""
    ntg = (T + K_LOGIT_TOKENS - 1) // K_LOGIT_TOKENS
    n_eb = E // K_EPI_WARPS
    cta_per_eb = grid // n_eb if n_eb > 0 else 0
    rounds = (ntg + cta_per_eb - 1) // cta_per_eb if cta_per_eb > 0 else 0
    free = (K_STAGES_32 - 4) * K_ATILE + K_STAGES_32 * K_BTILE_32
    need = K_EPI_WARPS * H * 4 + rounds * K_LOGIT_TOKENS * H * 2
    staged = E % K_EPI_WARPS == 0 and cta_per_eb > 0 and rounds <= 2 and need <= free
    if not staged:
        return None
    tasks = {}
    for b in range(grid):
        eb, q = b % n_eb, b // n_eb
        if not (q < cta_per_eb and q < ntg):
            continue
        for r in range(rounds):
            tg = q + r * cta_per_eb
            if tg >= ntg:
                break
            for w in range(K_EPI_WARPS):
                tasks.setdefault((tg, eb * K_EPI_WARPS + w), []).append(b)
    # The ring holds the router rows and every round's token rows from A stage 4 on.
    end = 4 * K_ATILE + need
    assert end <= K_STAGES_32 * K_ATILE + K_STAGES_32 * K_BTILE_32
    return ntg, rounds, tasks


@pytest.mark.parametrize("E,H", [(64, 2048), (8, 256), (16, 512), (256, 2048), (24, 1024)])
def test_staged_logit_tasks_cover_each_pair_once(E, H):
    staged_any = False
    for T in range(16, 257):  # gather mode
        res = staged_tasks(T, E, H, 148)
        if res is None:
            continue
        staged_any = True
        ntg, rounds, tasks = res
        assert 1 <= rounds <= 2
        assert len(tasks) == ntg * E, (E, H, T)
        assert all(len(v) == 1 for v in tasks.values()), (E, H, T)
    assert staged_any  # 256 experts: 32 expert blocks of 4 CTAs, staged up to 64 tokens (two rounds)


def test_v2lite_stages_both_rounds_at_256_tokens():
    """V2-Lite at the fused kernel's largest batch: 32 token groups over 18 CTAs per expert
    block, two rounds, 64 KB of router rows + 2 x 32 KB of token rows (of 136 KB free)."""
    ntg, rounds, tasks = staged_tasks(256, 64, 2048, 148)
    assert (ntg, rounds) == (32, 2)
    assert K_STAGES_32 == 10
    assert len(tasks) == 32 * 64
