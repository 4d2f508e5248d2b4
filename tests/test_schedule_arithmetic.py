"""The work-distribution arithmetic of the two kernels, restated in Python and
checked on random sizes (CPU): every output element is produced by exactly one
work item, every k-block of a tile is accumulated exactly once, and every push
unit of the output side lands where the owner's GEMM waits for it.

Each helper restates one device or host function and names it; the kernels
themselves are checked on the GPU by tests/test_gpu_kernel.py and
tests/test_gpu_oproj.py."""

from collections import Counter

from hypothesis import given, settings, strategies as st

BM, BN, BK = 128, 256, 64


# ---------------------------------------------------------------- forward (fu_qkv.cu)
def pair_grid(L, heads, pairs, retile=True):
    """fu_qkv_forward's pair branch: (T, units, full_units, grid pairs)."""
    nb = (heads + 1) // 2
    T = (L + 2 * BM - 1) // (2 * BM) * nb
    rem = T % pairs
    units, full = T, T
    if retile and rem > 0 and 2 * rem <= pairs:
        full, units = T - rem, T + rem
    return T, units, full, min(units, pairs), nb


def decode_unit(u, full_units, nb, m_tiles):
    """fu_qkv.cu::decode_unit: (m_blk, n_blk, half); half -1 = both heads.
    Tiles are numbered column-major (row block t mod m_tiles)."""
    if u < full_units:
        return u % m_tiles, u // m_tiles, -1
    j = u - full_units
    t = full_units + (j >> 1)
    return t % m_tiles, t // m_tiles, j & 1


@settings(max_examples=200, deadline=None)
@given(st.integers(1, 20000), st.integers(1, 40), st.integers(1, 80), st.booleans())
def test_pair_grid_emits_every_head_of_every_tile_once(L, heads, pairs, retile):
    T, units, full, grid, nb = pair_grid(L, heads, pairs, retile)
    emitted = Counter()
    for pair in range(grid):                       # make_sched<true>: first, stride
        for u in range(pair, units, grid):
            m, n, half = decode_unit(u, full, nb, T // nb)
            for h in ((0, 1) if half < 0 else (half,)):
                if 2 * n + h < heads:              # an odd head count leaves one slot empty
                    emitted[(m, 2 * n + h)] += 1
    m_blocks = (L + 2 * BM - 1) // (2 * BM)
    assert emitted == Counter({(m, h): 1 for m in range(m_blocks) for h in range(heads)})


# ---------------------------------------------------------------- output side (fu_oproj.cu)
def slice_rows_for(cpm, unit_bytes=32 * 1024):
    """fu_oproj_forward: push units of ~32 KiB, 8 to 128 rows."""
    rows = 8
    while rows < BM and 2 * rows * cpm * 2 <= unit_bytes:
        rows *= 2
    return rows


def push_units(L, S, me, cpm):
    """run_gather's decoding of every unit u: (mb, peer s, row0, rows)."""
    rows_per = slice_rows_for(cpm)
    slices = BM // rows_per
    num_m = (L + BM - 1) // BM
    per_m = (S - 1) * slices
    out = []
    for u in range(num_m * per_m):
        mb, rest = divmod(u, per_m)
        sv = rest // slices
        s = sv + (1 if sv >= me else 0)
        row0 = mb * BM + (rest - sv * slices) * rows_per
        out.append((mb, s, row0, max(0, min(rows_per, L - row0))))
    return out, slices


@settings(max_examples=200, deadline=None)
@given(st.integers(1, 3000), st.integers(2, 8), st.integers(1, 8), st.data())
def test_push_units_cover_every_peer_row_once_and_fill_the_counters(L, S, heads_per, data):
    me = data.draw(st.integers(0, S - 1))
    cpm = heads_per * 128
    units, slices = push_units(L, S, me, cpm)
    rows = Counter()
    counts = Counter()                            # per (owner s, m-block)
    for mb, s, row0, n in units:
        assert s != me and 0 <= s < S             # own columns are never pushed
        assert row0 // BM == mb
        for r in range(row0, row0 + n):
            rows[(s, r)] += 1
        counts[(s, mb)] += 1
    assert rows == Counter({(s, r): 1 for s in range(S) if s != me for r in range(L)})
    # Owner s's producer waits for (S - 1) * slices counts per m-block; in a full
    # world every member pushes its units to s, so each member contributes slices.
    num_m = (L + BM - 1) // BM
    assert all(counts[(s, mb)] == slices for s in range(S) if s != me for mb in range(num_m))


def test_push_unit_sizes():
    # ~32 KiB per unit at every column width, never fewer than 8 rows.
    assert [slice_rows_for(c) for c in (128, 256, 512, 1024, 2048, 4096)] == \
        [128, 64, 32, 16, 8, 8]
    # The multiply-high division of run_gather is exact over a unit's chunks.
    for cpm in range(128, 8192 + 1, 128):
        cpr = cpm // 8
        magic = 0xFFFFFFFF // cpr + 1
        chunks = slice_rows_for(cpm) * cpr
        assert chunks < (1 << 32) // cpr
        for i in (0, cpr - 1, cpr, chunks - 1):
            assert (i * magic) >> 32 == i // cpr


@settings(max_examples=150, deadline=None)
@given(st.integers(1, 9000), st.sampled_from([256, 512, 1024, 2048, 4096, 8192]),
       st.integers(1, 74), st.booleans(), st.booleans())
def test_oproj_tiles_cover_the_output_once(L, H, pairs, pair, col_major):
    """fu_oproj_forward's tiling and Sched<kPair>::m_block / n_block (tiles
    numbered row by row with peers, column by column for a world of one):
    every (row block, column block) of out [L, H] is stored by exactly one CTA."""
    num_m = (L + BM - 1) // BM
    row_tiles = (L + 2 * BM - 1) // (2 * BM) if pair else num_m
    slots = pairs if pair else 148
    bn = 64
    for c in (256, 128):
        if row_tiles * (H // c) * 2 >= slots:
            bn = c
            break
    num_n = H // bn
    tiles = row_tiles * num_n
    stored = Counter()
    ctas = 2 * min(tiles, pairs) if pair else min(tiles, 148)
    for cta in range(ctas):
        rank = cta % 2 if pair else 0
        first, stride = (cta // 2, ctas // 2) if pair else (cta, ctas)
        for t in range(first, tiles, stride):
            mt, nb = (t % row_tiles, t // row_tiles) if col_major else divmod(t, num_n)
            mb = 2 * mt + rank if pair else mt
            if mb < num_m:                        # a pair's second CTA may have no rows
                stored[(mb, nb)] += 1
    assert stored == Counter({(m, n): 1 for m in range(num_m) for n in range(num_n)})
