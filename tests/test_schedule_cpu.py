"""The decode's balanced work split, restated on the CPU and checked
exhaustively over many batch shapes.

The kernel (kimi_b200/csrc/decode_common.cuh: `balanced_schedule`,
`cta_of_tile`, the cursor; kimi_b200/csrc/mla_decode_fp4.cu: the empty-run
and span records; kimi_b200/csrc/mla_reduce.cu: the slots a merge reads)
lays the batch's 128-token tiles end to end, T in all, and gives run
[c T / G, (c + 1) T / G) to CTA c of G.  The part of sequence b inside the
run of CTA c is a piece; it writes its partial into slot b + c.  The CTA
holding a sequence's first tile records the sequence's CTA span
[c(first tile), c(last tile)], and the merge reads slots b + c for c in the
span.  An empty run (T < G) still names the sequence at its position and
writes LSE -inf into that sequence's slot b + c, so that a span it sits in
reads no stale weight.

Checked here: `cta_of_tile` names the run holding each tile; every tile is in
one run; every written slot is unique and inside the B + G slots of the
workspace; every slot a merge reads was written by this call (a piece or an
empty run); a sequence held by one CTA is written directly and merged by
nobody.
"""
import itertools
import random

import pytest


def cta_of_tile(x, total, ctas):
    """decode_common.cuh `cta_of_tile`: the largest c with c T / G <= x."""
    return ((x + 1) * ctas - 1) // total


def plan(tiles, ctas):
    """Pieces, empty-run records, spans and direct outputs of one call."""
    total = sum(tiles)
    starts = list(itertools.accumulate([0] + tiles[:-1]))
    writes = {}      # slot -> ("piece", b, c, lo, hi) or ("empty", b, c)
    direct = set()   # sequences written straight to o
    spans = {}       # sequence -> (first CTA, last CTA), recorded by its first tile's CTA
    covered = [0] * total
    for c in range(ctas):
        lo, hi = c * total // ctas, (c + 1) * total // ctas
        if lo == hi:
            if lo < total:  # the sequence at this position names the slot
                b = max(i for i in range(len(tiles)) if starts[i] <= lo and tiles[i] > 0)
                assert b + c not in writes
                writes[b + c] = ("empty", b, c)
            continue
        x = lo
        while x < hi:
            b = max(i for i in range(len(tiles)) if starts[i] <= x and tiles[i] > 0)
            p_lo, p_hi = x - starts[b], min(hi, starts[b] + tiles[b]) - starts[b]
            for t in range(starts[b] + p_lo, starts[b] + p_hi):
                covered[t] += 1
            if p_lo == 0 and p_hi == tiles[b]:
                direct.add(b)
            else:
                assert b + c not in writes, "two pieces share a slot"
                writes[b + c] = ("piece", b, c, p_lo, p_hi)
            if p_lo == 0:
                spans[b] = (c, cta_of_tile(starts[b] + tiles[b] - 1, total, ctas))
            x = starts[b] + p_hi
    return total, writes, direct, spans, covered


def check(tiles, ctas):
    total, writes, direct, spans, covered = plan(tiles, ctas)
    # cta_of_tile is the run holding the tile
    for x in range(total):
        c = cta_of_tile(x, total, ctas)
        assert c * total // ctas <= x < (c + 1) * total // ctas
    assert all(n == 1 for n in covered)
    assert all(0 <= s < len(tiles) + ctas for s in writes)
    for b, t in enumerate(tiles):
        if t == 0:
            assert b not in spans and b not in direct  # the merge writes zeros
            continue
        lo, hi = spans[b]
        if b in direct:
            assert lo == hi  # written by the decode itself; the merge skips it
            continue
        assert lo < hi
        for c in range(lo, hi + 1):  # every slot the merge reads was written now
            rec = writes.get(b + c)
            assert rec is not None and rec[1] == b and rec[2] == c, (tiles, ctas, b, c)


@pytest.mark.parametrize("ctas", [1, 2, 3, 7, 16, 37, 74, 148])
def test_uniform_batches(ctas):
    for batch, tiles in ((64, 64), (128, 32), (8, 1024), (1, 5), (3, 1), (200, 3)):
        check([tiles] * batch, ctas)


def test_ragged_batches_with_empty_sequences():
    rng = random.Random(3)
    for _ in range(300):
        batch = rng.randint(1, 40)
        tiles = [rng.choice([0, 1, 2, 3, 8, 50, 257]) for _ in range(batch)]
        if sum(tiles) == 0:
            tiles[0] = 1
        check(tiles, rng.choice([1, 2, 5, 13, 74, 148]))


def test_fewer_tiles_than_ctas_leaves_empty_runs_inside_spans():
    # 3 tiles over 8 CTAs: five runs are empty and their -inf records sit in
    # the spans of the sequences at their positions
    total, writes, direct, spans, _ = plan([2, 1], 8)
    assert total == 3
    assert sum(1 for r in writes.values() if r[0] == "empty") == 5
    check([2, 1], 8)
