"""Paged-cache bookkeeping on the host (no GPU): PageTable against the reference's token-list model.

The paged layout's contract is that the logical cache equals the reference's contiguous cache
after the same appends and splices (threadcut/kv.py:28-41, 64-77). Here the pool holds token ids,
so after every operation the pool gathered in run order must equal the list the reference would
hold; the tests also check that new slots never land on a live row, that no page leaks or is
freed twice, and that the tile table covers exactly the runs with tiles the decode kernel accepts.
"""
import random

import numpy as np
import pytest

from oracle.paged import gather_ref
from threadcut_b200.match import Split
from threadcut_b200.paged import TILE_ROWS, PageTable


def check_invariants(tab, pool, model):
    assert tab.n == len(model)
    assert gather_ref(pool, tab.runs).ravel().tolist() == model
    used = {r[0] for r in tab.runs}
    assert not used & set(tab.free), "a page is both in use and free"
    assert len(set(tab.free)) == len(tab.free), "a page was freed twice"
    assert used | set(tab.free) == set(range(tab.num_pages)), "a page leaked"
    for page, r0, cnt in tab.runs:
        assert 0 <= r0 and cnt >= 1 and r0 + cnt <= tab.page_rows
    tiles = tab.tiles()
    assert tiles.shape == (sum(-(-r[2] // TILE_ROWS) for r in tab.runs), 3)
    if tiles.size:
        assert (tiles[:, 2] >= 1).all() and (tiles[:, 2] <= TILE_ROWS).all()
        assert (tiles[:, 1] + tiles[:, 2] <= tab.page_rows).all()
    cover = [(p, r) for p, r0, cnt in tiles.tolist() for r in range(r0, r0 + cnt)]
    assert cover == [tuple(x) for x in tab.positions().tolist()]


@pytest.mark.parametrize("seed", range(12))
@pytest.mark.parametrize("page_rows", [32, 64, 96])
def test_random_appends_and_splices_match_the_list_model(seed, page_rows):
    rng = random.Random(seed * 7 + page_rows)
    pages = 48
    tab = PageTable(pages, page_rows)
    pool = np.full((pages, 1, page_rows, 1), -1, np.int64)
    model, next_id = [], 0
    for _ in range(80):
        if rng.random() < 0.6 or not model:
            t = rng.choice([1, 1, 1, 2, 5, 31, 32, 33, 64, 100])
            if (len(tab.free) - 1) * page_rows < t:
                continue
            live = {tuple(x) for x in tab.positions().tolist()}
            slots = tab.reserve(t)
            assert slots.shape == (t, 2)
            assert not live & {tuple(x) for x in slots.tolist()}, "a new slot overwrote a live token"
            pool[slots[:, 0], 0, slots[:, 1], 0] = np.arange(next_id, next_id + t)
            model += list(range(next_id, next_id + t))
            next_id += t
        else:
            n = len(model)
            a = rng.randint(0, n)
            c0 = rng.randint(a, n)
            c = rng.randint(0, n - c0)
            runs_c, freed = tab.splice(Split(a, c0, c))
            assert sum(r[2] for r in runs_c) == c
            assert gather_ref(pool, runs_c).ravel().tolist() == model[c0:c0 + c]
            model = model[:a] + model[c0:c0 + c]
        check_invariants(tab, pool, model)


def test_whole_pages_of_b_and_the_tail_are_freed():
    tab = PageTable(16, 64)
    tab.reserve(64 * 10)                                      # pages 0..9, full
    runs_c, freed = tab.splice(Split(70, 300, 200))           # A = pages 0-1, B = rest of 1..4, C = 4..7
    assert runs_c[0].tolist() == [4, 300 - 256, 64 - (300 - 256)]      # C starts inside page 4
    assert freed == [2, 3, 8, 9]                              # wholly inside B, and the stale tail
    assert tab.n == 270
    assert {r[0] for r in tab.runs} == {0, 1, 4, 5, 6, 7}


def test_append_after_splice_reuses_the_last_page_tail():
    tab = PageTable(8, 64)
    tab.reserve(200)                         # pages 0..3 (page 3 holds rows 0..7)
    tab.splice(Split(10, 100, 50))           # C = rows 36..63 of page 1, 0..21 of page 2; stale tail dropped
    slots = tab.reserve(5)
    assert slots.tolist() == [[2, 22], [2, 23], [2, 24], [2, 25], [2, 26]]
    assert 3 in tab.free


def test_crop_and_empty_cases():
    tab = PageTable(4, 32)
    assert tab.tiles().shape == (0, 3)
    tab.reserve(70)
    freed = tab.truncate(33)
    assert freed == [2] and tab.n == 33
    tab.splice(Split(0, 0, 0))
    assert tab.n == 0 and tab.runs == [] and sorted(tab.free) == [0, 1, 2, 3]
    with pytest.raises(ValueError):
        tab.splice(Split(0, 1, 0))
    with pytest.raises(ValueError):
        PageTable(4, 16)


def test_pool_exhaustion_raises():
    tab = PageTable(2, 32)
    tab.reserve(64)
    with pytest.raises(MemoryError):
        tab.reserve(1)
