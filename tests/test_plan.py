"""Host-side level planning (no GPU): level tables, ancestor ranges, tiles, readout layout."""

import numpy as np

from janus_b200 import synthetic
from janus_b200.plan import build_levels, build_readout


def test_tree_levels_and_ranges():
    packs = [synthetic.tiny_request(seed=s, mode="tree") for s in (1, 2)]
    levels, index = build_levels(packs)
    assert [lv.depth for lv in levels] == [0, 1, 2]
    l0, l1, l2 = levels
    assert l0.B == 2 and l0.T == 512
    assert l1.B == 6 and l2.B == 2 * (4 + 3 + 1)
    # children of one parent are consecutive and child_start covers every row
    assert l2.child_start[0] == 0 and l2.child_start[-1] == l2.B
    assert (np.diff(l2.parent) >= 0).all()
    # every leaf sees its request's state and its block
    for r in range(l2.B):
        b = l2.parent[r]
        assert l2.anc_lo[1][r] == l1.row_start[b] and l2.anc_hi[1][r] == l1.row_start[b + 1]
        st = l1.parent[b]
        assert l2.anc_lo[0][r] == l0.row_start[st] and l2.anc_hi[0][r] == l0.row_start[st + 1]
    assert l0.keep and l1.keep and not l2.keep
    # token content matches the packs
    i, seg, a = l2.rows[3]
    n = l2.row_start[4] - l2.row_start[3]
    assert (l2.ids[l2.row_start[3]:l2.row_start[4]] == packs[i].input_ids[0, a:a + n].numpy()).all()


def test_tiles_cover_every_token_once_and_stay_in_one_request():
    packs = [synthetic.q4b_request(vocab=4096, seed=s, state_tokens=300, questions=3) for s in range(3)]
    levels, _ = build_levels(packs)
    for lv in levels:
        for n in (1, 8, 16, 32, 64, 128):
            tiles = lv.attention_tiles(n)
            cover = np.zeros(lv.T, dtype=int)
            for a, b in tiles:
                assert 0 < b - a <= n
                cover[a:b] += 1
                if lv.depth > 0:  # one state per tile
                    rows = lv.row_of_token[a:b]
                    assert len(set(lv.anc_lo[0][rows].tolist())) == 1
                else:
                    assert len(set(lv.row_of_token[a:b].tolist())) == 1
            assert (cover == 1).all()


def test_fork_chunks_pack_whole_sibling_rows():
    packs = [synthetic.q4b_request(vocab=4096, seed=s, state_tokens=300, questions=5) for s in range(3)]
    levels, _ = build_levels(packs)
    assert levels[0].fork_chunks() is None  # the state level has no parent
    leaves = levels[-1]
    starts, parents = leaves.fork_chunks()
    assert starts[0] == 0 and starts[-1] == leaves.T and (np.diff(starts) > 0).all()
    assert (np.diff(starts) <= 64).all()
    row_bounds = set(leaves.row_start.tolist())
    for i, p in enumerate(parents.tolist()):
        a, b = int(starts[i]), int(starts[i + 1])
        assert a in row_bounds and b in row_bounds  # whole rows only
        rows = set(leaves.row_of_token[a:b].tolist())
        assert all(int(leaves.parent[r]) == p for r in rows)  # siblings of one parent
    assert (np.diff(parents) >= 0).all()
    # a row longer than a run cannot be packed
    assert leaves.fork_chunks(max_tokens=1) is None or int(np.diff(leaves.row_start).max()) <= 1


def test_readout_layout_tree_and_listwise():
    packs = [synthetic.tiny_request(seed=0, mode="tree")]
    levels, index = build_levels(packs)
    ro = build_readout(packs, levels, index, "tree")
    layout = ro.layout[0]
    assert [len(q) for q in layout] == [4, 3, 2]
    assert layout[2][0] is None and layout[2][1] is not None  # noul: [0, z]
    assert ro.n_slots == 4 + 3 + 1
    packs = [synthetic.tiny_request(seed=0, mode="listwise")]
    levels, index = build_levels(packs)
    ro = build_readout(packs, levels, index, "listwise")
    assert ro.n_slots == 4 + 3 + 2
    orows, oq, drows, slots = ro.pointer[1]
    assert len(drows) == 3 and oq.tolist() == [0] * 4 + [1] * 3 + [2] * 2


def _greedy_tiles(lv, n):
    """The tile rule written as a plain walk over the rows: tiles of n tokens fill across rows, closed where the
    row's long ancestors (> LONG_ANCESTOR keys) change and after every long row (> LONG_OWN tokens)."""
    from janus_b200.plan import LONG_ANCESTOR, LONG_OWN
    out, start, count, prev = [], None, 0, None
    for r in range(lv.B):
        a, b = int(lv.row_start[r]), int(lv.row_start[r + 1])
        key = tuple(int(lo[r]) if int(hi[r]) - int(lo[r]) > LONG_ANCESTOR else -1
                    for lo, hi in zip(lv.anc_lo, lv.anc_hi))
        if start is not None and key != prev:
            out.append((start, start + count)); start, count = None, 0
        prev = key
        t = a
        while t < b:
            if start is None:
                start, count = t, 0
            take = min(n - count, b - t)
            count += take
            t += take
            if count == n:
                out.append((start, start + count)); start, count = None, 0
        if start is not None and b - a > LONG_OWN:
            out.append((start, start + count)); start, count = None, 0
    if start is not None:
        out.append((start, start + count))
    return np.asarray(out, dtype=np.int32).reshape(-1, 2)


def test_vectorised_tables_equal_a_row_by_row_restatement():
    packs = [synthetic.q4b_request(vocab=4096, seed=s, state_tokens=st, questions=q)
             for s, st, q in ((0, 300, 3), (1, 70, 5), (2, 1000, 2))]
    packs += [synthetic.tiny_request(seed=3, mode="tree")]
    levels, _ = build_levels(packs)
    for lv in levels:
        for r, (i, seg, a) in enumerate(lv.rows):  # every row's tokens and positions are its pack's slice
            s, e = int(lv.row_start[r]), int(lv.row_start[r + 1])
            assert (lv.ids[s:e] == packs[i].input_ids[0, a:a + e - s].numpy()).all()
            assert (lv.positions[s:e] == packs[i].position_ids[0, a:a + e - s].numpy()).all()
        for n in (1, 7, 16, 32, 64, 128):
            assert np.array_equal(lv.attention_tiles(n), _greedy_tiles(lv, n)), (lv.depth, n)
