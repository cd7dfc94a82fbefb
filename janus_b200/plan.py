"""Host-side level plan of a batch of packed requests (the CPU part of janus/hybrid.py `_levels`/`_branch_levels`,
:1661-1853, restated for packed levels without padding).

Level d holds every segment at depth d of every pack, in (pack, parent row, segment) order, packed back to back:
T_d tokens, B_d rows. Because rows are sorted by parent, the children of one parent row are consecutive, which is
what the fork kernel (a parent's state read in place by its children) and the tree attention tiles rely on. For
every row the plan records its parent row in level d-1 and its ancestor row's token range at every earlier level
(the keys it may attend to). Attention tiles are runs of at most `tokens` query tokens (the attention kernel's
tile: 128 or 64 rows over the GQA group) that never cross a change of long ancestor (so a tile reads one state,
not two) nor leave a long row of their own level.

Everything here is numpy on the host; `DevicePlan` moves the int32 tables to the GPU in one copy.
"""

from dataclasses import dataclass, field

import numpy as np
import torch

from .packing import tree_levels

LONG_ANCESTOR = 128   # ancestor rows longer than this split attention tiles at their boundaries
LONG_OWN = 64         # own rows longer than this end a tile at their last token


@dataclass
class Level:
    depth: int
    ids: np.ndarray            # [T] int32 token ids
    positions: np.ndarray      # [T] int32
    row_start: np.ndarray      # [B+1] int32
    row_of_token: np.ndarray   # [T] int32
    parent: np.ndarray         # [B] int32 row in level depth-1 (-1 at depth 0)
    anc_lo: list               # per ancestor level l < depth: [B] int32 first key (token of level l)
    anc_hi: list               # per ancestor level: [B] int32 end key
    child_start: np.ndarray    # [P+1] int32, P = rows of level depth-1 (depth 0: [0..B], each row its own group)
    chunk_start: np.ndarray    # [B+1] int32, first 64-token chunk of each row (the chunked delta rule)
    rows: list                 # (pack, segment, first packed position) per row
    keep: bool = False         # a deeper level reads this level's states
    tiles: dict = field(default_factory=dict)  # tokens per tile -> [n, 2] int32

    @property
    def T(self):
        return int(self.ids.shape[0])

    @property
    def B(self):
        return int(self.row_start.shape[0] - 1)

    def fork_chunks(self, max_tokens=64):
        """The rows packed into chunks for the segmented chunk scan: whole sibling rows (consecutive, same parent)
        are gathered into runs of at most `max_tokens` tokens. Returns (token start of each run [n+1], parent row of
        each run [n]) as int32, or None when a row is longer than max_tokens (or at depth 0)."""
        key = ("fork", max_tokens)
        if key in self.tiles:
            return self.tiles[key]
        out = None
        lengths = np.diff(self.row_start)
        if self.depth > 0 and (lengths.size == 0 or int(lengths.max()) <= max_tokens):
            starts, parents = [], []
            for p in range(self.child_start.shape[0] - 1):
                a, b = int(self.child_start[p]), int(self.child_start[p + 1])
                run_start, run_len = None, 0
                for r in range(a, b):
                    n = int(lengths[r])
                    if run_start is None or run_len + n > max_tokens:
                        if run_start is not None:
                            starts.append(run_start)
                            parents.append(p)
                        run_start, run_len = int(self.row_start[r]), 0
                    run_len += n
                if run_start is not None and run_len > 0:
                    starts.append(run_start)
                    parents.append(p)
            starts.append(self.T)
            out = (np.asarray(starts, dtype=np.int32), np.asarray(parents, dtype=np.int32))
        self.tiles[key] = out
        return out

    def attention_tiles(self, tokens):
        """Query tiles of at most `tokens` tokens (janus_b200_tree_attention_tile_tokens): the level's tokens are cut
        where a row's long ancestors change (a tile reads one state) and after every long row (a tile never leaves
        one); between cuts, consecutive tiles of `tokens` tokens, the last one shorter."""
        if tokens in self.tiles:
            return self.tiles[tokens]
        tq = max(1, int(tokens))
        rs = self.row_start.astype(np.int64)
        cuts = [np.array([0, self.T], dtype=np.int64), rs[np.flatnonzero(np.diff(rs) > LONG_OWN) + 1]]
        if self.B > 1 and self.anc_lo:
            key = np.stack([np.where((hi - lo) > LONG_ANCESTOR, lo, -1) for lo, hi in zip(self.anc_lo, self.anc_hi)], 1)
            cuts.append(rs[np.flatnonzero((key[1:] != key[:-1]).any(axis=1)) + 1])
        b = np.unique(np.concatenate(cuts))
        s, e = b[:-1], b[1:]
        n = (e - s + tq - 1) // tq
        first = np.repeat(np.cumsum(n) - n, n)
        starts = np.repeat(s, n) + (np.arange(int(n.sum()), dtype=np.int64) - first) * tq
        ends = np.minimum(starts + tq, np.repeat(e, n))
        arr = np.stack([starts, ends], axis=1).astype(np.int32).reshape(-1, 2)
        self.tiles[tokens] = arr
        return arr


@dataclass
class Readout:
    """Where each question's options are read: per level, the flat token rows and their logit slots."""
    mode: str
    # tree: per level d: (token rows [n], slot [n]) -> logits_flat[slot] = head(row)
    scalar: dict = field(default_factory=dict)
    # listwise: per level d: (option rows [n], option question idx [n] into decision rows, decision rows [Q], slots [n])
    pointer: dict = field(default_factory=dict)
    n_slots: int = 0
    # per pack: per question: list of slots (None: constant 0 logit for the false option of a tree-mode noul)
    layout: list = field(default_factory=list)


def build_levels(packs):
    """Levels of a batch of packs (module docstring)."""
    per_pack = [tree_levels(p.segment_ids, p.parents) for p in packs]
    depth = max(len(t) for t in per_pack)
    # every pack's tokens and positions once, back to back: a level's tokens are one gather from them
    all_ids = np.concatenate([np.asarray(p.input_ids[0], dtype=np.int32) for p in packs])
    all_pos = np.concatenate([np.asarray(p.position_ids[0], dtype=np.int32) for p in packs])
    pack_off = np.zeros(len(packs) + 1, dtype=np.int64)
    np.cumsum([int(p.input_ids.shape[1]) for p in packs], out=pack_off[1:])
    parents = [p.parents.tolist() for p in packs]
    levels = []
    row_index = {}  # (pack, segment) -> (depth, row, first packed position)
    for d in range(depth):
        entries = []  # (parent_row, pack, seg, start, end)
        for i, (p, tree) in enumerate(zip(packs, per_pack)):
            if d >= len(tree):
                continue
            par = parents[i]
            for seg, a, b in tree[d]:
                prow = -1 if d == 0 else row_index[(i, par[seg])][1]
                entries.append((prow, i, seg, a, b))
        if d > 0:
            entries.sort(key=lambda e: (e[0], e[1], e[2]))
        B = len(entries)
        lengths = np.array([b - a for _, _, _, a, b in entries], dtype=np.int64)
        row_start = np.zeros(B + 1, dtype=np.int64)
        np.cumsum(lengths, out=row_start[1:])
        T = int(row_start[-1])
        rot = np.repeat(np.arange(B, dtype=np.int32), lengths)
        src = np.array([pack_off[i] + a for _, i, _, a, _ in entries], dtype=np.int64)
        gather = np.arange(T, dtype=np.int64) + np.repeat(src - row_start[:-1], lengths)
        ids, pos = all_ids[gather], all_pos[gather]
        parent = np.array([prow for prow, _, _, _, _ in entries], dtype=np.int32).reshape(B)
        rows = []
        for r, (prow, i, seg, a, b) in enumerate(entries):
            row_index[(i, seg)] = (d, r, a)
            rows.append((i, seg, a))
        if d == 0:
            child_start = np.arange(B + 1, dtype=np.int32)
            anc_lo, anc_hi = [], []
        else:
            prev = levels[d - 1]
            P = prev.B
            counts = np.bincount(parent, minlength=P)
            child_start = np.zeros(P + 1, dtype=np.int32)
            np.cumsum(counts, out=child_start[1:])
            prev.keep = True
            anc_lo = [lo[parent] for lo in prev.anc_lo] + [prev.row_start[:-1][parent].astype(np.int32)]
            anc_hi = [hi[parent] for hi in prev.anc_hi] + [prev.row_start[1:][parent].astype(np.int32)]
        chunk_start = np.zeros(B + 1, dtype=np.int64)
        np.cumsum((lengths + 63) // 64, out=chunk_start[1:])
        levels.append(Level(d, ids, pos, row_start.astype(np.int32), rot, parent, anc_lo, anc_hi,
                            child_start.astype(np.int32), chunk_start.astype(np.int32), rows))
    return levels, row_index


def build_readout(packs, levels, row_index, mode):
    """Readout rows of every question (janus/model.py:319-366): tree mode reads each leaf's last token through the
    ScalarHead (a noul question's single leaf gives the true option, the false option is the constant 0); listwise
    reads each option's last token against the branch's decision token through the PointerHead."""
    ro = Readout(mode)
    slot = 0
    scal = {}
    ptr = {}
    for i, p in enumerate(packs):
        segs = p.segment_ids.numpy()

        def flat(pos):
            d, r, a = row_index[(i, int(segs[pos]))]
            return d, int(levels[d].row_start[r]) + pos - a

        layout = [[None] * k for k in p.option_counts]
        for br in p.branches:
            if mode == "tree":
                for oi, pos in zip(br.option_indices if br.kind != "noul" else (1,), br.option_positions):
                    d, t = flat(pos)
                    scal.setdefault(d, ([], []))
                    scal[d][0].append(t); scal[d][1].append(slot)
                    layout[br.question_index][oi] = slot
                    slot += 1
            else:
                d, dec = flat(br.decision_position)
                e = ptr.setdefault(d, ([], [], [], []))
                qidx = len(e[2])
                e[2].append(dec)
                for oi, pos in zip(br.option_indices, br.option_positions):
                    d2, t = flat(pos)
                    if d2 != d:
                        raise ValueError("listwise options must sit in the decision's level")
                    e[0].append(t); e[1].append(qidx); e[3].append(slot)
                    layout[br.question_index][oi] = slot
                    slot += 1
        ro.layout.append(layout)
    ro.scalar = {d: (np.asarray(a, np.int32), np.asarray(b, np.int64)) for d, (a, b) in scal.items()}
    ro.pointer = {d: (np.asarray(a, np.int32), np.asarray(b, np.int32), np.asarray(c, np.int32), np.asarray(s, np.int64))
                  for d, (a, b, c, s) in ptr.items()}
    ro.n_slots = slot
    return ro


class DevicePlan:
    """The int32 tables of every level on one device, moved with a single host-to-device copy."""

    def __init__(self, levels, readout, device, tile_tokens=()):
        chunks, index = [], {}

        def add(key, arr):
            arr = np.ascontiguousarray(arr, dtype=np.int32).reshape(-1)
            index[key] = (sum(c.size for c in chunks), arr.size)
            chunks.append(arr)

        for lv in levels:
            d = lv.depth
            add((d, "ids"), lv.ids)
            add((d, "pos"), lv.positions)
            add((d, "row_start"), lv.row_start)
            add((d, "row_of_token"), lv.row_of_token)
            add((d, "parent"), np.maximum(lv.parent, 0))
            add((d, "child_start"), lv.child_start)
            add((d, "chunk_start"), lv.chunk_start)
            for l, (lo, hi) in enumerate(zip(lv.anc_lo, lv.anc_hi)):
                add((d, "lo", l), lo)
                add((d, "hi", l), hi)
            for n in tile_tokens:
                add((d, "tiles", n), lv.attention_tiles(n))
            fc = lv.fork_chunks()
            if fc is not None:
                add((d, "fc_start"), fc[0])
                add((d, "fc_parent"), fc[1])
                add((d, "fc_chunks"), np.arange(fc[1].shape[0] + 1, dtype=np.int32))
        for d, (rows, slots) in readout.scalar.items():
            add((d, "scalar_rows"), rows)
            add((d, "scalar_slots"), slots)
        for d, (orows, oq, drows, slots) in readout.pointer.items():
            add((d, "opt_rows"), orows)
            add((d, "opt_q"), oq)
            add((d, "dec_rows"), drows)
            add((d, "pointer_slots"), slots)
        host = np.concatenate(chunks) if chunks else np.zeros(0, np.int32)
        pinned = torch.from_numpy(host).pin_memory() if torch.cuda.is_available() else torch.from_numpy(host)
        self.buffer = pinned.to(device, non_blocking=True)
        self.h2d_bytes = host.size * 4
        self.index = index

    def __getitem__(self, key):
        off, n = self.index[key]
        return self.buffer[off:off + n]
