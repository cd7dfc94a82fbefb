"""The packed prefix-tree request: the input format of the decision readout.

Mirrors `PackedRequest` / `Branch` of the reference (janus/packing.py:20-64) field for field, so a pack made by
the reference's `pack_request` (janus/packing.py:89-202) can be handed over unchanged, and builds the same layout
directly from token ids for synthetic workloads (the benchmark has no tokenizer or text). One segment is the
shared state (segment 0); every other segment is a question branch whose parent is an earlier segment.

Layouts (janus/packing.py:127-183):
  tree      per question a block segment (parent 0) and one leaf segment per option (parent: the block); a leaf's
            decision position is its last token. Positions "continue": the block continues from the state's end
            and the leaves of a question continue one after another from the block's end (:157-163).
  listwise  per question one segment (parent 0) holding the question and all options; the options are read at
            the last token of each option, the decision at the branch's last token; positions restart at the
            state's end for every question (:176-183).
"""

from dataclasses import dataclass, field

import numpy as np
import torch


@dataclass
class Branch:
    start: int
    end: int
    question_index: int
    option_indices: tuple
    option_positions: tuple
    decision_position: int
    kind: str = "choice"
    leaves: tuple = ()


@dataclass
class PackedRequest:
    input_ids: torch.Tensor      # [1, n] int64
    position_ids: torch.Tensor   # [1, n] int64
    segment_ids: torch.Tensor    # [n] int64
    parents: torch.Tensor        # [segments] int64, parents[0] = 0
    branches: list
    state_length: int
    option_counts: tuple
    branch_packs: list = field(default_factory=list)
    images: tuple = None

    @property
    def token_count(self):
        return self.input_ids.shape[1]


@dataclass(frozen=True)
class Question:
    """A synthetic question: its kind, the token ids of its header and of each option."""
    kind: str                    # "choice" | "score" | "noul"
    header: tuple                # token ids of the block (tree) or the question text (listwise)
    options: tuple               # per option a tuple of token ids (noul: the single decision leaf in tree mode)
    suffix: tuple = ()           # listwise: the "Decision:" tokens after the options


def pack_tree(state, questions):
    """Tree layout with tree_positions="continue" (the released configs, janus/packing.py:127-170)."""
    tokens = list(state)
    s = len(tokens)
    positions = list(range(s))
    segments, branches = [], []
    for qi, q in enumerate(questions):
        block_start = len(tokens)
        tokens.extend(q.header)
        block_end = len(tokens)
        positions.extend(range(s, s + block_end - block_start))
        segments.append((block_start, block_end, 0))
        block_segment = len(segments)
        nxt = s + block_end - block_start
        leaves, decisions = [], []
        for leaf in q.options:
            start = len(tokens)
            tokens.extend(leaf)
            end = len(tokens)
            positions.extend(range(nxt, nxt + end - start))
            nxt += end - start
            segments.append((start, end, block_segment))
            leaves.append((start, end))
            decisions.append(end - 1)
        count = 2 if q.kind == "noul" else len(q.options)
        branches.append(Branch(block_start, block_end, qi, tuple(range(count)), tuple(decisions), block_end - 1,
                               q.kind, tuple(leaves)))
    return _finish(tokens, positions, segments, branches, s,
                   tuple(2 if q.kind == "noul" else len(q.options) for q in questions))


def pack_listwise(state, questions):
    """Listwise layout (janus/packing.py:171-183): one branch per question, options read at their last token."""
    tokens = list(state)
    s = len(tokens)
    positions = list(range(s))
    segments, branches = [], []
    for qi, q in enumerate(questions):
        start = len(tokens)
        tokens.extend(q.header)
        option_positions = []
        for option in q.options:
            tokens.extend(option)
            option_positions.append(len(tokens) - 1)
        tokens.extend(q.suffix)
        end = len(tokens)
        positions.extend(range(s, s + end - start))
        segments.append((start, end, 0))
        branches.append(Branch(start, end, qi, tuple(range(len(q.options))), tuple(option_positions), end - 1, q.kind))
    return _finish(tokens, positions, segments, branches, s, tuple(len(q.options) for q in questions))


def _finish(tokens, positions, segments, branches, state_length, option_counts):
    n = len(tokens)
    segment_ids = torch.zeros(n, dtype=torch.long)
    parents = torch.zeros(len(segments) + 1, dtype=torch.long)
    for index, (start, end, parent) in enumerate(segments, start=1):
        segment_ids[start:end] = index
        parents[index] = parent
    return PackedRequest(torch.tensor([tokens], dtype=torch.long), torch.tensor([positions], dtype=torch.long),
                         segment_ids, parents, branches, state_length, option_counts)


def tree_levels(segment_ids, parents):
    """Segments grouped by depth, [(segment, start, end)] per level (janus/hybrid.py:128-153): level 0 is the state,
    level d the children of level d-1. Raises ValueError for an empty or non-contiguous segment or a parent that
    does not precede its child."""
    seg = np.asarray(segment_ids.cpu() if torch.is_tensor(segment_ids) else segment_ids)
    par = np.asarray(parents.cpu() if torch.is_tensor(parents) else parents)
    count = par.shape[0]
    starts = np.full(count, -1, dtype=np.int64)
    ends = np.full(count, -1, dtype=np.int64)
    sizes = np.bincount(seg, minlength=count) if seg.size else np.zeros(count, dtype=np.int64)
    if seg.size:
        change = np.flatnonzero(np.diff(seg)) + 1
        run_starts = np.concatenate([[0], change])
        run_ends = np.concatenate([change, [seg.size]])
        for a, b in zip(run_starts, run_ends):
            s = int(seg[a])
            if s >= count or s < 0:
                raise ValueError(f"segment id {s} out of range")
            if starts[s] >= 0:
                raise ValueError(f"segment {s} is not contiguous")
            starts[s], ends[s] = a, b
    depth = [0] * count
    levels = {}
    for s in range(count):
        if sizes[s] == 0 or starts[s] < 0:
            raise ValueError(f"segment {s} has no tokens")
        p = int(par[s])
        if s > 0:
            if p >= s:
                raise ValueError("a segment's parent must precede it")
            depth[s] = depth[p] + 1
        levels.setdefault(depth[s], []).append((s, int(starts[s]), int(ends[s])))
    return [levels[d] for d in range(max(depth) + 1)]
