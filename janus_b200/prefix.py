"""Prefix snapshots: what a request's state segment (level 0) leaves for its branch levels, so a repeated state is
run once and its questions are answered from the snapshot (janus/hybrid.py:1641-1646 `encode_prefixes`,
:1898-1906 `PrefixSnapshot`; the serving cache of janus/server.py:98-136 `PrefixCache`).

A snapshot holds, per layer and on the device, exactly what the children of the state row read in place:
DeltaNet layers the conv tail [K-1, C] (bf16) and the recurrent state [Hv, Dk, Dv] (fp32) after the state's last
token, attention layers the keys and values [tokens, Hkv, D] (bf16) of the state. `DecisionReadout.encode_prefixes`
makes them (copied out of the level batch, so they outlive it); `DecisionReadout.prepare(packs, prefixes=...)`
stacks them back into a level-0 batch in pack order and the pass starts at level 1.
"""

import math

import numpy as np
import torch


class PrefixSnapshot:
    """The per-layer states after a state's last token. `states[i]` is (conv tail, recurrent state) for a DeltaNet
    layer and (keys, values) for an attention layer (`attention[i]` True); `ids` the state's token ids (host int32),
    checked against the pack a snapshot is used for; `bytes` its device memory and `kv_bytes` the part that grows
    with the token count (the attention keys and values)."""

    def __init__(self, states, attention, ids):
        self.states = list(states)
        self.attention = [bool(a) for a in attention]
        if len(self.states) != len(self.attention):
            raise ValueError("one (state, state) pair per layer")
        self.ids = np.array(ids, dtype=np.int32).reshape(-1)
        self.tokens = int(self.ids.shape[0])
        self.bytes = sum(t.numel() * t.element_size() for s in self.states for t in s)
        self.kv_bytes = sum(t.numel() * t.element_size() for s, a in zip(self.states, self.attention) if a for t in s)

    @property
    def device(self):
        return self.states[0][0].device if self.states else None


def stack_level0(snapshots, attention):
    """The level-0 entry of the pass history for a batch whose every pack comes with a snapshot (rows in pack
    order): per layer the DeltaNet tails and states stacked on a new row axis, the attention keys and values
    concatenated along the tokens (the level's token order)."""
    out = []
    for i, att in enumerate(attention):
        first = [s.states[i][0] for s in snapshots]
        second = [s.states[i][1] for s in snapshots]
        out.append((torch.cat(first), torch.cat(second)) if att else (torch.stack(first), torch.stack(second)))
    return out


class PrefixCache:
    """LRU of prefix snapshots keyed by the caller (a hash of the state's tokens), capacity in tokens
    (janus/server.py:98-136). A snapshot is charged its tokens scaled by bytes / kv_bytes, i.e. its state tokens
    plus its fixed per-state memory (the DeltaNet matrices) expressed in tokens of attention keys and values, so the
    capacity bounds the device memory whatever the state lengths. Not thread-safe: one inference thread uses it."""

    def __init__(self, capacity):
        self.capacity = capacity
        self.entries = {}  # key -> (snapshot, charge); insertion order is the recency order
        self.charged = self.hits = self.misses = 0

    @staticmethod
    def charge(snapshot):
        if snapshot.kv_bytes <= 0:
            return snapshot.tokens
        return math.ceil(snapshot.bytes * snapshot.tokens / snapshot.kv_bytes)

    def get(self, key):
        entry = self.entries.pop(key, None)
        if entry is None:
            self.misses += 1
            return None
        self.entries[key] = entry  # back to the most recent end
        self.hits += 1
        return entry[0]

    def put(self, key, snapshot):
        charge = self.charge(snapshot)
        if charge > self.capacity:
            return
        old = self.entries.pop(key, None)
        if old is not None:
            self.charged -= old[1]
        while self.entries and self.charged + charge > self.capacity:
            self.charged -= self.entries.pop(next(iter(self.entries)))[1]
        self.entries[key] = (snapshot, charge)
        self.charged += charge

    def clear(self):
        self.entries.clear()
        self.charged = self.hits = self.misses = 0

    def snapshot(self):
        entries = list(self.entries.values())
        return {"entries": len(entries), "tokens": sum(s.tokens for s, _ in entries), "charged_tokens": self.charged,
                "capacity_tokens": self.capacity, "bytes": sum(s.bytes for s, _ in entries), "hits": self.hits,
                "misses": self.misses}
