"""Loads the golden fixtures written by tests/golden/make_golden.py (reference outputs on seeded inputs)."""

import json
from pathlib import Path

import torch

from janus_b200.config import SHAPES
from janus_b200.packing import Branch, PackedRequest
from janus_b200 import synthetic

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_cases():
    return json.loads((GOLDEN / "readout_cases.json").read_text())


def pack_from_dict(d):
    return PackedRequest(torch.tensor([d["input_ids"]]), torch.tensor([d["position_ids"]]),
                         torch.tensor(d["segment_ids"]), torch.tensor(d["parents"]),
                         [Branch(b["start"], b["end"], b["question_index"], tuple(b["option_indices"]),
                                 tuple(b["option_positions"]), b["decision_position"], b["kind"],
                                 tuple(tuple(x) for x in b["leaves"])) for b in d["branches"]],
                         d["state_length"], tuple(d["option_counts"]))


def case_model(case):
    """(shape, weights, mode, packs) of one golden case, weights regenerated from the seed and checked."""
    base = SHAPES[case["shape"]]
    over = dict(case["overrides"])
    layers = over.pop("layers", base.layers)
    shape = base.with_layers(layers, **over)
    weights = synthetic.make_weights(shape, seed=case["seed"], head="scalar" if case["mode"] == "tree" else "pointer")
    got = synthetic.weight_checksum(weights)
    assert abs(got - case["checksum"]) <= 1e-9 * max(1.0, abs(case["checksum"])), "weight generator drifted"
    return shape, weights, case["mode"], [pack_from_dict(p) for p in case["packs"]]


def load_full_cases():
    """The benchmark configurations at full depth (tests/golden/make_golden.py --full); {} if not generated."""
    path = GOLDEN / "readout_full.json"
    return json.loads(path.read_text()) if path.exists() else {}


def full_case_model(case, device="cpu"):
    """(shape, weights, mode, packs) of one full-size case: requests rebuilt from their seeds and checked against
    the stored crc of their ids, weights regenerated from the seed and checked."""
    import zlib
    base = SHAPES[case["shape"]]
    over = dict(case["overrides"])
    layers = over.pop("layers", base.layers)
    shape = base.with_layers(layers, **over)
    packs = []
    for r in case["requests"]:
        p = getattr(synthetic, r["builder"])(**r["kwargs"])
        assert zlib.crc32(p.input_ids[0].numpy().astype("int64").tobytes()) == r["ids_crc"], "request builder drifted"
        packs.append(p)
    weights = synthetic.make_weights(shape, seed=case["seed"], head="scalar" if case["mode"] == "tree" else "pointer",
                                     device=device, std=case.get("std"))
    got = synthetic.weight_checksum(weights)
    assert abs(got - case["checksum"]) <= 1e-9 * max(1.0, abs(case["checksum"])), "weight generator drifted"
    return shape, weights, case["mode"], packs
