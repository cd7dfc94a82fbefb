"""The wire step (janus_b200/wire.py) against the reference's own server functions, on CPU: for the same logits and
calibration file, the probability lists and the response envelope are identical (json text compared byte for byte).

Needs the reference checkout (REFERENCE_ROOT, default /root/reference) for the comparison; the fallback rules of
the temperature lookup are also checked on their own."""

import json
import os
import sys
from pathlib import Path

import pytest
import torch

from janus_b200 import wire

REFERENCE = Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))
HAVE_REF = (REFERENCE / "janus" / "server.py").exists()

CALIBRATION = {"temperature": 1.7, "by_kind": {"noul": 0.9},
               "by_family": {"medqa": {"temperature": 1.3, "by_cardinality": {"4": 1.1, "8": 2.5}},
                             "bool": {"temperature": 0.8}}}


def _bodies():
    choice = {"type": "choice", "instructions": "Pick one.", "criteria": {f"o{i}": f"option {i}" for i in range(7)}}
    score = {"type": "score", "instructions": "Rate it.", "criteria": ["bad", "fine", "good", "great"]}
    noul = {"type": "noul", "instructions": "Is it so?"}
    big = {"type": "choice", "instructions": "Pick.", "criteria": {f"k{i}": None for i in range(255)}}
    return [({"state": "s", "questions": {"a": choice, "b": score, "c": noul}, "group_id": "medqa:17"}, 11),
            ({"state": "s", "questions": {"x": noul, "y": big}, "group_id": "other"}, 900),
            ({"state": "s", "questions": {"q": score}, "group_id": "bool:1"}, 3)]


def test_temperature_lookup_falls_back_in_order():
    assert wire.bucket(1) == "2" and wire.bucket(2) == "2" and wire.bucket(3) == "4" and wire.bucket(8) == "8"
    assert wire.bucket(9) == "16" and wire.bucket(255) == "256"
    assert wire.temperature_for(CALIBRATION, "medqa", 4) == 1.1
    assert wire.temperature_for(CALIBRATION, "medqa", 2) == 1.3
    assert wire.temperature_for(CALIBRATION, "bool", 8) == 0.8
    assert wire.temperature_for(CALIBRATION, "x", 4, "noul") == 0.9
    assert wire.temperature_for(CALIBRATION, "x", 4, "choice") == 1.7


@pytest.mark.skipif(not HAVE_REF, reason="reference not present")
def test_probabilities_and_envelope_equal_the_reference_server():
    sys.path.insert(0, str(REFERENCE))
    from janus.calibration_sets import temperature_for
    from janus.schema import Request
    from janus.server import Worker, envelope, null_criteria
    g = torch.Generator().manual_seed(7)
    for body, tokens in _bodies():
        request = Request.from_dict(null_criteria(json.loads(json.dumps(body))))
        logits = [torch.randn(len(q.options), generator=g) * 3 for q in request.questions]
        fake = type("W", (), {"temperature": 1.7, "calibration": CALIBRATION})()
        temps_ref = Worker.temperatures(fake, request)
        temps = wire.temperatures(CALIBRATION, request)
        assert temps == temps_ref
        assert temps == [temperature_for(CALIBRATION, wire.family_of(request), len(q.options), q.kind)
                         for q in request.questions]
        for t in (None, temps):
            ref = Worker.probabilities(fake, logits, t)
            got = wire.probabilities(logits, t, default=1.7)
            assert json.dumps(got) == json.dumps(ref)
        dists = wire.probabilities(logits, temps)
        assert json.dumps(wire.envelope(request, dists, "janus-4b", tokens)) == \
            json.dumps(envelope(request, dists, "janus-4b", tokens))
