"""The calibration and wire step after the readout: temperatures per question, the temperature softmax as plain
Python lists, and the response envelope, byte for byte what the reference's server returns for the same logits.

What it reproduces (the outputs must be identical, so the arithmetic is the same torch / Python operations in the
same order):
- `probabilities`: `Worker.probabilities` (janus/server.py:277-282): the request's logits concatenated, one host
  copy in fp32, then per question softmax(z / T) as a list of Python floats;
- `temperature_for` / `temperatures`: janus/calibration_sets.py:13-18, 40-46 and `Worker.temperatures`
  (janus/server.py:237-242): (family, power-of-two cardinality bucket), then the family, then the question kind's
  entry, then the global temperature; the family is the request's group_id up to the first ':';
- `decode` / `envelope`: janus/schema.py:16-21, 158-174 and janus/server.py:66-87: per question the option
  probabilities keyed by option, the argmax option (choice) or the expected level and legend (score), the
  probability of "true" (noul), the largest probability as the confidence, and the usage block.
Requests are read by attribute (`questions`, each with `id`, `kind`, `options` of `key` / `description`; `group_id`),
so the reference's `janus.schema.Request` is taken as it is.
"""

import math

import torch


def bucket(cardinality):
    """The power-of-two cardinality bucket of a question with `cardinality` options ("2" for 1-2, "4" for 3-4, ...)."""
    n = max(1, (int(cardinality) - 1).bit_length())
    return str(1 << n)


def family_of(request):
    return getattr(request, "group_id", "").split(":", 1)[0]


def temperature_for(calibration, family, cardinality, kind=None):
    """The most specific temperature of a calibration dict: by_family[family].by_cardinality[bucket], then
    by_family[family].temperature, else by_kind[kind], else the global temperature."""
    fam = (calibration.get("by_family") or {}).get(family)
    if fam is not None:
        return fam.get("by_cardinality", {}).get(bucket(cardinality), fam["temperature"])
    return (calibration.get("by_kind") or {}).get(kind, calibration["temperature"])


def temperatures(calibration, request):
    """One temperature per question of `request`."""
    family = family_of(request)
    return [temperature_for(calibration, family, len(q.options), q.kind) for q in request.questions]


def probabilities(logits, temperatures=None, default=1.0):
    """Per question softmax(logits / T) as lists of floats. `logits`: one request's per-question logit tensors (any
    device: one copy to the host for all of them); `temperatures`: one per question, or None for `default`."""
    sizes = [int(z.numel()) for z in logits]
    flat = torch.cat([z.reshape(-1) for z in logits]).float().cpu()
    temps = [default] * len(sizes) if temperatures is None else temperatures
    return [(z / t).softmax(-1).tolist() for z, t in zip(flat.split(sizes), temps)]


def validate_distribution(values, size):
    vals = tuple(float(x) for x in values)
    ok = len(vals) == size and all(math.isfinite(x) and x >= 0 for x in vals) and math.isclose(sum(vals), 1, abs_tol=1e-5)
    if not ok:
        raise ValueError(f"Expected {size} finite nonnegative probabilities summing to one")
    return vals


def decode(request, distributions):
    """question id -> answer body: choice {probabilities, choice}, score {probabilities, score, legend}, noul: the
    probability of its second option."""
    if len(distributions) != len(request.questions):
        raise ValueError("Wrong number of question distributions")
    answers = {}
    for q, values in zip(request.questions, distributions):
        p = validate_distribution(values, len(q.options))
        if q.kind == "noul":
            answers[q.id] = p[1]
            continue
        body = {"probabilities": dict(zip((o.key for o in q.options), p))}
        if q.kind == "choice":
            best = max(range(len(p)), key=p.__getitem__)
            body["choice"] = q.options[best].key
        else:
            body["score"] = sum(i * x for i, x in enumerate(p))
            body["legend"] = {o.key: o.description for o in q.options}
        answers[q.id] = body
    return answers


def confidence(probabilities):
    return max(probabilities)


def envelope(request, distributions, model_id, input_tokens):
    """The response body of one request: model id, per question its typed answer (with the confidence except for
    noul), usage."""
    answers = decode(request, distributions)
    for q, p in zip(request.questions, distributions):
        if q.kind == "noul":
            answers[q.id] = {"type": "noul", "noul": answers[q.id]}
        else:
            answers[q.id] = {"type": q.kind, **answers[q.id], "confidence": confidence(p)}
    return {"model": model_id, "answers": answers, "usage": {"input_tokens": input_tokens, "output_tokens": 0}}
