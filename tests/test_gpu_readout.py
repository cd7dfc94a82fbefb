"""The full B200 readout against the reference's own probabilities (golden fixtures) and the CPU oracle.

Per question the fixtures hold three probability vectors, all from seeded weights and requests:

- p_ref:  the reference (janus.hybrid.HybridBackbone + the janus.model heads) in fp32: the truth;
- p_ref16: the same reference readout with its backbone cast to bf16 (its plain CPU path);
- p_o16:  the CPU oracle with bf16 storage (oracle/hybrid.py `Oracle(storage="bf16")`): the reference's algorithm
          with every tensor the B200 path keeps in bf16 between its kernels rounded at that point, the rest fp32.
          The oracle itself is pinned to p_ref (fp32 storage: 2e-5, tests/test_oracle.py).

On these random-init models the bf16 rounding of the stored tensors alone moves probabilities by up to ~1e-2 at the
0.8B/4B widths (p_o16 against p_ref; rounding one class of tensors at a time on the CPU shows no single dominant
one: the DeltaNet projections, the normed GEMM inputs, q/k/v and the delta rule's output each move the 4B-width case
by 1.5-4e-3), the reference's own bf16 run by as much, and the MoE widths by ~0.1 (top-k routing near-ties flip
under any rounding). No bf16 path meets 2e-3 against the fp32 truth on these models; the gates are therefore the
north star's 2e-3 where the model's bf16 noise floor is below it, and that floor otherwise:

- per case: max |p - p_ref| <= max(2e-3, 1.5 x floor), floor = the larger of max |p_ref16 - p_ref| and
  max |p_o16 - p_ref| (the same for the RMS);
- argmax(p) == argmax(p_ref) wherever p_ref's top-2 margin exceeds twice that bound;
- over all cases: RMS |p - p_ref| <= 1.25 x RMS |p_ref16 - p_ref| (the B200 path is about as close to the fp32 truth
  as the reference's own bf16 run).
Each case prints max and RMS of |p - p_ref|, |p - p_ref16|, |p_ref16 - p_ref|, |p_o16 - p_ref| and |p - p_o16|.

Cases: the small golden set (tests/golden/readout_cases.json: tiny models and 4-layer slices at 0.8B/4B/A3B
widths) and the benchmark configurations (tests/golden/readout_full.json): cfg 2 (0.8B, 24 layers, 2048-token
state, listwise), cfg 3 (4B, 32 layers, 8192-token state, 8 tree questions), cfg 4 (0.8B, 24 layers, the
255-option stress pack on a 4096-token state), cfg 5 at A3B widths with all 256 experts at 4 layers.
"""

import numpy as np
import pytest

from tests.golden_cases import case_model, full_case_model, load_cases, load_full_cases

pytestmark = pytest.mark.gpu
PROB_ATOL = 2e-3
SMALL = load_cases()
FULL = load_full_cases()
_RESULTS = {}
_REPORT = {}


def _flat(per_pack):
    return np.concatenate([np.asarray(p, dtype=np.float64).ravel() for per in per_pack for p in per])


def _margins(per_pack):
    out = []
    for per in per_pack:
        for p in per:
            p = np.sort(np.asarray(p, dtype=np.float64))
            out.append(p[-1] - p[-2] if p.size > 1 else 1.0)
    return np.array(out)


def _argmax(per_pack):
    return np.array([int(np.argmax(p)) for per in per_pack for p in per])


def _cuda(shape, weights, mode, packs):
    from janus_b200.model import DecisionReadout
    model = DecisionReadout(shape, weights, mode)
    return [[p.numpy() for p in per] for per in model.probabilities(packs)]


def _check(name, got, ref, ref16, o16):
    d = lambda a, b: (float(np.abs(_flat(a) - _flat(b)).max()), float(np.sqrt(np.mean((_flat(a) - _flat(b)) ** 2))))
    rows = {"|p-p_ref|": d(got, ref), "|p-p_ref16|": d(got, ref16), "|p_ref16-p_ref|": d(ref16, ref),
            "|p_o16-p_ref|": d(o16, ref), "|p-p_o16|": d(got, o16)}
    print(f"\n{name}: " + "; ".join(f"{k} max {m:.2e} rms {r:.2e}" for k, (m, r) in rows.items()))
    _REPORT[name] = (got, ref, ref16)
    floor_max = max(rows["|p_ref16-p_ref|"][0], rows["|p_o16-p_ref|"][0])
    floor_rms = max(rows["|p_ref16-p_ref|"][1], rows["|p_o16-p_ref|"][1])
    bound = max(PROB_ATOL, 1.5 * floor_max)
    worst, rms = rows["|p-p_ref|"]
    assert worst <= bound, f"{name}: max |p - p_ref| = {worst:.2e} > {bound:.2e}"
    assert rms <= max(PROB_ATOL, 1.5 * floor_rms), f"{name}: rms |p - p_ref| = {rms:.2e}"
    clear = _margins(ref) > 2 * bound
    assert np.array_equal(_argmax(got)[clear], _argmax(ref)[clear]), name


@pytest.mark.parametrize("name", sorted(SMALL))
def test_readout_small_cases(name):
    from oracle import hybrid as oracle
    case = SMALL[name]
    shape, weights, mode, packs = case_model(case)
    got = _cuda(shape, weights, mode, packs)
    model16 = oracle.Oracle(shape, weights, storage="bf16")
    o16 = [[p.numpy() for p in oracle.probabilities(model16.logits(pack, mode))] for pack in packs]
    _check(name, got, case["probs"], case["probs_bf16"], o16)


@pytest.mark.parametrize("name", sorted(FULL))
def test_readout_benchmark_configs(name):
    case = FULL[name]
    shape, weights, mode, packs = full_case_model(case)
    got = _cuda(shape, weights, mode, packs)
    del weights
    _check(name, got, case["probs"], case["probs_bf16"], case["probs_oracle_bf16"])


def test_aggregate_deviation_is_within_the_reference_bf16_noise():
    """Runs after the per-case tests (same module): over every case they ran, the B200 path is about as close to the
    fp32 reference as the reference's own bf16 run (within 25% in RMS)."""
    if not _REPORT:
        pytest.skip("no readout case ran")
    ours = np.concatenate([_flat(g) - _flat(r) for g, r, _ in _REPORT.values()])
    theirs = np.concatenate([_flat(r16) - _flat(r) for _, r, r16 in _REPORT.values()])
    rms = lambda x: float(np.sqrt(np.mean(x ** 2)))
    print(f"\nRMS |p - p_ref| over {len(_REPORT)} cases: janus_b200 {rms(ours):.3e}, reference bf16 {rms(theirs):.3e}")
    assert rms(ours) <= 1.25 * rms(theirs)


def test_batch_composition_does_not_change_results():
    """A request's probabilities do not depend on the other requests of its batch (rows are independent)."""
    from janus_b200.model import DecisionReadout
    case = SMALL["tiny_tree"]
    shape, weights, mode, packs = case_model(case)
    model = DecisionReadout(shape, weights, mode)
    both = model.probabilities(packs)
    alone = model.probabilities(packs[1:])
    for a, b in zip(both[1], alone[0]):
        np.testing.assert_allclose(a.numpy(), b.numpy(), atol=1e-6)
