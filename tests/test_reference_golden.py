"""The boundary's pure-Python behaviour against the reference's own code: @config /
.override() / override() and the Einsum metadata functions, run through the same scenarios
(tests/golden/reference_scenarios.py) whose results make_reference_golden.py recorded by
executing the reference's configurator.py and einsum.py functions unchanged."""
import json
import sys
from pathlib import Path

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))

import reference_scenarios as sc  # noqa: E402

from macrogpt_jax_b200.configurator import config, override  # noqa: E402
from macrogpt_jax_b200.einsum import compute_weight_metadata, parse_einsum_expr  # noqa: E402


def _json(x):
    return json.loads(json.dumps(x, sort_keys=True))


def _reference():
    return json.loads((GOLDEN / "reference_behaviour.json").read_text())


def test_configurator_matches_reference():
    ref = _reference()["configurator"]
    ours = _json(sc.configurator_results(config, override))
    assert sorted(ours) == sorted(ref)
    for key in ref:
        assert ours[key] == ref[key], key


def test_einsum_metadata_matches_reference():
    ref = _reference()["einsum"]
    ours = _json(sc.metadata_results(parse_einsum_expr, compute_weight_metadata))
    assert ours["parse"] == ref["parse"]
    assert len(ours["metadata"]) == len(ref["metadata"])
    for case, got, want in zip(sc.METADATA_CASES, ours["metadata"], ref["metadata"]):
        assert got == want, case
