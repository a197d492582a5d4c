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


def test_layer_constructors_match_reference_signatures():
    """Same positional parameters in the same order with the same defaults (a JAX default
    maps to its PyTorch counterpart), and the reference's keyword-only parameters first, with
    the same defaults; additions are keyword-only and come after them."""
    import inspect

    import torch

    from macrogpt_jax_b200.einsum import Einsum, lecun_normal_init
    from macrogpt_jax_b200.mlp import GMLP, MLP, swish
    from macrogpt_jax_b200.soft_attn import SoftmaxAttention

    same_as = {"jnp.bfloat16": torch.bfloat16, "nnx.swish": swish, "Einsum": Einsum,
               "lecun_normal_init": lecun_normal_init, "None": None, "''": "", "64": 64, "1": 1,
               "10000.0": 10000.0, "'sp'": "sp"}
    ref = _reference()["constructors"]
    for cls in (Einsum, GMLP, MLP, SoftmaxAttention):
        want = ref[cls.__name__]
        params = list(inspect.signature(cls.__init__).parameters.values())[1:]
        pos = [p for p in params if p.kind is inspect.Parameter.POSITIONAL_OR_KEYWORD]
        kwo = [p.name for p in params if p.kind is inspect.Parameter.KEYWORD_ONLY]
        assert [p.name for p in pos] == [n for n, _ in want["positional"]], cls.__name__
        for p, (name, default) in zip(pos, want["positional"]):
            if default is None:
                assert p.default is inspect.Parameter.empty, (cls.__name__, name)
            else:
                assert p.default == same_as[default], (cls.__name__, name)
        kw = {p.name: p for p in params if p.kind is inspect.Parameter.KEYWORD_ONLY}
        assert kwo[:len(want["keyword_only"])] == [n for n, _ in want["keyword_only"]], cls.__name__
        for name, default in want["keyword_only"]:
            if default is None:
                assert kw[name].default is inspect.Parameter.empty, (cls.__name__, name)
            else:
                assert kw[name].default == same_as[default], (cls.__name__, name)
