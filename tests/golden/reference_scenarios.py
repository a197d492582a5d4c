"""Behaviour scenarios for the pure-Python parts of the path's boundary, written once and run
twice: against the reference's own code (by make_reference_golden.py, which records the
results) and against this package (by tests/test_reference_golden.py, which compares).

Covered: `@config` / `.override()` / `override()` on functions and classes
(ueaj/utils/configurator.py), and `parse_einsum_expr` / `compute_weight_metadata` for the
Einsum expressions the reference's layers build (ueaj/model/einsum.py:81-147).
"""
from __future__ import annotations

from dataclasses import asdict

# (weight_expr, output_expr, batch_dims, size_dict) of the Einsums the reference builds:
# GMLP fused / down (ueaj/model/mlp.py:78-96), MLP up / down, attention k / v / q / o
# (ueaj/model/soft_attn.py:82-124), a fused QKV, and two made-up layouts.
METADATA_CASES = [
    ("idh", "ibnh", "i", {"i": 2, "d": 768, "h": 3072}),
    ("hd", "bnd", "", {"h": 3072, "d": 768}),
    ("dh", "bnh", "", {"d": 768, "h": 3072}),
    ("dhk", "bnhk", "", {"d": 2048, "h": 16, "k": 128}),
    ("dhik", "bnhik", "", {"d": 2048, "h": 8, "i": 2, "k": 128}),
    ("hivd", "bnd", "", {"h": 8, "i": 2, "v": 128, "d": 2048}),
    ("fdhk", "fbnhk", "f", {"f": 3, "d": 2048, "h": 16, "k": 128}),
    ("dvh", "bnvh", "", {"d": 64, "v": 3, "h": 5}),
    ("hdi", "ibnd", "i", {"h": 7, "d": 9, "i": 2}),
]

PARSE_CASES = ["bnd,idh->ibnh", "bnh,hd->bnd", " bnd , dh -> bnh ", "bnd,dh", "bnd,dh,hk->bnk", "bnd->bnh"]


def metadata_results(parse_einsum_expr, compute_weight_metadata) -> dict:
    out = {"metadata": [], "parse": []}
    for w, o, b, sizes in METADATA_CASES:
        m = asdict(compute_weight_metadata(w, o, b, sizes))
        out["metadata"].append({k: list(v) if isinstance(v, tuple) else v for k, v in m.items()})
    for expr in PARSE_CASES:
        try:
            out["parse"].append({"ok": list(parse_einsum_expr(expr))})
        except ValueError as e:
            out["parse"].append({"error": type(e).__name__})
    return out


def configurator_results(config, override) -> dict:
    out = {}

    @config
    def make(a, b=2, *, c=3):
        return [a, b, c]

    out["plain"] = make(1)
    f = make.override(b=5)
    out["override"] = f(1)
    out["override_beats_call_site"] = f(1, b=9)
    g = f.override(c=7)
    out["chained"] = [g(0), f(0)]
    out["chain_later_wins"] = make.override(b=5).override(b=6)(0)
    try:
        make.override(zz=1)
        out["bad_key"] = None
    except TypeError as e:
        out["bad_key"] = str(e)

    @config
    def outer(x, inner=make):
        return inner(x)

    out["nested_marker_on_function"] = outer.override(inner=override(b=11))(4)
    out["replace_default_function"] = outer.override(inner=make.override(c=0))(4)

    @config
    def takes_kwargs(a, **kw):
        return [a, sorted(kw.items())]

    out["kwargs_forwarding"] = takes_kwargs.override(extra=1, more="m")(0)

    class Thing:
        def __init__(self, x, inner=make, **kw):
            self.x, self.inner, self.kw = x, inner, kw

    Thing = config(Thing)

    def attempt(fn):
        try:
            return {"ok": fn()}
        except TypeError:
            return {"error": "TypeError"}

    def summary(t):
        return [t.x, sorted(t.kw.items()), t.inner(0)]

    out["class_override"] = attempt(lambda: summary(Thing.override(x=4, extra=1)()))
    out["class_override_beats_call_site_keyword"] = attempt(lambda: summary(Thing.override(extra=2)(0, extra=3)))
    out["class_override_and_positional"] = attempt(lambda: summary(Thing.override(x=4)(0)))
    out["class_replace_default_function"] = attempt(lambda: summary(Thing.override(inner=make.override(b=8))(1)))
    out["class_chained"] = attempt(lambda: summary(Thing.override(extra=1).override(extra=5, more=0)(2)))
    out["class_nested_marker_forwarded"] = attempt(
        lambda: list(Thing.override(inner=override(b=11))(1).inner[1].items()))
    out["class_factory_is_not_a_class"] = not isinstance(Thing.override(x=1), type)
    return out
