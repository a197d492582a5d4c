"""Records the reference's own behaviour for tests/golden/reference_scenarios.py.

    python tests/golden/make_reference_golden.py REFERENCE_ROOT

REFERENCE_ROOT is the macrogpt-jax checkout (or set MACROGPT_JAX_REFERENCE).  The reference's
package imports JAX at the top of ueaj/utils/__init__.py and ueaj/model/einsum.py, which is not
installed here, so this script loads only pure-Python code from it, unchanged:
ueaj/utils/configurator.py as a standalone module, and the EinsumMetadata dataclass plus the
parse_einsum_expr / compute_weight_metadata functions of ueaj/model/einsum.py (their source,
extracted with ast and executed with the standard-library names they use); and the
constructor signatures of Einsum, GMLP, MLP and SoftmaxAttention (parsed, not executed).
Writes reference_behaviour.json next to this script; the reference is not read at test time.
"""
from __future__ import annotations

import ast
import importlib.util
import json
import operator
import os
import sys
from dataclasses import dataclass
from functools import reduce
from pathlib import Path
from typing import Dict, List, Tuple

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import reference_scenarios as sc  # noqa: E402


def load_configurator(root: Path):
    spec = importlib.util.spec_from_file_location("ref_configurator", root / "ueaj/utils/configurator.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def load_einsum_metadata(root: Path):
    src = (root / "ueaj/model/einsum.py").read_text()
    tree = ast.parse(src)
    keep = [n for n in tree.body if isinstance(n, (ast.ClassDef, ast.FunctionDef))
            and n.name in ("EinsumMetadata", "parse_einsum_expr", "compute_weight_metadata")]
    assert len(keep) == 3, "reference functions not found"
    ns = {"dataclass": dataclass, "Tuple": Tuple, "List": List, "Dict": Dict, "reduce": reduce,
          "operator": operator}
    exec(compile(ast.Module(body=keep, type_ignores=[]), "ueaj/model/einsum.py", "exec"), ns)
    return ns["parse_einsum_expr"], ns["compute_weight_metadata"]


def constructor_signatures(root: Path) -> dict:
    """Positional and keyword-only parameters with their default expressions (source text;
    None where there is no default) of the layer constructors on the path, read from the
    reference's source."""
    out = {}
    for rel, cls in (("ueaj/model/einsum.py", "Einsum"), ("ueaj/model/mlp.py", "GMLP"), ("ueaj/model/mlp.py", "MLP"),
                     ("ueaj/model/soft_attn.py", "SoftmaxAttention")):
        tree = ast.parse((root / rel).read_text())
        init = next(f for n in tree.body if isinstance(n, ast.ClassDef) and n.name == cls
                    for f in n.body if isinstance(f, ast.FunctionDef) and f.name == "__init__")
        a = init.args
        pos = [x.arg for x in a.args][1:]
        defaults = [None] * (len(pos) - len(a.defaults)) + [ast.unparse(d) for d in a.defaults]
        kw_defaults = [None if d is None else ast.unparse(d) for d in a.kw_defaults]
        out[cls] = {"positional": [[n, d] for n, d in zip(pos, defaults)],
                    "keyword_only": [[x.arg, d] for x, d in zip(a.kwonlyargs, kw_defaults)]}
    return out


def main() -> None:
    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MACROGPT_JAX_REFERENCE")
    if not arg:
        raise SystemExit("usage: make_reference_golden.py REFERENCE_ROOT (or set MACROGPT_JAX_REFERENCE)")
    root = Path(arg)
    cfg = load_configurator(root)
    parse, meta = load_einsum_metadata(root)
    out = {"configurator": sc.configurator_results(cfg.config, cfg.override),
           "einsum": sc.metadata_results(parse, meta),
           "constructors": constructor_signatures(root)}
    (HERE / "reference_behaviour.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print("wrote", HERE / "reference_behaviour.json")


if __name__ == "__main__":
    main()
