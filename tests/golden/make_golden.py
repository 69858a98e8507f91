"""Regenerate ``reference_cases.json`` from the dflash-mlx test sources.

The reference's tests need MLX (Apple only), so they cannot run here; their
literal test data are read from the source text with ``ast`` (nothing is
imported or executed) and stored as a fixture the CPU and GPU tests load:

* ``tests/test_engine_acceptance.py``   -- the acceptance-length table;
* ``tests/test_verify_qmm_parity.py``   -- REAL_MLP_SHAPES, REAL_MLP_M4_SHAPES,
  the random-shape generator's constants (seed, M levels, K/N ranges) and the
  tolerances;
* ``tests/test_verify_linear_parity.py`` -- the eligibility fixture shapes.

Usage: ``python tests/golden/make_golden.py <path to the dflash-mlx checkout>``.
"""

from __future__ import annotations

import ast
import json
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent / "reference_cases.json"


def _module(path: Path) -> ast.Module:
    return ast.parse(path.read_text(), filename=str(path))


def _assigned(tree: ast.AST, name: str):
    for node in ast.walk(tree):
        if isinstance(node, ast.Assign):
            for t in node.targets:
                if isinstance(t, ast.Name) and t.id == name:
                    return ast.literal_eval(node.value)
                if isinstance(t, ast.Tuple):  # a, b = 1, 2
                    names = [e.id for e in t.elts if isinstance(e, ast.Name)]
                    if name in names:
                        return ast.literal_eval(node.value)[names.index(name)]
    raise KeyError(name)


def _function(tree: ast.AST, name: str) -> ast.FunctionDef:
    for node in ast.walk(tree):
        if isinstance(node, ast.FunctionDef) and node.name == name:
            return node
    raise KeyError(name)


def _int_calls(fn: ast.FunctionDef, attr: str):
    """Constant arguments of every ``<x>.<attr>(a, b)`` call inside fn."""
    out = []
    for node in ast.walk(fn):
        if isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute) and node.func.attr == attr:
            out.append([ast.literal_eval(a) for a in node.args])
    return out


def main(ref: Path) -> None:
    tests = ref / "tests"
    acc = _module(tests / "test_engine_acceptance.py")
    cases = _assigned(_function(acc, "test_acceptance_length_cases"), "cases")
    qmm = _module(tests / "test_verify_qmm_parity.py")
    gen = _function(qmm, "_gen_random_shapes")
    defaults = [ast.literal_eval(d) for d in gen.args.defaults]
    ranges = _int_calls(gen, "integers")
    lin = _module(tests / "test_verify_linear_parity.py")
    small = _function(lin, "small_ql")
    large = _function(lin, "test_eligibility_rejects_large_N")
    data = {
        "source": "dflash-mlx tests (literal data read with ast)",
        "acceptance_cases": [{"drafted": d, "posterior": p, "expected": e} for d, p, e in cases],
        "qmm_group_size": _assigned(qmm, "GROUP_SIZE"),
        "qmm_bits": _assigned(qmm, "BITS"),
        "qmm_real_mlp_shapes": _assigned(qmm, "REAL_MLP_SHAPES"),
        "qmm_real_mlp_m4_shapes": _assigned(qmm, "REAL_MLP_M4_SHAPES"),
        "qmm_random_shapes": {"n": defaults[0], "seed": defaults[1],
                              "m_levels": _assigned(gen, "M_levels"),
                              "k_blocks_range": ranges[0], "n_blocks_range": ranges[1]},
        "qmm_tolerance_bf16": {"abs": 8e-3, "rel": 2e-2},
        "linear_small": {"in_dims": _assigned(small, "in_dims"), "out_dims": _assigned(small, "out_dims")},
        "linear_large_n": _int_calls(large, "Linear")[0][1],
    }
    OUT.write_text(json.dumps(data, indent=1) + "\n")
    print(f"wrote {OUT}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(Path(sys.argv[1]))
