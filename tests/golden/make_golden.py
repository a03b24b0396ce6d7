"""Extracts the reference's known-answer vectors into tests/golden/reference_kats.json.

Run in a checkout where the reference tree is available:
    python tests/golden/make_golden.py /path/to/tt-thrml
The reference is read as text (its Python imports JAX/thrml, which cannot run
here); the literal values of its own known-answer tests are pulled out with
`ast` so the committed fixture is exactly what those tests assert:

* tests/test_compiler_lowering.py — flat gather offsets of the mixed program
  (KAT 1), the spin-with-categorical-source kernel (KAT 2), superblock
  simultaneity (KAT 3);
* scripts/probe_gather_pipeline.py — gather, field and threshold stage
  vectors (KATs 4-6).
"""

from __future__ import annotations

import ast
import json
import sys
from pathlib import Path


def _literal(node):
    """Literal value of a list/number expression, unwrapping jnp/np.asarray/array calls."""
    if isinstance(node, ast.Call) and node.args:
        return _literal(node.args[0])
    return ast.literal_eval(node)


def _assignments(fn: ast.FunctionDef) -> dict:
    out = {}
    for st in ast.walk(fn):
        if isinstance(st, ast.Assign) and len(st.targets) == 1 and isinstance(st.targets[0], ast.Name):
            try:
                out[st.targets[0].id] = _literal(st.value)
            except (ValueError, TypeError, SyntaxError):
                pass
    return out


def _functions(path: Path) -> dict:
    tree = ast.parse(path.read_text())
    return {n.name: n for n in ast.walk(tree) if isinstance(n, ast.FunctionDef)}


def lowering_kats(ref: Path) -> dict:
    src = ref / "tests" / "test_compiler_lowering.py"
    fns = _functions(src)
    kat1 = []
    for st in ast.walk(fns["test_mixed_program_global_slices_lower_to_flat_offsets"]):
        if isinstance(st, ast.Assert) and isinstance(st.test, ast.Compare):
            lhs = ast.unparse(st.test.left)
            # np.asarray(_spec_for(program, B).interactions[I].gather_indices[0]).tolist()
            call = st.test.left.func.value.args[0]  # _spec_for(...).interactions[I].gather_indices[0]
            inter_sub = call.value.value  # _spec_for(...).interactions[I]
            block = ast.literal_eval(inter_sub.value.value.args[1])
            inter = ast.literal_eval(inter_sub.slice)
            src_idx = ast.literal_eval(call.slice)
            kat1.append(
                {"block": block, "interaction": inter, "source": src_idx,
                 "expected": ast.literal_eval(st.test.comparators[0]), "expr": lhs}
            )
    fn2 = fns["test_spin_kernel_selects_categorical_source_axis"]
    a2 = _assignments(fn2)
    kat2 = {"block": 0, "rng": a2["rng"], "cases": []}
    for st in ast.walk(fn2):
        if isinstance(st, ast.Assert) and isinstance(st.test, ast.Compare):
            state_name = st.test.left.value.args[0].args[0].id  # np.asarray(kernel(<state>, rng))[0]
            kat2["cases"].append({"state": a2[state_name], "expected_out0": ast.literal_eval(st.test.comparators[0])})
    fn3 = fns["test_sampling_group_kernel_updates_blocks_simultaneously"]
    kat3 = {}
    for st in ast.walk(fn3):
        if isinstance(st, ast.Assign) and isinstance(st.targets[0], ast.Name) and st.targets[0].id == "out":
            args = st.value.args
            kat3["state"] = _literal(args[0])
            kat3["rng"] = [_literal(a) for a in args[1:]]
        if isinstance(st, ast.Expr) and isinstance(st.value, ast.Call) and "assert_array_equal" in ast.unparse(st.value.func):
            kat3["expected"] = _literal(st.value.args[1])
        if isinstance(st, ast.Call) and ast.unparse(st.func) == "SpinEBMFactor":
            kat3["coupling"] = _literal(st.args[1])
    return {"kat1_flat_offsets": kat1, "kat2_categorical_source": kat2, "kat3_superblock": kat3}


def probe_kats(ref: Path) -> dict:
    fns = _functions(ref / "scripts" / "probe_gather_pipeline.py")
    s1 = _assignments(fns["stage1_pure_gather"])
    s2 = _assignments(fns["stage2_gather_arith"])
    s3 = _assignments(fns["stage3_full_sweep"])
    return {
        "kat4_gather": {"global_state": s1["global_state_np"], "indices": s1["indices_np"]},
        "kat5_gamma": {
            "global_state": s2["global_state_np"],
            "indices": s2["gather_indices_np"],
            "weights": s2["weights_np"],
            "mask": s2["mask_np"],
        },
        "kat6_threshold": {
            "global_state": s3["global_state_np"],
            "indices": s3["gather_indices_np"],
            "weights": s3["weights_np"],
            "mask": s3["mask_np"],
            "rng": s3["rng_slice_np"],
            "compares": "gamma > rng",
        },
    }


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    ref = Path(sys.argv[1])
    if not (ref / "tests" / "test_compiler_lowering.py").exists():
        sys.exit(f"{ref} does not look like the reference checkout (tests/test_compiler_lowering.py missing)")
    out = {"source": "reference tests/test_compiler_lowering.py and scripts/probe_gather_pipeline.py"}
    out.update(lowering_kats(ref))
    out.update(probe_kats(ref))
    path = Path(__file__).with_name("reference_kats.json")
    path.write_text(json.dumps(out, indent=1) + "\n")
    print(path)


if __name__ == "__main__":
    main()
