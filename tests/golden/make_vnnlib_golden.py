"""Record Luna's reading of the VNN-LIB corpus in tests/golden/vnnlib/.

Luna's own parser (VnnLibInputParser + OutputConstraintSet::toCMatrix,
compiled from the reference sources by oracle/Makefile, run through
oracle/_ref/luna_ref_vnnlib) reads every property of the corpus for the
network sizes listed below; its results are stored in
tests/golden/vnnlib_golden.json with every float as a hex literal.

    make -C oracle && python tests/golden/make_vnnlib_golden.py
"""
from __future__ import annotations

import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import luna_ref  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
CORPUS = os.path.join(HERE, "vnnlib")
OUT = os.path.join(HERE, "vnnlib_golden.json")

# (file, n_in, n_out): the network sizes each property is read for.
SIZES = [
    ("box_conjunction.vnnlib", 3, 4),
    ("or_branches.vnnlib", 2, 4),
    ("linear_exprs.vnnlib", 1, 3),
    ("quirks.vnnlib", 4, 3),
    ("crlf_no_final_newline.vnnlib", 1, 2),
    ("top_and_or.vnnlib", 1, 3),
    ("or_with_inputs.vnnlib", 2, 2),
    ("and_nested_desync.vnnlib", 2, 2),
    ("dropped_index.vnnlib", 1, 3),
    ("dropped_scalar.vnnlib", 1, 1),
    ("bad_input.vnnlib", 1, 1),
    ("joined_lines.vnnlib", 1, 1),
    ("inputs_only.vnnlib", 2, 2),
    ("empty.vnnlib", 2, 2),
    ("hex_and_inf.vnnlib", 2, 2),
]


def hexes(a):
    return [float(x).hex() for x in a.reshape(-1)]


def main():
    cases = []
    for name, n_in, n_out in SIZES:
        with open(os.path.join(CORPUS, name), "rb") as f:
            cases.append((f.read(), n_in, n_out))
    results = luna_ref.vnnlib_parse_many(cases)
    out = []
    for (name, n_in, n_out), r in zip(SIZES, results):
        e = {"file": name, "n_in": n_in, "n_out": n_out}
        if isinstance(r, ValueError):
            e["input_error"] = True
        else:
            e.update(input_error=False, lower=hexes(r["lower"]), upper=hexes(r["upper"]), C=hexes(r["C"]),
                     thresholds=hexes(r["thresholds"]), branches=r["branches"].tolist(),
                     nspec=int(r["C"].shape[0]), n_branches=int(r["n_branches"]),
                     spec_dropped=bool(r["spec_dropped"]))
        out.append(e)
    with open(OUT, "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")
    print(f"wrote {len(out)} properties to {OUT}")


if __name__ == "__main__":
    main()
