"""VNN-LIB properties: the engine's parser and verdict against Luna's.

Luna's own parser (VnnLibInputParser + OutputConstraintSet::toCMatrix) and
verdict (OutputConstraintSet::evaluateORBranches and the CLI's
evaluatePropertyStatus), compiled from the reference sources by
oracle/Makefile, are the ground truth: through the committed golden file for
the corpus in tests/golden/vnnlib/, and live on seeded random properties
(including unbalanced and otherwise malformed ones) when oracle/_ref is built.
Everything here runs on the CPU: parsing and the host verdict touch no GPU.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

from luna_b200 import abi
from luna_b200.engine import EngineError
from luna_b200.vnnlib import Property

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "vnnlib_golden.json")
CORPUS = os.path.join(HERE, "golden", "vnnlib")


def _ref():
    from oracle import luna_ref
    if not (luna_ref.available() and os.path.exists(luna_ref.PARSE_BIN)):
        pytest.skip("oracle/_ref is not built (make -C oracle)")
    return luna_ref


def _ours(text, n_in, n_out):
    try:
        return Property(text, n_in, n_out)
    except EngineError as e:
        assert "input bounds" in str(e), e
        return None


def _same(p: Property, r: dict) -> list[str]:
    """Names of the fields where our reading differs from Luna's (bitwise)."""
    diff = []
    for name, ours in (("lower", p.lower), ("upper", p.upper), ("C", p.C), ("thresholds", p.thresholds)):
        theirs = np.asarray(r[name], np.float32).reshape(ours.shape) if np.size(r[name]) == ours.size else None
        if theirs is None or ours.tobytes() != theirs.tobytes():
            diff.append(name)
    if p.branches.tolist() != list(np.asarray(r["branches"]).reshape(-1)):
        diff.append("branches")
    if p.n_branches != r["n_branches"]:
        diff.append("n_branches")
    if p.spec_dropped != r["spec_dropped"]:
        diff.append("spec_dropped")
    return diff


def test_corpus_matches_luna_golden():
    with open(GOLDEN) as f:
        golden = json.load(f)
    assert len(golden) >= 15
    for e in golden:
        with open(os.path.join(CORPUS, e["file"]), "rb") as f:
            text = f.read()
        p = _ours(text, e["n_in"], e["n_out"])
        if e["input_error"]:
            assert p is None, e["file"]
            continue
        assert p is not None, e["file"]
        r = {k: np.array([float.fromhex(x) for x in e[k]], np.float32) for k in ("lower", "upper", "C", "thresholds")}
        r.update(branches=e["branches"], n_branches=e["n_branches"], spec_dropped=e["spec_dropped"])
        assert p.nspec == e["nspec"], e["file"]
        assert _same(p, r) == [], (e["file"], _same(p, r))


def test_corpus_readings():
    """A few readings stated outright (they follow Luna's rules)."""
    read = lambda name, n_in, n_out: Property(open(os.path.join(CORPUS, name), "rb").read(), n_in, n_out)
    p = read("or_branches.vnnlib", 2, 4)
    assert p.n_branches == 3 and p.branches.tolist() == [0, 1, 2, 2]
    # (>= Y_0 Y_2) reads as -Y_0 + Y_2 <= 0.
    assert p.C[0].tolist() == [-1, 0, 1, 0] and p.thresholds[0] == 0
    p = read("quirks.vnnlib", 4, 3)
    assert p.C[0].tolist() == [1, 0, 0]          # (- Y_0): unary minus keeps the sign
    assert p.C[1].tolist() == [0, 2, 0]          # (* 2 Y_0 Y_1): the last variable takes the product
    assert p.C[2].tolist() == [0, 0, 1]          # (+ Y_2 Y_2): a column is stored, not summed
    assert p.lower[3] == -np.inf and p.upper[3] == np.inf  # X_7 is beyond 4 inputs
    p = read("and_nested_desync.vnnlib", 2, 2)
    assert p.lower[0] == -np.inf and p.upper[0] == np.inf  # the bounds after (+ ...) in the AND are not read
    assert read("dropped_index.vnnlib", 1, 3).spec_dropped
    assert not read("inputs_only.vnnlib", 2, 2).has_spec
    with pytest.raises(EngineError):
        read("bad_input.vnnlib", 1, 1)


# ------------------------------------------------------------------ fuzzing
_NUMS = ["0", "1", "-1", "0.5", "-0.25", "2.0", "1e-3", "-2.5E-1", "3E2", ".5", "-.75", "7.", "0x1p-3", "inf",
         "1e999", "-1e-320", "abc", "1.2.3", "1e", "1e-", "--1", "0.1", "1.000000059604644775390625"]
_GOOD_NUMS = _NUMS[:13] + ["0.1", "12.5", "-3"]


def _var(rng, prefix, n):
    k = int(rng.integers(0, n + 2))
    r = rng.random()
    if r < 0.03:
        return f"{prefix}__{k}"
    if r < 0.05:
        return f"_{prefix}_{k}"
    if r < 0.06:
        return f"{prefix}_{k}x"
    return f"{prefix}_{k}"


def _num(rng, bad_rate):
    pool = _NUMS if rng.random() < bad_rate else _GOOD_NUMS
    return pool[int(rng.integers(0, len(pool)))]


def _expr(rng, n_out, depth, bad):
    r = rng.random()
    if depth <= 0 or r < 0.35:
        return _var(rng, "Y", n_out) if rng.random() < 0.7 else _num(rng, bad)
    op = ["+", "-", "*"][int(rng.integers(0, 3))]
    k = int(rng.integers(1, 4))
    if op == "*":
        parts = [_num(rng, bad)] + [_expr(rng, n_out, depth - 1, bad) for _ in range(k - 1)]
        rng.shuffle(parts)
    else:
        parts = [_expr(rng, n_out, depth - 1, bad) for _ in range(k)]
    return f"({op} {' '.join(parts)})"


def _out_cmp(rng, n_out, bad):
    op = "<=" if rng.random() < 0.5 else ">="
    return f"({op} {_expr(rng, n_out, 2, bad)} {_expr(rng, n_out, 2, bad)})"


def _in_cmp(rng, n_in, bad):
    op = "<=" if rng.random() < 0.5 else ">="
    v, x = _num(rng, bad), _var(rng, "X", n_in)
    return f"({op} {x} {v})" if rng.random() < 0.7 else f"({op} {v} {x})"


def _property(rng, n_in, n_out):
    bad = 0.05 if rng.random() < 0.3 else 0.0
    lines = ["; generated"]
    for k in range(n_in + int(rng.integers(0, 2))):
        lines.append(f"(declare-const X_{k} {'Real' if rng.random() < 0.95 else 'Int'})")
    for k in range(n_out):
        lines.append(f"(declare-const Y_{k} Real)")
    for _ in range(int(rng.integers(0, 2 * n_in + 1))):
        lines.append(f"(assert {_in_cmp(rng, n_in, bad)})")
    if rng.random() < 0.3:
        lines.append("(assert (and " + " ".join(_in_cmp(rng, n_in, bad) for _ in range(3)) + "))")
    for _ in range(int(rng.integers(0, 3))):
        lines.append(f"(assert {_out_cmp(rng, n_out, bad)})")
    if rng.random() < 0.5:
        branches = []
        for _ in range(int(rng.integers(1, 4))):
            items = [_out_cmp(rng, n_out, bad) for _ in range(int(rng.integers(1, 3)))]
            if rng.random() < 0.3:
                items.append(_in_cmp(rng, n_in, bad))
            if rng.random() < 0.1:
                items.append(f"(or {_out_cmp(rng, n_out, bad)})")
            rng.shuffle(items)
            branches.append("(and " + " ".join(items) + ")" if rng.random() < 0.8 else items[0])
        lines.append("(assert (or " + " ".join(branches) + "))")
    if rng.random() < 0.2:
        lines.append("(check-sat)")
    if rng.random() < 0.1:
        lines.append("\t; tabbed comment")
    body = lines[1:]
    rng.shuffle(body)
    text = "\n".join(lines[:1] + body)
    if rng.random() < 0.1:
        text = text.replace("\n", "\r\n")
    if rng.random() < 0.2:
        # Malformed: drop or duplicate a parenthesis, or truncate.
        pos = [i for i, ch in enumerate(text) if ch in "()"]
        i = pos[int(rng.integers(0, len(pos)))]
        m = rng.random()
        text = text[:i] + text[i + 1:] if m < 0.4 else (text[:i] + text[i] + text[i:] if m < 0.8 else text[:i])
    return text


def test_fuzz_matches_luna():
    luna_ref = _ref()
    rng = np.random.default_rng(20240611)
    cases = []
    for _ in range(400):
        n_in, n_out = int(rng.integers(1, 6)), int(rng.integers(1, 6))
        cases.append((_property(rng, n_in, n_out), n_in, n_out))
    theirs = luna_ref.vnnlib_parse_many(cases)
    kinds = {"input_error": 0, "dropped": 0, "or": 0, "conj": 0, "none": 0}
    for (text, n_in, n_out), r in zip(cases, theirs):
        p = _ours(text, n_in, n_out)
        if isinstance(r, ValueError):
            assert p is None, text
            kinds["input_error"] += 1
            continue
        assert p is not None, (text, r)
        assert _same(p, r) == [], (text, _same(p, r))
        kinds["dropped" if p.spec_dropped else "or" if p.has_or else "conj" if p.has_spec else "none"] += 1
    # The generator reaches every kind of outcome.
    assert all(v > 5 for v in kinds.values()), kinds


# ------------------------------------------------------------------ verdicts
def _status_cases(rng, n_boxes, nspec, n_branches):
    thr = rng.normal(size=nspec).astype(np.float32)
    lb = (thr + rng.normal(size=(n_boxes, nspec)) - 1.5 - 0.3 * nspec).astype(np.float32)
    ub = (lb + 2 * np.abs(rng.normal(size=(n_boxes, nspec)))).astype(np.float32)
    # Ties, NaN and infinities.
    lb[rng.random(lb.shape) < 0.05] = np.nan
    ub[rng.random(ub.shape) < 0.05] = np.nan
    tie = rng.random(lb.shape) < 0.1
    lb[tie] = np.broadcast_to(thr, lb.shape)[tie]
    tie = rng.random(ub.shape) < 0.1
    ub[tie] = np.broadcast_to(thr, ub.shape)[tie]
    ub[rng.random(ub.shape) < 0.03] = np.inf
    lb[rng.random(lb.shape) < 0.03] = -np.inf
    branches = rng.integers(0, max(n_branches, 1), nspec).astype(np.int32)
    return lb, ub, thr, branches


def _host_status(lb, ub, thr, branches, n_branches):
    import ctypes as C
    from luna_b200.abi import fptr
    from luna_b200.engine import _check, load_library
    out = np.zeros(lb.shape[0], np.int32)
    ip = C.POINTER(C.c_int32)
    _check(load_library().lb200_property_status(fptr(lb), fptr(ub), lb.shape[0], lb.shape[1], fptr(thr),
                                                branches.ctypes.data_as(ip), n_branches, out.ctypes.data_as(ip)),
           "lb200_property_status")
    return out


def test_status_matches_luna():
    luna_ref = _ref()
    rng = np.random.default_rng(7)
    seen = {False: set(), True: set()}
    for nspec, n_branches in ((1, 0), (4, 0), (9, 0), (3, 2), (6, 3), (9, 9), (5, 7), (2, 1)):
        lb, ub, thr, br = _status_cases(rng, 300, nspec, n_branches)
        ours = _host_status(lb, ub, thr, br, n_branches)
        theirs = luna_ref.property_status(lb, ub, thr, br, n_branches)
        assert (ours == theirs).all(), (nspec, n_branches, np.nonzero(ours != theirs))
        seen[n_branches > 0] |= set(ours.tolist())
    assert seen[False] == seen[True] == {abi.STATUS_UNKNOWN, abi.STATUS_UNSAT, abi.STATUS_SAT}, seen


def test_status_rules():
    thr = np.zeros(2, np.float32)
    st = lambda lb, ub, br=(0, 0), nb=0: _host_status(np.array([lb], np.float32), np.array([ub], np.float32), thr,
                                                     np.array(br, np.int32), nb)[0]
    assert st([0.1, -5], [1, 1]) == abi.STATUS_UNSAT            # one row breaks the conjunction
    assert st([-1, -1], [0, 0]) == abi.STATUS_SAT               # ub <= thr everywhere
    assert st([-1, -1], [0, 0.5]) == abi.STATUS_UNKNOWN
    assert st([0.1, -1], [1, 0], (0, 1), 2) == abi.STATUS_SAT   # branch 1 always satisfiable
    assert st([0.1, 0.2], [1, 1], (0, 1), 2) == abi.STATUS_UNSAT
    assert st([-1, -1], [np.nan, np.nan]) == abi.STATUS_UNKNOWN          # NaN never satisfies a conjunction
    assert st([-1, -1], [np.nan, 1], (0, 1), 2) == abi.STATUS_SAT        # ... but does not block a branch
    assert st([-1, -1], [-1, -1], (0, 0), 2) == abi.STATUS_SAT           # branch 1 has no rows
    with pytest.raises(EngineError):
        st([0, 0], [1, 1], (0, 2), 2)                                    # branch id out of range


def test_property_status_method():
    p = Property(open(os.path.join(CORPUS, "or_branches.vnnlib"), "rb").read(), 2, 4)
    # Rows: branch 0 {0}, branch 1 {1}, branch 2 {2, 3} with thresholds 0, 0, 0, 10.
    lb = np.array([[0.1, 0.1, 0.1, -1], [0.1, 0.1, -1, -1], [0.1, 0.1, -1, -1]], np.float32)
    ub = lb + 1
    ub[2, 3] = 11
    assert p.status(lb, ub).tolist() == [abi.STATUS_UNSAT, abi.STATUS_SAT, abi.STATUS_UNKNOWN]
    assert p.status(lb[0], ub[0]) == abi.STATUS_UNSAT
