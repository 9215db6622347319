"""The C-ABI library: it loads, exports every entry point include/luna_b200.h
declares, and the ctypes mirror lays structures out as the C header does."""
import ctypes as C
import os
import re
import subprocess

import pytest

from luna_b200 import abi, engine

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "luna_b200.h")


def declared_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"LB200_API\s+\w+\s+(lb200_\w+)\s*\(", src)))


def test_header_declares_the_python_exports():
    assert set(declared_functions()) == set(engine.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = engine.load_library()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_options_default_matches_luna_defaults():
    lib = engine.load_library()
    o = abi.Options()
    assert lib.lb200_options_default(C.byref(o)) == 0
    ref = abi.default_options()
    for f, _ in abi.Options._fields_:
        assert getattr(o, f) == pytest.approx(getattr(ref, f)), f


def test_errors_are_reported_not_thrown():
    lib = engine.load_library()
    h = C.c_void_p()
    desc = abi.GraphDesc(0, None, 0, 0)
    assert lib.lb200_model_create(C.byref(desc), 0, C.byref(h)) != 0
    buf = C.create_string_buffer(256)
    lib.lb200_last_error(buf, 256)
    assert buf.value


def test_warm_start_entry_points_reject_missing_arguments():
    """The warm-start calls fail with a message, not a crash, on a null model
    or null outputs (no device is touched)."""
    lib = engine.load_library()
    buf = C.create_string_buffer(256)
    assert lib.lb200_set_warm_start(None, 1) != 0
    lib.lb200_last_error(buf, 256)
    assert b"null model" in buf.value
    parent = (C.c_int64 * 2)(0, 1)
    assert lib.lb200_set_warm_parents(None, parent, 2) != 0
    lib.lb200_last_error(buf, 256)
    assert b"null model" in buf.value
    rows, cols = C.c_int64(), C.c_int64()
    assert lib.lb200_warm_alpha(None, 1, 2, 0, None, 0, C.byref(rows), C.byref(cols), None) != 0
    lib.lb200_last_error(buf, 256)
    assert b"null argument" in buf.value


@pytest.mark.skipif(not os.path.exists("/usr/bin/gcc") and not os.path.exists("/opt/gcc/bin/gcc"),
                    reason="no C compiler")
def test_struct_layout_matches_header(tmp_path):
    prog = tmp_path / "layout.c"
    checks = []
    for st, cls in (("lb200_node_desc", abi.NodeDesc), ("lb200_graph_desc", abi.GraphDesc),
                    ("lb200_options", abi.Options), ("lb200_stats", abi.Stats)):
        checks.append(f'printf("{st} size %zu\\n", sizeof({st}));')
        for f, _ in cls._fields_:
            checks.append(f'printf("{st}.{f} %zu\\n", offsetof({st}, {f}));')
    prog.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "luna_b200.h"\nint main(void){'
                    + "\n".join(checks) + "return 0;}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(prog), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = dict(line.rsplit(" ", 1) for line in out if line)
    for st, cls in (("lb200_node_desc", abi.NodeDesc), ("lb200_graph_desc", abi.GraphDesc),
                    ("lb200_options", abi.Options), ("lb200_stats", abi.Stats)):
        assert int(got[f"{st} size"]) == C.sizeof(cls), st
        for f, _ in cls._fields_:
            assert int(got[f"{st}.{f}"]) == getattr(cls, f).offset, (st, f)


def test_shard_range_matches_the_host_sharding():
    """lb200_shard_range (the native multi-GPU split) and luna_b200.shard agree,
    cover every box once and differ in size by at most one."""
    from luna_b200.engine import shard_range as native
    from luna_b200.shard import shard_range as host
    for n in (0, 1, 7, 512, 1000):
        for world in (1, 2, 3, 8):
            spans = [native(r, world, n) for r in range(world)]
            assert spans == [host(r, world, n) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
