"""Static check (no GPU): every name a function of bench.py, __graft_entry__.py
or the aestrix_b200 package reads as a global is defined at module level or is
a builtin. The bench's GPU paths only run on a B200, so a misspelled or
unimported name there would otherwise surface only at measurement time."""
import builtins
import os
import symtable

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FILES = ["bench.py", "__graft_entry__.py"] + [
    os.path.join("aestrix_b200", f) for f in sorted(os.listdir(os.path.join(ROOT, "aestrix_b200"))) if f.endswith(".py")
]


def _undefined(path):
    src = open(os.path.join(ROOT, path)).read()
    top = symtable.symtable(src, path, "exec")
    module_names = {s.get_name() for s in top.get_symbols() if s.is_assigned() or s.is_imported()}
    known = module_names | set(dir(builtins))
    bad = []

    def walk(tab, scope):
        for sym in tab.get_symbols():
            if tab.get_type() == "function" and sym.is_global() and sym.is_referenced():
                if sym.get_name() not in known:
                    bad.append(f"{scope}: {sym.get_name()}")
        for child in tab.get_children():
            walk(child, f"{scope}.{child.get_name()}")

    walk(top, path)
    return bad


@pytest.mark.parametrize("path", FILES)
def test_no_undefined_globals(path):
    assert _undefined(path) == []
