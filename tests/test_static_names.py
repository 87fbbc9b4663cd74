"""Every name the driver-facing scripts and the timing tools read is defined
(a static check, no GPU: these files' GPU paths cannot run on the CPU)."""
from __future__ import annotations

import builtins
import os
import symtable

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FILES = ["bench.py", "__graft_entry__.py", "megacu_b200/shapes_bench.py",
         "megacu_b200/mlp_bench.py", "megacu_b200/timeline.py", "megacu_b200/measure.py",
         "megacu_b200/api.py", "megacu_b200/build.py"]


def undefined_globals(path):
    src = open(path).read()
    top = symtable.symtable(src, path, "exec")
    defined = set(top.get_identifiers())
    missing = []

    def walk(table, where):
        for child in table.get_children():
            for sym in child.get_symbols():
                name = sym.get_name()
                if (sym.is_global() and not sym.is_assigned() and name not in defined
                        and not hasattr(builtins, name)):
                    missing.append(f"{where}{child.get_name()}: {name}")
            walk(child, f"{where}{child.get_name()}/")

    walk(top, "")
    return missing


@pytest.mark.parametrize("rel", FILES)
def test_no_undefined_names(rel):
    assert undefined_globals(os.path.join(ROOT, rel)) == []
