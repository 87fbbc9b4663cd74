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
    # plus the module attributes Python defines for every module
    defined = set(top.get_identifiers()) | {"__file__", "__name__", "__doc__", "__spec__",
                                             "__package__", "__loader__"}
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


def _sources():
    tests = sorted(f for f in os.listdir(os.path.join(ROOT, "tests")) if f.endswith(".py"))
    return FILES + [os.path.join("tests", f) for f in tests]


@pytest.mark.parametrize("rel", _sources())
def test_no_undefined_names(rel):
    assert undefined_globals(os.path.join(ROOT, rel)) == []


# Module aliases whose attributes the GPU-only code paths use; every
# attribute read through them must exist (run on the CPU, these paths never
# execute, so a misspelt or removed name would only show on a B200).
MODULES = {"megacu_b200": "megacu_b200", "mb": "megacu_b200", "_capi": "megacu_b200._capi",
           "oracle_lib": "oracle_lib", "measure": "megacu_b200.measure",
           "build": "megacu_b200.build", "timeline": "megacu_b200.timeline",
           "shapes_bench": "megacu_b200.shapes_bench", "gpu_util": "gpu_util"}


def missing_attributes(path):
    import ast
    import importlib

    tree = ast.parse(open(path).read())
    aliases = {}
    for node in ast.walk(tree):
        if isinstance(node, ast.Import):
            for a in node.names:
                name = a.asname or a.name
                if a.name in MODULES.values():
                    aliases[name] = a.name
        elif isinstance(node, ast.ImportFrom) and node.module:
            for a in node.names:
                full = f"{node.module}.{a.name}"
                if full in MODULES.values():
                    aliases[a.asname or a.name] = full
    missing = []
    for node in ast.walk(tree):
        if (isinstance(node, ast.Attribute) and isinstance(node.value, ast.Name)
                and node.value.id in aliases):
            mod = importlib.import_module(aliases[node.value.id])
            if not hasattr(mod, node.attr):
                missing.append(f"{node.value.id}.{node.attr} (line {node.lineno})")
    return missing


@pytest.mark.parametrize("rel", _sources())
def test_module_attributes_exist(rel):
    assert missing_attributes(os.path.join(ROOT, rel)) == []


def bad_calls(path):
    """Calls `alias.f(...)` into the modules above whose keyword names or
    positional count do not fit f's signature (classes: their __init__)."""
    import ast
    import importlib
    import inspect

    tree = ast.parse(open(path).read())
    aliases = {}
    for node in ast.walk(tree):
        if isinstance(node, ast.Import):
            for a in node.names:
                if a.name in MODULES.values():
                    aliases[a.asname or a.name] = a.name
    bad = []
    for node in ast.walk(tree):
        if not (isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute)
                and isinstance(node.func.value, ast.Name) and node.func.value.id in aliases):
            continue
        mod = importlib.import_module(aliases[node.func.value.id])
        fn = getattr(mod, node.func.attr, None)
        if fn is None or not callable(fn):
            continue
        try:
            sig = inspect.signature(fn)
        except (TypeError, ValueError):
            continue  # ctypes functions and builtins
        if any(isinstance(a, ast.Starred) for a in node.args) or any(
                k.arg is None for k in node.keywords):
            continue
        try:
            sig.bind(*range(len(node.args)), **{k.arg: None for k in node.keywords})
        except TypeError as exc:
            bad.append(f"{node.func.value.id}.{node.func.attr} line {node.lineno}: {exc}")
    return bad


@pytest.mark.parametrize("rel", _sources())
def test_calls_fit_signatures(rel):
    assert bad_calls(os.path.join(ROOT, rel)) == []


def _ast_signature(fn):
    """inspect.Signature of an ast.FunctionDef (defaults as placeholders)."""
    import inspect
    P = inspect.Parameter
    a = fn.args
    positional = [(x, P.POSITIONAL_ONLY) for x in a.posonlyargs] + \
                 [(x, P.POSITIONAL_OR_KEYWORD) for x in a.args]
    first_default = len(positional) - len(a.defaults)
    params = [P(x.arg, kind, default=None if i >= first_default else P.empty)
              for i, (x, kind) in enumerate(positional)]
    if a.vararg:
        params.append(P(a.vararg.arg, P.VAR_POSITIONAL))
    for x, d in zip(a.kwonlyargs, a.kw_defaults):
        params.append(P(x.arg, P.KEYWORD_ONLY, default=P.empty if d is None else None))
    if a.kwarg:
        params.append(P(a.kwarg.arg, P.VAR_KEYWORD))
    return inspect.Signature(params)


def _importable(module):
    """Modules the check may import: this package and the test helpers."""
    return (module == "megacu_b200" or module.startswith("megacu_b200.")
            or os.path.exists(os.path.join(ROOT, "tests", module + ".py")))


def bad_bare_calls(path):
    """Calls `f(...)` by a bare name whose arguments do not fit f: f imported
    by `from <module> import f` (this package, relative imports included, or
    a test helper) or a function defined once in the file itself outside a
    class."""
    import ast
    import importlib
    import inspect

    tree = ast.parse(open(path).read())
    rel_dir = os.path.relpath(os.path.dirname(path), ROOT)
    package = "" if rel_dir in (".", "tests") else rel_dir.replace(os.sep, ".")
    sigs, assigned, defined = {}, set(), {}

    def visit(node, in_class):
        for child in ast.iter_child_nodes(node):
            if isinstance(child, (ast.FunctionDef, ast.AsyncFunctionDef)) and not in_class:
                defined.setdefault(child.name, []).append(child)
            if isinstance(child, ast.Name) and isinstance(child.ctx, ast.Store):
                assigned.add(child.id)
            if isinstance(child, ast.arg):
                assigned.add(child.arg)
            visit(child, isinstance(child, ast.ClassDef))

    visit(tree, False)
    for name, defs in defined.items():
        if len(defs) == 1 and name not in assigned and not defs[0].decorator_list:
            sigs[name] = _ast_signature(defs[0])
    for node in ast.walk(tree):
        if not isinstance(node, ast.ImportFrom):
            continue
        module = node.module or ""
        if node.level:
            base = package.split(".")[:len(package.split(".")) - (node.level - 1)]
            module = ".".join([*base, module] if module else base)
        if not _importable(module):
            continue
        mod = importlib.import_module(module)
        for a in node.names:
            obj = getattr(mod, a.name, None)
            name = a.asname or a.name
            if callable(obj) and not inspect.ismodule(obj) and name not in assigned:
                try:
                    sigs[name] = inspect.signature(obj)
                except (TypeError, ValueError):
                    pass
    bad = []
    for node in ast.walk(tree):
        if not (isinstance(node, ast.Call) and isinstance(node.func, ast.Name)
                and node.func.id in sigs):
            continue
        if any(isinstance(a, ast.Starred) for a in node.args) or any(
                k.arg is None for k in node.keywords):
            continue
        try:
            sigs[node.func.id].bind(*range(len(node.args)),
                                    **{k.arg: None for k in node.keywords})
        except TypeError as exc:
            bad.append(f"{node.func.id} line {node.lineno}: {exc}")
    return bad


@pytest.mark.parametrize("rel", _sources())
def test_bare_calls_fit_signatures(rel):
    assert bad_bare_calls(os.path.join(ROOT, rel)) == []


def test_bare_call_check_catches_a_mismatch(tmp_path):
    """The check itself: a wrong keyword, a missing argument and a surplus
    positional are each found, in a local function and an imported one."""
    src = tmp_path / "probe.py"
    src.write_text(
        "from megacu_b200.measure import interleaved\n"
        "def f(a, b=1, *, c):\n    return a\n"
        "f(1, c=2)\n"            # fits
        "f(1, d=2)\n"            # unknown keyword, c missing
        "f(c=1)\n"               # a missing
        "f(1, 2, 3, c=4)\n"      # surplus positional
        "interleaved([], 1, 1, None, None, 1, device=None)\n"   # fits
        "interleaved([], 1, 1, None, None)\n")                  # world missing
    found = bad_bare_calls(str(src))
    assert [x.split(" line ")[1].split(":")[0] for x in found] == ["5", "6", "7", "9"], found


@pytest.mark.parametrize("argv", [["bench.py", "--help"],
                                  ["-m", "megacu_b200.shapes_bench", "--help"],
                                  ["-m", "megacu_b200.mlp_bench", "--help"],
                                  ["-m", "megacu_b200.timeline", "--help"]])
def test_tools_parse_their_arguments(argv):
    """The timing tools start and parse their options without a GPU."""
    import subprocess
    import sys
    proc = subprocess.run([sys.executable, *argv], cwd=ROOT, capture_output=True, text=True,
                          timeout=300)
    assert proc.returncode == 0 and "usage" in proc.stdout.lower(), proc.stderr[-2000:]


def test_same_process_team_sets_what_team_init_sets():
    """tests/gpu_util.same_process_team builds Team objects without __init__
    (one process, several GPUs): it must set every attribute __init__ sets,
    or the multi-GPU tests would fail only on a B200."""
    import ast

    def assigned(fn, name):
        out = set()
        for node in ast.walk(fn):
            targets = node.targets if isinstance(node, ast.Assign) else []
            for t in targets:
                elts = t.elts if isinstance(t, ast.Tuple) else [t]
                for x in elts:
                    if (isinstance(x, ast.Attribute) and isinstance(x.value, ast.Name)
                            and x.value.id == name):
                        out.add(x.attr)
        return out

    api = ast.parse(open(os.path.join(ROOT, "megacu_b200", "api.py")).read())
    team = next(n for n in api.body if isinstance(n, ast.ClassDef) and n.name == "Team")
    init = next(n for n in team.body if isinstance(n, ast.FunctionDef) and n.name == "__init__")
    util = ast.parse(open(os.path.join(ROOT, "tests", "gpu_util.py")).read())
    spt = next(n for n in util.body
               if isinstance(n, ast.FunctionDef) and n.name == "same_process_team")
    want = assigned(init, "self") - {"_finalizer"}  # close() tolerates its absence
    assert want and want <= assigned(spt, "t"), want - assigned(spt, "t")
