"""The C ABI library: loads, exports what include/megacu_b200.h declares, and
validates arguments the way megacu's launcher does (no GPU needed: a null
stream means "validate only", megacu_gemm_allreduce_phased.cu:160-165)."""
from __future__ import annotations

import ctypes
import os

import pytest

import megacu_b200 as mb
from megacu_b200 import _capi


def test_library_exports_every_declared_symbol():
    lib = _capi.load()
    names = _capi.declared_functions()
    assert len(names) >= 24
    for name in names:
        assert hasattr(lib, name), name
    assert lib.megacu_b200_version().startswith(b"megacu_b200")


def test_checked_build_exports_the_same_symbols():
    """The bounds-checked library (MEGACU_B200_LIBRARY=checked) is the same
    C ABI."""
    from megacu_b200 import build
    if not os.path.exists(build.CHECKED_LIB_PATH):
        pytest.skip("checked library not built")
    lib = ctypes.CDLL(build.CHECKED_LIB_PATH)
    for name in _capi.declared_functions():
        assert hasattr(lib, name), name


def test_component_link_anchors():
    """tests/build/runtime_components_contracts.cc:60-64."""
    lib = _capi.load()
    for name in ("megacu_dispatcher_explicit_attrs_component",
                 "megacu_scheduler_explicit_asap_component", "megacu_platform_cuda_component",
                 "megacu_backend_nvshmem_component", "megacu_target_runtime_component"):
        assert getattr(lib, name)() == 1


def _status(fn, *args):
    s = fn(*args)
    return s.code, s.detail


FAKE = 0x100000  # never dereferenced: validation-only calls


def test_f32_validation_only():
    """direct_orchestrate_smoke.cc: null stream + team of 2 -> ok, no launch."""
    d = mb.driver_view(None, 0)
    d.team.team_n_pes, d.team.world_n_pes = 2, 2
    p = _capi.GemmArProblem(m=1, n=1, k=1, tile_m=1, tile_n=1)
    lib = _capi.load()
    assert _status(lib.megacu_cuda_gemm_allreduce_f32_orchestrate, d, FAKE, FAKE, FAKE, FAKE,
                   FAKE, p) == (0, 0)
    assert _status(lib.megacu_cuda_gemm_allreduce_phased_f32, d, FAKE, FAKE, FAKE, FAKE, FAKE,
                   p) == (0, 0)
    bad = _capi.GemmArProblem(m=0, n=1, k=1, tile_m=1, tile_n=1)
    assert _status(lib.megacu_cuda_gemm_allreduce_phased_f32, d, FAKE, FAKE, FAKE, FAKE, FAKE,
                   bad) == (1, 1)
    assert _status(lib.megacu_cuda_gemm_allreduce_phased_f32, d, None, FAKE, FAKE, FAKE, FAKE,
                   p) == (1, 2)


def test_bf16_validation_only():
    lib = _capi.load()
    d = mb.driver_view(None, 0)
    good = mb.Problem(256, 512, 128).to_c()
    for fn in (lib.megacu_cuda_gemm_allreduce_bf16, lib.megacu_cuda_gemm_allreduce_bf16_orchestrate,
               lib.megacu_cuda_gemm_reduce_scatter_bf16):
        assert _status(fn, d, FAKE, FAKE, FAKE, FAKE, FAKE, good) == (0, 0)
    cases = [
        (mb.Problem(0, 512, 128), (1, 1)),
        (mb.Problem(256, 510, 128), (1, 21)),
        (mb.Problem(256, 512, 100), (1, 21)),
        (mb.Problem(256, 512, 128, tile_n=96), (2, 22)),
        (mb.Problem(256, 512, 128, mode=7), (1, 1)),
    ]
    for prob, want in cases:
        assert _status(lib.megacu_cuda_gemm_allreduce_bf16_orchestrate, d, FAKE, FAKE, FAKE, FAKE,
                       FAKE, prob.to_c()) == want
    p = mb.Problem(256, 512, 128).to_c()
    p.dtype = 3
    assert _status(lib.megacu_cuda_gemm_allreduce_bf16, d, FAKE, FAKE, FAKE, FAKE, FAKE, p) == (2, 20)
    # missing storage / misaligned
    assert _status(lib.megacu_cuda_gemm_allreduce_bf16, d, None, FAKE, FAKE, FAKE, FAKE,
                   good) == (1, 2)
    assert _status(lib.megacu_cuda_gemm_allreduce_bf16, d, FAKE + 2, FAKE, FAKE, FAKE, FAKE,
                   good) == (1, 21)
    # remote PEs without a team backend (megacu's detail 13)
    d2 = mb.driver_view(None, 0)
    d2.team.team_n_pes = 2
    assert _status(lib.megacu_cuda_gemm_allreduce_bf16, d2, FAKE, FAKE, FAKE, FAKE, FAKE,
                   good) == (2, 13)
    # reduce-scatter needs m divisible by tp * 128
    rs = mb.Problem(300, 512, 128).to_c()
    assert _status(lib.megacu_cuda_gemm_reduce_scatter_bf16, d, FAKE, FAKE, FAKE, FAKE, FAKE,
                   rs) == (2, 26)


@pytest.mark.parametrize("m,n,k,n_pes,mode", [(4096, 8192, 8192, 1, 0), (4096, 8192, 1024, 8, 0),
                                              (8192, 8192, 3584, 8, 1), (16, 8192, 3584, 8, 0),
                                              (2048, 4096, 1024, 2, 0)])
def test_plan_sizes(m, n, k, n_pes, mode):
    prob = mb.Problem(m, n, k, mode=mode)
    pl = mb.plan(prob, n_pes)
    assert pl.tile_m == 128 and pl.tile_n in (64, 128, 256)
    assert pl.m_tiles == -(-m // 128) and pl.n_tiles == -(-n // pl.tile_n)
    ws = mb.workspace_bytes(prob, n_pes)
    ev = mb.events_bytes(prob, n_pes)
    assert ev == 256 + 4 * (2 * n_pes * pl.tiles * 4 + 2 * n_pes)
    if n_pes == 1:
        assert ws == 0 and pl.slots_per_src == 0
    else:
        # each PE keeps its own partial of every tile, two parity planes
        assert pl.slots_per_src == pl.tiles
        assert ws == 2 * pl.tiles * 128 * pl.tile_n * pl.wire_bytes
        if mode == 0 and m <= 128:
            assert pl.one_shot


def test_status_layout_matches_cpp():
    assert ctypes.sizeof(_capi.Status) == 16
    assert ctypes.sizeof(_capi.DriverView) == 64
    assert ctypes.sizeof(_capi.GemmArProblem) == 32


def test_header_is_plain_c_and_links():
    """include/megacu_b200.h is a C header: a C99 translation unit that calls
    every declared function compiles warning-free and links against the
    library (the binding a C, cgo or FFI host would make)."""
    import shutil
    import subprocess
    import tempfile

    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("no C compiler")
    from megacu_b200 import build
    names = _capi.declared_functions()
    body = "\n".join(f"  (void)&{n};" for n in names)
    src = f"#include <megacu_b200.h>\nint main(void) {{\n{body}\n  return 0;\n}}\n"
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "abi.c")
        with open(path, "w") as f:
            f.write(src)
        cmd = [cc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror",
               "-I" + os.path.join(build.ROOT, "include"), path, "-L" + build.LIB_DIR,
               "-lmegacu_b200", "-o", os.path.join(tmp, "abi")]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        assert proc.returncode == 0, proc.stderr


def test_team_context_manager_closes_once():
    """`with Team(...) as t:` closes the team on exit; close() is idempotent
    (a team object without a handle, as after close(), does nothing)."""
    t = mb.Team.__new__(mb.Team)
    t.handle = None
    with t as same:
        assert same is t
    t.close()
    assert t.handle is None


def _c_declarations():
    """name -> (return kind, [parameter kinds]) of every function declared in
    include/megacu_b200.h."""
    import re
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    src = open(os.path.join(root, "include", "megacu_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    kinds = {
        "megacu_driver_view": "driver", "megacu_gemm_ar_problem": "problem",
        "megacu_gemm_ar_problem_v2": "problem_v2", "megacu_mlp_chain_problem": "chain_problem",
        "int32_t": "i32", "int64_t": "i64", "const char *": "str", "void **": "ptr*",
        "const void *const *": "ptr*", "int32_t *": "i32*", "int64_t *": "i64*",
        "uint64_t *": "u64*",
    }
    out = {}
    decl = r"\b(megacu_status|int|const char \*)\s*(megacu_\w+)\s*\(([^;{]*?)\)\s*;"
    for ret, name, params in re.findall(decl, src, re.S):
        got = []
        if params.strip() not in ("", "void"):
            for p in params.split(","):
                p = " ".join(p.split())
                array = re.match(r"(.*?)\s*\w+\[\d+\]$", p)
                t = array.group(1) + " *" if array else re.sub(r"\s*\b\w+$", "", p)
                t = t.replace("const ", "") if t not in kinds else t
                got.append(kinds.get(t, "ptr" if t.endswith("*") else t))
        out[name] = ({"megacu_status": "status", "int": "int"}.get(ret, "str"), got)
    return out


def test_ctypes_prototypes_match_the_c_header():
    """Every declared function has a ctypes prototype with the same return
    type and the same parameter count and kinds (a mismatch would pass
    garbage to the library only on a GPU call)."""
    import ctypes

    from megacu_b200 import _capi
    P = ctypes.POINTER
    kind_of = {_capi.DriverView: "driver", _capi.GemmArProblem: "problem",
               _capi.GemmArProblemV2: "problem_v2", _capi.MlpChainProblem: "chain_problem",
               ctypes.c_int32: "i32", ctypes.c_int64: "i64", ctypes.c_char_p: "str",
               ctypes.c_void_p: "ptr", P(ctypes.c_void_p): "ptr*", P(ctypes.c_int32): "i32*",
               P(ctypes.c_int64): "i64*", P(ctypes.c_uint64): "u64*"}
    decls = _c_declarations()
    assert len(decls) >= 40
    assert set(decls) == set(_capi._PROTOTYPES), set(decls) ^ set(_capi._PROTOTYPES)
    for name, (ret, params) in decls.items():
        res, args = _capi._PROTOTYPES[name]
        want = {_capi.Status: "status", ctypes.c_int: "int", ctypes.c_char_p: "str"}[res]
        assert want == ret, name
        assert [kind_of.get(a, repr(a)) for a in args] == params, name


def test_ctypes_struct_layouts_match_the_c_header(tmp_path):
    """Size and every field offset of the C ABI's structs, as the C compiler
    lays them out from include/megacu_b200.h, equal the ctypes mirrors'."""
    import shutil
    import subprocess

    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("no C compiler")
    from megacu_b200 import build
    structs = {"megacu_status": _capi.Status, "megacu_launch_view": _capi.LaunchView,
               "megacu_team_view": _capi.TeamView, "megacu_driver_view": _capi.DriverView,
               "megacu_gemm_ar_problem": _capi.GemmArProblem,
               "megacu_gemm_ar_problem_v2": _capi.GemmArProblemV2,
               "megacu_mlp_chain_problem": _capi.MlpChainProblem}
    lines, want = [], []
    for c_name, py in structs.items():
        lines.append(f'  printf("%zu\\n", sizeof({c_name}));')
        want.append(ctypes.sizeof(py))
        for field, _ in py._fields_:
            lines.append(f'  printf("%zu\\n", offsetof({c_name}, {field}));')
            want.append(getattr(py, field).offset)
    src = ("#include <stddef.h>\n#include <stdio.h>\n#include <megacu_b200.h>\n"
           "int main(void) {\n" + "\n".join(lines) + "\n  return 0;\n}\n")
    (tmp_path / "layout.c").write_text(src)
    exe = str(tmp_path / "layout")
    proc = subprocess.run([cc, "-std=c99", "-Wall", "-Werror",
                           "-I" + os.path.join(build.ROOT, "include"),
                           str(tmp_path / "layout.c"), "-o", exe], capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr
    got = [int(x) for x in subprocess.run([exe], capture_output=True, text=True,
                                          check=True).stdout.split()]
    assert got == want


def test_problem_struct_is_rebuilt_after_a_field_changes():
    """Problem.to_c caches the C struct of a call without a trace; changing a
    field must rebuild it, and a traced call always gets a fresh one."""
    p = mb.Problem(256, 512, 128)
    first = p.to_c()
    assert p.to_c() is first
    p.tile_n = 128
    again = p.to_c()
    assert again is not first and again.tile_n == 128 and first.tile_n == 0
    traced = p.to_c(0x1000, 4)
    assert traced.trace == 0x1000 and traced.trace_capacity == 4 and p.to_c() is again
    assert p == mb.Problem(256, 512, 128, tile_n=128)  # equality still compares fields only


@pytest.mark.parametrize("m,n,k,tile_n", [
    (16, 8192, 3584, 128),   # config 4: 64 tiles, each split over K between two CTAs
    (128, 8192, 3584, 128),
    (64, 1024, 1024, 64),    # 16 tiles of 64: split in two fills more SMs than wider tiles
    (1, 65536, 256, 256),    # 256 tiles of 256 already cover the SMs: no split
    (16, 8192, 64, 64),      # one k-block: no split; the narrowest tiles give the most CTAs
])
def test_one_tile_row_plan_width(m, n, k, tile_n):
    """One tile row (decode shapes): the plan picks the tile width that, with
    the K split the launcher may add, keeps the most SMs busy."""
    assert mb.plan(mb.Problem(m, n, k), 8).tile_n == tile_n
