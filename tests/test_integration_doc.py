"""The code in INTEGRATION.md works as written (no GPU): the ctypes stub runs
a validate-only call (null stream) against the built library, and every C++
snippet compiles against include/ once its free variables are declared (the
co-resident one with nvcc, since it instantiates the device loop)."""
from __future__ import annotations

import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DOC = os.path.join(ROOT, "INTEGRATION.md")
FAKE = 0x100000  # never dereferenced: validate-only call


def blocks(lang):
    text = open(DOC).read()
    return [body for tag, body in re.findall(r"```(\w*)\n(.*?)```", text, re.S) if tag == lang]


def test_ctypes_stub_validates():
    (stub,) = blocks("python")
    env = {"stream_handle": None, "a_ptr": FAKE, "b_ptr": FAKE, "out_ptr": FAKE,
           "events_ptr": FAKE}
    exec(compile(stub, "INTEGRATION.md", "exec"), env)  # asserts st.code == 0 itself
    assert env["st"].code == 0 and env["prob"].dtype == 2


# Declarations of each snippet's free variables, keyed by a line the snippet
# starts with; the snippet becomes the body of one function.
PRELUDE = {
    "void *team = nullptr;\nmegacu_b200_team_create(": """
        int my_pe = 0, n_pes = 1, device = 0;
        int64_t heap_bytes = 1 << 20, partial_bytes = 4096, event_bytes = 4096;
        unsigned char const *all_handles = nullptr;
        cudaStream_t stream = nullptr;
        float const *a = nullptr, *b = nullptr;
        float *out = nullptr;
        gemm_ar_problem problem{};""",
    "void *team = nullptr;\nmegacu_status st = megacu_b200_team_create_local(": """
        int my_pe = 0, n_pes = 1, device = 0;
        int64_t heap_bytes = 1 << 20;""",
    "unsigned char mc_mine": """
        void *team = nullptr, *workspace = nullptr, *out = nullptr;
        int64_t ws_bytes = 4096, out_bytes = 4096;
        bool all_valid = true;
        unsigned char const *all_mc_handles = nullptr;""",
    "void *scratch = nullptr;\nmegacu_b200_noalloc_scratch(": """
        int device = 0;
        cudaStream_t stream = nullptr;
        void const *a = nullptr, *b = nullptr;
        void *out = nullptr;
        megacu_driver_view driver{};
        megacu_gemm_ar_problem_v2 problem{};""",
}

HEADERS = """
#include <cstdint>
#include <cuda_runtime.h>
#include <megacu_b200.h>
#include <megacu/gemm_allreduce.h>
"""

CO_RESIDENT_PRELUDE = """
namespace snippet {
struct driver_t {
  megacu::cuda::launch_view launch;
  megacu::nvshmem::team_view team;
};
struct ops_t {
  template <class Context, class Task, class Work>
  __device__ void invoke(Context, Task, Work) const {}
};
}  // namespace snippet
using namespace megacu::runtime;
"""

CO_RESIDENT_VARS = """
    snippet::driver_t driver{};
    megacu::scheduler::device::co_resident_state *state = nullptr;
    snippet::ops_t ops{};
    megacu::nvshmem::peer_table peers{};
    unsigned long long timeout_ns = 1000000000ull;
    int device = 0;
    cudaStream_t stream = nullptr;
"""


def _split_includes(body):
    inc = [x for x in body.splitlines() if x.startswith("#include")]
    rest = [x for x in body.splitlines() if not x.startswith("#include")]
    return "\n".join(inc), "\n".join(rest)


def _host_snippets():
    out = []
    for body in blocks("cpp"):
        for start, prelude in PRELUDE.items():
            if body.startswith(start.split("\n")[0]) and start.split("\n")[-1] in body:
                out.append((body, prelude))
                break
    return out


def test_every_cpp_snippet_is_checked():
    cpp = blocks("cpp")
    assert len(_host_snippets()) + sum("co_resident" in b for b in cpp) == len(cpp)


@pytest.mark.parametrize("i", range(4))
def test_host_snippet_compiles(tmp_path, i):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not found")
    body, prelude = _host_snippets()[i]
    src = tmp_path / "snippet.cc"
    src.write_text(f"{HEADERS}\nvoid snippet_{i}() {{\n{prelude}\n{body}\n}}\n")
    proc = subprocess.run([gxx, "-std=c++20", "-fsyntax-only", "-Wall",
                           "-I" + os.path.join(ROOT, "include"), "-I/usr/local/cuda/include",
                           str(src)], capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr[-3000:]


def test_co_resident_snippet_compiles(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not found")
    (body,) = [b for b in blocks("cpp") if "co_resident" in b]
    inc, rest = _split_includes(body)
    src = tmp_path / "snippet.cu"
    src.write_text(f"{HEADERS}\n#include <megacu/runtime.h>\n{inc}\n{CO_RESIDENT_PRELUDE}\n"
                   f"megacu::status snippet_co_resident() {{\n{CO_RESIDENT_VARS}\n{rest}\n"
                   f"  return st;\n}}\n")
    proc = subprocess.run([nvcc, "-std=c++20", "-gencode", "arch=compute_100a,code=sm_100a",
                           "-I" + os.path.join(ROOT, "include"), "-c", str(src), "-o",
                           str(tmp_path / "snippet.o")], capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr[-3000:]
