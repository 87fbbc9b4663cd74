"""Source-level drop-in: megacu's own orchestration source
(examples/cuda_nvshmem/gemm_allreduce/phased/megacu/
gemm_allreduce_phased_orchestrate.cc), compiled unchanged against this
repository's headers and linked with libmegacu_b200.so by oracle/Makefile
(oracle/_ref/libref_orchestrate_on_b200.so, built only where the reference
tree is present), answers like the reference: validate-only calls and
argument errors, no GPU needed."""
from __future__ import annotations

import ctypes
import os

import pytest

import megacu_b200 as mb
from megacu_b200 import _capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DROPIN = os.path.join(ROOT, "oracle", "_ref", "libref_orchestrate_on_b200.so")
FAKE = 0x100000  # never dereferenced: validation-only calls


def load_dropin():
    if not os.path.exists(DROPIN):
        pytest.skip("reference orchestration not built here (no reference tree)")
    _capi.load()  # libmegacu_b200.so first, RTLD_GLOBAL
    lib = ctypes.CDLL(DROPIN)
    fn = lib.dropin_orchestrate
    fn.restype = _capi.Status
    fn.argtypes = [_capi.DriverView] + [ctypes.c_void_p] * 5 + [_capi.GemmArProblem]
    return fn


def test_reference_orchestration_validates_through_our_runtime():
    fn = load_dropin()
    d = mb.driver_view(None, 0)
    d.team.team_n_pes, d.team.world_n_pes = 2, 2
    good = _capi.GemmArProblem(m=512, n=512, k=512, tile_m=128, tile_n=128)
    st = fn(d, FAKE, FAKE, FAKE, FAKE, FAKE, good)
    assert (st.code, st.detail) == (0, 0)
    # the launcher's own validation, reached through the reference's phase
    st = fn(d, None, FAKE, FAKE, FAKE, FAKE, good)
    assert (st.code, st.detail) == (_capi.INVALID_ARGUMENT, 2)
    bad = _capi.GemmArProblem(m=0, n=512, k=512, tile_m=128, tile_n=128)
    st = fn(d, FAKE, FAKE, FAKE, FAKE, FAKE, bad)
    assert (st.code, st.detail) == (_capi.INVALID_ARGUMENT, 1)


REF_DIR = os.path.join(ROOT, "oracle", "_ref")


def run_reference_program(name, **env):
    """Runs one of megacu's own test programs, built unchanged against this
    repository's headers and libmegacu_b200.so by oracle/Makefile."""
    import subprocess
    path = os.path.join(REF_DIR, name)
    if not os.path.exists(path):
        pytest.skip(f"{name} not built here (no reference tree)")
    proc = subprocess.run([path], env=dict(os.environ, **env), capture_output=True, text=True,
                          timeout=120)
    return proc.returncode, proc.stdout + proc.stderr


@pytest.mark.parametrize("name", [
    "ref_test_components",          # tests/build/runtime_components_contracts.cc
    "ref_test_surface",             # tests/build/runtime_linked_surface_contract.cc
    "ref_test_direct_orchestrate",  # tests/runtime/direct_orchestrate_smoke.cc
])
def test_reference_host_programs_pass(name):
    code, out = run_reference_program(name)
    assert code == 0, out
