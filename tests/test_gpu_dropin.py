"""Source-level drop-in on the GPU: megacu's own orchestration source,
compiled unchanged against this repository's headers (see test_dropin.py),
runs the reference's single-PE known-answer test through libmegacu_b200's
runtime and fp32 launcher."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

import megacu_b200 as mb
from test_dropin import load_dropin

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kat_gemm_allreduce.json")


def test_reference_orchestration_runs_the_kat():
    fn = load_dropin()
    from megacu_b200 import _capi
    with open(GOLDEN) as f:
        kat = json.load(f)["single_pe"]
    m, n, k = kat["m"], kat["n"], kat["k"]
    dev = torch.device("cuda", 0)
    a = torch.tensor(np.array(kat["a"], np.float32).reshape(m, k), device=dev)
    b = torch.tensor(np.array(kat["b"], np.float32).reshape(k, n), device=dev)
    partial = torch.zeros(m * n, dtype=torch.float32, device=dev)
    out = torch.zeros(m, n, dtype=torch.float32, device=dev)
    tiles = -(-m // kat["tile_m"]) * -(-n // kat["tile_n"])
    events = torch.zeros(max(tiles, 32), dtype=torch.int32, device=dev)
    d = mb.driver_view(torch.cuda.current_stream(), 0)
    st = fn(d, a.data_ptr(), b.data_ptr(), partial.data_ptr(), out.data_ptr(), events.data_ptr(),
            _capi.GemmArProblem(m=m, n=n, k=k, tile_m=kat["tile_m"], tile_n=kat["tile_n"]))
    assert st.code == 0, st
    torch.cuda.synchronize()
    want = np.array(kat["expected"], np.float32).reshape(m, n)
    assert np.max(np.abs(out.cpu().numpy() - want)) < kat["tolerance"]
    assert events[:tiles].cpu().tolist() == list(range(1, tiles + 1))


def test_reference_cuda_orchestrate_smoke_passes():
    """tests/runtime/cuda_orchestrate_smoke.cc, unchanged, on our library."""
    from test_dropin import run_reference_program
    code, out = run_reference_program("ref_test_cuda_orchestrate", MEGACU_TEST_CUDA_DEVICE="0")
    assert code == 0, out


def test_reference_cuda_multicard_smoke_passes():
    """tests/runtime/cuda_multicard_smoke.cc, unchanged (exit 77 = fewer than
    two GPUs, megacu's skip code)."""
    from test_dropin import run_reference_program
    code, out = run_reference_program("ref_test_cuda_multicard")
    if code == 77:
        pytest.skip("megacu's multicard smoke needs two GPUs")
    assert code == 0, out
