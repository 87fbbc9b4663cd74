"""Regenerates the golden fixtures in tests/golden/ (needs the reference tree).

* ``ref_host_runtime.json`` — answers of the reference's own host runtime
  (its src/**/*.cc, compiled by ``make -C oracle ref`` into
  oracle/_ref/libref_host_harness.so) on tests/host_scenarios.py.
* ``kat_gemm_allreduce.json`` — the known-answer tests of the reference,
  read as text from its test sources:
    tests/runtime/cuda_gemm_allreduce_correctness.cc:16-18,92-99 (A 2x4,
    B 4x3, tile 1x2, expected = A @ B with the reference's own host loop
    `expected()` at :44-52, tolerance 1e-4) and
    tests/runtime/nvshmem_two_rank_smoke.cc:16-18,29-36,101-102 (2 PEs,
    A = pe + 1, B = 1, K = 4 -> every output 12, tolerance 1e-4).

Run: ``python tests/golden/make_golden.py [REFERENCE_ROOT]``.
"""
from __future__ import annotations

import ctypes
import json
import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))

import host_scenarios  # noqa: E402


def _floats(text: str, name: str) -> list[float]:
    m = re.search(r"std::vector<float>\s+" + name + r"\s*\{([^}]*)\}", text)
    assert m, f"{name} not found"
    return [float(v.strip().rstrip("f")) for v in m.group(1).split(",") if v.strip()]


def _const(text: str, name: str) -> int:
    m = re.search(r"constexpr int " + name + r"\s*=\s*(\d+);", text)
    assert m, name
    return int(m.group(1))


def kat(ref: str) -> dict:
    src = open(os.path.join(ref, "tests/runtime/cuda_gemm_allreduce_correctness.cc")).read()
    m, n, k = _const(src, "kM"), _const(src, "kN"), _const(src, "kK")
    a, b = _floats(src, "host_a"), _floats(src, "host_b")
    # The reference's expected(): value += a[row*K + kk] * b[kk*N + col].
    want = []
    for r in range(m):
        for c in range(n):
            v = 0.0
            for kk in range(k):
                v += a[r * k + kk] * b[kk * n + c]
            want.append(v)
    tile = re.search(r"gemm_ar_problem\{\.m = kM, \.n = kN, \.k = kK, \.tile_m = (\d+), "
                     r"\.tile_n = (\d+)\}", src)
    two = open(os.path.join(ref, "tests/runtime/nvshmem_two_rank_smoke.cc")).read()
    m2, n2, k2 = _const(two, "kM"), _const(two, "kN"), _const(two, "kK")
    want2 = sum(k2 * 1.0 * (pe + 1) for pe in range(2))
    return {
        "single_pe": {"m": m, "n": n, "k": k, "a": a, "b": b, "tile_m": int(tile.group(1)),
                      "tile_n": int(tile.group(2)), "expected": want, "tolerance": 1e-4,
                      "source": "tests/runtime/cuda_gemm_allreduce_correctness.cc:92-99"},
        "two_pe": {"m": m2, "n": n2, "k": k2, "a_value_per_pe": [1.0, 2.0], "b_value": 1.0,
                   "tile_m": m2, "tile_n": n2, "expected_value": want2, "tolerance": 1e-4,
                   "source": "tests/runtime/nvshmem_two_rank_smoke.cc:101-102,46-61"},
    }


def main() -> None:
    sys.path.insert(0, ROOT)
    from megacu_b200.build import reference_root
    ref = sys.argv[1] if len(sys.argv) > 1 else reference_root()
    if not ref:
        raise SystemExit("the reference tree (BASELINE.json reference_path) is not present")
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref", f"REF={ref}"],
                   check=True)
    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_host_harness.so"))
    runs = {sc["name"]: host_scenarios.run_scenario(lib, sc) for sc in host_scenarios.scenarios()}
    fixed = host_scenarios.run_fixed(lib)
    with open(os.path.join(HERE, "ref_host_runtime.json"), "w") as f:
        json.dump({"scenarios": runs, "fixed": fixed,
                   "generated_by": "tests/golden/make_golden.py from the reference's src/**/*.cc"},
                  f, indent=1, sort_keys=True)
    with open(os.path.join(HERE, "kat_gemm_allreduce.json"), "w") as f:
        json.dump(kat(ref), f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
