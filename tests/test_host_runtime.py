"""Host runtime (phase / dispatcher / ASAP scheduler) parity with the reference.

tests/golden/ref_host_runtime.json holds the answers of the reference's own
src/**/*.cc (compiled by oracle/Makefile) on tests/host_scenarios.py; this
repository's runtime must give the same answers — dispatch counts, the order
operator bodies run in, status codes and detail numbers.
"""
from __future__ import annotations

import ctypes
import json
import os

import pytest

import host_scenarios
import oracle_lib

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ref_host_runtime.json")


@pytest.fixture(scope="module")
def ours():
    from megacu_b200 import build
    return ctypes.CDLL(build.build_harness())


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as f:
        return json.load(f)


@pytest.mark.parametrize("sc", host_scenarios.scenarios(), ids=lambda s: s["name"])
def test_scenario_matches_reference(ours, golden, sc):
    assert host_scenarios.run_scenario(ours, sc) == golden["scenarios"][sc["name"]]


def test_fixed_contracts_match_reference(ours, golden):
    assert host_scenarios.run_fixed(ours) == golden["fixed"]


def test_contract_values(ours):
    """The reference's contract tests' literal expectations
    (runtime_components_contracts.cc:59-184)."""
    fixed = host_scenarios.run_fixed(ours)
    assert fixed["attr_capacity"] == 8
    assert fixed["components"] == [0, 1, 1, 0, 2, 1, 7, 7]
    assert fixed["capacity_3_1"]["status"] == [1, 4] and fixed["capacity_3_1"]["task_invalid"]
    assert fixed["missing_entry"]["status"] == [1, 1]
    by_name = {s["name"]: s for s in host_scenarios.scenarios()}
    r = host_scenarios.run_scenario(ours, by_name["tile_grid"])
    assert r["counts"][2:4] == [1, 6]
    r = host_scenarios.run_scenario(ours, by_name["event_sync"])
    assert r["counts"] == [3, 1, 0, 0, 1, 6, 1, 1, 1] and r["order"] == [0, 2]
    r = host_scenarios.run_scenario(ours, by_name["launcher_only"])
    assert r["order"] == [-2]  # run(launcher) calls only the launcher
    assert host_scenarios.run_scenario(ours, by_name["cycle"])["status"] == [1, 2]
    assert host_scenarios.run_scenario(ours, by_name["progress_unsupported"])["status"] == [2, 1]


@pytest.mark.skipif(not os.path.exists(oracle_lib.REF_HOST_PATH),
                    reason="reference host runtime not built here")
def test_live_reference_build(ours):
    ref = ctypes.CDLL(oracle_lib.REF_HOST_PATH)
    for sc in host_scenarios.scenarios():
        assert host_scenarios.run_scenario(ours, sc) == host_scenarios.run_scenario(ref, sc)
