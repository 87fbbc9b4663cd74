"""Exhaustive check of the single-CTA stage ring of the fused kernel with the
first tile's loads issued during the set-up (race and deadlock detection
without a GPU).

An explicit-state model of one CTA's TMA producer and MMA issuer over a ring
of `n_stages` shared-memory stages explores every order of their steps, of the
loads landing (in any order) and of the MMA commits completing (in issue
order), and checks that
  * every k-block the MMA consumes is the one it expects, from a load that
    has landed (no stale or foreign stage);
  * no load lands in a stage whose previous k-block the MMA has not consumed
    (no overwrite);
  * nothing is stuck (some step enabled until both threads are done).

It follows the kernel (megacu_b200/csrc/kernels/gemm_ar_kernel.cuh):
  * mbarrier waits take a parity: `wait(p)` passes once the barrier's current
    phase has a parity other than p (a fresh barrier passes `wait(1)` at once);
  * set-up (single-CTA plain tiles): the first `pre = min(n_stages, kbs)`
    k-blocks of the CTA's first tile are issued into stages 0..pre-1 with no
    wait;
  * producer loop: it starts at it = pre, stage = pre % n_stages, phase =
    pre / n_stages, skips the first tile's first `pre` k-blocks, and before
    each load waits `empty[stage]` with parity `phase ^ 1`; a load arrives on
    `full[stage]` with its bytes (the phase completes when it lands);
  * MMA: from stage 0, phase 0, waits `full[stage]` with parity `phase`,
    consumes, and commits to `empty[stage]` (one arrive once the MMA is done);
  * both advance stage by one and flip phase on wrapping.

Planted mistakes (the first tile's pre-issued k-blocks loaded again; the
phase not flipped when the set-up filled the whole ring; no pre-issue but the
loop started past the ring) must each be found: the check has teeth.
"""
from __future__ import annotations

import pytest


def producer_ops(n_stages, tiles, kbs, mistake=None):
    """(stage, tag, wait parity or None) per load, in the producer's order."""
    ops = []
    pre = min(n_stages, kbs) if tiles > 0 else 0
    if mistake == "no_pre_issue":
        pre_loads = 0
    else:
        pre_loads = pre
    for s in range(pre_loads):
        ops.append((s, (0, s), None))
    stage = 0 if pre == n_stages else pre
    phase = 1 if pre == n_stages else 0
    if mistake == "no_phase_flip":
        phase = 0
    for n in range(tiles):
        first = pre if n == 0 else 0
        if mistake == "reload_pre_issued":
            first = 0
        for kb in range(first, kbs):
            ops.append((stage, (n, kb), phase ^ 1))
            stage += 1
            if stage == n_stages:
                stage = 0
                phase ^= 1
    return ops


def mma_ops(n_stages, tiles, kbs):
    """(stage, expected tag, wait parity) per consumed k-block."""
    ops = []
    stage = phase = 0
    for n in range(tiles):
        for kb in range(kbs):
            ops.append((stage, (n, kb), phase))
            stage += 1
            if stage == n_stages:
                stage = 0
                phase ^= 1
    return ops


def passes(count, parity):
    """mbarrier try_wait.parity: the current phase (completed count) has
    another parity than the one waited on."""
    return (count & 1) != parity


class Violation(Exception):
    pass


def explore(n_stages, tiles, kbs, mistake=None, limit=2_000_000):
    """Visits every reachable state; raises Violation on a race or a stuck
    state. Returns the number of states."""
    prod = producer_ops(n_stages, tiles, kbs, mistake)
    mma = mma_ops(n_stages, tiles, kbs)
    # state: producer index, MMA index, full counts, empty counts,
    # stage contents ((tag, consumed) or None), loads in flight
    # (frozenset of (stage, tag)), commits in flight (tuple of stages, FIFO)
    start = (0, 0, (0,) * n_stages, (0,) * n_stages, (None,) * n_stages, frozenset(), ())
    seen = {start}
    todo = [start]
    while todo:
        st = todo.pop()
        pi, mi, full, empty, slots, loads, commits = st
        nxt = []
        if pi < len(prod):
            s, tag, parity = prod[pi]
            if parity is None or passes(empty[s], parity):
                if any(ls == s for ls, _ in loads):
                    raise Violation(f"two loads in flight into stage {s}")
                nxt.append((pi + 1, mi, full, empty, slots, loads | {(s, tag)}, commits))
        for ls, tag in loads:
            cur = slots[ls]
            if cur is not None and not cur[1]:
                raise Violation(f"load {tag} lands on unconsumed {cur[0]} in stage {ls}")
            f = list(full)
            f[ls] += 1
            sl = list(slots)
            sl[ls] = (tag, False)
            nxt.append((pi, mi, tuple(f), empty, tuple(sl), loads - {(ls, tag)}, commits))
        if mi < len(mma):
            s, want, parity = mma[mi]
            if passes(full[s], parity):
                cur = slots[s]
                if cur is None or cur[0] != want or cur[1]:
                    raise Violation(f"MMA expected {want} in stage {s}, found {cur}")
                sl = list(slots)
                sl[s] = (want, True)
                nxt.append((pi, mi + 1, full, empty, tuple(sl), loads, commits + (s,)))
        if commits:
            e = list(empty)
            e[commits[0]] += 1
            nxt.append((pi, mi, full, tuple(e), slots, loads, commits[1:]))
        if not nxt:
            if pi < len(prod) or mi < len(mma) or loads:
                raise Violation(f"stuck: producer {pi}/{len(prod)}, MMA {mi}/{len(mma)}")
            continue
        for s2 in nxt:
            if s2 not in seen:
                seen.add(s2)
                if len(seen) > limit:
                    raise RuntimeError("state space larger than the limit")
                todo.append(s2)
    return len(seen)


CASES = [(n, t, k) for n in (1, 2, 3) for t in (1, 2, 3) for k in (1, 2, 3, 4)]


@pytest.mark.parametrize("n_stages,tiles,kbs", CASES)
def test_stage_ring_with_set_up_loads_has_no_race_or_deadlock(n_stages, tiles, kbs):
    assert explore(n_stages, tiles, kbs) > 1


def test_producer_issues_every_k_block_once():
    for n_stages, tiles, kbs in CASES:
        tags = [tag for _, tag, _ in producer_ops(n_stages, tiles, kbs)]
        assert tags == [(n, kb) for n in range(tiles) for kb in range(kbs)]


@pytest.mark.parametrize("mistake,case", [
    ("reload_pre_issued", (2, 1, 3)),   # the first tile's first k-blocks loaded twice
    ("reload_pre_issued", (3, 2, 2)),
    ("no_phase_flip", (2, 1, 3)),       # set-up filled the ring, phase left at 0
    ("no_phase_flip", (1, 2, 1)),
    ("no_pre_issue", (2, 1, 3)),        # loop starts past loads that were never issued
])
def test_planted_ring_mistakes_are_found(mistake, case):
    with pytest.raises(Violation):
        explore(*case, mistake=mistake)
