"""Exhaustive check of the cross-GPU flag protocol of the fused kernel over
consecutive calls (race detection without a GPU).

An explicit-state model of `tp` PEs, each running `calls` launches of the
kernel one after another on its stream, explores every interleaving of their
steps and checks that
  * no read of a peer's partial slot (or, for all-gather, of a peer's A
    shard) sees data of another call than its own;
  * no PE's output is overwritten by a later call before its own call ends
    (at the end of call e every output element it owns holds call e's value);
  * no state is stuck (some PE not finished, no step enabled).

The model follows the kernel's protocol (megacu_b200/csrc/kernels/
gemm_ar_kernel.cuh), one step per flag store or acquired wait:
  * call e (epoch e, from the launch counter) uses parity plane e & 1 of the
    partial slots and of the `arrive` / `done` flags; waits compare a flag
    for equality with e (`wait_flag`);
  * GEMM step W(t): the tile's partial goes into this PE's own slot, then the
    `arrive` flag (source me, tile t) is stored into the event tensor of each
    PE that reduces t: every PE (one-shot), the owner t mod tp (two-shot), the
    owner of t's row block (reduce-scatter);
  * reduce step R(q, t) of a reducer, once its flag from q equals e: load q's
    slot of tile t; final step F(t) after every source: store the sum into
    this PE's out (one-shot, reduce-scatter) or into every PE's out
    (two-shot);
  * in-switch two-shot: the owner's reduce is one step (one
    `multimem.ld_reduce` over every PE's slot, once every flag equals e) and
    its final step stores into every PE's out through the multicast mapping;
  * two-shot completion (both kinds): once a PE's reduce steps are all done it stores
    `done` (source me) = e into every PE; a launch ends only after all tp
    `done` flags equal e;
  * all-gather: at launch start the PE's A shard (written by the host before
    the launch) is announced by `ready` = e on every peer (one slot per
    source, no parity plane); copy step C(q) once `ready` from q equals e,
    after which `read_done` (source me) = e is stored into q; a launch ends
    only after `read_done` from every peer equals e.
A launch ends only after all its own steps and waits (kernel completion), and
call e + 1 of a PE starts after its call e ended (stream order).

The single-launch MLP chain's protocol (`ChainModel`) is checked the same
way over consecutive launches.

Planted mistakes (one parity plane, no `done` wait, no `read_done` wait; for
the chain: arrive flags zeroed with the counters, no final wait, no wait for
the previous block) must each be found: the check has teeth.
"""
from __future__ import annotations

import itertools

import pytest

ONE_SHOT, TWO_SHOT, REDUCE_SCATTER, ALL_GATHER = "one_shot", "two_shot", "reduce_scatter", "gather"
IN_SWITCH = "in_switch"  # two-shot whose owner reads and stores through the NVSwitch


class Model:
    def __init__(self, mode, tp, tiles, calls, planes=2, wait_done=True, wait_reads=True):
        self.mode, self.tp, self.tiles, self.calls = mode, tp, tiles, calls
        self.planes, self.wait_done, self.wait_reads = planes, wait_done, wait_reads

    # ---- roles ----
    def reducers(self, t):
        if self.mode == ONE_SHOT:
            return range(self.tp)
        if self.mode in (TWO_SHOT, IN_SWITCH):
            return [t % self.tp]
        return [t * self.tp // self.tiles]  # the PE whose output rows hold tile t

    def owned(self, p):
        return [t for t in range(self.tiles) if p in self.reducers(t)]

    def out_targets(self, p):
        return range(self.tp) if self.mode in (TWO_SHOT, IN_SWITCH) else [p]

    def out_tiles(self, p):
        """Output tiles PE p's out holds at the end of a call."""
        if self.mode in (ONE_SHOT, TWO_SHOT, IN_SWITCH):
            return range(self.tiles)
        return self.owned(p)

    # ---- state ----
    # state = (pes, mem); pes[p] = (call, frozenset(progress)); mem is a dict
    # frozen as a sorted tuple of items.
    def initial(self):
        mem = {}
        for p in range(self.tp):
            for pl, t in itertools.product(range(self.planes), range(self.tiles)):
                mem[("slot", p, pl, t)] = 0
            for t in range(self.tiles):
                mem[("out", p, t)] = 0
            mem[("shard", p)] = 0
            for q in range(self.tp):
                for pl in range(self.planes):
                    mem[("done", p, pl, q)] = 0
                    for t in range(self.tiles):
                        mem[("arrive", p, pl, q, t)] = 0
                mem[("ready", p, q)] = 0
                mem[("read_done", p, q)] = 0
        return (tuple((1, frozenset()) for _ in range(self.tp)), tuple(sorted(mem.items())))

    def steps(self, p, e, prog, mem):
        """(name, enabled, effect) of PE p's steps in call e; effect(mem) -> error or None."""
        pl = e % self.planes
        tp = self.tp
        out = []
        if self.mode == ALL_GATHER:
            if "S" not in prog:
                def start(m):
                    m[("shard", p)] = e  # the host wrote this call's shard
                    for x in range(tp):
                        if x != p:
                            m[("ready", x, p)] = e
                out.append(("S", True, start))
                return out
            for q in range(tp):
                if q == p or ("C", q) in prog:
                    continue

                def copy(m, q=q):
                    if m[("shard", q)] != e:
                        return f"PE {p} call {e} copied PE {q}'s shard of call {m[('shard', q)]}"
                    m[("read_done", q, p)] = e
                out.append((("C", q), mem[("ready", p, q)] == e, copy))
            return out
        for t in range(self.tiles):
            if ("W", t) not in prog:
                def write(m, t=t):
                    m[("slot", p, pl, t)] = e
                    for r in self.reducers(t):
                        m[("arrive", r, pl, p, t)] = e
                out.append((("W", t), True, write))
        for t in self.owned(p):
            if self.mode == IN_SWITCH:
                # one multimem.ld_reduce over every PE's slot, after every flag
                if ("R", t) not in prog:
                    def reduce_all(m, t=t):
                        for q in range(tp):
                            if m[("slot", q, pl, t)] != e:
                                return (f"PE {p} call {e} reduced PE {q}'s slot of tile {t} "
                                        f"holding call {m[('slot', q, pl, t)]}")
                    ready = all(mem[("arrive", p, pl, q, t)] == e for q in range(tp))
                    out.append((("R", t), ready, reduce_all))
                if ("F", t) not in prog:
                    def store_all(m, t=t):
                        for x in range(tp):
                            m[("out", x, t)] = e
                    out.append((("F", t), ("R", t) in prog, store_all))
                continue
            for q in range(tp):
                if ("R", q, t) in prog:
                    continue

                def read(m, q=q, t=t):
                    if m[("slot", q, pl, t)] != e:
                        return (f"PE {p} call {e} read PE {q}'s slot of tile {t} holding call "
                                f"{m[('slot', q, pl, t)]}")
                out.append((("R", q, t), mem[("arrive", p, pl, q, t)] == e, read))
            if ("F", t) not in prog:
                def final(m, t=t):
                    for x in self.out_targets(p):
                        m[("out", x, t)] = e
                ready = all(("R", q, t) in prog for q in range(tp))
                out.append((("F", t), ready, final))
        if self.mode in (TWO_SHOT, IN_SWITCH) and "D" not in prog:
            def done(m):
                for x in range(tp):
                    m[("done", x, pl, p)] = e
            out.append(("D", all(("F", t) in prog for t in self.owned(p)), done))
        return out

    def can_end(self, p, e, prog, mem):
        pl = e % self.planes
        if self.mode == ALL_GATHER:
            if "S" not in prog or any(("C", q) not in prog for q in range(self.tp) if q != p):
                return False
            return not self.wait_reads or all(
                mem[("read_done", p, q)] == e for q in range(self.tp) if q != p)
        if any(("W", t) not in prog for t in range(self.tiles)):
            return False
        if any(("F", t) not in prog for t in self.owned(p)):
            return False
        if self.mode in (TWO_SHOT, IN_SWITCH):
            if "D" not in prog:
                return False
            if self.wait_done and any(mem[("done", p, pl, q)] != e for q in range(self.tp)):
                return False
        return True

    def check_end(self, p, e, mem):
        if self.mode == ALL_GATHER:
            return None
        for t in self.out_tiles(p):
            if mem[("out", p, t)] != e:
                return f"PE {p} ended call {e} with out tile {t} of call {mem[('out', p, t)]}"
        return None

    def begin(self, p, e, mem):
        """Host work on PE p between its launches, before call e."""

    def explore(self):
        """Depth-first over every interleaving; returns (states, first error)."""
        start = self.initial()
        seen = {start}
        stack = [start]
        while stack:
            pes, mem_t = stack.pop()
            mem = dict(mem_t)
            if all(e > self.calls for e, _ in pes):
                continue
            moves = []
            for p, (e, prog) in enumerate(pes):
                if e > self.calls:
                    continue
                for name, enabled, effect in self.steps(p, e, prog, mem):
                    if enabled:
                        moves.append((p, e, prog | {name}, effect))
                if self.can_end(p, e, prog, mem):
                    moves.append((p, e + 1, frozenset(), None))
            if not moves:
                state = ", ".join(f"PE {p} call {e} did {sorted(map(str, prog))}"
                                  for p, (e, prog) in enumerate(pes))
                return len(seen), f"stuck: {state}"
            for p, e_next, prog_next, effect in moves:
                m = dict(mem)
                if effect is not None:
                    err = effect(m)
                else:  # the launch of call e_next - 1 ended
                    err = self.check_end(p, e_next - 1, m)
                    if err is None and e_next <= self.calls:
                        self.begin(p, e_next, m)
                if err:
                    return len(seen), err
                nxt = list(pes)
                nxt[p] = (e_next, prog_next)
                s = (tuple(nxt), tuple(sorted(m.items())))
                if s not in seen:
                    seen.add(s)
                    stack.append(s)
        return len(seen), None


class ChainModel(Model):
    """The single-launch MLP chain (megacu_b200/csrc/kernels/chain_kernel.cuh):
    `layers` blocks in one launch per call, `rows` token row blocks, per row
    block `gu` gate/up tiles (local) and `dn` down tiles, DN tile (r, j) owned
    by PE (r * dn + j) mod tp. Data values are (call, block) pairs.

      GU(l, r, c)  block 0, or x_ready[l-1][r] holds all dn counts: read the
                   row block of x (block 0) or of block l-1's output, write
                   act[r][c], count act_ready[l][r]
      DN(l, r, j)  act_ready[l][r] holds all gu counts: read act[r][*], write
                   this PE's slot[r][j] (one plane, shared by the blocks),
                   store arrive[l][me][(r, j)] = call into the owner
      X(l, r, j)   (owner) every PE's arrive equals the call: read every PE's
                   slot[r][j], store the sum into block l's output on every
                   PE, count x_ready[l][r] there
    Block outputs alternate between two buffers, the last one `out`. A launch
    ends after its steps and once x_ready[layers-1][r] holds all dn counts for
    every r; then the host zeroes the counters (act_ready, x_ready; the arrive
    flags are epoch-tagged and kept) and writes the next call's x.
    """

    def __init__(self, tp, layers, rows, gu, dn, calls, zero_arrive=False, final_wait=True,
                 wait_x=True):
        super().__init__("chain", tp, rows * dn, calls)
        self.layers, self.rows, self.gu, self.dn = layers, rows, gu, dn
        self.zero_arrive, self.final_wait, self.wait_x = zero_arrive, final_wait, wait_x

    def owner(self, r, j):
        return (r * self.dn + j) % self.tp

    def buf(self, l):
        return "out" if (self.layers - 1 - l) % 2 == 0 else "work"

    def initial(self):
        mem = {}
        L, R = self.layers, self.rows
        for p in range(self.tp):
            for r in range(R):
                mem[("x", p, r)] = (1, -1)
                for c in range(self.gu):
                    mem[("act", p, r, c)] = (0, 0)
                for j in range(self.dn):
                    mem[("slot", p, r, j)] = (0, 0)
                    for b in ("out", "work"):
                        mem[(b, p, r, j)] = (0, 0)
                for l in range(L):
                    mem[("act_ready", p, l, r)] = 0
                    mem[("x_ready", p, l, r)] = 0
                    for q in range(self.tp):
                        for j in range(self.dn):
                            mem[("arrive", p, l, q, r, j)] = 0
        return (tuple((1, frozenset()) for _ in range(self.tp)), tuple(sorted(mem.items())))

    def steps(self, p, e, prog, mem):
        L, R, tp = self.layers, self.rows, self.tp
        out = []
        for l, r in itertools.product(range(L), range(R)):
            for c in range(self.gu):
                if ("GU", l, r, c) in prog:
                    continue

                def gu(m, l=l, r=r, c=c):
                    for j in range(self.dn):
                        src = m[("x", p, r)] if l == 0 else m[(self.buf(l - 1), p, r, j)]
                        want = (e, -1) if l == 0 else (e, l - 1)
                        if src != want:
                            return f"PE {p} call {e} GU{l} read input {src}, want {want}"
                    m[("act", p, r, c)] = (e, l)
                    m[("act_ready", p, l, r)] += 1
                ready = (l == 0 or not self.wait_x
                         or mem[("x_ready", p, l - 1, r)] == self.dn)
                out.append((("GU", l, r, c), ready, gu))
            for j in range(self.dn):
                if ("DN", l, r, j) not in prog:
                    def dn(m, l=l, r=r, j=j):
                        for c in range(self.gu):
                            if m[("act", p, r, c)] != (e, l):
                                return f"PE {p} call {e} DN{l} read act {m[('act', p, r, c)]}"
                        m[("slot", p, r, j)] = (e, l)
                        m[("arrive", self.owner(r, j), l, p, r, j)] = e
                    out.append((("DN", l, r, j), mem[("act_ready", p, l, r)] == self.gu, dn))
                if self.owner(r, j) != p or ("X", l, r, j) in prog:
                    continue

                def x(m, l=l, r=r, j=j):
                    for q in range(tp):
                        if m[("slot", q, r, j)] != (e, l):
                            return (f"PE {p} call {e} X{l} read PE {q}'s slot holding "
                                    f"{m[('slot', q, r, j)]}")
                    for y in range(tp):
                        m[(self.buf(l), y, r, j)] = (e, l)
                        m[("x_ready", y, l, r)] += 1
                ready = all(mem[("arrive", p, l, q, r, j)] == e for q in range(tp))
                out.append((("X", l, r, j), ready, x))
        return out

    def can_end(self, p, e, prog, mem):
        L, R = self.layers, self.rows
        for l, r in itertools.product(range(L), range(R)):
            if any(("GU", l, r, c) not in prog for c in range(self.gu)):
                return False
            for j in range(self.dn):
                if ("DN", l, r, j) not in prog:
                    return False
                if self.owner(r, j) == p and ("X", l, r, j) not in prog:
                    return False
        return not self.final_wait or all(
            mem[("x_ready", p, L - 1, r)] == self.dn for r in range(R))

    def check_end(self, p, e, mem):
        for r, j in itertools.product(range(self.rows), range(self.dn)):
            if mem[("out", p, r, j)] != (e, self.layers - 1):
                return f"PE {p} ended call {e} with out {mem[('out', p, r, j)]}"
        return None

    def begin(self, p, e, mem):
        for key in list(mem):
            if key[0] in ("act_ready", "x_ready") and key[1] == p:
                mem[key] = 0
            if self.zero_arrive and key[0] == "arrive" and key[1] == p:
                mem[key] = 0
        for r in range(self.rows):
            mem[("x", p, r)] = (e, -1)


CHAIN_CASES = [
    # tp, layers, rows, gu, dn, calls
    (2, 3, 1, 1, 2, 2),   # three blocks: the output buffers are reused (l, l + 2)
    (2, 2, 2, 1, 1, 3),   # two row blocks, one DN tile each, owned by different PEs
    (2, 2, 2, 1, 2, 3),   # two row blocks of two DN tiles, three calls
    (3, 3, 1, 1, 3, 2),   # three PEs, each owning one DN tile
    (3, 2, 1, 1, 3, 3),
]


@pytest.mark.parametrize("tp,layers,rows,gu,dn,calls", CHAIN_CASES)
def test_chain_protocol_has_no_race_or_deadlock(tp, layers, rows, gu, dn, calls):
    states, err = ChainModel(tp, layers, rows, gu, dn, calls).explore()
    assert err is None, err
    assert states > 10


def test_chain_planted_mistakes_are_found():
    """Zeroing the arrive flags with the counters loses a fast peer's flag of
    the next call; ending before the last block's counts ends with an
    incomplete out; a GU tile that does not wait for the previous block reads
    an old input."""
    _, err = ChainModel(2, 1, 1, 1, 2, 2, zero_arrive=True).explore()
    assert err is not None and "stuck" in err, err
    _, err = ChainModel(2, 1, 1, 1, 2, 2, final_wait=False).explore()
    assert err is not None and "ended call" in err, err
    _, err = ChainModel(2, 2, 1, 1, 1, 1, wait_x=False).explore()
    assert err is not None and "GU1 read input" in err, err


CASES = [
    (ONE_SHOT, 2, 2, 3),
    (ONE_SHOT, 3, 1, 3),
    (TWO_SHOT, 2, 2, 3),
    (TWO_SHOT, 3, 2, 3),   # one PE owns no tile: only the done flags hold it back
    (IN_SWITCH, 2, 2, 3),
    (IN_SWITCH, 3, 2, 3),
    (REDUCE_SCATTER, 2, 2, 3),
    (REDUCE_SCATTER, 3, 3, 3),
    (ALL_GATHER, 3, 1, 4),
]


@pytest.mark.parametrize("mode,tp,tiles,calls", CASES)
def test_protocol_has_no_race_or_deadlock(mode, tp, tiles, calls):
    states, err = Model(mode, tp, tiles, calls).explore()
    assert err is None, err
    assert states > 10


@pytest.mark.parametrize("mode,tp,tiles", [(ONE_SHOT, 2, 1), (REDUCE_SCATTER, 2, 2)])
def test_one_parity_plane_races(mode, tp, tiles):
    """One-shot and reduce-scatter have no call-wide barrier: with one plane a
    PE's next call overwrites a slot a slower peer has not yet read (or that
    peer waits forever on a flag already at e + 1)."""
    _, err = Model(mode, tp, tiles, 3, planes=1).explore()
    assert err is not None and ("read PE" in err or "stuck" in err), err


def test_two_shot_done_wait_alone_protects_the_slots():
    """Two-shot: a PE ends call e only after every PE's done flag, which each
    PE stores after its last read, so even one plane would be safe there; the
    second plane matters for one-shot and reduce-scatter."""
    assert Model(TWO_SHOT, 2, 2, 3, planes=1).explore()[1] is None
    _, err = Model(TWO_SHOT, 2, 2, 3, planes=1, wait_done=False).explore()
    assert err is not None, err


@pytest.mark.parametrize("mode", [TWO_SHOT, IN_SWITCH])
def test_two_shot_without_done_wait_races(mode):
    """Without the done wait a PE ends its call before every owner stored its
    tiles into its out."""
    _, err = Model(mode, 2, 2, 2, wait_done=False).explore()
    assert err is not None and "ended call" in err, err


def test_all_gather_without_read_done_wait_races():
    """Without the read_done wait a PE's host overwrites its shard while a
    peer still copies it (or the peer misses this call's ready flag)."""
    _, err = Model(ALL_GATHER, 2, 1, 3, wait_reads=False).explore()
    assert err is not None and ("copied" in err or "stuck" in err), err
