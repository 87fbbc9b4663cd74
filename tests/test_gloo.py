"""World-size-2 gloo runs on the CPU: the host side of the N > 1 path.

* The team handle exchange (`megacu_b200.torch_exchange`) delivers every
  PE's handle in PE order, and ends with an error (not a hang) when a rank
  has died.
* The product's tile plan (`plan_tile`, the device queue's schedule) drives a
  CPU emulation of the two-shot allreduce, the reduce-scatter and the
  all-gather + GEMM (each rank's own raster) across real processes: each rank sends its partial tiles to their owners, owners reduce
  in PE order, two-shot owners send the sums back to everyone. The result
  must equal the oracle's n-PE graph bit for bit, and the owners must
  partition the tiles with dense local indices.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _emulate(rank, world, m, n, k, mode):
    import sys
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    import megacu_b200 as mb
    import oracle_lib

    prob = mb.Problem(m, n, k, mode=mode, algo=mb.ALGO_TWO_SHOT)
    pl = mb.plan(prob, world)
    rng = np.random.default_rng(42)
    a = [oracle_lib.round_bf16(rng.normal(0, 1, (m, k)).astype(np.float32)) for _ in range(world)]
    b = [oracle_lib.round_bf16(rng.normal(0, 0.1, (k, n)).astype(np.float32)) for _ in range(world)]
    partial = oracle_lib.round_bf16(oracle_lib.gemm_f32(a[rank], b[rank], threads=2))
    tn = pl.tile_n
    owned = {}
    # every raster index: the tile's owner receives this rank's partial tile
    for r in range(pl.tiles):
        row, col, owner, local = mb.plan_tile(prob, world, r)
        tile = partial[row * 128:(row + 1) * 128, col * tn:(col + 1) * tn].copy()
        gathered = [None] * world
        dist.all_gather_object(gathered, (owner, local, tile))
        if owner == rank:
            assert local not in owned
            acc = np.zeros_like(tile)
            for src in range(world):  # PE order
                acc = acc + gathered[src][2]
            owned[local] = (row, col, acc)
    # owners' local indices are dense
    assert sorted(owned) == list(range(len(owned)))
    rows = m // world if mode == mb.MODE_REDUCE_SCATTER else m
    out = np.zeros((rows, n), np.float32)
    everyone = [None] * world
    dist.all_gather_object(everyone, list(owned.values()))
    total = sum(len(x) for x in everyone)
    assert total == pl.tiles
    for pe, items in enumerate(everyone):
        for row, col, acc in items:
            if mode == mb.MODE_REDUCE_SCATTER:
                if pe != rank:
                    continue
                r0 = row * 128 - rank * rows
                out[r0:r0 + acc.shape[0], col * tn:col * tn + acc.shape[1]] = acc[: rows - r0]
            else:
                h = min(128, m - row * 128)
                w = min(tn, n - col * tn)
                out[row * 128:row * 128 + h, col * tn:col * tn + w] = acc[:h, :w]
    ref = oracle_lib.bf16_call(a, b, m=m, n=n, k=k, tile_n=tn, mode=mode, one_shot=False,
                               wire_bytes=2, epoch=1, threads=2)
    assert out.tobytes() == ref["out"][rank].tobytes()


def _emulate_allgather(rank, world, m, n, k):
    """The all-gather + GEMM across real processes, driven by the product's
    per-PE plan: each rank fetches the shards in its copy order (the shared
    chunk decode), computes its tiles in its own raster order from the rows
    it has, and must match the oracle bit for bit (gathered A and output)."""
    import sys
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    import megacu_b200 as mb
    import oracle_lib

    prob = mb.Problem(m, n, k, mode=mb.MODE_ALLGATHER)
    pl = mb.plan(prob, world)
    rows = m // world
    rng = np.random.default_rng(77)
    shards = [oracle_lib.round_bf16(rng.normal(0, 1, (rows, k)).astype(np.float32))
              for _ in range(world)]
    b = [oracle_lib.round_bf16(rng.normal(0, 0.1, (k, n)).astype(np.float32))
         for _ in range(world)]
    everyone = [None] * world
    dist.all_gather_object(everyone, shards[rank])          # what the peers expose
    gathered = np.full((m, k), np.nan, np.float32)
    gathered[rank * rows:(rank + 1) * rows] = everyone[rank]  # own shard: read in place
    have = {rank}
    out = np.full((m, n), np.nan, np.float32)
    tn = pl.tile_n
    last_hops = 0
    for r in range(pl.tiles):
        row, col, shard, _ = mb.plan_tile(prob, world, r, rank)
        hops = (shard - rank) % world
        assert hops >= last_hops     # whole shards, own first, then 1, 2, ... PEs away
        last_hops = hops
        if shard not in have:                                 # the copy of the next shard
            gathered[shard * rows:(shard + 1) * rows] = everyone[shard]
            have.add(shard)
        a = gathered[row * 128:(row + 1) * 128]
        assert not np.isnan(a).any()
        w = min(tn, n - col * tn)
        out[row * 128:(row + 1) * 128, col * tn:col * tn + w] = oracle_lib.gemm_f32(
            a, b[rank][:, col * tn:col * tn + w], threads=2)
    ref = oracle_lib.allgather_gemm(shards, b, m=m, n=n, k=k, tile_n=tn, threads=2)
    assert gathered.tobytes() == ref["gathered"][rank].tobytes()
    assert out.tobytes() == ref["out"][rank].tobytes()


def _worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    status = "ok"
    try:
        import sys
        sys.path.insert(0, os.path.dirname(HERE))
        import megacu_b200 as mb
        ex = mb.torch_exchange()
        mine = bytes([rank]) * 128
        got = ex(mine)
        assert [g[0] for g in got] == list(range(world)) and all(len(g) == 128 for g in got)
        _emulate(rank, world, 300, 520, 64, mb.MODE_ALLREDUCE)
        _emulate(rank, world, 512, 256, 48, mb.MODE_REDUCE_SCATTER)
        _emulate_allgather(rank, world, 512, 200, 72)
    except Exception as exc:  # reported through the result file
        status = f"fail: {exc!r}"
    finally:
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write(status)
        dist.destroy_process_group()


def test_two_rank_gloo(tmp_path):
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        if p.is_alive():
            p.kill()
    results = [open(tmp_path / f"rank{r}").read() if (tmp_path / f"rank{r}").exists() else "missing"
               for r in range(world)]
    assert results == ["ok"] * world, results


def _dying_worker(rank, world, port, result_dir):
    """Rank 1 leaves right after joining; rank 0's handle exchange must end
    with an error (within the process group's timeout), not hang."""
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    status = "ok"
    try:
        if rank == 1:
            os._exit(0)  # a rank that dies between steps
        import sys
        sys.path.insert(0, os.path.dirname(HERE))
        import megacu_b200 as mb
        try:
            mb.torch_exchange()(bytes(128))
            status = "exchange returned without the peer"
        except Exception as exc:  # noqa: BLE001 - any error is the expected outcome
            status = f"error: {type(exc).__name__}"
    finally:
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write(status)


def test_exchange_fails_when_a_rank_dies(tmp_path):
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, world, port, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    result = (tmp_path / "rank0").read_text() if (tmp_path / "rank0").exists() else "missing"
    assert result.startswith("error:"), result
