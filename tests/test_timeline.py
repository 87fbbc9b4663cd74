"""The timeline tool's summary of trace records (no GPU: synthetic records)."""
import numpy as np

from megacu_b200 import timeline


def test_summary_reads_every_kind_relative_to_first_event():
    # kind, start ns, end ns
    recs = [(0, 1000, 5000), (0, 3000, 9000), (2, 4000, 20000), (2, 6000, 30000),
            (3, 21000, 40000), (3, 31000, 41000), (4, 41000, 42000), (5, 35000, 43000)]
    tr = {"kind": np.array([r[0] for r in recs], np.int64),
          "t0": np.array([r[1] for r in recs], np.uint64),
          "t1": np.array([r[2] for r in recs], np.uint64)}
    s = timeline._summary(tr, np)
    assert s["gemm_tiles"] == 2 and s["gemm_end_us"] == 8.0 and s["gemm_end_p50_us"] == 6.0
    assert s["reduce_tasks"] == 2 and s["reduce_first_start_us"] == 3.0
    assert s["reduce_end_us"] == 29.0 and s["reduce_task_p50_us"] == 20.0
    assert s["fence_start_us"] == [20.0, 30.0] and s["fence_end_us"] == [39.0, 40.0]
    assert s["done_flags_end_us"] == [41.0, 41.0] and s["final_wait_start_us"] == [34.0, 34.0]


def test_summary_reads_copy_chunks_by_shard_distance():
    recs = [(0, 0, 10000), (6, 1000, 3000, 1), (6, 2000, 4000, 1), (6, 2500, 9000, 2)]
    tr = {"kind": np.array([r[0] for r in recs], np.int64),
          "sub": np.array([r[3] if len(r) > 3 else 0 for r in recs], np.int64),
          "t0": np.array([r[1] for r in recs], np.uint64),
          "t1": np.array([r[2] for r in recs], np.uint64)}
    s = timeline._summary(tr, np)
    assert s["copy_chunks"] == 3 and s["copy_first_start_us"] == 1.0 and s["copy_end_us"] == 9.0
    assert s["copy_end_by_hops_us"] == {1: 4.0, 2: 9.0}
    assert s["copy_chunk_p50_us"] == 2.0


def test_summary_of_an_empty_trace():
    empty = np.zeros(0, np.uint64)
    tr = {"kind": empty.astype(np.int64), "sub": empty.astype(np.int64), "t0": empty, "t1": empty}
    assert timeline._summary(tr, np) == {"records": 0}
