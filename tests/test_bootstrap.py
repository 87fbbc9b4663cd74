"""The local rendezvous (megacu_b200_exchange_local), host only: every PE's
blob to every PE in PE order, across real processes; bounded failure when a
PE is missing or claims another's index; argument validation."""
from __future__ import annotations

import ctypes
import multiprocessing as mp
import os
import uuid

import pytest

from megacu_b200 import _capi


def _session():
    return f"test.{os.getpid()}.{uuid.uuid4().hex[:12]}"


def _exchange(session, pe, n_pes, blob, timeout_ms):
    lib = _capi.load()
    out = ctypes.create_string_buffer(len(blob) * n_pes)
    st = lib.megacu_b200_exchange_local(session.encode(), pe, n_pes, blob, len(blob), out,
                                        timeout_ms)
    return st.code, st.detail, out.raw


def _worker(session, pe, n_pes, blob, timeout_ms, q):
    q.put((pe, _exchange(session, pe, n_pes, blob, timeout_ms)))


def _run(jobs, timeout_ms):
    """jobs: [(pe claimed, n_pes, blob)], one process each; -> {index: result}."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    session = _session()
    procs = [ctx.Process(target=_worker, args=(session, pe, n, blob, timeout_ms, q))
             for pe, n, blob in jobs]
    for p in procs:
        p.start()
    results = [q.get(timeout=60) for _ in procs]
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    return results


@pytest.mark.parametrize("n_pes,size", [(2, 128), (4, 128), (8, 1000)])
def test_every_pe_gets_every_blob(n_pes, size):
    blobs = [os.urandom(size) for _ in range(n_pes)]
    res = _run([(pe, n_pes, blobs[pe]) for pe in range(n_pes)], 20_000)
    for pe, (code, detail, raw) in res:
        assert (code, detail) == (0, 0)
        assert raw == b"".join(blobs)


def test_missing_pe_times_out():
    res = dict(_run([(0, 3, b"a" * 64), (1, 3, b"b" * 64)], 500))
    assert res[0][:2] == (_capi.BACKEND_ERROR, 39)
    assert res[1][:2] == (_capi.BACKEND_ERROR, 39)


def test_no_server_times_out():
    code, detail, _ = _exchange(_session(), 1, 2, b"x" * 16, 300)
    assert (code, detail) == (_capi.BACKEND_ERROR, 39)


def test_duplicate_pe_is_refused():
    res = _run([(0, 3, b"a" * 32), (1, 3, b"b" * 32), (1, 3, b"c" * 32)], 2_000)
    assert all(r[1][:2] == (_capi.BACKEND_ERROR, 39) for r in res)


def test_validation_and_single_pe():
    lib = _capi.load()
    out = ctypes.create_string_buffer(64)

    def call(session, pe, n, blob, size, timeout=100):
        st = lib.megacu_b200_exchange_local(session, pe, n, blob, size, out, timeout)
        return st.code, st.detail

    assert call(b"s", 0, 1, b"z" * 8, 8) == (0, 0) and out.raw[:8] == b"z" * 8
    assert call(b"", 0, 2, b"z" * 8, 8) == (1, 1)
    assert call(b"s" * 65, 0, 2, b"z" * 8, 8) == (1, 1)
    assert call(b"s", 0, 2, b"z" * 8, 0) == (1, 1)
    assert call(b"s", 0, 2, b"z" * 8, 8, 0) == (1, 1)
    assert call(b"s", 2, 2, b"z" * 8, 8) == (1, 23)
    assert call(b"s", 0, 0, b"z" * 8, 8) == (1, 23)
    assert call(None, 0, 2, b"z" * 8, 8) == (1, 2)
