"""The allocation-free entry point, megacu_cuda_gemm_bf16_noalloc.

It exists for callers that cannot allocate device memory for the kernel's
scratch — a plugin host that hands an operator only its inputs and outputs,
a process whose device memory belongs to another allocator, a serving loop
that must not call cudaMalloc. The kernel's scratch lives in a fixed array
built into the library instead. This file is collected last on purpose.

The GPU tests call it through the C ABI and compare every output bit for bit
with the regular entry point's (the same kernel, given a caller-allocated
events buffer): two calls in a row of each shape; a stream-ordered sequence
of different shapes on the one shared array (CTA-pair tiles, 64-column
tiles, a traced call); and a call after an error word was left set in the
array. After every call the array's error word is read (and cleared) with
megacu_b200_events_status, and the completion counters it gained are
compared with the oracle's graph. The array is shared by every call in the
process, so the tests compare counter increments, not totals, and pass
alone or after any other test. The CPU test checks the limits that need no
GPU.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import megacu_b200 as mb
import oracle_lib
from megacu_b200 import _capi
from conftest import gpu_count
from gpu_util import SinglePE, inputs, trace_records


def test_noalloc_rejects_what_it_cannot_hold():
    lib = _capi.load()
    d = mb.driver_view(None, 0)
    fake = 0x100000
    ok = lib.megacu_cuda_gemm_bf16_noalloc(d, fake, fake, fake, mb.Problem(512, 1024, 256).to_c())
    assert (ok.code, ok.detail) == (0, 0)  # null stream: validate only
    big = lib.megacu_cuda_gemm_bf16_noalloc(d, fake, fake, fake,
                                            mb.Problem(16384, 65536, 64).to_c())
    assert (big.code, big.detail) == (1, 52) and b"256 KiB" in big.message
    d2 = mb.driver_view(None, 0)
    d2.team.team_n_pes = 2
    two = lib.megacu_cuda_gemm_bf16_noalloc(d2, fake, fake, fake, mb.Problem(256, 256, 64).to_c())
    assert (two.code, two.detail) == (2, 51)
    missing = lib.megacu_b200_noalloc_scratch(0, None, None)
    assert (missing.code, missing.detail) == (1, 2)


def _scratch(device: int = 0):
    """Device address and size of the built-in scratch (looked up, not allocated)."""
    ptr, nbytes = ctypes.c_void_p(), ctypes.c_int64()
    mb.check(_capi.load().megacu_b200_noalloc_scratch(device, ctypes.byref(ptr),
                                                      ctypes.byref(nbytes)))
    return ptr.value, nbytes.value


class _ControlWords:
    """The first 64 int32 words of the scratch (its control block) as a CUDA
    array, so a test can write into them with torch."""

    def __init__(self, ptr: int):
        self.__cuda_array_interface__ = {"shape": (64,), "typestr": "<i4",
                                         "data": (ptr, False), "version": 3}


def _graph_counters(prob: mb.Problem, tile_n: int) -> list[int]:
    """Completion counters of one one-PE call in the oracle's graph (they
    depend on m, n and the tiles, not on k or the data, so k = 8 here)."""
    m, n = prob.m, prob.n
    zeros_a = np.zeros((m, 8), np.float32)
    zeros_b = np.zeros((8, n), np.float32)
    ref = oracle_lib.bf16_call([zeros_a], [zeros_b], m=m, n=n, k=8, tile_n=tile_n)
    return ref["counters"][0].tolist()


def _noalloc_call(prob: mb.Problem, a, b, stream, trace=None):
    """One allocation-free call through the C ABI into a NaN-filled output;
    returns it with the counters the call added to the shared array."""
    events, _ = _scratch()
    before = mb.events_counters(events, stream)
    got = torch.full((prob.m, prob.n), float("nan"), dtype=torch.bfloat16, device="cuda")
    trace_ptr = trace.data_ptr() if trace is not None else None
    capacity = trace.numel() // 4 if trace is not None else 0
    st = _capi.load().megacu_cuda_gemm_bf16_noalloc(
        mb.driver_view(stream, 0), a.data_ptr(), b.data_ptr(), got.data_ptr(),
        prob.to_c(trace_ptr, capacity))
    assert st.code == 0, (st.code, st.detail, st.message)
    mb.events_status(events, stream)  # raises if a device wait of this call failed
    after = mb.events_counters(events, stream)
    return got, [x - y for x, y in zip(after, before)]


def _regular_call(prob: mb.Problem, a, b):
    ctx = SinglePE(prob)
    out = ctx.run(a, b).clone()
    return out, mb.events_counters(ctx.events), ctx.plan


@pytest.mark.gpu
@pytest.mark.skipif(gpu_count() < 1, reason="needs a CUDA GPU")
@pytest.mark.parametrize("m,n,k", [(512, 1024, 384), (200, 136, 72), (4096, 8192, 1024)])
def test_noalloc_matches_regular_entry_twice(m, n, k):
    a, b = inputs(31, 1, m, n, k)
    ad, bd = a[0].cuda(), b[0].cuda()
    prob = mb.Problem(m, n, k)
    want, want_counters, plan = _regular_call(prob, ad, bd)
    assert want_counters == _graph_counters(prob, plan.tile_n)
    stream = torch.cuda.Stream()
    for _ in range(2):
        got, added = _noalloc_call(prob, ad, bd, stream)
        assert torch.equal(got, want)  # the same kernel: the same bits
        assert added == want_counters


@pytest.mark.gpu
@pytest.mark.skipif(gpu_count() < 1, reason="needs a CUDA GPU")
def test_noalloc_shape_sequence_on_the_shared_array():
    """Stream-ordered calls of different tilings on the one shared array: CTA
    pairs, then single CTAs with 64-column tiles, then a traced call whose
    device queue must hand out its tiles in the oracle's order."""
    stream = torch.cuda.Stream()
    cases = [(mb.Problem(2048, 4096, 512, cta_pairs=mb.CTA_PAIRS_ON), None),
             (mb.Problem(256, 192, 64, tile_n=64), None),
             (mb.Problem(512, 768, 320, tile_n=128), "trace")]
    for i, (prob, traced) in enumerate(cases):
        a, b = inputs(40 + i, 1, prob.m, prob.n, prob.k)
        ad, bd = a[0].cuda(), b[0].cuda()
        want, want_counters, plan = _regular_call(prob, ad, bd)
        trace = (torch.zeros(plan.tiles * 4 * 4, dtype=torch.int64, device="cuda")
                 if traced else None)
        got, added = _noalloc_call(prob, ad, bd, stream, trace)
        assert torch.equal(got, want), prob
        assert added == want_counters == _graph_counters(prob, plan.tile_n), prob
        if trace is not None:
            tr = trace_records(trace)
            assert len(tr["kind"]) == plan.tiles and np.all(tr["kind"] == 0)
            assert sorted(tr["ticket"].tolist()) == list(range(plan.tiles))
            ref = oracle_lib.bf16_call([np.zeros((prob.m, 8), np.float32)],
                                       [np.zeros((8, prob.n), np.float32)], m=prob.m,
                                       n=prob.n, k=8, tile_n=plan.tile_n)
            assert np.array_equal(ref["gemm_order"][tr["ticket"]], tr["tile"])


@pytest.mark.gpu
@pytest.mark.skipif(gpu_count() < 1, reason="needs a CUDA GPU")
def test_noalloc_error_word_left_set_does_not_stop_the_next_call():
    """An error word left in the array (as a timed-out wait of an earlier
    call would leave it, if nobody read it) is cleared by the next call,
    which then computes its whole output."""
    m, n, k = 512, 1024, 256
    a, b = inputs(47, 1, m, n, k)
    ad, bd = a[0].cuda(), b[0].cuda()
    prob = mb.Problem(m, n, k)
    want, want_counters, _ = _regular_call(prob, ad, bd)
    events, _ = _scratch()
    words = torch.as_tensor(_ControlWords(events), device="cuda")
    stream = torch.cuda.current_stream()
    # error_code (word 4) = 41, a local pipeline timeout; error_info (words 5-7)
    words[4:8] = torch.tensor([41, 7, 0, 3], dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    got, added = _noalloc_call(prob, ad, bd, stream)
    assert torch.equal(got, want)
    assert added == want_counters
