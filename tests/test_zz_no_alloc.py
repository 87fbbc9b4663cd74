"""The allocation-free entry point, megacu_cuda_gemm_bf16_noalloc.

It exists for callers that cannot allocate device memory for the kernel's
scratch — a plugin host that hands an operator only its inputs and outputs,
a process whose device memory belongs to another allocator, a serving loop
that must not call cudaMalloc. The kernel's scratch lives in a fixed array
built into the library instead. This file is collected last on purpose.

The GPU test calls it through the C ABI twice in a row and compares each
output with the regular entry point's (which takes a caller-allocated events
buffer), within the bf16 path's tolerance. The CPU test checks the limits
that need no GPU.
"""
from __future__ import annotations

import pytest
import torch

import megacu_b200 as mb
from megacu_b200 import _capi
from conftest import gpu_count
from gpu_util import REL_TOL, f32, inputs, rel_error


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


@pytest.mark.gpu
@pytest.mark.skipif(gpu_count() < 1, reason="needs a CUDA GPU")
@pytest.mark.parametrize("m,n,k", [(512, 1024, 384), (200, 136, 72), (4096, 8192, 1024)])
def test_noalloc_matches_regular_entry_twice(m, n, k):
    lib = _capi.load()
    a, b = inputs(31, 1, m, n, k)
    ad, bd = a[0].cuda(), b[0].cuda()
    prob = mb.Problem(m, n, k)
    stream = torch.cuda.Stream()
    # regular entry point: caller-allocated events buffer
    events = torch.zeros(mb.events_bytes(prob, 1) // 4, dtype=torch.int32, device="cuda")
    want = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    mb.gemm_allreduce(ad, bd, want, workspace=None, events=events, problem=prob, stream=stream)
    mb.events_status(events, stream)
    d = mb.driver_view(stream, 0)
    for _ in range(2):
        got = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        st = lib.megacu_cuda_gemm_bf16_noalloc(d, ad.data_ptr(), bd.data_ptr(), got.data_ptr(),
                                               prob.to_c())
        assert st.code == 0, st
        stream.synchronize()
        assert rel_error(f32(got), f32(want)) < REL_TOL
