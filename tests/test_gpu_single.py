"""Single-GPU parity of the sm_100a megakernel and megacu's fp32 launcher,
through the C ABI, against the CPU oracle (and, where built, the reference's
own fp32 kernel compiled from its sources)."""
from __future__ import annotations

import ctypes
import json
import os

import numpy as np
import pytest
import torch

import megacu_b200 as mb
import oracle_lib
from conftest import gpu_count
from gpu_util import REL_TOL, SinglePE, assert_close, f32, inputs, rel_error, trace_records

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(gpu_count() < 1, reason="needs a CUDA GPU")]

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kat_gemm_allreduce.json")


@pytest.mark.parametrize("m,n,k,tile_n", [
    (128, 256, 64, 256),     # one tile, one k-block
    (256, 512, 256, 0),      # several tiles and k-blocks
    (200, 136, 72, 64),      # ragged m, n and k (zero-filled TMA edges)
    (384, 384, 520, 128),
    (1024, 1024, 1024, 256),
    (16, 8192, 3584, 0),     # decode shape: one 16-row tile row, tile_n 64
    (1, 1024, 704, 0),       # one token: an 8-row A box, 19 stages
    (37, 520, 200, 128),     # ragged token count (40-row box), ragged n and k
    (100, 2048, 3584, 256),  # 104-row box, tile_n 256
    (64, 4096, 1024, 0),     # the 64-row box
    (130, 264, 8, 64),       # k shorter than one k-block
    (200, 264, 72, 128),     # one CTA pair: ragged lower tile, ragged last column tile
    (512, 768, 1000, 256),   # pairs with tile_n 256, k not a multiple of 64
])
@pytest.mark.parametrize("pairs", [mb.CTA_PAIRS_OFF, mb.CTA_PAIRS_AUTO])
def test_bf16_tp1_matches_oracle(m, n, k, tile_n, pairs):
    a, b = inputs(1, 1, m, n, k)
    prob = mb.Problem(m, n, k, tile_n=tile_n, cta_pairs=pairs)
    ctx = SinglePE(prob)
    out = ctx.run(a[0].cuda(), b[0].cuda())
    torch.cuda.synchronize()
    want = oracle_lib.bf16_call([f32(a[0])], [f32(b[0])], m=m, n=n, k=k,
                                tile_n=ctx.plan.tile_n)["out"][0]
    assert_close(f32(out), want)


@pytest.mark.parametrize("pairs", [mb.CTA_PAIRS_OFF, mb.CTA_PAIRS_ON])
def test_bf16_tp1_events_counters_trace_and_determinism(pairs):
    m, n, k = 512, 768, 320
    a, b = inputs(2, 1, m, n, k)
    prob = mb.Problem(m, n, k, tile_n=128, cta_pairs=pairs)
    ctx = SinglePE(prob)
    assert ctx.plan.cta_pairs == (pairs == mb.CTA_PAIRS_ON)
    tiles = ctx.plan.tiles
    trace = torch.zeros(tiles * 4 * 4, dtype=torch.int64, device="cuda")
    ev0 = ctx.event_words()
    out1 = ctx.run(a[0].cuda(), b[0].cuda(), trace=trace).clone()
    ev1 = ctx.event_words()
    counters = mb.events_counters(ctx.events)
    ref = oracle_lib.bf16_call([f32(a[0])], [f32(b[0])], m=m, n=n, k=k, tile_n=128, epoch=1,
                               events=[ev0])
    # event tensor and completion counts: bit-exact with the oracle's graph
    assert np.array_equal(ev1, ref["events"][0])
    assert counters == ref["counters"][0].tolist()
    # the device queue handed tiles out in the oracle's order
    tr = trace_records(trace)
    assert len(tr["kind"]) == tiles and np.all(tr["kind"] == 0)
    assert np.array_equal(ref["gemm_order"][tr["ticket"]], tr["tile"])
    assert sorted(tr["ticket"].tolist()) == list(range(tiles))
    # second call: epoch 2 lands in the other parity plane; same bits out
    out2 = ctx.run(a[0].cuda(), b[0].cuda())
    assert torch.equal(out1, out2)
    ev2 = ctx.event_words()
    ref2 = oracle_lib.bf16_call([f32(a[0])], [f32(b[0])], m=m, n=n, k=k, tile_n=128, epoch=2,
                                events=[ev1])
    assert np.array_equal(ev2, ref2["events"][0])
    assert mb.events_counters(ctx.events)[6] == 2


def test_bf16_tp1_pairs_equal_single_ctas_bitwise():
    """A 256-row pair MMA sums each output element over k in the same order as
    two 128-row MMAs: both tilings give the same bits."""
    m, n, k = 1024, 2048, 1536
    a, b = inputs(4, 1, m, n, k)
    ad, bd = a[0].cuda(), b[0].cuda()
    outs = []
    for pairs in (mb.CTA_PAIRS_OFF, mb.CTA_PAIRS_ON):
        ctx = SinglePE(mb.Problem(m, n, k, tile_n=256, cta_pairs=pairs))
        outs.append(ctx.run(ad, bd).clone())
    torch.cuda.synchronize()
    assert rel_error(f32(outs[1]), f32(outs[0])) < REL_TOL
    assert torch.equal(outs[0], outs[1])


def test_bf16_tp1_direct_launcher_equals_orchestrated():
    m, n, k = 256, 256, 128
    a, b = inputs(3, 1, m, n, k)
    ctx = SinglePE(mb.Problem(m, n, k))
    o1 = ctx.run(a[0].cuda(), b[0].cuda(), orchestrate=True).clone()
    o2 = ctx.run(a[0].cuda(), b[0].cuda(), orchestrate=False).clone()
    assert torch.equal(o1, o2)


def test_bf16_bench_shape_sampled_tiles():
    """C2 at tp = 1 (4096 x 8192 x 8192): sampled tiles against the oracle,
    the whole output against torch's fp32 GEMM of the same bf16 inputs."""
    m, n, k = 4096, 8192, 8192
    a, b = inputs(2, 1, m, n, k, std_a=0.02, std_b=0.02)
    ad, bd = a[0].cuda(), b[0].cuda()
    ctx = SinglePE(mb.Problem(m, n, k))
    out = ctx.run(ad, bd)
    torch.cuda.synchronize()
    full = torch.matmul(ad.float(), bd.float())
    assert_close(out.float().cpu().numpy(), full.cpu().numpy(), what="whole output vs torch fp32")
    pl = ctx.plan
    rng = np.random.default_rng(0)
    ids = np.sort(rng.choice(pl.tiles, 6, replace=False)).astype(np.int32)
    want = oracle_lib.bf16_tiles([f32(a[0])], [f32(b[0])], ids, m=m, n=n, k=k,
                                 tile_n=pl.tile_n)
    got = f32(out)
    for t in ids:
        r0, c0 = (t // pl.n_tiles) * 128, (t % pl.n_tiles) * pl.tile_n
        sl = (slice(r0, r0 + 128), slice(c0, c0 + pl.tile_n))
        assert_close(got[sl], want[sl], what=f"tile {t}")


# ---- megacu's fp32 phased launcher ------------------------------------------------

def _f32_call(a, b, m, n, k, tile_m, tile_n, orchestrate=True):
    dev = torch.device("cuda")
    ad = torch.tensor(a, device=dev)
    bd = torch.tensor(b, device=dev)
    partial = torch.zeros(m * n, dtype=torch.float32, device=dev)
    out = torch.zeros(m, n, dtype=torch.float32, device=dev)
    tiles = -(-m // tile_m) * -(-n // tile_n)
    events = torch.zeros(max(tiles, 32), dtype=torch.int32, device=dev)
    d = mb.driver_view(torch.cuda.current_stream(), 0)
    fn = (mb.cuda_nvshmem_gemm_allreduce_phased_orchestrate if orchestrate
          else mb.megacu_cuda_gemm_allreduce_phased_f32)
    mb.check(fn(d, ad, bd, partial, out, events, m, n, k, tile_m, tile_n))
    torch.cuda.synchronize()
    return out.cpu().numpy(), events[:tiles].cpu().numpy()


def test_f32_kat_single_pe():
    with open(GOLDEN) as f:
        kat = json.load(f)["single_pe"]
    a = np.array(kat["a"], np.float32).reshape(kat["m"], kat["k"])
    b = np.array(kat["b"], np.float32).reshape(kat["k"], kat["n"])
    for orch in (True, False):
        out, events = _f32_call(a, b, kat["m"], kat["n"], kat["k"], kat["tile_m"], kat["tile_n"],
                                orch)
        want = np.array(kat["expected"], np.float32).reshape(kat["m"], kat["n"])
        assert np.max(np.abs(out - want)) < kat["tolerance"]
        assert events.tolist() == list(range(1, len(events) + 1))


def test_f32_bit_exact_with_oracle_and_reference_kernel():
    rng = np.random.default_rng(5)
    m, n, k, tm, tn = 200, 136, 70, 16, 32
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((k, n), dtype=np.float32)
    out, _ = _f32_call(a, b, m, n, k, tm, tn)
    want, _ = oracle_lib.phased_f32([a], [b], m, n, k, tm, tn)
    assert out.tobytes() == want[0].tobytes()
    if os.path.exists(oracle_lib.REF_F32_PATH):
        ref = ctypes.CDLL(oracle_lib.REF_F32_PATH)
        fn = ref.megacu_cuda_gemm_allreduce_phased_f32
        from megacu_b200 import _capi
        fn.restype = _capi.Status
        fn.argtypes = [_capi.DriverView] + [ctypes.c_void_p] * 5 + [_capi.GemmArProblem]
        dev = torch.device("cuda")
        ad, bd = torch.tensor(a, device=dev), torch.tensor(b, device=dev)
        partial = torch.zeros(m * n, dtype=torch.float32, device=dev)
        rout = torch.zeros(m, n, dtype=torch.float32, device=dev)
        events = torch.zeros(4096, dtype=torch.int32, device=dev)
        d = mb.driver_view(torch.cuda.current_stream(), 0)
        st = fn(d, ad.data_ptr(), bd.data_ptr(), partial.data_ptr(), rout.data_ptr(),
                events.data_ptr(), _capi.GemmArProblem(m=m, n=n, k=k, tile_m=tm, tile_n=tn))
        assert st.code == 0
        torch.cuda.synchronize()
        assert rout.cpu().numpy().tobytes() == out.tobytes()
