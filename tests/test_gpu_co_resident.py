"""megacu's fp32 phase with co-resident persistent progress on the GPU: one
cooperative persistent launch of the generic device loop over the lowered
unit graph. Its operators are the phased launcher's, so the output must
match that launcher and the oracle bit for bit, and the event tensor must
hold megacu's ready values (tile + 1 in every PE's slot).

Every case and the example have passed on B200s. The lowering and
validation are covered without a GPU in test_co_resident.py.
"""
from __future__ import annotations


import numpy as np
import pytest
import torch

import megacu_b200 as mb
import oracle_lib
from conftest import gpu_count
from gpu_util import same_process_team

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k,tm,tn", [(200, 136, 70, 16, 32), (256, 256, 64, 128, 128),
                                         (64, 4096, 33, 64, 64)])
def test_one_pe_bit_exact_with_phased_launcher(m, n, k, tm, tn):
    rng = np.random.default_rng(11)
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((k, n), dtype=np.float32)
    dev = torch.device("cuda", 0)
    ad, bd = torch.tensor(a, device=dev), torch.tensor(b, device=dev)
    tiles = -(-m // tm) * -(-n // tn)
    outs, events = [], []
    control = torch.empty(mb.co_resident_control_bytes(), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    for co in (False, True):
        partial = torch.zeros(m * n, dtype=torch.float32, device=dev)
        out = torch.zeros(m, n, dtype=torch.float32, device=dev)
        ev = torch.full((tiles,), -5, dtype=torch.int32, device=dev)
        d = mb.driver_view(stream, 0)
        for _ in range(2):
            if co:
                st = mb.megacu_cuda_gemm_allreduce_f32_co_resident(d, ad, bd, partial, out, ev,
                                                                   control, m, n, k, tm, tn)
            else:
                st = mb.megacu_cuda_gemm_allreduce_phased_f32(d, ad, bd, partial, out, ev, m, n,
                                                              k, tm, tn)
            mb.check(st)
        if co:
            mb.co_resident_status(control, stream)
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy())
        events.append(ev.cpu().numpy())
    want, _ = oracle_lib.phased_f32([a], [b], m, n, k, tm, tn)
    assert outs[1].tobytes() == outs[0].tobytes() == want[0].tobytes()
    assert events[1].tolist() == events[0].tolist() == list(range(1, tiles + 1))


@pytest.mark.skipif(gpu_count() < 2, reason="needs two GPUs")
def test_two_pes_match_oracle():
    m, n, k, tm, tn = 256, 384, 96, 64, 128
    rng = np.random.default_rng(12)
    a = [rng.standard_normal((m, k), dtype=np.float32) for _ in range(2)]
    b = [rng.standard_normal((k, n), dtype=np.float32) for _ in range(2)]
    teams = same_process_team([0, 1])
    try:
        tiles = -(-m // tm) * -(-n // tn)
        bufs = []
        for pe, t in enumerate(teams):
            dev = torch.device("cuda", t.device)
            bufs.append(dict(
                a=torch.tensor(a[pe], device=dev), b=torch.tensor(b[pe], device=dev),
                partial=t.tensor((m * n,), torch.float32),
                events=t.tensor((2 * tiles,), torch.int32),
                out=torch.zeros(m, n, dtype=torch.float32, device=dev),
                control=torch.empty(mb.co_resident_control_bytes(), dtype=torch.uint8,
                                    device=dev),
                stream=torch.cuda.Stream(device=dev)))
        for pe in range(2):
            torch.cuda.synchronize(pe)
        for pe, t in enumerate(teams):
            x = bufs[pe]
            d = mb.driver_view(x["stream"], t.device, t)
            with torch.cuda.device(t.device):
                mb.check(mb.megacu_cuda_gemm_allreduce_f32_co_resident(
                    d, x["a"], x["b"], x["partial"], x["out"], x["events"], x["control"],
                    m, n, k, tm, tn))
        for pe in range(2):
            mb.co_resident_status(bufs[pe]["control"], bufs[pe]["stream"])
        want, want_ev = oracle_lib.phased_f32(a, b, m, n, k, tm, tn)
        for pe in range(2):
            assert bufs[pe]["out"].cpu().numpy().tobytes() == want[pe].tobytes()
            ev = bufs[pe]["events"].cpu().numpy().reshape(2, tiles)
            assert np.array_equal(ev, want_ev[pe])
    finally:
        for pe in range(2):
            torch.cuda.synchronize(pe)
        for t in teams:
            t.close()


def test_three_task_example_with_two_acquired_tensors(tmp_path):
    """tests/cpp/co_resident_example.cu: fill -> scale -> sum, the last task
    acquiring both tensors, one persistent launch, checked on the host."""
    import subprocess

    from test_co_resident import build_example
    exe = build_example(str(tmp_path))
    proc = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0 and proc.stdout.strip() == "ok", proc.stdout + proc.stderr
