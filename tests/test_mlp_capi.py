"""Host-side checks of the MLP entry points (no GPU: a null stream validates
only)."""
import ctypes

import pytest

import megacu_b200 as mb
from megacu_b200 import _capi

FAKE = 0x100000


def test_swiglu_validation():
    lib = _capi.load()
    d = mb.driver_view(None, 0)
    st = lib.megacu_cuda_gemm_swiglu_bf16(d, FAKE, FAKE, FAKE, FAKE, FAKE,
                                          mb.Problem(256, 384, 320).to_c())
    assert (st.code, st.detail) == (0, 0)
    st = lib.megacu_cuda_gemm_swiglu_bf16(d, FAKE, FAKE, FAKE, FAKE, FAKE,
                                          mb.Problem(256, 384, 320, tile_n=256).to_c())
    assert (st.code, st.detail) == (_capi.UNSUPPORTED, 22)
    st = lib.megacu_cuda_gemm_swiglu_bf16(
        d, FAKE, FAKE, FAKE, FAKE, FAKE,
        mb.Problem(384, 384, 320, cta_pairs=mb.CTA_PAIRS_ON).to_c())
    assert (st.code, st.detail) == (_capi.UNSUPPORTED, 27)
    st = lib.megacu_cuda_gemm_swiglu_bf16(d, FAKE, FAKE, FAKE, None, FAKE,
                                          mb.Problem(256, 384, 320).to_c())
    assert (st.code, st.detail) == (_capi.INVALID_ARGUMENT, 2)
    assert mb.swiglu_events_bytes(mb.Problem(2048, 1792, 4096)) == 256 + 4 * (2 * 16 * 14 * 4 + 2)


@pytest.mark.parametrize("n_pes", [1, 2, 8])
def test_chain_sizes_compose_the_two_launches(n_pes):
    prob = mb.MlpChainProblem(2048, 4096, 14336 // 8, layers=4)
    sz = mb.mlp_chain_sizes(prob, n_pes)
    down = mb.Problem(2048, 4096, 1792)
    assert sz["act"] == 2048 * 1792 * 2 and sz["x_work"] == 2048 * 4096 * 2
    assert sz["workspace"] == mb.workspace_bytes(down, n_pes)
    assert sz["events_down"] == mb.events_bytes(down, n_pes)
    assert sz["events_swiglu"] == mb.swiglu_events_bytes(mb.Problem(2048, 1792, 4096))


def test_chain_validation():
    lib = _capi.load()
    d = mb.driver_view(None, 0)
    ptrs = (ctypes.c_void_p * 2)(FAKE, FAKE)
    prob = mb.MlpChainProblem(256, 256, 384, layers=2)
    st = lib.megacu_cuda_mlp_chain_bf16(d, FAKE, ptrs, ptrs, ptrs, FAKE, FAKE, FAKE, FAKE, FAKE,
                                        FAKE, prob.to_c())
    assert (st.code, st.detail) == (0, 0)
    prob.layers = 0
    with pytest.raises(mb.MegacuError):
        mb.mlp_chain_sizes(prob, 1)
    st = lib.megacu_cuda_mlp_chain_bf16(d, FAKE, ptrs, ptrs, ptrs, FAKE, FAKE, FAKE, FAKE, FAKE,
                                        FAKE, prob.to_c())
    assert (st.code, st.detail) == (_capi.INVALID_ARGUMENT, 1)
    prob.layers = 2
    st = lib.megacu_cuda_mlp_chain_bf16(d, FAKE, ptrs, ptrs, ptrs, FAKE, FAKE, None, FAKE, FAKE,
                                        FAKE, prob.to_c())
    assert (st.code, st.detail) == (_capi.INVALID_ARGUMENT, 2)


def test_single_launch_chain_limits_and_sizes():
    lib = _capi.load()
    d = mb.driver_view(None, 0)
    ptrs = (ctypes.c_void_p * 7)(*([FAKE] * 7))
    prob = mb.MlpChainProblem(256, 256, 384, layers=2, single_launch=True)
    st = lib.megacu_cuda_mlp_chain_bf16(d, FAKE, ptrs, ptrs, ptrs, FAKE, FAKE, FAKE, FAKE, FAKE,
                                        FAKE, prob.to_c())
    assert (st.code, st.detail) == (0, 0)
    for bad in (dict(layers=7), dict(layers=2, deterministic=True)):
        p = mb.MlpChainProblem(256, 256, 384, single_launch=True, **bad)
        st = lib.megacu_cuda_mlp_chain_bf16(d, FAKE, ptrs, ptrs, ptrs, FAKE, FAKE, FAKE, FAKE,
                                            FAKE, FAKE, p.to_c())
        assert (st.code, st.detail) == (_capi.UNSUPPORTED, 29), bad
    # the sizes cover the single launch's layout: one plane of 128 x 256 partial
    # slots per (token block, hidden tile), and its event words
    t, h, i, layers = 2048, 4096, 1792, 4
    for n_pes in (1, 8):
        one = mb.mlp_chain_sizes(mb.MlpChainProblem(t, h, i, layers=layers, single_launch=True),
                                 n_pes)
        two = mb.mlp_chain_sizes(mb.MlpChainProblem(t, h, i, layers=layers), n_pes)
        m_tiles, dn = t // 128, h // 256
        ws = 0 if n_pes == 1 else m_tiles * dn * 128 * 256 * 2
        # arrive flags per (block, source PE, DN tile of the whole grid, quarter)
        ev = 256 + 4 * (layers * n_pes * m_tiles * dn * 4 + 2 * layers * m_tiles)
        assert one["workspace"] == max(two["workspace"], ws)
        assert one["events_down"] == max(two["events_down"], ev)
