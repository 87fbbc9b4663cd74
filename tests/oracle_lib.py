"""ctypes binding of the CPU oracle (oracle/liboracle.so) — test infrastructure.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use
this module, as the checker / the timed CPU baseline.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_PATH = os.path.join(ROOT, "oracle", "liboracle.so")
REF_HOST_PATH = os.path.join(ROOT, "oracle", "_ref", "libref_host_harness.so")
REF_F32_PATH = os.path.join(ROOT, "oracle", "_ref", "libref_phased_f32.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_lib = None


class OracleBf16Problem(ctypes.Structure):
    _fields_ = [("m", ctypes.c_int64), ("n", ctypes.c_int64), ("k", ctypes.c_int64),
                ("tile_m", ctypes.c_int32), ("tile_n", ctypes.c_int32),
                ("n_pes", ctypes.c_int32), ("mode", ctypes.c_int32),
                ("one_shot", ctypes.c_int32), ("group_m", ctypes.c_int32),
                ("wire_bytes", ctypes.c_int32), ("threads", ctypes.c_int32),
                ("epoch", ctypes.c_uint32)]


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_PATH):
            raise ImportError(f"oracle not built: make -C oracle ({ORACLE_PATH})")
        lib = ctypes.CDLL(ORACLE_PATH)
        lib.oracle_gemm_f32.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_int64, ctypes.c_int32]
        lib.oracle_round_bf16.argtypes = [ctypes.c_float]
        lib.oracle_round_bf16.restype = ctypes.c_float
        lib.oracle_phased_f32.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                          ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                          ctypes.POINTER(_f32p), ctypes.POINTER(_f32p),
                                          ctypes.POINTER(_f32p),
                                          ctypes.POINTER(ctypes.POINTER(ctypes.c_int32))]
        lib.oracle_locate.argtypes = [ctypes.c_int32] * 6 + [ctypes.POINTER(ctypes.c_int32)]
        lib.oracle_pair_raster.argtypes = [ctypes.c_int32] * 3 + [ctypes.POINTER(ctypes.c_int32)]
        lib.oracle_bf16_call.argtypes = [ctypes.POINTER(OracleBf16Problem),
                                         ctypes.POINTER(_f32p), ctypes.POINTER(_f32p),
                                         ctypes.POINTER(_f32p),
                                         ctypes.POINTER(ctypes.POINTER(ctypes.c_uint32)),
                                         ctypes.POINTER(ctypes.c_uint64),
                                         ctypes.POINTER(ctypes.c_int32),
                                         ctypes.POINTER(ctypes.POINTER(ctypes.c_int32))]
        lib.oracle_bf16_tiles.argtypes = [ctypes.POINTER(OracleBf16Problem),
                                          ctypes.POINTER(_f32p), ctypes.POINTER(_f32p),
                                          ctypes.POINTER(ctypes.c_int32), ctypes.c_int32, _f32p]
        lib.oracle_mlp_chain.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _f32p,
                                         ctypes.POINTER(_f32p), ctypes.POINTER(_f32p),
                                         ctypes.POINTER(_f32p), _f32p, ctypes.c_int32]
        lib.oracle_allgather_gemm.argtypes = [ctypes.POINTER(OracleBf16Problem),
                                              ctypes.POINTER(_f32p), ctypes.POINTER(_f32p),
                                              ctypes.POINTER(_f32p), ctypes.POINTER(_f32p),
                                              ctypes.POINTER(ctypes.POINTER(ctypes.c_uint32)),
                                              ctypes.POINTER(ctypes.c_uint64),
                                              ctypes.POINTER(ctypes.POINTER(ctypes.c_int32))]
        lib.oracle_locate_gather.argtypes = [ctypes.c_int32] * 6 + [ctypes.POINTER(ctypes.c_int32)]
        lib.oracle_gather_chunk_rows.argtypes = [ctypes.c_int64]
        lib.oracle_gather_chunk_rows.restype = ctypes.c_int32
        lib.oracle_gather_events_words.argtypes = [ctypes.c_int32] * 3
        lib.oracle_gather_events_words.restype = ctypes.c_int64
        lib.oracle_chain_events_words.argtypes = [ctypes.c_int32, ctypes.c_int32,
                                                  ctypes.c_int64, ctypes.c_int64]
        lib.oracle_chain_events_words.restype = ctypes.c_int64
        lib.oracle_chain_events.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
                                            ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                            ctypes.c_uint32,
                                            ctypes.POINTER(ctypes.POINTER(ctypes.c_uint32)),
                                            ctypes.POINTER(ctypes.c_uint64)]
        _lib = lib
    return _lib


def _fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def _fp_array(arrs):
    return (_f32p * len(arrs))(*[_fp(x) for x in arrs])


def gemm_f32(a: np.ndarray, b: np.ndarray, threads: int = 0) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    load().oracle_gemm_f32(_fp(a), _fp(b), _fp(c), m, n, k, threads or os.cpu_count() or 1)
    return c


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bf16, returned as fp32 (vectorised; matches the C oracle)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7F800000) == 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000)
    quiet = np.where((u & np.uint64(0x007FFFFF)) != 0, np.uint64(0x00400000), np.uint64(0))
    r = np.where(nan, (u | quiet) & np.uint64(0xFFFF0000), r)
    return r.astype(np.uint32).view(np.float32)


def phased_f32(a_list, b_list, m, n, k, tile_m, tile_n):
    """megacu's fp32 phased graph on len(a_list) logical PEs -> (outs, events)."""
    n_pes = len(a_list)
    a_list = [np.ascontiguousarray(x, np.float32) for x in a_list]
    b_list = [np.ascontiguousarray(x, np.float32) for x in b_list]
    tiles = -(-m // tile_m) * -(-n // tile_n)
    outs = [np.zeros((m, n), np.float32) for _ in range(n_pes)]
    evs = [np.zeros(tiles * n_pes, np.int32) for _ in range(n_pes)]
    evp = (ctypes.POINTER(ctypes.c_int32) * n_pes)(
        *[e.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)) for e in evs])
    rc = load().oracle_phased_f32(m, n, k, tile_m, tile_n, n_pes, _fp_array(a_list),
                                  _fp_array(b_list), _fp_array(outs), evp)
    assert rc == 0, rc
    return outs, [e.reshape(n_pes, tiles) for e in evs]


def locate(m_tiles, n_tiles, n_pes, mode, group_m, r):
    out = (ctypes.c_int32 * 4)()
    load().oracle_locate(m_tiles, n_tiles, n_pes, mode, group_m, r, out)
    return tuple(out)


def pair_raster(n_pes, mode, q):
    out = (ctypes.c_int32 * 2)()
    load().oracle_pair_raster(n_pes, mode, q, out)
    return tuple(out)


def bf16_call(a_list, b_list, *, m, n, k, tile_n, mode=0, one_shot=False, group_m=16,
              wire_bytes=2, epoch=1, events=None, threads=0):
    """The megakernel's task graph for one call on len(a_list) logical PEs.

    Returns dict(out=[...], events=[...] or None, counters=(n_pes, 8),
    gemm_order=[tiles], reduce_order=[[tiles*4] per PE]).
    """
    n_pes = len(a_list)
    a_list = [np.ascontiguousarray(x, np.float32) for x in a_list]
    b_list = [np.ascontiguousarray(x, np.float32) for x in b_list]
    m_tiles, n_tiles = -(-m // 128), -(-n // tile_n)
    tiles = m_tiles * n_tiles
    rows = m // n_pes if mode == 1 else m
    outs = [np.zeros((rows, n), np.float32) for _ in range(n_pes)]
    p = OracleBf16Problem(m, n, k, 128, tile_n, n_pes, mode, 1 if one_shot else 0, group_m,
                          wire_bytes, threads or os.cpu_count() or 1, epoch)
    evp = None
    if events is not None:
        events = [np.ascontiguousarray(e, np.uint32) for e in events]
        evp = (ctypes.POINTER(ctypes.c_uint32) * n_pes)(
            *[e.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)) for e in events])
    counters = np.zeros((n_pes, 8), np.uint64)
    gemm_order = np.zeros(tiles, np.int32)
    reduce_orders = [np.full(tiles * 4 * (tile_n // 64), -1, np.int32) for _ in range(n_pes)]
    rop = (ctypes.POINTER(ctypes.c_int32) * n_pes)(
        *[r.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)) for r in reduce_orders])
    rc = load().oracle_bf16_call(ctypes.byref(p), _fp_array(a_list), _fp_array(b_list),
                                 _fp_array(outs), evp,
                                 counters.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)),
                                 gemm_order.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), rop)
    assert rc == 0, rc
    return dict(out=outs, events=events, counters=counters, gemm_order=gemm_order,
                reduce_order=reduce_orders)


def bf16_tiles(a_list, b_list, tile_ids, *, m, n, k, tile_n, wire_bytes=2, threads=0):
    """Summed output of the listed tiles only (CPU-baseline sample)."""
    n_pes = len(a_list)
    out = np.zeros((m, n), np.float32)
    ids = np.ascontiguousarray(tile_ids, np.int32)
    p = OracleBf16Problem(m, n, k, 128, tile_n, n_pes, 0, 0, 16, wire_bytes,
                          threads or os.cpu_count() or 1, 1)
    load().oracle_bf16_tiles(ctypes.byref(p), _fp_array(list(a_list)), _fp_array(list(b_list)),
                             ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(ids),
                             _fp(out))
    return out


def mlp_chain(x, wg, wu, wd, *, wire_bytes=2, threads=0):
    """The MLP chain's output. x: [t, h]; wg, wu: [layers][n_pes] of [h, i];
    wd: [layers][n_pes] of [i, h] (bf16 values as float32)."""
    layers, n_pes = len(wg), len(wg[0])
    t, h = x.shape
    i = wg[0][0].shape[1]
    x = np.ascontiguousarray(x, np.float32)
    flat = lambda ws: [np.ascontiguousarray(w, np.float32) for layer in ws for w in layer]
    g, u, d = flat(wg), flat(wu), flat(wd)
    out = np.empty((t, h), np.float32)
    load().oracle_mlp_chain(t, h, i, layers, n_pes, wire_bytes, _fp(x), _fp_array(g), _fp_array(u),
                            _fp_array(d), _fp(out), threads or os.cpu_count() or 1)
    return out


def event_tensor_words(n_pes: int, tiles: int) -> int:
    """uint32 words of the event tensor after the control block
    (arrive [2][n_pes][tiles][4], then done [2][n_pes])."""
    return 2 * n_pes * tiles * 4 + 2 * n_pes


def locate_gather(m_tiles, n_tiles, n_pes, my_pe, group_m, r):
    out = (ctypes.c_int32 * 4)()
    load().oracle_locate_gather(m_tiles, n_tiles, n_pes, my_pe, group_m, r, out)
    return tuple(out)


def gather_chunk_rows(k):
    return load().oracle_gather_chunk_rows(k)


def gather_events_words(n_pes, tiles, m_tiles_per_pe):
    return load().oracle_gather_events_words(n_pes, tiles, m_tiles_per_pe)


def allgather_gemm(a_shards, b_list, *, m, n, k, tile_n, group_m=16, epoch=1, events=None,
                   threads=0):
    """The all-gather + GEMM graph for one call on len(a_shards) logical PEs.

    Returns dict(gathered=[...], out=[...], events=[...] or None,
    counters=(n_pes, 8), gemm_order=[[tiles] per PE]).
    """
    n_pes = len(a_shards)
    a_shards = [np.ascontiguousarray(x, np.float32) for x in a_shards]
    b_list = [np.ascontiguousarray(x, np.float32) for x in b_list]
    tiles = (m // 128) * -(-n // tile_n)
    gathered = [np.zeros((m, k), np.float32) for _ in range(n_pes)]
    outs = [np.zeros((m, n), np.float32) for _ in range(n_pes)]
    p = OracleBf16Problem(m, n, k, 128, tile_n, n_pes, 2, 0, group_m, 2,
                          threads or os.cpu_count() or 1, epoch)
    evp = None
    if events is not None:
        events = [np.ascontiguousarray(e, np.uint32) for e in events]
        evp = (ctypes.POINTER(ctypes.c_uint32) * n_pes)(
            *[e.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)) for e in events])
    counters = np.zeros((n_pes, 8), np.uint64)
    orders = [np.full(tiles, -1, np.int32) for _ in range(n_pes)]
    op = (ctypes.POINTER(ctypes.c_int32) * n_pes)(
        *[o.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)) for o in orders])
    rc = load().oracle_allgather_gemm(ctypes.byref(p), _fp_array(a_shards), _fp_array(b_list),
                                      _fp_array(gathered), _fp_array(outs), evp,
                                      counters.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), op)
    assert rc == 0, rc
    return dict(gathered=gathered, out=outs, events=events, counters=counters, gemm_order=orders)


def chain_events(layers, n_pes, tokens, hidden, inter, *, epoch=1, events=None, group_m=16):
    """The single-launch chain's event words (per PE, after the control block)
    and per-call counter deltas. `events` (optional) is updated in place."""
    words = load().oracle_chain_events_words(layers, n_pes, tokens, hidden)
    if events is None:
        events = [np.zeros(words, np.uint32) for _ in range(n_pes)]
    events = [np.ascontiguousarray(e, np.uint32) for e in events]
    evp = (ctypes.POINTER(ctypes.c_uint32) * n_pes)(
        *[e.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)) for e in events])
    counters = np.zeros((n_pes, 8), np.uint64)
    load().oracle_chain_events(layers, n_pes, tokens, hidden, inter, group_m, epoch, evp,
                               counters.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)))
    return dict(events=events, counters=counters, words=words)
