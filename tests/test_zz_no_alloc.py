"""kv800_decode_noalloc, the decode entry point for callers that cannot allocate device memory while decoding (it
uses a scratch array built into the library instead of a caller-provided workspace).  Called through the C ABI
twice in a row on the same inputs; each output must match kv800_decode's (the workspace entry point) within the
decode tolerance of the other tests, and the CPU oracle on the same pools.  Both schedule forms are covered: the
persistent quantized pass (spb = 0, counters cleared by the schedule kernel) and the grid of fixed splits (spb = 4,
cleared by a memset), plus a large decode followed by a small one (the small one must not pick up the large one's
leftover scratch).  After each call the status word inside the array reads 0.  This file is named to run last."""
import ctypes

import numpy as np
import pytest
import torch

import inputs as I
from _util import assert_parity, assert_parity_ulp, nb, tb
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _store(kv800, win, n, B, seed):
    K, V, q = I.parity_inputs(win, n, B=B, seed=seed)
    st = kv800.PagedStore(B, n + 8, DEV, window=win)
    st.append(tb(K, DEV), tb(V, DEV))
    return st, q


def _oracle(st, q, cs, sn):
    P = st.paged()
    Pn = dict(qpool=P.qpool.cpu().numpy(), boff=P.boff.cpu().numpy(), epool=nb(P.epool), eoff=P.eoff.cpu().numpy(),
              ebs=P.ebs, e_hs=P.e_hs, e_ts=P.e_ts, e_v=P.e_v, sk=None if P.sk is None else nb(P.sk),
              sv=None if P.sv is None else nb(P.sv), skoff=P.skoff.cpu().numpy(), svoff=P.svoff.cpu().numpy(),
              N=P.N.cpu().numpy(), NQ=P.NQ.cpu().numpy(), nqmax=P.nqmax, win=P.win)
    return O.decode(Pn, q, cs, sn)


def _noalloc(L, kv800, st, qd, c32, s32, spb):
    B = qd.shape[0]
    s, keep = kv800._paged_struct(st.paged(), torch.device(DEV), B)
    out = torch.full((B, 16, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.kv800_decode_noalloc(ctypes.byref(s), ctypes.c_void_p(qd.data_ptr()), ctypes.c_void_p(c32.data_ptr()),
                                ctypes.c_void_p(s32.data_ptr()), c32.shape[0], B, spb,
                                ctypes.c_void_p(out.data_ptr()), stream)
    assert rc == 0, L.kv800_last_error()
    status = ctypes.c_int(-1)
    assert L.kv800_decode_noalloc_status(ctypes.byref(status), stream) == 0, L.kv800_last_error()
    assert status.value == 0
    del keep
    return nb(out)


@pytest.mark.parametrize("win,n,spb", [(0, 1500, 0), (0, 1500, 4), (256, 700, 0)])
def test_noalloc_matches_workspace_decode_twice(win, n, spb):
    from lfm3_kv800 import _lib, kv800
    st, q = _store(kv800, win, n, 3, 4)
    cs, sn = I.rope_tables(4096)
    qd, c32, s32 = tb(q, DEV), tb(cs, DEV), tb(sn, DEV)
    ref = nb(kv800.decode(st.paged(), qd, c32, s32, st.H, spb=spb or None))
    oracle = _oracle(st, q, cs, sn)
    L = _lib.lib()
    for call in range(2):
        got = _noalloc(L, kv800, st, qd, c32, s32, spb)
        assert_parity(got, ref, f"no-alloc decode vs kv800_decode, call {call + 1}")
        # these synthetic outputs reach magnitude 4, where one bf16 ulp exceeds 2e-2: max(2e-2, 1 ulp) per element
        assert_parity_ulp(got, oracle, f"no-alloc decode vs oracle, call {call + 1}")


def test_noalloc_large_then_small():
    """A 24-row decode fills more of the array than the 2-row decode after it; the small one's counters, status
    word and partials must all be its own."""
    from lfm3_kv800 import _lib, kv800
    cs, sn = I.rope_tables(4096)
    c32, s32 = tb(cs, DEV), tb(sn, DEV)
    L = _lib.lib()
    big, qb = _store(kv800, 0, 2100, 24, 8)
    small, qs = _store(kv800, 0, 900, 2, 9)
    for spb in (0, 4):
        gb = _noalloc(L, kv800, big, tb(qb, DEV), c32, s32, spb)
        gs = _noalloc(L, kv800, small, tb(qs, DEV), c32, s32, spb)
        assert_parity(gb, nb(kv800.decode(big.paged(), tb(qb, DEV), c32, s32, spb=spb or None)), f"large, spb {spb}")
        assert_parity(gs, nb(kv800.decode(small.paged(), tb(qs, DEV), c32, s32, spb=spb or None)), f"small, spb {spb}")
    assert_parity_ulp(gs, _oracle(small, qs, cs, sn), "small vs oracle")


def test_noalloc_rejects_oversized_decode():
    from lfm3_kv800 import _lib, kv800
    L = _lib.lib()
    s = _lib.Paged()
    s.win, s.nqmax = 0, 127
    # 4096 rows x 127 sub-blocks at spb = 1 needs far more than the built-in scratch: rejected on the host
    rc = L.kv800_decode_noalloc(ctypes.byref(s), None, None, None, 1, 4096, 1, None, None)
    assert rc == _lib.ERR_RANGE
    assert b"scratch" in L.kv800_last_error()
