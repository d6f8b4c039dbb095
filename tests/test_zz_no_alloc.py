"""kv800_decode_noalloc, the decode entry point for callers that cannot allocate device memory while decoding (it
uses a scratch array built into the library instead of a caller-provided workspace).  Called through the C ABI
twice in a row on the same inputs; each output must match kv800_decode's (the workspace entry point) within the
decode tolerance of the other tests.  This file is named to run last."""
import ctypes

import numpy as np
import pytest
import torch

import inputs as I
from _util import assert_parity, nb, tb

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("win,n", [(0, 1500), (256, 700)])
def test_noalloc_matches_workspace_decode_twice(win, n):
    from lfm3_kv800 import _lib, kv800
    K, V, q = I.parity_inputs(win, n, B=3, seed=4)
    cs, sn = I.rope_tables(4096)
    st = kv800.PagedStore(3, n + 8, DEV, window=win)
    st.append(tb(K, DEV), tb(V, DEV))
    qd, c32, s32 = tb(q, DEV), tb(cs, DEV), tb(sn, DEV)
    ref = nb(kv800.decode(st.paged(), qd, c32, s32, st.H))

    s, keep = kv800._paged_struct(st.paged(), torch.device(DEV), 3)
    L = _lib.lib()
    for call in range(2):
        out = torch.full((3, 16, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
        rc = L.kv800_decode_noalloc(ctypes.byref(s), ctypes.c_void_p(qd.data_ptr()), ctypes.c_void_p(c32.data_ptr()),
                                    ctypes.c_void_p(s32.data_ptr()), c32.shape[0], 3, 0,
                                    ctypes.c_void_p(out.data_ptr()),
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, L.kv800_last_error()
        torch.cuda.synchronize()
        assert_parity(nb(out), ref, f"no-alloc decode, call {call + 1}")
    del keep


def test_noalloc_rejects_oversized_decode():
    from lfm3_kv800 import _lib, kv800
    L = _lib.lib()
    s = _lib.Paged()
    s.win, s.nqmax = 0, 127
    # 4096 rows x 127 sub-blocks at spb = 1 needs far more than the built-in scratch: rejected on the host
    rc = L.kv800_decode_noalloc(ctypes.byref(s), None, None, None, 1, 4096, 1, None, None)
    assert rc == _lib.ERR_RANGE
    assert b"scratch" in L.kv800_last_error()
