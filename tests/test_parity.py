"""Decode parity, the reference's own test (tests/test_parity.py: 12 cases, quantized layer at n = 50 .. 5000 and
window + sinks layer at n = 3 .. 1500, B = 2, the last 5 tokens appended one at a time) run through this package's
CUDA backend: the output must be within rel-L2 1e-2 and max-abs 2e-2 of the reference's torch_decode (golden
fixtures) and of the CPU oracle on the same pools; the backend that ran must be the one requested."""
import numpy as np
import pytest
import torch

import inputs as I
from _util import assert_parity, nb, tb
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DG = np.load(I.__file__.replace("inputs.py", "decode.npz"))
DEV = "cuda"


@pytest.fixture(scope="module")
def kv800():
    from lfm3_kv800 import kv800 as m
    return m


@pytest.fixture(scope="module")
def tables():
    cs, sn = I.rope_tables(8192)
    return cs, sn, tb(cs, DEV), tb(sn, DEV)


def run_case(kv800, tables, win, n, backend="cuda", spb=None):
    cs, sn, c32, s32 = tables
    K, V, q = I.parity_inputs(win, n)
    st = kv800.PagedStore(2, n + 8, DEV, window=win)
    pre = max(1, n - 5)
    st.append(tb(K[:, :pre], DEV), tb(V[:, :pre], DEV))
    for i in range(pre, n):
        st.append(tb(K[:, i:i + 1], DEV), tb(V[:, i:i + 1], DEV))
    kv800.set_backend(backend)
    try:
        o = kv800.decode(st.paged(), tb(q, DEV), c32, s32, st.H, spb=spb)
        ran = kv800.get_backend()
    finally:
        kv800.set_backend(None)
    return nb(o), ran, st, q


@pytest.mark.parametrize("win,n", I.parity_cases())
def test_parity_vs_reference(kv800, tables, win, n):
    o, ran, st, q = run_case(kv800, tables, win, n)
    assert ran == "cuda"
    assert_parity(o, DG[f"w{win}_n{n}_out"], f"win={win} n={n} vs reference torch_decode")


@pytest.mark.parametrize("win,n", [(0, 1500), (0, 5000), (256, 1500)])
def test_parity_vs_oracle_same_pools(kv800, tables, win, n):
    """The oracle decodes the CUDA-built pools (copied to the host): isolates the decode from the flush."""
    o, _, st, q = run_case(kv800, tables, win, n)
    P = st.paged()
    Pn = dict(qpool=P.qpool.cpu().numpy(), boff=P.boff.cpu().numpy(), epool=nb(P.epool), eoff=P.eoff.cpu().numpy(),
              ebs=P.ebs, e_hs=P.e_hs, e_ts=P.e_ts, e_v=P.e_v, sk=None if P.sk is None else nb(P.sk),
              sv=None if P.sv is None else nb(P.sv), skoff=P.skoff.cpu().numpy(), svoff=P.svoff.cpu().numpy(),
              N=P.N.cpu().numpy(), NQ=P.NQ.cpu().numpy(), nqmax=P.nqmax, win=P.win)
    ref = O.decode(Pn, q, tables[0], tables[1])
    assert_parity(o, ref, f"win={win} n={n} vs oracle")


@pytest.mark.parametrize("spb", [1, 2, 3, 100])
def test_split_sizes_agree(kv800, tables, spb):
    """Every split size gives the reference's answer (split-K + combine is exact up to fp32 rounding)."""
    o, _, _, _ = run_case(kv800, tables, 0, 5000, spb=spb)
    assert_parity(o, DG["w0_n5000_out"], f"spb={spb}")


@pytest.mark.parametrize("win,n", [(0, 1500), (256, 700)])
def test_decode_timed_matches_decode(kv800, tables, win, n):
    """kv800.decode_timed (the phase-timed entry the bench uses for its roofline) returns decode()'s exact output and
    phase times (the exact phase, which also merges the partials, always runs; the quantized phase only for quantized
    layers; the merge has no launch of its own, so its phase is the gap between two events)."""
    K, V, q = I.parity_inputs(win, n)
    st = kv800.PagedStore(2, n + 8, DEV, window=win)
    st.append(tb(K, DEV), tb(V, DEV))
    _, _, c32, s32 = tables
    ref = nb(kv800.decode(st.paged(), tb(q, DEV), c32, s32, st.H))
    out, ms = kv800.decode_timed(st.paged(), tb(q, DEV), c32, s32)
    assert np.array_equal(nb(out), ref)
    assert ms["exact_ms"] > 0 and ms["combine_ms"] >= 0 and ms["quantized_ms"] >= 0
    if win == 0:
        assert ms["quantized_ms"] > 0
