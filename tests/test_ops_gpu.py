"""The reference's three-op decode path on this package's kernels: torch.ops.kv800.qdecode -> xdecode -> combine,
called with the arguments and split sizing of the reference's kv800_sycl.decode (kv800_sycl.py:94-112: ns splits of
spb sub-blocks, slot ns = sinks + exact tokens, partials MO / LO / AO allocated by the caller), which reach the C ABI
entry points kv800_qdecode / kv800_xdecode / kv800_combine.  The merged output must meet the decode bar against
the reference's torch_decode goldens on the 12 parity cases and against the oracle on a 4 x 32K layer; the Python
kv800.combine (the reference's combine(MO, LO, AO, ns, H), kv800.py:231-236) must give the op's bytes on the same
partials."""
import math

import numpy as np
import pytest
import torch

import inputs as I
from _util import assert_parity, assert_parity_ulp, nb, tb
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
DG = np.load(I.__file__.replace("inputs.py", "decode.npz"))
SCALE = 128 ** -0.5 * 1.4426950408889634


@pytest.fixture(scope="module")
def mods():
    from lfm3_kv800 import kv800, ops
    return kv800, ops.ops()


def three_op_decode(kv800, o, P, q, c32, s32, spb=None, target=2048):
    """kv800_sycl.decode (kv800_sycl.py:94-112), step by step, on torch.ops.kv800 -> (out, MO, LO, AO, ns)."""
    B = q.shape[0]
    nqmax = 0 if P.win else P.nqmax
    if spb is None:
        spb = max(1, math.ceil(nqmax * B * 4 / target)) if nqmax else 1
    ns = math.ceil(nqmax / spb) if nqmax else 0
    MO = torch.empty(B, ns + 1, 16, device=q.device, dtype=torch.float32)
    LO = torch.empty_like(MO)
    AO = torch.empty(B, ns + 1, 16, 128, device=q.device, dtype=torch.float32)
    if ns:
        o.qdecode(q, P.qpool, P.boff, P.NQ, c32, s32, MO, LO, AO, ns, spb, SCALE, 1)
    sk = P.sk if P.sk is not None else P.epool
    sv = P.sv if P.sv is not None else P.epool
    dummy = P.N.to(torch.int64) if P.skoff is None else None
    skoff = P.skoff if P.skoff is not None else dummy
    svoff = P.svoff if P.svoff is not None else dummy
    nsink = kv800.NSINK if (P.win and P.sk is not None) else 0
    o.xdecode(q, P.epool, P.eoff, P.ebs, P.e_hs, P.e_ts, P.e_v, sk, sv, skoff, svoff, P.N, P.NQ, c32, s32, MO, LO,
              AO, ns, SCALE, P.win, nsink)
    return o.combine(MO, LO, AO, ns), MO, LO, AO, ns


@pytest.mark.parametrize("win,n", I.parity_cases())
@pytest.mark.parametrize("spb", [None, 2])
def test_three_ops_vs_reference(mods, win, n, spb):
    kv800, o = mods
    K, V, q = I.parity_inputs(win, n)
    cs, sn = I.rope_tables(8192)
    st = kv800.PagedStore(2, n + 8, DEV, window=win)
    pre = max(1, n - 5)
    st.append(tb(K[:, :pre], DEV), tb(V[:, :pre], DEV))
    for i in range(pre, n):
        st.append(tb(K[:, i:i + 1], DEV), tb(V[:, i:i + 1], DEV))
    out, MO, LO, AO, ns = three_op_decode(kv800, o, st.paged(), tb(q, DEV), tb(cs, DEV), tb(sn, DEV), spb=spb)
    assert_parity(nb(out), DG[f"w{win}_n{n}_out"], f"three ops, win={win} n={n} spb={spb}")
    # the Python combine on the same partials: the same kernel, the same bytes
    assert np.array_equal(nb(kv800.combine(MO, LO, AO, ns, st.H)), nb(out))
    # and the single-call decode agrees with the three-op path within the bar
    assert_parity(nb(kv800.decode(st.paged(), tb(q, DEV), tb(cs, DEV), tb(sn, DEV), st.H)), nb(out), "decode vs ops")


def test_three_ops_long_context_vs_oracle(mods):
    """4 rows x 32,768 tokens (127 sub-blocks + 256 exact tokens each), spb 8 (16 quantized splits per row)."""
    kv800, o = mods
    B, N = 4, 32768
    g = torch.Generator(device=DEV).manual_seed(77)
    K = (torch.randn(B, N, 4, 128, device=DEV, generator=g) +
         3 * torch.randn(1, 1, 4, 128, device=DEV, generator=g)).to(torch.bfloat16)
    V = torch.randn(B, N, 4, 128, device=DEV, generator=g).to(torch.bfloat16)
    st = kv800.PagedStore(B, N + 8, DEV)
    st.append(K, V)
    del K, V
    P = st.paged()
    rs = np.random.RandomState(5)
    q = I.f32_to_bf16((2.0 * rs.standard_normal((B, 16, 128))).astype(np.float32))
    cs, sn = I.rope_tables(N + 64)
    out, *_ = three_op_decode(kv800, o, P, tb(q, DEV), tb(cs, DEV), tb(sn, DEV), spb=8)
    Pn = dict(qpool=P.qpool.cpu().numpy(), boff=P.boff.cpu().numpy(), epool=nb(P.epool), eoff=P.eoff.cpu().numpy(),
              ebs=P.ebs, e_hs=P.e_hs, e_ts=P.e_ts, e_v=P.e_v, sk=None, sv=None, skoff=P.skoff.cpu().numpy(),
              svoff=P.svoff.cpu().numpy(), N=P.N.cpu().numpy(), NQ=P.NQ.cpu().numpy(), nqmax=P.nqmax, win=0)
    assert_parity_ulp(nb(out), O.decode(Pn, q, cs, sn), "three ops, 4 x 32K")


def test_ops_reject_bad_arguments(mods):
    kv800, o = mods
    B = 2
    q = torch.zeros(B, 16, 128, dtype=torch.bfloat16, device=DEV)
    MO = torch.zeros(B, 2, 16, device=DEV)
    with pytest.raises(ValueError):
        o.combine(MO, MO, torch.zeros(B, 2, 16, 64, device=DEV), 1)          # AO of the wrong shape
    with pytest.raises(ValueError):
        o.combine(MO.double(), MO, torch.zeros(B, 2, 16, 128, device=DEV), 1)
    with pytest.raises(ValueError):
        o.qdecode(q.float(), torch.zeros(51200, dtype=torch.uint8, device=DEV), torch.zeros(B, 1, dtype=torch.int64,
                  device=DEV), torch.ones(B, dtype=torch.int32, device=DEV), q[0, :, :32], q[0, :, :32], MO, MO,
                  torch.zeros(B, 2, 16, 128, device=DEV), 1, 1, SCALE, 1)
