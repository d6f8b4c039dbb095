"""One process decoding on two GPUs: the kernels' shared-memory attributes are per device, so the library sets them on
each device it is used on.  The same pools and query decoded on cuda:0 and then on cuda:1 must give identical
outputs and meet the bar against the oracle.  Skipped unless two GPUs are visible."""
import numpy as np
import pytest
import torch

import inputs as I
from _util import assert_parity_ulp, nb, tb
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("win", [0, 256])
def test_decode_on_two_devices(win):
    from lfm3_kv800 import kv800
    K, V, q = I.parity_inputs(win, 1500, B=3, seed=12)
    cs, sn = I.rope_tables(4096)
    outs = []
    for d in ("cuda:0", "cuda:1"):
        with torch.cuda.device(d):
            st = kv800.PagedStore(3, 1508, d, window=win)
            st.append(tb(K, d), tb(V, d))
            outs.append(nb(kv800.decode(st.paged(), tb(q, d), tb(cs, d), tb(sn, d), st.H)))
            torch.cuda.synchronize()
            P = st.paged()
            Pn = dict(qpool=P.qpool.cpu().numpy(), boff=P.boff.cpu().numpy(), epool=nb(P.epool),
                      eoff=P.eoff.cpu().numpy(), ebs=P.ebs, e_hs=P.e_hs, e_ts=P.e_ts, e_v=P.e_v,
                      sk=None if P.sk is None else nb(P.sk), sv=None if P.sv is None else nb(P.sv),
                      skoff=P.skoff.cpu().numpy(), svoff=P.svoff.cpu().numpy(), N=P.N.cpu().numpy(),
                      NQ=P.NQ.cpu().numpy(), nqmax=P.nqmax, win=P.win)
            assert_parity_ulp(outs[-1], O.decode(Pn, q, cs, sn), f"{d} win={win}")
    assert np.array_equal(outs[0], outs[1]), "the two devices decoded the same pools differently"
