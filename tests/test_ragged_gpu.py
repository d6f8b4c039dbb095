"""Ragged batches through the decode (BASELINE config 4 in small): rows of different lengths, including an empty row
and rows without quantized sub-blocks, with sub-blocks and exact pages at shuffled pool slots.  The pools are built
on the host with the oracle's quantizer and decoded by both the CUDA path (persistent schedule and explicit split
sizes) and the oracle; the outputs must agree within the decode tolerance."""
import numpy as np
import pytest
import torch

import inputs as I
from _util import assert_parity_ulp, nb, tb
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
EBS = 64


def build(lengths, win, seed, distinct=None, ebs=EBS, pitch=256):
    """Host pools for rows of `lengths`; `distinct` = quantize only that many different sub-blocks and scatter them
    at random over the rows' tables (the quantized part need not match the exact pages).  Exact pages hold `ebs`
    slots per head with rows of `pitch` elements (K at 0, V at 128; 256 is the reference's layout)."""
    EBS = ebs
    rs = np.random.RandomState(seed)
    B = len(lengths)
    nqs = [0 if win else max(0, n - 128) // 256 for n in lengths]
    nslot = sum(nqs) + 5
    slots = rs.permutation(nslot)
    qpool = np.zeros((nslot, 51200), np.uint8)
    maxpg = max(lengths) // EBS + 2
    boff = np.zeros((B, max(1, max(nqs))), np.int64)
    eoff = np.zeros((B, maxpg), np.int64)
    npages = sum(n // EBS + 1 for n in lengths) + 3
    pages = rs.permutation(npages)
    epool = np.zeros((npages, 4, EBS, pitch), np.uint16)
    # token data: every position when the sub-blocks are built from it, else only what the decode reads (the exact
    # positions [256 nq, n) and the 4 sink positions); other positions stay zero
    K_all, V_all = [], []
    for b, n in enumerate(lengths):
        lo = 0 if not distinct else 256 * nqs[b]
        K = np.zeros((n, 4, 128), np.uint16)
        V = np.zeros((n, 4, 128), np.uint16)
        for a_, z_ in ((0, min(4, n)), (lo, n)):
            if z_ > a_:
                K[a_:z_] = I.f32_to_bf16(rs.standard_normal((z_ - a_, 4, 128)).astype(np.float32) +
                                        2 * rs.standard_normal((1, 4, 128)).astype(np.float32))
                V[a_:z_] = I.f32_to_bf16(rs.standard_normal((z_ - a_, 4, 128)).astype(np.float32))
        K_all.append(K)
        V_all.append(V)
    # all full sub-blocks in one oracle call, placed at the shuffled slots
    if distinct:
        k, v = I.quant_inputs("parity", distinct, seed=seed)
        pool = O.quantize_blocks(k, v)
        sbs = pool[rs.randint(0, distinct, sum(nqs))]
    else:
        ks = [K_all[b][256 * j:256 * j + 256] for b in range(B) for j in range(nqs[b])]
        vs = [V_all[b][256 * j:256 * j + 256] for b in range(B) for j in range(nqs[b])]
        sbs = O.quantize_blocks(np.stack(ks), np.stack(vs)) if ks else None
    if sum(nqs):
        si = 0
        for b in range(B):
            for j in range(nqs[b]):
                qpool[slots[si]] = sbs[si]
                boff[b, j] = slots[si] * 51200
                si += 1
    pi = 0
    for b, n in enumerate(lengths):
        npg = n // EBS + 1
        eoff[b, :npg] = pages[pi:pi + npg] * 4 * EBS * pitch
        pi += npg
        if n:
            t = np.arange(n)
            pg = eoff[b, t // EBS] // (4 * EBS * pitch)
            epool[pg, :, t % EBS, :128] = K_all[b]
            epool[pg, :, t % EBS, 128:256] = V_all[b]
    sk = np.zeros((B, 4, 4, 128), np.uint16)
    for b, n in enumerate(lengths):
        m = min(4, n)
        sk[b, :m] = K_all[b][:m]
    sv = np.zeros_like(sk)
    for b, n in enumerate(lengths):
        m = min(4, n)
        sv[b, :m] = V_all[b][:m]
    q = I.f32_to_bf16(2 * rs.standard_normal((B, 16, 128)).astype(np.float32))
    P = dict(qpool=qpool, boff=boff, epool=epool, eoff=eoff, ebs=EBS, e_hs=EBS * pitch, e_ts=pitch, e_v=128,
             sk=sk if win else None, sv=sv if win else None, skoff=np.arange(B, dtype=np.int64) * 2048,
             svoff=np.arange(B, dtype=np.int64) * 2048, N=np.array(lengths, np.int32), NQ=np.array(nqs, np.int32),
             nqmax=max(nqs), win=win)
    return P, q


def to_dev(kv800, P):
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(DEV)
    return kv800.Paged(qpool=t(P["qpool"]), boff=t(P["boff"]), epool=tb(P["epool"], DEV), eoff=t(P["eoff"]),
                       ebs=P["ebs"], e_hs=P["e_hs"], e_ts=P["e_ts"], e_v=P["e_v"],
                       sk=None if P["sk"] is None else tb(P["sk"], DEV),
                       sv=None if P["sv"] is None else tb(P["sv"], DEV), skoff=t(P["skoff"]), svoff=t(P["svoff"]),
                       N=t(P["N"]), NQ=t(P["NQ"]), nqmax=P["nqmax"], win=P["win"])


LENGTHS = [0, 3, 383, 384, 900, 2000, 5000, 1, 640]


@pytest.mark.parametrize("win", [0, 256])
@pytest.mark.parametrize("spb", [None, 1, 4])
def test_ragged_vs_oracle(win, spb):
    from lfm3_kv800 import kv800
    P, q = build(LENGTHS, win, seed=17 + win)
    cs, sn = I.rope_tables(5200)
    out = kv800.decode(to_dev(kv800, P), tb(q, DEV), tb(cs, DEV), tb(sn, DEV), spb=spb)
    ref = O.decode(P, q, cs, sn)
    got = nb(out)
    assert_parity_ulp(got, ref, f"ragged win={win} spb={spb}")
    assert np.all(got[0] == 0), "the empty row must decode to zeros"


@pytest.mark.parametrize("ebs,pitch", [(16, 256), (128, 256), (24, 256), (64, 384)])
@pytest.mark.parametrize("win", [0, 256])
def test_exact_page_layouts(ebs, pitch, win, monkeypatch):
    """Both forms of the exact partials against the oracle: pages of a multiple of 16 slots with 512-byte K | V rows
    (the reference's layout) take the tensor-map form, other page sizes and padded rows the gather form.  Windows
    start at positions that are not multiples of 16, so first and last tiles are partly masked.  The status word
    must stay 0 (no spurious range flags)."""
    from lfm3_kv800 import kv800
    monkeypatch.setattr(kv800, "_CHECK", True)
    P, q = build(LENGTHS, win, seed=31 + ebs + pitch + win, ebs=ebs, pitch=pitch)
    cs, sn = I.rope_tables(5200)
    for spb in (None, 3):
        got = nb(kv800.decode(to_dev(kv800, P), tb(q, DEV), tb(cs, DEV), tb(sn, DEV), spb=spb))
        assert_parity_ulp(got, O.decode(P, q, cs, sn), f"ebs={ebs} pitch={pitch} win={win} spb={spb}")
        assert np.all(got[0] == 0)


@pytest.mark.parametrize("win", [0, 256])
def test_exact_pages_off_the_row_grid(win, monkeypatch):
    """Page offsets that keep every row 16-byte aligned but are not multiples of 256 elements (the pool starts 8
    elements into its buffer): the reference's strides select the tensor-map form, which loads such tiles with plain
    loads.  Must meet the bar against the oracle with the status word 0, as the gather form did for them."""
    from lfm3_kv800 import kv800
    monkeypatch.setattr(kv800, "_CHECK", True)
    P, q = build(LENGTHS, win, seed=41 + win)
    P["epool"] = np.concatenate([np.zeros(8, np.uint16), P["epool"].ravel()])
    P["eoff"] = P["eoff"] + 8
    cs, sn = I.rope_tables(5200)
    for spb in (None, 3):
        got = nb(kv800.decode(to_dev(kv800, P), tb(q, DEV), tb(cs, DEV), tb(sn, DEV), spb=spb))
        assert_parity_ulp(got, O.decode(P, q, cs, sn), f"off-grid pages win={win} spb={spb}")
        assert np.all(got[0] == 0)


def test_persistent_many_rows():
    """More rows than persistent CTAs with tiny sub-block lists: every CTA range crosses several rows."""
    from lfm3_kv800 import kv800
    lengths = [384 + 256 * (i % 3) for i in range(400)]
    P, q = build(lengths, 0, seed=5, distinct=24)
    cs, sn = I.rope_tables(1200)
    out = kv800.decode(to_dev(kv800, P), tb(q, DEV), tb(cs, DEV), tb(sn, DEV))
    assert_parity_ulp(nb(out), O.decode(P, q, cs, sn), "400 short rows")


@pytest.mark.parametrize("sinks", [True, False])
def test_sliding_layer_without_tables(sinks):
    """Native sliding layers (keys stored post-RoPE) decode without tables: bit-identical to the reference's way of
    running them, all-ones / all-zeros tables (vllm_attn.py:256-257), and within the bar of the oracle with those
    tables.  Quantized layers still refuse null tables."""
    from lfm3_kv800 import kv800
    P, q = build(LENGTHS, 256, seed=23)
    if not sinks:
        P["sk"] = P["sv"] = None
    one = I.f32_to_bf16(np.ones((5200, 32), np.float32))
    zero = I.f32_to_bf16(np.zeros((5200, 32), np.float32))
    Pd = to_dev(kv800, P)
    got = nb(kv800.decode(Pd, tb(q, DEV), None, None))
    ident = nb(kv800.decode(Pd, tb(q, DEV), tb(one, DEV), tb(zero, DEV)))
    assert np.array_equal(got, ident), "no-rotation decode differs from identity tables"
    assert_parity_ulp(got, O.decode(P, q, one, zero), f"sliding layer sinks={sinks}")
    Pq, qq = build([900, 2000], 0, seed=3)
    with pytest.raises(ValueError):
        kv800.decode(to_dev(kv800, Pq), tb(qq, DEV), None, None)
