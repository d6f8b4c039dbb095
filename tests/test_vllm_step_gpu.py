"""The vLLM step on the device (lfm3_kv800/vllm_step.py, the data path of the reference's vllm_attn.py:244-402) driven
through a simulated vLLM schedule: chunked prefill, an extend with quantized history, and decode steps that cross the
flush boundary, for two quantized layers (which are also the sink hosts), a window layer with sinks and a native
sliding layer.  Every cache has its own shuffled block table, as vLLM's allocator hands out pages.

Checked against the oracle after every step:
  * quant caches: every flushed sub-block bit-identical to the oracle quantizer on the same tokens
  * exact caches and sink rows: the written bf16 rows
  * decode rows: the oracle decode over copies of the very caches the GPU holds, within the decode tolerance
  * prefill / extend rows: a dense fp32 attention over the oracle's dequantized history (the reference's fp32 prefill,
    vllm_attn.py:170-187) within 2e-2 relative, the bar the reference applies to its bf16 SDPA prefill
    (vllm_attn.py:393-396)
  * kv800_prefill_kv directly: the assembled K / V bit-identical to the oracle's dequantize + bf16 RoPE."""
import numpy as np
import pytest
import torch

import inputs as I
from _util import assert_parity_ulp, f32, nb, tb
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
EBS = 128                   # vLLM's 64-token page doubled by the page-size unification with the quant pages
MAXPOS = 2048
LAYERS = {6: "quant", 10: "quant", 2: "window", 0: "slide"}


def f32_bf16(x):
    return I.f32_to_bf16(np.asarray(x, np.float32))


def rope_np(K, pos, cs, sn):
    """HF RoPE of bf16 K (S, 4, 128) at positions pos with [P, 32] tables, in the reference's fp32 operation order."""
    kf = f32(K)
    c, s = f32(cs[pos]), f32(sn[pos])
    one, zero = np.ones_like(c), np.zeros_like(s)
    c128 = np.concatenate((c, one, c, one), 1)[:, None]
    s128 = np.concatenate((s, zero, s, zero), 1)[:, None]
    rot = np.concatenate((-kf[..., 64:], kf[..., :64]), -1)
    return f32_bf16((kf * c128).astype(np.float32) + (rot * s128).astype(np.float32))


class Sim:
    def __init__(self, lengths, seed=0):
        from lfm3_kv800 import vllm_step as S
        self.S = S
        rs = np.random.RandomState(seed)
        self.rs = rs
        R = len(lengths)
        self.R, self.L = R, lengths
        # per (layer, request) token data (pre-RoPE K, V) and a running length
        self.K = {l: [I.f32_to_bf16((rs.standard_normal((n, 4, 128)) + 1.5 * rs.standard_normal((1, 4, 128)))
                                    .astype(np.float32)) for n in lengths] for l in LAYERS}
        self.V = {l: [I.f32_to_bf16(rs.standard_normal((n, 4, 128)).astype(np.float32)) for n in lengths]
                  for l in LAYERS}
        self.n = [0] * R
        # every cache gets its own shuffled, disjoint pages per request (a few spare pages stay unused)
        pages = -(-max(lengths) // EBS)
        qpages = -(-max(lengths) // S.QBLOCK)
        NBLK, NQPG = R * pages + 3, R * qpages + 2
        self.bt = {l: rs.permutation(NBLK)[:R * pages].reshape(R, pages).astype(np.int32) for l in LAYERS}
        self.qbt = {l: rs.permutation(NQPG)[:R * qpages].reshape(R, qpages).astype(np.int32)
                    for l, k in LAYERS.items() if k == "quant"}
        self.ev = {l: torch.zeros(NBLK, 4, EBS, 256, dtype=torch.bfloat16, device=DEV) for l in LAYERS}
        self.qraw = {l: torch.zeros(NQPG * S.QPAGE, dtype=torch.uint8, device=DEV) for l in self.qbt}
        # the vLLM-shaped view: (pages, 2, 1280, 4, 25) uint8 with the page stride padded to 262,144 B
        self.qv = {l: torch.as_strided(self.qraw[l], (NQPG, 2, S.QBLOCK, 4, S.QCONTENT),
                                       (S.QPAGE, S.QBLOCK * 4 * S.QCONTENT, 4 * S.QCONTENT, S.QCONTENT, 1))
                   for l in self.qbt}
        self.attn = {l: S.KV800Attention(l, MAXPOS, slide=(k == "slide")) for l, k in LAYERS.items()}
        cs, sn, one, zero = S.tables(torch.device(DEV), MAXPOS)
        self.cs, self.sn = nb(cs), nb(sn)
        self.one, self.zero = nb(one), nb(zero)

    # ------------------------------------------------------------ one step
    def step(self, sched):
        """sched: [(request, new tokens)] in vLLM's order (decodes first).  Returns {layer: (out bits, q bits)}."""
        S = self.S
        order = [r for r, _ in sched]
        qlen = [t for _, t in sched]
        qsl = np.concatenate(([0], np.cumsum(qlen))).astype(np.int32)
        sl = np.array([self.n[r] + t for r, t in sched], np.int32)
        T = int(qsl[-1])
        pos = np.concatenate([np.arange(self.n[r], self.n[r] + t) for r, t in sched]).astype(np.int64)
        nd = 0
        while nd < len(sched) and qlen[nd] == 1:
            nd += 1
        res = {}
        for l, kind in LAYERS.items():
            bt = self.bt[l][order]
            slot = np.concatenate([self.bt[l][r][np.arange(self.n[r], self.n[r] + t) // EBS] * EBS +
                                   np.arange(self.n[r], self.n[r] + t) % EBS for r, t in sched]).astype(np.int64)
            res[l] = dict(bt=bt, slot=slot)
        metas = {}
        for l in LAYERS:
            bt_t = torch.from_numpy(res[l]["bt"]).to(DEV)
            metas[l] = S.build_meta(bt_t, torch.from_numpy(res[l]["slot"]).to(DEV), torch.from_numpy(sl).to(DEV),
                                    torch.from_numpy(qsl).to(DEV), torch.from_numpy(sl), torch.from_numpy(qsl),
                                    num_decodes=nd)
        qmetas = {l: S.build_meta(torch.from_numpy(self.qbt[l][order]).to(DEV), metas[l].slot_mapping,
                                  metas[l].seq_lens, metas[l].query_start_loc, metas[l].seq_lens_cpu,
                                  metas[l].query_start_loc_cpu, metas[l].positions, nd) for l in self.qbt}
        assert np.array_equal(metas[0].positions.cpu().numpy(), pos)
        out = {}
        for l, kind in LAYERS.items():
            k = np.concatenate([self.K[l][r][self.n[r]:self.n[r] + t] for r, t in sched])
            v = np.concatenate([self.V[l][r][self.n[r]:self.n[r] + t] for r, t in sched])
            q = I.f32_to_bf16(self.rs.standard_normal((T, 16, 128)).astype(np.float32))
            kw = {}
            if kind == "quant":
                kw = dict(mq=qmetas[l], qv=self.qv[l])
            elif kind == "window":
                kw = dict(hosts=((qmetas[6], self.qv[6]), (qmetas[10], self.qv[10])))
            o = self.attn[l].forward(tb(q, DEV), tb(k, DEV), tb(v, DEV), metas[l], self.ev[l], **kw)
            out[l] = (nb(o), q)
        torch.cuda.synchronize()
        prev = list(self.n)
        for r, t in sched:
            self.n[r] += t
        self.check(sched, prev, nd, out)
        return out

    # ------------------------------------------------------------ checks
    def boff(self, l, r, nq):
        bsq = self.S.QBLOCK
        return np.array([self.qbt[l][r][(256 * j) // bsq] * self.S.QPAGE + ((256 * j % bsq) // 256) * 51200
                         for j in range(nq)], np.int64)

    def check(self, sched, prev, nd, out):
        S = self.S
        qbytes = {l: self.qraw[l].cpu().numpy() for l in self.qraw}
        ev = {l: nb(self.ev[l]).reshape(-1) for l in LAYERS}
        s0, s1, s2 = 4 * EBS * 256, EBS * 256, 256
        aux = (S.QBLOCK // 256) * 25600
        for r in range(self.R):
            n = self.n[r]
            for l in LAYERS:
                # exact rows of every position
                p = np.arange(n)
                base = self.bt[l][r][p // EBS].astype(np.int64) * s0 + (p % EBS) * s2
                idx = base[:, None, None] + np.arange(4)[None, :, None] * s1 + np.arange(128)
                assert np.array_equal(ev[l][idx], self.K[l][r][:n]), f"exact K layer {l} req {r}"
                assert np.array_equal(ev[l][idx + 128], self.V[l][r][:n]), f"exact V layer {l} req {r}"
            for l in self.qbt:
                nq = S.nq_of(n)
                if nq:
                    got = qbytes[l][self.boff(l, r, nq)[:, None] + np.arange(51200)]
                    ref = O.quantize_blocks(self.K[l][r][:256 * nq].reshape(nq, 256, 4, 128),
                                            self.V[l][r][:256 * nq].reshape(nq, 256, 4, 128))
                    assert np.array_equal(got, ref), f"quant cache layer {l} req {r}: sub-blocks differ"
            # sinks of the window layer in the hosts' aux areas
            ns = min(4, n)
            for host, src in ((6, self.K[2][r]), (10, self.V[2][r])):
                hb = qbytes[host].view(np.uint16)
                a = int(self.qbt[host][r][0]) * (S.QPAGE // 2) + aux
                assert np.array_equal(hb[a:a + ns * 512].reshape(ns, 4, 128), src[:ns]), f"sinks host {host} req {r}"
        # decode rows: the oracle over copies of the same caches
        order = [r for r, _ in sched]
        if nd:
            rows = order[:nd]
            for l, kind in LAYERS.items():
                o, q = out[l]
                N = np.array([self.n[r] for r in rows], np.int32)
                eoff = self.bt[l][rows].astype(np.int64) * s0
                P = dict(epool=ev[l], eoff=eoff, ebs=EBS, e_hs=s1, e_ts=s2, e_v=128, N=N, sk=None, sv=None)
                cs, sn = (self.one, self.zero) if kind == "slide" else (self.cs, self.sn)
                if kind == "quant":
                    NQ = np.array([S.nq_of(n) for n in N], np.int32)
                    nqmax = int(NQ.max())
                    boff = np.zeros((nd, max(1, nqmax)), np.int64)
                    for i, r in enumerate(rows):
                        boff[i, :NQ[i]] = self.boff(l, r, NQ[i])
                    P.update(qpool=qbytes[l], boff=boff, NQ=NQ, nqmax=nqmax, win=0)
                else:
                    P.update(qpool=np.zeros(1, np.uint8), boff=np.zeros((nd, 1), np.int64),
                             NQ=np.zeros(nd, np.int32), nqmax=0, win=256)
                    if kind == "window":
                        P.update(sk=qbytes[6].view(np.uint16), sv=qbytes[10].view(np.uint16),
                                 skoff=self.qbt[6][rows, 0].astype(np.int64) * (S.QPAGE // 2) + aux,
                                 svoff=self.qbt[10][rows, 0].astype(np.int64) * (S.QPAGE // 2) + aux)
                ref = O.decode(P, q[:nd], cs, sn)
                assert_parity_ulp(o[:nd], ref, f"decode layer {l} rows {rows}")
        # prefill / extend rows: dense fp32 attention over the oracle's history
        qsl = np.concatenate(([0], np.cumsum([t for _, t in sched])))
        for i in range(nd, len(sched)):
            r = order[i]
            n0, n = prev[r], self.n[r]
            for l, kind in LAYERS.items():
                o, q = out[l]
                K, V, kp = self.history(l, kind, r, n0, n)
                ref = dense(f32(q[qsl[i]:qsl[i + 1]]), f32(K), f32(V), kp, n0, n, kind)
                got = f32(o[qsl[i]:qsl[i + 1]])
                rel = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
                assert rel < 2e-2, f"prefill layer {l} req {r} [{n0}, {n}): rel {rel:.3e}"

    def history(self, l, kind, r, n0, n):
        """the reference's K (rotated, bf16) / V (bf16) / positions for request r's chunk [n0, n) on layer l."""
        Kr, Vr = self.K[l][r], self.V[l][r]
        parts_k, parts_v, parts_p = [], [], []
        if kind == "quant":
            nqp = self.S.nq_of(n0)
            lo = 256 * nqp
            if nqp:
                kq, vq = O.dequantize_blocks(O.quantize_blocks(Kr[:lo].reshape(nqp, 256, 4, 128),
                                                               Vr[:lo].reshape(nqp, 256, 4, 128)))
                parts_k.append(kq.reshape(-1, 4, 128))
                parts_v.append(f32_bf16(vq.reshape(-1, 4, 128)))
                parts_p.append(np.arange(lo))
        else:
            lo = max(0, n0 - 255)
            ns = 0 if kind == "slide" else min(4, lo)
            if ns:
                parts_k.append(Kr[:ns])
                parts_v.append(Vr[:ns])
                parts_p.append(np.arange(ns))
        parts_k.append(Kr[lo:n])
        parts_v.append(Vr[lo:n])
        parts_p.append(np.arange(lo, n))
        K, V, kp = np.concatenate(parts_k), np.concatenate(parts_v), np.concatenate(parts_p)
        if kind != "slide":
            K = rope_np(K, kp, self.cs, self.sn)
        return K, V, kp


def dense(q, K, V, kp, n0, n, kind):
    """fp32 attention of queries at positions n0 .. n - 1 (vllm_attn.py:170-187)."""
    Kf = np.repeat(K, 4, axis=1).transpose(1, 0, 2)
    Vf = np.repeat(V, 4, axis=1).transpose(1, 0, 2)
    qi = q.transpose(1, 0, 2)
    qp = np.arange(n0, n)[:, None]
    m = kp[None] <= qp
    if kind == "slide":
        m &= kp[None] > qp - 256
    elif kind == "window":
        m &= (kp[None] > qp - 256) | (kp[None] < 4)
    sc = np.einsum("hqd,hkd->hqk", qi, Kf) * np.float32(128 ** -0.5)
    sc = np.where(m[None], sc, -np.inf)
    sc -= sc.max(-1, keepdims=True)
    p = np.exp(sc)
    p /= p.sum(-1, keepdims=True)
    return np.einsum("hqk,hkd->hqd", p, Vf).transpose(1, 0, 2)


def test_vllm_schedule():
    sim = Sim([1160, 1320, 12], seed=5)
    sim.step([(0, 1150), (1, 600), (2, 3)])             # prefills; request 0 flushes 3 sub-blocks in its prefill
    sim.step([(0, 1), (2, 1), (1, 700)])                # decodes (request 2 writes sink position 3) + an extend with
    #                                                     a quantized sub-block of history; request 1 flushes 3
    sim.step([(0, 1), (2, 1), (1, 1)])                  # request 0 reaches 1152 = 256 * 3 + 384: one flush
    for _ in range(4):
        sim.step([(1, 1), (0, 1), (2, 1)])
    assert sim.n == [1156, 1305, 9]


def test_flush_boundary_many_requests():
    """Many decode rows crossing the flush boundary in the same step (one flushed sub-block each), others not."""
    lengths = [640 + 1 + (i % 3) for i in range(12)]
    sim = Sim([n + 4 for n in lengths], seed=11)
    sim.step([(r, n) for r, n in enumerate(lengths)])
    for _ in range(3):
        sim.step([(r, 1) for r in range(len(lengths))])


def test_prefill_kv_bits():
    """kv800_prefill_kv alone: quantized history + exact tail + chunk, and window sinks + exact window, bit-identical to
    the oracle's dequantize + bf16 RoPE."""
    sim = Sim([1400, 700], seed=3)
    sim.step([(0, 1300), (1, 690)])
    S = sim.S
    cs, sn, _, _ = S.tables(torch.device(DEV), MAXPOS)
    for l, kind in LAYERS.items():
        if kind == "slide":
            continue
        for r, (n0, n) in enumerate(((1300, 1340), (690, 700))):
            chunk_k, chunk_v = sim.K[l][r][n0:n], sim.V[l][r][n0:n]
            bt = torch.from_numpy(sim.bt[l][r]).to(DEV)
            if kind == "quant":
                K, V, kp = S.prefill_kv(n0, n, tb(chunk_k, DEV), tb(chunk_v, DEV), sim.ev[l], bt, qv=sim.qv[l],
                                        qbt_row=torch.from_numpy(sim.qbt[l][r]).to(DEV), nqp=S.nq_of(n0), cos_t=cs,
                                        sin_t=sn)
            else:
                lo = max(0, n0 - 255)
                ns = min(4, lo)
                sk = tb(sim.K[l][r][:ns], DEV)
                sv = tb(sim.V[l][r][:ns], DEV)
                K, V, kp = S.prefill_kv(n0, n, tb(chunk_k, DEV), tb(chunk_v, DEV), sim.ev[l], bt, sk=sk, sv=sv,
                                        ns=ns, lo=lo, cos_t=cs, sin_t=sn)
            torch.cuda.synchronize()
            # the reference's parts: the exact chunk rows are the same tokens as the cache rows
            Kr, Vr, kpr = sim.history(l, kind, r, n0, n)
            assert np.array_equal(kp.cpu().numpy(), kpr)
            assert np.array_equal(nb(K), Kr), f"prefill K layer {l} req {r}"
            assert np.array_equal(nb(V), Vr), f"prefill V layer {l} req {r}"
