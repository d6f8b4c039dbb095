"""Drop-in: the reference's own modules running on this package's CUDA kv800.

The staged copy of the reference package (oracle/stage_reference.py -> oracle/_ref) sits on sys.path after this
package; lfm3_kv800/__init__.py's pkgutil.extend_path serves the modules this package does not ship from there, and
their `from . import kv800` binds this package's kv800.  Checked on the GPU:
  * the reference's unmodified tests/test_parity.py, run as `python test_parity.py --device cuda cuda`: its 12 cases
    against its own dense reference, through this package's decode (the backend it reports must be "cuda");
  * the reference's torch_decode.decode (which calls kv800.dequantize_blocks, here the CUDA kernel) against
    kv800.decode on the same pools;
  * the reference's vLLM layer vllm_attn.KV800Attention.forward (exact write, sink write, flush plan +
    kv800.quantize_blocks, decode tables + kv800.decode, dequantized prefill history) driven through a simulated
    schedule with a stand-in for vLLM's config and forward context, side by side with this package's device-side
    vllm_step.KV800Attention on copies of the same caches: caches bit-identical after every step, outputs within the
    decode bar of each other."""
import os
import subprocess
import sys
import types

import numpy as np
import pytest
import torch

import inputs as I
from _util import assert_parity, nb, tb

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")
PKG = os.path.join(ROOT, "lfm3-kv800_b200")
staged = pytest.mark.skipif(not os.path.exists(os.path.join(REF, "lfm3_kv800", "vllm_attn.py")),
                            reason="the reference package is not staged under oracle/_ref (oracle/stage_reference.py)")


@staged
def test_reference_test_parity_unmodified():
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([PKG, REF]))
    r = subprocess.run([sys.executable, os.path.join(REF, "tests", "test_parity.py"), "--device", "cuda", "cuda"],
                       capture_output=True, text=True, env=env, timeout=900)
    print(r.stdout[-3000:])
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "PARITY cuda on cuda: OK" in r.stdout
    assert r.stdout.count("ran cuda") == 12


@staged
@pytest.mark.parametrize("win,n", [(0, 1500), (256, 700)])
def test_reference_torch_decode_on_cuda(win, n):
    from lfm3_kv800 import kv800
    import lfm3_kv800.torch_decode as td
    assert td.kv800 is kv800, "the reference's torch_decode must bind this package's kv800"
    K, V, q = I.parity_inputs(win, n, seed=3)
    cs, sn = I.rope_tables(4096)
    st = kv800.PagedStore(2, n + 8, DEV, window=win)
    st.append(tb(K, DEV), tb(V, DEV))
    ref = td.decode(st.paged(), tb(q, DEV), tb(cs, DEV), tb(sn, DEV), st.H)
    got = kv800.decode(st.paged(), tb(q, DEV), tb(cs, DEV), tb(sn, DEV), st.H)
    assert_parity(nb(got), nb(ref), f"kv800.decode vs reference torch_decode on CUDA, win={win} n={n}")


# ---------------------------------------------------------------- the reference's vLLM layer, side by side
EBS, MAXPOS = 128, 2048
LAYERS = {6: "quant", 10: "quant", 2: "window", 0: "slide"}


class _Ctx:
    """Stand-in for vLLM's config (the layers register their caches in static_forward_context) and forward context
    (attn_metadata: cache name -> the reference's KV800Meta)."""

    def __init__(self):
        self.static = {}
        self.cfg = types.SimpleNamespace(compilation_config=types.SimpleNamespace(static_forward_context=self.static))
        self.fc = types.SimpleNamespace(attn_metadata=None)


@staged
def test_reference_vllm_attn_matches_vllm_step():
    from lfm3_kv800 import kv800
    from lfm3_kv800 import vllm_step as S
    import lfm3_kv800.vllm_attn as va
    assert va.kv800 is kv800, "the reference's vllm_attn must bind this package's kv800"
    ctx = _Ctx()
    saved = (va.get_current_vllm_config, va.get_forward_context)
    va.get_current_vllm_config = lambda: ctx.cfg
    va.get_forward_context = lambda: ctx.fc
    try:
        _run_schedule(kv800, S, va, ctx)
    finally:
        va.get_current_vllm_config, va.get_forward_context = saved


def _run_schedule(kv800, S, va, ctx):
    rs = np.random.RandomState(21)
    lengths = [720, 560, 380]
    R = len(lengths)
    prefix = {l: f"model.layers.{l}.self_attn" for l in LAYERS}
    ref_attn = {l: va.KV800Attention(l, prefix[l], MAXPOS, slide=(k == "slide")) for l, k in LAYERS.items()}
    our_attn = {l: S.KV800Attention(l, MAXPOS, slide=(k == "slide")) for l, k in LAYERS.items()}
    pages, qpages = -(-max(lengths + [1200]) // EBS), -(-1200 // S.QBLOCK)
    NBLK, NQPG = R * pages + 3, R * qpages + 2
    bt = {l: rs.permutation(NBLK)[:R * pages].reshape(R, pages).astype(np.int32) for l in LAYERS}
    qbt = {l: rs.permutation(NQPG)[:R * qpages].reshape(R, qpages).astype(np.int32)
           for l, k in LAYERS.items() if k == "quant"}
    ev = {side: {l: torch.zeros(NBLK, 4, EBS, 256, dtype=torch.bfloat16, device=DEV) for l in LAYERS}
          for side in ("ref", "ours")}
    qraw = {side: {l: torch.zeros(NQPG * S.QPAGE, dtype=torch.uint8, device=DEV) for l in qbt}
            for side in ("ref", "ours")}

    def qview(t):
        # pages of 262,144 B holding (2, 1280 tokens, 4 heads x 25 B): the reference views a host's page as bf16 for
        # the sink rows of its aux area, so the last dimension is the 4 heads' 100 bytes of a token
        return torch.as_strided(t, (NQPG, 2, S.QBLOCK, 4 * S.QCONTENT),
                                (S.QPAGE, S.QBLOCK * 4 * S.QCONTENT, 4 * S.QCONTENT, 1))
    qv = {side: {l: qview(qraw[side][l]) for l in qbt} for side in qraw}
    for l in LAYERS:
        ref_attn[l].xc.kv_cache = ev["ref"][l]
        if l in qbt:
            ref_attn[l].qc.kv_cache = qv["ref"][l]
    n = [0] * R
    # chunked prefill, decodes crossing the flush boundary at 384 (request 2), an extend with quantized history
    schedule = [[(0, 512), (1, 560), (2, 380)], [(2, 1), (0, 208)], [(2, 1), (0, 1), (1, 1)], [(2, 1), (0, 1)],
                [(2, 1), (0, 1), (1, 1)], [(2, 1), (0, 1), (1, 150)]]
    for step, sched in enumerate(schedule):
        order = [r for r, _ in sched]
        qlen = [t for _, t in sched]
        qsl = np.concatenate(([0], np.cumsum(qlen))).astype(np.int32)
        sl = np.array([n[r] + t for r, t in sched], np.int32)
        T = int(qsl[-1])
        pos = np.concatenate([np.arange(n[r], n[r] + t) for r, t in sched]).astype(np.int64)
        nd = 0
        while nd < len(sched) and qlen[nd] == 1:
            nd += 1
        amd, ours = {}, {}
        for l in LAYERS:
            slot = np.concatenate([bt[l][r][np.arange(n[r], n[r] + t) // EBS] * EBS + np.arange(n[r], n[r] + t) % EBS
                                   for r, t in sched]).astype(np.int64)
            btl = torch.from_numpy(bt[l][order]).to(DEV)
            slot_d, sl_d, pos_d = (torch.from_numpy(x).to(DEV) for x in (slot, sl, pos))
            amd[ref_attn[l].x_name] = va.KV800Meta(btl, slot_d, sl_d, torch.from_numpy(sl), torch.from_numpy(qsl),
                                                   pos_d, len(sched), T, nd)
            ours[l] = S.build_meta(btl, slot_d, sl_d, torch.from_numpy(qsl).to(DEV), torch.from_numpy(sl),
                                   torch.from_numpy(qsl), pos_d, nd)
            if l in qbt:
                qb = torch.from_numpy(qbt[l][order]).to(DEV)
                amd[ref_attn[l].q_name] = va.KV800Meta(qb, slot_d, sl_d, torch.from_numpy(sl), torch.from_numpy(qsl),
                                                       pos_d, len(sched), T, nd)
                ours[("q", l)] = S.build_meta(qb, slot_d, sl_d, torch.from_numpy(qsl).to(DEV), torch.from_numpy(sl),
                                              torch.from_numpy(qsl), pos_d, nd)
        ctx.fc.attn_metadata = amd
        for l, kind in LAYERS.items():
            q = tb(I.f32_to_bf16(rs.standard_normal((T, 16, 128)).astype(np.float32)), DEV)
            k = tb(I.f32_to_bf16((rs.standard_normal((T, 4, 128)) + 1.5).astype(np.float32)), DEV)
            v = tb(I.f32_to_bf16(rs.standard_normal((T, 4, 128)).astype(np.float32)), DEV)
            o_ref = ref_attn[l].forward(q, k, v)
            kw = {}
            if kind == "quant":
                kw = dict(mq=ours[("q", l)], qv=qv["ours"][l])
            elif kind == "window":
                kw = dict(hosts=((ours[("q", 6)], qv["ours"][6]), (ours[("q", 10)], qv["ours"][10])))
            o_ours = our_attn[l].forward(q, k, v, ours[l], ev["ours"][l], **kw)
            torch.cuda.synchronize()
            assert_parity(nb(o_ours[:T]), nb(o_ref[:T]), f"step {step}, layer {l} ({kind}): vllm_step vs vllm_attn")
        for r, t in sched:
            n[r] += t
        for l in LAYERS:
            assert torch.equal(ev["ref"][l].view(torch.int16), ev["ours"][l].view(torch.int16)), \
                f"step {step}: exact cache of layer {l} differs"
        for l in qbt:
            assert torch.equal(qraw["ref"][l], qraw["ours"][l]), f"step {step}: quant cache of layer {l} differs"
    assert n[2] >= 384 and int((qraw["ours"][6] != 0).sum()) > 0
