"""One vLLM step of an LFM3 full-attention layer over the 800h caches, on the device.

This is the data path of the reference's vLLM attention layer (lfm3_kv800/vllm_attn.py:244-402, KV800Attention.forward)
with the host work taken out: the exact-cache scatter, the sink write, the flush plan and its gather/quantize/scatter,
and the decode tables are single CUDA launches over vLLM's own metadata tensors (block tables, slot mapping, seq_lens,
query_start_loc), so a step builds no index tensors, runs no Python loop over requests or sub-blocks and makes no
host sync.  Host values come only from the CPU copies vLLM already keeps (seq_lens_cpu, query_start_loc_cpu): the
flush pair count and the decode nqmax.

It is written against plain tensors rather than vLLM's forward context, so the vLLM glue (KV800Backend, the cache
specs, the metadata builder) stays a thin layer: `KV800Attention.forward(q, k, v, meta, ...)` takes the layer's
caches and the step metadata explicitly.  The cache geometry follows vllm_attn.py:1-12,125-142:
  quant cache  per quantized layer, pages of QPAGE = 262,144 B holding QBLOCK / 256 = 5 sub-blocks of 51,200 B
               (the 6,144-byte tail of a request's first page is the aux area holding the 4 sink rows of a window
               layer); a uint8 view whose shape[2] is the page's token count and stride(0) the page bytes
  exact cache  per layer, [blocks, 4, ebs, 256] bf16: K (pre-RoPE) in the first 128 of the last dimension, V after.
Decode rows go through kv800.decode (the sm_100a split-K kernels); prefill / extend rows attend with torch's fused
scaled_dot_product_attention in bf16 over the history assembled by kv800_prefill_kv (dequantized sub-blocks, sinks,
exact window and the chunk, K rotated), the reference's flash prefill (vllm_attn.py:190-211)."""
import ctypes
from dataclasses import dataclass, field

import torch

from . import _lib, get_logger, kv800
from .kv800 import BLK, LAG, NSINK, SUB, WIN, _cuda, _extent, _ptr, _stream

_log = get_logger()
QUANT_LAYERS, WINDOW_LAYERS = (6, 10, 14, 22), (2, 18)
SINK_HOST = {2: (6, 10), 18: (14, 22)}     # window layer -> (layer whose aux holds its sink K, ... its sink V)
EXACT_WINDOW = 640
QBLOCK, QCONTENT, QPAGE = 1280, 25, 262144
PREFILL_CHUNK = 2048                       # queries per SDPA call (vllm_attn.py:195)


def nq_of(n):
    """sub-blocks flushed once a sequence holds n tokens (the flush rule: n >= 256 j + 384)."""
    return max(0, int(n) - LAG) // BLK


def aux_offset(qv):
    """bf16 element offset, inside a quant page, of the aux area (after the page's sub-blocks)."""
    return (qv.shape[2] // BLK) * (SUB // 2)


@dataclass
class StepMeta:
    """Per-step attention metadata of one KV cache group (vllm_attn.py:61-72); `cache` holds values shared by the
    layers of the group within the step."""
    block_table: torch.Tensor          # (R, pages) int32, device
    slot_mapping: torch.Tensor         # (T,) int64, device
    seq_lens: torch.Tensor             # (R,) int32, device
    seq_lens_cpu: torch.Tensor         # (R,) host copy
    query_start_loc: torch.Tensor      # (R + 1,) int32, device
    query_start_loc_cpu: torch.Tensor  # (R + 1,) host copy
    positions: torch.Tensor            # (T,) int64, device
    num_reqs: int
    num_actual_tokens: int
    num_decodes: int
    cache: dict = field(default_factory=dict)


def build_meta(block_table, slot_mapping, seq_lens, query_start_loc, seq_lens_cpu=None, query_start_loc_cpu=None,
               positions=None, num_decodes=None):
    """KV800Builder.build (vllm_attn.py:84-101) on plain tensors.  Requests are ordered decodes first (vLLM's
    reorder_batch_threshold 1); num_decodes defaults to the leading run of one-token requests.  positions default to
    seq_len - qlen + (i - qsl) per token, computed on the device."""
    dev = seq_lens.device
    qsl_cpu = (query_start_loc_cpu if query_start_loc_cpu is not None else query_start_loc.cpu()).to(torch.int64)
    R = qsl_cpu.numel() - 1
    sl_cpu = (seq_lens_cpu if seq_lens_cpu is not None else seq_lens[:R].cpu()).to(torch.int64)
    T = int(qsl_cpu[R])
    qlen_cpu = qsl_cpu[1:] - qsl_cpu[:-1]
    if num_decodes is None:
        nd = 0
        while nd < R and int(qlen_cpu[nd]) == 1:
            nd += 1
    else:
        nd = int(num_decodes)
    qsl = query_start_loc.to(device=dev, dtype=torch.int32)
    if positions is None:
        qlen = (qsl[1:] - qsl[:-1]).long()
        start = seq_lens[:R].long() - qlen
        positions = torch.repeat_interleave(start - qsl[:-1].long(), qlen, output_size=T) + torch.arange(T, device=dev)
    return StepMeta(block_table.to(torch.int32), slot_mapping[:T].long(), seq_lens[:R].to(torch.int32), sl_cpu, qsl,
                    qsl_cpu, positions[:T].long(), R, T, nd)


_TABLES: dict = {}


def tables(device, max_pos):
    """(cos32, sin32) [P, 32] bf16 for the kernels as the HF Lfm3 full layers build them (theta 1e6, 32 rotating
    frequencies over head_dim 128, fp32 product, bf16 cast), plus the identity tables of the native sliding layers
    (vllm_attn.py:147-159)."""
    key = (str(device), max_pos)
    if key not in _TABLES:
        inv = 1.0 / (1e6 ** (torch.arange(0, 64, 2, dtype=torch.float32, device=device) / 128))
        fr = torch.arange(max_pos, device=device, dtype=torch.float32)[:, None] * inv[None]
        c32, s32 = fr.cos().to(torch.bfloat16).contiguous(), fr.sin().to(torch.bfloat16).contiguous()
        _TABLES[key] = (c32, s32, torch.ones_like(c32), torch.zeros_like(s32))
    return _TABLES[key]


def _status(C, dev):
    if "status" not in C:
        C["status"] = torch.zeros(1, dtype=torch.int32, device=dev)
    return C["status"]


def bf16_flat(t):
    """1-D bf16 view of t's storage from t's first byte on (the quant caches are uint8 pages; the sink rows in their
    aux areas are bf16), and the page stride in bf16 elements."""
    off = t.storage_offset() * t.element_size()
    n = (t.untyped_storage().nbytes() - off) // 2
    flat = torch.empty(0, dtype=torch.bfloat16, device=t.device).set_(t.untyped_storage(), off // 2, (n,), (1,))
    return flat, t.stride(0) * t.element_size() // 2


def _bf(t):
    return t if t.dtype == torch.bfloat16 and t.is_contiguous() else t.to(torch.bfloat16).contiguous()


# ---------------------------------------------------------------- the device ops of a step
def write_slots(ev, k, v, slot_mapping, status=None):
    """Exact K / V of every scheduled token into the window pages: token i -> block slot[i] // ebs, row slot[i] % ebs
    (vllm_attn.py:261-269); negative slots (padding) are skipped."""
    dev = _cuda(ev, "write_slots").device
    T = slot_mapping.numel()
    if T == 0:
        return
    k, v = _bf(k[:T]), _bf(v[:T])
    slot = slot_mapping.to(device=dev, dtype=torch.int64).contiguous()
    _lib.call("kv800_write_slots", _ptr(ev), _extent(ev), ev.stride(0), ev.stride(1), ev.stride(2), ev.shape[2],
              _ptr(k), _ptr(v), _ptr(slot), T, _ptr(status), _stream(dev))


def write_sinks(host_k, bt_k, host_v, bt_v, k, v, positions, slot_mapping, query_start_loc, status=None):
    """Positions < 4 of a window layer into the aux area of the request's first page of two host quant caches
    (vllm_attn.py:276-291): K rows into host_k, V rows into host_v (uint8 quant-cache views)."""
    dev = _cuda(host_k, "write_sinks").device
    T = positions.numel()
    R = query_start_loc.numel() - 1
    if T == 0 or R <= 0:
        return
    (hk, hk0), (hv, hv0) = bf16_flat(host_k), bf16_flat(host_v)
    k, v = _bf(k[:T]), _bf(v[:T])
    bk, bv = bt_k.to(torch.int32), bt_v.to(torch.int32)
    _lib.call("kv800_write_sinks", _ptr(hk), hk.numel(), hk0, aux_offset(host_k), _ptr(bk), bk.stride(0),
              _ptr(hv), hv.numel(), hv0, aux_offset(host_v), _ptr(bv), bv.stride(0), _ptr(k), _ptr(v),
              _ptr(positions.contiguous()), _ptr(slot_mapping.contiguous()), _ptr(query_start_loc.contiguous()), R, T,
              _ptr(status), _stream(dev))


def flush_pairs(seq_lens_cpu, query_start_loc_cpu):
    """Sub-blocks the step flushes, from the host copies (no device sync)."""
    sl = seq_lens_cpu.to(torch.int64)
    qsl = query_start_loc_cpu.to(torch.int64)
    prev = sl - (qsl[1:] - qsl[:-1])
    nq = lambda n: torch.clamp(n - LAG, min=0) // BLK   # noqa: E731
    return int((nq(sl) - nq(prev)).clamp(min=0).sum())


def flush_step(ev, block_table, qv, qblock_table, seq_lens, query_start_loc, max_pairs, status=None, workspace=None):
    """Quantize every sub-block that became eligible this step (n >= 256 j + 384) from the exact cache into the quant
    cache (vllm_attn.py:298-317): plan, gather, quantize and scatter on the device in two launches."""
    dev = _cuda(ev, "flush_step").device
    R = seq_lens.numel()
    if R == 0 or max_pairs <= 0:
        return
    need = int(_lib.lib().kv800_flush_step_workspace_size(int(max_pairs)))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    bt, qbt = block_table.to(torch.int32).contiguous(), qblock_table.to(torch.int32).contiguous()
    _lib.call("kv800_flush_step", _ptr(ev), _extent(ev), ev.stride(0), ev.stride(1), ev.stride(2), ev.shape[2],
              _ptr(bt), bt.stride(0), _ptr(qv), _extent(qv) * qv.element_size(), qv.stride(0) * qv.element_size(),
              qv.shape[2], _ptr(qbt), qbt.stride(0), _ptr(seq_lens.to(torch.int32).contiguous()),
              _ptr(query_start_loc.to(torch.int32).contiguous()), R, int(max_pairs), _ptr(workspace), workspace.numel(),
              _ptr(status), _stream(dev))


def decode_tables(seq_lens, nd, block_table, s0, qblock_table=None, qs0=0, bsq=0, nqw=0, sinks=None):
    """N, NQ, EOFF (and BOFF, or the sink offsets) of the first nd requests in one launch (vllm_attn.py:320-349).
    sinks: ((bt_k, s0_k, aux_k), (bt_v, s0_v, aux_v)) of the two host layers.  Returns a dict of device tensors."""
    dev = seq_lens.device
    bt = block_table.to(torch.int32).contiguous()     # the kernel reads bt_stride columns per row
    out = {"N": torch.empty(nd, dtype=torch.int32, device=dev), "NQ": torch.empty(nd, dtype=torch.int32, device=dev),
           "eoff": torch.empty(nd, bt.shape[1], dtype=torch.int64, device=dev)}
    args_q = [None, 0, 0, 0, 0, None]
    if nqw:
        qbt = qblock_table.to(torch.int32).contiguous()
        out["boff"] = torch.empty(nd, nqw, dtype=torch.int64, device=dev)
        args_q = [_ptr(qbt), qbt.stride(0), int(qs0), int(bsq), int(nqw), _ptr(out["boff"])]
        out["_qbt"] = qbt
    args_s = [None, 0, 0, 0, None] * 2
    if sinks is not None:
        (bk, sk0, ak), (bv, sv0, av) = sinks
        bk, bv = bk.to(torch.int32), bv.to(torch.int32)
        out["skoff"] = torch.empty(nd, dtype=torch.int64, device=dev)
        out["svoff"] = torch.empty(nd, dtype=torch.int64, device=dev)
        args_s = [_ptr(bk), bk.stride(0), int(sk0), int(ak), _ptr(out["skoff"]),
                  _ptr(bv), bv.stride(0), int(sv0), int(av), _ptr(out["svoff"])]
        out["_sbt"] = (bk, bv)
    if nd:
        _lib.call("kv800_decode_tables", _ptr(seq_lens.to(torch.int32).contiguous()), nd, _ptr(bt), bt.stride(0),
                  int(s0), _ptr(out["N"]), _ptr(out["NQ"]), _ptr(out["eoff"]), *args_q, *args_s, _stream(dev))
    return out


def prefill_kv(n0, n, k, v, ev, bt_row, qv=None, qbt_row=None, nqp=0, sk=None, sv=None, ns=0, lo=None, cos_t=None,
               sin_t=None, status=None):
    """K / V (bf16, (S, 4, 128)) and positions of one prefill / extend request in the reference's order: nqp
    dequantized sub-blocks, ns sinks, exact rows [lo, n0), then the chunk k / v at positions n0 .. n - 1; K rotated
    with cos_t / sin_t ([P, 32] bf16) unless they are None (vllm_attn.py:355-388)."""
    dev = _cuda(ev, "prefill_kv").device
    lo = nqp * BLK if lo is None else int(lo)
    if k.shape[0] != n - n0 or v.shape[0] != n - n0 or tuple(k.shape[1:]) != (4, 128):
        raise ValueError(f"prefill_kv: the chunk must be ({n - n0}, 4, 128), got {tuple(k.shape)} / {tuple(v.shape)}")
    if ns and (sk is None or sv is None or sk.numel() < ns * 512 or sv.numel() < ns * 512):
        raise ValueError(f"prefill_kv: {ns} sink rows need sk / sv of at least ({ns}, 4, 128)")
    bt_row = bt_row.to(torch.int32).contiguous()
    if qbt_row is not None:
        qbt_row = qbt_row.to(torch.int32).contiguous()
    S = nqp * BLK + ns + (n0 - lo) + (n - n0)
    K = torch.empty(S, 4, 128, dtype=torch.bfloat16, device=dev)
    V = torch.empty(S, 4, 128, dtype=torch.bfloat16, device=dev)
    k, v = _bf(k), _bf(v)
    if ns:
        sk, sv = _bf(sk), _bf(sv)
    npos = cos_t.shape[0] if cos_t is not None else 0
    qbytes = _extent(qv) * qv.element_size() if qv is not None else 0
    qs0 = qv.stride(0) * qv.element_size() if qv is not None else 0
    bsq = qv.shape[2] if qv is not None else 0
    _lib.call("kv800_prefill_kv", _ptr(qv) if nqp else None, qbytes, qs0, bsq, _ptr(qbt_row) if nqp else None,
              qbt_row.numel() if qbt_row is not None else 0, int(nqp), _ptr(sk) if ns else None,
              _ptr(sv) if ns else None, int(ns), _ptr(ev), _extent(ev), ev.stride(0), ev.stride(1), ev.stride(2),
              ev.shape[2], _ptr(bt_row), bt_row.numel(), lo, int(n0), _ptr(k), _ptr(v), int(n), _ptr(cos_t),
              _ptr(sin_t), npos, _ptr(K), _ptr(V), _ptr(status), _stream(dev))
    parts = []
    if nqp:
        parts.append(torch.arange(nqp * BLK, device=dev))
    if ns:
        parts.append(torch.arange(ns, device=dev))
    parts.append(torch.arange(lo, n, device=dev))
    return K, V, torch.cat(parts)


def attend(q, K, V, kp, n0, n, slide, win):
    """Prefill attention of queries at positions n0 .. n - 1 over K / V at positions kp: torch's fused SDPA in bf16,
    2048 queries per call, one boolean mask shared by the heads (causal, plus the 256-window and sinks), as the
    reference's flash prefill (vllm_attn.py:190-211)."""
    import torch.nn.functional as F
    Kh = K.repeat_interleave(4, 1).transpose(0, 1)[None]
    Vh = V.repeat_interleave(4, 1).transpose(0, 1)[None]
    qi = q.to(torch.bfloat16).transpose(0, 1)[None]
    qp = torch.arange(n0, n, device=q.device)
    out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
    for a in range(0, n - n0, PREFILL_CHUNK):
        qa = qp[a:a + PREFILL_CHUNK, None]
        m = kp[None] <= qa
        if slide:
            m = m & (kp[None] > qa - WIN)
        elif win:
            m = m & ((kp[None] > qa - WIN) | (kp[None] < NSINK))
        o = F.scaled_dot_product_attention(qi[:, :, a:a + PREFILL_CHUNK], Kh, Vh, attn_mask=m[None, None],
                                           scale=128 ** -0.5)
        out[a:a + PREFILL_CHUNK] = o[0].transpose(0, 1)
    return out


# ---------------------------------------------------------------- the layer
class KV800Attention:
    """Attention core of one LFM3 full-attention layer with the 800h cache (vllm_attn.py:214-402).  forward(q, k, v):
    q (T, 16, 128) post-RoPE, k (T, 4, 128) PRE-RoPE, v (T, 4, 128) -> (T, 16, 128) bf16.  slide=True is a native
    sliding layer (window 256, no sinks, K stored post-RoPE, identity rotation in the kernels)."""

    def __init__(self, layer_idx, max_pos, slide=False):
        self.l, self.max_pos, self.slide = layer_idx, max_pos, slide
        self.win = slide or layer_idx in WINDOW_LAYERS

    def forward(self, q, k, v, mx, ev, mq=None, qv=None, hosts=None):
        """mx: StepMeta of this layer's exact-cache group, ev its exact cache; mq / qv: the quant cache's metadata and
        uint8 view (quantized layers); hosts: ((meta, qv) of the sink-K host, (meta, qv) of the sink-V host) for
        window layers."""
        dev = q.device
        out = torch.zeros(q.shape, dtype=torch.bfloat16, device=dev)
        T, R, nd = mx.num_actual_tokens, mx.num_reqs, mx.num_decodes
        if T == 0:
            return out
        c32, s32, one32, zero32 = tables(dev, self.max_pos)
        if self.slide:
            c32, s32 = one32, zero32
        C = mx.cache
        st = _status(C, dev)
        s0, s1, s2, ebs = ev.stride(0), ev.stride(1), ev.stride(2), ev.shape[2]
        # 1. exact K / V of every scheduled token
        write_slots(ev, k, v, mx.slot_mapping, st)
        if "prev" not in C:
            qsl = mx.query_start_loc_cpu
            C["prev"] = mx.seq_lens_cpu - (qsl[1:] - qsl[:-1])
        prev = C["prev"]
        if self.slide:
            pass
        elif self.win:
            # 2a. sinks: only a step holding a position < 4 writes them (decided on host data)
            if bool((prev < NSINK).any()):
                (hmk, hvk), (hmv, hvv) = hosts
                write_sinks(hvk, hmk.block_table, hvv, hmv.block_table, k, v, mx.positions, mx.slot_mapping,
                            mx.query_start_loc, st)
        else:
            # 2b. flush of the sub-blocks that became eligible this step
            if "npairs" not in C:
                C["npairs"] = flush_pairs(mx.seq_lens_cpu, mx.query_start_loc_cpu)
            flush_step(ev, mx.block_table, qv, mq.block_table, mx.seq_lens, mx.query_start_loc, C["npairs"], st)
        # 3. decode rows
        if nd:
            if self.slide or self.win:
                tkey = ("dec", "win" if not self.slide else "slide", s0, nd)
                if tkey not in C:
                    sinks = None
                    if not self.slide:
                        (hmk, hvk), (hmv, hvv) = hosts
                        sinks = ((hmk.block_table[:nd], bf16_flat(hvk)[1], aux_offset(hvk)),
                                 (hmv.block_table[:nd], bf16_flat(hvv)[1], aux_offset(hvv)))
                    C[tkey] = decode_tables(mx.seq_lens[:nd], nd, mx.block_table[:nd], s0, sinks=sinks)
                tb = C[tkey]
                sk = sv = None
                if not self.slide:
                    sk, sv = bf16_flat(hosts[0][1])[0], bf16_flat(hosts[1][1])[0]
                P = kv800.Paged(qpool=ev, boff=tb["eoff"], epool=ev, eoff=tb["eoff"], ebs=ebs, e_hs=s1, e_ts=s2,
                                e_v=128, sk=sk, sv=sv, skoff=tb.get("skoff"), svoff=tb.get("svoff"), N=tb["N"],
                                NQ=tb["NQ"], nqmax=0, win=WIN)
            else:
                qs0, bsq = qv.stride(0) * qv.element_size(), qv.shape[2]
                tkey = ("dec", "quant", s0, qs0, bsq, nd)
                if tkey not in C:
                    nqmax = nq_of(int(mx.seq_lens_cpu[:nd].max()))
                    tb = decode_tables(mx.seq_lens[:nd], nd, mx.block_table[:nd], s0, mq.block_table[:nd], qs0, bsq,
                                       nqmax)
                    tb["nqmax"] = nqmax
                    C[tkey] = tb
                tb = C[tkey]
                P = kv800.Paged(qpool=qv, boff=tb.get("boff"), epool=ev, eoff=tb["eoff"], ebs=ebs, e_hs=s1, e_ts=s2,
                                e_v=128, N=tb["N"], NQ=tb["NQ"], nqmax=tb["nqmax"], win=0)
            rot = (None, None) if self.slide else (c32, s32)     # sliding layers: no rotation at all
            out[:nd] = kv800.decode(P, q[:nd].contiguous(), *rot)
        # 4. prefill / extend rows
        qsl, sl = mx.query_start_loc_cpu, mx.seq_lens_cpu
        for i in range(nd, R):
            s, e = int(qsl[i]), int(qsl[i + 1])
            n, n0 = int(sl[i]), int(prev[i])
            if e == s:
                continue
            rope = (None, None) if self.slide else (c32, s32)
            if self.win:
                lo = max(0, n0 - (WIN - 1))
                ns = 0 if self.slide else min(NSINK, lo)
                sk = sv = None
                if ns:
                    (hmk, hvk), (hmv, hvv) = hosts
                    sk = self._sink_rows(hvk, hmk, i, ns)
                    sv = self._sink_rows(hvv, hmv, i, ns)
                K, V, kp = prefill_kv(n0, n, k[s:e], v[s:e], ev, mx.block_table[i], sk=sk, sv=sv, ns=ns, lo=lo,
                                      cos_t=rope[0], sin_t=rope[1], status=st)
            else:
                nqp = nq_of(n0)
                K, V, kp = prefill_kv(n0, n, k[s:e], v[s:e], ev, mx.block_table[i], qv=qv, qbt_row=mq.block_table[i],
                                      nqp=nqp, cos_t=c32, sin_t=s32, status=st)
            out[s:e] = attend(q[s:e], K, V, kp, n0, n, self.slide, self.win)
        kv800._check_status(st, dev, "vllm step")
        return out

    @staticmethod
    def _sink_rows(hv, hm, i, ns):
        """(ns, 4, 128) bf16 view of request i's sink rows in a host quant cache's first page (vllm_attn.py:360-363)."""
        flat, ps = bf16_flat(hv)
        a = int(hm.block_table[i, 0]) * ps + aux_offset(hv)
        return flat[a:a + ns * 512].view(ns, 4, 128)
