"""Paged 800h KV cache (the layout vLLM pages hold) with one CUDA backend for B200 (sm_100a).

Same layout, operator surface and semantics as the reference module (riceharvest/lfm3-kv800, lfm3_kv800/kv800.py):
quantized layer state = 256-token SUB-BLOCKS of 51,200 bytes addressed by BOFF[b, j] (byte offset from the quant
pool's base pointer).  Sub-block layout:
  [0, 32768)      kc   [256, 4, 32]  planar 2-bit K (byte j = dims j, j+32, j+64, j+96 at bits 0-1/2-3/4-5/6-7)
  [32768, 49152)  vb   [256, 4, 16]  planar 1-bit V after per-head Hadamard (byte j = dims j + 16i at bit i)
  [49152, 49664)  vlo  [256, 2] fp8   per (token, 2-head group)
  [49664, 50176)  vsc  [256, 2] fp8
  [50176, 50688)  klo  [4, 128] fp8   per (head, channel) over the 256 tokens, PRE-RoPE
  [50688, 51200)  ksc  [4, 128] fp8
Exact tokens (pre-RoPE K, unrotated V, bf16) live in pages of EBS tokens addressed by EOFF[b, p // EBS] (element
offset of the page in the exact pool); inside a page: K of (head h, slot t) at + h*e_hs + t*e_ts, V at + e_v from K.
Sinks (window layers): K/V of positions 0..3 at element offsets SKOFF[b] / SVOFF[b] in their pools, layout [4, 4, 128].
Semantics: sub-block j of a full layer is quantized once n >= 256 j + 384 (the newest 128..383 tokens stay exact);
window layers = 4 sinks + the last 256 tokens, all exact.

Backend: the reference's sycl -> triton -> torch chain (kv800.py:251-349) is replaced by ONE backend, "cuda": the
hand-written sm_100a kernels of libkv800_b200.so behind the C ABI of include/kv800_b200.h.  There is no CPU path and
no fallback: a call on a non-CUDA tensor, or without the built library, raises.  Env LFM3KV_BACKEND=cuda|auto (or
set_backend()) selects it; any other name raises ValueError as the reference does for unknown names.  Env
LFM3KV_CHECK=1 reads back the device status word after every call (a host sync) and raises on a range-check event."""
import ctypes
import math
import os

import torch

from . import _lib, get_logger
from . import ops as _ops

BLK, LAG, NSINK, WIN = 256, 128, 4, 256
SUB = 51200
KC_O, VB_O, VLO_O, VSC_O, KLO_O, KSC_O = 0, 32768, 49152, 49664, 50176, 50688
F8 = torch.float8_e4m3fn
LOG2E = 1.4426950408889634
BACKENDS = ("cuda",)
_log = get_logger()
_ops.register()          # torch.ops.kv800.{qdecode, xdecode, combine}: the reference's op schema on these kernels

__all__ = ["BLK", "LAG", "NSINK", "WIN", "SUB", "KC_O", "VB_O", "VLO_O", "VSC_O", "KLO_O", "KSC_O", "F8", "LOG2E",
           "BACKENDS", "hadamard", "flat", "quantize_blocks", "dequantize_blocks", "Paged", "PagedStore", "decode",
           "combine", "set_backend", "get_backend", "flush", "write_exact"]


def hadamard(n=128, device=None):
    """Orthonormal Sylvester Hadamard (n x n, fp32), the reference's hadamard() (kv800.py:43-46)."""
    H = torch.ones(1, 1)
    while H.shape[0] < n:
        H = torch.cat((torch.cat((H, H), 1), torch.cat((H, -H), 1)), 0)
    return (H / n ** 0.5).to(device)


def flat(t):
    """1-D view of t's storage starting at t's first element (t may be a strided view into a shared buffer)."""
    n = t.untyped_storage().nbytes() // t.element_size() - t.storage_offset()
    return torch.as_strided(t, (n,), (1,), t.storage_offset())


# ---------------------------------------------------------------- boundary helpers
def _extent(t):
    """elements of t's storage from t's first element on (the range a pool offset may address)."""
    return t.untyped_storage().nbytes() // t.element_size() - t.storage_offset()


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _cuda(t, what):
    if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
        dev = t.device if isinstance(t, torch.Tensor) else type(t).__name__
        raise RuntimeError(f"{what}: the 800h CUDA backend needs CUDA tensors (got {dev}); this package has no CPU "
                           f"path (the reference's torch backend is its test oracle, not a fallback)")
    return t


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _i64(t, dev):
    return t.to(device=dev, dtype=torch.int64).contiguous()


def _i32(t, dev):
    return t.to(device=dev, dtype=torch.int32).contiguous()


def _bf16(t):
    if t.dtype == torch.float16:                      # accepted and upcast, as the reference does for q
        t = t.to(torch.bfloat16)
    if t.dtype != torch.bfloat16:
        raise TypeError(f"expected a bf16 tensor, got {t.dtype}")
    return t.contiguous()


def _bits(t):
    """bf16 tensor -> its storage seen as int16 (same pointer)."""
    return t.view(torch.int16)


_CHECK = os.environ.get("LFM3KV_CHECK", "0") not in ("", "0")


def _check_status(status, dev, who):
    if status is None or not _CHECK:
        return
    host = ctypes.c_int(0)
    _lib.call("kv800_check_status", _ptr(status), ctypes.byref(host), _stream(dev))


# ---------------------------------------------------------------- quantizer (kv800.py:56-92)
def quantize_blocks(k, v, H=None):
    """k, v: (M, 256, 4, 128) bf16 (pre-RoPE K, unrotated V) -> (M, 51200) uint8 sub-blocks, bit-exact with the
    reference quantizer.  H is accepted for signature compatibility and must be hadamard(128): the kernel applies the
    normalized 128-point Hadamard itself."""
    _cuda(k, "quantize_blocks")
    if k.dim() != 4 or tuple(k.shape[1:]) != (BLK, 4, 128) or v.shape != k.shape:
        raise ValueError(f"quantize_blocks: k, v must be (M, 256, 4, 128), got {tuple(k.shape)} / {tuple(v.shape)}")
    if k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise TypeError(f"quantize_blocks: k, v must be bf16 (the values the cache stores), got {k.dtype} / {v.dtype}")
    k, v = k.contiguous(), v.contiguous()
    M = k.shape[0]
    out = torch.empty(M, SUB, dtype=torch.uint8, device=k.device)
    _lib.call("kv800_quantize_blocks", _ptr(k), _ptr(v), M, _ptr(out), _stream(k.device))
    return out


def dequantize_blocks(sb, H=None):
    """(M, 51200) uint8 -> pre-RoPE K (M, 256, 4, 128) bf16 and unrotated V (M, 256, 4, 128) fp32 (kv800.py:79-92)."""
    _cuda(sb, "dequantize_blocks")
    if sb.dim() != 2 or sb.shape[1] != SUB or sb.dtype != torch.uint8:
        raise ValueError(f"dequantize_blocks: expected (M, {SUB}) uint8, got {tuple(sb.shape)} {sb.dtype}")
    sb = sb.contiguous()
    M = sb.shape[0]
    k = torch.empty(M, BLK, 4, 128, dtype=torch.bfloat16, device=sb.device)
    v = torch.empty(M, BLK, 4, 128, dtype=torch.float32, device=sb.device)
    _lib.call("kv800_dequantize_blocks", _ptr(sb), M, _ptr(k), _ptr(v), _stream(sb.device))
    return k, v


def flush(epool, eoff, ebs, e_hs, e_ts, e_v, qpool, boff, seq, blk, status=None):
    """Quantize sub-blocks blk[m] of sequences seq[m] from the exact pages into qpool at boff[seq, blk] (the flush of
    kv800.py:433-440 / vllm_attn.py:298-317 in one launch).  epool: bf16 pool (EOFF base), qpool: uint8 pool (BOFF
    base), eoff / boff: int64 (nseq, *) tables, seq / blk: int tensors of equal length."""
    dev = _cuda(qpool, "flush").device
    eoff, boff = _i64(eoff, dev), _i64(boff, dev)
    seq, blk = _i32(seq, dev), _i32(blk, dev)
    M = seq.numel()
    if M == 0:
        return
    _lib.call("kv800_flush", _ptr(epool), _extent(epool), _ptr(eoff), eoff.stride(0), ebs, e_hs, e_ts, e_v,
              _ptr(qpool), _extent(qpool), _ptr(boff), boff.stride(0), _ptr(seq), _ptr(blk), M, eoff.shape[0],
              _ptr(status), _stream(dev))


def write_exact(epool, eoff, ebs, e_hs, e_ts, e_v, k, v, seq, pos, status=None):
    """Scatter tokens (T, 4, 128) of k / v into the exact pages of sequences seq[i] at positions pos[i]
    (kv800.py:423-428 / vllm_attn.py:261-269)."""
    dev = _cuda(epool, "write_exact").device
    eoff = _i64(eoff, dev)
    k, v = _bf16(k.to(torch.bfloat16)), _bf16(v.to(torch.bfloat16))
    seq, pos = _i32(seq, dev), _i64(pos, dev)
    T = seq.numel()
    if T == 0:
        return
    _lib.call("kv800_write_exact", _ptr(epool), _extent(epool), _ptr(eoff), eoff.stride(0), ebs, e_hs, e_ts, e_v,
              _ptr(k), _ptr(v), _ptr(seq), _ptr(pos), T, eoff.shape[0], _ptr(status), _stream(dev))


# ---------------------------------------------------------------- decode input record (kv800.py:239-248)
class Paged:
    """The decode's view of one layer's cache for a batch of rows (the reference's 16-slot record).

    Offsets are relative to the first element of the tensor they index into:
      qpool  uint8 pool of sub-blocks; boff[b, j] = byte offset of row b's sub-block j
      epool  bf16 pool of exact pages; eoff[b, p] = element offset of the page holding row b's positions
             [p ebs, (p + 1) ebs); K of (head h, slot t) at + h e_hs + t e_ts, V at + e_v from K
      sk, sv bf16 sink pools (window layers); skoff[b] / svoff[b] = element offset of row b's [4, 4, 128] sink rows
      N      int32 row lengths, the current token included; NQ int32 sub-blocks flushed per row
      nqmax  host int, an upper bound of NQ; win 0 for a quantized layer, 256 for a window layer with sinks."""
    __slots__ = ("qpool", "boff", "epool", "eoff", "ebs", "e_hs", "e_ts", "e_v", "sk", "sv", "skoff", "svoff",
                 "N", "NQ", "nqmax", "win")

    def __init__(self, **kw):
        for k in self.__slots__:
            setattr(self, k, kw.get(k))


# ---------------------------------------------------------------- backend selection (kv800.py:251-349)
_FORCED = None
_CHOSEN = {}
_LAST = [None]


def _requested():
    v = _FORCED if _FORCED is not None else os.environ.get("LFM3KV_BACKEND", "auto")
    v = (v or "auto").strip().lower()
    if v not in BACKENDS + ("auto",):
        raise ValueError(f"LFM3KV_BACKEND={v!r}: expected one of {', '.join(BACKENDS)}, auto (this build has a single "
                         f"CUDA backend)")
    return v


def set_backend(name=None):
    """Force the decode backend ('cuda'), or 'auto' / None (env LFM3KV_BACKEND is read when this is None)."""
    global _FORCED
    _FORCED = None if name is None else str(name).strip().lower()
    _requested()
    _CHOSEN.clear()


def get_backend(device_type=None):
    """Backend used by the last decode() (or the one in use on `device_type`)."""
    return _CHOSEN.get(device_type) if device_type else _LAST[0]


def _available(name, dt):
    """(ok, detail) for backend `name` on device type `dt`."""
    if name != "cuda":
        return False, f"backend {name!r} does not exist in this build (only 'cuda')"
    if dt != "cuda":
        return False, f"the CUDA backend runs on cuda devices only (device type {dt!r})"
    try:
        _lib.lib()
    except ImportError as e:
        return False, str(e)
    return True, f"libkv800_b200.so (sm_100a), {_lib.LIB_PATH}"


def _resolve(dt):
    if dt in _CHOSEN:
        return _CHOSEN[dt]
    req = _requested()
    ok, why = _available("cuda", dt)
    if not ok:
        raise RuntimeError(f"800h decode on {dt}: no backend available ({why}); requested {req!r}")
    _log.info("decode backend on %s: cuda (%s%s)", dt, why, "; forced" if req != "auto" else "")
    _CHOSEN[dt] = "cuda"
    return "cuda"


def _paged_struct(P, dev, B):
    """kv800_paged record for Paged P (keeps the converted tensors alive in the returned tuple)."""
    win = int(P.win or 0)
    nqmax = 0 if win else int(P.nqmax or 0)
    keep = []
    N, NQ = _i32(P.N, dev), _i32(P.NQ, dev)
    eoff = _i64(P.eoff, dev)
    if eoff.dim() == 1:
        eoff = eoff.view(B, -1)
    keep += [N, NQ, eoff]
    s = _lib.Paged()
    if nqmax:
        boff = _i64(P.boff, dev)
        if boff.dim() == 1:
            boff = boff.view(B, -1)
        if boff.shape[0] != B:
            raise ValueError(f"decode: boff has {boff.shape[0]} rows for batch {B}")
        keep.append(boff)
        s.qpool, s.qpool_bytes = P.qpool.data_ptr(), _extent(P.qpool) * P.qpool.element_size()
        s.boff, s.boff_stride = boff.data_ptr(), boff.stride(0)
    s.epool, s.epool_elems = P.epool.data_ptr(), _extent(P.epool)
    s.eoff, s.eoff_stride = eoff.data_ptr(), eoff.stride(0)
    s.ebs, s.e_hs, s.e_ts, s.e_v = int(P.ebs), int(P.e_hs), int(P.e_ts), int(P.e_v)
    if win and P.sk is not None:
        skoff = _i64(P.skoff, dev)
        svoff = _i64(P.svoff if P.svoff is not None else P.skoff, dev)
        keep += [skoff, svoff]
        s.sk, s.sv = P.sk.data_ptr(), P.sv.data_ptr()
        s.sk_elems, s.sv_elems = _extent(P.sk), _extent(P.sv)
        s.skoff, s.svoff = skoff.data_ptr(), svoff.data_ptr()
        s.nsink = NSINK
    s.N, s.NQ = N.data_ptr(), NQ.data_ptr()
    s.nqmax, s.win = nqmax, win
    return s, keep


def decode(P, q, cos_t, sin_t, H=None, spb=None, target=None):
    """q: (B, 16, 128) bf16 post-RoPE -> (B, 16, 128) bf16. cos_t / sin_t: (P, 32) bf16 tables of the 32 rotating
    frequencies (dims d and d + 64 share frequency d, d < 32), or both None for a layer without quantized sub-blocks
    whose keys need no rotation (native sliding layers); H: accepted for signature compatibility (the kernels
    apply the normalized 128-point Hadamard themselves).  spb: sub-blocks per split; target: the reference's split
    sizing knob (spb = ceil(nqmax * B * 4 / target)); both None = the library's choice for 148 SMs."""
    return _decode(P, q, cos_t, sin_t, spb, target, None)


def decode_timed(P, q, cos_t, sin_t, spb=None):
    """decode() with CUDA-event timing of its phases (benchmarks; no counterpart in the reference).  Synchronizes.
    -> (out, {"quantized_ms": schedule + qdecode_mma, "exact_ms": the exact partials with the merge of each row's
    partials (done by the last exact-partial CTA of each row or (row, head)), "combine_ms": the gap after it (about zero)})."""
    ms = (ctypes.c_float * 3)()
    out = _decode(P, q, cos_t, sin_t, spb, None, ms)
    return out, {"quantized_ms": ms[0], "exact_ms": ms[1], "combine_ms": ms[2]}


def _decode(P, q, cos_t, sin_t, spb, target, ms):
    """decode() / decode_timed(); ms: a ctypes float[3] for the phase timings, or None."""
    _cuda(q, "decode")
    dt = q.device.type
    _LAST[0] = _resolve(dt)
    dev = q.device
    if q.dim() != 3 or tuple(q.shape[1:]) != (16, 128):
        raise ValueError(f"decode: q must be (B, 16, 128), got {tuple(q.shape)}")
    q = _bf16(q)
    B = q.shape[0]
    out = torch.empty(B, 16, 128, dtype=torch.bfloat16, device=dev)
    if B == 0:
        return out
    if cos_t is None and sin_t is None:
        # native sliding layers: keys stored post-RoPE, no rotation (the reference passes identity tables there)
        cs = sn = None
        npos = 0
    else:
        cs, sn = _bf16(cos_t), _bf16(sin_t)
        if cs.dim() != 2 or cs.shape[1] != 32 or sn.shape != cs.shape:
            raise ValueError(f"decode: cos_t / sin_t must be (P, 32), got {tuple(cs.shape)} / {tuple(sn.shape)}")
        for name, t in (("cos_t", cs), ("sin_t", sn)):
            _cuda(t, f"decode ({name})")
        npos = cs.shape[0]
    _cuda(P.epool, "decode (epool)")
    s, keep = _paged_struct(P, dev, B)
    nqmax = s.nqmax
    if spb is None and target is not None and nqmax:
        spb = max(1, math.ceil(nqmax * B * 4 / target))
    spb = int(spb or 0)
    ws_bytes = int(_lib.lib().kv800_decode_workspace_size(B, nqmax, s.win, spb))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    if ms is None:
        _lib.call("kv800_decode", ctypes.byref(s), _ptr(q), _ptr(cs), _ptr(sn), npos, B, spb, _ptr(out),
                  _ptr(ws), ws_bytes, _stream(dev))
    else:
        _lib.call("kv800_decode_timed", ctypes.byref(s), _ptr(q), _ptr(cs), _ptr(sn), npos, B, spb, _ptr(out),
                  _ptr(ws), ws_bytes, _stream(dev), ms)
    _check_status(ws[:4].view(torch.int32), dev, "decode")
    del keep
    return out


def combine(MO, LO, AO, ns, H=None):
    """Merge split partials (the reference's combine, kv800.py:231-236): MO / LO (B, ns + 1, 16), AO (B, ns + 1, 16,
    128) fp32; slots < ns are quantized (Hadamard domain), slot ns exact.  -> (B, 16, 128) bf16."""
    dev = _cuda(MO, "combine").device
    MO, LO, AO = (t.to(torch.float32).contiguous() for t in (MO, LO, AO))
    B = MO.shape[0]
    out = torch.empty(B, 16, 128, dtype=torch.bfloat16, device=dev)
    _lib.call("kv800_combine", _ptr(MO), _ptr(LO), _ptr(AO), B, int(ns), _ptr(out), _stream(dev))
    return out


# ---------------------------------------------------------------- harness store with the paged layout (kv800.py:387)
class PagedStore:
    """A cache for `batch` rows that all grow together, laid out like the vLLM pages (the reference's test and
    benchmark harness, kv800.py:387-441).  Each row's exact tokens live in a ring of `nring` pages of `ebs` tokens
    (vLLM's sliding window frees older pages the same way), its sub-blocks at fixed slots of `qpool`.  append() writes
    new tokens into the pages with the CUDA scatter kernel and, whenever a row's length reaches 256 j + 384, quantizes
    sub-block j from the pages with the CUDA flush kernel (one launch per 128-token slice of the appended tokens)."""

    def __init__(self, batch, max_len, device, window=0, ebs=64, nring=10):
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError(f"PagedStore: the 800h CUDA backend needs a cuda device, got {device}")
        self.B, self.win, self.dev, self.ebs, self.nring = batch, window, device, ebs, nring
        self.H = hadamard(128, device)
        nsub = 0 if window else max_len // BLK + 1
        self.qpool = torch.zeros(max(1, batch * nsub), SUB, dtype=torch.uint8, device=device)
        self.boff = (torch.arange(batch * max(nsub, 1), device=device, dtype=torch.int64) * SUB).view(batch, max(nsub, 1))
        # exact pages: [B * nring, 4 heads, ebs tokens, K 128 | V 128] bf16
        self.epool = torch.zeros(batch * nring, 4, ebs, 256, dtype=torch.bfloat16, device=device)
        npg = max_len // ebs + 2
        pg = torch.arange(npg, device=device) % nring
        self.eoff = ((torch.arange(batch, device=device)[:, None] * nring + pg[None]) * (4 * ebs * 256)).to(torch.int64)
        self.e_hs, self.e_ts, self.e_v = ebs * 256, 256, 128
        self.sk = torch.zeros(batch, NSINK, 4, 128, dtype=torch.bfloat16, device=device)
        self.sv = torch.zeros_like(self.sk)
        self.skoff = torch.arange(batch, device=device, dtype=torch.int64) * NSINK * 512
        self.N = torch.zeros(batch, dtype=torch.int32, device=device)
        self.NQ = torch.zeros_like(self.N)
        self.n, self.nq = 0, 0
        self._seq = torch.arange(batch, device=device, dtype=torch.int32)
        assert nring * ebs >= 512 + ebs

    def paged(self):
        return Paged(qpool=self.qpool, boff=self.boff, epool=self.epool, eoff=self.eoff, ebs=self.ebs,
                     e_hs=self.e_hs, e_ts=self.e_ts, e_v=self.e_v, sk=self.sk if self.win else None,
                     sv=self.sv if self.win else None, skoff=self.skoff, svoff=self.skoff, N=self.N, NQ=self.NQ,
                     nqmax=self.nq, win=self.win)

    def append(self, k, v):
        """k: pre-RoPE keys, v: values, (B, T, 4, 128)."""
        T = k.shape[1]
        for s in range(0, T, 128):
            kk = k[:, s:s + 128].to(device=self.dev, dtype=torch.bfloat16)
            vv = v[:, s:s + 128].to(device=self.dev, dtype=torch.bfloat16)
            t = kk.shape[1]
            pos = torch.arange(self.n, self.n + t, device=self.dev)
            write_exact(self.epool, self.eoff, self.ebs, self.e_hs, self.e_ts, self.e_v,
                        kk.reshape(-1, 4, 128), vv.reshape(-1, 4, 128),
                        self._seq.repeat_interleave(t), pos.repeat(self.B))
            if self.win and self.n < NSINK:
                m = pos < NSINK
                self.sk[:, pos[m]], self.sv[:, pos[m]] = kk[:, m], vv[:, m]
            self.n += t
            while not self.win and (self.n - LAG) // BLK > self.nq:
                flush(self.epool, self.eoff, self.ebs, self.e_hs, self.e_ts, self.e_v, self.qpool, self.boff,
                      self._seq, torch.full((self.B,), self.nq, dtype=torch.int32, device=self.dev))
                self.nq += 1
        self.N.fill_(self.n)
        self.NQ.fill_(self.nq)
