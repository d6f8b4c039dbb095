"""CPU oracle for the 800h hot path -- TEST INFRASTRUCTURE ONLY.

numpy front end of oracle/kv800_oracle.c (a plain-C restatement of the reference's quantizer, dequantizer, paged
flush and torch decode).  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import
this module; it is the checker, never the thing measured or shipped.  The product package has no CPU path.

Reference anchors (riceharvest/lfm3-kv800 v0.1.1):
  quantize_blocks      lfm3_kv800/kv800.py:56-76
  dequantize_blocks    lfm3_kv800/kv800.py:79-92
  decode               lfm3_kv800/torch_decode.py:27-80
  Store                lfm3_kv800/kv800.py:387-441 (PagedStore: exact ring pages, flush rule n >= 256 j + 384)
  fake_quant_k / _v    lfm3_kv800/train.py:82-100
Parity of this oracle with the reference is pinned by the fixtures in tests/golden (made by make_golden.py, which
imports the reference)."""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkv800_oracle.so")

BLK, LAG, NSINK, WIN = 256, 128, 4, 256
SUB = 51200
KC_O, VB_O, VLO_O, VSC_O, KLO_O, KSC_O = 0, 32768, 49152, 49664, 50176, 50688

_lib = None
_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int


def build():
    """Compile the oracle with its Makefile (gcc only; no GPU needed)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.orc_f8_encode.restype = ctypes.c_uint8
        L.orc_f8_encode.argtypes = [ctypes.c_float]
        L.orc_f8_decode.restype = ctypes.c_float
        L.orc_f8_decode.argtypes = [ctypes.c_uint8]
        L.orc_quantize_blocks.argtypes = [_p, _p, _i64, _p, _int]
        L.orc_dequantize_blocks.argtypes = [_p, _i64, _p, _p, _p]
        L.orc_flush.argtypes = [_p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _i64, _p, _p, _i64, _int]
        L.orc_decode.argtypes = [_p, _p, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _i64,
                                 _i64, _p, _p, _p, _i64, _p, _int]
        L.orc_f8_encode_array.argtypes = [_p, _i64, _p]
        L.orc_fake_quant_k.argtypes = [_p, _i64, _i64, _p, _int]
        L.orc_fake_quant_v.argtypes = [_p, _i64, _p, _int]
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def threads():
    return os.cpu_count() or 1


# ---------------------------------------------------------------- formats
def f8_encode(x):
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint8)
    lib().orc_f8_encode_array(_ptr(x), x.size, _ptr(out))
    return out


def f8_decode(b):
    """fp8 e4m3fn bytes -> float32 (numpy restatement of the reference's integer decode, kv800.py:97-104)."""
    b = np.asarray(b, dtype=np.uint8).astype(np.uint32)
    e, m = (b >> 3) & 15, b & 7
    nrm = (((e + 120) << 23) | (m << 20)).astype(np.uint32).view(np.float32)
    mag = np.where(e == 0, m.astype(np.float32) * np.float32(0.001953125), nrm).astype(np.float32)
    mag = np.where((e == 15) & (m == 7), np.float32(np.nan), mag)
    return np.where(b & 0x80, -mag, mag).astype(np.float32)


def hadamard(n=128):
    H = np.ones((1, 1), np.float32)
    while H.shape[0] < n:
        H = np.block([[H, H], [H, -H]])
    return (H / np.float32(np.sqrt(np.float32(n)))).astype(np.float32)


# ---------------------------------------------------------------- quantizer
def quantize_blocks(k, v, nthreads=None):
    """k, v: (M, 256, 4, 128) bf16 bits -> (M, 51200) uint8 (kv800.py:56-76)."""
    k = _c(k, np.uint16)
    v = _c(v, np.uint16)
    M = k.shape[0]
    assert k.shape == (M, BLK, 4, 128) and v.shape == k.shape
    out = np.zeros((M, SUB), np.uint8)
    lib().orc_quantize_blocks(_ptr(k), _ptr(v), M, _ptr(out), nthreads or threads())
    return out


def dequantize_blocks(sb):
    """(M, 51200) uint8 -> K (M,256,4,128) bf16 bits, V (M,256,4,128) float32 (kv800.py:79-92)."""
    sb = _c(sb, np.uint8)
    M = sb.shape[0]
    k = np.empty((M, BLK, 4, 128), np.uint16)
    v = np.empty((M, BLK, 4, 128), np.float32)
    lib().orc_dequantize_blocks(_ptr(sb), M, _ptr(k), _ptr(v), None)
    return k, v


# ---------------------------------------------------------------- training fake quant (train.py:82-100)
def fake_quant_k(x, nthreads=None):
    """x (..., G, 256, C) float32 -> the 800h K quantize-dequantize round trip (float32), per 256-token group and
    channel."""
    x = _c(x, np.float32)
    C = x.shape[-1]
    G = x.size // (BLK * C)
    out = np.empty_like(x)
    lib().orc_fake_quant_k(_ptr(x), G, C, _ptr(out), nthreads or threads())
    return out


def fake_quant_v(v, nthreads=None):
    """v (..., 4, 128) float32 -> the 800h V round trip through the Hadamard domain (float32)."""
    v = _c(v, np.float32)
    out = np.empty_like(v)
    lib().orc_fake_quant_v(_ptr(v), v.size // 512, _ptr(out), nthreads or threads())
    return out


# ---------------------------------------------------------------- paged decode
def decode(P, q, cos_t, sin_t, nthreads=None):
    """P: dict with the reference's Paged slots as numpy arrays (qpool u8, boff int64 [B, *], epool bf16 bits, eoff
    int64 [B, *], ebs, e_hs, e_ts, e_v, sk / sv bf16 bits or None, skoff / svoff int64, N / NQ int32, nqmax, win);
    q (B, 16, 128) bf16 bits; cos_t / sin_t (P, 32) bf16 bits -> (B, 16, 128) bf16 bits (torch_decode.py:27-80)."""
    q = _c(q, np.uint16)
    B = q.shape[0]
    out = np.zeros((B, 16, 128), np.uint16)
    boff = _c(P["boff"], np.int64)
    eoff = _c(P["eoff"], np.int64)
    sk = None if P.get("sk") is None else _c(P["sk"], np.uint16)
    sv = None if P.get("sv") is None else _c(P["sv"], np.uint16)
    skoff = _c(P["skoff"], np.int64) if P.get("skoff") is not None else np.zeros(B, np.int64)
    svoff = _c(P["svoff"], np.int64) if P.get("svoff") is not None else np.zeros(B, np.int64)
    qpool, epool = _c(P["qpool"], np.uint8), _c(P["epool"], np.uint16)
    N, NQ = _c(P["N"], np.int32), _c(P["NQ"], np.int32)
    cs, sn = _c(cos_t, np.uint16), _c(sin_t, np.uint16)
    lib().orc_decode(_ptr(qpool), _ptr(boff), boff.shape[1] if boff.ndim == 2 else 1, _ptr(epool), _ptr(eoff),
                     eoff.shape[1] if eoff.ndim == 2 else 1, int(P["ebs"]), int(P["e_hs"]), int(P["e_ts"]),
                     int(P["e_v"]), _ptr(sk), _ptr(sv), _ptr(skoff), _ptr(svoff), _ptr(N), _ptr(NQ),
                     int(P.get("nqmax") or 0), int(P.get("win") or 0), _ptr(q), _ptr(cs), _ptr(sn), B, _ptr(out),
                     nthreads or threads())
    return out


def flush(epool, eoff, ebs, e_hs, e_ts, e_v, qpool, boff, seq, blk, nthreads=None):
    """Quantize the listed (sequence, sub-block) pairs from the exact pages into qpool (in place)."""
    eoff, boff = _c(eoff, np.int64), _c(boff, np.int64)
    seq, blk = _c(seq, np.int32), _c(blk, np.int32)
    assert epool.flags.c_contiguous and qpool.flags.c_contiguous
    lib().orc_flush(_ptr(epool), _ptr(eoff), eoff.shape[1], ebs, e_hs, e_ts, e_v, _ptr(qpool), _ptr(boff),
                    boff.shape[1], _ptr(seq), _ptr(blk), len(seq), nthreads or threads())


# ---------------------------------------------------------------- paged store (kv800.py:387-441)
class Store:
    """numpy mirror of the reference's PagedStore: `batch` equal-length sequences, exact pages in a ring of `nring`
    pages of `ebs` tokens per sequence, quantized sub-blocks at BOFF, sinks for window layers; the same flush rule."""

    def __init__(self, batch, max_len, window=0, ebs=64, nring=10):
        self.B, self.win, self.ebs, self.nring = batch, window, ebs, nring
        nsub = 0 if window else max_len // BLK + 1
        self.qpool = np.zeros((max(1, batch * nsub), SUB), np.uint8)
        self.boff = (np.arange(batch * max(nsub, 1), dtype=np.int64) * SUB).reshape(batch, max(nsub, 1))
        self.epool = np.zeros((batch * nring, 4, ebs, 256), np.uint16)
        npg = max_len // ebs + 2
        pg = np.arange(npg) % nring
        self.eoff = ((np.arange(batch)[:, None] * nring + pg[None]) * (4 * ebs * 256)).astype(np.int64)
        self.e_hs, self.e_ts, self.e_v = ebs * 256, 256, 128
        self.sk = np.zeros((batch, NSINK, 4, 128), np.uint16)
        self.sv = np.zeros_like(self.sk)
        self.skoff = np.arange(batch, dtype=np.int64) * NSINK * 512
        self.n = self.nq = 0
        assert nring * ebs >= 512 + ebs

    def _rows(self, pos):
        """element offsets (B, len(pos), 4) of the K rows of positions `pos` for each head."""
        pg = self.eoff[:, pos // self.ebs]
        return pg[..., None] + np.arange(4) * self.e_hs + (pos % self.ebs)[None, :, None] * self.e_ts

    def append(self, k, v):
        """k: pre-RoPE keys, v: values, (B, T, 4, 128) bf16 bits."""
        T = k.shape[1]
        ef = self.epool.reshape(-1)
        for s in range(0, T, 128):
            kk, vv = k[:, s:s + 128], v[:, s:s + 128]
            t = kk.shape[1]
            pos = np.arange(self.n, self.n + t)
            idx = self._rows(pos)[..., None] + np.arange(128)
            ef[idx] = kk
            ef[idx + self.e_v] = vv
            if self.win and self.n < NSINK:
                m = pos < NSINK
                self.sk[:, pos[m]] = kk[:, m]
                self.sv[:, pos[m]] = vv[:, m]
            self.n += t
            while not self.win and (self.n - LAG) // BLK > self.nq:
                j = self.nq
                flush(self.epool, self.eoff, self.ebs, self.e_hs, self.e_ts, self.e_v, self.qpool, self.boff,
                      np.arange(self.B), np.full(self.B, j))
                self.nq += 1

    def paged(self):
        B = self.B
        return dict(qpool=self.qpool, boff=self.boff, epool=self.epool, eoff=self.eoff, ebs=self.ebs, e_hs=self.e_hs,
                    e_ts=self.e_ts, e_v=self.e_v, sk=self.sk if self.win else None, sv=self.sv if self.win else None,
                    skoff=self.skoff, svoff=self.skoff, N=np.full(B, self.n, np.int32),
                    NQ=np.full(B, self.nq, np.int32), nqmax=self.nq, win=self.win)
