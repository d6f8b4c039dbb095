"""The CUDA quantizer / flush / dequantizer against the reference (golden fixtures made from the reference package)
and the CPU oracle: packed bytes bit-exact, dequantized K bit-exact, dequantized V bit-exact (the same FMA chain)."""
import numpy as np
import pytest
import torch

import inputs as I
from _util import nb, tb
from oracle import oracle as O

pytestmark = pytest.mark.gpu
QG = np.load(I.__file__.replace("inputs.py", "quant.npz"))
DG = np.load(I.__file__.replace("inputs.py", "decode.npz"))
DEV = "cuda"


@pytest.fixture(scope="module")
def kv800():
    from lfm3_kv800 import kv800 as m
    return m


@pytest.mark.parametrize("kind", I.QUANT_KINDS)
def test_quantize_blocks_matches_reference(kv800, kind):
    M = int(QG[f"{kind}_M"])
    k, v = I.quant_inputs(kind, M)
    out = kv800.quantize_blocks(tb(k, DEV), tb(v, DEV), kv800.hadamard(128, DEV)).cpu().numpy()
    if f"{kind}_bytes" in QG:
        ref = QG[f"{kind}_bytes"]
        bad = np.nonzero(out != ref)
        assert bad[0].size == 0, f"{bad[0].size} bytes differ, first at {bad[1][:8]}"
    assert [I.digest(out[m]) for m in range(M)] == list(QG[f"{kind}_sha"])


@pytest.mark.parametrize("kind,M", [("outlier", 37), ("wide", 9), ("normal", 64)])
def test_quantize_blocks_matches_oracle_many(kv800, kind, M):
    k, v = I.quant_inputs(kind, M, seed=5)
    out = kv800.quantize_blocks(tb(k, DEV), tb(v, DEV)).cpu().numpy()
    np.testing.assert_array_equal(out, O.quantize_blocks(k, v))


def test_dequantize_blocks_matches_reference(kv800):
    kd, vd = kv800.dequantize_blocks(torch.from_numpy(QG["outlier_bytes"]).to(DEV))
    assert I.digest(nb(kd)) == str(QG["outlier_deq_k_sha"])
    assert I.digest(vd.cpu().numpy()) == str(QG["outlier_deq_v_sha"])


def test_round_trip_idempotent(kv800):
    """quantize(dequantize(quantize(x))) keeps K codes of the dequantized keys: a size-independent property."""
    k, v = I.quant_inputs("normal", 8, seed=11)
    sb = kv800.quantize_blocks(tb(k, DEV), tb(v, DEV))
    kd, _ = kv800.dequantize_blocks(sb)
    sb2 = kv800.quantize_blocks(kd.contiguous(), tb(v, DEV))
    np.testing.assert_array_equal(sb2[:, :32768].cpu().numpy(), sb[:, :32768].cpu().numpy())


def _cuda_store(kv800, win, n, B=2):
    K, V, q = I.parity_inputs(win, n, B=B)
    st = kv800.PagedStore(B, n + 8, DEV, window=win)
    pre = max(1, n - 5)
    st.append(tb(K[:, :pre], DEV), tb(V[:, :pre], DEV))
    for i in range(pre, n):
        st.append(tb(K[:, i:i + 1], DEV), tb(V[:, i:i + 1], DEV))
    return st


@pytest.mark.parametrize("win,n", [c for c in I.parity_cases() if c[0] == 0])
def test_paged_flush_matches_reference(kv800, win, n):
    """PagedStore.append (CUDA page scatter + flush) gives the reference's pools byte for byte."""
    st = _cuda_store(kv800, win, n)
    key = f"w{win}_n{n}"
    assert st.nq == int(DG[f"{key}_nq"])
    assert I.digest(st.qpool.cpu().numpy()) == str(DG[f"{key}_qpool_sha"])
    assert I.digest(nb(st.epool)) == str(DG[f"{key}_epool_sha"])


def test_flush_scattered_tables(kv800):
    """Flush through shuffled page / sub-block tables, many sequences at once, against the oracle."""
    g = np.random.RandomState(3)
    B, nsub, ebs = 6, 3, 64
    npg = nsub * 256 // ebs
    K = I.f32_to_bf16(g.standard_normal((B, nsub * 256, 4, 128)).astype(np.float32) * 2)
    V = I.f32_to_bf16(g.standard_normal((B, nsub * 256, 4, 128)).astype(np.float32))
    pages = g.permutation(B * npg + 5)[:B * npg].reshape(B, npg)
    epool = np.zeros((B * npg + 5, 4, ebs, 256), np.uint16)
    for b in range(B):
        for p in range(nsub * 256):
            epool[pages[b, p // ebs], :, p % ebs, :128] = K[b, p]
            epool[pages[b, p // ebs], :, p % ebs, 128:] = V[b, p]
    eoff = (pages * 4 * ebs * 256).astype(np.int64)
    boff = (g.permutation(B * nsub + 2)[:B * nsub].reshape(B, nsub) * 51200).astype(np.int64)
    seq = np.repeat(np.arange(B), nsub).astype(np.int32)
    blk = np.tile(np.arange(nsub), B).astype(np.int32)
    qref = np.zeros((B * nsub + 2, 51200), np.uint8)
    O.flush(epool, eoff, ebs, ebs * 256, 256, 128, qref, boff, seq, blk)
    qp = torch.zeros(B * nsub + 2, 51200, dtype=torch.uint8, device=DEV)
    ep = tb(epool, DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    kv800.flush(ep, torch.from_numpy(eoff), ebs, ebs * 256, 256, 128, qp, torch.from_numpy(boff),
                torch.from_numpy(seq), torch.from_numpy(blk), status=status)
    assert int(status.item()) == 0
    np.testing.assert_array_equal(qp.cpu().numpy(), qref)


def test_flush_rejects_out_of_range_offsets(kv800):
    """A sub-block offset past the pool is skipped by the kernel's own range check and reported in the status word:
    the bad entry is never read or written (a host-made failure, no device fault)."""
    B, ebs = 1, 64
    ep = torch.zeros(10, 4, ebs, 256, dtype=torch.bfloat16, device=DEV)
    eoff = torch.arange(10, dtype=torch.int64).view(1, 10) * 4 * ebs * 256
    qp = torch.zeros(2, 51200, dtype=torch.uint8, device=DEV)
    boff = torch.tensor([[51200 * 2, 0]], dtype=torch.int64)          # sub-block 0 points one past the pool
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    kv800.flush(ep, eoff, ebs, ebs * 256, 256, 128, qp, boff, torch.tensor([0]), torch.tensor([0]), status=status)
    assert int(status.item()) & 1
    assert int(qp.sum().item()) == 0


def _stress_v(kind, M, rs):
    """V rows that probe the quantizer's fast-transform decisions: heavy tails, values far apart in scale, tiny
    (subnormal-range) values, near-constant rows, exact zeros and ties, and rows sitting on rounding boundaries."""
    shape = (M, 256, 4, 128)
    g = rs.standard_normal(shape)
    if kind == "heavy":
        v = g / (np.abs(rs.standard_normal(shape)) + 1e-3)
    elif kind == "scales":
        v = np.where(rs.random_sample(shape) < 0.05, 300.0 * g, 1e-3 * g)
    elif kind == "tiny":
        v = g * 1e-38
    elif kind == "flat":
        v = 1.0 + 1e-3 * g
    elif kind == "ties":
        v = np.round(g * 2) / 2                      # many exact ties and zeros
        v[:, ::7] = 0.0
    else:                                           # "grid": values on a coarse grid, rotated sums hit boundaries
        v = rs.randint(-3, 4, shape) * 0.0625
    return I.f32_to_bf16(np.clip(v, -3e38, 3e38).astype(np.float32))


@pytest.mark.parametrize("kind", ["heavy", "scales", "tiny", "flat", "ties", "grid"])
def test_quantizer_stress_matches_oracle(kv800, kind):
    """Bit-exact against the oracle (the reference's sequential FMA chain) on adversarial V rows: the quantizer takes
    its V decisions from a fast transform with a proven error bound and redoes undecided tokens with the chain."""
    rs = np.random.RandomState(hash(kind) % 2**31)
    M = 24
    k = I.f32_to_bf16(rs.standard_normal((M, 256, 4, 128)).astype(np.float32))
    v = _stress_v(kind, M, rs)
    got = kv800.quantize_blocks(tb(k, DEV), tb(v, DEV)).cpu().numpy()
    ref = O.quantize_blocks(k, v)
    bad = np.nonzero((got != ref).any(1))[0]
    assert bad.size == 0, f"{kind}: sub-blocks {bad[:8].tolist()} differ"


KLO_O, KSC_O = 50176, 50688


def test_fp8_bytes_match_torch_cast_on_every_bf16(kv800):
    """The device fp8 e4m3fn encoder against torch's own fp32 -> float8_e4m3fn cast (the cast of kv800.py:63-64) on
    every non-NaN bf16 value, infinities and magnitudes past 464 included.  Each value fills one K channel of one
    sub-block for all 256 tokens, so that channel's lo = hi = the value: its lo byte is the encoder's output for the
    value, and its scale byte the output for (hi - lo) / 3 clamped at 1e-8 (NaN for the infinities, compared without
    the NaN's sign, which is the platform's).  A second pass
    fills each channel with two random finite values (tokens 0..127 and 128..255) so the scale bytes also sweep fp32
    quotients that are not bf16 values."""
    bits = np.arange(65536, dtype=np.uint32)
    f = (bits << 16).view(np.float32)
    vals = bits[~np.isnan(f)].astype(np.uint16)
    n = vals.size
    M = -(-n // 512)
    ch = np.zeros(M * 512, dtype=np.uint16)
    ch[:n] = vals
    k = np.ascontiguousarray(np.broadcast_to(ch.reshape(M, 1, 4, 128), (M, 256, 4, 128)))
    v = np.zeros_like(k)
    out = kv800.quantize_blocks(tb(k, DEV), tb(v, DEV)).cpu().numpy()
    x = torch.from_numpy((ch.astype(np.uint32) << 16).view(np.float32))
    f8 = torch.float8_e4m3fn
    np.testing.assert_array_equal(out[:, KLO_O:KSC_O].reshape(-1), x.to(f8).view(torch.uint8).numpy())
    # the infinities' scale is inf - inf = NaN, whose sign is the platform's default NaN (positive on the GPU,
    # negative on x86, where torch runs here): NaN scale bytes are compared without the sign bit
    sc, ref_sc = out[:, KSC_O:].reshape(-1), ((x - x) / 3).clamp_min(1e-8).to(f8).view(torch.uint8).numpy()
    nan = (ref_sc & 0x7F) == 0x7F
    assert int(nan.sum()) == 2   # +inf and -inf
    np.testing.assert_array_equal(sc[~nan], ref_sc[~nan])
    np.testing.assert_array_equal(sc[nan] & 0x7F, ref_sc[nan] & 0x7F)
    # two values per channel: lo = min, hi = max, scale = (hi - lo) / 3
    rs = np.random.RandomState(17)
    M2 = 64
    a = I.f32_to_bf16((rs.standard_normal(M2 * 512) * np.exp(rs.uniform(-12, 6, M2 * 512))).astype(np.float32))
    b = I.f32_to_bf16((rs.standard_normal(M2 * 512) * np.exp(rs.uniform(-12, 6, M2 * 512))).astype(np.float32))
    k2 = np.empty((M2, 256, 4, 128), dtype=np.uint16)
    k2[:, :128] = a.reshape(M2, 1, 4, 128)
    k2[:, 128:] = b.reshape(M2, 1, 4, 128)
    out2 = kv800.quantize_blocks(tb(k2, DEV), tb(np.zeros_like(k2), DEV)).cpu().numpy()
    xa = torch.from_numpy((a.astype(np.uint32) << 16).view(np.float32))
    xb = torch.from_numpy((b.astype(np.uint32) << 16).view(np.float32))
    lo, hi = torch.minimum(xa, xb), torch.maximum(xa, xb)
    np.testing.assert_array_equal(out2[:, KLO_O:KSC_O].reshape(-1), lo.to(f8).view(torch.uint8).numpy())
    np.testing.assert_array_equal(out2[:, KSC_O:].reshape(-1),
                                  ((hi - lo) / 3).clamp_min(1e-8).to(f8).view(torch.uint8).numpy())


def test_fp8_decode_of_every_byte(kv800):
    """The device fp8 decoder on all 256 bytes: a sub-block whose K codes are 0 and scales 0 dequantizes to
    K = bf16(0 * 0 + lo) (kv800.py:84-86), compared with the same expression in torch on the float8_e4m3fn -> fp32
    decode of each byte (NaN bytes: NaN)."""
    sb = np.zeros((1, 51200), dtype=np.uint8)
    sb[0, KLO_O:KSC_O] = np.tile(np.arange(256, dtype=np.uint8), 2)
    kd, _ = kv800.dequantize_blocks(torch.from_numpy(sb).to(DEV))
    got = kd[0, 0].reshape(-1).float().cpu()
    lo = torch.from_numpy(np.tile(np.arange(256, dtype=np.uint8), 2)).view(torch.float8_e4m3fn).float()
    zero = torch.zeros_like(lo)
    ref = (zero * zero + lo).to(torch.bfloat16).float()   # the reference's codes * ksc + klo (-0 byte -> +0)
    nan = torch.isnan(ref)
    assert torch.equal(torch.isnan(got), nan)
    assert torch.equal(got[~nan].view(torch.int32), ref[~nan].view(torch.int32))
