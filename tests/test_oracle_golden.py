"""The CPU oracle (oracle/) against the reference's own outputs recorded in tests/golden (made by make_golden.py from
the reference package): the quantizer and dequantizer bit-exact, the paged append + flush rule bit-exact on the pool
bytes, the decode within a couple of bf16 ulps.  Also the oracle's fp8 encoder against torch's cast over a dense
sweep.  CPU only."""
import numpy as np
import pytest
import torch

import inputs as I
from oracle import oracle as O

QG = np.load(I.__file__.replace("inputs.py", "quant.npz"))
DG = np.load(I.__file__.replace("inputs.py", "decode.npz"))


@pytest.mark.parametrize("kind", I.QUANT_KINDS)
def test_quantize_blocks_bit_exact(kind):
    M = int(QG[f"{kind}_M"])
    k, v = I.quant_inputs(kind, M)
    assert [I.digest(k), I.digest(v)] == list(QG[f"{kind}_in_sha"]), "input generator drifted"
    out = O.quantize_blocks(k, v)
    if f"{kind}_bytes" in QG:
        np.testing.assert_array_equal(out, QG[f"{kind}_bytes"])
    assert [I.digest(out[m]) for m in range(M)] == list(QG[f"{kind}_sha"])


def test_dequantize_blocks_bit_exact():
    kd, vd = O.dequantize_blocks(QG["outlier_bytes"])
    assert I.digest(kd) == str(QG["outlier_deq_k_sha"])
    assert I.digest(vd) == str(QG["outlier_deq_v_sha"])


def test_f8_encoder_matches_torch():
    """Dense sweep: every bf16-representable float, their midpoints and neighbours, the fp8 boundaries."""
    u = np.arange(1 << 16, dtype=np.uint32) << 16
    base = u.view(np.float32)
    mids = ((u | 0x8000).view(np.float32))
    rs = np.random.RandomState(7)
    rnd = rs.randint(0, 1 << 32, 1 << 20, dtype=np.uint64).astype(np.uint32).view(np.float32)
    edge = np.array([464.0, 448.0, 480.0, 2.0 ** -6, 2.0 ** -9, 2.0 ** -10, 1.5 * 2.0 ** -9, 0.0, -0.0, 1e-8,
                     np.inf, -np.inf, np.nan], np.float32)
    x = np.concatenate([base, mids, rnd, edge, np.nextafter(edge, np.float32(np.inf)),
                        np.nextafter(edge, np.float32(-np.inf))]).astype(np.float32)
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    got = O.f8_encode(x)
    nan_in = np.isnan(x)
    np.testing.assert_array_equal(got[~nan_in], want[~nan_in])
    assert np.all((got[nan_in] & 0x7F) == 0x7F)


def _store(win, n):
    K, V, q = I.parity_inputs(win, n)
    st = O.Store(2, n + 8, window=win)
    pre = max(1, n - 5)
    st.append(K[:, :pre], V[:, :pre])
    for i in range(pre, n):
        st.append(K[:, i:i + 1], V[:, i:i + 1])
    return st, q


@pytest.mark.parametrize("win,n", I.parity_cases())
def test_decode_matches_reference(win, n):
    cs, sn = I.rope_tables(8192)
    assert [I.digest(cs), I.digest(sn)] == list(DG["tables_sha"])
    st, q = _store(win, n)
    key = f"w{win}_n{n}"
    assert st.nq == int(DG[f"{key}_nq"])
    assert I.digest(st.qpool) == str(DG[f"{key}_qpool_sha"]), "flushed pool bytes differ from the reference"
    assert I.digest(st.epool) == str(DG[f"{key}_epool_sha"])
    o = I.bf16_to_f32(O.decode(st.paged(), q, cs, sn))
    r = I.bf16_to_f32(DG[f"{key}_out"])
    rel = np.linalg.norm(o - r) / np.linalg.norm(r)
    # the oracle sums in another order (quantized V rotated once per row): a bf16 ulp here and there
    assert rel < 1e-3, rel
    assert np.all(np.abs(o - r) <= 2.0 ** -6 * np.abs(r) + 1e-4)


@pytest.mark.parametrize("i", [0, 382, 383, 384, 638, 639, 1099])
def test_flush_rule(i):
    """Reference tests/test_train_hook.py:116-126: a query at index i (cache length i + 1) reads nq = max(0, i + 1 -
    128) // 256 sub-blocks quantized; the store flushes exactly those."""
    n = i + 1
    st = O.Store(1, n + 8)
    z = np.zeros((1, n, 4, 128), np.uint16)
    st.append(z, z)
    assert st.nq == max(0, n - 128) // 256


FG = np.load(I.__file__.replace("inputs.py", "fakequant.npz"))


@pytest.mark.parametrize("kind", ["normal", "outlier", "edge"])
def test_fake_quant_matches_reference(kind):
    """The training-side fake quant (train.py:82-100): K bit-exact, V bit-exact (same FMA chain as the CPU BLAS)."""
    k, v = I.quant_inputs(kind, 2, seed=3)
    fk = O.fake_quant_k(I.bf16_to_f32(k).reshape(2, 256, 512))
    fv = O.fake_quant_v(I.bf16_to_f32(v))
    if kind == "outlier":
        np.testing.assert_array_equal(fk[0, :16], FG["outlier_k16"])
        np.testing.assert_array_equal(fv[0, :16], FG["outlier_v16"])
    assert I.digest(fk) == str(FG[f"{kind}_k_sha"])
    assert I.digest(fv) == str(FG[f"{kind}_v_sha"])


def test_fake_quant_k_equals_cache_round_trip():
    """Reference tests/test_train_hook.py:92-106: the K fake quant equals dequantize(quantize(.)) of the cache."""
    k, v = I.quant_inputs("outlier", 3, seed=8)
    kd, vd = O.dequantize_blocks(O.quantize_blocks(k, v))
    fk = O.fake_quant_k(I.bf16_to_f32(k).reshape(3, 256, 512)).reshape(3, 256, 4, 128)
    np.testing.assert_array_equal(I.f32_to_bf16(fk), kd)
    fv = O.fake_quant_v(I.bf16_to_f32(v))
    np.testing.assert_allclose(fv, vd, atol=1e-5, rtol=0)
