"""Generate the golden fixtures in this directory by running the REFERENCE package (riceharvest/lfm3-kv800 v0.1.1,
Python/torch) on the deterministic inputs of inputs.py.

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --ref <path of the reference checkout>

It needs the reference importable (its lfm3_kv800 package), so it runs only where the reference is mounted; the
fixtures it writes are committed and are all the tests need elsewhere.  What is recorded:
  quant.npz   kv800.quantize_blocks(k, v, H) (kv800.py:56-76) on every input kind of inputs.QUANT_KINDS: per-sub-block
              sha256 of the packed bytes, raw bytes for the 'outlier' and 'edge' kinds, and sha256 of
              kv800.dequantize_blocks (kv800.py:79-92) of the 'outlier' bytes
  decode.npz  the 12 cases of the reference parity test (tests/test_parity.py:17-18,80-96) driven through
              kv800.PagedStore.append (flush rule, kv800.py:421-441) and torch_decode.decode (torch_decode.py:27-80):
              the bf16 outputs, the sha256 of the quantized pool and the exact pool after the appends, and the error
              of the reference's own torch backend against the test's dense re-derivation
  fakequant.npz  train.fake_quant_k / fake_quant_v (train.py:82-100) on three input kinds: sha256 of the fp32
              outputs, the first 16 tokens raw for the 'outlier' kind"""
import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import inputs as I  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference checkout (contains lfm3_kv800/)")
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    import torch
    from lfm3_kv800 import kv800, torch_decode
    assert os.path.abspath(os.path.dirname(kv800.__file__)).startswith(os.path.abspath(a.ref)), kv800.__file__
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    def tb(x):                                           # bf16 bits (numpy uint16) -> torch bf16
        return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).view(torch.bfloat16)

    def nb(t):                                           # torch bf16 -> bf16 bits
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    H = kv800.hadamard(128)
    # ------------------------------------------------------------ quantizer
    q = {"kinds": np.array(I.QUANT_KINDS)}
    M = {"normal": 2, "outlier": 2, "parity": 2, "edge": 1, "wide": 2}
    for kind in I.QUANT_KINDS:
        k, v = I.quant_inputs(kind, M[kind])
        out = kv800.quantize_blocks(tb(k), tb(v), H).numpy()
        q[f"{kind}_M"] = np.int64(M[kind])
        q[f"{kind}_in_sha"] = np.array([I.digest(k), I.digest(v)])
        q[f"{kind}_sha"] = np.array([I.digest(out[m]) for m in range(out.shape[0])])
        if kind in ("outlier", "edge"):
            q[f"{kind}_bytes"] = out
        if kind == "outlier":
            kd, vd = kv800.dequantize_blocks(torch.from_numpy(out), H)
            q["outlier_deq_k_sha"] = np.array(I.digest(nb(kd)))
            q["outlier_deq_v_sha"] = np.array(I.digest(vd.numpy()))
        print(f"quant {kind}: M={M[kind]} ok", flush=True)
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **q)

    # ------------------------------------------------------------ decode parity cases
    cs, sn = I.rope_tables(8192)
    c32, s32 = tb(cs), tb(sn)
    d = {"cases": np.array(I.parity_cases(), dtype=np.int64), "tables_sha": np.array([I.digest(cs), I.digest(sn)])}
    # full 128-dim tables for the test's dense re-derivation (tests/test_parity.py:67-73, :45-64)
    c128 = torch.cat((c32.float(), torch.ones(8192, 32), c32.float(), torch.ones(8192, 32)), 1).bfloat16()
    s128 = torch.cat((s32.float(), torch.zeros(8192, 32), s32.float(), torch.zeros(8192, 32)), 1).bfloat16()
    sys.path.insert(0, os.path.join(a.ref, "tests"))
    import test_parity as tp
    for win, n in I.parity_cases():
        K, V, qq = I.parity_inputs(win, n)
        Kh, Vh, qt = tb(K), tb(V), tb(qq)
        st = kv800.PagedStore(2, n + 8, "cpu", window=win)
        pre = max(1, n - 5)
        st.append(Kh[:, :pre], Vh[:, :pre])
        for i in range(pre, n):
            st.append(Kh[:, i:i + 1], Vh[:, i:i + 1])
        o = torch_decode.decode(st.paged(), qt, c32, s32, st.H)
        r = tp.reference(qt, Kh, Vh, c128, s128, window=win)
        rel = ((o.float() - r).norm() / r.norm()).item()
        key = f"w{win}_n{n}"
        d[f"{key}_out"] = nb(o)
        d[f"{key}_qpool_sha"] = np.array(I.digest(st.qpool.numpy()))
        d[f"{key}_epool_sha"] = np.array(I.digest(nb(st.epool)))
        d[f"{key}_nq"] = np.int64(st.nq)
        d[f"{key}_rel_vs_dense"] = np.float64(rel)
        print(f"decode win={win} n={n}: nq={st.nq} rel(torch_decode vs dense)={rel:.3e}", flush=True)
    np.savez_compressed(os.path.join(HERE, "decode.npz"), **d)

    # ------------------------------------------------------------ training fake quant (train.py:82-100)
    from lfm3_kv800 import train as kt
    f = {}
    for kind in ("normal", "outlier", "edge"):
        k, v = I.quant_inputs(kind, 2, seed=3)
        kf = I.bf16_to_f32(k).reshape(2, 256, 512)        # groups of 256 tokens x 512 channels, as fq_k feeds it
        vf = I.bf16_to_f32(v)
        fk = kt.fake_quant_k(torch.from_numpy(kf.copy())).numpy()
        fv = kt.fake_quant_v(torch.from_numpy(vf.copy()), kt.hadamard(128)).numpy()
        f[f"{kind}_k_sha"] = np.array(I.digest(fk))
        f[f"{kind}_v_sha"] = np.array(I.digest(fv))
        if kind == "outlier":                             # a slice of raw values for readable diffs
            f["outlier_k16"] = fk[0, :16]
            f["outlier_v16"] = fv[0, :16]
        print(f"fake quant {kind} ok", flush=True)
    np.savez_compressed(os.path.join(HERE, "fakequant.npz"), **f)


if __name__ == "__main__":
    main()
