"""Helpers shared by the GPU tests: bf16-bit numpy arrays <-> torch tensors, the parity metrics and tolerances."""
import numpy as np
import torch

# north-star tolerance of the decode output against the reference's torch_decode on the same inputs
REL_TOL, ABS_TOL = 1e-2, 2e-2


def tb(x, dev=None):
    """numpy bf16 bits (uint16) -> torch bf16 (optionally moved to dev)."""
    t = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).view(torch.bfloat16)
    return t if dev is None else t.to(dev)


def nb(t):
    """torch bf16 -> numpy bf16 bits."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def metrics(got_bits, ref_bits):
    g, r = f32(got_bits), f32(ref_bits)
    rel = float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30))
    return rel, float(np.abs(g - r).max())


def assert_parity(got_bits, ref_bits, what=""):
    rel, mx = metrics(got_bits, ref_bits)
    assert np.all(np.isfinite(f32(got_bits))), f"{what}: non-finite output"
    assert rel <= REL_TOL and mx <= ABS_TOL, f"{what}: rel {rel:.3e} (<= {REL_TOL}), max-abs {mx:.3e} (<= {ABS_TOL})"
    return rel, mx


def assert_parity_ulp(got_bits, ref_bits, what=""):
    """The decode bar with a one-bf16-ulp allowance: rel-L2 <= 1e-2, and per element |got - ref| <= max(2e-2, one
    bf16 ulp of |ref|).  Outputs whose magnitude reaches 4 have a bf16 ulp of 2^-5 or more, above the 2e-2 bar, and
    two correct fp32 implementations that sum in different orders can round such an element one ulp apart.  Synthetic
    cases whose outputs reach that range (1-bit V of a dominant token) use this form; the reference's own parity cases
    (outputs below 4) use the strict `assert_parity`."""
    g, r = f32(got_bits), f32(ref_bits)
    rel = float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30))
    ulp = np.ldexp(1.0, (np.floor(np.log2(np.maximum(np.abs(r), 1e-30))) - 7).astype(np.int64)).astype(np.float32)
    bound = np.maximum(np.float32(ABS_TOL), ulp)
    bad = np.abs(g - r) > bound
    assert np.all(np.isfinite(g)), f"{what}: non-finite output"
    assert rel <= REL_TOL and not bad.any(), (
        f"{what}: rel {rel:.3e}, {int(bad.sum())} elements beyond max(2e-2, 1 ulp); worst "
        f"{float(np.abs(g - r).max()):.3e}")
    return rel
