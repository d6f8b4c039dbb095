"""torch.ops.kv800: the reference's three native decode ops, registered for CUDA tensors and backed by this package's
C ABI (kv800_qdecode / kv800_xdecode / kv800_combine in libkv800_b200.so).

Same names, schema and argument meaning as the reference's op library (lfm3_kv800/csrc/kv800_sycl.sycl:554-566, the
ops that kv800_sycl.decode binds at kv800_sycl.py:94-112):

    kv800::qdecode(Tensor q, Tensor qp, Tensor boff, Tensor nq, Tensor cos, Tensor sin, Tensor(a!) mo,
                   Tensor(b!) lo, Tensor(c!) ao, int ns, int spb, float scale, int xmx) -> ()
    kv800::xdecode(Tensor q, Tensor ep, Tensor eoff, int ebs, int e_hs, int e_ts, int e_v, Tensor skp, Tensor svp,
                   Tensor skoff, Tensor svoff, Tensor n, Tensor nq, Tensor cos, Tensor sin, Tensor(a!) mo,
                   Tensor(b!) lo, Tensor(c!) ao, int ns, float scale, int win, int nsink) -> ()
    kv800::combine(Tensor mo, Tensor lo, Tensor ao, int ns) -> Tensor

Partials: MO / LO (B, ns + 1, 16) fp32, AO (B, ns + 1, 16, 128) fp32; slots [0, ns) hold the quantized splits of spb
sub-blocks each (V in the Hadamard domain), slot ns the sinks + exact tokens.  `xmx` selects the SYCL kernel variant
in the reference and is accepted and ignored here (one CUDA kernel).  Ops run on the current CUDA stream.  The
reference's kernels take any tensors; these check dtypes, shapes and devices first and raise ValueError, because a
wrong pointer on the GPU is a fault, not an exception.

register() is idempotent and runs when lfm3_kv800.kv800 is imported; ops() returns torch.ops.kv800 (the reference's
kv800_sycl.ops())."""
import ctypes

import torch

from . import _lib

SCHEMAS = {
    "qdecode": "qdecode(Tensor q, Tensor qp, Tensor boff, Tensor nq, Tensor cos, Tensor sin, Tensor(a!) mo, "
               "Tensor(b!) lo, Tensor(c!) ao, int ns, int spb, float scale, int xmx) -> ()",
    "xdecode": "xdecode(Tensor q, Tensor ep, Tensor eoff, int ebs, int e_hs, int e_ts, int e_v, Tensor skp, "
               "Tensor svp, Tensor skoff, Tensor svoff, Tensor n, Tensor nq, Tensor cos, Tensor sin, Tensor(a!) mo, "
               "Tensor(b!) lo, Tensor(c!) ao, int ns, float scale, int win, int nsink) -> ()",
    "combine": "combine(Tensor mo, Tensor lo, Tensor ao, int ns) -> Tensor",
}
_LIB = None


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _extent(t):
    return t.untyped_storage().nbytes() // t.element_size() - t.storage_offset()


def _stream(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _need(t, name, dtype, dim=None, contiguous=True):
    if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
        raise ValueError(f"kv800 op: {name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"kv800 op: {name} must be {dtype}, got {t.dtype}")
    if dim is not None and t.dim() != dim:
        raise ValueError(f"kv800 op: {name} must have {dim} dims, got {tuple(t.shape)}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"kv800 op: {name} must be contiguous")


def _partials(mo, lo, ao, B, ns):
    for t, name in ((mo, "mo"), (lo, "lo")):
        _need(t, name, torch.float32)
        if tuple(t.shape) != (B, ns + 1, 16):
            raise ValueError(f"kv800 op: {name} must be ({B}, {ns + 1}, 16), got {tuple(t.shape)}")
    _need(ao, "ao", torch.float32)
    if tuple(ao.shape) != (B, ns + 1, 16, 128):
        raise ValueError(f"kv800 op: ao must be ({B}, {ns + 1}, 16, 128), got {tuple(ao.shape)}")


def _tables(cos, sin):
    for t, name in ((cos, "cos"), (sin, "sin")):
        _need(t, name, torch.bfloat16, 2)
        if t.shape[1] != 32 or t.shape != cos.shape:
            raise ValueError(f"kv800 op: {name} must be (P, 32), got {tuple(t.shape)}")


def _q(q):
    _need(q, "q", torch.bfloat16, 3)
    if tuple(q.shape[1:]) != (16, 128):
        raise ValueError(f"kv800 op: q must be (B, 16, 128), got {tuple(q.shape)}")
    return q.shape[0]


def _qdecode(q, qp, boff, nq, cos, sin, mo, lo, ao, ns, spb, scale, xmx):
    """Quantized split partials: split s of row b covers sub-blocks [s spb, min((s + 1) spb, NQ[b]))
    (kv800_sycl.sycl:509-526; kv800.py:119-170)."""
    B = _q(q)
    if ns <= 0 or B == 0:
        return
    _need(qp, "qp", torch.uint8, contiguous=False)
    _need(boff, "boff", torch.int64, 2, contiguous=False)
    if boff.stride(1) != 1 or boff.shape[0] < B:
        raise ValueError("kv800 op: boff must be (B, >= ns * spb) with unit column stride")
    _need(nq, "nq", torch.int32, 1)
    _tables(cos, sin)
    _partials(mo, lo, ao, B, ns)
    _lib.call("kv800_qdecode", _p(q), _p(qp), _extent(qp), _p(boff), boff.stride(0), _p(nq), _p(cos), _p(sin),
              cos.shape[0], _p(mo), _p(lo), _p(ao), B, int(ns), int(spb), int(ns) * int(spb), float(scale), None,
              _stream(q))


def _xdecode(q, ep, eoff, ebs, e_hs, e_ts, e_v, skp, svp, skoff, svoff, n, nq, cos, sin, mo, lo, ao, ns, scale, win,
             nsink):
    """Sinks + exact tokens of each row into slot ns (kv800_sycl.sycl:528-541; kv800.py:173-228)."""
    B = _q(q)
    if B == 0:
        return
    _need(ep, "ep", torch.bfloat16, contiguous=False)
    _need(eoff, "eoff", torch.int64, 2, contiguous=False)
    if eoff.stride(1) != 1 or eoff.shape[0] < B:
        raise ValueError("kv800 op: eoff must be (B, pages) with unit column stride")
    _need(n, "n", torch.int32, 1)
    _need(nq, "nq", torch.int32, 1)
    _tables(cos, sin)
    _partials(mo, lo, ao, B, ns)
    s = _lib.Paged()
    s.epool, s.epool_elems = ep.data_ptr(), _extent(ep)
    s.eoff, s.eoff_stride = eoff.data_ptr(), eoff.stride(0)
    s.ebs, s.e_hs, s.e_ts, s.e_v = int(ebs), int(e_hs), int(e_ts), int(e_v)
    s.N, s.NQ = n.data_ptr(), nq.data_ptr()
    s.win, s.nqmax = int(win), 0
    keep = []
    if win and nsink:
        for t, name in ((skp, "skp"), (svp, "svp")):
            _need(t, name, torch.bfloat16, contiguous=False)
        sko, svo = skoff.to(torch.int64).contiguous(), svoff.to(torch.int64).contiguous()
        keep += [sko, svo]
        s.sk, s.sv, s.sk_elems, s.sv_elems = skp.data_ptr(), svp.data_ptr(), _extent(skp), _extent(svp)
        s.skoff, s.svoff, s.nsink = sko.data_ptr(), svo.data_ptr(), int(nsink)
    _lib.call("kv800_xdecode", _p(q), ctypes.byref(s), _p(cos), _p(sin), cos.shape[0], _p(mo), _p(lo), _p(ao), B,
              int(ns), float(scale), None, _stream(q))
    del keep


def _combine(mo, lo, ao, ns):
    """Log-sum-exp merge of the ns + 1 slots, Hadamard on the quantized part (kv800.py:231-236) -> (B, 16, 128)."""
    B = mo.shape[0]
    _partials(mo, lo, ao, B, ns)
    out = torch.empty(B, 16, 128, dtype=torch.bfloat16, device=mo.device)
    if B:
        _lib.call("kv800_combine", _p(mo), _p(lo), _p(ao), B, int(ns), _p(out), _stream(mo))
    return out


def register():
    """Define kv800::qdecode / xdecode / combine (if no library in this process has) and bind their CUDA kernels."""
    global _LIB
    if _LIB is not None:
        return
    lib = torch.library.Library("kv800", "FRAGMENT")
    for name, schema in SCHEMAS.items():
        try:
            lib.define(schema)
        except RuntimeError as e:                      # defined already (another build of the ops in this process)
            if "already" not in str(e) and "multiple times" not in str(e):
                raise
    lib.impl("qdecode", _qdecode, "CUDA")
    lib.impl("xdecode", _xdecode, "CUDA")
    lib.impl("combine", _combine, "CUDA")
    _LIB = lib


def ops():
    """torch.ops.kv800 with the CUDA kernels registered."""
    register()
    return torch.ops.kv800
