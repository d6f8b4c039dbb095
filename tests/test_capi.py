"""The C-ABI library without a GPU: it loads, exports every entry point include/kv800_b200.h declares, and rejects
bad arguments on the host before any launch (no kernel runs in these tests)."""
import ctypes
import os
import re

import pytest

from lfm3_kv800 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kv800_b200.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"KV800_API\s+[\w\s\*]+?\b(kv800_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared()
    for n in ("kv800_quantize_blocks", "kv800_dequantize_blocks", "kv800_flush", "kv800_write_exact", "kv800_decode",
              "kv800_qdecode", "kv800_xdecode", "kv800_combine"):
        assert n in names


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for n in declared():
        assert hasattr(L, n), n
    assert set(declared()) <= set(_lib.SIGNATURES), "a declared entry point has no ctypes signature"


def test_abi_and_constants():
    L = _lib.lib()
    assert L.kv800_abi_version() == 1
    v = [ctypes.c_int64() for _ in range(5)]
    assert L.kv800_constants(*[ctypes.byref(x) for x in v]) == 0
    assert [x.value for x in v] == [256, 51200, 128, 4, 256]


def test_struct_layout_matches_header():
    # 23 eight-byte fields in the order of struct kv800_paged
    assert ctypes.sizeof(_lib.Paged) == 23 * 8
    src = open(HEADER).read()
    body = src[src.index("typedef struct kv800_paged"):src.index("} kv800_paged;")]
    fields = re.findall(r"\*?\s*(\w+)\s*[;,]", body.split("{", 1)[1])
    assert [f for f, _ in _lib.Paged._fields_] == fields


def test_host_argument_checks():
    L = _lib.lib()
    assert L.kv800_quantize_blocks(None, None, -1, None, None) == _lib.ERR_ARG
    assert b"negative" in L.kv800_last_error()
    assert L.kv800_quantize_blocks(None, None, 0, None, None) == _lib.OK          # empty: nothing to do
    assert L.kv800_quantize_blocks(None, None, 4, None, None) == _lib.ERR_ARG
    assert L.kv800_flush(None, 0, None, 1, 64, 0, 0, 0, None, 0, None, 1, None, None, -3, 1, None, None) == _lib.ERR_ARG
    assert L.kv800_decode(None, None, None, None, 1, 1, 0, None, None, 0, None) == _lib.ERR_ARG
    assert b"Paged" in L.kv800_last_error()
    P = _lib.Paged()
    assert L.kv800_decode(ctypes.byref(P), None, None, None, 1, 1, 0, None, None, 0, None) == _lib.ERR_ARG
    assert L.kv800_check_status(None, None, None) == _lib.ERR_ARG
    assert L.kv800_decode_timed(None, None, None, None, 1, 1, 0, None, None, 0, None, None) == _lib.ERR_ARG
    assert L.kv800_decode_timed(ctypes.byref(P), None, None, None, 1, 1, 0, None, None, 0, None, None) == _lib.ERR_ARG


def test_step_entry_argument_checks():
    """The vLLM-step entry points reject bad arguments on the host and treat empty work as a no-op."""
    L = _lib.lib()
    # write_slots: negative T, empty, null pointers
    assert L.kv800_write_slots(None, 0, 0, 0, 0, 64, None, None, None, -1, None, None) == _lib.ERR_ARG
    assert L.kv800_write_slots(None, 0, 0, 0, 0, 64, None, None, None, 0, None, None) == _lib.OK
    assert L.kv800_write_slots(None, 0, 0, 0, 0, 64, None, None, None, 5, None, None) == _lib.ERR_ARG
    # flush_step: workspace sizing, nothing to flush, bad bsq, short workspace
    assert L.kv800_flush_step_workspace_size(0) == 256
    assert L.kv800_flush_step_workspace_size(3) == 512
    assert L.kv800_flush_step_workspace_size(-1) == -1
    args = [None, 0, 0, 0, 0, 64, None, 1, None, 0, 262144, 1280, None, 1, None, None]
    assert L.kv800_flush_step(*args, 4, 0, None, 0, None, None) == _lib.OK
    assert L.kv800_flush_step(*args, 4, 2, None, 0, None, None) == _lib.ERR_ARG
    fake = ctypes.c_void_p(256)        # never dereferenced: every check below fails before a launch
    good = [fake, 0, 0, 0, 0, 64, fake, 1, fake, 0, 262144, 1280, fake, 1, fake, fake]
    bad_bsq = list(good)
    bad_bsq[11] = 1000
    assert L.kv800_flush_step(*bad_bsq, 4, 2, fake, 4096, None, None) == _lib.ERR_ARG
    assert L.kv800_flush_step(*good, 4, 2, fake, 16, None, None) == _lib.ERR_RANGE
    assert b"workspace" in L.kv800_last_error()
    # write_sinks / decode_tables / prefill_kv
    assert L.kv800_write_sinks(*[None, 0, 0, 0, None, 0] * 2, None, None, None, None, None, 2, -1, None, None) == _lib.ERR_ARG
    assert L.kv800_write_sinks(*[None, 0, 0, 0, None, 0] * 2, None, None, None, None, None, 2, 0, None, None) == _lib.OK
    tab = [None, 0, 0, 0, None] * 2
    assert L.kv800_decode_tables(None, 0, None, 0, 0, None, None, None, None, 0, 0, 0, 0, None, *tab, None) == _lib.OK
    assert L.kv800_decode_tables(None, 3, None, 0, 0, None, None, None, None, 0, 0, 0, 0, None, *tab, None) == _lib.ERR_ARG
    assert L.kv800_decode_tables(fake, 3, fake, 4, 0, fake, fake, fake, None, 0, 0, 1280, 5, fake, *tab,
                                 None) == _lib.ERR_ARG
    assert b"quant block table" in L.kv800_last_error()
    none_pf = [None, 0, 0, 0, None, 0]
    assert L.kv800_prefill_kv(*none_pf, 0, None, None, 5, *[None, 0, 0, 0, 0, 0, None, 0], 0, 0, None, None, 0,
                              None, None, 0, None, None, None, None) == _lib.ERR_ARG                  # ns > 4
    assert L.kv800_prefill_kv(*none_pf, 0, None, None, 0, *[None, 0, 0, 0, 0, 0, None, 0], 0, 0, None, None, 0,
                              None, None, 0, None, None, None, None) == _lib.OK                       # nothing
    assert L.kv800_prefill_kv(*none_pf, 2, None, None, 0, *[None, 0, 0, 0, 0, 0, None, 0], 0, 0, None, None, 0,
                              None, None, 0, fake, fake, None, None) == _lib.ERR_ARG                  # no quant cache


def _plan_bytes(B, nqmax, win, spb, G0=444):
    up = lambda x: (x + 255) & ~255
    nq = 0 if win else nqmax
    persistent = spb <= 0 and nq > 0
    ns = 0 if (nq == 0 or persistent) else -(-nq // spb)
    nx = 3 if win else 4                           # exact splits per row: 3 for window layers, 4 otherwise
    nslots = (G0 + B + nx * B) if persistent else B * (ns + nx)
    prefix = up(256 + 16 * B)                      # status word | arrival counters per (row, head)
    mo = up(prefix + ((B + 1) * 8 if persistent else 0))
    lo = up(mo + nslots * 64)
    ao = up(lo + nslots * 64)
    return up(ao + nslots * 16 * 128 * 4)


@pytest.mark.parametrize("B,nqmax,win,spb", [(64, 127, 0, 0), (4, 7, 0, 0), (64, 0, 256, 0), (2048, 127, 0, 0),
                                             (2, 19, 0, 3), (64, 127, 0, 7)])
def test_workspace_size(B, nqmax, win, spb):
    """Workspace plan: status word, arrival counters, schedule prefix (persistent), MO / LO / AO partials
    (no GPU: the persistent CTA count falls back to 3 x 148 when no device answers)."""
    L = _lib.lib()
    assert L.kv800_decode_workspace_size(B, nqmax, win, spb) == _plan_bytes(B, nqmax, win, spb)
