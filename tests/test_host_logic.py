"""Host-side logic of the package without a GPU: the backend surface keeps the reference's names and error
behaviour (kv800.py:251-349) with a single 'cuda' backend, and nothing silently runs on the CPU."""
import numpy as np
import pytest
import torch

from lfm3_kv800 import kv800
from oracle import oracle as O


def test_constants_match_reference_layout():
    assert (kv800.BLK, kv800.LAG, kv800.NSINK, kv800.WIN, kv800.SUB) == (256, 128, 4, 256, 51200)
    assert (kv800.KC_O, kv800.VB_O, kv800.VLO_O, kv800.VSC_O, kv800.KLO_O, kv800.KSC_O) == (
        0, 32768, 49152, 49664, 50176, 50688)
    assert kv800.F8 is torch.float8_e4m3fn
    assert kv800.BACKENDS == ("cuda",)


def test_hadamard_and_flat():
    H = kv800.hadamard(128)
    np.testing.assert_array_equal(H.numpy(), O.hadamard(128))
    assert torch.allclose(H @ H.T, torch.eye(128), atol=1e-6)
    base = torch.arange(100, dtype=torch.float32)
    v = base[10:20]
    f = kv800.flat(v)
    assert f.shape == (90,) and f[0] == 10 and f.data_ptr() == v.data_ptr()


def test_backend_selection_names():
    try:
        kv800.set_backend("cuda")
        kv800.set_backend("auto")
        kv800.set_backend(None)
        for bad in ("triton", "sycl", "torch", "nope"):
            with pytest.raises(ValueError):
                kv800.set_backend(bad)
    finally:
        kv800.set_backend(None)
    ok, why = kv800._available("cuda", "cpu")
    assert not ok and "cuda devices only" in why
    ok, why = kv800._available("triton", "cuda")
    assert not ok


def test_env_backend(monkeypatch):
    monkeypatch.setenv("LFM3KV_BACKEND", "triton")
    with pytest.raises(ValueError):          # set_backend(None) re-reads the env, as in the reference
        kv800.set_backend(None)
    with pytest.raises(ValueError):
        kv800._requested()
    monkeypatch.setenv("LFM3KV_BACKEND", "cuda")
    assert kv800._requested() == "cuda"


def test_no_cpu_path():
    """Every product entry point refuses CPU tensors instead of computing on the host."""
    k = torch.zeros(1, 256, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        kv800.quantize_blocks(k, k, kv800.hadamard())
    with pytest.raises(RuntimeError, match="CUDA"):
        kv800.dequantize_blocks(torch.zeros(1, 51200, dtype=torch.uint8))
    with pytest.raises(RuntimeError, match="cuda"):
        kv800.PagedStore(1, 300, "cpu")
    P = kv800.Paged(qpool=torch.zeros(1, 51200, dtype=torch.uint8), boff=torch.zeros(1, 1, dtype=torch.int64),
                    epool=torch.zeros(10, 4, 64, 256, dtype=torch.bfloat16), eoff=torch.zeros(1, 8, dtype=torch.int64),
                    ebs=64, e_hs=64 * 256, e_ts=256, e_v=128, N=torch.ones(1, dtype=torch.int32),
                    NQ=torch.zeros(1, dtype=torch.int32), nqmax=0, win=0)
    q = torch.zeros(1, 16, 128, dtype=torch.bfloat16)
    cs = torch.ones(16, 32, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        kv800.decode(P, q, cs, cs, kv800.hadamard())


def test_paged_slots():
    P = kv800.Paged(win=256, nqmax=3)
    assert P.win == 256 and P.nqmax == 3 and P.sk is None
    assert set(kv800.Paged.__slots__) == {"qpool", "boff", "epool", "eoff", "ebs", "e_hs", "e_ts", "e_v", "sk", "sv",
                                          "skoff", "svoff", "N", "NQ", "nqmax", "win"}


def test_vllm_step_host_values():
    """Host values of a vLLM step come from the CPU copies of the metadata: the flushed sub-block count (the flush
    rule n >= 256 j + 384 between the lengths before and after the step) and the positions of the scheduled tokens."""
    import torch
    from lfm3_kv800 import vllm_step as S
    assert [S.nq_of(n) for n in (0, 383, 384, 639, 640, 1151, 1152)] == [0, 0, 1, 1, 2, 3, 4]
    sl = torch.tensor([1151, 384, 2000, 5], dtype=torch.int32)
    qsl = torch.tensor([0, 1, 2, 2002, 2007], dtype=torch.int32)    # decodes, a 2000-token prefill, a 5-token prefill
    # prev = 1150, 383, 0, 0 -> flushes 3-3, 1-0, 7-0, 0
    assert S.flush_pairs(sl, qsl) == 0 + 1 + 7 + 0
    m = S.build_meta(torch.zeros(4, 16, dtype=torch.int32), torch.arange(2007), sl, qsl, sl, qsl)
    assert m.num_decodes == 2 and m.num_reqs == 4 and m.num_actual_tokens == 2007
    pos = m.positions.numpy()
    assert pos[0] == 1150 and pos[1] == 383 and list(pos[2:5]) == [0, 1, 2] and pos[2001] == 1999
    assert list(pos[2002:]) == [0, 1, 2, 3, 4]
    qv = torch.zeros(3 * S.QPAGE, dtype=torch.uint8)
    view = torch.as_strided(qv, (3, 2, S.QBLOCK, 4, S.QCONTENT), (S.QPAGE, 128000, 100, 25, 1))
    assert S.aux_offset(view) == 5 * 25600                              # bf16 elements: after 5 sub-blocks
    flat, ps = S.bf16_flat(view[1:])
    assert ps == S.QPAGE // 2 and flat.numel() == 2 * S.QPAGE // 2 and flat.dtype == torch.bfloat16


def test_bench_stdout_stays_one_json_line():
    """bench.py points file descriptor 1 at stderr while NCCL creates its communicator (NCCL prints its version banner
    to stdout): output written to fd 1 inside the guard, even by native code, lands on stderr, and stdout is back
    afterwards for the JSON line."""
    import os
    import subprocess
    import sys
    code = ("import os, sys; sys.path.insert(0, sys.argv[1]); import bench; "
            "bench.stdout_to_stderr(lambda: os.write(1, b'NCCL version banner\\n')); print('{\"metric\": 1}')")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code, root], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout == '{"metric": 1}\n'
    assert "NCCL version banner" in r.stderr
