"""Multi-rank host logic of the data-parallel decode on CPU (world size 2, gloo): the shard assignment is balanced and
covers every row exactly once, max-over-ranks returns the slowest rank, and decoding each rank's shard (the CPU
oracle stands in for the per-GPU kernels) then gathering to rank 0 reproduces the full-batch decode exactly --
sequences are independent, so sharding needs no collective on the decode itself."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lfm3_kv800 import dp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_rows_balanced_and_complete():
    rs = np.random.RandomState(0)
    lengths = list(rs.randint(1024, 32769, 2048))
    world = 8
    shards = [dp.shard_rows(lengths, world, r) for r in range(world)]
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(len(lengths)))
    loads = [sum(dp.row_cost(lengths[i]) for i in s) for s in shards]
    assert max(loads) / min(loads) < 1.01


def _worker(rank, world, port, result):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "lfm3-kv800_b200"), root, os.path.join(root, "tests"),
                    os.path.join(root, "tests", "golden")]
    import inputs as I
    import test_ragged_gpu as R
    from lfm3_kv800 import dp as D
    from oracle import oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        lengths = [700, 3, 384, 1500, 0, 900, 260, 5000]
        P, q = R.build(lengths, 0, seed=9)                         # same global pools on every rank (seeded)
        cs, sn = I.rope_tables(5200)
        rows = D.shard_rows(lengths, world, rank)
        sub = dict(P, boff=P["boff"][rows], eoff=P["eoff"][rows], N=P["N"][rows], NQ=P["NQ"][rows],
                   skoff=P["skoff"][rows], svoff=P["svoff"][rows])
        # the bf16 bits as int16, the dtype the bench gathers; every collective of gather_rows must use a dtype
        # NCCL moves (it has no int16 / uint16)
        out = torch.from_numpy(O.decode(sub, q[rows], cs, sn, nthreads=2).view(np.int16))
        seen = []
        real = dist.all_gather
        def recording(outs, t, *args, **kw):
            seen.append(t.dtype)
            return real(outs, t, *args, **kw)
        dist.all_gather = recording
        try:
            full = D.gather_rows(out, rows, len(lengths))
        finally:
            dist.all_gather = real
        slowest = D.max_over_ranks(1.0 + rank)
        if rank == 0:
            ref = O.decode(P, q, cs, sn, nthreads=2).view(np.int16)
            result["equal"] = bool(full.dtype == torch.int16 and np.array_equal(full.numpy(), ref))
            result["dtypes"] = sorted({str(d) for d in seen})
            result["max"] = slowest
            result["rows0"] = rows
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_sharded_decode_gathers_to_full_batch():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, result)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(240)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        assert result["equal"], "gathered shards differ from the full-batch decode"
        assert set(result["dtypes"]) <= {"torch.uint8", "torch.int64"}, result["dtypes"]
        assert result["max"] == 2.0
        assert 0 < len(result["rows0"]) < 8
