"""Benchmark of the 800h hot path on B200: paged GQA decode over the 800h cache at 64 sequences x 32,768 tokens per GPU,
all 6 attention layers of the LFM3-1.7B shape (4 quantized layers: 127 sub-blocks + a 256-token exact tail; 2 window
layers: 4 sinks + 256 exact tokens), one decode query per sequence per layer (the metric's
config).  Sub-blocks and exact pages sit at a seeded random permutation of pool slots.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cuda|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

A step = the decode of all 6 layers for the rank's 64 sequences (one token per sequence).  `value` = sequences x
steps x ranks / max-over-ranks device time (tok/s, weak scaling: 64 sequences per GPU).  `e2e` = the same metric
through the public API with the step's inputs (6 x q, the current token's K / V) copied from pinned host memory, the
current token written into its exact page, and the 6 outputs read back, all inside the timed region (the copies on a
second stream, overlapped with the neighbouring layers' decode).  `roofline` =
the quantized-split kernel (the dominant one) timed alone with CUDA events: algorithmic bytes (51,200 per sub-block)
/ duration against the measured HBM copy bandwidth.  `cpu_baseline` = the CPU oracle (a C port of the reference's
torch decode, OpenMP over (sequence, kv head)) on the 64 sequences, all 6 layers, on this host's cores.
--workload ragged: BASELINE config 4 instead (2,048 ragged rows sharded over the ranks, strong scaling).

--impl reference: the reference's CPU path for this step (the oracle port, all host threads) on a bounded sample of
the same workload, printed as the reference arm's line; on N > 1 ranks only rank 0 runs it."""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "lfm3-kv800_b200"), ROOT, os.path.join(ROOT, "tests", "golden")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "800h paged-decode tok/s and HBM GB/s (vs 8 TB/s) at 64x32K ctx, 1/2/4/8 B200"
B_PER_GPU, N_CTX = 64, 32768
QUANT_LAYERS, WINDOW_LAYERS = 4, 2
EBS, NSINK, WIN, SUB = 64, 4, 256, 51200
FALLBACK_HBM_GBS = 6650.0


def stdout_to_stderr(fn):
    """Run fn with file descriptor 1 pointed at stderr.  NCCL writes to stdout while it creates a communicator (its
    version banner, at NCCL_DEBUG=WARN or above), and the bench's stdout must be its one JSON line."""
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        return fn()
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------- workload (one rank)
class Layer:
    """One attention layer's 800h cache for B sequences of n tokens, pages at random pool slots."""

    def __init__(self, kv800, torch, dev, B, n, win, gen, chunk=512):
        self.win = win
        self.B, self.n = B, n
        nq = 0 if win else max(0, n - 128) // 256
        self.nq = nq
        lo = nq * 256 if not win else max(0, n - win)
        self.exact = n - lo
        npg_row = n // EBS + 1
        first_pg, last_pg = lo // EBS, (n - 1) // EBS
        pages_per_seq = last_pg - first_pg + 1
        npages = B * pages_per_seq
        perm = torch.randperm(npages + 3, generator=gen)[:npages].view(B, pages_per_seq)
        self.eoff = torch.zeros(B, npg_row, dtype=torch.int64)
        self.eoff[:, first_pg:last_pg + 1] = perm * (4 * EBS * 256)
        self.eoff = self.eoff.to(dev)
        self.epool = torch.zeros(npages + 3, 4, EBS, 256, dtype=torch.bfloat16, device=dev)
        # exact tokens [lo, n): written through the library's page scatter
        seq = torch.arange(B, dtype=torch.int32).repeat_interleave(n - lo).to(dev)
        pos = torch.arange(lo, n, dtype=torch.int64).repeat(B).to(dev)
        kk = torch.randn(B * (n - lo), 4, 128, device=dev).to(torch.bfloat16)
        vv = torch.randn(B * (n - lo), 4, 128, device=dev).to(torch.bfloat16)
        kv800.write_exact(self.epool, self.eoff, EBS, EBS * 256, 256, 128, kk, vv, seq, pos)
        if nq:
            nslot = B * nq + 7
            slots = torch.randperm(nslot, generator=gen)[:B * nq].view(B, nq)
            self.boff = (slots * SUB).to(torch.int64).to(dev)
            self.qpool = torch.empty(nslot, SUB, dtype=torch.uint8, device=dev)
            flat_slots = slots.reshape(-1).to(dev)
            for c0 in range(0, B * nq, chunk):
                c1 = min(c0 + chunk, B * nq)
                k = torch.randn(c1 - c0, 256, 4, 128, device=dev).to(torch.bfloat16)
                v = torch.randn(c1 - c0, 256, 4, 128, device=dev).to(torch.bfloat16)
                self.qpool[flat_slots[c0:c1]] = kv800.quantize_blocks(k, v)
        else:
            self.qpool = torch.zeros(1, SUB, dtype=torch.uint8, device=dev)
            self.boff = torch.zeros(B, 1, dtype=torch.int64, device=dev)
        if win:
            self.sk = torch.randn(B, NSINK, 4, 128, device=dev).to(torch.bfloat16)
            self.sv = torch.randn(B, NSINK, 4, 128, device=dev).to(torch.bfloat16)
            self.skoff = (torch.arange(B, dtype=torch.int64) * NSINK * 512).to(dev)
        else:
            self.sk = self.sv = self.skoff = None
        self.N = torch.full((B,), n, dtype=torch.int32, device=dev)
        self.NQ = torch.full((B,), nq, dtype=torch.int32, device=dev)
        self.P = kv800.Paged(qpool=self.qpool, boff=self.boff, epool=self.epool, eoff=self.eoff, ebs=EBS,
                             e_hs=EBS * 256, e_ts=256, e_v=128, sk=self.sk, sv=self.sv, skoff=self.skoff,
                             svoff=self.skoff, N=self.N, NQ=self.NQ, nqmax=nq, win=win)

    def algo_bytes(self):
        """Cache bytes one decode of this layer must read (the reference's formula, nvidia/check_nvidia.py:563)."""
        ex = self.exact + (NSINK if self.win else 0)
        return self.B * (self.nq * 256 * 200 + ex * 2048)


def build_workload(kv800, torch, dev, rank, B=B_PER_GPU, n=N_CTX):
    import inputs as I
    gen = torch.Generator().manual_seed(1234 + rank)
    torch.manual_seed(1234 + rank)
    layers = [Layer(kv800, torch, dev, B, n, 0, gen) for _ in range(QUANT_LAYERS)]
    layers += [Layer(kv800, torch, dev, B, n, WIN, gen) for _ in range(WINDOW_LAYERS)]
    cs, sn = I.rope_tables(n + 64)
    c32 = torch.from_numpy(cs.view(np.int16)).view(torch.bfloat16).to(dev)
    s32 = torch.from_numpy(sn.view(np.int16)).view(torch.bfloat16).to(dev)
    qs = [torch.randn(B, 16, 128, device=dev).to(torch.bfloat16) for _ in layers]
    return layers, qs, c32, s32


# ---------------------------------------------------------------- config 4: ragged rows in a big pool
RAGGED_ROWS, RAGGED_LO, RAGGED_HI = 2048, 1024, 32768


class RaggedLayer:
    """One layer's 800h cache for rows of different lengths: sub-blocks at distinct random slots
    of a shared pool (a view into a buffer of --pool-gb), exact pages at random slots of the layer's page pool.
    Sub-block contents come from a pool of `uniq` distinct quantized sub-blocks (the decode's cost does not depend on
    the values)."""

    def __init__(self, kv800, torch, dev, lengths, win, gen, pool, slots, uniq):
        self.win, self.B = win, len(lengths)
        N = torch.tensor(lengths, dtype=torch.int64)
        nq = torch.zeros_like(N) if win else torch.clamp(N - 128, min=0) // 256
        lo = torch.clamp(N - win, min=0) if win else nq * 256
        self.nqmax = int(nq.max())
        self.lengths, self.nq_rows = lengths, nq.tolist()
        self.exact_rows = (N - lo).tolist()
        # exact pages: rows' pages [lo // EBS, (n - 1) // EBS] at random slots
        first, last = lo // EBS, (N - 1) // EBS
        cnt = (last - first + 1).clamp(min=0)
        npages = int(cnt.sum())
        perm = torch.randperm(npages + 3, generator=gen)[:npages]
        npg_row = int(N.max()) // EBS + 1
        self.eoff = torch.zeros(self.B, npg_row, dtype=torch.int64)
        o = 0
        for b in range(self.B):
            c = int(cnt[b])
            self.eoff[b, int(first[b]):int(first[b]) + c] = perm[o:o + c] * (4 * EBS * 256)
            o += c
        self.eoff = self.eoff.to(dev)
        self.epool = torch.randn(npages + 3, 4, EBS, 256, device=dev).to(torch.bfloat16)
        if not win:
            self.qpool = pool
            self.boff = torch.zeros(self.B, max(1, self.nqmax), dtype=torch.int64)
            o = 0
            for b in range(self.B):
                k = int(nq[b])
                self.boff[b, :k] = slots[o:o + k] * SUB
                o += k
            self.boff = self.boff.to(dev)
            pick = torch.randint(0, uniq.shape[0], (o,), generator=gen).to(dev)
            pool.view(-1, SUB)[slots[:o].to(dev)] = uniq[pick]
            self.used = o
        else:
            self.qpool = torch.zeros(1, SUB, dtype=torch.uint8, device=dev)
            self.boff = torch.zeros(self.B, 1, dtype=torch.int64, device=dev)
            self.used = 0
        if win:
            self.sk = torch.randn(self.B, NSINK, 4, 128, device=dev).to(torch.bfloat16)
            self.sv = torch.randn(self.B, NSINK, 4, 128, device=dev).to(torch.bfloat16)
            self.skoff = (torch.arange(self.B, dtype=torch.int64) * NSINK * 512).to(dev)
        else:
            self.sk = self.sv = self.skoff = None
        self.N = N.to(torch.int32).to(dev)
        self.NQ = nq.to(torch.int32).to(dev)
        self.P = kv800.Paged(qpool=self.qpool, boff=self.boff, epool=self.epool, eoff=self.eoff, ebs=EBS,
                             e_hs=EBS * 256, e_ts=256, e_v=128, sk=self.sk, sv=self.sv, skoff=self.skoff,
                             svoff=self.skoff, N=self.N, NQ=self.NQ, nqmax=self.nqmax, win=win)

    def algo_bytes(self):
        return sum(q * 256 * 200 + (e + (NSINK if self.win else 0)) * 2048
                   for q, e in zip(self.nq_rows, self.exact_rows))


def build_ragged(kv800, torch, dev, rank, world, pool_gb):
    """Config 4: 2,048 rows with lengths ~ U[1024, 32768] (seeded, the same on every rank), sharded over the ranks by
    longest-processing-time on their read bytes; this rank's rows in 4 quantized + 2 window layers.  The quantized
    layers' sub-blocks are scattered over one pool of pool_gb GB."""
    from lfm3_kv800 import dp
    rs = np.random.RandomState(2048)
    lengths_all = rs.randint(RAGGED_LO, RAGGED_HI + 1, RAGGED_ROWS).tolist()
    rows = dp.shard_rows(lengths_all, world, rank)
    lengths = [lengths_all[i] for i in rows]
    gen = torch.Generator().manual_seed(4321 + rank)
    nsub = sum(max(0, n - 128) // 256 for n in lengths) * QUANT_LAYERS
    # exact pages of 6 layers (<= 8 pages of 32 KB x 4 heads per row) and their fp32 staging, then the pool in what is
    # left of the GPU's free memory minus 8 GB
    exact_bytes = 6 * len(lengths) * 8 * 4 * EBS * 256 * 2 * 3
    free = torch.cuda.mem_get_info(dev)[0]
    pool_bytes = min(int(pool_gb * 1e9), free - exact_bytes - int(8e9)) // SUB * SUB
    pool_bytes = max(pool_bytes, (nsub + 16) * SUB)
    pool = torch.empty(pool_bytes, dtype=torch.uint8, device=dev)
    slots = torch.randperm(pool_bytes // SUB, generator=gen)[:nsub]
    k = torch.randn(256, 256, 4, 128, device=dev).to(torch.bfloat16)
    v = torch.randn(256, 256, 4, 128, device=dev).to(torch.bfloat16)
    uniq = kv800.quantize_blocks(k, v)
    layers, o = [], 0
    for li in range(QUANT_LAYERS + WINDOW_LAYERS):
        win = 0 if li < QUANT_LAYERS else WIN
        L = RaggedLayer(kv800, torch, dev, lengths, win, gen, pool, slots[o:], uniq)
        o += L.used
        layers.append(L)
    qs = [torch.randn(len(lengths), 16, 128, device=dev).to(torch.bfloat16) for _ in layers]
    import inputs as I
    cs, sn = I.rope_tables(RAGGED_HI + 64)
    c32 = torch.from_numpy(cs.view(np.int16)).view(torch.bfloat16).to(dev)
    s32 = torch.from_numpy(sn.view(np.int16)).view(torch.bfloat16).to(dev)
    return layers, qs, c32, s32, rows, pool_bytes


# ---------------------------------------------------------------- clocks sampled during the timed region
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx, self.proc, self.path = gpu_index, None, None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:  # noqa: BLE001
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except Exception:  # noqa: BLE001
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return None
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- CPU oracle on a bounded sample
def cpu_sample(layers, qs, c32, s32, S, reps=1):
    """Time the oracle (C port of the reference decode) on sequences [0, S) of every layer; -> (tok/s, sec/step)."""
    from oracle import oracle as O

    def nb(t):
        import torch
        return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)

    cs, sn = nb(c32), nb(s32)
    per_layer = []
    for L, q in zip(layers, qs):
        if L.nq:
            rows = L.boff[:S].cpu().numpy()
            qpool = L.qpool[(L.boff[:S] // SUB).reshape(-1)].cpu().numpy()
            boff = (np.arange(S * L.nq, dtype=np.int64) * SUB).reshape(S, L.nq)
            del rows
        else:
            qpool, boff = np.zeros((1, SUB), np.uint8), np.zeros((S, 1), np.int64)
        P = dict(qpool=qpool, boff=boff, epool=nb(L.epool), eoff=L.eoff[:S].cpu().numpy(), ebs=EBS, e_hs=EBS * 256,
                 e_ts=256, e_v=128, sk=None if L.sk is None else nb(L.sk), sv=None if L.sv is None else nb(L.sv),
                 skoff=None if L.skoff is None else L.skoff[:S].cpu().numpy(),
                 svoff=None if L.skoff is None else L.skoff[:S].cpu().numpy(), N=L.N[:S].cpu().numpy(),
                 NQ=L.NQ[:S].cpu().numpy(), nqmax=L.nq, win=L.win)
        per_layer.append((P, nb(q[:S])))
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        for P, q in per_layer:
            O.decode(P, q, cs, sn)
        ts.append(time.perf_counter() - t0)
    med = statistics.median(ts)
    return S / med, med


# ---------------------------------------------------------------- flush / quantize (config 2)
def flush_bench(kv800, torch, dev, reps=10):
    """Config 2 of BASELINE: K / V ~ N(0, 1) bf16 with 1 % of the channels x 8.  (a) prefill: 16 sequences x 2048
    tokens = 112 full sub-blocks quantized in one quantize_blocks call; (b) decode step: 256 sequences whose new token
    completes a flush boundary, one 256-token sub-block each gathered from shuffled exact pages by the paged flush.
    Reports sub-blocks/s and the bytes moved (524,288 read + 51,200 written per sub-block)."""
    g = torch.Generator(device="cpu").manual_seed(7)
    def kvgen(M):
        k = torch.randn(M, 256, 4, 128, generator=g)
        v = torch.randn(M, 256, 4, 128, generator=g)
        mk = torch.rand(4, 128, generator=g) < 0.01
        mv = torch.rand(4, 128, generator=g) < 0.01
        k = torch.where(mk, k * 8, k).to(torch.bfloat16).to(dev)
        v = torch.where(mv, v * 8, v).to(torch.bfloat16).to(dev)
        return k, v
    k, v = kvgen(112)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / reps

    t_pre = timed(lambda: kv800.quantize_blocks(k, v))
    # 256 sequences: exact pages of 64 tokens at shuffled slots, sub-block 0 of each (positions 0..255) flushed
    B, ebs = 256, 64
    kk, vv = kvgen(B)
    perm = torch.randperm(B * 4 + 5, generator=g)[:B * 4].view(B, 4)
    eoff = (perm * (4 * ebs * 256)).to(torch.int64).to(dev)
    epool = torch.zeros(B * 4 + 5, 4, ebs, 256, dtype=torch.bfloat16, device=dev)
    seq = torch.arange(B, dtype=torch.int32, device=dev).repeat_interleave(256)
    pos = torch.arange(256, dtype=torch.int64, device=dev).repeat(B)
    kv800.write_exact(epool, eoff, ebs, ebs * 256, 256, 128, kk.reshape(-1, 4, 128), vv.reshape(-1, 4, 128), seq,
                      pos)
    qpool = torch.zeros(B + 3, 51200, dtype=torch.uint8, device=dev)
    boff = (torch.randperm(B + 3, generator=g)[:B] * 51200).to(torch.int64).view(B, 1).to(dev)
    sidx = torch.arange(B, dtype=torch.int32, device=dev)
    zero = torch.zeros(B, dtype=torch.int32, device=dev)
    t_step = timed(lambda: kv800.flush(epool, eoff, ebs, ebs * 256, 256, 128, qpool, boff, sidx, zero))
    per = 524288 + 51200
    return {"prefill_subblocks": 112, "prefill_us": round(t_pre * 1e6, 1),
            "prefill_subblocks_per_s": round(112 / t_pre, 1), "prefill_tok_per_s": round(112 * 256 / t_pre, 1),
            "prefill_gbs": round(112 * per / t_pre / 1e9, 1),
            "step_flush_subblocks": B, "step_flush_us": round(t_step * 1e6, 1),
            "step_flush_gbs": round(B * per / t_step / 1e9, 1),
            "bound": "issue: V rotation by a fast Walsh-Hadamard estimate with certified decisions (exact FMA chain "
                     "only for tokens with an undecided byte or bit), K codes by a certified reciprocal quotient"}


def next_rows_bench(kv800, torch, dev, reps=10):
    """The rows after the decode, each on its own seeded synthetic case:
    vllm_step   one decode step of a quantized layer through vllm_step.KV800Attention.forward for 64 requests at
                ~32K tokens with vLLM-shaped caches (exact blocks of 128 tokens, 262,144-B quant pages, shuffled
                block tables; half of the requests cross the flush boundary this step, so the step flushes 32
                sub-blocks), against kv800.decode alone on the same caches;
    prefill_kv  the K / V a 32,768-token extend attends to: 127 dequantized sub-blocks + 256 exact rows + a 1-token
                chunk, rotated, bf16 (output bytes / time);
    train       fake_quant_k (as (8, 16, 256, 512) groups) / fake_quant_v on (8, 4096, 4, 128) fp32 activations
                (bytes in + out / time);
    sliding     a native sliding layer's decode (64 rows, window 256) without tables vs with identity tables."""
    from lfm3_kv800 import train as T
    from lfm3_kv800 import vllm_step as S
    g = torch.Generator(device="cpu").manual_seed(11)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / reps

    out = {}
    # ---- vLLM step over vLLM-shaped caches
    R, ebs = 64, 128
    n_new = [32640 if r % 2 == 0 else 32641 for r in range(R)]   # 32,640 = 256 x 126 + 384: flushes sub-block 126
    pages, qpages = -(-max(n_new) // ebs), -(-max(n_new) // S.QBLOCK)
    live = 6                                             # exact blocks a request keeps (the 640-token window + slack)
    nblk = R * live + 1
    bt = torch.zeros(R, pages, dtype=torch.int32)
    perm = torch.randperm(nblk - 1, generator=g) + 1
    for r in range(R):
        last = (n_new[r] - 1) // ebs
        bt[r, last - live + 1:last + 1] = perm[r * live:(r + 1) * live].to(torch.int32)
    qperm = torch.randperm(R * qpages, generator=g).view(R, qpages).to(torch.int32)
    ev = (torch.randn(nblk, 4, ebs, 256, generator=g)).to(torch.bfloat16).to(dev)
    npg = R * qpages
    qraw = torch.zeros(npg * S.QPAGE, dtype=torch.uint8, device=dev)
    pv = qraw.view(npg, S.QPAGE)
    for p0 in range(0, npg, 64):                        # every sub-block slot holds real quantized data
        p1 = min(npg, p0 + 64)
        m = (p1 - p0) * 5
        k = torch.randn(m, 256, 4, 128, device=dev).to(torch.bfloat16)
        v = torch.randn(m, 256, 4, 128, device=dev).to(torch.bfloat16)
        pv[p0:p1, :5 * SUB] = kv800.quantize_blocks(k, v).view(p1 - p0, 5 * SUB)
    qv = torch.as_strided(qraw, (R * qpages, 2, S.QBLOCK, 4, S.QCONTENT),
                          (S.QPAGE, S.QBLOCK * 4 * S.QCONTENT, 4 * S.QCONTENT, S.QCONTENT, 1))
    sl = torch.tensor(n_new, dtype=torch.int32)
    qsl = torch.arange(R + 1, dtype=torch.int32)
    pos = sl.long() - 1
    slot = (bt[torch.arange(R), (pos // ebs)].long() * ebs + pos % ebs)
    q = torch.randn(R, 16, 128, generator=g).to(torch.bfloat16).to(dev)
    k1 = torch.randn(R, 4, 128, generator=g).to(torch.bfloat16).to(dev)
    v1 = torch.randn(R, 4, 128, generator=g).to(torch.bfloat16).to(dev)
    attn = S.KV800Attention(6, 33000)
    bt_d, slot_d, sl_d, qsl_d, pos_d, qbt_d = (t.to(dev) for t in (bt, slot, sl, qsl, pos, qperm))

    def vstep():                                        # the metadata lives on the device, as vLLM keeps it
        mx = S.build_meta(bt_d, slot_d, sl_d, qsl_d, sl, qsl, pos_d, R)
        mq = S.build_meta(qbt_d, slot_d, sl_d, qsl_d, sl, qsl, pos_d, R)
        return attn.forward(q, k1, v1, mx, ev, mq=mq, qv=qv)
    t_step = timed(vstep)
    # the step has no host sync, so it also runs as one CUDA graph: the graph replay is its device time without the
    # Python / launch overhead of eager mode
    t_graph = None
    try:
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            vstep()
        torch.cuda.current_stream(dev).wait_stream(side)
        with torch.cuda.graph(graph):
            vstep()
        t_graph = timed(graph.replay)
        del graph
    except Exception as ex:                             # report, do not fail the bench
        t_graph = f"capture failed: {type(ex).__name__}: {str(ex)[:120]}"
    mx = S.build_meta(bt_d, slot_d, sl_d, qsl_d, sl, qsl, pos_d, R)
    c32, s32, _, _ = S.tables(dev, 33000)
    qs0 = qv.stride(0)
    nqmax = max(S.nq_of(n) for n in n_new)
    tb = S.decode_tables(mx.seq_lens, R, mx.block_table, ev.stride(0), qbt_d, qs0, S.QBLOCK, nqmax)
    P = kv800.Paged(qpool=qv, boff=tb["boff"], epool=ev, eoff=tb["eoff"], ebs=ebs, e_hs=ev.stride(1),
                    e_ts=ev.stride(2), e_v=128, N=tb["N"], NQ=tb["NQ"], nqmax=nqmax, win=0)
    t_dec = timed(lambda: kv800.decode(P, q, c32, s32))
    out["vllm_step"] = {"requests": R, "flushed_subblocks": R // 2, "eager_step_us": round(t_step * 1e6, 1),
                        "graph_step_us": round(t_graph * 1e6, 1) if isinstance(t_graph, float) else t_graph,
                        "decode_only_us": round(t_dec * 1e6, 1),
                        "launches": "write_slots, flush plan + flush, decode tables, 3 decode kernels"}
    # ---- prefill / extend history assembly for one 32K request
    r0 = 0
    nq0 = S.nq_of(n_new[r0] - 1)
    ch_k, ch_v = k1[:1], v1[:1]

    def pk():
        return S.prefill_kv(n_new[r0] - 1, n_new[r0], ch_k, ch_v, ev, mx.block_table[r0], qv=qv,
                            qbt_row=qbt_d[r0], nqp=nq0, cos_t=c32, sin_t=s32)
    t_pk = timed(pk)
    rows = nq0 * 256 + (n_new[r0] - nq0 * 256)
    out["prefill_kv"] = {"tokens": rows, "us": round(t_pk * 1e6, 1),
                         "out_gbs": round(rows * 2048 / t_pk / 1e9, 1),
                         "in_bytes": nq0 * SUB + (rows - nq0 * 256) * 2048}
    # ---- training fake quant
    x = torch.randn(8, 4096, 4, 128, device=dev)
    xk = x.view(8, 16, 256, 512)                         # (B, groups of 256 tokens, 256, 4 heads x 128 channels)
    t_k = timed(lambda: T.fake_quant_k(xk))
    t_v = timed(lambda: T.fake_quant_v(x))
    nbytes = x.numel() * 8
    out["train_fake_quant"] = {"shape": [8, 4096, 4, 128], "k_us": round(t_k * 1e6, 1), "v_us": round(t_v * 1e6, 1),
                               "k_gbs": round(nbytes / t_k / 1e9, 1), "v_gbs": round(nbytes / t_v / 1e9, 1)}
    # ---- native sliding layer (window 256, no sinks): no tables vs identity tables
    Ps = kv800.Paged(qpool=ev, boff=tb["eoff"], epool=ev, eoff=tb["eoff"], ebs=ebs, e_hs=ev.stride(1),
                     e_ts=ev.stride(2), e_v=128, N=tb["N"], NQ=torch.zeros_like(tb["NQ"]), nqmax=0, win=WIN)
    _, _, one, zero = S.tables(dev, 33000)
    t_nt = timed(lambda: kv800.decode(Ps, q, None, None))
    t_id = timed(lambda: kv800.decode(Ps, q, one, zero))
    sb_bytes = R * WIN * 2048
    out["sliding"] = {"rows": R, "window": WIN, "no_tables_us": round(t_nt * 1e6, 1),
                      "identity_tables_us": round(t_id * 1e6, 1), "gbs_no_tables": round(sb_bytes / t_nt / 1e9, 1)}
    return out


# ---------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="cuda", choices=("cuda", "reference"))
    ap.add_argument("--cpu-seqs", type=int, default=64, help="sequences of the CPU-baseline sample")
    ap.add_argument("--cpu-reps", type=int, default=3, help="passes of the CPU-baseline sample (median)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline (profiling runs)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-flush", action="store_true", help="skip the quantize / flush measurement")
    ap.add_argument("--no-next", action="store_true", help="skip the vLLM-step / prefill / train / sliding measurement")
    ap.add_argument("--seqs", type=int, default=B_PER_GPU, help="sequences per GPU (profiling: smaller cases)")
    ap.add_argument("--ctx", type=int, default=N_CTX, help="context length (profiling: smaller cases)")
    ap.add_argument("--workload", default="config3", choices=("config3", "ragged"),
                    help="config3 (the metric's workload) or ragged (BASELINE config 4: 2,048 rows of U[1K, 32K] "
                         "tokens sharded over the ranks, strong scaling)")
    ap.add_argument("--pool-gb", type=float, default=150.0, help="ragged: the sub-block pool per GPU (GB)")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)

    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n_gpus = max(world, 1)

    if a.impl == "reference":
        return reference_arm(a, rank, world, n_gpus)

    from lfm3_kv800 import _lib, kv800
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        def init():
            dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
            dist.barrier()   # the communicator is created by now
        stdout_to_stderr(init)

    if a.workload == "ragged":
        return ragged_main(a, kv800, torch, dist, dev, rank, world, local, n_gpus)
    layers, qs, c32, s32 = build_workload(kv800, torch, dev, rank, B=a.seqs, n=a.ctx)
    torch.cuda.synchronize()
    step_bytes = sum(L.algo_bytes() for L in layers)

    def step():
        return [kv800.decode(L.P, q, c32, s32) for L, q in zip(layers, qs)]

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        torch.cuda.synchronize()
        ev0.record()
        for _ in range(a.steps):
            step()
        ev1.record()
        torch.cuda.synchronize()
    t = ev0.elapsed_time(ev1) / 1e3
    if world > 1:
        tt = torch.tensor([t], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt.item())
        dist.barrier()
    clocks = clk.summary()
    value = a.seqs * a.steps * n_gpus / t
    launches_per_step = sum(3 if L.nq else 1 for L in layers)   # qsched + qdecode + xdecode (merge included)

    # ---- dominant kernel: qdecode_mma (87.5 % of the decode kernels' device time in the ncu launch list), timed by
    # CUDA events around the quantized phase of one quantized-layer decode (schedule + qdecode_mma) with L2 flushed
    # before every launch; algorithmic bytes = the layer's sub-blocks read once, 64 x 127 x 51,200 B
    L0, q0 = layers[0], qs[0]
    kreps = 10
    flushbuf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(3):
        kv800.decode(L0.P, q0, c32, s32)
    kt, lt = [], []
    for _ in range(kreps):
        flushbuf.fill_(1)
        _, ms = kv800.decode_timed(L0.P, q0, c32, s32)
        kt.append(ms["quantized_ms"] / 1e3)
        lt.append((ms["quantized_ms"] + ms["exact_ms"] + ms["combine_ms"]) / 1e3)
    kdur, ldur = statistics.median(kt), statistics.median(lt)
    kbytes = L0.B * L0.nq * SUB
    hbm, peak_kind = peaks()
    # DRAM traffic of qdecode_mma from one ncu capture on 64 x 16,384 (4,032 sub-blocks: 209.5 MB read + 5.1 MB
    # written), scaled to this launch by sub-blocks (traffic grows in proportion: reads are the sub-blocks plus
    # the cos / sin rows, writes the split partials)
    traffic = round((209.5e6 + 5.1e6) * (L0.B * L0.nq) / 4032) if a.ctx == N_CTX and a.seqs == B_PER_GPU else None
    roofline = {"bound": "hbm", "achieved": round(kbytes / kdur / 1e9, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(kbytes / kdur / 1e9 / hbm, 4), "traffic": traffic, "peak_source": peak_kind,
                "kernel": "qdecode_mma (+ its 1-CTA schedule scan)", "bytes_per_launch": kbytes,
                "launch_us": round(kdur * 1e6, 1),
                "layer_decode": {"bytes": L0.algo_bytes(), "us": round(ldur * 1e6, 1),
                                 "achieved_gbs": round(L0.algo_bytes() / ldur / 1e9, 1),
                                 "kernels": "qsched + qdecode_mma + xdecode_mma (with the merge of each row's partials)"}}

    # ---- end to end through the public API with host buffers
    e2e = None
    if not a.no_e2e:
        B = a.seqs
        nl = len(layers)
        hq = [q.cpu().pin_memory() for q in qs]
        hk = torch.randn(nl, B, 4, 128).to(torch.bfloat16).pin_memory()
        hv = torch.randn(nl, B, 4, 128).to(torch.bfloat16).pin_memory()
        hout = [torch.empty(B, 16, 128, dtype=torch.bfloat16).pin_memory() for _ in layers]
        seqs = torch.arange(B, dtype=torch.int32, device=dev)
        posv = torch.full((B,), a.ctx - 1, dtype=torch.int64, device=dev)
        # copies run on their own stream: all layers' uploads are queued at the step's start, so layer i + 1's
        # inputs arrive while layer i decodes, and layer i's output is read back while layer i + 1 decodes.  The
        # device input buffers are reused across steps: the next step's uploads queue behind this step's last
        # read-back, which waits for the last decode, so no upload overwrites an input still in use.
        main, cps = torch.cuda.current_stream(dev), torch.cuda.Stream(dev)
        dq = [torch.empty_like(q) for q in qs]
        dk = torch.empty(nl, B, 4, 128, dtype=torch.bfloat16, device=dev)
        dv = torch.empty_like(dk)
        ready = [torch.cuda.Event() for _ in layers]
        done = [torch.cuda.Event() for _ in layers]

        def e2e_step():
            with torch.cuda.stream(cps):
                for i in range(nl):
                    dq[i].copy_(hq[i], non_blocking=True)
                    dk[i].copy_(hk[i], non_blocking=True)
                    dv[i].copy_(hv[i], non_blocking=True)
                    ready[i].record(cps)
            for i, L in enumerate(layers):
                main.wait_event(ready[i])
                kv800.write_exact(L.epool, L.eoff, EBS, EBS * 256, 256, 128, dk[i], dv[i], seqs, posv)
                o = kv800.decode(L.P, dq[i], c32, s32)
                done[i].record(main)
                cps.wait_event(done[i])
                with torch.cuda.stream(cps):
                    hout[i].copy_(o, non_blocking=True)
                o.record_stream(cps)
            main.wait_stream(cps)      # the step ends when its last read-back has landed
            return hout

        for _ in range(a.warmup):
            e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        te = e0.elapsed_time(e1) / 1e3
        if world > 1:
            tt = torch.tensor([te], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            te = float(tt.item())
        h2d = sum(x.numel() * x.element_size() for x in hq) + hk.numel() * 2 + hv.numel() * 2
        d2h = sum(x.numel() * x.element_size() for x in hout)
        e2e = {"value": round(a.seqs * a.steps * n_gpus / te, 1), "unit": "tok/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": round(te / a.steps * 1e3, 4)}

    # ---- flush / quantize: a 16 x 2048-token prefill (112 sub-blocks through quantize_blocks)
    # and a decode step of 256 sequences that crosses a flush boundary (one sub-block each through the paged flush)
    flush = None
    if not a.no_flush:
        flush = flush_bench(kv800, torch, dev)
    nxt = None
    if not a.no_next and world == 1:
        nxt = next_rows_bench(kv800, torch, dev)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:
        S = a.cpu_seqs
        tps, sec = cpu_sample(layers, qs, c32, s32, S, reps=a.cpu_reps)
        cpu = {"value": round(tps, 2), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{S} of the {a.seqs} sequences x {a.ctx:,} tokens, all 6 layers, oracle/kv800_oracle.c "
                         f"(OpenMP over sequence x kv head), median of {a.cpu_reps} passes of {sec:.2f} s"}

    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": n_gpus, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": round(t / a.steps * 1e3, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "u8+bf16 (fp32 math)", "data": "synthetic",
                "config": {"workload": "config 3: 64 seq x 32768 ctx per GPU, 4 quantized (127 sub-blocks + 256 "
                                       "exact) + 2 window (4 sinks + 256) layers, 16q/4kv/128, shuffled pages",
                           "seqs_per_gpu": a.seqs, "ctx": a.ctx, "layers": QUANT_LAYERS + WINDOW_LAYERS,
                           "parallelism": f"dp{n_gpus} (sequence sharding, no collective)",
                           "l2": "inputs larger than L2 (1.87 GB per step); kernel timing flushes L2 per launch"},
                "hbm_gbs_step": round(step_bytes * a.steps / t / 1e9, 1),
                "hbm_frac_step": round(step_bytes * a.steps / t / 1e9 / peaks()[0], 4),
                "bytes_per_step_per_gpu": step_bytes, "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": launches_per_step * a.steps, "clocks": clocks, "flush": flush, "next_rows": nxt}
        print(json.dumps(line), flush=True)


def ragged_main(a, kv800, torch, dist, dev, rank, world, local, n_gpus):
    """Config 4: every rank decodes its LPT share of the 2,048 ragged rows through all 6 layers per step; value =
    2,048 x steps / max-over-ranks device time (strong scaling: the total work is fixed)."""
    layers, qs, c32, s32, rows, pool_bytes = build_ragged(kv800, torch, dev, rank, world, a.pool_gb)
    torch.cuda.synchronize()
    step_bytes = sum(L.algo_bytes() for L in layers)

    def step():
        return [kv800.decode(L.P, q, c32, s32) for L, q in zip(layers, qs)]

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        torch.cuda.synchronize()
        ev0.record()
        for _ in range(a.steps):
            step()
        ev1.record()
        torch.cuda.synchronize()
    t = ev0.elapsed_time(ev1) / 1e3
    tmax = t
    bytes_all = step_bytes
    if world > 1:
        tt = torch.tensor([t], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        tmax = float(tt.item())
        bb = torch.tensor([float(step_bytes)], device=dev, dtype=torch.float64)
        dist.all_reduce(bb)
        bytes_all = float(bb.item())
        dist.barrier()
    # dominant kernel on this rank: the quantized phase of layer 0 (L2 flushed)
    L0, q0 = layers[0], qs[0]
    flushbuf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    kt = []
    for _ in range(10):
        flushbuf.fill_(1)
        _, ms = kv800.decode_timed(L0.P, q0, c32, s32)
        kt.append(ms["quantized_ms"] / 1e3)
    kdur = statistics.median(kt)
    kbytes = sum(L0.nq_rows) * SUB
    hbm, peak_kind = peaks()
    clocks = clk.summary()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        line = {"metric": METRIC, "value": round(RAGGED_ROWS * a.steps / tmax, 1), "unit": "tok/s", "n_gpus": n_gpus,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(tmax / a.steps * 1e3, 4),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8+bf16 (fp32 math)",
                "data": "synthetic",
                "config": {"workload": f"config 4: {RAGGED_ROWS} rows, lengths U[{RAGGED_LO}, {RAGGED_HI}] (seed "
                                       f"2048), LPT-sharded over {n_gpus} GPU(s), 4 quantized + 2 window layers, "
                                       f"sub-blocks scattered over a {pool_bytes / 1e9:.0f} GB pool per GPU",
                           "rows_rank0": len(rows), "parallelism": f"dp{n_gpus} (LPT row sharding, no collective)"},
                "hbm_gbs_step": round(bytes_all * a.steps / tmax / 1e9, 1),
                "bytes_per_step_all_gpus": int(bytes_all),
                "roofline": {"bound": "hbm", "achieved": round(kbytes / kdur / 1e9, 1), "peak": hbm, "unit": "GB/s",
                             "frac": round(kbytes / kdur / 1e9 / hbm, 4), "traffic": None, "peak_source": peak_kind,
                             "kernel": "qdecode_mma (+ its 1-CTA schedule scan), rank 0, layer 0",
                             "bytes_per_launch": kbytes, "launch_us": round(kdur * 1e6, 1)},
                "cpu_baseline": None, "e2e": None,
                "gpu_launches": sum(3 if L.nqmax else 1 for L in layers) * a.steps, "clocks": clocks}
        print(json.dumps(line), flush=True)


def reference_arm(a, rank, world, n_gpus):
    """The reference's CPU path for this step (the oracle port of torch_decode, all host threads) on a bounded sample:
    S = cores / 4 (at most 4) sequences of the 64 x 32K, 6-layer workload per step, so that every host thread has a
    (sequence, kv head) item (about 0.2 s per step on 16 cores), exactly K steps after W warm-ups."""
    if rank != 0:
        return
    import torch
    from oracle import oracle as O
    O.lib()
    S = max(1, min(4, (os.cpu_count() or 4) // 4))   # the oracle runs (sequence x kv head) items in parallel
    # the workload built on the CPU side with the oracle's own quantizer (no GPU used by this arm)
    rs = np.random.RandomState(99)
    import inputs as I
    cs, sn = I.rope_tables(N_CTX + 64)
    per_layer = []
    for li in range(QUANT_LAYERS + WINDOW_LAYERS):
        win = 0 if li < QUANT_LAYERS else WIN
        nq = 0 if win else (N_CTX - 128) // 256
        lo = nq * 256 if not win else N_CTX - win
        npg = N_CTX // EBS + 1
        first = lo // EBS
        pps = (N_CTX - 1) // EBS - first + 1
        epool = np.zeros((S * pps, 4, EBS, 256), np.uint16)
        eoff = np.zeros((S, npg), np.int64)
        eoff[:, first:first + pps] = (rs.permutation(S * pps).reshape(S, pps) * 4 * EBS * 256)
        epool[...] = I.f32_to_bf16(rs.standard_normal(epool.shape).astype(np.float32))
        if nq:
            M = S * nq
            qpool = np.zeros((M, SUB), np.uint8)
            for c0 in range(0, M, 64):
                c1 = min(M, c0 + 64)
                k = I.f32_to_bf16(rs.standard_normal((c1 - c0, 256, 4, 128)).astype(np.float32))
                v = I.f32_to_bf16(rs.standard_normal((c1 - c0, 256, 4, 128)).astype(np.float32))
                qpool[c0:c1] = O.quantize_blocks(k, v)
            boff = (rs.permutation(M).reshape(S, nq) * SUB).astype(np.int64)
        else:
            qpool, boff = np.zeros((1, SUB), np.uint8), np.zeros((S, 1), np.int64)
        sk = I.f32_to_bf16(rs.standard_normal((S, NSINK, 4, 128)).astype(np.float32)) if win else None
        P = dict(qpool=qpool, boff=boff, epool=epool, eoff=eoff, ebs=EBS, e_hs=EBS * 256, e_ts=256, e_v=128, sk=sk,
                 sv=sk, skoff=np.arange(S, dtype=np.int64) * NSINK * 512, svoff=np.arange(S, dtype=np.int64) * NSINK * 512,
                 N=np.full(S, N_CTX, np.int32), NQ=np.full(S, nq, np.int32), nqmax=nq, win=win)
        q = I.f32_to_bf16(rs.standard_normal((S, 16, 128)).astype(np.float32))
        per_layer.append((P, q))

    def step():
        for P, q in per_layer:
            O.decode(P, q, cs, sn)

    for _ in range(a.warmup):
        step()
    steps = a.steps
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = (time.perf_counter() - t0) / steps
    v = S / dt
    cores = os.cpu_count()
    line = {"metric": METRIC, "value": round(v, 2), "unit": "tok/s", "n_gpus": n_gpus, "steps": steps,
            "warmup": a.warmup, "ms_per_step": round(dt * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8+bf16 (fp32 math)", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "config 3: 64 seq x 32768 ctx per GPU, 4 quantized (127 sub-blocks + 256 exact) + "
                                   "2 window (4 sinks + 256) layers, 16q/4kv/128, shuffled pages",
                       "seqs_per_gpu": B_PER_GPU, "ctx": N_CTX, "layers": QUANT_LAYERS + WINDOW_LAYERS,
                       "parallelism": "host cores (reference CPU path)"},
            "cpu_baseline": {"value": round(v, 2), "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"{S} sequences x 32,768 tokens x 6 layers per step (of the 64 per GPU), "
                                       f"oracle/kv800_oracle.c decode with OpenMP over sequence x kv head"},
            "e2e": {"value": round(v, 2), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
