"""Benchmark of the 800h hot path on B200: paged GQA decode over the 800h cache at 64 sequences x 32,768 tokens per GPU,
all 6 attention layers of the LFM3-1.7B shape (4 quantized layers: 127 sub-blocks + a 256-token exact tail; 2 window
layers: 4 sinks + 256 exact tokens), one decode query per sequence per layer (the metric's
config).  Sub-blocks and exact pages sit at a seeded random permutation of pool slots.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--windows R] [--impl cuda|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

A step = the decode of all 6 layers for the rank's 64 sequences (one token per sequence), captured once as a CUDA
graph and replayed (--eager: launched eagerly; the eager median is reported beside the graph's in config.timing).
Timing: R windows of exactly K steps, each bracketed by a barrier and a device synchronize and timed with CUDA
events, max over ranks per window; `value` = sequences x K x ranks / the median window (tok/s, weak scaling: 64 sequences per GPU), with the
windows' spread in config.timing.  Keys of the line:
  e2e          the same metric through the public API with the step's inputs (6 x q, the current token's K / V)
               copied from pinned host memory, the token written into its exact page, and the 6 outputs read back,
               all inside the timed region (copies on a second stream, overlapped with the neighbouring layers);
  roofline     the quantized-split kernel (the dominant one) timed alone with CUDA events, L2 flushed: algorithmic
               bytes (51,200 per sub-block) / duration against the measured HBM copy bandwidth;
  parity       rows of the timed outputs against the CPU oracle on the same pools (gathered to rank 0 over NCCL at
               N > 1: the only collective besides the timing reduction);
  cpu_baseline the reference's own torch_decode.decode (staged under oracle/_ref, run in a child process on all host
               threads) on a bounded sample of the same workload; cpu_baseline_port: its C restatement
               (oracle/kv800_oracle.c) on 64 sequences;
  config1      BASELINE config 1 (one quantized layer, 4 x 2,048): per-call latency, roofline, parity, CPU baseline;
  flush        BASELINE config 2 (the quantizer / flush) with every packed byte compared to the oracle quantizer;
  ragged       BASELINE config 4 (2,048 ragged rows, LPT-sharded over the ranks, strong scaling) in the same run;
  next_rows    the rows after the decode (vLLM step, prefill K / V, training fake quant, sliding layers), N = 1.
--workload ragged prints config 4's line alone.

--impl reference: the reference's CPU path for this step (its own torch_decode on the host cores, or the C port of it
when the reference is not staged) on a bounded sample of the same workload, printed as the reference arm's line; on
N > 1 ranks only rank 0 runs it."""
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
REF_STAGED = os.path.join(ROOT, "oracle", "_ref")       # oracle/stage_reference.py: the reference package's sources
if "--ref-worker" not in sys.argv:                      # the reference CPU worker imports the reference alone
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


# ---------------------------------------------------------------- the reference's CPU decode (separate process)
def ref_worker(argv):
    """Runs in a child process whose sys.path holds only the staged reference package (oracle/_ref): times the
    reference's own torch_decode.decode (lfm3_kv800/torch_decode.py:27-80, the reference's CPU path for this step) on
    the host cores.  argv: JSON {"seqs": S, "ctx": n, "steps": K, "warmup": W, "config1_reps": R}.  Workloads: S
    rows x n tokens through 4 quantized + 2 window layers per step (config 3's shape; sub-blocks made by the
    reference's quantize_blocks on the CPU, pages at shuffled slots), and config 1 (one quantized layer, 4 rows x
    2,048 tokens).  Prints one JSON line with the per-step and per-call seconds."""
    import json as _json
    cfg = _json.loads(argv)
    sys.path[:0] = [REF_STAGED]
    import torch
    from lfm3_kv800 import kv800 as RK, torch_decode as TD
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(17)
    H = RK.hadamard(128)

    def tables(P):
        inv = 1.0 / (1e6 ** (torch.arange(0, 64, 2, dtype=torch.float32) / 128))
        fr = torch.arange(P, dtype=torch.float32)[:, None] * inv[None]
        return fr.cos().to(torch.bfloat16).contiguous(), fr.sin().to(torch.bfloat16).contiguous()

    def layer(B, n, win):
        nq = 0 if win else max(0, n - 128) // 256
        lo = max(0, n - win) if win else nq * 256
        npg = n // EBS + 1
        first, last = lo // EBS, (n - 1) // EBS
        pps = last - first + 1
        perm = torch.randperm(B * pps + 3, generator=g)[:B * pps].view(B, pps)
        eoff = torch.zeros(B, npg, dtype=torch.int64)
        eoff[:, first:last + 1] = perm * (4 * EBS * 256)
        epool = torch.randn(B * pps + 3, 4, EBS, 256, generator=g).to(torch.bfloat16)
        if nq:
            slots = torch.randperm(B * nq + 5, generator=g)[:B * nq].view(B, nq)
            qpool = torch.zeros(B * nq + 5, SUB, dtype=torch.uint8)
            for c0 in range(0, B * nq, 64):
                c1 = min(B * nq, c0 + 64)
                k = torch.randn(c1 - c0, 256, 4, 128, generator=g).to(torch.bfloat16)
                v = torch.randn(c1 - c0, 256, 4, 128, generator=g).to(torch.bfloat16)
                qpool[slots.view(-1)[c0:c1]] = RK.quantize_blocks(k, v, H)
            boff = slots * SUB
        else:
            qpool, boff = torch.zeros(1, SUB, dtype=torch.uint8), torch.zeros(B, 1, dtype=torch.int64)
        sk = torch.randn(B, NSINK, 4, 128, generator=g).to(torch.bfloat16) if win else None
        skoff = torch.arange(B, dtype=torch.int64) * NSINK * 512 if win else None
        return RK.Paged(qpool=qpool, boff=boff, epool=epool, eoff=eoff, ebs=EBS, e_hs=EBS * 256, e_ts=256, e_v=128,
                        sk=sk, sv=sk, skoff=skoff, svoff=skoff, N=torch.full((B,), n, dtype=torch.int32),
                        NQ=torch.full((B,), nq, dtype=torch.int32), nqmax=nq, win=win)

    S, n = cfg["seqs"], cfg["ctx"]
    out = {"threads": threads, "torch": torch.__version__}
    if S > 0:
        layers = [layer(S, n, 0) for _ in range(QUANT_LAYERS)] + [layer(S, n, WIN) for _ in range(WINDOW_LAYERS)]
        qs = [torch.randn(S, 16, 128, generator=g).to(torch.bfloat16) for _ in layers]
        c32, s32 = tables(n + 64)
        times = []
        for i in range(cfg["warmup"] + cfg["steps"]):
            t0 = time.perf_counter()
            for P, q in zip(layers, qs):
                TD.decode(P, q, c32, s32, H)
            if i >= cfg["warmup"]:
                times.append(time.perf_counter() - t0)
        out["step_s"] = times
        del layers
    if cfg.get("config1_reps", 0):
        P1 = layer(4, 2048, 0)
        q1 = torch.randn(4, 16, 128, generator=g).to(torch.bfloat16)
        c32, s32 = tables(4096)
        for _ in range(3):
            TD.decode(P1, q1, c32, s32, H)
        calls = []
        for _ in range(cfg["config1_reps"]):
            t0 = time.perf_counter()
            TD.decode(P1, q1, c32, s32, H)
            calls.append(time.perf_counter() - t0)
        out["config1_call_s"] = calls
    print("REFJSON " + _json.dumps(out), flush=True)


def run_ref_worker(seqs, ctx, steps, warmup, config1_reps=0, timeout=1800):
    """The reference's torch_decode timed in a child process (ref_worker); None when the reference is not staged
    (then the C port of it stands in, and the line says so)."""
    if not os.path.exists(os.path.join(REF_STAGED, "lfm3_kv800", "torch_decode.py")):
        return None
    arg = json.dumps({"seqs": seqs, "ctx": ctx, "steps": steps, "warmup": warmup, "config1_reps": config1_reps})
    env = dict(os.environ, PYTHONPATH="", CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, os.path.abspath(__file__), "--ref-worker", arg], capture_output=True,
                       text=True, env=env, timeout=timeout)
    for line in r.stdout.splitlines():
        if line.startswith("REFJSON "):
            return json.loads(line[8:])
    raise RuntimeError(f"reference CPU worker failed (rc {r.returncode}): {r.stderr[-800:]}")


# ---------------------------------------------------------------- CPU oracle on a bounded sample
def _bits(t):
    """torch bf16 (any device) -> numpy bf16 bits."""
    import torch
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def oracle_view(L, rows):
    """The oracle's numpy Paged dict for rows `rows` of layer L (the rows' sub-blocks copied into a compact pool)."""
    import torch
    rows = list(rows)
    S = len(rows)
    ri = np.asarray(rows, np.int64)
    if L.nq:
        slots = torch.from_numpy(L.boff.cpu().numpy()[ri].reshape(-1) // SUB).to(L.qpool.device)
        qpool = L.qpool.view(-1, SUB)[slots].cpu().numpy()
        boff = (np.arange(S * L.nq, dtype=np.int64) * SUB).reshape(S, L.nq)
    else:
        qpool, boff = np.zeros((1, SUB), np.uint8), np.zeros((S, 1), np.int64)
    sk = None if L.sk is None else _bits(L.sk)
    skoff = None if L.skoff is None else L.skoff.cpu().numpy()[ri]
    return dict(qpool=qpool, boff=boff, epool=_bits(L.epool), eoff=L.eoff.cpu().numpy()[ri], ebs=EBS, e_hs=EBS * 256,
                e_ts=256, e_v=128, sk=sk, sv=None if L.sv is None else _bits(L.sv), skoff=skoff, svoff=skoff,
                N=L.N.cpu().numpy()[ri], NQ=L.NQ.cpu().numpy()[ri], nqmax=L.nq, win=L.win)


def cpu_sample(layers, qs, c32, s32, S, reps=1):
    """Time the oracle (C port of the reference decode) on sequences [0, S) of every layer; -> (tok/s, sec/step)."""
    from oracle import oracle as O
    cs, sn = _bits(c32), _bits(s32)
    per_layer = [(oracle_view(L, range(S)), _bits(q[:S])) for L, q in zip(layers, qs)]
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        for P, q in per_layer:
            O.decode(P, q, cs, sn)
        ts.append(time.perf_counter() - t0)
    med = statistics.median(ts)
    return S / med, med


def parity_metrics(got_bits, ref_bits):
    """rel-L2 and max-abs of bf16 outputs against the oracle's (1e-2 and 2e-2)."""
    g = (got_bits.astype(np.uint32) << 16).view(np.float32)
    r = (ref_bits.astype(np.uint32) << 16).view(np.float32)
    return float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30)), float(np.abs(g - r).max())


def sample_refs(layers, qs, c32, s32, rows):
    """The oracle's outputs (bf16 bits, (layers, len(rows), 16, 128)) for rows `rows` of every layer."""
    from oracle import oracle as O
    cs, sn = _bits(c32), _bits(s32)
    return np.stack([O.decode(oracle_view(L, rows), _bits(q[list(rows)]), cs, sn) for L, q in zip(layers, qs)])


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
    # bit-exactness of what was timed, outside the timed region: every packed byte against the oracle quantizer (the
    # C restatement of kv800.quantize_blocks, pinned to the reference's own bytes by the golden fixtures)
    from oracle import oracle as O
    pre_ok = bool(np.array_equal(kv800.quantize_blocks(k, v).cpu().numpy(), O.quantize_blocks(_bits(k), _bits(v))))
    step_bytes = qpool.view(-1, SUB)[(boff.view(-1) // SUB)].cpu().numpy()
    step_ok = bool(np.array_equal(step_bytes, O.quantize_blocks(_bits(kk), _bits(vv))))
    return {"prefill_subblocks": 112, "prefill_us": round(t_pre * 1e6, 1),
            "prefill_subblocks_per_s": round(112 / t_pre, 1), "prefill_tok_per_s": round(112 * 256 / t_pre, 1),
            "prefill_gbs": round(112 * per / t_pre / 1e9, 1),
            "step_flush_subblocks": B, "step_flush_us": round(t_step * 1e6, 1),
            "step_flush_gbs": round(B * per / t_step / 1e9, 1),
            "bit_exact": pre_ok and step_ok,
            "bit_exact_detail": {"prefill_112_subblocks": pre_ok, "step_flush_256_subblocks": step_ok,
                                 "against": "oracle/kv800_oracle.c quantize_blocks (pinned to reference goldens)"},
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


# ---------------------------------------------------------------- timing helpers
def timed_windows(torch, step, steps, windows, world, dist, dev):
    """`windows` timed windows of exactly `steps` steps each, every window bracketed by a barrier (N > 1) and a
    device synchronize on both sides and timed with CUDA events on the launching stream; the max over ranks per window.
    -> list of window seconds."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out = []
    for _ in range(windows):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 1e3
        if world > 1:
            tt = torch.tensor([t], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        out.append(t)
    return out


def window_summary(ts, steps):
    return {"windows": len(ts), "steps_per_window": steps, "reported": "median window",
            "ms_per_step_median": round(statistics.median(ts) / steps * 1e3, 4),
            "ms_per_step_min": round(min(ts) / steps * 1e3, 4), "ms_per_step_max": round(max(ts) / steps * 1e3, 4)}


def kernel_roofline(kv800, torch, dev, L0, q0, c32, s32, reps=10):
    """The dominant kernel, timed alone: the quantized phase of one quantized-layer decode (the schedule scan +
    qdecode_mma) by CUDA events on the launching stream, L2 flushed before every launch; algorithmic bytes = the
    layer's sub-blocks read once.  Also the whole layer decode (quantized + exact partials + merge)."""
    flushbuf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(3):
        kv800.decode(L0.P, q0, c32, s32)
    kt, lt = [], []
    for _ in range(reps):
        flushbuf.fill_(1)
        _, ms = kv800.decode_timed(L0.P, q0, c32, s32)
        kt.append(ms["quantized_ms"] / 1e3)
        lt.append((ms["quantized_ms"] + ms["exact_ms"] + ms["combine_ms"]) / 1e3)
    del flushbuf
    return statistics.median(kt), statistics.median(lt)


def config1_bench(kv800, torch, dev, hbm, peak_kind, reps=50):
    """one quantized attention layer, 4 sequences x 2,048 tokens (7 sub-blocks + 256
    exact tokens each), shuffled pages; 3,530,752 cache bytes per call.  Per-call device time by CUDA events with L2
    flushed before every call (the data would otherwise sit in L2), and back-to-back for context; parity of all 4
    rows against the oracle."""
    import inputs as I
    gen = torch.Generator().manual_seed(31)
    torch.manual_seed(31)
    L = Layer(kv800, torch, dev, 4, 2048, 0, gen)
    q = torch.randn(4, 16, 128, device=dev).to(torch.bfloat16)
    cs, sn = I.rope_tables(2048 + 64)
    c32 = torch.from_numpy(cs.view(np.int16)).view(torch.bfloat16).to(dev)
    s32 = torch.from_numpy(sn.view(np.int16)).view(torch.bfloat16).to(dev)
    flushbuf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(5):
        out = kv800.decode(L.P, q, c32, s32)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cold = []
    for _ in range(reps):
        flushbuf.fill_(1)
        e0.record()
        kv800.decode(L.P, q, c32, s32)
        e1.record()
        torch.cuda.synchronize()
        cold.append(e0.elapsed_time(e1) / 1e3)
    e0.record()
    for _ in range(200):
        kv800.decode(L.P, q, c32, s32)
    e1.record()
    torch.cuda.synchronize()
    warm = e0.elapsed_time(e1) / 1e3 / 200
    # the call's device time without the host's launch gaps: one decode captured in a CUDA graph (it makes no host
    # sync), replayed with L2 flushed before each replay
    graph_t = None
    try:
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            kv800.decode(L.P, q, c32, s32)
        torch.cuda.current_stream(dev).wait_stream(side)
        with torch.cuda.graph(g):
            gout = kv800.decode(L.P, q, c32, s32)
        gt = []
        for _ in range(reps):
            flushbuf.fill_(1)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            gt.append(e0.elapsed_time(e1) / 1e3)
        assert np.array_equal(_bits(gout), _bits(out))
        graph_t = statistics.median(gt)
        del g
    except Exception as ex:                                   # report, do not fail the bench
        graph_t = f"capture failed: {type(ex).__name__}: {str(ex)[:120]}"
    t = statistics.median(cold)
    nbytes = L.algo_bytes()
    rel, mx = parity_metrics(_bits(out), sample_refs([L], [q], c32, s32, range(4))[0])
    del flushbuf
    return {"workload": "config 1: 1 quantized layer, 4 seq x 2048 tokens (7 sub-blocks + 256 exact each), "
                        "16q/4kv/128, shuffled pages", "bytes_per_call": nbytes,
            "us_per_call": round(t * 1e6, 2), "us_per_call_back_to_back": round(warm * 1e6, 2),
            "device_us_per_call": round(graph_t * 1e6, 2) if isinstance(graph_t, float) else graph_t,
            "timing": f"us_per_call: kv800.decode from Python, median of {reps} calls, L2 flushed before each "
                      f"(host launch gaps included); back-to-back: 200 calls, L2-resident; device_us_per_call: the "
                      f"same call as a CUDA graph, median of {reps} replays, L2 flushed before each",
            "tok_per_s": round(4 / t, 1),
            "roofline": {"bound": "hbm", "achieved": round(nbytes / t / 1e9, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(nbytes / t / 1e9 / hbm, 4), "peak_source": peak_kind,
                         "note": "3.5 MB per call: launch / latency bound, not bandwidth bound"},
            "parity": {"rows": 4, "rel_l2": rel, "max_abs": mx, "ok": rel <= 1e-2 and mx <= 2e-2,
                       "against": "oracle/kv800_oracle.c decode (pinned to reference torch_decode goldens)"},
            "gpu_launches_per_call": 3}


# ---------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--windows", type=int, default=25, help="timed windows of --steps steps; the median is reported")
    ap.add_argument("--impl", default="cuda", choices=("cuda", "reference"))
    ap.add_argument("--cpu-seqs", type=int, default=64, help="sequences of the oracle-port CPU sample")
    ap.add_argument("--cpu-reps", type=int, default=3, help="passes of the CPU samples (median)")
    ap.add_argument("--ref-seqs", type=int, default=1, help="sequences per step of the reference torch_decode sample")
    ap.add_argument("--check-rows", type=int, default=2, help="rows per GPU checked against the oracle")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baselines (profiling runs)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--eager", action="store_true",
                    help="time the step as eager launches instead of one CUDA graph of the 6 layer decodes")
    ap.add_argument("--no-flush", action="store_true", help="skip the quantize / flush measurement")
    ap.add_argument("--no-next", action="store_true", help="skip the vLLM-step / prefill / train / sliding measurement")
    ap.add_argument("--no-config1", action="store_true", help="skip the config 1 measurement")
    ap.add_argument("--no-ragged", action="store_true", help="skip the config 4 (ragged rows) measurement")
    ap.add_argument("--seqs", type=int, default=B_PER_GPU, help="sequences per GPU (profiling: smaller cases)")
    ap.add_argument("--ctx", type=int, default=N_CTX, help="context length (profiling: smaller cases)")
    ap.add_argument("--workload", default="config3", choices=("config3", "ragged"),
                    help="config3 (the metric's workload) or ragged (BASELINE config 4 alone: 2,048 rows of U[1K, 32K] "
                         "tokens sharded over the ranks, strong scaling)")
    ap.add_argument("--pool-gb", type=float, default=150.0, help="ragged: the sub-block pool per GPU (GB)")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)
    a.windows = max(a.windows, 1)

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
        line = ragged_main(a, kv800, torch, dist, dev, rank, world, local, n_gpus)
        if world > 1:
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(line), flush=True)
        return
    layers, qs, c32, s32 = build_workload(kv800, torch, dev, rank, B=a.seqs, n=a.ctx)
    torch.cuda.synchronize()
    step_bytes = sum(L.algo_bytes() for L in layers)
    quant_bytes = sum(L.B * L.nq * SUB for L in layers)   # the sub-block part; the rest is exact tokens and sinks
    hbm, peak_kind = peaks()

    def step():
        return [kv800.decode(L.P, q, c32, s32) for L, q in zip(layers, qs)]

    for _ in range(a.warmup):
        outs = step()
    torch.cuda.synchronize()
    # the step's 6 layer decodes captured once as a CUDA graph and replayed, as a serving engine replays its decode
    # step (the decode makes no host sync, so it captures; the launches keep their programmatic dependencies); the
    # eager step is timed beside it
    timed_step, graph = step, None
    if not a.eager:
        gs = torch.cuda.Stream()
        gs.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(gs):
            step()
            gs.synchronize()
            with torch.cuda.graph(graph, stream=gs):
                outs = step()
        torch.cuda.current_stream().wait_stream(gs)
        torch.cuda.synchronize()
        timed_step = graph.replay
        for _ in range(a.warmup):
            graph.replay()
        torch.cuda.synchronize()
    with Clocks(local) as clk:
        wins = timed_windows(torch, timed_step, a.steps, a.windows, world, dist, dev)
    t = statistics.median(wins)
    wins_eager = wins if graph is None else timed_windows(torch, step, a.steps, max(3, a.windows // 5), world, dist,
                                                          dev)
    clocks = clk.summary()
    value = a.seqs * a.steps * n_gpus / t
    launches_per_step = sum(3 if L.nq else 1 for L in layers)   # qsched + qdecode + xdecode (merge included)

    # ---- correctness of what was timed: rows of this rank's outputs against the oracle on the same pools, gathered
    # to rank 0 over NCCL at N > 1 (the only use of a collective besides the timing reduction)
    rows = list(range(min(a.check_rows, a.seqs)))
    got = np.stack([_bits(o[rows]) for o in outs])                  # (layers, rows, 16, 128)
    ref = sample_refs(layers, qs, c32, s32, rows)
    if world > 1:
        from lfm3_kv800 import dp
        gtot = dp.gather_rows(torch.from_numpy(got.view(np.int16)).to(dev).transpose(0, 1).contiguous(),
                              [rank * len(rows) + i for i in range(len(rows))], world * len(rows), dev)
        rtot = dp.gather_rows(torch.from_numpy(ref.view(np.int16)).to(dev).transpose(0, 1).contiguous(),
                              [rank * len(rows) + i for i in range(len(rows))], world * len(rows), dev)
        if rank == 0:
            got = gtot.cpu().numpy().view(np.uint16).swapaxes(0, 1)
            ref = rtot.cpu().numpy().view(np.uint16).swapaxes(0, 1)
    per_layer = [parity_metrics(got[i], ref[i]) for i in range(len(layers))]
    parity = {"rows_per_gpu": len(rows), "rows_checked": int(got.shape[1]), "layers": len(layers),
              "rel_l2_max": max(r for r, _ in per_layer), "max_abs_max": max(m for _, m in per_layer),
              "ok": all(r <= 1e-2 and m <= 2e-2 for r, m in per_layer),
              "against": "oracle/kv800_oracle.c decode on the same pools (pinned to reference torch_decode goldens)",
              "gathered": "NCCL all_gather of every rank's checked rows to rank 0" if world > 1 else None}

    # ---- dominant kernel: qdecode_mma (the largest share of the decode kernels' device time in the ncu launch list)
    L0, q0 = layers[0], qs[0]
    kdur, ldur = kernel_roofline(kv800, torch, dev, L0, q0, c32, s32)
    kbytes = L0.B * L0.nq * SUB
    # DRAM traffic of qdecode_mma from one ncu capture on 64 x 16,384 (4,032 sub-blocks: 209.5 MB read + 5.1 MB
    # written), scaled to this launch by sub-blocks (traffic grows in proportion: reads are the sub-blocks plus
    # the cos / sin rows, writes the split partials)
    traffic = round((209.5e6 + 5.1e6) * (L0.B * L0.nq) / 4032) if a.ctx == N_CTX and a.seqs == B_PER_GPU else None
    roofline = {"bound": "hbm", "achieved": round(kbytes / kdur / 1e9, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(kbytes / kdur / 1e9 / hbm, 4), "traffic": traffic, "peak_source": peak_kind,
                "kernel": "qdecode_mma (+ its 1-CTA schedule scan)", "bytes_per_launch": kbytes,
                "launch_us": round(kdur * 1e6, 1),
                "layer_decode": {"bytes": L0.algo_bytes(), "bytes_quantized": kbytes,
                                 "bytes_exact": L0.algo_bytes() - kbytes, "us": round(ldur * 1e6, 1),
                                 "achieved_gbs": round(L0.algo_bytes() / ldur / 1e9, 1),
                                 "kernels": "qsched + qdecode_mma + xdecode_tma (with the merge of each row's partials)"}}
    # a window layer (4 sinks + 256 exact tokens per row): xdecode_tma with each row's merge, L2 flushed
    LW, qw = layers[QUANT_LAYERS], qs[QUANT_LAYERS]
    _, wdur = kernel_roofline(kv800, torch, dev, LW, qw, c32, s32)
    window = {"bytes": LW.algo_bytes(), "us": round(wdur * 1e6, 1),
              "achieved_gbs": round(LW.algo_bytes() / wdur / 1e9, 1), "frac": round(LW.algo_bytes() / wdur / 1e9 / hbm, 4),
              "kernel": "xdecode_tma (one warp per row, split and head) with the merges, one window layer, L2 flushed"}

    # ---- end to end through the public API with host buffers
    e2e = None
    if not a.no_e2e:
        e2e = e2e_bench(a, kv800, torch, dist, dev, world, n_gpus, layers, qs, c32, s32)

    # ---- flush / quantize
    flush = None if a.no_flush else flush_bench(kv800, torch, dev)
    nxt = None
    if not a.no_next and world == 1:
        nxt = next_rows_bench(kv800, torch, dev)
    cfg1 = None
    if not a.no_config1 and world == 1:
        cfg1 = config1_bench(kv800, torch, dev, hbm, peak_kind)

    cpu = cpu_port = None
    if rank == 0 and world == 1 and not a.no_cpu:
        S = min(a.cpu_seqs, a.seqs)
        tps, sec = cpu_sample(layers, qs, c32, s32, S, reps=a.cpu_reps)
        cpu_port = {"value": round(tps, 2), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                    "sample": f"{S} of the {a.seqs} sequences x {a.ctx:,} tokens, all 6 layers, oracle/kv800_oracle.c "
                              f"(the C restatement of torch_decode, OpenMP over sequence x kv head), median of "
                              f"{a.cpu_reps} passes of {sec:.2f} s"}
        rw = run_ref_worker(a.ref_seqs, a.ctx, a.cpu_reps, 1, config1_reps=0 if cfg1 is None else 20)
        if rw is not None:
            st = statistics.median(rw["step_s"])
            cpu = {"value": round(a.ref_seqs / st, 3), "unit": "tok/s", "cores": rw["threads"], "kind": "reference",
                   "sample": f"{a.ref_seqs} sequence(s) x {a.ctx:,} tokens x 6 layers per step (4 quantized + 2 "
                             f"window, the config 3 shape), the reference's own torch_decode.decode on the host "
                             f"CPU (torch {rw['torch']}, {rw['threads']} threads), median of {len(rw['step_s'])} "
                             f"steps of {st:.2f} s"}
            if cfg1 is not None and rw.get("config1_call_s"):
                c1 = statistics.median(rw["config1_call_s"])
                cfg1["cpu_baseline"] = {"value": round(c1 * 1e6, 1), "unit": "us per call", "cores": rw["threads"],
                                        "kind": "reference",
                                        "sample": f"torch_decode.decode, 4 x 2048, median of "
                                                  f"{len(rw['config1_call_s'])} calls"}
                cfg1["speedup_vs_reference_cpu"] = round(c1 / (cfg1["us_per_call"] * 1e-6), 1)
        else:
            cpu = dict(cpu_port, note="the reference package is not staged (oracle/_ref); its C port stands in")

    ragged = None
    if not a.no_ragged:
        del outs, layers, qs, L0, q0
        torch.cuda.empty_cache()
        ragged = ragged_main(a, kv800, torch, dist, dev, rank, world, local, n_gpus, windows=min(a.windows, 10))

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
                           "l2": "inputs larger than L2 (1.87 GB per step); kernel timing flushes L2 per launch",
                           "timing": dict(window_summary(wins, a.steps),
                                          step="eager launches" if graph is None else
                                          "one CUDA graph of the 6 layer decodes, replayed",
                                          eager_ms_per_step_median=round(statistics.median(wins_eager) / a.steps
                                                                         * 1e3, 4))},
                "hbm_gbs_step": round(step_bytes * a.steps / t / 1e9, 1),
                "hbm_frac_step": round(step_bytes * a.steps / t / 1e9 / hbm, 4),
                "bytes_per_step_per_gpu": step_bytes,
                "bytes_per_step_split": {"quantized": quant_bytes, "exact": step_bytes - quant_bytes},
                "roofline": roofline, "window_layer": window, "parity": parity,
                "cpu_baseline": cpu,
                "cpu_baseline_port": cpu_port, "e2e": e2e,
                "gpu_launches": launches_per_step * a.steps, "clocks": clocks, "config1": cfg1, "flush": flush,
                "ragged": ragged, "next_rows": nxt}
        print(json.dumps(line), flush=True)


def e2e_bench(a, kv800, torch, dist, dev, world, n_gpus, layers, qs, c32, s32):
    """The metric through the public API with host buffers: every step uploads its inputs (6 x q, the current token's
    K / V) from pinned host memory, writes the token into its exact page (kv800.write_exact), decodes (kv800.decode)
    and reads the 6 outputs back, all inside the timed region.  Uploads and token writes run on their own stream,
    queued at the step's start, so layer i + 1's inputs arrive and its token lands while layer i decodes; layer i's
    decode waits for its own layer's write, and its output is read back while layer i + 1 decodes.  The device input
    buffers and pages are reused across steps: the next step's uploads and writes queue behind this step's last
    read-back, which waits for the last decode, so nothing overwrites data a decode still reads."""
    B = a.seqs
    nl = len(layers)
    hq = [q.cpu().pin_memory() for q in qs]
    hk = torch.randn(nl, B, 4, 128).to(torch.bfloat16).pin_memory()
    hv = torch.randn(nl, B, 4, 128).to(torch.bfloat16).pin_memory()
    hout = [torch.empty(B, 16, 128, dtype=torch.bfloat16).pin_memory() for _ in layers]
    seqs = torch.arange(B, dtype=torch.int32, device=dev)
    posv = torch.full((B,), a.ctx - 1, dtype=torch.int64, device=dev)
    main_s, cps = torch.cuda.current_stream(dev), torch.cuda.Stream(dev)
    dq = [torch.empty_like(q) for q in qs]
    dk = torch.empty(nl, B, 4, 128, dtype=torch.bfloat16, device=dev)
    dv = torch.empty_like(dk)
    ready = [torch.cuda.Event() for _ in layers]
    done = [torch.cuda.Event() for _ in layers]

    def e2e_step():
        with torch.cuda.stream(cps):
            for i, L in enumerate(layers):
                dq[i].copy_(hq[i], non_blocking=True)
                dk[i].copy_(hk[i], non_blocking=True)
                dv[i].copy_(hv[i], non_blocking=True)
                kv800.write_exact(L.epool, L.eoff, EBS, EBS * 256, 256, 128, dk[i], dv[i], seqs, posv)
                ready[i].record(cps)
        for i, L in enumerate(layers):
            main_s.wait_event(ready[i])
            o = kv800.decode(L.P, dq[i], c32, s32)
            done[i].record(main_s)
            cps.wait_event(done[i])
            with torch.cuda.stream(cps):
                hout[i].copy_(o, non_blocking=True)
            o.record_stream(cps)
        main_s.wait_stream(cps)      # the step ends when its last read-back has landed
        return hout

    for _ in range(a.warmup):
        e2e_step()
    torch.cuda.synchronize()
    wins = timed_windows(torch, e2e_step, a.steps, max(1, a.windows // 3), world, dist, dev)
    te = statistics.median(wins)
    h2d = sum(x.numel() * x.element_size() for x in hq) + hk.numel() * 2 + hv.numel() * 2
    d2h = sum(x.numel() * x.element_size() for x in hout)
    return {"value": round(a.seqs * a.steps * n_gpus / te, 1), "unit": "tok/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": round(te / a.steps * 1e3, 4),
            "timing": window_summary(wins, a.steps)}


def ragged_main(a, kv800, torch, dist, dev, rank, world, local, n_gpus, windows=None):
    """Config 4: every rank decodes its LPT share of the 2,048 ragged rows through all 6 layers per step; value =
    2,048 x steps / max-over-ranks device time (strong scaling: the total work is fixed).  -> the line's dict (with
    --workload ragged the whole line, otherwise the "ragged" object of the config 3 line)."""
    layers, qs, c32, s32, rows, pool_bytes = build_ragged(kv800, torch, dev, rank, world, a.pool_gb)
    torch.cuda.synchronize()
    step_bytes = sum(L.algo_bytes() for L in layers)

    def step():
        return [kv800.decode(L.P, q, c32, s32) for L, q in zip(layers, qs)]

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    nwin = windows or a.windows
    with Clocks(local) as clk:
        wins = timed_windows(torch, step, a.steps, nwin, world, dist, dev)
    tmax = statistics.median(wins)
    bytes_all = step_bytes
    if world > 1:
        bb = torch.tensor([float(step_bytes)], device=dev, dtype=torch.float64)
        dist.all_reduce(bb)
        bytes_all = float(bb.item())
        dist.barrier()
    # dominant kernel on this rank: the quantized phase of layer 0 (L2 flushed)
    L0, q0 = layers[0], qs[0]
    kdur, _ = kernel_roofline(kv800, torch, dev, L0, q0, c32, s32)
    kbytes = sum(L0.nq_rows) * SUB
    hbm, peak_kind = peaks()
    clocks = clk.summary()
    launches_per_step = sum(3 if L.nqmax else 1 for L in layers)   # qsched + qdecode + xdecode (merge included)
    del layers, qs, L0, q0
    torch.cuda.empty_cache()
    return {"metric": METRIC, "value": round(RAGGED_ROWS * a.steps / tmax, 1), "unit": "tok/s", "n_gpus": n_gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(tmax / a.steps * 1e3, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8+bf16 (fp32 math)",
            "data": "synthetic",
            "config": {"workload": f"config 4: {RAGGED_ROWS} rows, lengths U[{RAGGED_LO}, {RAGGED_HI}] (seed "
                                   f"2048), LPT-sharded over {n_gpus} GPU(s), 4 quantized + 2 window layers, "
                                   f"sub-blocks scattered over a {pool_bytes / 1e9:.0f} GB pool per GPU",
                       "rows_rank0": len(rows), "parallelism": f"dp{n_gpus} (LPT row sharding, no collective)",
                       "timing": window_summary(wins, a.steps)},
            "hbm_gbs_step": round(bytes_all * a.steps / tmax / 1e9, 1),
            "bytes_per_step_all_gpus": int(bytes_all),
            "roofline": {"bound": "hbm", "achieved": round(kbytes / kdur / 1e9, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(kbytes / kdur / 1e9 / hbm, 4), "traffic": None, "peak_source": peak_kind,
                         "kernel": "qdecode_mma (+ its 1-CTA schedule scan), rank 0, layer 0",
                         "bytes_per_launch": kbytes, "launch_us": round(kdur * 1e6, 1)},
            "cpu_baseline": None, "e2e": None,
            "gpu_launches": launches_per_step * a.steps, "clocks": clocks}


def reference_arm(a, rank, world, n_gpus):
    """The reference's CPU path for this step on the host cores: its own torch_decode.decode (imported from the staged
    copy under oracle/_ref in a child process, all host threads) on a bounded sample of the config 3 workload, S
    sequences x 32,768 tokens through the 4 quantized + 2 window layers per step, exactly K steps after W warm-ups,
    scaled to tok/s.  When the reference is not staged, the C port of torch_decode (oracle/kv800_oracle.c) stands in
    and the line says so.  On N > 1 ranks only rank 0 runs it."""
    if rank != 0:
        return
    S = max(1, a.ref_seqs)
    rw = run_ref_worker(S, N_CTX, a.steps, a.warmup)
    if rw is not None:
        dt = statistics.median(rw["step_s"])
        v = S / dt
        cores = rw["threads"]
        base = {"value": round(v, 3), "unit": "tok/s", "cores": cores, "kind": "reference",
                "sample": f"{S} sequence(s) x 32,768 tokens x 6 layers per step (of the 64 per GPU), the reference's "
                          f"own torch_decode.decode (lfm3_kv800/torch_decode.py:27-80) on the host CPU, torch "
                          f"{rw['torch']}, {cores} threads, median of {len(rw['step_s'])} steps"}
    else:
        v, dt, base = port_arm(a)
    line = {"metric": METRIC, "value": round(v, 3), "unit": "tok/s", "n_gpus": n_gpus, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(dt * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8+bf16 (fp32 math)", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "config 3: 64 seq x 32768 ctx per GPU, 4 quantized (127 sub-blocks + 256 exact) + "
                                   "2 window (4 sinks + 256) layers, 16q/4kv/128, shuffled pages",
                       "seqs_per_gpu": B_PER_GPU, "ctx": N_CTX, "layers": QUANT_LAYERS + WINDOW_LAYERS,
                       "parallelism": "host cores (reference CPU path)"},
            "cpu_baseline": base,
            "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def port_arm(a):
    """The C port of torch_decode (oracle/kv800_oracle.c, all host threads) on cores / 4 (at most 4) sequences per
    step, for the K steps after W warm-ups: the reference arm when the reference package is not staged."""
    import torch  # noqa: F401  (the oracle front end imports numpy only; torch keeps the import order of the main arm)
    from oracle import oracle as O
    O.lib()
    S = max(1, min(4, (os.cpu_count() or 4) // 4))
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
                 sv=sk, skoff=np.arange(S, dtype=np.int64) * NSINK * 512,
                 svoff=np.arange(S, dtype=np.int64) * NSINK * 512, N=np.full(S, N_CTX, np.int32),
                 NQ=np.full(S, nq, np.int32), nqmax=nq, win=win)
        q = I.f32_to_bf16(rs.standard_normal((S, 16, 128)).astype(np.float32))
        per_layer.append((P, q))

    def step():
        for P, q in per_layer:
            O.decode(P, q, cs, sn)

    for _ in range(a.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        step()
    dt = (time.perf_counter() - t0) / a.steps
    base = {"value": round(S / dt, 2), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{S} sequences x 32,768 tokens x 6 layers per step, oracle/kv800_oracle.c decode (OpenMP over "
                      f"sequence x kv head); the reference package was not staged under oracle/_ref"}
    return S / dt, dt, base


if __name__ == "__main__":
    if len(sys.argv) >= 3 and sys.argv[1] == "--ref-worker":
        ref_worker(sys.argv[2])
    else:
        main()
