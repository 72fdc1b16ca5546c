"""Benchmark of the B200 paged-MLA attention path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config decode|decode_fp8|mtp|prefill|longctx|cpu|kv_write|kv_write_fp8|
                              sparse|sparse_fp8|prologue|prologue_nope]
                    [--cpu-sample S]

A step is one launch of the attention path (scheduler, tcgen05 attention kernel, combine) over
one batch of synthetic, seeded input already resident in HBM. The default workload is bf16 paged
decode: 64 sequences x 1 query token, 128 heads, 576-wide latent+RoPE rows, 512-wide output,
cached lengths uniform in [4096, 8192], 64-row pages from a permuted pool. The pool (~0.5 GB)
exceeds L2 (126 MB), so every step reads its rows from HBM; no L2 flush is needed.
``--config decode_fp8`` is the same batch with FP8 E4M3 rows (512 codes + 4 f32 scales, stored
544 bytes apart; q 512 wide). ``--config kv_write_fp8`` / ``kv_write`` time the KV cache writer
instead: 128 sequences x 2048 new bf16 latent rows per step (512 wide, quantized to FP8 rows at
stride 544; or 576 wide, copied to 1152-byte rows) scattered into a permuted page pool; the metric
is rows written per second. ``--config sparse`` / ``sparse_fp8`` time sparse top-k decode: 64
sequences x 1 token, 32 heads, 32K cached positions, 2051 index entries per token of which 2048
are valid, bf16 or FP8 rows; four index sets rotate between steps so the rows read are not
L2-resident. ``--config prologue`` / ``prologue_nope`` time the MLA prologue of one decode step
(64 tokens: projections, norms, absorption, RoPE, cache write) with L2 flushed between steps.

With N ranks (torchrun, one GPU each) the job holds N x 64 sequences drawn from the same seeded
stream and sharded by token count (weak scaling); there is no collective on the data path.
``value`` is total query tokens / max-over-ranks device time. ``e2e`` is the same metric
through the C ABI with the step's inputs (q, block tables, positions, lengths) copied from
pinned host memory and the results (out, lse) copied back inside the timed region.
``--impl reference`` times the reference's CPU algorithm (the oracle's float64 restatement of
``mla_attention_core``; the reference itself is Python and is not present on the GPU host) on
all host cores, on a bounded sample of the same workload, on rank 0 only.
"""

import argparse
import contextlib
import json
import math
import multiprocessing as mp
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "tensorquay-engine_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "MLA paged decode tokens/s"
UNIT = "tokens/s"
LAUNCHES_PER_STEP = 3  # scheduler + attention + combine


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), \
            "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# Sequences per rank when a job of N ranks is sharded (weak scaling: N times the one-GPU batch).
SHARD_BASE = {"decode": 64, "decode_fp8": 64, "mtp": 512, "prefill": 8, "longctx": 4, "cpu": 4,
              "sparse": 64, "sparse_fp8": 64}


def job_batch(name, world, strong):
    """Sequences of the whole job: the configuration's batch (one GPU, or strong scaling) or
    N times it (weak scaling over N ranks)."""
    return None if (world == 1 or strong or name == "cpu") else SHARD_BASE[name] * world


def workload_for(name, world, rank, strong=False):
    """This rank's share of the job: whole sequences, balanced by token count."""
    from tq_mla import inputs

    full = inputs.config(name, batch=job_batch(name, world, strong))
    return full if world == 1 else inputs.shard(full, world, rank)


def config_block(name, world, sequences, tokens, heads, width, pool_bytes, parallelism=None,
                 strong=False):
    """The line's ``config``: the workload's fixed description (no measured values), the same
    for the GPU arm and the reference arm of one configuration and rank count. ``sequences``,
    ``tokens`` and ``pool_bytes`` are the whole job's."""
    return {
        "workload": name if world == 1 else (
            f"{name} over {world} ranks (fixed batch)" if strong
            else f"{name} x{world} ranks (token-sharded)"),
        "sequences": int(sequences), "query_tokens": int(tokens), "heads": int(heads),
        "row_width": int(width), "value_width": 512, "page_rows": 64,
        "parallelism": parallelism or f"sequence-shard x{world}",
        "l2": "inputs larger than L2 (KV pool %.0f MB per GPU on average), no flush"
              % (pool_bytes / world / 1e6),
    }


# ------------------------------------------------------------------------- clocks

def clock_log_path(args, rank):
    """Where the nvidia-smi samples of the timed region go: ``--clock-log`` (a file name, with
    ``{rank}`` replaced), else a file in the system temporary directory."""
    if getattr(args, "clock_log", None):
        return args.clock_log.replace("{rank}", str(rank))
    return os.path.join(tempfile.gettempdir(), f"tq_bench_clocks_rank{rank}.csv")


class ClockSampler:
    def __init__(self, device_index, path):
        self.path = path
        self.proc = None
        self.device_index = device_index

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not Path(self.path).exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------- CPU leg

BLAS_ENV = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS", "BLIS_NUM_THREADS",
            "NUMEXPR_NUM_THREADS", "VECLIB_MAXIMUM_THREADS")


def _cpu_proc(conn, name, batch, seqs):
    """One CPU worker: builds its sequences' inputs once from the seeded generator (untimed),
    then, per step, times the block-table gather plus the float64 attention of each of them.

    Inputs come from the oracle's NumPy generator: the same Philox streams as the GPU batch,
    with no product library loaded. FP8 rows are random finite codes with a fixed tile scale
    (their values do not change the float64 work); the timed part then also decodes them.
    """
    sys.path.insert(0, str(ROOT))
    from oracle import fp8 as ofp8, generate as ogen, mla as omla

    w = ogen.config(name, batch=batch)
    fp8 = w.kv_format == "fp8_e4m3"
    jobs = []
    for b in seqs:
        n, t = int(w.kv_len[b]), int(w.q_per_seq[b])
        pages = (n + 63) // 64
        table = w.page_table[b:b + 1, :pages].copy()
        # A private pool holding just this sequence's pages, at their permuted page slots.
        local = np.argsort(np.argsort(table[0])).astype(np.int32)[None, :]
        pos = np.arange(n)
        rows = local[0, pos // 64].astype(np.int64) * 64 + pos % 64
        if fp8:
            rng = np.random.default_rng(int(w.seed) * 1000 + b)
            pool = np.zeros((pages * 64, 544), np.uint8)
            codes = rng.integers(0, 0x7E, size=(n, 512), dtype=np.uint8)
            codes |= rng.integers(0, 2, size=(n, 512), dtype=np.uint8) << 7
            pool[rows, :512] = codes
            pool[rows, 512:528] = np.full((n, 4), 4.0 / 448.0, np.float32).view(np.uint8)
        else:
            pool = np.zeros((pages * 64, w.width))
            pool[rows] = w.sequence_rows(b)
        q = w.sequence_queries(b)
        q_pos = (w.prefix[b] + np.arange(t)).astype(np.int32)
        jobs.append((q, pool, local, np.zeros(t, np.int32), q_pos, np.array([n]), t))
    conn.send(("ready", sum(j[-1] for j in jobs)))
    while True:
        msg = conn.recv()
        if msg is None:
            break
        t0 = time.perf_counter()
        for q, pool, table, seq_id, q_pos, kv_len, _ in jobs:
            values = ofp8.dequant_rows(pool) if fp8 else pool
            omla.paged_attention(q, values, table, seq_id, q_pos, kv_len, scale=w.scale,
                                 value_dim=512)
        conn.send(time.perf_counter() - t0)
    conn.close()


class CpuTeam:
    """``procs`` spawned processes, each with one BLAS thread, over a fixed set of sequences.

    The thread limits are put into this process's environment before the children start, so
    each child's BLAS library sees them when it loads; the parent's own settings are restored
    afterwards. A step sends every worker its go signal and ends when the last one replies: the
    step time is that wall-clock interval (the slowest process plus the message round trip).
    """

    def __init__(self, name, batch, seqs, procs):
        seqs = list(seqs)
        procs = max(1, min(procs, len(seqs)))
        saved = {k: os.environ.get(k) for k in BLAS_ENV}
        for k in BLAS_ENV:
            os.environ[k] = "1"
        ctx = mp.get_context("spawn")
        self.conns, self.procs = [], []
        try:
            for i in range(procs):
                a, b = ctx.Pipe()
                p = ctx.Process(target=_cpu_proc, args=(b, name, batch, seqs[i::procs]),
                                daemon=True)
                p.start()
                self.conns.append(a)
                self.procs.append(p)
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v
        self.tokens = sum(c.recv()[1] for c in self.conns)
        self.sequences = len(seqs)

    def step(self):
        t0 = time.perf_counter()
        for c in self.conns:
            c.send(True)
        busy = max(c.recv() for c in self.conns)
        return time.perf_counter() - t0, busy

    def close(self):
        for c in self.conns:
            c.send(None)
        for p in self.procs:
            p.join(timeout=30)


def cpu_sample(name, world, strong=False):
    """The sequences a CPU step covers: the whole batch for the decode batches, else a fixed
    spread of sequences of the (unsharded) job, so a step stays within about a second."""
    sys.path.insert(0, str(ROOT))
    from oracle import generate as ogen

    batch = job_batch(name, world, strong)
    w = ogen.config(name, batch=batch)
    cap = {"decode": 64, "decode_fp8": 64, "cpu": 4, "mtp": 16, "prefill": 1,
           "longctx": 1}.get(name, 8)
    n = min(w.sequences, cap)
    picks = np.unique(np.linspace(0, w.sequences - 1, n).astype(int))
    return w, batch, picks


def single_process_seconds(name, batch, seqs):
    """The same work in this process with its default BLAS threads (the second timing)."""
    from oracle import fp8 as ofp8, generate as ogen, mla as omla

    w = ogen.config(name, batch=batch)
    total, tokens = 0.0, 0
    for b in seqs:
        n, t = int(w.kv_len[b]), int(w.q_per_seq[b])
        if w.kv_format == "fp8_e4m3":
            rng = np.random.default_rng(b)
            raw = np.zeros((n, 544), np.uint8)
            raw[:, :512] = rng.integers(0, 0x7E, size=(n, 512), dtype=np.uint8)
            raw[:, 512:528] = np.full((n, 4), 4.0 / 448.0, np.float32).view(np.uint8)
            rows = None
        else:
            rows = w.sequence_rows(b)
        q = w.sequence_queries(b)
        table = np.arange((n + 63) // 64, dtype=np.int32)[None, :]
        q_pos = (w.prefix[b] + np.arange(t)).astype(np.int32)
        t0 = time.perf_counter()
        values = ofp8.dequant_rows(raw) if rows is None else rows
        omla.paged_attention(q, values, table, np.zeros(t, np.int32), q_pos, np.array([n]),
                             scale=w.scale, value_dim=512)
        total += time.perf_counter() - t0
        tokens += t
    return tokens, total


def _fp8_note(w):
    return " and FP8 E4M3 row decoding" if getattr(w, "kv_format", None) == "fp8_e4m3" or \
        getattr(w, "extra", {}).get("kv_format") == "fp8_e4m3" else ""


def kv_format_of(w):
    from tq_mla import _abi

    return _abi.KV_FP8_E4M3 if w.extra.get("kv_format") == "fp8_e4m3" else None


def cpu_measure(name, world, steps, warmup, single_seqs=8, strong=False):
    """Times the CPU path: ``steps`` steps of the sample over one process per host core, plus
    one pass over a few of its sequences in a single process with default BLAS threads."""
    w, batch, picks = cpu_sample(name, world, strong)
    cores = os.cpu_count() or 1
    team = CpuTeam(name, batch, picks, cores)
    try:
        for _ in range(warmup):
            team.step()
        walls = [team.step()[0] for _ in range(steps)]
    finally:
        team.close()
    st, ss = single_process_seconds(name, batch, picks[:single_seqs])
    value = team.tokens * len(walls) / sum(walls)
    sample = (f"{team.tokens} query tokens per step ({team.sequences} of {w.sequences} "
              f"sequences{'' if team.sequences == w.sequences else ', spread over the batch'}) of "
              f"{w.name}; inputs from the seeded generator (oracle/generate.py, no product "
              f"library); timed part = block-table gather{_fp8_note(w)} + float64 attention "
              f"(oracle restatement of mla_attention_core); {len(team.procs)} spawned processes x "
              f"1 BLAS thread, step = wall time until the last process finishes")
    return {
        "value": value, "unit": UNIT, "cores": len(team.procs), "kind": "port",
        "sample": sample, "steps": len(walls), "warmup": warmup,
        "ms_per_step": 1e3 * float(np.mean(walls)),
        "ms_per_step_p10_p50_p90": [1e3 * float(np.percentile(walls, p)) for p in (10, 50, 90)],
        "single_process": {"value": st / ss if ss > 0 else None, "unit": UNIT,
                           "tokens": st, "seconds": ss,
                           "sample": f"first {len(picks[:single_seqs])} sequences of the sample "
                                     f"in one process, default BLAS threads"},
        "host_cores": cores,
    }


def cpu_baseline(name, world):
    """The ``cpu_baseline`` object of the GPU arm's line (rank 0, one GPU)."""
    return cpu_measure(name, world, steps=10, warmup=1)


# ------------------------------------------------------------------------- KV writer

WRITER_SEQS, WRITER_ROWS_PER_SEQ = 128, 2048


KV_FP8_E4M3, KV_BF16_ROPE576 = 1, 2  # row formats of include/tq_mla.h


def writer_workload(name, rank=0):
    """Host arrays of one writer step: bf16 bits [R, W], page table, seq_id, pos (seeded)."""
    fmt = KV_FP8_E4M3 if name == "kv_write_fp8" else KV_BF16_ROPE576
    width = 512 if fmt == KV_FP8_E4M3 else 576
    stride = 544 if fmt == KV_FP8_E4M3 else 1152
    rng = np.random.default_rng(1000 + rank)
    slots = WRITER_ROWS_PER_SEQ // 64
    pages = WRITER_SEQS * slots
    table = rng.permutation(pages).astype(np.int32).reshape(WRITER_SEQS, slots)
    seq_id = np.repeat(np.arange(WRITER_SEQS, dtype=np.int32), WRITER_ROWS_PER_SEQ)
    pos = np.tile(np.arange(WRITER_ROWS_PER_SEQ, dtype=np.int32), WRITER_SEQS)
    return fmt, width, stride, pages, table, seq_id, pos, rng


def writer_cpu_baseline(name, rows=16384):
    """The oracle writer (numpy quantization + scatter) on a bounded sample of the step."""
    from oracle import kv_write as okw

    fmt, width, stride, pages, table, seq_id, pos, rng = writer_workload(name)
    x = (rng.standard_normal((rows, width))).astype(np.float32)
    bits = (x.view(np.uint32) >> 16).astype(np.uint16)
    pool = np.zeros((pages, 64, stride), np.uint8)
    t0 = time.perf_counter()
    okw.write(pool, bits, table, seq_id[:rows], pos[:rows], fmt)
    sec = time.perf_counter() - t0
    return {"value": rows / sec, "unit": "rows/s", "cores": 1, "kind": "port",
            "sample": f"{rows} of the step's {len(seq_id)} rows through oracle/kv_write.py "
                      f"(numpy, one process)", "seconds": sec}


def run_writer(args, world, rank, local_rank):
    import torch
    import torch.distributed as dist
    from tq_mla import ops

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    fmt, width, stride, pages, table, seq_id, pos, rng = writer_workload(args.config, rank)
    rows = len(seq_id)
    h_src = torch.randn((rows, width), generator=torch.Generator().manual_seed(7 + rank),
                        dtype=torch.float32).to(torch.bfloat16).pin_memory()
    src = h_src.to(dev)
    pool = torch.zeros((pages, 64, stride), dtype=torch.uint8, device=dev)
    d_table = torch.from_numpy(table).to(dev)
    d_seq = torch.from_numpy(seq_id).to(dev)
    d_pos = torch.from_numpy(pos).to(dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        ops.kv_write(src, pool, d_table, d_seq, d_pos, kv_format=fmt, flags=flags, stream=stream)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clock = ClockSampler(local_rank, clock_log_path(args, rank))
    barrier()
    torch.cuda.synchronize(dev)
    with clock:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    ms_step = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    # End to end: the step's rows copied in from pinned host memory, the flags read back.
    h_flags = torch.zeros(1, dtype=torch.int32).pin_memory()
    e2e_steps = max(3, min(args.steps, 50))
    barrier()
    torch.cuda.synchronize(dev)
    ev0.record(stream)
    for _ in range(e2e_steps):
        src.copy_(h_src, non_blocking=True)
        step()
        h_flags.copy_(flags, non_blocking=True)
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1)) / e2e_steps
    assert int(flags.item()) == 0, "writer flagged rows"
    payload = 528 if stride == 544 else 1152
    bytes_per_row = width * 2 + payload + 8  # bf16 source, payload written, seq_id + pos
    hbm, _, _, src_name = peaks()
    ach = rows * bytes_per_row / (ms_step * 1e-3) / 1e9
    result = {
        "metric": "KV rows written/s", "value": world * rows / (ms_step * 1e-3), "unit": "rows/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 -> fp8_e4m3" if stride == 544 else "bf16", "data": "synthetic",
        "config": {"workload": f"{args.config}: {WRITER_SEQS} sequences x {WRITER_ROWS_PER_SEQ} "
                               f"rows, width {width}, pool stride {stride}",
                   "rows": rows, "l2": "source %.0f MB + pool %.0f MB per step, above L2; no "
                   "flush" % (rows * width * 2 / 1e6, pages * 64 * stride / 1e6)},
        "e2e": {"value": world * rows / (e2e_ms * 1e-3), "unit": "rows/s",
                "h2d_bytes_per_step": rows * width * 2, "d2h_bytes_per_step": 4,
                "ms_per_step": e2e_ms},
        "gpu_launches": args.steps,
        "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                     "frac": ach / hbm, "traffic": None, "kernel": "kv_write_kernel",
                     "peak_source": f"{src_name} (MEASURED_PEAKS.json)",
                     "algorithmic_bytes_per_row": bytes_per_row},
        "clocks": clock.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = writer_cpu_baseline(args.config)
    if rank == 0:
        print(json.dumps(result), flush=True)


# ------------------------------------------------------------------------- MLA prologue

# One decode step's prologue: every sequence's new token, x -> (absorbed q, cache row).
# "prologue": the 576-wide form at the decode batch (128 heads of 128 + 64 RoPE, hidden 7168,
# Q rank 1536); "prologue_nope": the reference's no-RoPE model (64 heads of 256, hidden 4096,
# Q rank 1536) writing 528-byte FP8 rows.
PROLOGUE = {
    "prologue": dict(tokens=64, dm=7168, rq=1536, heads=128, dn=128, dr=64, fmt=2, row=1152),
    "prologue_nope": dict(tokens=64, dm=4096, rq=1536, heads=64, dn=256, dr=0, fmt=1, row=544),
}
L2_FLUSH_BYTES = 256 << 20


def prologue_host(name, seed=5):
    """Seeded weights and one decode token per sequence (positions uniform in [4096, 8192)),
    float32 arrays holding bf16-rounded values."""
    import torch

    c = PROLOGUE[name]
    g = np.random.default_rng(seed)
    dm, rq, h, dn, dr, t = c["dm"], c["rq"], c["heads"], c["dn"], c["dr"], c["tokens"]

    def bf(a):
        return torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16).float().numpy()

    w = dict(x=bf(g.standard_normal((t, dm))),
             w_qa=bf(g.standard_normal((rq, dm)) / math.sqrt(dm)),
             q_norm=bf(g.uniform(0.5, 1.5, rq)),
             w_qb=bf(g.standard_normal((h * (dn + dr), rq)) / math.sqrt(rq)),
             w_uk=bf(g.standard_normal((h, dn, 512)) / math.sqrt(dn)),
             w_kva=bf(g.standard_normal((512 + dr, dm)) / math.sqrt(dm)),
             kv_norm=bf(g.uniform(0.5, 1.5, 512)))
    pos = g.integers(4096, 8192, t).astype(np.int32)
    seq = np.arange(t, dtype=np.int32)
    slots = 128
    table = g.permutation(t * slots).astype(np.int32).reshape(t, slots)
    return c, w, pos, seq, table


def prologue_bytes(c):
    """Algorithmic bytes of one step: the weights, x, q and the rows written (plus pos, seq_id)."""
    dm, rq, h, dn, dr, t = c["dm"], c["rq"], c["heads"], c["dn"], c["dr"], c["tokens"]
    payload = {0: 1024, 1: 528, 2: 1152}[c["fmt"]]
    weights = 2 * (rq * dm + rq + h * (dn + dr) * rq + h * dn * 512 + (512 + dr) * dm + 512)
    return weights + t * (2 * dm + 2 * h * (512 + dr) + payload + 8)


def prologue_cpu_baseline(name, min_seconds=10.0):
    """The oracle's float64 prologue of the whole step (numpy BLAS on every host thread), repeated
    for at least ``min_seconds``, in tokens/s."""
    from oracle import prologue as opro

    c, w, pos, seq, table = prologue_host(name)
    w = {k: v.astype(np.float64) for k, v in w.items()}
    reps = 0
    t0 = time.perf_counter()
    while True:
        opro.prologue(**w, pos=pos, heads=c["heads"], nope_dim=c["dn"], rope_dim=c["dr"],
                      q_eps=1e-6, kv_eps=1e-6, rope_theta=10000.0)
        reps += 1
        sec = time.perf_counter() - t0
        if sec >= min_seconds:
            break
    return {"value": reps * c["tokens"] / sec, "unit": UNIT, "cores": os.cpu_count(),
            "kind": "port", "seconds": sec / reps,
            "sample": f"{name}: the whole {c['tokens']}-token step through the oracle's float64 "
                      f"prologue (numpy BLAS, all host threads), {reps} repetitions in "
                      f"{sec:.1f} s; the reference ships no prologue of its own"}


def run_prologue(args, world, rank, local_rank):
    import torch
    import torch.distributed as dist
    from tq_mla import ops

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    c, w, pos, seq, table = prologue_host(args.config, seed=5 + rank)
    d = {k: torch.from_numpy(v).to(torch.bfloat16).to(dev) for k, v in w.items()}
    h_x = torch.from_numpy(w["x"]).to(torch.bfloat16).pin_memory()
    h_ids = torch.from_numpy(np.stack([pos, seq])).pin_memory()
    d_ids = h_ids.to(dev)
    d_table = torch.from_numpy(table).to(dev)
    pool = torch.zeros((table.size, 64, c["row"]), dtype=torch.uint8, device=dev)
    q = torch.empty((c["tokens"], c["heads"], 512 + c["dr"]), dtype=torch.bfloat16, device=dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    pro = ops.MlaPrologue(d["x"], d["w_qa"], d["q_norm"], d["w_qb"], d["w_uk"], d["w_kva"],
                          d["kv_norm"], d_ids[0], d_ids[1], d_table, pool, q, heads=c["heads"],
                          nope_dim=c["dn"], rope_dim=c["dr"], kv_format=c["fmt"])
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(args.warmup, 3)):
        pro(flags=flags, stream=stream)
    torch.cuda.synchronize(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    clock = ClockSampler(local_rank, clock_log_path(args, rank))
    barrier()
    torch.cuda.synchronize(dev)
    with clock:
        for a, b in evs:
            flush.fill_(1)                        # L2 flushed between timed steps (256 MB write)
            a.record(stream)
            pro(flags=flags, stream=stream)
            b.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    times = [a.elapsed_time(b) for a, b in evs]
    ms_step = max_over_ranks(sum(times) / len(times))
    # The same step captured once in a CUDA graph and replayed (launch gaps removed), L2 flushed
    # before each replay as above.
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(dev)
    with torch.cuda.graph(graph, stream=cap):
        pro(flags=flags, stream=cap)
    torch.cuda.synchronize(dev)
    gevs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(args.steps)]
    for a, b in gevs:
        flush.fill_(1)
        a.record(stream)
        graph.replay()
        b.record(stream)
    torch.cuda.synchronize(dev)
    graph_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in gevs) / len(gevs))
    del graph
    # End to end: x, positions and sequence ids copied in from pinned host memory, the device
    # flags read back (q stays on the device for the attention step that consumes it).
    h_flags = torch.zeros(1, dtype=torch.int32).pin_memory()
    e2e = []
    for _ in range(max(3, min(args.steps, 50))):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        d["x"].copy_(h_x, non_blocking=True)
        d_ids.copy_(h_ids, non_blocking=True)
        pro(flags=flags, stream=stream)
        h_flags.copy_(flags, non_blocking=True)
        b.record(stream)
        e2e.append((a, b))
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in e2e) / len(e2e))
    assert int(flags.item()) == 0, "prologue flagged rows"
    # Self-check of the timed output against the oracle (q of every token).
    from oracle import prologue as opro

    q_ref, _ = opro.prologue(**{k: v.astype(np.float64) for k, v in w.items()}, pos=pos,
                             heads=c["heads"], nope_dim=c["dn"], rope_dim=c["dr"], q_eps=1e-6,
                             kv_eps=1e-6, rope_theta=10000.0)
    got = q.float().cpu().numpy().astype(np.float64)
    rms = np.sqrt(np.mean(q_ref ** 2, axis=-1, keepdims=True))
    ok = bool(np.all(np.abs(got - q_ref) <= 2.0 ** -6 * np.abs(q_ref) + 2.0 ** -6 * rms) and
              np.linalg.norm(got - q_ref) <= 2.0 ** -8 * np.linalg.norm(q_ref))
    nbytes = prologue_bytes(c)
    hbm, _, _, src_name = peaks()
    ach = nbytes / (ms_step * 1e-3) / 1e9
    ours = 2 + (2 if c["dr"] else 0)
    t = c["tokens"]
    result = {
        "metric": "MLA prologue tokens/s", "value": world * t / (ms_step * 1e-3), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (f32 accumulate)", "data": "synthetic",
        "config": {"workload": f"{args.config}: {t} decode tokens, hidden {c['dm']}, Q rank "
                               f"{c['rq']}, {c['heads']} heads x ({c['dn']} + {c['dr']}), rows "
                               f"{ {0: 1024, 1: 528, 2: 1152}[c['fmt']] } B",
                   "l2": "flushed between timed steps (256 MB write outside the events)"},
        "e2e": {"value": world * t / (e2e_ms * 1e-3), "unit": UNIT,
                "h2d_bytes_per_step": t * c["dm"] * 2 + 8 * t, "d2h_bytes_per_step": 4,
                "ms_per_step": e2e_ms},
        "gpu_launches": ours * args.steps,
        "library_launches_per_step": 4,
        "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                     "frac": ach / hbm, "traffic": None,
                     "kernel": "whole prologue step (q_a, q_b and kv_a projections, absorption, norms, RoPE, writer)",
                     "peak_source": f"{src_name} (MEASURED_PEAKS.json)",
                     "algorithmic_bytes_per_step": nbytes},
        "self_check": {"q_within_tolerance": ok, "tokens": t},
        "graph": {"ms_per_step": graph_ms, "value": world * t / (graph_ms * 1e-3),
                  "frac": nbytes / (graph_ms * 1e-3) / 1e9 / hbm,
                  "what": "the step captured in one CUDA graph, replayed; L2 flushed before "
                          "each replay"},
        "clocks": clock.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = prologue_cpu_baseline(args.config)
    if rank == 0:
        print(json.dumps(result), flush=True)


# ------------------------------------------------------------------------- sparse top-k

SPARSE_K, SPARSE_VALID, SPARSE_SETS = 2051, 2048, 4


def sparse_indices(w, set_id):
    """Index set ``set_id`` of a sparse workload: per token 2048 unique random positions in
    [0, q_pos], then three -1 entries, all in one shuffled row of 2051."""
    rng = np.random.default_rng(7000 + 31 * set_id + int(w.seed))
    seq, q_pos = w.seq_id(), w.q_pos()
    idx = np.full((w.tokens, SPARSE_K), -1, np.int32)
    for t in range(w.tokens):
        vis = int(min(w.kv_len[seq[t]], q_pos[t] + 1))
        sel = rng.choice(vis, size=min(vis, SPARSE_VALID), replace=False).astype(np.int32)
        row = np.concatenate([sel, np.full(SPARSE_K - len(sel), -1, np.int32)])
        rng.shuffle(row)
        idx[t] = row
    return idx, np.full(w.tokens, SPARSE_K, np.int32)


def sparse_cpu_baseline(name, tokens=8):
    """The oracle (float64 sparse gather + attention) on a bounded sample of tokens."""
    from oracle import generate as ogen, mla as omla
    from oracle import fp8 as ofp8

    w = ogen.config(name)
    idx, k_len = sparse_indices(w, 0)
    rng = np.random.default_rng(3)
    t0 = time.perf_counter()
    for t in range(tokens):
        q = rng.standard_normal((1, w.heads, 512))
        if w.kv_format == "fp8_e4m3":
            raw = np.zeros((SPARSE_VALID, 544), np.uint8)
            raw[:, :512] = rng.integers(0, 0x7E, size=(SPARSE_VALID, 512), dtype=np.uint8)
            raw[:, 512:528] = np.full((SPARSE_VALID, 4), 0.01, np.float32).view(np.uint8)
            rows = ofp8.dequant_rows(raw)
        else:
            rows = rng.standard_normal((SPARSE_VALID, 512))
        v = omla.sparse_entries(idx[t], k_len[t], w.q_pos()[t], w.kv_len[w.seq_id()[t]])
        omla.identity_core(q[0], rows[: len(v)], w.scale, 512)
    sec = time.perf_counter() - t0
    return {"value": tokens / sec, "unit": UNIT, "cores": 1, "kind": "port",
            "sample": f"{tokens} of {w.tokens} query tokens of {w.name}: float64 entry "
                      f"validation, row gather{_fp8_note(w)} and attention (oracle/mla.py), one "
                      f"process", "seconds": sec}


def run_sparse(args, world, rank, local_rank):
    import torch
    import torch.distributed as dist
    from tq_mla import inputs, ops

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    w = workload_for(args.config, world, rank)
    batch = inputs.materialize(w, dev)
    fmt = kv_format_of(w)
    out = torch.empty((w.tokens, w.heads, 512), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((w.tokens, w.heads), dtype=torch.float32, device=dev)
    sets = [sparse_indices(w, i) for i in range(SPARSE_SETS)]
    d_sets = [(torch.from_numpy(i).to(dev), torch.from_numpy(k).to(dev)) for i, k in sets]
    launches = [ops.MlaLaunch(batch.q, batch.kv, batch.page_table, batch.seq_id, batch.q_pos,
                              batch.kv_len, out, lse, scale=w.scale,
                              query_counts=batch.query_counts, kv_format=fmt, idx=i, k_len=k)
                for i, k in d_sets]
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for i in range(max(args.warmup, SPARSE_SETS)):
        launches[i % SPARSE_SETS](stream)
    torch.cuda.synchronize(dev)
    assert all(l.device_error() == 0 for l in launches)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clock = ClockSampler(local_rank, clock_log_path(args, rank))
    barrier()
    torch.cuda.synchronize(dev)
    with clock:
        ev0.record(stream)
        for i in range(args.steps):
            launches[i % SPARSE_SETS](stream)
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    ms_step = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    # The attention kernel alone (events around it; a second pass, as for dense decode).
    k_steps = min(args.steps, 300)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(k_steps)]
    for b_, e_ in kev:
        b_.record(stream)
        e_.record(stream)
    torch.cuda.synchronize(dev)
    for i, (b_, e_) in enumerate(kev):
        ops.set_kernel_timer(b_, e_)
        launches[i % SPARSE_SETS](stream)
    torch.cuda.synchronize(dev)
    ops.set_kernel_timer()
    kernel_ms = sum(b_.elapsed_time(e_) for b_, e_ in kev) / k_steps
    # End to end: q and the step's indices copied in from pinned memory, out and lse copied back.
    h_q = batch.q.cpu().pin_memory()
    h_sets = [(torch.from_numpy(i).pin_memory(), torch.from_numpy(k).pin_memory()) for i, k in sets]
    h_out = torch.empty_like(out, device="cpu").pin_memory()
    h_lse = torch.empty_like(lse, device="cpu").pin_memory()
    e2e_steps = max(SPARSE_SETS, min(args.steps, 200))
    barrier()
    torch.cuda.synchronize(dev)
    ev0.record(stream)
    for i in range(e2e_steps):
        j = i % SPARSE_SETS
        batch.q.copy_(h_q, non_blocking=True)
        d_sets[j][0].copy_(h_sets[j][0], non_blocking=True)
        d_sets[j][1].copy_(h_sets[j][1], non_blocking=True)
        launches[j](stream)
        h_out.copy_(out, non_blocking=True)
        h_lse.copy_(lse, non_blocking=True)
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1)) / e2e_steps
    assert all(l.device_error() == 0 for l in launches)
    # Parity of a timed launch's output with the oracle (index set 0).
    launches[0](stream)
    torch.cuda.synchronize(dev)
    check = self_check(w, batch, out, lse, fp8=fmt is not None, sparse=sets[0])
    ok_all = max_over_ranks(0.0 if check["pass"] else 1.0) == 0.0
    row_bytes = 528 if fmt is not None else 1024
    valid = sum(int(min(SPARSE_VALID, k)) for k in w.kv_len[w.seq_id()])
    bytes_step = (valid * row_bytes + w.tokens * w.heads * 512 * 2 + w.tokens * SPARSE_K * 4
                  + w.tokens * 4 + w.tokens * w.heads * (512 * 2 + 4))
    flops_step = 2.0 * valid * w.heads * (512 + 512)
    hbm, tc_burst, _, src = peaks()
    ach_gbs = bytes_step / (kernel_ms * 1e-3) / 1e9
    tokens_all = w.tokens * world
    h2d = h_q.numel() * 2 + h_sets[0][0].numel() * 4 + h_sets[0][1].numel() * 4
    d2h = h_out.numel() * 2 + h_lse.numel() * 4
    result = {
        "metric": "MLA sparse top-k decode tokens/s", "value": tokens_all / (ms_step * 1e-3),
        "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp8_e4m3 rows, bf16 operands" if fmt is not None else "bf16",
        "data": "synthetic",
        "config": {"workload": w.name if world == 1 else f"{w.name} x{world} ranks",
                   "query_tokens": tokens_all, "heads": w.heads, "topk_entries": SPARSE_K,
                   "valid_entries_per_token": SPARSE_VALID,
                   "l2": f"{SPARSE_SETS} index sets rotate: %.0f MB of rows per step, %.0f MB "
                         "across the sets (L2 126 MB)" % (valid * row_bytes / 1e6,
                                                          SPARSE_SETS * valid * row_bytes / 1e6)},
        "e2e": {"value": tokens_all / (e2e_ms * 1e-3), "unit": UNIT,
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "ms_per_step": e2e_ms},
        "gpu_launches": (LAUNCHES_PER_STEP + 1) * args.steps,
        "roofline": {"bound": "hbm", "achieved": ach_gbs, "peak": hbm, "unit": "GB/s",
                     "frac": ach_gbs / hbm, "traffic": None, "kernel": "mla_paged_kernel",
                     "kernel_ms_per_launch": kernel_ms,
                     "peak_source": f"{src} (MEASURED_PEAKS.json)",
                     "algorithmic_bytes_per_launch": bytes_step, "flops_per_launch": flops_step,
                     "tflops": flops_step / (kernel_ms * 1e-3) / 1e12,
                     "step_frac": bytes_step / (ms_step * 1e-3) / 1e9 / hbm},
        "clocks": clock.summary(),
    }
    result["self_check"] = check
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = sparse_cpu_baseline(args.config)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if not ok_all:
        raise SystemExit(f"self-check failed: the timed output does not match the oracle: {check}")


# ------------------------------------------------------------------------- reference arm

def run_reference(args, world, rank):
    if rank != 0:
        return
    if args.config.startswith("sparse"):
        base = sparse_cpu_baseline(args.config, tokens=16)
        line = {"impl": "reference", "metric": "MLA sparse top-k decode tokens/s",
                "value": base["value"], "unit": UNIT, "n_gpus": world, "steps": 1, "warmup": 0,
                "ms_per_step": 1e3 * base["seconds"], "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
                "config": {"workload": args.config}, "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if args.config.startswith("prologue"):
        base = prologue_cpu_baseline(args.config)
        line = {"impl": "reference", "metric": "MLA prologue tokens/s", "value": base["value"],
                "unit": UNIT, "n_gpus": world, "steps": 1, "warmup": 0,
                "ms_per_step": 1e3 * base["seconds"], "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
                "config": {"workload": args.config}, "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if args.config.startswith("kv_write"):
        base = writer_cpu_baseline(args.config)
        line = {"impl": "reference", "metric": "KV rows written/s", "value": base["value"],
                "unit": "rows/s", "n_gpus": world, "steps": 1, "warmup": 0,
                "ms_per_step": 1e3 * base["seconds"], "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": args.config}, "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "rows/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    # Dense configurations: the oracle's float64 restatement of mla_attention_core over the same
    # seeded inputs, one spawned process per host core; no product library is loaded.
    strong = args.scaling == "strong"
    base = cpu_measure(args.config, world, steps=args.steps, warmup=args.warmup, strong=strong)
    w, _, _ = cpu_sample(args.config, world, strong)
    dtype = "f64" + (" (FP8 E4M3 rows decoded to f64)" if _fp8_note(w) else "")
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT,
        "n_gpus": world, "steps": base["steps"], "warmup": base["warmup"],
        "ms_per_step": base["ms_per_step"], "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": dtype, "data": "synthetic",
        "config": job_config(args.config, world, w, strong),
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def job_config(name, world, w, strong=False):
    """``config`` of a dense configuration from its whole-job workload (product or oracle)."""
    fp8 = getattr(w, "kv_format", None) == "fp8_e4m3" or \
        getattr(w, "extra", {}).get("kv_format") == "fp8_e4m3"
    row_stride = 544 if fp8 else 2 * w.width
    par = None
    if strong and world > 1:
        par = (f"context split x{world} (each sequence's pages over the ranks, NCCL all-gather "
               f"+ LSE merge)" if name == "longctx"
               else f"sequence-shard x{world} of the fixed batch (token-balanced)")
    return config_block(w.name, world, w.sequences, w.tokens, w.heads, w.width,
                        w.pool_pages * 64 * row_stride, parallelism=par, strong=strong)


# ------------------------------------------------------------------------- our arm

def self_check(w, batch, out, lse, *, count=8, fp8=False, sparse=None):
    """Compares ``count`` query tokens of a finished step with the oracle, computed in float64
    from the very device inputs the kernel read (out max-abs 2e-2 and
    relative L2 1e-2, lse 1e-3). Returns the errors; the caller fails the run on a mismatch.

    The oracle is the checker here: it runs after the timed regions, on copies of the inputs.
    """
    import torch
    from oracle import fp8 as ofp8, mla as omla

    T = w.tokens
    if T == 0:
        return {"tokens": 0, "pass": True}
    picks = np.unique(np.linspace(0, T - 1, min(count, T)).astype(int))
    seq, qpos = w.seq_id(), w.q_pos()
    table = w.extra["page_table"]
    dev = out.device
    got_o, got_l, ref_o, ref_l = [], [], [], []
    for t in picks:
        s_ = int(seq[t])
        if sparse is not None:
            idx, k_len = sparse
            v = omla.sparse_entries(idx[t], k_len[t], qpos[t], w.kv_len[s_])
            prow = table[s_][v // 64].astype(np.int64) * 64 + v % 64
            raw = batch.kv.reshape(-1, batch.kv.shape[-1])[torch.from_numpy(prow).to(dev)]
        else:
            n = int(min(w.kv_len[s_], int(qpos[t]) + 1))
            pages = torch.from_numpy(table[s_, : (n + 63) // 64].astype(np.int64)).to(dev)
            raw = batch.kv[pages].reshape(-1, batch.kv.shape[-1])[:n]
        if fp8:
            rows = ofp8.operand_rows(raw.cpu().numpy())
        else:
            rows = raw.double().cpu().numpy()
        q = batch.q[int(t)].double().cpu().numpy()
        o, l_ = omla.identity_core(q, rows, w.scale, 512)
        ref_o.append(o)
        ref_l.append(l_)
        got_o.append(out[int(t)].double().cpu().numpy())
        got_l.append(lse[int(t)].double().cpu().numpy())
    ro, rl, go, gl = map(np.stack, (ref_o, ref_l, got_o, got_l))
    fin = np.isfinite(rl)
    res = {
        "tokens": int(len(picks)),
        "out_max_abs": float(np.abs(go - ro).max()),
        "out_rel_l2": float(np.linalg.norm(go - ro) / max(np.linalg.norm(ro), 1e-300)),
        "lse_max_abs": float(np.abs(gl[fin] - rl[fin]).max()) if fin.any() else 0.0,
        "lse_inf_pattern_equal": bool(np.array_equal(np.isneginf(gl), np.isneginf(rl))),
    }
    res["pass"] = bool(np.isfinite(go).all() and res["out_max_abs"] <= 2e-2 and
                       res["out_rel_l2"] <= 1e-2 and res["lse_max_abs"] <= 1e-3 and
                       res["lse_inf_pattern_equal"])
    return res


def step_percentiles(launch_step, stream, runs=50, steps_per_run=10):
    """Per-step time over ``runs`` runs of ``steps_per_run`` back-to-back steps, with events only
    at run boundaries (an event between two launches breaks their programmatic overlap)."""
    import torch

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(runs + 1)]
    torch.cuda.synchronize()
    ev[0].record(stream)
    for r in range(runs):
        for _ in range(steps_per_run):
            launch_step()
        ev[r + 1].record(stream)
    torch.cuda.synchronize()
    per = np.array([ev[r].elapsed_time(ev[r + 1]) / steps_per_run for r in range(runs)])
    p10, p25, p50, p75, p90 = (float(np.percentile(per, q)) for q in (10, 25, 50, 75, 90))
    return {"runs": runs, "steps_per_run": steps_per_run, "ms_p10": p10, "ms_median": p50,
            "ms_p90": p90, "ms_iqr": p75 - p25, "ms_mean": float(per.mean())}


def host_link(h_in, d_in, d_out, h_out, stream, reps=20):
    """Host<->device copy rates of one step's buffers: each direction alone, then both at once
    on two streams (PCIe is full duplex). This bounds what an end-to-end step can reach."""
    import torch

    def timed(pairs_by_stream):
        evs = []
        for st, pairs in pairs_by_stream:
            b, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            b.record(st)
            with torch.cuda.stream(st):
                for _ in range(reps):
                    for dst, src in pairs:
                        dst.copy_(src, non_blocking=True)
            e.record(st)
            evs.append((b, e))
        torch.cuda.synchronize()
        return [b.elapsed_time(e) / reps for b, e in evs]

    nbytes = lambda pairs: sum(d.numel() * d.element_size() for d, _ in pairs)
    h2d, d2h = list(zip(d_in, h_in)), list(zip(h_out, d_out))
    s2 = torch.cuda.Stream(stream.device)
    timed([(stream, h2d)])  # warm-up
    (t_in,) = timed([(stream, h2d)])
    (t_out,) = timed([(stream, d2h)])
    t_in2, t_out2 = timed([(stream, h2d), (s2, d2h)])
    bi, bo = nbytes(h2d), nbytes(d2h)
    return {"h2d_gbs": bi / t_in / 1e6, "d2h_gbs": bo / t_out / 1e6,
            "h2d_gbs_concurrent": bi / t_in2 / 1e6, "d2h_gbs_concurrent": bo / t_out2 / 1e6,
            "h2d_ms": t_in, "d2h_ms": t_out, "both_ms": max(t_in2, t_out2)}


def traffic_from_profiles(workload_name):
    p = ROOT / "profiles" / "ncu_traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.lstrip().startswith("#"):
            continue
        kv = dict(x.split("=", 1) for x in line.split() if "=" in x)
        if kv.get("workload") == workload_name and "dram_bytes_per_launch" in kv:
            return float(kv["dram_bytes_per_launch"])
    return None


NATIVE_CONFIGS = ("decode", "prefill", "longctx", "mtp", "cpu")


def native_binary():
    """Path of the native benchmark binary (built next to libtq_mla.so), or None."""
    path = ROOT / "tensorquay-engine_b200" / "tq_mla" / "tq_bench"
    return path if path.exists() and os.access(path, os.X_OK) else None


def run_native(args, world, rank, local_rank, strong, dump_path):
    """Times the step with the native binary (C ABI only, no Python on the timed path) on this
    rank's GPU and share of the job; returns its JSON result."""
    cmd = [str(native_binary()), "--config", args.config, "--steps", str(args.steps),
           "--warmup", str(args.warmup), "--world", str(world), "--rank", str(rank),
           "--device", str(local_rank), "--graph", "--dump-out", dump_path]
    if strong:
        cmd.append("--strong")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", ""))
    if not env["CUDA_VISIBLE_DEVICES"]:
        env.pop("CUDA_VISIBLE_DEVICES")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    if r.returncode != 0:
        raise SystemExit(f"tq_bench failed ({r.returncode}): {r.stderr[-2000:]}")
    return json.loads(r.stdout.strip().splitlines()[-1])


def run_ours(args, world, rank, local_rank):
    import torch
    import torch.distributed as dist
    from tq_mla import inputs, ops

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    strong = args.scaling == "strong"
    w = workload_for(args.config, world, rank, strong)

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- the timed step, from the native binary (C ABI only) when it is built for this
    # configuration: K steps back to back on this rank's GPU, bracketed by barriers.
    native, dump = None, None
    clock = ClockSampler(local_rank, clock_log_path(args, rank))
    if native_binary() is not None and args.config in NATIVE_CONFIGS:
        dump = os.path.join(tempfile.gettempdir(), f"tq_bench_out_rank{rank}_{os.getpid()}.bin")
        barrier()
        torch.cuda.synchronize(dev)
        with clock:
            native = run_native(args, world, rank, local_rank, strong, dump)
        barrier()
    batch = inputs.materialize(w, dev)
    out = torch.empty((w.tokens, w.heads, 512), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((w.tokens, w.heads), dtype=torch.float32, device=dev)
    launch = ops.MlaLaunch(batch.q, batch.kv, batch.page_table, batch.seq_id, batch.q_pos,
                           batch.kv_len, out, lse, scale=w.scale,
                           query_counts=batch.query_counts, prefill=args.config == "prefill",
                           kv_format=kv_format_of(w))
    stream = torch.cuda.current_stream(dev)

    # Host copies for the end-to-end leg (pinned). The four int32 metadata arrays travel as one
    # packed buffer (one copy per step instead of four), each array 16-byte aligned in it.
    h_q = batch.q.cpu().pin_memory()
    d_meta = [batch.page_table, batch.seq_id, batch.q_pos, batch.kv_len]
    meta_offsets, n_meta = [], 0
    for t in d_meta:
        meta_offsets.append(n_meta)
        n_meta += -(-t.numel() // 4) * 4
    h_meta = torch.zeros(n_meta, dtype=torch.int32).pin_memory()
    for t, o in zip(d_meta, meta_offsets):
        h_meta[o:o + t.numel()].copy_(t.reshape(-1).cpu())
    h_out = torch.empty_like(out, device="cpu").pin_memory()
    h_lse = torch.empty_like(lse, device="cpu").pin_memory()
    h2d = h_q.numel() * 2 + h_meta.numel() * 4
    d2h = h_out.numel() * 2 + h_lse.numel() * 4

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    for _ in range(args.warmup):
        launch(stream)
    torch.cuda.synchronize(dev)
    assert launch.device_error() == 0, "device error flag set during warm-up"

    # ---- device-resident timing through the Python front end (ctypes -> C ABI)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    with (clock if native is None else contextlib.nullcontext()):
        ev0.record(stream)
        for _ in range(args.steps):
            launch(stream)
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms)
    ms_step = ms_max / args.steps

    # ---- the attention kernel alone: a second pass with events recorded around it in every
    # step (recorded once beforehand so that they exist). An event between two launches breaks
    # their programmatic overlap, so this pass is not the one that gives the step time above, and
    # each kernel interval also holds the kernel's own launch latency (conservative).
    k_steps = min(args.steps, 300)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(k_steps)]
    for b, e in kev:
        b.record(stream)
        e.record(stream)
    torch.cuda.synchronize(dev)
    for b, e in kev:
        ops.set_kernel_timer(b, e)
        launch(stream)
    torch.cuda.synchronize(dev)
    ops.set_kernel_timer()
    kernel_ms = sum(b.elapsed_time(e) for b, e in kev) / k_steps

    # ---- end-to-end through the C ABI with host buffers, pipelined as a serving loop would be:
    # two sets of device buffers, each with its own validated launch; per step k (set k % 2) the
    # inputs are copied in on a copy-in stream, the attention runs on the compute stream once
    # they have landed, and the results are copied out on a copy-out stream once it finishes.
    # Step k+1's copies in and step k-1's copies out overlap step k's compute; every step's own
    # copies (all of its inputs, all of its results) stay inside the timed region.
    s_in = torch.cuda.Stream(dev)
    s_out = torch.cuda.Stream(dev)
    sets = []
    for _ in range(2):
        q_d = torch.empty_like(batch.q)
        meta_packed = torch.empty(n_meta, dtype=torch.int32, device=dev)
        meta_d = [meta_packed[o:o + t.numel()].view(t.shape) for t, o in zip(d_meta, meta_offsets)]
        out_d = torch.empty_like(out)
        lse_d = torch.empty_like(lse)
        lk = ops.MlaLaunch(q_d, batch.kv, meta_d[0], meta_d[1], meta_d[2], meta_d[3], out_d, lse_d,
                           scale=w.scale, query_counts=batch.query_counts,
                           prefill=args.config == "prefill", kv_format=kv_format_of(w))
        h_o = torch.empty_like(out, device="cpu").pin_memory()
        h_l = torch.empty_like(lse, device="cpu").pin_memory()
        ev = [torch.cuda.Event() for _ in range(3)]  # inputs landed, computed, copied out
        for e in ev:
            e.record(stream)
        sets.append((q_d, meta_packed, out_d, lse_d, lk, h_o, h_l, ev))

    def e2e_step(i):
        q_d, meta_packed, out_d, lse_d, lk, h_o, h_l, (ev_in, ev_done, ev_out) = sets[i % 2]
        s_in.wait_event(ev_done)  # step i-2 finished reading this set's inputs
        with torch.cuda.stream(s_in):
            q_d.copy_(h_q, non_blocking=True)
            meta_packed.copy_(h_meta, non_blocking=True)
        ev_in.record(s_in)
        stream.wait_event(ev_in)
        stream.wait_event(ev_out)  # step i-2's results have left this set's output buffers
        lk(stream)
        ev_done.record(stream)
        s_out.wait_event(ev_done)
        with torch.cuda.stream(s_out):
            h_o.copy_(out_d, non_blocking=True)
            h_l.copy_(lse_d, non_blocking=True)
        ev_out.record(s_out)

    for i in range(max(2, args.warmup)):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    ev0.record(stream)
    s_in.wait_event(ev0)
    s_out.wait_event(ev0)
    for i in range(args.steps):
        e2e_step(i)
    stream.wait_stream(s_in)
    stream.wait_stream(s_out)
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    assert sets[0][4].device_error() == 0 and sets[1][4].device_error() == 0
    err = launch.device_error()
    # The end-to-end results equal the resident run's bit for bit (same inputs, deterministic).
    e2e_same = all(torch.equal(st[5], out.cpu()) and torch.equal(st[6], lse.cpu())
                   for st in sets)
    stats = step_percentiles(lambda: launch(stream), stream)
    link = host_link([h_q, h_meta], [sets[0][0], sets[0][1]], [sets[0][2], sets[0][3]],
                     [sets[0][5], sets[0][6]], stream)
    # Parity of the timed output with the oracle (after every timed region; all ranks check
    # their own tokens, then the verdict is combined).
    check = self_check(w, batch, out, lse, fp8=kv_format_of(w) is not None)
    native_same = True
    if native is not None:
        # The binary's last output: bitwise equal to this front end's (same seeded inputs,
        # deterministic kernels), hence also checked against the oracle above.
        raw = np.fromfile(dump, dtype=np.uint8)
        os.remove(dump)
        n_out = out.numel() * 2
        nat_out = torch.from_numpy(raw[:n_out].copy()).view(torch.bfloat16).view(out.shape)
        nat_lse = torch.from_numpy(raw[n_out:].copy()).view(torch.float32).view(lse.shape)
        native_same = bool(torch.equal(nat_out, out.cpu()) and torch.equal(nat_lse, lse.cpu()))
        native_same = native_same and native["e2e"]["results_equal_resident_run"] and \
            native["device_error_flags"] == 0
        check["native_output_equal"] = native_same
    ok_all = max_over_ranks(0.0 if (check["pass"] and e2e_same and err == 0 and native_same)
                            else 1.0) == 0.0
    py = {"ms_per_step": ms_step, "kernel_ms_per_launch": kernel_ms, "e2e_ms_per_step": e2e_ms,
          "step_stats": stats}
    if native is not None:
        ms = max_over_ranks(native["ms_per_step"]) * args.steps
        ms_step = ms / args.steps
        kernel_ms = max_over_ranks(native["kernel_ms_per_launch"])
        e2e_ms = max_over_ranks(native["e2e"]["ms_per_step"])
        stats = native["step_stats"]
        h2d, d2h = native["e2e"]["h2d_bytes_per_step"], native["e2e"]["d2h_bytes_per_step"]

    tokens_all = sum_over_ranks(float(w.tokens))
    flops_all = sum_over_ranks(w.flops())
    bytes_mine = w.bytes()
    value = tokens_all / (ms_step * 1e-3)
    e2e_value = tokens_all / (e2e_ms * 1e-3)
    hbm, tc_burst, tc_sus, src = peaks()
    # Dominant kernel: the attention kernel, timed by the events recorded around each launch.
    ach_gbs = bytes_mine / (kernel_ms * 1e-3) / 1e9
    ach_tflops = w.flops() / (kernel_ms * 1e-3) / 1e12
    ai = w.flops() / bytes_mine
    ridge = tc_burst * 1e12 / (hbm * 1e9)
    bound = "hbm" if ai < ridge else "tensor"
    traffic = traffic_from_profiles(w.name) if world == 1 else None
    roofline = {
        "bound": bound,
        "achieved": ach_gbs if bound == "hbm" else ach_tflops,
        "peak": hbm if bound == "hbm" else tc_burst,
        "unit": "GB/s" if bound == "hbm" else "TFLOP/s",
        "frac": (ach_gbs / hbm) if bound == "hbm" else (ach_tflops / tc_burst),
        "traffic": traffic,
        "peak_source": f"{src} (MEASURED_PEAKS.json)" if src == "measured" else "fallback",
        "hbm_gbs": ach_gbs, "hbm_frac": ach_gbs / hbm,
        "tflops": ach_tflops, "tensor_frac_burst": ach_tflops / tc_burst,
        "tensor_frac_sustained": ach_tflops / tc_sus,
        "kernel": "mla_paged_kernel", "kernel_ms_per_launch": kernel_ms,
        "roofline_time_us": 1e6 * max(bytes_mine / (hbm * 1e9), w.flops() / (tc_burst * 1e12)),
        "step_roofline_frac": 1e6 * max(bytes_mine / (hbm * 1e9), w.flops() / (tc_burst * 1e12))
        / (1e3 * ms / args.steps),
        "algorithmic_bytes_per_launch": bytes_mine, "flops_per_launch": w.flops(),
        "arithmetic_intensity": ai,
    }
    result = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None,
        "dtype": "fp8_e4m3 rows, bf16 operands" if kv_format_of(w) is not None else "bf16",
        "data": "synthetic",
        "config": job_config(args.config, world, inputs.config(
            args.config, batch=job_batch(args.config, world, strong)), strong),
        "tflops_total": flops_all / (ms_step * 1e-3) / 1e12,
        "step_stats": stats,
        "timed_by": ("tq_bench (native binary, C ABI only)" if native is not None
                     else "bench.py through the C ABI (ctypes)"),
        "graph_stats": native.get("graph_stats") if native is not None else None,
        "python_front_end": py,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_ms,
                "pipeline": "copy-in, compute and copy-out streams, two buffer sets",
                "results_equal_resident_run": bool(e2e_same and native_same),
                "host_link": link,
                "ceiling_tokens_per_s": float(w.tokens) * world / (1e-3 * max(
                    link["both_ms"], ms_step))},
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "roofline": roofline,
        "clocks": clock.summary(),
        "device_error_flags": err,
        "self_check": check,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(args.config, world)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if not ok_all:
        raise SystemExit("self-check failed: the timed output does not match the oracle "
                         f"(rank {rank}: {check}, e2e equal {e2e_same}, device flags {err})")


def run_context(args, world, rank, local_rank):
    """The long-context batch as configured: every sequence's 131072 cached positions are split
    over the ranks by page range. Per step each rank decodes its range into f32 partials, then
    ``tq_mla_context_merge`` (NCCL all-gather of the partials + the LSE merge kernel; with
    ``--merge peer`` one kernel reading the peers' partials over NVLink) leaves the
    merged output on every rank. ``value`` = the batch's query tokens / the slowest rank's step
    time (strong scaling: the work is fixed, the ranks share it)."""
    import torch
    import torch.distributed as dist
    from tq_mla import dist as tdist, inputs, ops

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    full = inputs.config(args.config)
    part = tdist.context_split(full, world, rank)
    batch = inputs.materialize(part, dev)
    T, H = part.tokens, part.heads
    comm = tdist.Comm.from_process_group()
    peer = args.merge == "peer"
    pm = tdist.PeerMerge(comm, T, H) if peer else None
    if peer:  # the partials are decoded straight into this rank's exchange region
        p_out, p_lse = pm.part_out, pm.part_lse
    else:
        p_out = torch.empty((T, H, 512), dtype=torch.float32, device=dev)
        p_lse = torch.empty((T, H), dtype=torch.float32, device=dev)
    out = torch.empty((T, H, 512), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((T, H), dtype=torch.float32, device=dev)
    launch = ops.MlaLaunch(batch.q, batch.kv, batch.page_table, batch.seq_id, batch.q_pos,
                           batch.kv_len, p_out, p_lse, scale=part.scale,
                           query_counts=batch.query_counts)
    stream = torch.cuda.current_stream(dev)

    def merge():
        if peer:
            pm.merge(out, lse, stream)
        else:
            tdist.context_merge(comm, p_out, p_lse, out, lse, stream)

    def step():
        launch(stream)
        merge()

    def max_over_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    try:
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize(dev)
        assert launch.device_error() == 0
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clock = ClockSampler(local_rank, clock_log_path(args, rank))
        dist.barrier()
        torch.cuda.synchronize(dev)
        with clock:
            ev0.record(stream)
            for _ in range(args.steps):
                step()
            ev1.record(stream)
            torch.cuda.synchronize(dev)
        dist.barrier()
        ms_step = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
        # The merge alone (all-gather + merge kernel), then the attention kernel alone.
        dist.barrier()
        torch.cuda.synchronize(dev)
        ev0.record(stream)
        for _ in range(args.steps):
            merge()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
        merge_ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
        k_steps = min(args.steps, 300)
        kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(k_steps)]
        for b_, e_ in kev:
            b_.record(stream)
            e_.record(stream)
        torch.cuda.synchronize(dev)
        for b_, e_ in kev:
            ops.set_kernel_timer(b_, e_)
            launch(stream)
        torch.cuda.synchronize(dev)
        ops.set_kernel_timer()
        kernel_ms = max_over_ranks(sum(b_.elapsed_time(e_) for b_, e_ in kev) / k_steps)
        # End to end: the step's queries from pinned host memory on every rank, the merged
        # output and lse back to the host, one stream.
        h_q = batch.q.cpu().pin_memory()
        h_out = torch.empty_like(out, device="cpu").pin_memory()
        h_lse = torch.empty_like(lse, device="cpu").pin_memory()
        dist.barrier()
        torch.cuda.synchronize(dev)
        ev0.record(stream)
        for _ in range(args.steps):
            batch.q.copy_(h_q, non_blocking=True)
            step()
            h_out.copy_(out, non_blocking=True)
            h_lse.copy_(lse, non_blocking=True)
        ev1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
        err = launch.device_error()
        # Parity: every rank's partial against the oracle of its own range; rank 0 merges the
        # oracle partials of all ranks and compares the merged device output with that.
        from oracle import mla as omla

        step()
        torch.cuda.synchronize(dev)
        part_check = self_check(part, batch, p_out, p_lse, count=T)
        table = part.extra["page_table"]
        ref_o, ref_l = [], []
        for t in range(T):
            n = int(part.kv_len[t])
            pages = torch.from_numpy(table[t, : (n + 63) // 64].astype(np.int64)).to(dev)
            rows = batch.kv[pages].reshape(-1, batch.kv.shape[-1])[:n].double().cpu().numpy()
            o, l_ = omla.identity_core(batch.q[t].double().cpu().numpy(), rows, part.scale, 512)
            ref_o.append(o)
            ref_l.append(l_)
        gathered = [None] * world
        dist.all_gather_object(gathered, (np.stack(ref_o), np.stack(ref_l)))
        m_o, m_l = omla.combine_partials(np.stack([g[0] for g in gathered]),
                                         np.stack([g[1] for g in gathered]))
        go, gl = out.double().cpu().numpy(), lse.double().cpu().numpy()
        merged_check = {
            "out_max_abs": float(np.abs(go - m_o).max()),
            "out_rel_l2": float(np.linalg.norm(go - m_o) / np.linalg.norm(m_o)),
            "lse_max_abs": float(np.abs(gl - m_l).max()),
        }
        merged_check["pass"] = bool(merged_check["out_max_abs"] <= 2e-2 and
                                    merged_check["out_rel_l2"] <= 1e-2 and
                                    merged_check["lse_max_abs"] <= 1e-3)
        merge_err = pm.device_error(stream) if peer else 0
        ok_all = max_over_ranks(0.0 if (part_check["pass"] and merged_check["pass"] and
                                        err == 0 and merge_err == 0) else 1.0) == 0.0
    finally:
        if pm is not None:
            pm.destroy()
        comm.destroy()

    hbm, tc_burst, tc_sus, src = peaks()
    bytes_rank, flops_rank = part.bytes(), part.flops()
    ach = bytes_rank / (kernel_ms * 1e-3) / 1e9
    tokens = full.tokens
    gather_bytes = (world - 1) * T * H * (512 + 1) * 4
    result = {
        "metric": METRIC, "value": tokens / (ms_step * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": dict(job_config(args.config, world, full, strong=True),
                       parallelism=f"context split x{world} (each sequence's pages over the "
                                   "ranks; " + ("partials read over NVLink by one merge kernel "
                                                "per rank" if peer else "NCCL all-gather + LSE "
                                                "merge") + ")"),
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": UNIT,
                "h2d_bytes_per_step": int(h_q.numel() * 2),
                "d2h_bytes_per_step": int(h_out.numel() * 2 + h_lse.numel() * 4),
                "ms_per_step": e2e_ms, "per_rank": "each rank copies the queries in and the "
                                                 "merged result out"},
        "gpu_launches": (LAUNCHES_PER_STEP + 1) * args.steps,
        "merge": {"ms": merge_ms, "received_bytes_per_rank": gather_bytes,
                  "what": ("tq_peer_merge: one kernel per rank reads the peers' f32 partials and "
                           "lse over NVLink (CUDA IPC mappings) and merges them" if peer else
                           "tq_mla_context_merge: NCCL all-gather of f32 partials + lse, then "
                           "the LSE merge kernel"), "kernel_ms": kernel_ms},
        "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                     "frac": ach / hbm, "traffic": None, "kernel": "mla_paged_kernel",
                     "kernel_ms_per_launch": kernel_ms,
                     "peak_source": f"{src} (MEASURED_PEAKS.json)",
                     "algorithmic_bytes_per_launch": bytes_rank,
                     "flops_per_launch": flops_rank,
                     "tflops": flops_rank / (kernel_ms * 1e-3) / 1e12,
                     "step_roofline_frac": max(full.bytes() / (hbm * 1e9),
                                               full.flops() / (tc_burst * 1e12))
                     / world / (ms_step * 1e-3)},
        "clocks": clock.summary(),
        "device_error_flags": err,
        "self_check": {"partial": part_check, "merged": merged_check},
    }
    if rank == 0:
        print(json.dumps(result), flush=True)
    if not ok_all:
        raise SystemExit(f"self-check failed on rank {rank}: {result['self_check']}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="decode",
                    choices=["decode", "decode_fp8", "mtp", "prefill", "longctx", "cpu",
                             "kv_write", "kv_write_fp8", "sparse", "sparse_fp8", "prologue",
                             "prologue_nope"])
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="weak: N ranks hold N times the one-GPU batch; strong: the batch stays "
                         "fixed and is shared (longctx: each sequence's pages split over the "
                         "ranks, merged over NCCL)")
    ap.add_argument("--merge", choices=["nccl", "peer"], default="peer",
                    help="long-context split (--config longctx --scaling strong, N > 1): merge "
                         "the ranks' partials by an NCCL all-gather + merge kernel, or by one "
                         "kernel reading the peers' partials over NVLink")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--clock-log", default=None,
                    help="file for the nvidia-smi clock samples ({rank} is replaced)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.config.startswith("kv_write"):
            run_writer(args, world, rank, local_rank)
        elif args.config.startswith("prologue"):
            run_prologue(args, world, rank, local_rank)
        elif args.config.startswith("sparse"):
            run_sparse(args, world, rank, local_rank)
        elif args.config == "longctx" and args.scaling == "strong" and world > 1:
            run_context(args, world, rank, local_rank)
        else:
            run_ours(args, world, rank, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
