"""Paged-KV decode benchmark for B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: one attention layer, bf16 K/V,
14 query / 2 KV heads, head_dim 64, page size 16, a pool of 65 536 pages,
64 sequences with context lengths U[256, 4096] (seed 2) whose block tables
are a random permutation of the free page ids (seed 3), Q/K/V ~ N(0, 1)
(seed 4).  One step = append one token per sequence, then paged decode
attention over every sequence, in one kernel launch (the append is fused
into the decode kernel).

  value  decode tokens/s over all ranks: the K timed steps replayed back to
         back (one CUDA graph each) between two CUDA events, inputs resident
         in HBM.  The steps rotate through 6 disjoint 64-sequence batches, so
         no step finds its K/V in L2 (inputs larger than L2, no flush);
         per_step_l2_flushed_us re-times the same steps one by one after an
         L2-flushing 256 MiB write.
  e2e    the same step through the C ABI with pinned HOST buffers: Q, new
         K/V and seq_lens (packed in one staging buffer per step) copied
         host->device and the output copied back inside the timed region.
  roofline  the decode kernel: algorithmic bytes per launch / its mean
         CUDA-event time, against MEASURED_PEAKS.json hbm_gbs.
  cpu_baseline  the reference algorithm on the host cores (oracle port of
         the cat-grown contiguous cache decode step), bounded sample.

Multi-GPU: replicas only.  Every rank runs its own pool and sequences; no
data-path collective.  torch.distributed (NCCL) only provides the barrier
and the max-over-ranks of the device time.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tokens/s & paged-attn KV-read HBM GB/s vs peak"
N_SEQS, HQ, HKV, D, PS, NUM_PAGES = 64, 14, 2, 64, 16, 65536
L_LO, L_HI = 256, 4096
B_TOK = 2 * HKV * D * 2  # K+V bytes per token per layer (bf16)


def workload_config(extra=None):
    cfg = {
        "workload": "BASELINE config 2: isolated paged-KV microbench, 1 layer, bf16 K/V, GQA 14q/2kv, head_dim 64, "
                    "page 16, pool 65536 pages, 64 seqs, ctx U[256,4096]; step = append 1 token/seq + decode",
        "n_seqs": N_SEQS, "num_q_heads": HQ, "num_kv_heads": HKV, "head_dim": D, "page_size": PS,
        "num_pages": NUM_PAGES, "ctx_range": [L_LO, L_HI], "seeds": {"lens": 2, "tables": 3, "qkv": 4},
        "l2": f"inputs larger than L2, no flush: steps rotate through {N_BATCHES} disjoint 64-sequence batches "
              f"(~71 MB of K/V each), so a step's K/V were last read {N_BATCHES - 1} steps (~355 MB) earlier; "
              "per_step_l2_flushed_us re-times the same steps one by one after a 256 MiB L2-flushing write",
    }
    if extra:
        cfg.update(extra)
    return cfg


def make_lens(n=N_SEQS):
    rng = np.random.default_rng(2)
    return rng.integers(L_LO, L_HI + 1, size=n).astype(np.int64)


def decode_bytes(seq_lens: np.ndarray) -> int:
    """Algorithmic bytes of one decode (K+V read once, Q in, O out, page ids, lens/indptr)."""
    pages = np.ceil(seq_lens / PS).astype(np.int64)
    return int(seq_lens.sum() * B_TOK + N_SEQS * HQ * D * 2 * 2 + 4 * pages.sum() + 8 * N_SEQS)


def append_bytes(n_tok: int) -> int:
    """Algorithmic bytes of appending n_tok tokens (read new K/V, write them into pages)."""
    return int(2 * n_tok * HKV * D * 2)


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling during the timed region (one GPU)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.tmp = None

    def __enter__(self):
        try:
            self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.tmp,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or self.tmp is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.tmp.flush()
        rows = []
        with open(self.tmp.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
                except ValueError:
                    continue
        os.unlink(self.tmp.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(rows), "reasons": reasons}


# ------------------------------------------------------------ distributed
def dist_setup(n_gpus: int):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus and world > 1:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
        pg = dist
    return rank, world, local, pg


def _coll_device(pg) -> str:
    """Where the small collective tensors live: the GPU under NCCL, the host under gloo."""
    return "cuda" if pg.get_backend() == "nccl" else "cpu"


def barrier(pg):
    import torch

    if torch.cuda.is_available():
        torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    if torch.cuda.is_available():
        torch.cuda.synchronize()


def max_over_ranks(pg, x: float) -> float:
    if pg is None:
        return x
    import torch

    t = torch.tensor([x], dtype=torch.float64, device=_coll_device(pg))
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(pg, x: float) -> float:
    if pg is None:
        return x
    import torch

    t = torch.tensor([x], dtype=torch.float64, device=_coll_device(pg))
    pg.all_reduce(t, op=pg.ReduceOp.SUM)
    return float(t.item())


def job_throughput(pg, units_local: float, seconds_local: float) -> tuple[float, float]:
    """Whole-job rate over the replicas: every rank's units over the slowest rank's time."""
    t_max = max_over_ranks(pg, seconds_local)
    return sum_over_ranks(pg, units_local) / t_max, t_max


# ---------------------------------------------------------------- our arm
N_BATCHES = 6  # disjoint 64-sequence batches the steps rotate through (inputs > L2 without a flush)


def build_state(steps_total: int, device, n_batches: int = N_BATCHES):
    """The pool and n_batches disjoint batches of the config-2 workload.

    Every batch has the same 64 context lengths (seed 2); the block tables of
    all batches are disjoint slices of one random permutation of the pool's
    page ids (seed 3).  Step j runs batch j % n_batches, whose sequences then
    grow by one token, so a step's K/V were last read n_batches - 1 steps
    (about 355 MB of other K/V) earlier: more than the 126 MB L2 holds.
    """
    import torch

    from mitten_b200 import paged

    lens0 = make_lens()
    per_batch_steps = (steps_total + n_batches - 1) // n_batches
    need = [(int(L) + per_batch_steps + 1 + PS - 1) // PS for L in lens0]
    assert sum(need) * n_batches <= NUM_PAGES
    rng = np.random.default_rng(3)
    perm = rng.permutation(NUM_PAGES).astype(np.int32)
    indptr = np.zeros(N_SEQS + 1, np.int32)
    indptr[1:] = np.cumsum(need)
    pool = paged.PagedKVPool(1, NUM_PAGES, PS, HKV, D, device=device)
    gen = torch.Generator(device=device)
    gen.manual_seed(4)
    batches = []
    for b in range(n_batches):
        tables = perm[b * indptr[-1]: (b + 1) * indptr[-1]]
        # initial context: L_s tokens per sequence, written with the append kernel
        slots = np.concatenate([tables[indptr[s] + np.arange(L) // PS].astype(np.int64) * PS + np.arange(L) % PS
                                for s, L in enumerate(lens0)])
        n0 = len(slots)
        for lo in range(0, n0, 1 << 18):
            hi = min(n0, lo + (1 << 18))
            k = torch.randn((hi - lo, HKV, D), generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
            v = torch.randn((hi - lo, HKV, D), generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
            pool.append(0, k, v, torch.from_numpy(slots[lo:hi]).to(device))
        batches.append({"tables": tables.copy(), "indices": torch.from_numpy(tables.copy()).to(device)})
    torch.cuda.synchronize()
    return {"pool": pool, "lens0": lens0, "indptr": torch.from_numpy(indptr).to(device), "indptr_np": indptr,
            "batches": batches, "n_batches": n_batches, "gen": gen,
            # batch 0 under the names the single-batch tools use
            "indices": batches[0]["indices"], "tables": batches[0]["tables"]}


def step_batch(st, step: int) -> int:
    return step % st["n_batches"]


def step_inputs(st, step: int, device):
    """Slots and seq_lens (host numpy) of step `step`: batch step % n_batches, grown step // n_batches times."""
    b = step_batch(st, step)
    pos = st["lens0"] + step // st["n_batches"]  # position of the appended token
    tables, indptr = st["batches"][b]["tables"], st["indptr_np"]
    slots = (tables[indptr[:-1] + pos // PS].astype(np.int64) * PS + pos % PS).astype(np.int64)
    return slots, (pos + 1).astype(np.int32)


def run_ours(args, rank, world, local, pg):
    import torch

    from mitten_b200 import paged

    device = torch.device("cuda", local)
    total_steps = args.warmup + args.steps
    st = build_state(total_steps + 1, device)
    pool = st["pool"]
    ws = paged.DecodeWorkspace.for_shape(pool, N_SEQS, HQ)
    gen = st["gen"]
    q_all = torch.randn((total_steps, N_SEQS, HQ, D), generator=gen, device=device).to(torch.bfloat16)
    k_all = torch.randn((total_steps, N_SEQS, HKV, D), generator=gen, device=device).to(torch.bfloat16)
    v_all = torch.randn((total_steps, N_SEQS, HKV, D), generator=gen, device=device).to(torch.bfloat16)
    lens_np = [step_inputs(st, i, device)[1] for i in range(total_steps)]
    lens_all = torch.from_numpy(np.stack(lens_np)).to(device)
    out = torch.empty((N_SEQS, HQ, D), dtype=torch.bfloat16, device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    scale = D ** -0.5

    def step(i):
        # One launch: append this step's K/V at position len-1, then decode.
        b = st["batches"][step_batch(st, i)]
        paged.paged_decode(pool, 0, q_all[i], st["indptr"], b["indices"], lens_all[i], scale=scale,
                           phantom=False, k_new=k_all[i], v_new=v_all[i], out=out, workspace=ws)

    for i in range(args.warmup):  # also configures the kernel before capture
        step(i)
    torch.cuda.synchronize()
    # All K timed steps in one CUDA graph: consecutive decode launches keep
    # their programmatic-dependent-launch edges (the next step's CTAs start
    # their prologue on SMs the previous step frees, then wait for it).
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for j in range(args.steps):
            step(args.warmup + j)
    torch.cuda.synchronize()
    barrier(pg)
    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(pg)
        ev0.record(stream)
        graph.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier(pg)
    t_step = ev0.elapsed_time(ev1) * 1e-3
    del graph
    # The same steps again, one at a time after an L2-flushing write, for
    # comparison (their appends rewrite the same rows with the same values).
    graphs = []
    for j in range(args.steps):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step(args.warmup + j)
        graphs.append(g)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    for j in range(args.steps):
        flush.zero_()
        evs[j][0].record(stream)
        graphs[j].replay()
        evs[j][1].record(stream)
    torch.cuda.synchronize()
    t_flushed = sum(evs[j][0].elapsed_time(evs[j][1]) * 1e-3 for j in range(args.steps))
    code, detail = paged.device_error(local)
    if code:
        raise SystemExit(f"device error {code} (detail {detail}) during the bench")
    dec_bytes = [decode_bytes(lens_np[args.warmup + j].astype(np.int64)) + append_bytes(N_SEQS)
                 for j in range(args.steps)]
    kv_bytes = sum(int(lens_np[args.warmup + j].sum()) * B_TOK for j in range(args.steps))
    del graphs

    # ---- e2e through the C ABI with pinned host buffers
    e2e = run_e2e(args, st, pool, ws, device, stream, total_steps)
    # ---- the other two HBM-bound kernels of the path, on free pages
    extras = run_append_and_copy(st, pool, device, stream)

    value, t_max = job_throughput(pg, float(N_SEQS * args.steps), t_step)
    e2e_value, _ = job_throughput(pg, float(N_SEQS * e2e["steps"]), e2e["t"])
    peaks = load_peaks()
    achieved = (sum(dec_bytes) / len(dec_bytes)) / (t_step / args.steps) / 1e9
    res = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * t_max / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) Q/K/V)",
        "config": workload_config(),
        "execution": {"replicas": world, "step": "one fused append+decode launch per step; the K timed steps "
                                                  "captured in one CUDA graph, replayed between two events"},
        "kv_read_gbs": sum_over_ranks(pg, kv_bytes) / t_max / 1e9,
        "decode_us_per_step": 1e6 * t_step / args.steps,
        "per_step_l2_flushed_us": 1e6 * t_flushed / args.steps,
        "roofline": {"bound": "hbm", "kernel": "paged_decode_kernel<64,7> (append fused)", "achieved": achieved,
                     "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     "peak_source": peaks["source"], "traffic": traffic_from_profile(),
                     "algorithmic_bytes_per_launch": sum(dec_bytes) / len(dec_bytes)},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": e2e["h2d"],
                "d2h_bytes_per_step": e2e["d2h"], "steps": e2e["steps"],
                "path": "per step: Q/K/V/seq_lens packed in one pinned host buffer -> one H2D copy -> "
                        "mtn_paged_decode (C ABI) -> D2H output; steps in groups of 8: group g+1's H2D and "
                        "group g-1's D2H overlap group g's kernels (upload/download streams, 16 staging and 16 "
                        "output buffers, only a group's first launch waits on copy events), batches rotating "
                        "as above"},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
        "kv_append_bulk": extras["append"],
        "page_copy": extras["copy"],
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    return res


def run_append_and_copy(st, pool, device, stream) -> dict:
    """Bandwidth of the bulk KV append (64 sequences x 512 tokens per call, the prefill-append shape)
    and of the copy-on-write page copy (3072 pages per call), each timed as 24 calls captured in one
    CUDA graph (so host launch cost is not timed) that rotate through sources and destinations larger
    than L2 together.  Destinations are pool pages no batch uses; page-copy sources are batch pages
    (read only)."""
    import torch

    peak = load_peaks()["hbm_gbs"]
    used = st["n_batches"] * int(st["indptr_np"][-1])
    free = np.random.default_rng(3).permutation(NUM_PAGES).astype(np.int64)[used:]
    res = {}
    # bulk append: 32768 tokens, 2 x 32768 x HKV x D bf16 read + the same written + 8 B slots
    n_tok, n_calls = 64 * 512, 24
    pages_per_call = n_tok // PS
    gen = torch.Generator(device=device)
    gen.manual_seed(6)
    srcs = [(torch.randn((n_tok, HKV, D), generator=gen, device=device).to(torch.bfloat16),
             torch.randn((n_tok, HKV, D), generator=gen, device=device).to(torch.bfloat16)) for _ in range(6)]
    dsts = []
    for j in range(max(1, min(3, len(free) // pages_per_call))):
        pg = free[j * pages_per_call:(j + 1) * pages_per_call]
        dsts.append(torch.from_numpy((np.repeat(pg, PS) * PS + np.tile(np.arange(PS), len(pg))).astype(np.int64))
                    .to(device))

    def app(i):
        k, v = srcs[i % len(srcs)]
        pool.append(0, k, v, dsts[i % len(dsts)])

    def timed(fn):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(n_calls):
                fn(i)
        g.replay()  # warm
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        g.replay()
        b.record(stream)
        b.synchronize()
        del g
        return a.elapsed_time(b) * 1e-3 / n_calls

    t = timed(app)
    nbytes = append_bytes(n_tok) * 2 + 8 * n_tok
    res["append"] = {"kernel": "kv_append_kernel<bf16>", "tokens_per_call": n_tok, "bytes_per_call": nbytes,
                     "us_per_call": 1e6 * t, "gbs": nbytes / t / 1e9, "frac": nbytes / t / 1e9 / peak,
                     "peak_gbs": peak}
    # page copy: 3072 pages of one layer, K and V (2 x 3072 x PS x HKV x D x 2 B read, the same written)
    n_pg = 3072
    n_dst = max(1, min(3, len(free) // n_pg))
    batch_pages = np.random.default_rng(3).permutation(NUM_PAGES).astype(np.int32)[:used]
    src_sets = [torch.from_numpy(batch_pages[j * n_pg:(j + 1) * n_pg].copy()).to(device)
                for j in range(min(6, used // n_pg))]
    dst_sets = [torch.from_numpy(free[j * n_pg:(j + 1) * n_pg].astype(np.int32)).to(device) for j in range(n_dst)]

    def cp(i):
        pool.page_copy(src_sets[i % len(src_sets)], dst_sets[i % len(dst_sets)])

    t = timed(cp)
    nbytes = 2 * n_pg * 2 * PS * HKV * D * 2 + 8 * n_pg
    res["copy"] = {"kernel": "page_copy_bulk_kernel", "pages_per_call": n_pg, "bytes_per_call": nbytes,
                   "us_per_call": 1e6 * t, "gbs": nbytes / t / 1e9, "frac": nbytes / t / 1e9 / peak,
                   "peak_gbs": peak}
    return res


def e2e_schedule(n: int, group: int = 8) -> list:
    """Host issue order of run_e2e's pipeline for n steps: (op, step, deps) with op one of
    "upload" (host -> staging buffer step % 2group, upload stream), "kernel" (the decode of that
    step, compute stream) or "download" (its output buffer step % 2group -> host, download stream);
    deps are the (op, step) events the op's stream waits for first.  Groups of `group` steps: the
    uploads of group g+2 are issued once group g's kernels are, each waiting for the kernel that
    last read its staging buffer; only a group's first kernel waits, for its group's uploads and
    for the downloads of group g-2 (the last users of the output buffers the group writes)."""
    nb = 2 * group
    ops = []

    def upload(j):
        ops.append(("upload", j, [("kernel", j - nb)] if j >= nb else []))

    for j in range(min(n, nb)):  # groups 0 and 1
        upload(j)
    for j in range(n):
        deps = []
        if j % group == 0:
            deps = [("upload", u) for u in range(j, min(n, j + group))]
            deps += [("download", u) for u in range(j - nb, j - nb + group) if u >= 0]
        ops.append(("kernel", j, deps))
        ops.append(("download", j, [("kernel", j)]))
        if j % group == group - 1:
            for u in range(j + 1 + group, min(n, j + 1 + nb)):
                upload(u)
    return ops


def run_e2e(args, st, pool, ws, device, stream, total_steps):
    """Append + decode through the C ABI with host inputs/outputs copied inside the timed region.

    Each step's Q, new K/V and seq_lens are packed in one pinned host buffer and copied in with one
    H2D copy; O comes back with one D2H copy.  Copies overlap the kernels: the steps run in groups
    of G = 8; the uploads of group g+1 (on an upload stream) and the downloads of group g-1 (on a
    download stream) run while group g's kernels run, through 2G device staging and 2G output
    buffers.  Only the first launch of a group waits (by events) for its group's uploads and for
    the downloads that free its output buffers, so the other seven keep the kernel-to-kernel edge
    that lets a decode launch start while the previous one finishes (an event wait in front of
    every launch measured ~3 us more per step).  All K steps are captured in one CUDA graph and
    replayed between two events.
    """
    import ctypes as C

    import torch

    from mitten_b200 import _lib

    lib = _lib.lib()
    steps = args.steps
    G = 8
    NB = 2 * G  # staging and output buffers
    gen = torch.Generator()
    gen.manual_seed(5)
    q_h = torch.randn((N_SEQS, HQ, D), generator=gen).to(torch.bfloat16)
    k_h = torch.randn((N_SEQS, HKV, D), generator=gen).to(torch.bfloat16)
    v_h = torch.randn((N_SEQS, HKV, D), generator=gen).to(torch.bfloat16)
    parts = [q_h.view(torch.uint8).reshape(-1), k_h.view(torch.uint8).reshape(-1), v_h.view(torch.uint8).reshape(-1)]
    offs = np.cumsum([0] + [x.numel() for x in parts]).tolist()  # byte offsets (multiples of 16)
    nbytes = offs[-1] + N_SEQS * 4
    stage_h = []
    for i in range(total_steps):
        buf = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        for x, o in zip(parts, offs):
            buf[o:o + x.numel()].copy_(x)
        lens_i = np.ascontiguousarray(step_inputs(st, i, device)[1], np.int32)
        buf[offs[3]:].copy_(torch.from_numpy(lens_i).view(torch.uint8))
        stage_h.append(buf)
    o_h = [torch.empty((N_SEQS, HQ, D), dtype=torch.bfloat16).pin_memory() for _ in range(total_steps)]
    stage_d = [torch.empty(nbytes, dtype=torch.uint8, device=device) for _ in range(NB)]
    o_d = [torch.empty((N_SEQS, HQ, D), dtype=torch.bfloat16, device=device) for _ in range(NB)]
    scale = D ** -0.5
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def call(i, buf):
        sp = int(torch.cuda.current_stream().cuda_stream)
        b = st["batches"][step_batch(st, i)]
        base = stage_d[buf].data_ptr()
        q_p, k_p, v_p, l_p = (base + o for o in offs)
        _lib.check(lib.mtn_paged_decode(C.byref(pool.layout), 0, q_p, _lib.MTN_DTYPE_BF16,
                                        o_d[buf].data_ptr(), _lib.MTN_DTYPE_BF16, k_p, v_p,
                                        _lib.MTN_DTYPE_BF16, N_SEQS, HQ, st["indptr"].data_ptr(),
                                        b["indices"].data_ptr(), l_p, scale, 0, ws.buf.data_ptr(),
                                        ws.nbytes, sp))

    def pipeline(first, n):
        """Steps first .. first+n-1 on the current (compute) stream with overlapped copies."""
        comp = torch.cuda.current_stream()
        ev = {kind: [torch.cuda.Event() for _ in range(n)] for kind in ("upload", "kernel", "download")}
        up.wait_stream(comp)
        down.wait_stream(comp)
        for op, j, deps in e2e_schedule(n, G):
            strm = {"upload": up, "kernel": comp, "download": down}[op]
            with torch.cuda.stream(strm):
                for kind, u in deps:
                    strm.wait_event(ev[kind][u])
                if op == "upload":
                    stage_d[j % NB].copy_(stage_h[first + j], non_blocking=True)
                elif op == "kernel":
                    call(first + j, j % NB)
                else:
                    o_h[first + j].copy_(o_d[j % NB], non_blocking=True)
                ev[op][j].record(strm)
        comp.wait_stream(up)
        comp.wait_stream(down)

    # the pool already holds the device arm's appends: these steps rewrite the same positions
    first = total_steps - steps
    pipeline(first, min(3, steps))
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        pipeline(first, steps)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    g.replay()
    b.record(stream)
    b.synchronize()
    t = a.elapsed_time(b) * 1e-3
    del g
    # the last step's output reached the host
    ref_out = o_d[(steps - 1) % NB].cpu()
    if not torch.equal(o_h[first + steps - 1], ref_out):
        raise SystemExit("e2e: the downloaded output differs from the device output")
    h2d = nbytes
    d2h = o_h[0].numel() * o_h[0].element_size()
    return {"t": t, "steps": steps, "h2d": h2d, "d2h": d2h}


# ------------------------------------------------------------ CPU baseline
def cpu_workload(n_steps_cap: int, seconds: float, threads_note: str):
    """Time the oracle port of the reference decode step (cat-grown caches) on the host."""
    import oracle

    lens = make_lens()
    rng = np.random.default_rng(4)
    kp, vp = [], []
    for L in lens:
        k = np.zeros((HKV, int(L) + 1, D), np.float32)
        v = np.zeros((HKV, int(L) + 1, D), np.float32)
        k[:, 1:] = rng.standard_normal((HKV, int(L), D), dtype=np.float32)
        v[:, 1:] = rng.standard_normal((HKV, int(L), D), dtype=np.float32)
        kp.append(k)
        vp.append(v)
    dec = oracle.CatGrownDecode(kp, vp, HQ, D ** -0.5)
    done, t = 0, 0.0
    while done < n_steps_cap and t < seconds:
        q = rng.standard_normal((N_SEQS, HQ, D), dtype=np.float32)
        kn = rng.standard_normal((N_SEQS, HKV, D), dtype=np.float32)
        vn = rng.standard_normal((N_SEQS, HKV, D), dtype=np.float32)
        t0 = time.perf_counter()
        dec.step(q, kn, vn)
        t += time.perf_counter() - t0
        done += 1
    dec.close()
    return done, t


def cpu_baseline(seconds: float) -> dict:
    import oracle

    oracle.build()
    cores = oracle.num_threads()
    done, t = cpu_workload(10 ** 9, seconds, "")
    return {"value": N_SEQS * done / t, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{done} decode steps of the full config-2 batch (64 seqs) through the oracle port of the "
                      f"reference cat-grown f32 decode (Tensor::cat growth, GQA repeat, -1e10 mask, softmax), "
                      f"{t:.1f} s, OpenMP {cores} threads"}


def run_reference(args, rank, world):
    """The reference's CPU algorithm (oracle port; the Rust reference cannot be built here)."""
    import oracle

    oracle.build()
    cores = oracle.num_threads()
    # bounded: every step is the whole 64-sequence decode step; cap total time
    warm, _ = cpu_workload(max(args.warmup, 0), 60.0, "")
    done, t = cpu_workload(args.steps, args.ref_seconds, "")
    value = N_SEQS * done / t
    return {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": done,
        "warmup": args.warmup, "ms_per_step": 1e3 * t / max(done, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) Q/K/V)",
        "config": workload_config(), "execution": {"host_cores": cores}, "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{done} of {args.steps} requested steps of the full config-2 batch "
                                   f"(cap {args.ref_seconds:.0f} s); the Rust reference cannot be built here"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------ configs 3 and 4 (kernels only)
def _graph_steps(fns, stream):
    """Capture each step function in its own CUDA graph; time all replays back to back."""
    import torch

    for f in fns[:3]:
        f()
    torch.cuda.synchronize()
    graphs = []
    for f in fns:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            f()
        graphs.append(g)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for g in graphs:
        g.replay()
    b.record(stream)
    b.synchronize()
    del graphs
    return a.elapsed_time(b) * 1e-3


def model_weights(shape, device, seed: int = 0, std: float = 0.02) -> dict:
    """Random N(0, std) weights of a QwenPagedModel shape, generated on the device (norm weights 0, i.e.
    a (1 + w) scale of 1), under the names the model reads."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    h, d, L = shape.hidden, shape.head_dim, shape.layers

    def rnd(*sz):
        return torch.randn(sz, generator=g, device=device, dtype=torch.float32) * std

    w = {"embedding.weight": rnd(shape.vocab, h), "norm.weight": torch.zeros(h, device=device)}
    for li in range(L):
        m, pfx = f"layers.{li}.mixer", f"layers.{li}"
        w[f"{m}.q_proj.weight"] = rnd(shape.hq * d * (2 if shape.gated_q else 1), h)
        w[f"{m}.k_proj.weight"] = rnd(shape.hkv * d, h)
        w[f"{m}.v_proj.weight"] = rnd(shape.hkv * d, h)
        w[f"{m}.o_proj.weight"] = rnd(h, shape.hq * d)
        if shape.qk_norm:
            w[f"{m}.q_norm.weight"] = torch.zeros(d, device=device)
            w[f"{m}.k_norm.weight"] = torch.zeros(d, device=device)
        w[f"{pfx}.norm.weight"] = torch.zeros(h, device=device)
        w[f"{pfx}.ffn_norm.weight"] = torch.zeros(h, device=device)
        w[f"{pfx}.mlp.gate_proj.weight"] = rnd(shape.inter, h)
        w[f"{pfx}.mlp.up_proj.weight"] = rnd(shape.inter, h)
        w[f"{pfx}.mlp.down_proj.weight"] = rnd(h, shape.inter)
    return w


def run_cfg1(args, local) -> dict:
    """BASELINE config 1 end to end through the engine: the Qwen2.5-0.5B-shaped model (24 layers, hidden
    896, 14 q / 2 kv heads, head_dim 64, SwiGLU 4864, vocab 151936, tied embeddings, random N(0, 0.02)
    f32 weights), page 16, 4 requests of 128 random prompt tokens (seed 1) and 32 greedy decode steps.
    Each engine iteration is the scheduler mirror (C++) -> QwenPagedModel.forward (dense parts on the
    device BLAS in f32, attention on the paged kernels) -> device argmax -> token hand-back.  Reported:
    decode tokens/s over the 32 decode iterations (CUDA events around the loop, so host scheduling and
    launches count) and the prefill iteration's time."""
    import torch

    from mitten_b200 import host, model as M

    dev = torch.device("cuda", local)
    shape = M.QWEN_CONFIG1
    n_req, prompt_len, steps = 4, 128, 32
    weights = model_weights(shape, dev, seed=0)
    prompts = np.random.default_rng(1).integers(0, shape.vocab, size=(n_req, prompt_len)).astype(np.uint32)
    times = []
    for trial in range(2):  # the first pass warms the kernels and the BLAS
        mdl = M.QwenPagedModel(shape, weights, num_pages=256, page_size=16, device=dev)
        sched = host.Scheduler(256, 16, max_prefill_tokens_per_iter=512, max_decode_batch_size=8,
                               eos_token_ids=(shape.vocab,))
        for rid in range(n_req):
            sched.add_request(rid, prompts[rid], temperature=0.0, max_new_tokens=steps)
        eng = M.Engine(mdl, sched)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        eng.step()  # the prefill iteration (all four prompts fit the 512-token budget)
        ev[1].record()
        eng.run()
        ev[2].record()
        torch.cuda.synchronize()
        times.append((ev[0].elapsed_time(ev[1]) * 1e-3, ev[1].elapsed_time(ev[2]) * 1e-3, eng.iterations))
        outs = [sched.request_output(r) for r in range(n_req)]
    t_pre, t_dec, iters = times[-1]
    dec_tokens = n_req * (steps - 1)  # the prefill iteration already emitted each request's first token
    # device time of one decode step alone: the batch-4 graph replayed back to back
    g = mdl._graphs.get(n_req)
    replay_ms = None
    if g is not None and g.graph is not None:
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record()
        for _ in range(10):
            g.graph.replay()
        ev[1].record()
        torch.cuda.synchronize()
        replay_ms = ev[0].elapsed_time(ev[1]) / 10
    return {"metric": "config 1 engine decode tokens/s (Qwen2.5-0.5B shape, random weights)",
            "value": dec_tokens / t_dec, "unit": "tokens/s", "n_gpus": 1, "steps": iters - 1, "warmup": 1,
            "ms_per_step": 1e3 * t_dec / max(iters - 1, 1), "higher_is_better": True, "dtype": "f32 dense, bf16 K/V",
            "data": "synthetic (random N(0,0.02) weights seed 0, random prompt tokens seed 1)",
            "config": {"workload": "BASELINE config 1: 4 requests x 128-token prompts, 32 greedy decode steps, "
                                   "page 16, whole engine loop (scheduler, model forward, device argmax)"},
            "prefill_iteration_ms": 1e3 * t_pre, "decode_graph_replay_ms": replay_ms,
            "outputs_per_request": [len(o) for o in outs],
            "gpu_launches": None}


def run_cfg3(args, local) -> dict:
    """BASELINE config 3's attention layer: 128 sequences share a 1032-token prefix (64 full pages and
    a partial one, refcounted), each with its own suffix U[64, 512] (seed 6) and its own copy of the
    partial page (copy-on-write), Qwen2.5-7B attention shapes (28 q / 4 kv heads, head_dim 128).
    One step = fused append + decode over all 128 sequences of one layer; steps rotate through 3
    disjoint copies of the workload (logical K/V per step far above L2; the shared prefix is read 128
    times within a step, which is the reuse the shared pages exist for)."""
    import torch

    from mitten_b200 import paged

    dev = torch.device("cuda", local)
    hq, hkv, d, ps, n = 28, 4, 128, 16, 128
    prefix = 1032
    suf = np.random.default_rng(6).integers(64, 513, size=n)
    steps = args.steps
    per_copy_pages = (prefix + ps - 1) // ps + sum((prefix + int(s) + steps + ps) // ps - prefix // ps for s in suf)
    n_copies = 3
    num_pages = n_copies * per_copy_pages + 64
    pool = paged.PagedKVPool(1, num_pages, ps, hkv, d, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    pool.storage.normal_(generator=gen)
    copies, nxt, cow_src, cow_dst = [], 0, [], []
    for c in range(n_copies):
        shared = list(range(nxt, nxt + (prefix + ps - 1) // ps))
        nxt += len(shared)
        tables = []
        for s in suf:
            own = list(shared[:-1]) + [nxt]  # private copy of the partial prefix page
            cow_src.append(shared[-1])
            cow_dst.append(nxt)
            nxt += 1
            need = (prefix + int(s) + steps + ps) // ps
            while len(own) < need:
                own.append(nxt)
                nxt += 1
            tables.append(own)
        indptr = np.concatenate([[0], np.cumsum([len(t) for t in tables])]).astype(np.int32)
        n_full = prefix // ps  # the full prefix pages every table starts with
        own = [t[n_full:] for t in tables]
        own_ptr = np.concatenate([[0], np.cumsum([len(t) for t in own])]).astype(np.int32)
        copies.append({"indptr": torch.from_numpy(indptr).to(dev),
                       "indices": torch.from_numpy(np.concatenate(tables).astype(np.int32)).to(dev),
                       "prefix": torch.tensor(shared[:n_full], dtype=torch.int32, device=dev),
                       "own_indptr": torch.from_numpy(own_ptr).to(dev),
                       "own_indices": torch.from_numpy(np.concatenate(own).astype(np.int32)).to(dev)})
    assert nxt <= num_pages
    # copy-on-write of every sequence's partial prefix page (128 pages per copy of the workload)
    src_t = torch.tensor(cow_src[:n], dtype=torch.int32, device=dev)
    dst_t = torch.tensor(cow_dst[:n], dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    t_cow = _graph_steps([lambda: pool.page_copy(src_t, dst_t)] * 8, stream) / 8
    ws = paged.DecodeWorkspace.for_shape(pool, n, hq)
    q = torch.randn((n, hq, d), generator=gen, device=dev).to(torch.bfloat16)
    kn = torch.randn((n, hkv, d), generator=gen, device=dev).to(torch.bfloat16)
    vn = torch.randn((n, hkv, d), generator=gen, device=dev).to(torch.bfloat16)
    out = torch.empty((n, hq, d), dtype=torch.bfloat16, device=dev)
    lens = [torch.from_numpy((prefix + suf + 1 + j // n_copies).astype(np.int32)).to(dev)
            for j in range(args.warmup + steps)]

    def step(j):
        c = copies[j % n_copies]
        return lambda: paged.paged_decode(pool, 0, q, c["indptr"], c["indices"], lens[j], k_new=kn, v_new=vn,
                                          out=out, workspace=ws)

    for j in range(args.warmup):
        step(j)()
    t = _graph_steps([step(args.warmup + j) for j in range(steps)], stream)
    # The same steps with the prefix's 64 full pages attended once for the
    # whole batch (mtn_paged_decode_shared_prefix), each sequence's own part
    # (the copied partial page and its suffix) by the decode kernel.
    n_full = prefix // ps
    own_lens = [l - n_full * ps for l in lens]
    sp_ws = paged.shared_prefix_workspace(pool, n, hq)
    out_sp = torch.empty_like(out)

    def step_sp(j):
        c = copies[j % n_copies]
        return lambda: paged.paged_decode_shared_prefix(pool, 0, q, c["prefix"], c["own_indptr"], c["own_indices"],
                                                        own_lens[j], k_new=kn, v_new=vn, out=out_sp,
                                                        workspace=sp_ws)

    for j in range(args.warmup):
        step_sp(j)()
    t_sp = _graph_steps([step_sp(args.warmup + j) for j in range(steps)], stream)
    b_tok = 2 * hkv * d * 2
    logical = float(sum((prefix + suf + 1).astype(np.int64))) * b_tok
    unique = (prefix + float(np.sum(suf + 1))) * b_tok
    peak = load_peaks()["hbm_gbs"]
    code, detail = paged.device_error(local)
    if code:
        raise SystemExit(f"device error {code} (detail {detail})")
    return {"metric": "config 3 decode attention over shared prefix pages", "value": n * steps / t,
            "unit": "tokens/s", "n_gpus": 1, "steps": steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * t / steps, "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "BASELINE config 3 attention layer: 128 seqs, 1032-token shared prefix "
                                   "(64 full + 1 partial page, copy-on-write), suffix U[64,512] seed 6, "
                                   "Hq 28 / Hkv 4 / D 128, page 16, 1 layer, append fused",
                       "l2": "3 disjoint copies of the workload rotate step to step"},
            "logical_kv_gbs": logical / (t / steps) / 1e9, "unique_kv_gbs": unique / (t / steps) / 1e9,
            "unique_frac_of_hbm": unique / (t / steps) / 1e9 / peak,
            "cow_page_copy_us_per_128_pages": 1e6 * t_cow, "gpu_launches": steps,
            "shared_prefix": {"call": "mtn_paged_decode_shared_prefix (prefix once per batch, LSE combine)",
                              "ms_per_step": 1e3 * t_sp / steps, "tokens_per_s": n * steps / t_sp,
                              "speedup": t / t_sp, "unique_kv_gbs": unique / (t_sp / steps) / 1e9,
                              "launches_per_step": 3}}


def run_cfg3_engine(args, local) -> dict:
    """BASELINE config 3 through the engine: the Qwen2.5-7B-shaped model (random N(0,0.02) bf16 weights),
    a parent request holding a 1032-token random prefix (seed 5) and 128 children forked off it
    (mtn_sched_fork: each shares the prefix pages, the partial last page included), each with its own
    random suffix of U[64, 512] tokens (lengths seed 6, tokens seed 7).  A child's first write into the
    shared partial page copies it (copy-on-write).  Once every request decodes, `steps` (at most 32)
    decode-only engine iterations of the 129-request batch are timed with CUDA events around the loop
    (scheduler, copies, the forward replayed from a CUDA graph, device argmax, token hand-back).
    Checked: exactly 128 copy-on-write copies of the partial page."""
    import torch

    from mitten_b200 import host, model as M

    dev = torch.device("cuda", local)
    shape = M.DecoderShape(**QWEN7B)
    n, prefix_len, ps = 128, 1032, 16
    timed = max(1, min(args.steps, 32))
    out_tokens = timed + 24  # the children decode during the later prefill iterations too
    prefix = np.random.default_rng(5).integers(0, shape.vocab, prefix_len).astype(np.uint32)
    suf_lens = np.random.default_rng(6).integers(64, 513, size=n)
    tok = np.random.default_rng(7)
    suffixes = [tok.integers(0, shape.vocab, int(k)).astype(np.uint32) for k in suf_lens]
    num_pages = (prefix_len + ps - 1) // ps + 1 + sum((int(k) + out_tokens + 2 * ps) // ps for k in suf_lens) + 64
    w = model_weights(shape, dev, seed=0)
    model = M.QwenPagedModel(shape, w, num_pages, ps, device=dev, split_bf16=False, dtype=torch.bfloat16)
    del w
    torch.cuda.empty_cache()
    sched = host.Scheduler(num_pages, ps, max_prefill_tokens_per_iter=8192, max_decode_batch_size=n + 1,
                           eos_token_ids=(shape.vocab,))
    sched.add_request(0, prefix, temperature=0.0, max_new_tokens=out_tokens + 32)
    eng = M.Engine(model, sched, cuda_graphs=True)
    cows, it = 0, 0
    t0 = time.perf_counter()
    while True:  # prefill: the parent, then the children's suffixes (their own pages, the partial page copied)
        b = sched.schedule()
        cows += len(b.cow_src)
        lg = model.forward(b)
        sched.process_tokens(M.paged.argmax_rows(lg).cpu().numpy().astype(np.uint32))
        if it == 0:
            for k, suf in enumerate(suffixes):
                sched.fork(0, k + 1, suf, temperature=0.0, max_new_tokens=out_tokens)
        it += 1
        if all(sched.request_info(r)["state"] == 2 for r in range(n + 1)):
            break
    torch.cuda.synchronize(dev)
    prefill_s = time.perf_counter() - t0
    eng.step()  # first decode-only batch: eager run + capture of the batch's CUDA graph
    torch.cuda.synchronize(dev)
    done0 = sum(len(sched.request_output(r)) for r in range(n + 1))
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(timed):
        eng.step()
    e.record()
    e.synchronize()
    t = a.elapsed_time(e) * 1e-3
    tokens = sum(len(sched.request_output(r)) for r in range(n + 1)) - done0
    code, detail = M.paged.device_error(local)
    if code:
        raise SystemExit(f"device error {code} (detail {detail}) in the config-3 engine run")
    if cows != n:
        raise SystemExit(f"config-3 engine run: {cows} copy-on-write copies, expected {n}")
    return {"metric": "config 3 engine decode tokens/s (Qwen2.5-7B shape, shared 1032-token prefix, CoW)",
            "value": tokens / t, "unit": "tokens/s", "n_gpus": 1, "steps": timed, "warmup": 1,
            "ms_per_step": 1e3 * t / timed, "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic (random N(0,0.02) bf16 weights seed 0, random tokens seeds 5-7)",
            "config": {"workload": "BASELINE config 3 through the engine: 128 children forked off a 1032-token "
                                   "prefix (64 full pages + 1 partial, refcounted), suffix U[64,512], "
                                   f"{timed} decode steps timed (trimmed from 128)", "requests": n + 1},
            "prefill_s": prefill_s, "prefill_iterations": it, "cow_copies": cows,
            "decode_tokens": tokens, "gpu_launches": None}


def run_cfg4_engine(args, local) -> dict:
    """BASELINE config 4 through the engine: the Gemma-2B-shaped model (MQA 8 q / 1 kv head, head_dim 256,
    GeGLU 16384, vocab 256000, random N(0,0.02) bf16 weights), continuous batching.  96 requests with
    prompts U[512, 8192] (seed 7) are prefilled first, under the same per-iteration token budget as the
    timed part (2048 prefill tokens plus the decode rows).  Then every timed iteration four new
    512-token requests arrive (tokens seed 8), so each iteration is one mixed batch: the decoding
    requests (96 at the start, four more each iteration) plus four 512-token prefill chunks through one
    forward (paged prefill and decode attention), device argmax, token hand-back.  Timed with CUDA
    events around 24 iterations (trimmed), host scheduling and launches included."""
    import torch

    from mitten_b200 import host, model as M

    dev = torch.device("cuda", local)
    shape = M.GEMMA_2B
    n_dec, n_new, chunk, ps = 96, 4, 512, 16
    timed = max(1, min(args.steps, 24))
    lens = np.random.default_rng(7).integers(512, 8193, size=n_dec)
    tok = np.random.default_rng(8)
    prompts = [tok.integers(0, shape.vocab, int(k)).astype(np.uint32) for k in lens]
    arrivals = [[tok.integers(0, shape.vocab, chunk).astype(np.uint32) for _ in range(n_new)] for _ in range(timed + 1)]
    max_dec = n_dec + n_new * (timed + 1)
    budget = n_new * chunk + max_dec
    out_cap = 512
    num_pages = sum((int(k) + out_cap + ps) // ps for k in lens)
    num_pages += (timed + 1) * n_new * ((chunk + out_cap + ps) // ps) + 64
    w = model_weights(shape, dev, seed=0)
    model = M.QwenPagedModel(shape, w, num_pages, ps, device=dev, split_bf16=False, dtype=torch.bfloat16)
    del w
    torch.cuda.empty_cache()
    sched = host.Scheduler(num_pages, ps, max_prefill_tokens_per_iter=budget, max_decode_batch_size=max_dec,
                           eos_token_ids=(shape.vocab,))
    for r in range(n_dec):
        sched.add_request(r, prompts[r], temperature=0.0, max_new_tokens=out_cap)
    eng = M.Engine(model, sched, cuda_graphs=False)
    t0 = time.perf_counter()
    while any(sched.request_info(r)["state"] in (0, 1) for r in range(n_dec)):  # waiting or prefilling
        eng.step()
    torch.cuda.synchronize(dev)
    prefill_s = time.perf_counter() - t0
    nxt = n_dec

    def arrive(k):
        nonlocal nxt
        for pr in arrivals[k]:
            sched.add_request(nxt, pr, temperature=0.0, max_new_tokens=out_cap)
            nxt += 1

    arrive(0)
    eng.step()  # warm-up: one mixed iteration
    torch.cuda.synchronize(dev)
    rows, pf_tokens = [], 0
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for k in range(timed):
        arrive(k + 1)
        b = sched.schedule()
        rows.append((b.n_reqs - b.n_prefill, b.n_prefill))
        pf_tokens += int(b.qo_indptr[b.n_prefill])
        lg = model.forward(b)
        sched.process_tokens(M.paged.argmax_rows(lg).cpu().numpy().astype(np.uint32))
    e.record()
    e.synchronize()
    t = a.elapsed_time(e) * 1e-3
    code, detail = M.paged.device_error(local)
    if code:
        raise SystemExit(f"device error {code} (detail {detail}) in the config-4 engine run")
    dec_rows = sum(r[0] for r in rows)
    return {"metric": "config 4 engine decode tokens/s (Gemma-2B shape, continuous batching)",
            "value": dec_rows / t, "unit": "tokens/s", "n_gpus": 1, "steps": timed, "warmup": 1,
            "ms_per_step": 1e3 * t / timed, "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic (random N(0,0.02) bf16 weights seed 0, random tokens seeds 7-8)",
            "config": {"workload": "BASELINE config 4 through the engine: decode rows (96, +4 per iteration) + 4 "
                                   "prefill chunks of 512 tokens per iteration (new requests), contexts "
                                   f"U[512, 8192], {timed} mixed iterations timed (trimmed)"},
            "prefill_tokens_per_s": pf_tokens / t,
            "decode_rows_first_last": [rows[0][0], rows[-1][0]], "prefill_rows_per_iteration": rows[0][1],
            "initial_prefill_s": prefill_s, "gpu_launches": None}


def run_cfg4(args, local) -> dict:
    """BASELINE config 4's attention layer (Gemma-2B shapes: 8 q / 1 kv head, head_dim 256): per step
    96 decoding sequences with context U[512, 8192] (seed 7) plus 4 prefill chunks of 512 tokens whose
    prior context is U{0, 512, ..., 7680} (seed 8), over one pool.  Decode (append fused) and prefill
    are timed separately: decode as KV GB/s, prefill as TFLOP/s against the measured bf16 peak."""
    import torch

    from mitten_b200 import paged

    dev = torch.device("cuda", local)
    hq, hkv, d, ps = 8, 1, 256, 16
    n_dec, n_pf, chunk = 96, 4, 512
    dl = np.random.default_rng(7).integers(512, 8193, size=n_dec)
    pp = np.random.default_rng(8).integers(0, 16, size=n_pf) * 512
    steps = args.steps
    dec_pages = [(int(L) + args.warmup + steps + 1 + ps - 1) // ps for L in dl]
    pf_pages = [(int(P) + chunk + ps - 1) // ps for P in pp]
    num_pages = sum(dec_pages) + sum(pf_pages) + 16
    perm = np.random.default_rng(3).permutation(num_pages).astype(np.int32)
    pool = paged.PagedKVPool(1, num_pages, ps, hkv, d, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(9)
    pool.storage.normal_(generator=gen)
    off = 0

    def take(k):
        nonlocal off
        t = perm[off:off + k]
        off += k
        return t

    dec_tables = [take(k) for k in dec_pages]
    pf_tables = [take(k) for k in pf_pages]
    d_indptr = torch.from_numpy(np.concatenate([[0], np.cumsum(dec_pages)]).astype(np.int32)).to(dev)
    d_indices = torch.from_numpy(np.concatenate(dec_tables)).to(dev)
    p_indptr = torch.from_numpy(np.concatenate([[0], np.cumsum(pf_pages)]).astype(np.int32)).to(dev)
    p_indices = torch.from_numpy(np.concatenate(pf_tables)).to(dev)
    qo = torch.from_numpy(np.arange(0, (n_pf + 1) * chunk, chunk).astype(np.int32)).to(dev)
    p_lens = torch.from_numpy((pp + chunk).astype(np.int32)).to(dev)
    qd = torch.randn((n_dec, hq, d), generator=gen, device=dev).to(torch.bfloat16)
    kn = torch.randn((n_dec, hkv, d), generator=gen, device=dev).to(torch.bfloat16)
    vn = torch.randn((n_dec, hkv, d), generator=gen, device=dev).to(torch.bfloat16)
    qp = torch.randn((n_pf * chunk, hq, d), generator=gen, device=dev).to(torch.bfloat16)
    od = torch.empty((n_dec, hq, d), dtype=torch.bfloat16, device=dev)
    op = torch.empty((n_pf * chunk, hq, d), dtype=torch.bfloat16, device=dev)
    ws = paged.DecodeWorkspace.for_shape(pool, n_dec, hq)
    pws = torch.zeros(max(256, paged.L.lib().mtn_paged_prefill_workspace_bytes(n_pf, n_pf * chunk, hq, hkv, d)),
                      dtype=torch.uint8, device=dev)
    lens = [torch.from_numpy((dl + 1 + j).astype(np.int32)).to(dev) for j in range(args.warmup + steps)]
    stream = torch.cuda.current_stream()

    def dec(j):
        return lambda: paged.paged_decode(pool, 0, qd, d_indptr, d_indices, lens[j], k_new=kn, v_new=vn, out=od,
                                          workspace=ws)

    def pre():
        paged.paged_prefill(pool, 0, qp, qo, p_indptr, p_indices, p_lens, chunk, out=op, workspace=pws)

    # The same kernel on the longest of the four chunks alone (one sequence, 32 units on 148 SMs:
    # the launch the split of long units is for).
    r1 = int(np.argmax(pp))
    s_indptr = torch.tensor([0, pf_pages[r1]], dtype=torch.int32, device=dev)
    s_indices = torch.from_numpy(pf_tables[r1].copy()).to(dev)
    s_qo = torch.tensor([0, chunk], dtype=torch.int32, device=dev)
    s_lens = torch.tensor([int(pp[r1]) + chunk], dtype=torch.int32, device=dev)
    s_q = qp[r1 * chunk:(r1 + 1) * chunk].contiguous()
    s_out = torch.empty_like(s_q)
    sws = torch.zeros(max(256, paged.L.lib().mtn_paged_prefill_workspace_bytes(1, chunk, hq, hkv, d)),
                      dtype=torch.uint8, device=dev)

    def pre1():
        paged.paged_prefill(pool, 0, s_q, s_qo, s_indptr, s_indices, s_lens, chunk, out=s_out, workspace=sws)

    for j in range(args.warmup):
        dec(j)()
        pre()
        pre1()
    t_dec = _graph_steps([dec(args.warmup + j) for j in range(steps)], stream)
    t_pre = _graph_steps([pre] * steps, stream)
    t_pre1 = _graph_steps([pre1] * steps, stream)
    peaks = load_peaks()
    kv = float(np.sum(dl + 1)) * 2 * hkv * d * 2
    flops = sum(4.0 * hq * d * chunk * (int(P) + (chunk + 1) / 2) for P in pp)
    flops1 = 4.0 * hq * d * chunk * (int(pp[r1]) + (chunk + 1) / 2)
    code, detail = paged.device_error(local)
    if code:
        raise SystemExit(f"device error {code} (detail {detail})")
    return {"metric": "config 4 mixed step: decode KV GB/s and chunked-prefill TFLOP/s", "value":
            (n_dec + n_pf * chunk) * steps / (t_dec + t_pre), "unit": "tokens/s", "n_gpus": 1, "steps": steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * (t_dec + t_pre) / steps, "higher_is_better": True,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "BASELINE config 4 attention layer: 96 decode seqs ctx U[512,8192] seed 7 + "
                                   "4 prefill chunks of 512 with prior ctx U{0,512..7680} seed 8, Hq 8 / Hkv 1 / "
                                   "D 256, page 16, 1 layer",
                       "l2": "decode reads ~430 MB of K/V per step (above L2)"},
            "decode": {"us_per_step": 1e6 * t_dec / steps, "kv_gbs": kv / (t_dec / steps) / 1e9,
                       "frac": kv / (t_dec / steps) / 1e9 / peaks["hbm_gbs"], "peak_gbs": peaks["hbm_gbs"]},
            "prefill": {"us_per_step": 1e6 * t_pre / steps, "tflops": flops / (t_pre / steps) / 1e12,
                        "frac": flops / (t_pre / steps) / 1e12 / peaks["bf16_tflops"],
                        "peak_tflops": peaks["bf16_tflops"]},
            "prefill_single_chunk": {"prior": int(pp[r1]), "us_per_step": 1e6 * t_pre1 / steps,
                                     "tflops": flops1 / (t_pre1 / steps) / 1e12,
                                     "frac": flops1 / (t_pre1 / steps) / 1e12 / peaks["bf16_tflops"]},
            "gpu_launches": 3 * steps}


def run_cfg5(args, local) -> dict:
    """BASELINE config 5's decode attention on one replica: with 1024 requests (prompts U[1024, 16384],
    seed 11) and the 16 long-context requests of 32768 tokens sharded round-robin over 8 replicas, a
    replica decodes 128 + 2 of them concurrently.  Qwen2.5-7B attention shapes (28 q / 4 kv heads,
    head_dim 128), page 16, block tables a random permutation of the pool, one layer.  One step =
    fused append of one token per sequence + split-KV decode over all 130 sequences; K/V read per
    step (~2.4 GB) is far above L2."""
    import torch

    from mitten_b200 import paged

    dev = torch.device("cuda", local)
    hq, hkv, d, ps = 28, 4, 128, 16
    lens0 = np.concatenate([np.random.default_rng(11).integers(1024, 16385, size=1024)[::8], [32768, 32768]])
    n = len(lens0)
    steps = args.steps
    pages = [(int(L) + args.warmup + steps + 1 + ps - 1) // ps for L in lens0]
    num_pages = sum(pages) + 16
    perm = np.random.default_rng(12).permutation(num_pages).astype(np.int32)
    pool = paged.PagedKVPool(1, num_pages, ps, hkv, d, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(13)
    pool.storage.normal_(generator=gen)
    indptr = torch.from_numpy(np.concatenate([[0], np.cumsum(pages)]).astype(np.int32)).to(dev)
    indices = torch.from_numpy(perm[:sum(pages)].copy()).to(dev)
    q = torch.randn((n, hq, d), generator=gen, device=dev).to(torch.bfloat16)
    kn = torch.randn((n, hkv, d), generator=gen, device=dev).to(torch.bfloat16)
    vn = torch.randn((n, hkv, d), generator=gen, device=dev).to(torch.bfloat16)
    out = torch.empty((n, hq, d), dtype=torch.bfloat16, device=dev)
    ws = paged.DecodeWorkspace.for_shape(pool, n, hq)
    lens = [torch.from_numpy((lens0 + 1 + j).astype(np.int32)).to(dev) for j in range(args.warmup + steps)]
    stream = torch.cuda.current_stream()

    def step(j):
        return lambda: paged.paged_decode(pool, 0, q, indptr, indices, lens[j], k_new=kn, v_new=vn, out=out,
                                          workspace=ws)

    for j in range(args.warmup):
        step(j)()
    t = _graph_steps([step(args.warmup + j) for j in range(steps)], stream)
    kv = float(np.mean([np.sum(lens0 + 1 + args.warmup + j) for j in range(steps)])) * 2 * hkv * d * 2
    peak = load_peaks()["hbm_gbs"]
    code, detail = paged.device_error(local)
    if code:
        raise SystemExit(f"device error {code} (detail {detail})")
    gbs = kv / (t / steps) / 1e9
    pre = run_cfg5_prefill(args, dev, stream)
    return {"metric": "config 5 replica decode attention: tokens/s and KV-read GB/s", "value": n * steps / t,
            "unit": "tokens/s", "n_gpus": 1, "steps": steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * t / steps, "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "BASELINE config 5, one replica's share at 8 GPUs: 128 seqs ctx U[1024,16384] "
                                   "seed 11 + 2 seqs at 32768, Hq 28 / Hkv 4 / D 128, page 16, 1 layer, "
                                   "append fused",
                       "l2": "K/V read per step ~2.4 GB, far above L2"},
            "kv_gbs": gbs, "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                                        "frac": gbs / peak, "traffic": None},
            "prefill": pre, "gpu_launches": steps + pre["launches"]}


def run_cfg5_prefill(args, dev, stream) -> dict:
    """Chunked prefill at config 5's shapes: 16 requests each with a 512-token chunk after a prior
    context drawn from its prompt range (U{0, 512, ..., 15872}, seed 14), Qwen2.5-7B attention shapes
    (28 q / 4 kv heads, head_dim 128), page 16, one layer.  1792 (query tile, head, sequence) units
    fill the grid several times over, so the kernel's per-SM rate shows rather than one unit's length."""
    import torch

    from mitten_b200 import paged

    hq, hkv, d, ps, n_pf, chunk = 28, 4, 128, 16, 16, 512
    pp = np.random.default_rng(14).integers(0, 32, size=n_pf) * 512
    pf_pages = [(int(P) + chunk + ps - 1) // ps for P in pp]
    num_pages = sum(pf_pages) + 16
    perm = np.random.default_rng(15).permutation(num_pages).astype(np.int32)
    pool = paged.PagedKVPool(1, num_pages, ps, hkv, d, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(16)
    pool.storage.normal_(generator=gen)
    p_indptr = torch.from_numpy(np.concatenate([[0], np.cumsum(pf_pages)]).astype(np.int32)).to(dev)
    p_indices = torch.from_numpy(perm[:sum(pf_pages)].copy()).to(dev)
    qo = torch.from_numpy(np.arange(0, (n_pf + 1) * chunk, chunk).astype(np.int32)).to(dev)
    p_lens = torch.from_numpy((pp + chunk).astype(np.int32)).to(dev)
    qp = torch.randn((n_pf * chunk, hq, d), generator=gen, device=dev).to(torch.bfloat16)
    op = torch.empty((n_pf * chunk, hq, d), dtype=torch.bfloat16, device=dev)

    def pre():  # two query tiles per CTA (the default at these shapes)
        paged.paged_prefill(pool, 0, qp, qo, p_indptr, p_indices, p_lens, chunk, out=op)

    def pre1():  # the one-tile kernel on the same inputs, for comparison
        paged.paged_prefill(pool, 0, qp, qo, p_indptr, p_indices, p_lens, chunk, out=op, one_tile=True)

    for _ in range(args.warmup):
        pre()
        pre1()
    steps = max(3, min(args.steps, 10))
    t = _graph_steps([pre] * steps, stream)
    t1 = _graph_steps([pre1] * steps, stream)
    flops = sum(4.0 * hq * d * chunk * (int(P) + (chunk + 1) / 2) for P in pp)
    peak = load_peaks()["bf16_tflops"]
    tf = flops / (t / steps) / 1e12
    return {"workload": "16 chunks of 512 after prior U{0,512..15872} seed 14, Hq 28 / Hkv 4 / D 128, page 16",
            "kernel": "paged_prefill_pair_kernel<128> (two query tiles per CTA)",
            "us_per_step": 1e6 * t / steps, "tflops": tf, "frac": tf / peak, "peak_tflops": peak,
            "launches": steps, "one_tile_us_per_step": 1e6 * t1 / steps}


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def traffic_from_profile():
    """DRAM bytes per decode launch from the committed ncu summary, if present."""
    p = ROOT / "profiles" / "decode_traffic.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["dram_bytes_per_launch"])
        except (KeyError, ValueError):
            return None
    return None


QWEN7B = dict(hidden=3584, layers=28, hq=28, hkv=4, head_dim=128, inter=18944, vocab=152064, theta=1e6)


def run_box_engine(args, rank, world, local, pg) -> dict:
    """Whole-box decode through the engine (trimmed): every rank is an independent
    replica with its own scheduler, KV pool and Qwen2.5-7B-shaped model (random bf16 weights, the
    reference's gated-q / qk-norm attention), serving its round-robin share of config 5's requests
    (request r goes to rank r % world).  Trimmed so a run fits in seconds: 64 requests per rank,
    prompts U[1024, 16384] (seed 9) capped at 4096 tokens, 48 greedy tokens each.  The decode phase
    (every request prefilled, then every decode step through the engine: schedule, forward replayed
    from a CUDA graph, device sampling, transition) is timed with CUDA events on each rank; value =
    decode tokens of all ranks / the slowest rank's decode time."""
    import torch

    from mitten_b200 import host, model as M

    dev = torch.device("cuda", local)
    per_rank, cap, out_tokens, timed_steps = 64, 4096, 48, 24
    rng = np.random.default_rng(9)
    lens = np.minimum(rng.integers(1024, 16385, size=per_rank * world), cap)
    toks = np.random.default_rng(10)
    mine = [r for r in range(per_rank * world) if r % world == rank]
    prompts = {r: toks.integers(0, QWEN7B["vocab"], int(lens[r])).astype(np.uint32) for r in range(per_rank * world)}
    shape = M.DecoderShape(**QWEN7B)
    w = model_weights(shape, dev, seed=0)
    page_bytes = 2 * shape.layers * 16 * shape.hkv * shape.head_dim * 2
    num_pages = int(sum((int(lens[r]) + out_tokens + 15) // 16 for r in mine) * 1.1) + 64
    model = M.QwenPagedModel(shape, w, num_pages, 16, device=dev, split_bf16=False, dtype=torch.bfloat16)
    del w
    torch.cuda.empty_cache()
    sched = host.Scheduler(num_pages, 16, max_prefill_tokens_per_iter=32768, max_decode_batch_size=per_rank,
                           eos_token_ids=(shape.vocab,))
    for r in mine:
        sched.add_request(r, prompts[r], temperature=0.0, max_new_tokens=out_tokens)
    eng = M.Engine(model, sched, cuda_graphs=True)
    t0 = time.perf_counter()
    while any(sched.request_info(r)["state"] != 2 for r in mine):  # until every request is decoding
        eng.step()
    torch.cuda.synchronize(dev)
    prefill_s = time.perf_counter() - t0
    eng.step()  # first decode-only batch: eager run + capture of the batch's CUDA graph
    torch.cuda.synchronize(dev)
    done0 = sum(len(sched.request_output(r)) for r in mine)
    # Every request has at most 1 + (prefill iterations) tokens here and asks
    # for 48, so all 64 stay in the batch for the timed steps: one graph size.
    assert all(len(sched.request_output(r)) + timed_steps < out_tokens for r in mine)
    barrier(pg)
    stream = torch.cuda.current_stream(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(timed_steps):
        eng.step()
    b.record(stream)
    b.synchronize()
    steps = timed_steps
    t = a.elapsed_time(b) * 1e-3
    tokens = sum(len(sched.request_output(r)) for r in mine) - done0
    assert tokens == len(mine) * timed_steps
    value, t_max = job_throughput(pg, float(tokens), t)
    code, detail = M.paged.device_error(local)
    if code:
        raise SystemExit(f"device error {code} (detail {detail}) in the engine run")
    res = {"metric": "decode tokens/s (whole box, engine, replicas)", "value": value, "unit": "tokens/s",
           "n_gpus": world, "decode_steps": steps, "decode_ms_per_step_max": 1e3 * t_max / max(steps, 1),
           "tokens_per_rank": tokens, "prefill_s_rank0": prefill_s, "kv_pool_gb": num_pages * page_bytes / 1e9,
           "config": {"workload": "BASELINE config 5 (trimmed): Qwen2.5-7B shape, random bf16 weights, requests "
                                  "round-robin over replicas", "requests_per_rank": per_rank,
                      "prompt_tokens": "U[1024, 16384] (seed 9) capped at 4096", "output_tokens": out_tokens,
                      "timed": f"{timed_steps} decode-only engine steps at a constant batch of {per_rank} per rank",
                      "trimmed_from": "1024 requests, prompts up to 16384, 256 output tokens, 16 x 32k long-context"}}
    del model, eng, sched
    torch.cuda.empty_cache()
    return res


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--ref-seconds", type=float, default=60.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-engine", action="store_true", help="skip the whole-box config-5 engine leg")
    ap.add_argument("--workload", choices=["cfg1", "cfg2", "cfg3", "cfg4", "cfg5", "cfg3e", "cfg4e"], default="cfg2",
                    help="cfg2 (default) is the headline; cfg3 / cfg4 / cfg5 time those configs' attention "
                         "layers; cfg1, cfg3e and cfg4e run configs 1, 3 and 4 through the engine")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(run_reference(args, rank, world)), flush=True)
        return 0
    rank, world, local, pg = dist_setup(args.gpus)
    if args.workload != "cfg2":
        res = {"cfg1": run_cfg1, "cfg3": run_cfg3, "cfg4": run_cfg4, "cfg5": run_cfg5, "cfg3e": run_cfg3_engine,
               "cfg4e": run_cfg4_engine}[args.workload](args, local)
        if rank == 0:
            print(json.dumps(res), flush=True)
        if pg is not None:
            pg.destroy_process_group()
        return 0
    try:
        res = run_ours(args, rank, world, local, pg)
        if not args.no_engine:
            import torch

            torch.cuda.empty_cache()
            res["box_engine"] = run_box_engine(args, rank, world, local, pg)
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        if pg is not None:
            pg.barrier()
            pg.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
