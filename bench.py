"""DiffSpec draft-context hot path benchmark.

One bench step is one retrieval period of the draft loop: the retrieval hook
(committed-query pick, chunk scores over the target's paged K history,
head-sharded exchange when N > 1, top-k selection) followed by
``retrieval_interval`` = 4 draft cycles, each one launch that builds the
history plan on the device and runs the fused gather + local-RoPE rebuild of
the working cache from it, and K = 4 draft attention steps.  That is 16 draft
steps (23 kernel launches) per bench step.

Workload (config 2, per 16-request group): 16 requests at 40960 tokens,
chunk 64, token budget 2048 (history budget 1984), rolling recent window 256
(27 ranked chunks + the newest; the plan's tail is the last 256 history
tokens), 32 query / 4 kv heads,
head_dim 128, bf16, RoPE theta 1e6, 8 planted high-score chunks per request,
paged target K with 16-token pages in a shuffled block table.  Data are
synthetic (seeded Gaussian); every buffer is larger than L2 except the
working cache, whose reuse inside a period is the real access pattern.

Multi-GPU (torchrun, N ranks): kv heads are sharded over hg = min(N, 4)
ranks and request groups over N / hg, so each GPU always holds 16 requests x
4 kv heads worth of (request, kv head) pairs (weak scaling).  Ranks of one
request group all-gather their per-kv-head chunk mass over NCCL before the
selection, which is bit-identical at any N.

``--impl reference`` times the reference's own PyTorch CPU path (the
package installed in baseline/_ref: chunk_attention_scores,
select_context_chunks, the _rebuild_working_cache and forward_attention CPU
loops) on the host cores over a bounded sample of the same workload; the
oracle port stands in only when that package does not import.
"""

from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
# the CPU baseline runs one numpy worker per core; keep BLAS single-threaded
os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
os.environ.setdefault("OMP_NUM_THREADS", "1")
# stdout carries exactly one JSON line: keep NCCL's version banner off it
if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
    os.environ["NCCL_DEBUG"] = "WARN"

# ---------------------------------------------------------------- config 2
B_GROUP = 16          # requests per request group
CTX = 40960           # committed context per request
CHUNK = 64
TOKEN_BUDGET = 2048
DEPTH = 4             # K speculative draft steps per cycle
INTERVAL = 4          # retrieval interval (cycles)
HQ, HK, D = 32, 4, 128
THETA = 1.0e6
PLANTED = 8
PAGE = 16             # paged target K block size
HISTORY_BUDGET = (TOKEN_BUDGET - DEPTH - 1) // CHUNK * CHUNK  # 1984
RECENT_WINDOW = 256   # rolling recent window of config 2 (window mode: 4 chunks)
REJECTED = 3          # rejected draft suffix at the retrieval pass
ACCEPT_PER_CYCLE = 2  # committed tokens added per cycle inside a period
METRIC = "DiffSpec draft steps/sec (B=16, 40k ctx, budget 2048) and % of HBM peak"
UNIT = "draft steps/s"
STEPS_PER_PERIOD = INTERVAL * DEPTH


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the
# period's kernels come from the committed ncu summary below: one row per
# launch kind with the kernel's source files, a digest of those sources at
# capture time, the cold-cache figure and the in-period figure.  A row whose
# sources have changed since the capture is reported as stale (null).
TRAFFIC_PROFILE = ROOT / "profiles" / "dram_traffic_config2.md"


def source_digest(files: str) -> str:
    """sha256 (16 hex) of the '+'-joined package source files, in order."""
    import hashlib

    h = hashlib.sha256()
    for name in files.split("+"):
        h.update((ROOT / "vllm-ascend-hust-diffspec_b200" / name.strip()).read_bytes())
    return h.hexdigest()[:16]


def profiled_traffic() -> dict:
    """{kind: dict(traffic, traffic_in_situ, source)} from TRAFFIC_PROFILE's
    table rows `| kind | kernel | sources | digest | cold bytes | in-period
    bytes |`; values are None when the digest no longer matches."""
    out = {}
    try:
        lines = TRAFFIC_PROFILE.read_text().splitlines()
    except OSError:
        return out
    for line in lines:
        cells = [c.strip().strip("`") for c in line.strip().strip("|").split("|")]
        if len(cells) != 6 or not cells[4].replace(",", "").isdigit():
            continue
        kind, _, files, digest, cold, warm = cells
        try:
            fresh = source_digest(files) == digest
        except OSError:
            fresh = False
        out[kind] = dict(traffic=int(cold.replace(",", "")) if fresh else None,
                         traffic_in_situ=int(warm.replace(",", "")) if fresh else None,
                         source=f"{TRAFFIC_PROFILE.relative_to(ROOT)}" +
                         ("" if fresh else f" (stale: {files} changed since the capture)"))
    return out


def _peaks() -> tuple[float, str]:
    try:
        data = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(data["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def algorithmic_bytes(retrieval_lens, history_lens_per_cycle, hk_local, group_requests):
    """Bytes the path must move per period (bf16 = 2 bytes)."""
    e = 2
    row = hk_local * D * e
    retrieval = sum(retrieval_lens) * row
    rebuild = 0
    attention = 0
    for hls in history_lens_per_cycle:
        rebuild += sum(4 * h * row for h in hls)          # read K,V + write K,V
        for j in range(DEPTH):
            attention += sum(2 * (h + j + 1) * row for h in hls)
    del group_requests
    return dict(retrieval=retrieval, rebuild=rebuild, attention=attention,
                total=retrieval + rebuild + attention)


class Workload:
    """Device buffers for one rank: `rows` requests x `hk` local kv heads."""

    def __init__(self, torch, dsb, device, rows, hk_local, hq_local, seed, ctx=None):
        CTX = ctx or globals()["CTX"]  # noqa: N806 - the context length of this workload
        self.ctx = CTX
        self.torch, self.dsb, self.device = torch, dsb, device
        self.rows, self.hk, self.hq = rows, hk_local, hq_local
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        bf = torch.bfloat16
        pages = CTX // PAGE
        nblocks = rows * pages
        self.key_cache = torch.empty((nblocks, PAGE, hk_local, D), dtype=bf, device=device)
        self.key_cache.normal_(generator=g)
        perm = torch.randperm(nblocks, generator=g, device=device)
        self.block_table = perm.view(rows, pages).to(torch.int32).contiguous()
        # verify pass: 5 query tokens per request (root + K drafts)
        self.query = torch.randn((5 * rows, hq_local, D), generator=g, device=device).to(bf)
        self.query_ends = (torch.arange(1, rows + 1, device=device, dtype=torch.int32) * 5)
        self.target_seq = torch.full((rows,), CTX, dtype=torch.int32, device=device)
        self.counts = torch.full((rows,), 5 - REJECTED, dtype=torch.int64, device=device)
        self.active = torch.arange(rows, dtype=torch.int32, device=device)
        self._plant(g)
        # draft side
        self.raw_key = torch.empty((rows, CTX + 64, hk_local, D), dtype=bf, device=device)
        self.raw_key.normal_(generator=g)
        self.raw_value = torch.empty_like(self.raw_key)
        self.raw_value.normal_(generator=g)
        self.working_key = torch.zeros((rows, hk_local, TOKEN_BUDGET, D), dtype=bf, device=device)
        self.working_value = torch.zeros_like(self.working_key)
        inv = 1.0 / (THETA ** (torch.arange(0, D, 2, dtype=torch.float64, device=device) / D))
        freqs = torch.arange(TOKEN_BUDGET, dtype=torch.float64, device=device)[:, None] * inv[None]
        self.cos_sin = torch.cat((freqs.cos(), freqs.sin()), -1).to(bf).contiguous()
        self.dq = torch.randn((rows, hq_local, D), generator=g, device=device).to(bf)
        self.dk = torch.randn((rows, hk_local, D), generator=g, device=device).to(bf)
        self.dv = torch.randn((rows, hk_local, D), generator=g, device=device).to(bf)
        self.out = torch.empty((rows, hq_local, D), dtype=bf, device=device)
        # retrieval scratch / state
        self.q_index = torch.empty(rows, dtype=torch.int32, device=device)
        self.r_len = torch.empty(rows, dtype=torch.int32, device=device)
        self.r_slot = torch.empty(rows, dtype=torch.int32, device=device)
        self.status = torch.zeros(2, dtype=torch.int32, device=device)
        self.max_chunks = (CTX + CHUNK - 1) // CHUNK
        self.parts = torch.zeros((rows, hk_local, self.max_chunks), dtype=torch.float32, device=device)
        self.sel_chunks = torch.zeros((rows, HISTORY_BUDGET // CHUNK), dtype=torch.int32, device=device)
        self.sel_count = torch.full((rows,), -1, dtype=torch.int32, device=device)
        self.plan = torch.zeros((rows, 5 + TOKEN_BUDGET // CHUNK), dtype=torch.int64, device=device)
        self.hist = torch.zeros(rows, dtype=torch.int32, device=device)
        self.committed = [
            torch.full((rows,), CTX - REJECTED + ACCEPT_PER_CYCLE * c, dtype=torch.int32, device=device)
            for c in range(INTERVAL)
        ]
        self.ws = dsb.attention.AttentionWorkspace(device)
        self.lse = self._true_lse()

    def _plant(self, g):
        """Make PLANTED chunks per request score high: keys = group-mean query + noise."""
        torch = self.torch
        group = self.hq // self.hk
        for r in range(self.rows):
            q_root = self.query[5 * r + (5 - REJECTED) - 1].float()       # committed query
            target = q_root.view(self.hk, group, D).mean(1)                 # [hk, D]
            chunks = torch.randperm(self.ctx // CHUNK - 1, generator=g, device=self.device)[:PLANTED]
            tok = (chunks[:, None] * CHUNK + torch.arange(CHUNK, device=self.device)).reshape(-1)
            pages = self.block_table[r].long()[tok // PAGE]
            noise = 0.1 * torch.randn((tok.numel(), self.hk, D), generator=g, device=self.device)
            self.key_cache[pages, tok % PAGE] = (target[None] + noise).to(torch.bfloat16)

    def _true_lse(self):
        """The target's softmax LSE of the committed queries (set-up only)."""
        torch = self.torch
        lse_rows = torch.empty((self.rows, self.hq), dtype=torch.float32, device=self.device)
        qi = torch.arange(self.rows, device=self.device) * 5 + (5 - REJECTED) - 1
        seq = torch.full((self.rows,), self.ctx - REJECTED, dtype=torch.int32, device=self.device)
        cmax, csum = self.dsb.kernels.paged_chunk_stats(
            self.query[qi].contiguous(), self.key_cache, self.block_table, seq,
            chunk_size=CHUNK, max_seq_len=self.ctx, scale=D ** -0.5)
        self.dsb.kernels.stats_to_head_scores(cmax, csum, seq, self.hk, chunk_size=CHUNK,
                                              lse_out=lse_rows)
        lse = torch.zeros((5 * self.rows, self.hq), dtype=torch.float32, device=self.device)
        lse[qi] = lse_rows
        return lse


def period_launches(w: "Workload", exchange=None, total_hq=None, gathered=None,
                    window=RECENT_WINDOW):
    """The kernels of one retrieval period as (kind, callable) in stream order.

    `exchange` (multi-GPU) all-gathers the local [rows, hk, N] mass into the
    request group's fixed rank-major [ranks, rows, hk, N] buffer `gathered`,
    which the selection then reads in place; it is inserted between scoring
    and selection.  `window` is the rolling recent window in tokens.
    """
    dsb, lib = w.dsb, w.dsb._lib
    total_hq = total_hq or w.hq
    flag = lib.error_flag(w.device)
    stream = lambda: lib.stream_ptr(w.device)  # noqa: E731

    def prepare():
        lib.call("dsb_prepare_retrieval_rows", w.query_ends.data_ptr(), w.target_seq.data_ptr(),
                 w.counts.data_ptr(), 1, w.active.data_ptr(), w.rows, w.q_index.data_ptr(),
                 w.r_len.data_ptr(), w.r_slot.data_ptr(), w.status.data_ptr(), stream())

    def scores():
        dsb.kernels.paged_chunk_head_scores(
            w.query, w.key_cache, w.lse, w.block_table, w.r_len, chunk_size=CHUNK,
            max_seq_len=w.ctx, scale=D ** -0.5, query_index=w.q_index, out=w.parts)

    def select(parts_fn=lambda: w.parts):
        dsb.selection.select_rows(parts_fn(), w.r_len, chunk_size=CHUNK, token_budget=HISTORY_BUDGET,
                                  normalize_heads=total_hq, row_slots=w.r_slot,
                                  sel_chunks=w.sel_chunks, sel_count=w.sel_count,
                                  recent_window=window)

    seq = [("prepare", prepare), ("scores", scores)]
    if exchange is not None:
        seq.append(("exchange", lambda: exchange(w.parts)))
        seq.append(("select", lambda: select(lambda: gathered)))
    else:
        seq.append(("select", select))
    for c in range(INTERVAL):
        def rebuild(c=c):  # plan + rebuild in one launch
            dsb.compact_kv.rebuild_working_cache(
                w.raw_key, w.raw_value, w.working_key, w.working_value, w.active, w.committed[c],
                w.sel_chunks, w.sel_count, w.cos_sin, chunk_size=CHUNK,
                history_budget=HISTORY_BUDGET, rotary_dim=D, is_neox_style=True, plan=w.plan,
                history_lens=w.hist, recent_window=window)

        seq.append(("rebuild", rebuild))
        for j in range(DEPTH):
            def attn(j=j):
                dsb.attention.draft_decode_attention(
                    w.dq, w.dk, w.dv, w.working_key, w.working_value, w.active, w.hist,
                    D ** -0.5, w.out, position_offset=j, workspace=w.ws)
            seq.append(("attention", attn))
    del flag
    return seq


class Graph:
    """A CUDA graph of a list of launches (captured once, replayed)."""

    def __init__(self, torch, launches, device):
        self.torch = torch
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            for _, fn in launches:  # warm-up: allocations and one-time attributes
                fn()
        torch.cuda.current_stream(device).wait_stream(s)
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            for _, fn in launches:
                fn()
        torch.cuda.synchronize(device)

    def replay(self):
        self.graph.replay()


def time_region(torch, device, fn, iters, flush=None):
    """Device time of `iters` calls of fn with CUDA events (ms per call)."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    start.record()
    for _ in range(iters):
        if flush is not None:
            flush()
        fn()
    end.record()
    torch.cuda.synchronize(device)
    return start.elapsed_time(end) / iters


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return self
        # nvidia-smi takes a moment to start: wait (bounded) for its first sample
        t_end = time.perf_counter() + 5.0
        while time.perf_counter() < t_end and self.proc.poll() is None:
            if Path(self.path).stat().st_size > 0:
                break
            time.sleep(0.05)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.path is None:
            return None
        rows = []
        for line in Path(self.path).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), f[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        sm = sorted(x[0] for x in rows)
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(x[1] for x in rows),
                "reasons": reasons, "samples": len(rows)}


def per_kernel_times(torch, device, launches, iters=5):
    """Average device time per launch kind inside a replay of the period.

    The period is captured once more with an external timing event between
    consecutive launches; deltas are attributed to the launch they bracket.
    Returns {kind: (launches, total_ms_per_period)} or None if the driver
    cannot time events recorded inside a graph.
    """
    try:
        events = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(len(launches) + 1)]
    except TypeError:
        return None
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    graph = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(graph, stream=s):
            events[0].record()
            for i, (_, fn) in enumerate(launches):
                fn()
                events[i + 1].record()
    except Exception:
        return None
    totals: dict[str, list[float]] = {}
    for _ in range(iters):
        graph.replay()
        torch.cuda.synchronize(device)
        for i, (kind, _) in enumerate(launches):
            try:
                dt = events[i].elapsed_time(events[i + 1])
            except Exception:
                return None
            totals.setdefault(kind, []).append(dt)
    return {k: (len(v) // iters, sum(v) / iters) for k, v in totals.items()}


def chain_time(torch, device, launches, kind, iters=20):
    """Average device time per launch of `kind` when its launches of one
    period run back to back in a CUDA graph (consecutive launches overlap
    their launch latency through programmatic dependent launch, as the
    consecutive draft steps of a cycle do).  Returns (launches, ms) or None."""
    fns = [fn for k, fn in launches if k == kind]
    if not fns:
        return None
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for fn in fns:
            fn()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        graph.replay()
    end.record()
    torch.cuda.synchronize(device)
    return len(fns), start.elapsed_time(end) / (iters * len(fns))


def _reference_runtime():
    """The reference's own runtime module from baseline/_ref (the package
    installed there from the reference's source, no dependencies), or
    (None, why) when it is not installed or does not import here."""
    ref_dir = ROOT / "baseline" / "_ref"
    if not (ref_dir / "diffspec" / "runtime.py").exists():
        return None, "baseline/_ref is not installed"
    if str(ref_dir) not in sys.path:
        sys.path.insert(0, str(ref_dir))
    try:
        from diffspec import runtime as ref_rt
        from vllm.model_executor.layers.rotary_embedding import RotaryEmbedding
    except Exception as error:  # noqa: BLE001 - reported in the JSON line
        return None, f"reference import failed: {type(error).__name__}: {error}"
    return (ref_rt, RotaryEmbedding), None


def cpu_reference_sample(budget_s: float, threads: int):
    """Time the reference's own PyTorch CPU path on config-2 requests.

    One sample unit = one request's retrieval period, run through the
    reference's functions exactly as its CPU path runs them:
    chunk_attention_scores over 40,957 tokens x 32 heads (LSE computed,
    diffspec/runtime.py:281-345), set_chunk_scores / select_context_chunks
    (:1554-1567, :348-414), then 4 cycles of _rebuild_working_cache (the CPU
    loop, :1683-1711, RoPE by vLLM's RotaryEmbedding.forward_static) and 4
    forward_attention steps (the CPU loop, :2040-2077).  fp32 (the
    reference's CPU attention loop needs fp32 caches); one request at a time
    (its loops are per request) with torch using `threads` host threads.
    The reference has no rolling-window mode, so its tail is one chunk.
    Returns (seconds per request-period, requests done) or None."""
    import torch

    mod, _ = _reference_runtime()
    if mod is None:
        return None
    torch.set_num_threads(threads)
    one_request = _REFERENCE_SETUP.get("one_request")
    if one_request is None:  # built once: the inputs take seconds to draw
        one_request = _REFERENCE_SETUP["one_request"] = _reference_request(mod)
    done = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s and done < 4 * B_GROUP:
        one_request()
        done += 1
    return (time.perf_counter() - t0) / max(done, 1), done


_REFERENCE_SETUP: dict = {}


def _reference_request(mod):
    """One config-2 request's period through the reference's functions
    (see cpu_reference_sample), as a closure over its inputs."""
    import torch

    ref_rt, rope = mod
    g = torch.Generator().manual_seed(7)
    L = CTX - REJECTED

    def bf16_exact(*shape):
        return torch.randn(shape, generator=g).bfloat16().float()

    keys = bf16_exact(L, HK, D)
    q = bf16_exact(HQ, D)
    inv = 1.0 / (THETA ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    fr = torch.arange(TOKEN_BUDGET, dtype=torch.float64)[:, None] * inv[None]
    table = torch.cat((fr.cos(), fr.sin()), -1).float()

    class Rotary:  # the attributes DiffSpecDraftCache reads; vLLM's own CPU rotation
        rotary_dim, head_size, is_neox_style, cos_sin_cache = D, D, True, table

        def forward_native(self, positions, query, key=None):
            return rope.forward_static(positions, query, key, D, D, table, True)

    cache = ref_rt.DiffSpecDraftCache(
        ref_rt.DiffSpecSettings(CHUNK, TOKEN_BUDGET, INTERVAL, 4, DEPTH, 0.7, False),
        max_num_reqs=1, max_model_len=CTX + 64, num_kv_heads=HK, head_dim=D, target_num_layers=2,
        dtype=torch.float32, device=torch.device("cpu"), rotary_embedding=Rotary())
    cache.raw_key[0] = bf16_exact(CTX + 64, HK, D)
    cache.raw_value[0] = bf16_exact(CTX + 64, HK, D)
    dq, dk = bf16_exact(1, HQ, D), bf16_exact(1, HK, D)
    out = torch.empty_like(dq)

    def one_request():
        scores = ref_rt.chunk_attention_scores(q, keys, CHUNK, None, D ** -0.5)
        cache.begin_cycle(["r"])
        cache.set_chunk_scores(0, scores, L)
        for c in range(INTERVAL):
            local = cache._rebuild_working_cache([0], [CTX - REJECTED + ACCEPT_PER_CYCLE * c])
            for j in range(DEPTH):
                cache._pending_request_indices = [0]
                cache._pending_local_positions = [local[0] + j]
                cache.forward_attention(dq, dk, dk, D ** -0.5, out)
        cache.end_cycle()

    return one_request


def cpu_baseline_sample(budget_s: float, threads: int):
    """The reference's own CPU path when baseline/_ref imports (kind
    "reference"), else the oracle port (kind "port", with the reason)."""
    got = cpu_reference_sample(budget_s, threads)
    if got is not None:
        t_req, done = got
        return t_req, done, threads, "reference", (
            f"{done} request-periods of config 2 through the reference's own PyTorch CPU path "
            f"(baseline/_ref: chunk_attention_scores, select_context_chunks, "
            f"_rebuild_working_cache, forward_attention; fp32, window = one chunk), "
            f"{threads} torch threads")
    why = _reference_runtime()[1]
    t_req, done, used = cpu_oracle_sample(budget_s, threads)
    return t_req, done, used, "port", (
        f"{done} request-periods of config 2 (oracle port, numpy fp32 scores, one worker per "
        f"core; the reference's own code is unavailable: {why})")


def cpu_oracle_sample(budget_s: float, threads: int, acc="float32"):
    """Time the oracle port of the reference's CPU path on config-2 requests.

    One sample unit = one request's retrieval period: chunk scores over 40957
    tokens x 32 heads, selection, 4 x (plan + rebuild of 1984 tokens + 4
    attention steps).  Requests are processed by `threads` workers until
    `budget_s` of wall time is spent.  Returns (seconds per request-period,
    requests done, threads).
    """
    import concurrent.futures

    import numpy as np

    from oracle import diffspec_oracle as O

    rng = np.random.Generator(np.random.PCG64(7))
    L = CTX - REJECTED
    keys = O.round_to(rng.standard_normal((L, HK, D), dtype=np.float32), "bf16")
    raw_k = O.round_to(rng.standard_normal((CTX + 64, HK, D), dtype=np.float32), "bf16")
    raw_v = O.round_to(rng.standard_normal((CTX + 64, HK, D), dtype=np.float32), "bf16")
    q = O.round_to(rng.standard_normal((HQ, D), dtype=np.float32), "bf16")
    inv = 1.0 / (THETA ** (np.arange(0, D, 2) / D))
    fr = np.arange(TOKEN_BUDGET)[:, None] * inv[None]
    cos_sin = O.round_to(np.concatenate([np.cos(fr), np.sin(fr)], -1).astype(np.float32), "bf16")
    dq = O.round_to(rng.standard_normal((1, HQ, D), dtype=np.float32), "bf16")
    dk = O.round_to(rng.standard_normal((1, HK, D), dtype=np.float32), "bf16")
    dtype = getattr(np, acc)
    table = np.arange(L // PAGE + 1, dtype=np.int64)[None]
    kc = np.zeros(((L // PAGE + 1) * PAGE, HK, D), np.float32)
    kc[:L] = keys
    kc = kc.reshape(-1, PAGE, HK, D)

    def one_request(_):
        scores = O.paged_chunk_attention_scores(q[None], kc, None, table, np.array([L]), CHUNK, L,
                                                D ** -0.5, acc=dtype)[0]
        n = (L + CHUNK - 1) // CHUNK
        chunks = O.select_context_chunks(scores[:n], L, CHUNK, HISTORY_BUDGET,
                                         recent_window=RECENT_WINDOW)[0].tolist()
        wk = np.zeros((1, HK, TOKEN_BUDGET, D), np.float32)
        wv = np.zeros_like(wk)
        for c in range(INTERVAL):
            committed = CTX - REJECTED + ACCEPT_PER_CYCLE * c
            plan = np.zeros((1, 5 + TOKEN_BUDGET // CHUNK), np.int64)
            row = O.history_plan(0, chunks, committed - 1, CHUNK, HISTORY_BUDGET,
                                 recent_window=RECENT_WINDOW)
            plan[0, : len(row)] = row
            O.rebuild_compact_kv_from_plan(raw_k[None], raw_v[None], wk, wv, plan, cos_sin, CHUNK,
                                           HISTORY_BUDGET, D, True, "bf16")
            for j in range(DEPTH):
                O.draft_decode_attention(dq, dk, dk, wk, wv, [0], [row[1] + j], D ** -0.5)
        return 1

    done = 0
    t0 = time.perf_counter()
    with concurrent.futures.ThreadPoolExecutor(threads) as pool:
        while time.perf_counter() - t0 < budget_s and done < 4 * B_GROUP:
            done += sum(pool.map(one_request, range(threads)))
    elapsed = time.perf_counter() - t0
    return elapsed / done, done, threads


def run_ours(args):
    import torch
    import torch.distributed as dist

    dsb = importlib.import_module("vllm-ascend-hust-diffspec_b200")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    hg = math.gcd(world, HK)  # kv-head shards per request group
    rg = world // hg
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
        groups = [dist.new_group(list(range(r * hg, (r + 1) * hg))) for r in range(rg)]
        group = groups[rank // hg]
    hk_local = HK // hg
    hq_local = HQ // hg
    rows = B_GROUP * hg
    w = Workload(torch, dsb, device, rows, hk_local, hq_local, seed=1234 + rank // hg)
    exchange = site = None
    if hg > 1:
        # rank-major [hg, rows, hk_local, N]: the all-gather writes it and the
        # selection reads it in place
        gathered = torch.empty((hg, rows, hk_local, w.max_chunks), dtype=torch.float32,
                               device=device)
        # auto: the peer gather for exchange groups of two ranks, where it has
        # been run and measured; NCCL for larger groups
        use_peer = args.retrieval_exchange == "peer" or (args.retrieval_exchange == "auto"
                                                         and hg == 2)
        if use_peer:
            # every rank must take the same exchange: if any rank cannot map
            # its peers' buffers, all of them use the NCCL all-gather
            try:
                site = dsb.parallel.PeerExchange.create(1, rows * hk_local * w.max_chunks,
                                                        device, group=group)
            except Exception as error:  # noqa: BLE001 - reported, then agreed on below
                print(f"rank {rank}: peer exchange unavailable ({error})", file=sys.stderr)
                site = None
            ok = torch.tensor([1 if site is not None else 0], device=device)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            if int(ok.item()) == 0 and site is not None:
                site.close()
                site = None
            dist.barrier()  # every rank's buffer is mapped before the first call
        if site is not None:
            exchange = lambda parts: dsb.parallel.peer_all_gather(parts, site, gathered)  # noqa: E731
        else:
            exchange = lambda parts: dsb.parallel.gather_head_scores(parts, group, out=gathered)  # noqa: E731
    launches = period_launches(w, exchange, total_hq=HQ,
                               gathered=gathered if exchange is not None else None)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    graphs = []
    res_mode = "one CUDA graph per bench step"
    if exchange is None:
        graphs.append(Graph(torch, launches, device))
        step = graphs[0].replay
    else:
        # The NCCL all-gather is captured inside the period's graph (after one
        # eager call has set up the communicator); if this build of PyTorch /
        # NCCL refuses, it runs eagerly between two captured halves.
        cut = [k for k, _ in launches].index("exchange")
        ex = launches[cut][1]
        ex()
        torch.cuda.synchronize(device)
        dist.barrier()
        try:
            graphs.append(Graph(torch, launches, device))
            step = graphs[0].replay
            res_mode = ("one CUDA graph per bench step, peer all-gather (NVLink, two launches) "
                        "captured in it" if site is not None else
                        "one CUDA graph per bench step, NCCL exchange captured in it")
        except Exception:  # noqa: BLE001 - fall back to the split graph
            graphs = [Graph(torch, launches[:cut], device), Graph(torch, launches[cut + 1:], device)]

            def step():
                graphs[0].replay()
                ex()
                graphs[1].replay()
            res_mode = "two CUDA graphs per bench step, NCCL exchange eager between them"

    step_ms = []
    for _ in range(args.warmup):
        w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0.record()
        step()
        w1.record()
        torch.cuda.synchronize(device)
        step_ms.append(w0.elapsed_time(w1))
    assert dsb._lib.read_and_clear_error_flag(device) == 0, "kernel index check tripped"
    # Steps that keep the GPU loaded for ~0.6 s before and ~0.3 s after the
    # timed region, so the clock sampler sees clocks under this load.  The
    # counts come from the slowest rank's fastest warm-up step, so every rank
    # issues the same collectives.
    est_ms = torch.tensor([max(min(step_ms, default=1.0), 1e-3)], device=device)
    if world > 1:
        dist.all_reduce(est_ms, op=dist.ReduceOp.MAX)
        dist.barrier()
    n_pre = max(1, math.ceil(600.0 / float(est_ms.item())))
    n_post = max(1, math.ceil(300.0 / float(est_ms.item())))
    with ClockSampler(local) as clocks:
        for _ in range(n_pre):
            step()
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        torch.cuda.synchronize(device)
        for _ in range(n_post):
            step()
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
    ms = start.elapsed_time(end) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = STEPS_PER_PERIOD * (B_GROUP * world // B_GROUP) / (ms / 1e3)
    # graphs holding NCCL work must be released before the process group
    del step
    graphs.clear()
    torch.cuda.synchronize(device)
    result = dict(ms=ms, value=value, clocks=clocks.summary(), w=w, launches=launches, rows=rows,
                  graph_mode=res_mode,
                  hk_local=hk_local, world=world, rank=rank, device=device, torch=torch, dsb=dsb,
                  dist=dist if world > 1 else None, flush=flush, group=group, hg=hg, site=site)
    return result


def run_e2e(res, args):
    """Same workload through the runtime's public API with host buffers: a
    DiffSpecDraftCache and its DraftPeriodGraph (one retrieval period
    captured as a CUDA graph).  Every period copies the verify pass's query,
    LSE, accepted counts and lengths of each cycle and every draft step's
    q/k/v from pinned host memory to the device, and every step's attention
    output back to pinned host memory; the copies are nodes of the graph on
    side streams, so they overlap the kernels."""
    torch, dsb, w, device = res["torch"], res["dsb"], res["w"], res["device"]

    rows = res["rows"]
    hg = res["hg"]
    settings = dsb.runtime.DiffSpecSettings(CHUNK, TOKEN_BUDGET, INTERVAL, 4, DEPTH, 0.7, False)
    cache = dsb.runtime.DiffSpecDraftCache(
        settings, max_num_reqs=rows, max_model_len=1, num_kv_heads=w.hk, head_dim=D,
        target_num_layers=2, dtype=torch.bfloat16, device=device, cos_sin_cache=w.cos_sin,
        rotary_dim=D, is_neox_style=True, target_tensor_parallel_size=hg,
        process_group=res["group"], recent_window=RECENT_WINDOW)
    cache.raw_key, cache.raw_value = w.raw_key, w.raw_value  # share the canonical cache
    cache.max_model_len = w.raw_key.shape[1]
    ids = [f"req{i}" for i in range(rows)]
    cache.set_active_requests(ids)
    g = dsb.runtime.DraftPeriodGraph(cache, ids, key_cache=w.key_cache,
                                     block_tables=w.block_table, query_rows_per_request=5,
                                     num_query_heads=w.hq, max_seq_len=CTX, scale=D ** -0.5)
    for c in range(INTERVAL):
        v = g.inputs["verify"][c]
        v["query"].copy_(w.query)
        v["lse"].copy_(w.lse)
        v["counts"].copy_(w.counts)
        v["query_ends"].copy_(w.query_ends)
        v["seq_lens"].copy_(w.target_seq)
        v["committed"].copy_(w.committed[c])
        for j in range(DEPTH):
            st = g.inputs["step"][c][j]
            st["q"].copy_(w.dq)
            st["k"].copy_(w.dk)
            st["v"].copy_(w.dv)

    for _ in range(max(args.warmup, 1)):
        g.replay()
    torch.cuda.synchronize(device)
    dist = res["dist"]
    if dist is not None:
        dist.barrier()
    steps = max(1, args.steps)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        g.replay()
    end.record()
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(end) / steps
    if dist is not None:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    assert dsb._lib.read_and_clear_error_flag(device) == 0
    h2d, d2h = g.h2d_bytes, g.d2h_bytes
    del g  # holds NCCL work when N > 1: released before the process group
    torch.cuda.synchronize(device)
    return dict(value=STEPS_PER_PERIOD * res["world"] / (ms / 1e3), unit=UNIT,
                ms_per_step=round(ms, 4), h2d_bytes_per_step=int(h2d),
                d2h_bytes_per_step=int(d2h),
                api="DiffSpecDraftCache + DraftPeriodGraph.replay (pinned host inputs and outputs)")


def period_bytes(res):
    """Algorithmic bytes of one period and per launch kind, from the history
    lengths the device plan kernel produces for each cycle of the period."""
    w = res["w"]
    hls = []
    for c in range(INTERVAL):
        w.dsb.selection.build_history_plan(
            w.active, w.committed[c], w.sel_chunks, w.sel_count, chunk_size=CHUNK,
            history_budget=HISTORY_BUDGET, working_budget=TOKEN_BUDGET, plan=w.plan,
            history_lens=w.hist, recent_window=RECENT_WINDOW)
        hls.append(w.hist[: res["rows"]].cpu().tolist())
    b = algorithmic_bytes([CTX - REJECTED] * res["rows"], hls, w.hk, res["rows"])
    per_launch = dict(scores=b["retrieval"], rebuild=b["rebuild"] / INTERVAL,
                      attention=b["attention"] / (INTERVAL * DEPTH))
    return b, per_launch


def emit_ours(args):
    res = run_ours(args)
    torch, device = res["torch"], res["device"]
    world, rank = res["world"], res["rank"]
    peak, peak_kind = _peaks()
    b, per_launch = period_bytes(res)
    kernel_t = per_kernel_times(torch, device, [x for x in res["launches"] if x[0] != "exchange"])
    roofline = None
    if kernel_t:
        dominant = max((k for k in kernel_t if k in per_launch), key=lambda k: kernel_t[k][1])
        chained = {k: chain_time(torch, device, res["launches"], k)
                   for k in per_launch if k in kernel_t}
        n, avg_ms = chained[dominant]
        achieved = per_launch[dominant] / (avg_ms / 1e3) / 1e9
        traffic = profiled_traffic().get(dominant, {})
        roofline = dict(bound="hbm", kernel=dominant, achieved=round(achieved, 1), peak=peak,
                        peak_kind=peak_kind, unit="GB/s", frac=round(achieved / peak, 4),
                        traffic=traffic.get("traffic"),
                        traffic_in_situ=traffic.get("traffic_in_situ"),
                        traffic_source=traffic.get("source", "no ncu capture committed"),
                        algorithmic_bytes_per_launch=int(per_launch[dominant]),
                        avg_launch_us=round(avg_ms * 1e3, 3),
                        timing="avg_launch_us: the kind's launches of one period back to back "
                               "in a CUDA graph; per_kind_us: each launch bracketed by events "
                               "inside the full period graph (adds the event gaps)",
                        chained_us={k: round(v[1] * 1e3, 3) for k, v in chained.items() if v},
                        per_kind_us={k: round(v[1] / v[0] * 1e3, 3) for k, v in kernel_t.items()},
                        per_kind_launches={k: v[0] for k, v in kernel_t.items()})
    e2e = None if args.no_e2e else run_e2e(res, args)
    cpu = None
    if world == 1 and not args.no_cpu:
        t_req, done, threads, kind, sample = cpu_baseline_sample(args.cpu_seconds, os.cpu_count() or 1)
        cpu = dict(value=round(1.0 / t_req, 4), unit=UNIT, cores=threads, kind=kind, sample=sample)
    period_ms = res["ms"]
    line = dict(
        metric=METRIC, value=round(res["value"], 2), unit=UNIT, n_gpus=world, steps=args.steps,
        warmup=args.warmup, ms_per_step=round(period_ms, 4), higher_is_better=True,
        scaling="weak", vs_baseline=None, dtype="bf16", data="synthetic",
        config=dict(workload="config 2: retrieval period (1 retrieval + 4 cycles x (plan + "
                    "rebuild, 4 draft attention steps)) over 16 requests x 40960 ctx per "
                    "request group", requests=B_GROUP * world, context=CTX, chunk=CHUNK,
                    token_budget=TOKEN_BUDGET, history_budget=HISTORY_BUDGET,
                    recent_window=RECENT_WINDOW, q_heads=HQ,
                    kv_heads=HK, head_dim=D, draft_steps_per_bench_step=STEPS_PER_PERIOD,
                    retrieval_interval=INTERVAL, page_size=PAGE,
                    parallelism=f"kv-head shards {res['hg']} x request groups {world // res['hg']}",
                    l2="inputs larger than L2 (target K 671 MB, raw KV 1.3 GB per group)",
                    bytes_per_step=int(b["total"]),
                    hbm_frac_whole_step=round(b["total"] / (period_ms / 1e3) / 1e9 / peak, 4),
                    graph=res["graph_mode"]),
        roofline=roofline, cpu_baseline=cpu, e2e=e2e,
        gpu_launches=(sum(1 for k, _ in res["launches"] if k != "exchange") +
                      (2 if res["site"] is not None else 0)) * args.steps,
        clocks=res["clocks"])
    if rank == 0:
        print(json.dumps(line), flush=True)
    if res["dist"] is not None:
        torch = res["torch"]
        torch.cuda.synchronize(res["device"])
        res["dist"].barrier()  # no rank still writes into another's exchange buffer
        if res["site"] is not None:
            res["site"].close()
            res["dist"].barrier()
        res["dist"].destroy_process_group()


def emit_reference(args):
    """The reference arm: the reference's own CPU path (baseline/_ref) timed
    on the host cores over bounded samples of the config-2 workload, on rank
    0 only; the oracle port stands in when the reference does not import."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    per_step = max(2.0, min(10.0, 150.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        cpu_baseline_sample(per_step / 4, threads)
    times, done_total, kind, sample = [], 0, "port", ""
    for _ in range(args.steps):
        t_req, done, used, kind, sample = cpu_baseline_sample(per_step, threads)
        times.append(t_req)
        done_total += done
    t_req = sum(times) / len(times)
    value = 1.0 / t_req
    sample = (f"{done_total} request-periods over {args.steps} steps (about {per_step:.0f} s of "
              f"CPU work each); " + sample.split(" ", 1)[1])
    line = dict(
        metric=METRIC, value=round(value, 4), unit=UNIT, n_gpus=world, steps=args.steps,
        warmup=args.warmup, ms_per_step=round(t_req * B_GROUP * 1e3, 3), higher_is_better=True,
        scaling="weak", vs_baseline=None, dtype="f32", data="synthetic", impl="reference",
        config=dict(workload="config 2: retrieval period (1 retrieval + 4 cycles x (plan + "
                    "rebuild, 4 draft attention steps)) over 16 requests x 40960 ctx per "
                    "request group", requests=B_GROUP, context=CTX, chunk=CHUNK,
                    token_budget=TOKEN_BUDGET, history_budget=HISTORY_BUDGET, q_heads=HQ,
                    kv_heads=HK, head_dim=D, retrieval_interval=INTERVAL,
                    implementation=("the reference's own PyTorch CPU path (baseline/_ref)"
                                    if kind == "reference" else "oracle port of the reference's "
                                    "CPU path")),
        cpu_baseline=dict(value=round(value, 4), unit=UNIT, cores=threads, kind=kind, sample=sample),
        e2e=dict(value=round(value, 4), unit=UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- config 4
C4_REQUESTS, C4_CTX, C4_HQ, C4_HK, C4_BUDGET = 32, 131072, 64, 8, 4096
C4_HISTORY_BUDGET = (C4_BUDGET - DEPTH - 1) // CHUNK * CHUNK  # 4032


class RetrievalWorkload:
    """Config 4 on one rank: the target's paged K for 32 requests x 131072
    tokens and this rank's contiguous kv heads [head_lo, head_hi) of 8 (with
    their 8 query heads each).  Every global kv head draws its keys, queries
    and planted-chunk noise from its own generator, and the block table and
    planted chunks from a shared one, so the data of a kv head is the same at
    any GPU count and the selection can be compared across counts."""

    def __init__(self, torch, dsb, device, head_lo, head_hi, seed=4242):
        self.torch, self.dsb, self.device = torch, dsb, device
        rows, ctx, group = C4_REQUESTS, C4_CTX, C4_HQ // C4_HK
        self.rows, self.hk, self.hq = rows, head_hi - head_lo, (head_hi - head_lo) * group
        bf = torch.bfloat16
        pages = ctx // PAGE
        nblocks = rows * pages
        shared = torch.Generator(device=device).manual_seed(seed)
        self.block_table = torch.randperm(nblocks, generator=shared, device=device).view(
            rows, pages).to(torch.int32).contiguous()
        planted = [torch.randperm(ctx // CHUNK - 1, generator=shared, device=device)[:PLANTED]
                   for _ in range(rows)]
        self.planted = [sorted(p.tolist()) for p in planted]
        self.key_cache = torch.empty((nblocks, PAGE, self.hk, D), dtype=bf, device=device)
        self.query = torch.empty((5 * rows, self.hq, D), dtype=bf, device=device)
        committed_q = 5 - REJECTED - 1
        for i, h in enumerate(range(head_lo, head_hi)):
            gh = torch.Generator(device=device).manual_seed(seed + 1 + h)
            keys = torch.randn((nblocks, PAGE, D), generator=gh, device=device).to(bf)
            q = torch.randn((5 * rows, group, D), generator=gh, device=device).to(bf)
            for r in range(rows):
                target = q[5 * r + committed_q].float().mean(0)
                tok = (planted[r][:, None] * CHUNK + torch.arange(CHUNK, device=device)).reshape(-1)
                noise = 0.1 * torch.randn((tok.numel(), D), generator=gh, device=device)
                keys[self.block_table[r].long()[tok // PAGE], tok % PAGE] = (target + noise).to(bf)
            self.key_cache[:, :, i] = keys
            self.query[:, i * group:(i + 1) * group] = q
            del keys
        self.query_ends = torch.arange(1, rows + 1, device=device, dtype=torch.int32) * 5
        self.target_seq = torch.full((rows,), ctx, dtype=torch.int32, device=device)
        self.counts = torch.full((rows,), 5 - REJECTED, dtype=torch.int64, device=device)
        self.active = torch.arange(rows, dtype=torch.int32, device=device)
        self.q_index = torch.empty(rows, dtype=torch.int32, device=device)
        self.r_len = torch.empty(rows, dtype=torch.int32, device=device)
        self.r_slot = torch.empty(rows, dtype=torch.int32, device=device)
        self.status = torch.zeros(2, dtype=torch.int32, device=device)
        self.max_chunks = (ctx + CHUNK - 1) // CHUNK
        self.parts = torch.zeros((rows, self.hk, self.max_chunks), dtype=torch.float32,
                                 device=device)
        self.sel_chunks = torch.zeros((rows, C4_HISTORY_BUDGET // CHUNK), dtype=torch.int32,
                                      device=device)
        self.sel_count = torch.full((rows,), -1, dtype=torch.int32, device=device)
        # the target's softmax LSE of the committed queries, per local query head
        qi = torch.arange(rows, device=device) * 5 + committed_q
        seq = torch.full((rows,), ctx - REJECTED, dtype=torch.int32, device=device)
        cmax, csum = dsb.kernels.paged_chunk_stats(
            self.query[qi].contiguous(), self.key_cache, self.block_table, seq, chunk_size=CHUNK,
            max_seq_len=ctx, scale=D ** -0.5)
        lse_rows = torch.empty((rows, self.hq), dtype=torch.float32, device=device)
        dsb.kernels.stats_to_head_scores(cmax, csum, seq, self.hk, chunk_size=CHUNK,
                                         lse_out=lse_rows)
        self.lse = torch.zeros((5 * rows, self.hq), dtype=torch.float32, device=device)
        self.lse[qi] = lse_rows


def retrieval_launches(w, exchange=None, gathered=None):
    """Config 4's retrieval as (kind, callable): committed-query pick, chunk
    scores of the local kv heads, the all-gather of their mass (N > 1), and
    the selection over all 64 query heads (replicated on every rank)."""
    dsb, lib = w.dsb, w.dsb._lib

    def prepare():
        lib.call("dsb_prepare_retrieval_rows", w.query_ends.data_ptr(), w.target_seq.data_ptr(),
                 w.counts.data_ptr(), 1, w.active.data_ptr(), w.rows, w.q_index.data_ptr(),
                 w.r_len.data_ptr(), w.r_slot.data_ptr(), w.status.data_ptr(),
                 lib.stream_ptr(w.device))

    def scores():
        dsb.kernels.paged_chunk_head_scores(
            w.query, w.key_cache, w.lse, w.block_table, w.r_len, chunk_size=CHUNK,
            max_seq_len=C4_CTX, scale=D ** -0.5, query_index=w.q_index, out=w.parts)

    def select():
        dsb.selection.select_rows(gathered if exchange is not None else w.parts, w.r_len,
                                  chunk_size=CHUNK, token_budget=C4_HISTORY_BUDGET,
                                  normalize_heads=C4_HQ, row_slots=w.r_slot,
                                  sel_chunks=w.sel_chunks, sel_count=w.sel_count)

    seq = [("prepare", prepare), ("scores", scores)]
    if exchange is not None:
        seq.append(("exchange", lambda: exchange(w.parts)))
    seq.append(("select", select))
    return seq


def run_config4(args):
    """head-sharded retrieval at fixed total work (strong
    scaling).  32 requests x 131072 tokens, 64 query / 8 kv heads, chunk 64,
    budget 4096 (history budget 4032, 62 ranked chunks + the newest); the 8
    kv heads are split evenly over the N ranks, each rank scores its heads
    over every request, the per-kv-head mass is all-gathered over NCCL and
    every rank runs the same selection.  One step = one retrieval of all 32
    requests; the line carries a digest of the selected chunk ids, which
    must be the same at every N."""
    import hashlib

    import torch
    import torch.distributed as dist

    dsb = importlib.import_module("vllm-ascend-hust-diffspec_b200")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus or C4_HK % world:
        raise SystemExit(f"config 4 runs on 1, 2, 4 or 8 ranks (--gpus {args.gpus}, "
                         f"WORLD_SIZE={world})")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    per = C4_HK // world
    w = RetrievalWorkload(torch, dsb, device, rank * per, (rank + 1) * per)
    exchange = gathered = None
    if world > 1:
        gathered = torch.empty((world, w.rows, per, w.max_chunks), dtype=torch.float32,
                               device=device)
        exchange = lambda parts: dsb.parallel.gather_head_scores(parts, None, out=gathered)  # noqa: E731
    launches = retrieval_launches(w, exchange, gathered)
    if exchange is not None:  # one eager collective sets up the communicator
        exchange(w.parts)
        torch.cuda.synchronize(device)
        dist.barrier()
    graph = Graph(torch, launches, device)
    for _ in range(max(3, args.warmup)):
        graph.replay()
    torch.cuda.synchronize(device)
    assert dsb._lib.read_and_clear_error_flag(device) == 0, "kernel index check tripped"
    with ClockSampler(local) as clocks:
        for _ in range(200):  # ~0.3 s of load before the timed region
            graph.replay()
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            graph.replay()
        end.record()
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
    ms = start.elapsed_time(end) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    kinds = [k for k, _ in launches if k != "exchange"]
    kernel_t = per_kernel_times(torch, device, [x for x in launches if x[0] != "exchange"]) or {}
    del graph
    torch.cuda.synchronize(device)
    sel = torch.cat((w.sel_chunks.flatten(), w.sel_count)).cpu().numpy().tobytes()
    planted_found = all(set(p) <= set(w.sel_chunks[r, : int(w.sel_count[r])].tolist())
                        for r, p in enumerate(w.planted))
    peak, peak_kind = _peaks()
    k_bytes = C4_REQUESTS * (C4_CTX - REJECTED) * per * D * 2
    line = dict(
        mode="config4", metric="config 4 head-sharded retrievals/s (32 x 131072 ctx, 64/8 heads, "
        "budget 4096)", value=round(1e3 / ms, 2), unit="retrievals/s", n_gpus=world,
        steps=args.steps, warmup=args.warmup, ms_per_step=round(ms, 4), higher_is_better=True,
        scaling="strong", dtype="bf16", data="synthetic (seeded Gaussian K/Q per kv head, 8 "
        "planted chunks per request)",
        config=dict(requests=C4_REQUESTS, context=C4_CTX, q_heads=C4_HQ, kv_heads=C4_HK,
                    kv_heads_per_gpu=per, head_dim=D, chunk=CHUNK, token_budget=C4_BUDGET,
                    history_budget=C4_HISTORY_BUDGET, page_size=PAGE,
                    l2=f"inputs larger than L2 (K {k_bytes / 1e9:.2f} GB per GPU)",
                    exchange="NCCL all-gather of per-kv-head mass, read in place by the selection"
                    if world > 1 else "none"),
        k_bytes_per_gpu=k_bytes,
        hbm_frac_per_gpu=round(k_bytes / (ms / 1e3) / 1e9 / peak, 4), peak=peak,
        peak_kind=peak_kind,
        per_kind_us={k: round(v[1] / v[0] * 1e3, 3) for k, v in kernel_t.items()},
        selection_digest=hashlib.sha256(sel).hexdigest()[:16], planted_found=planted_found,
        gpu_launches=len(kinds) * args.steps, clocks=clocks.summary())
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_only(args):
    """One kernel kind of the config-2 period, launched eagerly `--steps`
    times after `--warmup` launches (the command the ncu captures run)."""
    import torch

    dsb = importlib.import_module("vllm-ascend-hust-diffspec_b200")
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    w = Workload(torch, dsb, device, B_GROUP, HK, HQ, seed=1234)
    launches = period_launches(w)
    for kind, fn in launches:  # one full period so selection/plan state is real
        fn()
    if args.only == "gather":
        # the paged gather entry point over the period's selection: the raw
        # caches viewed as 16-token pages (identity block table), the selected
        # chunks expanded to token ids and padded with -1 to the token budget
        pages = w.raw_key.shape[1] // PAGE
        paged = [t.view(w.rows * pages, PAGE, w.hk, D) for t in (w.raw_key, w.raw_value)]
        table = torch.arange(w.rows * pages, dtype=torch.int32, device=device).view(w.rows, pages)
        tok = torch.full((w.rows, TOKEN_BUDGET), -1, dtype=torch.int64, device=device)
        n_sel = w.sel_chunks.shape[1]
        tok[:, : n_sel * CHUNK] = (w.sel_chunks.long()[:, :, None] * CHUNK
                                   + torch.arange(CHUNK, device=device)).view(w.rows, -1)
        launches = [("gather", lambda: dsb.kernels.gather_raw_kv_with_local_rope(
            paged[0], paged[1], table, tok, w.cos_sin, rope_dim=D, is_neox_style=True))]
    picked = [fn for kind, fn in launches if kind == args.only]
    if not picked:
        raise SystemExit(f"no launch of kind {args.only}")
    for i in range(args.warmup + args.steps):
        picked[i % len(picked)]()
    torch.cuda.synchronize(device)
    flag = dsb._lib.read_and_clear_error_flag(device)
    print(json.dumps({"only": args.only, "launches": args.warmup + args.steps, "error_flag": flag}))
    if flag:
        raise SystemExit(1)


def run_draft_step(args):
    """a random-init Eagle3-style draft layer (hidden 2048,
    qkv input 4096, 32 / 4 heads of 128, SwiGLU 6144, RMSNorm, bf16) drafting
    for 16 requests at 65536 context: one period = retrieval (committed-query
    pick, chunk scores over the paged target K, selection) + 4 cycles x (plan +
    rebuild, 4 draft steps through the layer: RMSNorm, query GEMM, K/V
    projection with the raw-cache write, RoPE, draft attention, output GEMM,
    RMSNorm, SwiGLU MLP).  The LM head is excluded (its vocabulary is
    unspecified).  Captured as one CUDA graph; prints draft tokens/s.

    Under torchrun (N ranks), --draft-parallel tp (default): the layer is
    tensor-parallel (Eagle3DraftLayerTP: qkv / gate_up column-split, o_proj /
    down_proj row-split with two fp32 all-reduces per step, kv heads
    replicated when N > 4; --tp-exchange peer (default) fuses each all-reduce
    into its row-split linear over NVLink peer memory, nccl calls
    torch.distributed.all_reduce) and the DiffSpec cache is sharded by kv head
    (retrieval mass all-gathered before the selection); every rank drafts
    the same 16 requests, so the total work is fixed (strong scaling).
    --draft-parallel dp: every rank drafts its own 16 requests with the
    whole layer and the whole cache (weak scaling, no collective)."""
    import torch
    import torch.distributed as dist

    dsb = importlib.import_module("vllm-ascend-hust-diffspec_b200")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    ctx = 65536
    tp = world > 1 and args.draft_parallel == "tp"
    if tp:
        hk_local = HK // world if world <= HK else 1
        rep = 1 if world <= HK else world // HK  # ranks holding each kv head
        hq_local = HQ // world
        kv_group = rank // rep  # this rank's kv-head shard
    else:  # one GPU, or data parallel: every rank drafts its own 16 requests
        hk_local, rep, hq_local, kv_group = HK, 1, HQ, rank
    w = Workload(torch, dsb, device, B_GROUP, hk_local, hq_local, seed=555 + kv_group, ctx=ctx)
    full = dsb.draft_layer.Eagle3DraftLayer(device, seed=5)
    sites = None
    if tp and args.tp_exchange == "peer":
        hidden = full.w_o.shape[0]
        sites = tuple(dsb.parallel.PeerExchange.create(B_GROUP, hidden, device) for _ in range(2))
        dist.barrier()  # every rank's buffers are mapped before the first call
    layer = dsb.draft_layer.Eagle3DraftLayerTP(full, rank, world, peer=sites) if tp else full
    g = torch.Generator(device=device).manual_seed(17)
    bf = torch.bfloat16
    x_in = torch.randn((B_GROUP, 4096), generator=g, device=device).to(bf)
    residual = torch.randn((B_GROUP, 2048), generator=g, device=device).to(bf)
    exchange = gathered = None
    if tp:
        full_gather = torch.empty((world, B_GROUP, hk_local, w.max_chunks), dtype=torch.float32,
                                  device=device)
        gathered = full_gather[::rep]  # one replica of every kv head, read in place
        exchange = lambda parts: dsb.parallel.gather_head_scores(parts, None, out=full_gather)  # noqa: E731
    launches = period_launches(w, exchange, total_hq=HQ, gathered=gathered, window=CHUNK)
    retrieval = [(k, fn) for k, fn in launches if k in ("prepare", "scores", "exchange", "select")]
    rebuilds = [fn for k, fn in launches if k == "rebuild"]
    abs_pos = [[(w.committed[c] + j).to(torch.int64) for j in range(DEPTH)] for c in range(INTERVAL)]
    outs = [torch.empty_like(residual) for _ in range(DEPTH)]

    def step(c, j):  # step j writes at the plan's history length + j
        layer.step(x_in, residual, slots=w.active, abs_positions=abs_pos[c][j],
                   local_positions=w.hist, position_offset=j, raw_key=w.raw_key,
                   raw_value=w.raw_value, working_key=w.working_key,
                   working_value=w.working_value, cos_sin=w.cos_sin, out=outs[j])

    seq = list(retrieval)
    for c in range(INTERVAL):
        seq.append(("rebuild", rebuilds[c]))
        for j in range(DEPTH):
            seq.append(("layer", lambda c=c, j=j: step(c, j)))
    if world > 1:  # one eager pass sets up the communicators before capture
        for _, fn in seq:
            fn()
        torch.cuda.synchronize(device)
        dist.barrier()
    graph = Graph(torch, seq, device)
    for _ in range(max(3, args.warmup)):
        graph.replay()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()

    def timed(gr):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
        a.record()
        for _ in range(args.steps):
            gr.replay()
        b.record()
        torch.cuda.synchronize(device)
        ms = a.elapsed_time(b) / args.steps
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    ms = timed(graph)
    assert dsb._lib.read_and_clear_error_flag(device) == 0
    steps_only = Graph(torch, [("layer", lambda j=j: step(0, j)) for j in range(DEPTH)], device)
    for _ in range(3):
        steps_only.replay()
    step_us = timed(steps_only) * 1e3 / DEPTH
    del graph, steps_only  # graphs holding NCCL work go before the process group
    torch.cuda.synchronize(device)
    tokens = B_GROUP * INTERVAL * DEPTH * (1 if tp else world)  # whole job, per period
    if rank == 0:
        print(json.dumps(dict(
            mode="draft_step", metric="draft tokens/s (config 5, one draft layer, LM head excluded)",
            value=round(tokens / (ms / 1e3), 1), unit="draft tokens/s", n_gpus=world,
            scaling=("strong" if tp else "weak") if world > 1 else None,
            ms_per_period=round(ms, 4),
            draft_tokens_per_period=tokens, layer_step_us=round(step_us, 2),
            layer_weight_bytes_per_gpu=layer.weight_bytes(),
            parallelism=("one GPU" if world == 1 else
                         f"tensor parallel over {world} GPUs: {hq_local} query heads and "
                         f"{hk_local} kv head(s) per GPU (each kv head on {rep} GPU(s)), "
                         + ("2 fp32 all-reduces per layer step fused into the row-split "
                            "linears over NVLink peer memory" if sites else
                            "2 fp32 NCCL all-reduces per layer step") if tp else
                         f"data parallel over {world} GPUs: every GPU drafts its own 16 "
                         "requests with the whole layer (no per-step collective)"),
            requests=B_GROUP * (1 if tp else world), context=ctx, token_budget=TOKEN_BUDGET, chunk=CHUNK,
            retrieval_interval=INTERVAL, draft_depth=DEPTH, dtype="bf16",
            data="synthetic (random weights and KV)")), flush=True)
    if world > 1:
        torch.cuda.synchronize(device)
        dist.barrier()  # no rank still writes into another's exchange buffer
        for site in sites or ():
            site.close()
        dist.barrier()
        dist.destroy_process_group()


def run_peer_exchange(args):
    """Under torchrun (N >= 2 ranks): the cost of one all-reduce of a row-split
    linear at config 5's shape (16 tokens x 2048 features fp32, a 2048 x 2048
    weight share), as a CUDA graph of 100 (linear + add + RMSNorm) pairs,
    max over ranks: fused over NVLink peer memory (dsb_draft_linear_peer +
    dsb_peer_add_rms_norm), the same kernels on a one-rank site of this GPU
    (no cross-GPU traffic), the partial linear + NCCL all_reduce +
    add_rms_norm, and the partial linear + add_rms_norm with no exchange."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    dsb = importlib.import_module("vllm-ascend-hust-diffspec_b200")
    dl = dsb.draft_layer
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world < 2 or world != args.gpus:
        raise SystemExit("--peer-exchange runs under torchrun with --gpus N = WORLD_SIZE >= 2")
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    feats, k, tokens = 2048, 2048, B_GROUP
    g = torch.Generator(device=device).manual_seed(rank)
    w = dl.pack_linear_weight((torch.randn((feats, k), generator=g, device=device) / k ** 0.5).bfloat16())
    x = torch.randn((tokens, k), generator=g, device=device).bfloat16()
    res = torch.randn((tokens, feats), generator=g, device=device).bfloat16()
    norm_w = torch.ones((feats,), device=device).bfloat16()
    part = torch.empty((tokens, feats), dtype=torch.float32, device=device)
    site = dsb.parallel.PeerExchange.create(tokens, feats, device)
    local = dsb.parallel.PeerExchange.local(1, tokens, feats, device)[0]
    dist.barrier()

    def fused(s):
        dl.draft_linear_peer(x, w, s, packed=True)
        dl.peer_add_rms_norm(s, res, norm_w, 1e-6)

    def nccl():
        dl.draft_linear(x, w, "partial", out=part, packed=True)
        dist.all_reduce(part)
        dl.add_rms_norm(part, res, norm_w, 1e-6)

    def none():
        dl.draft_linear(x, w, "partial", out=part, packed=True)
        dl.add_rms_norm(part, res, norm_w, 1e-6)

    out = {}
    for name, fn in (("peer_fused", lambda: fused(site)), ("fused_one_rank_site", lambda: fused(local)),
                     ("nccl_all_reduce", nccl), ("no_exchange", none)):
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            for _ in range(max(3, args.warmup)):
                fn()
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(100):
                fn()
        graph.replay()
        torch.cuda.synchronize(device)
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            graph.replay()
        b.record()
        torch.cuda.synchronize(device)
        t = torch.tensor([a.elapsed_time(b) * 1e3 / (100 * args.steps)], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out[name] = round(float(t.item()), 2)
        del graph
        torch.cuda.synchronize(device)
        dist.barrier()
    flag = dsb._lib.read_and_clear_error_flag(device)
    if rank == 0:
        print(json.dumps(dict(mode="peer_exchange", n_gpus=world, tokens=tokens, features=feats,
                              us_per_linear_and_add_rms_norm=out, error_flag=flag)), flush=True)
    torch.cuda.synchronize(device)
    dist.barrier()  # no rank still writes into another's exchange buffer
    site.close()
    local.close()
    dist.barrier()
    dist.destroy_process_group()


def run_kv_projection(args):
    """Time the draft-layer K/V projection + raw-cache write (config 5 decode
    step: 16 tokens, Eagle3 qkv input 4096, 4 kv heads x 128) against the
    library-call path it replaces (cuBLAS matmul, then the raw-cache scatter).
    The launches cycle through 24 weight copies (201 MB, more than L2), so
    every launch streams its weight from HBM."""
    import torch

    dsb = importlib.import_module("vllm-ascend-hust-diffspec_b200")
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device).manual_seed(99)
    tokens, hidden, hk = 16, 4096, HK
    bf = torch.bfloat16
    weights = [(torch.randn((2 * hk * D, hidden), generator=g, device=device) / 64).to(bf)
               for _ in range(24)]
    h = torch.randn((tokens, hidden), generator=g, device=device).to(bf)
    rk = torch.zeros((B_GROUP, 4096, hk, D), dtype=bf, device=device)
    rv = torch.zeros_like(rk)
    slots = torch.arange(tokens, dtype=torch.int32, device=device)
    pos = torch.full((tokens,), 1000, dtype=torch.int64, device=device)
    out = torch.empty((tokens, 2 * hk * D), dtype=bf, device=device)

    def ours(i):
        dsb.kernels.kv_projection_write_raw(h, weights[i % 24], slots, pos, rk, rv, out=out)

    def reference(i):
        kv = h @ weights[i % 24].t()
        rk[slots.long(), pos] = kv[:, : hk * D].view(tokens, hk, D)
        rv[slots.long(), pos] = kv[:, hk * D:].view(tokens, hk, D)

    def time_graph(fn):
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            for i in range(24):
                fn(i)
        torch.cuda.current_stream(device).wait_stream(s)
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(24):
                fn(i)
        for _ in range(max(3, args.warmup)):
            graph.replay()
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            graph.replay()
        b.record()
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) * 1e3 / (args.steps * 24)

    ours_us = time_graph(ours)
    assert dsb._lib.read_and_clear_error_flag(device) == 0
    ref_us = time_graph(reference)
    nbytes = 2 * hk * D * hidden * 2 + tokens * hidden * 2 + 2 * tokens * 2 * hk * D * 2
    peak, peak_kind = _peaks()
    gbs = nbytes / (ours_us * 1e-6) / 1e9
    print(json.dumps(dict(mode="kv_projection", tokens=tokens, hidden=hidden, kv_heads=hk,
                          head_dim=D, dtype="bf16", bytes_per_launch=nbytes,
                          us_per_launch=round(ours_us, 3), achieved_gbs=round(gbs, 1),
                          frac_of_hbm_peak=round(gbs / peak, 4), peak_kind=peak_kind,
                          cublas_matmul_plus_scatter_us=round(ref_us, 3))))


def run_draft_linear(args):
    """Time the config-5 draft layer's four linears at a 16-token decode step
    on the tcgen05 weight-streaming kernel (`us`: tile-packed weights, as the
    draft layer streams them; `us_row_major_weight`: the same launches on
    row-major weights; `us_prefetch_l2`: tile-packed with each CTA's next four weight blocks
    requested into L2 while the previous launch finishes, which the layer
    leaves off because it pushes the draft attention's working cache out of L2)
    (qkv with the raw-cache write,
    o_proj + residual, gate_up + SwiGLU, down_proj + residual) against cuBLAS
    for the same products (torch.mm; the K/V raw write, the residual add and
    SwiGLU not included on that side).  Each shape cycles enough weight copies
    (>= 300 MB, more than L2) that every launch streams its weight from HBM."""
    import torch

    dsb = importlib.import_module("vllm-ascend-hust-diffspec_b200")
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device).manual_seed(7)
    bf = torch.bfloat16
    tokens = 16
    dl = dsb.draft_layer
    rk = torch.zeros((B_GROUP, 4096, HK, D), dtype=bf, device=device)
    rv = torch.zeros_like(rk)
    slots = torch.arange(tokens, dtype=torch.int32, device=device)
    pos = torch.full((tokens,), 1000, dtype=torch.int64, device=device)
    shapes = {"qkv": (HQ * D + 2 * HK * D, 4096), "o_proj": (2048, HQ * D),
              "gate_up": (2 * 6144, 2048), "down_proj": (2048, 6144)}
    peak, peak_kind = _peaks()
    result = {}
    for name, (rows, k) in shapes.items():
        copies = int(300e6 // (rows * k * 2)) + 1
        ws = [(torch.randn((rows, k), generator=g, device=device) / k ** 0.5).to(bf)
              for _ in range(copies)]
        x = torch.randn((tokens, k), generator=g, device=device).to(bf)
        res = torch.randn((tokens, rows), generator=g, device=device).to(bf)
        out = torch.empty((tokens, rows), dtype=bf, device=device)
        half = torch.empty((tokens, rows // 2), dtype=bf, device=device)
        q_out = torch.empty((tokens, HQ * D), dtype=bf, device=device)
        kv_out = torch.empty((tokens, 2 * HK * D), dtype=bf, device=device)

        def ours(w, name=name, x=x, res=res, out=out, half=half, q_out=q_out, kv_out=kv_out,
                 packed=False, l2=False):
            if name == "qkv":
                dsb.kernels.qkv_projection_write_raw(x, w, HQ * D, slots, pos, rk, rv, q_out=q_out,
                                                     kv_out=kv_out, prefetch_weight=True,
                                                     packed_weight=packed, prefetch_l2=l2)
            elif name == "gate_up":  # the weight's tile order does not change the time
                dl.draft_linear(x, w, "swiglu", out=half, packed=packed, prefetch_l2=l2)
            else:
                dl.draft_linear(x, w, "residual", residual=res, out=out, packed=packed,
                                prefetch_l2=l2)

        def cublas(w, x=x, out=out):
            torch.mm(x, w.t(), out=out)

        def time_graph(fn):
            s = torch.cuda.Stream(device)
            s.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(s):
                for w in ws:
                    fn(w)
            torch.cuda.current_stream(device).wait_stream(s)
            torch.cuda.synchronize(device)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for w in ws:
                    fn(w)
            for _ in range(max(3, args.warmup)):
                graph.replay()
            torch.cuda.synchronize(device)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(args.steps):
                graph.replay()
            b.record()
            torch.cuda.synchronize(device)
            return a.elapsed_time(b) * 1e3 / (args.steps * len(ws))

        us_rowmajor = time_graph(ours)
        ws = [dl.pack_linear_weight(w) for w in ws]  # the layout Eagle3DraftLayer streams
        us = time_graph(lambda w: ours(w, packed=True))
        us_l2 = time_graph(lambda w: ours(w, packed=True, l2=True))
        assert dsb._lib.read_and_clear_error_flag(device) == 0
        del ws  # cuBLAS streams its own row-major copies
        ws = [(torch.randn((rows, k), generator=g, device=device) / k ** 0.5).to(bf)
              for _ in range(copies)]
        ref = time_graph(cublas)
        wbytes = rows * k * 2
        result[name] = dict(weight_rows=rows, k=k, us=round(us, 2), weight_gbs=round(wbytes / us / 1e3, 1),
                            frac_of_hbm_peak=round(wbytes / us / 1e3 / peak, 3),
                            us_row_major_weight=round(us_rowmajor, 2),
                            us_prefetch_l2=round(us_l2, 2), cublas_mm_us=round(ref, 2))
        del ws
        torch.cuda.empty_cache()
    print(json.dumps(dict(mode="draft_linear", tokens=tokens, dtype="bf16", peak_gbs=peak,
                          peak_kind=peak_kind, shapes=result)))


def run_target_attention(args):
    """Time the target paged decode attention with the LSE export at config 2's
    shape (16 decode rows x 40960 tokens, 32 / 4 heads of 128, 16-token pages
    in a shuffled block table: 1.34 GB of K/V per launch, more than L2) and
    report its K/V streaming rate against the measured HBM copy peak."""
    import torch

    dsb = importlib.import_module("vllm-ascend-hust-diffspec_b200")
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device).manual_seed(21)
    rows, ctx, bs = B_GROUP, CTX, 16
    cols = ctx // bs
    nblocks = rows * cols
    bf = torch.bfloat16
    kc = torch.randn((nblocks, bs, HK, D), generator=g, device=device).to(bf)
    vc = torch.randn((nblocks, bs, HK, D), generator=g, device=device).to(bf)
    table = torch.randperm(nblocks, generator=g, device=device).to(torch.int32).view(rows, cols)
    q = torch.randn((rows, HQ, D), generator=g, device=device).to(bf)
    lens = torch.full((rows,), ctx, dtype=torch.int32, device=device)
    out = torch.empty_like(q)
    lse = torch.empty((rows, HQ), dtype=torch.float32, device=device)

    def launch():
        dsb.kernels.paged_decode_attention_lse(q, kc, vc, table, lens, scale=D ** -0.5,
                                               max_seq_len=ctx, out=out, lse=lse,
                                               tokens_per_split=args.tokens_per_split)

    for _ in range(max(3, args.warmup)):
        launch()
    torch.cuda.synchronize(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        launch()
    b.record()
    torch.cuda.synchronize(device)
    assert dsb._lib.read_and_clear_error_flag(device) == 0
    us = a.elapsed_time(b) * 1e3 / args.steps
    nbytes = 2 * rows * ctx * HK * D * 2 + 2 * rows * HQ * D * 2 + rows * HQ * 4
    peak, peak_kind = _peaks()
    gbs = nbytes / us / 1e3
    print(json.dumps(dict(mode="target_attention", rows=rows, context=ctx, q_heads=HQ, kv_heads=HK,
                          head_dim=D, dtype="bf16", bytes_per_launch=nbytes,
                          us_per_launch=round(us, 2), achieved_gbs=round(gbs, 1),
                          frac_of_hbm_peak=round(gbs / peak, 3), peak_kind=peak_kind,
                          tokens_per_split=args.tokens_per_split,
                          l2="K/V 1.34 GB per launch, larger than L2")))


def run_reference_triton(args):
    """A secondary comparison arm on the GPU: the reference's two Triton
    kernels (diffspec/kernels.py:11-150 chunk scores, diffspec/compact_kv.py:
    8-242 plan-driven rebuild), imported from baseline/_ref and compiled by
    Triton for this B200, against this library's kernels on the same config-2
    inputs (16 requests x 40960 tokens, 32 / 4 heads of 128, chunk 64, budget
    2048).  Both sides run back to back in CUDA graphs (eager when a Triton
    launch cannot be captured); outputs are compared.  The product has no
    Triton: this only times the reference's own device code."""
    import torch

    ref_dir = ROOT / "baseline" / "_ref"
    stubs = ROOT / "tests" / "golden" / "ref_stubs"  # vllm_ascend import stand-ins
    for path in (str(stubs), str(ref_dir)):
        if path not in sys.path:
            sys.path.insert(0, path)
    try:
        from diffspec import compact_kv as ref_compact
        from diffspec import kernels as ref_kernels
    except Exception as error:  # noqa: BLE001
        print(json.dumps(dict(mode="reference_triton",
                              unavailable=f"reference import failed: {error}")))
        return
    dsb = importlib.import_module("vllm-ascend-hust-diffspec_b200")
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    w = Workload(torch, dsb, device, B_GROUP, HK, HQ, seed=1234)
    launches = period_launches(w, window=CHUNK)
    for _, fn in launches:  # selection state and plans of a real period
        fn()
    dsb.selection.build_history_plan(
        w.active, w.committed[0], w.sel_chunks, w.sel_count, chunk_size=CHUNK,
        history_budget=HISTORY_BUDGET, working_budget=TOKEN_BUDGET, plan=w.plan, history_lens=w.hist)
    torch.cuda.synchronize(device)
    q_rows = (torch.arange(B_GROUP, device=device) * 5 + (5 - REJECTED) - 1)
    query = w.query[q_rows].contiguous()
    lse = w.lse[q_rows].contiguous()
    seq = w.r_len.clone()
    wk_t, wv_t = torch.zeros_like(w.working_key), torch.zeros_like(w.working_value)

    def triton_scores():
        return ref_kernels.paged_chunk_attention_scores(
            query, w.key_cache, lse, w.block_table, seq, chunk_size=CHUNK, max_seq_len=CTX,
            scale=D ** -0.5)

    def ours_scores():
        return dsb.kernels.paged_chunk_attention_scores(
            query, w.key_cache, lse, w.block_table, seq, chunk_size=CHUNK, max_seq_len=CTX,
            scale=D ** -0.5)

    def triton_rebuild():
        ref_compact.rebuild_compact_kv_from_plan(
            w.raw_key, w.raw_value, wk_t, wv_t, w.plan, w.cos_sin, chunk_size=CHUNK,
            max_width=HISTORY_BUDGET, rotary_dim=D, is_neox_style=True)

    def ours_rebuild():
        dsb.compact_kv.rebuild_compact_kv_from_plan(
            w.raw_key, w.raw_value, w.working_key, w.working_value, w.plan, w.cos_sin,
            chunk_size=CHUNK, max_width=HISTORY_BUDGET, rotary_dim=D, is_neox_style=True)

    def timed(fn, n=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(device)
        mode = "graph"
        try:
            s = torch.cuda.Stream(device)
            s.wait_stream(torch.cuda.current_stream(device))
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                for _ in range(n):
                    fn()
            run = graph.replay
        except Exception:  # noqa: BLE001 - eager launches instead
            torch.cuda.synchronize(device)
            mode = "eager"

            def run():
                for _ in range(n):
                    fn()
        run()
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(max(1, args.steps)):
            run()
        b.record()
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) * 1e3 / (max(1, args.steps) * n), mode

    s_ref, s_ours = triton_scores(), ours_scores()
    rel = ((s_ref - s_ours).abs() / s_ref.abs().clamp_min(1e-30)).max().item()
    triton_rebuild()
    ours_rebuild()
    torch.cuda.synchronize(device)
    hmax = int(w.hist[: B_GROUP].max())
    same_v = bool(torch.equal(wv_t[:, :, :hmax], w.working_value[:, :, :hmax]))
    dk = (wk_t[:, :, :hmax].float() - w.working_key[:, :, :hmax].float()).abs().max().item()
    t_s, m_s = timed(triton_scores, 5)
    o_s, _ = timed(ours_scores, 5)
    t_r, m_r = timed(triton_rebuild)
    o_r, _ = timed(ours_rebuild)
    assert dsb._lib.read_and_clear_error_flag(device) == 0
    score_bytes = sum(int(x) for x in seq.tolist()) * HK * D * 2
    rebuild_bytes = sum(4 * int(h) * HK * D * 2 for h in w.hist[:B_GROUP].tolist())
    print(json.dumps(dict(
        mode="reference_triton", config="config 2 (16 x 40960, 32/4 heads, chunk 64, budget 2048)",
        scores=dict(triton_us=round(t_s, 1), ours_us=round(o_s, 1), speedup=round(t_s / o_s, 2),
                    triton_gbs=round(score_bytes / t_s / 1e3, 1), ours_gbs=round(score_bytes / o_s / 1e3, 1),
                    max_rel_diff=rel, triton_timing=m_s),
        rebuild=dict(triton_us=round(t_r, 2), ours_us=round(o_r, 2), speedup=round(t_r / o_r, 2),
                     triton_gbs=round(rebuild_bytes / t_r / 1e3, 1),
                     ours_gbs=round(rebuild_bytes / o_r / 1e3, 1), values_equal=same_v,
                     key_max_abs_diff=dk, triton_timing=m_r))), flush=True)


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--cpu-seconds", type=float, default=12.0)
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    p.add_argument("--no-e2e", action="store_true", help="skip the end-to-end API leg")
    p.add_argument("--only", choices=["prepare", "scores", "select", "rebuild", "attention",
                                      "gather"],
                   help="launch one kernel kind eagerly (for profiler captures)")
    p.add_argument("--kv-projection", action="store_true",
                   help="time the K/V projection + raw-cache write (config 5 decode step)")
    p.add_argument("--draft-step", action="store_true",
                   help="config 5: draft tokens/s of a draft layer over the DiffSpec cache")
    p.add_argument("--peer-exchange", action="store_true",
                   help="under torchrun: time one fused peer all-reduce of a row-split linear "
                        "against NCCL and against no exchange")
    p.add_argument("--retrieval-exchange", choices=["auto", "peer", "nccl"], default="auto",
                   help="multi-GPU retrieval: the per-kv-head mass all-gathered over NVLink peer "
                        "memory (two launches) or by NCCL; auto: peer for exchange groups of two "
                        "ranks, NCCL for larger ones")
    p.add_argument("--tp-exchange", choices=["peer", "nccl"], default="peer",
                   help="--draft-step --draft-parallel tp: the all-reduces fused into the "
                        "row-split linears over NVLink peer memory, or NCCL all-reduces")
    p.add_argument("--draft-parallel", choices=["tp", "dp"], default="tp",
                   help="--draft-step under torchrun: tensor parallel (one 16-request batch "
                        "over all GPUs) or data parallel (16 requests per GPU)")
    p.add_argument("--draft-linear", action="store_true",
                   help="time the config-5 draft layer's four linears against cuBLAS")
    p.add_argument("--target-attention", action="store_true",
                   help="time the target paged decode attention with the LSE export")
    p.add_argument("--config4", action="store_true",
                   help="config 4: head-sharded retrieval at fixed work over --gpus N ranks")
    p.add_argument("--tokens-per-split", type=int, default=0,
                   help="--target-attention: split length (0: the library default)")
    p.add_argument("--reference-triton", action="store_true",
                   help="time the reference's Triton kernels (compiled for this GPU) against ours")
    args = p.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.kv_projection:
        run_kv_projection(args)
    elif args.peer_exchange:
        run_peer_exchange(args)
    elif args.draft_step:
        run_draft_step(args)
    elif args.draft_linear:
        run_draft_linear(args)
    elif args.target_attention:
        run_target_attention(args)
    elif args.reference_triton:
        run_reference_triton(args)
    elif args.config4:
        run_config4(args)
    elif args.only:
        run_only(args)
    elif args.impl == "reference":
        emit_reference(args)
    else:
        emit_ours(args)


if __name__ == "__main__":
    main()
