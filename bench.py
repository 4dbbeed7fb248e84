"""Benchmark of the CSA / DSV4 decode path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload csa_batched|csa_cfg1|dsv4_c0|dsv4_c4|dsv4_c128|dsv4_splitkv|dsv4_indexer]

Default workload (the metric's batched case): one
dynamic CSA decode step for a batch of 64 requests x 32 heads, head_dim 128,
chunk 64, top-k 16, bf16, per-request context uniform over multiples of 64 in
[4096, 32768].  A step = score every valid chunk of K and select the top-16
per (request, head) (csa_select kernel), then split-K attention over the 16 x
64 selected tokens (csa_decode kernel).  K/V (34 GB) are larger than L2, so no
flush is needed between steps.

Multi-GPU (torchrun, one process per GPU): strong scaling.  The one batch of 64
requests is split over the ranks greedily by context length (sum of L_b per
rank balanced, ``csahca_b200.partition``); every rank materialises and decodes
only its share, with no collective on the data path.  ``value`` = 64 requests
/ the step time, max over ranks.  ``--workload dsv4_c*`` splits the DSV4 batch
by query (Q/N per rank), ``dsv4_indexer`` splits the config-5 indexer by
query and ``csa_cfg1`` splits config 1's 8 heads.

At N=1 the line also carries ``secondary``: DSV4 decode (configs 4 and 5: C0,
C4, C128), config 1 and the config-3 mini block, each timed alone with CUDA
events and each with a CPU baseline of the same case.

``--impl reference`` times the reference's CPU implementation of the same step
(the numpy port in ``oracle/``, one process per host core over requests) on
rank 0 only and prints the same metric.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "CSA batched dynamic decode throughput (score+top-k+split-K attention), config 2"
UNIT = "tokens/s"
CONFIG = {"workload": "csa_batched_dynamic_decode (BASELINE config 2)", "batch": 64, "heads": 32,
          "head_dim": 128, "max_seq_len": 32768, "min_seq_len": 4096, "chunk_size": 64, "top_k": 16,
          "dtype": "bf16", "l2": "inputs (K/V 34 GB at N=1) larger than L2; no flush"}
# DRAM bytes (read + write) per algorithmic byte of the scorer, from one ncu
# capture of csa_select_bulk_kernel on config 2's shapes at batch 4
# (--set full, one launch): 483.53 MB read + 9.77 MB written for 483.43 MB of
# algorithmic bytes.  Traffic grows in proportion to the valid K rows, so the
# full launch's traffic is this ratio times its algorithmic bytes.
NCU_TRAFFIC = {"csa_select": (483.53 + 9.77) / 483.43}


def _peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


# ------------------------------------------------------------------------------------------- clocks
REASONS = ["clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
           "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]


class ClockSampler:
    """nvidia-smi sampling (200 ms) of SM clock and throttle reasons while running."""

    def __init__(self, index: int) -> None:
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def __enter__(self):
        q = "clocks.sm,clocks.max.sm,power.draw," + ",".join(REASONS)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=lambda: self.lines.extend(iter(self.proc.stdout.readline, "")),
                                       daemon=True)
            self._t.start()
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self._t is not None:
                self._t.join(timeout=2)

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 3 + len(REASONS):
                continue
            try:
                sm.append(float(f[0]))
                mx.append(float(f[1]))
            except ValueError:
                continue
            for name, val in zip(REASONS, f[3:]):
                if val.lower().startswith("active"):
                    reasons.add(name.split(".")[-1])
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        busy = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": float(np.median(busy)), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------------- CPU legs
# The reference's CPU path for each case is restated by the numpy port in
# ``oracle/`` (kind "port"); these legs time it on the host cores of the GPU box
# beside the GPU numbers.  They are baselines, not targets.
_CPU_SAMPLE = None


def _cpu_model() -> str:
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _host(t: torch.Tensor) -> np.ndarray:
    """Device tensor -> the oracle's storage form (bf16 as uint16 bits)."""
    t = t.detach().contiguous().cpu()
    return t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()


def _cpu_request(i: int) -> int:
    from oracle import csa

    q, k, v, L, c, top_k = _CPU_SAMPLE[i]
    sel = csa.select_topk_chunks(q, k, c, top_k, "bf16")
    csa.csa_reference(q, k, v, chunk_size=c, top_k=top_k, dtype="bf16", selected_chunks=sel)
    return 1


def make_cpu_sample(n: int, seed: int = 0):
    """``n`` config-2 requests generated on the host with the same distributions
    (only each request's valid prefix is materialised)."""
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(4096 // 64, 32768 // 64 + 1, (n,), generator=g) * 64
    out = []
    for i in range(n):
        L = int(lens[i])
        q = torch.randn(1, 32, 128, generator=g).to(torch.bfloat16)
        k = torch.randn(1, 32, L // 64, 64, 128, generator=g)
        k += torch.randn(1, 32, L // 64, 1, 1, generator=g) * 0.5
        k = k.view(1, 32, L, 128).to(torch.bfloat16)
        v = torch.randn(1, 32, L, 128, generator=g).to(torch.bfloat16)
        out.append((_host(q), _host(k), _host(v), L, 64, 16))
    return out


def time_cpu_oracle(sample, workers: int, repeats: int = 1) -> tuple[float, list[float]]:
    """Requests decoded per second by the numpy port, ``workers`` processes over
    requests (BLAS one thread per process, so the processes use the cores)."""
    global _CPU_SAMPLE
    import concurrent.futures as cf
    import multiprocessing as mp

    from threadpoolctl import threadpool_limits

    _CPU_SAMPLE = sample
    times = []
    with threadpool_limits(1), cf.ProcessPoolExecutor(workers, mp_context=mp.get_context("fork")) as ex:
        list(ex.map(_cpu_request, range(min(len(sample), workers))))  # warm the workers
        for _ in range(repeats):
            t0 = time.perf_counter()
            n = sum(ex.map(_cpu_request, range(len(sample))))
            times.append(time.perf_counter() - t0)
    return n / float(np.median(times)), times


def _median_time(fn, repeats: int = 3) -> float:
    fn()  # warm
    ts = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return float(np.median(ts))


def cpu_cfg1(q, k, v) -> dict:
    """Config 1 on the host: select_topk_chunks + csa_reference over the whole
    request (numpy port, BLAS on every core)."""
    from oracle import csa

    qn, kn, vn = _host(q), _host(k), _host(v)

    def run():
        sel = csa.select_topk_chunks(qn, kn, 64, 8, "bf16")
        csa.csa_reference(qn, kn, vn, chunk_size=64, top_k=8, dtype="bf16", selected_chunks=sel)

    t = _median_time(run)
    return {"value": round(1.0 / t, 3), "unit": "tokens/s", "ms_per_step": round(t * 1e3, 2),
            "cores": os.cpu_count(), "kind": "port", "cpu": _cpu_model(),
            "sample": "the whole config-1 step (1 request x 8 heads), median of 3"}


def cpu_mini_block(blk, hidden, k, v) -> dict:
    """Config 3 on the host: one dynamic decode step of the reference-form block."""
    from oracle import mini_block

    args = [_host(hidden), _host(k), _host(v)] + [_host(m.weight) for m in
                                                  (blk.q_proj, blk.out_proj, blk.up_proj, blk.down_proj)]
    t = _median_time(lambda: mini_block.block_forward(*args, chunk_size=64, top_k=8, dtype="bf16"))
    return {"value": round(t * 1e3, 2), "unit": "ms/token", "cores": os.cpu_count(), "kind": "port",
            "cpu": _cpu_model(), "sample": "one dynamic step of the GELU block (d1024 H8 S32768), median of 3"}


def cpu_dsv4(b, n: int = 8) -> dict:
    """Configs 4/5 on the host: the fp32 sink-softmax oracle over ``n`` queries
    of the benched batch (their pages copied to the host first, untimed), scaled
    linearly to tokens/s."""
    from oracle import dsv4

    def compact(cache, idx, ps):
        valid = idx >= 0
        pages = np.unique(idx[valid] // ps)
        sub = cache[torch.from_numpy(pages).to(cache.device)].cpu().numpy()
        new = np.full_like(idx, -1)
        new[valid] = np.searchsorted(pages, idx[valid] // ps) * ps + idx[valid] % ps
        return sub, new

    qs = torch.arange(min(n, b.q.shape[0]), device=b.q.device)
    cache, idx = compact(b.cache, b.token_indices[qs].cpu().numpy(), b.page_size)
    extra = {}
    if b.extra_cache is not None:
        xc, xi = compact(b.extra_cache, b.extra_token_indices[qs].cpu().numpy(), b.extra_page_size)
        extra = dict(extra_cache=xc, extra_token_indices=xi,
                     extra_topk_lengths=b.extra_topk_lengths[qs].cpu().numpy(), extra_page_size=b.extra_page_size)
    qn, lens, sink = _host(b.q[qs]), b.topk_lengths[qs].cpu().numpy(), b.attn_sink.cpu().numpy()
    t = _median_time(lambda: dsv4.reference_attention(qn, "bf16", cache, idx, lens, sink, page_size=b.page_size,
                                                      softmax_scale=b.softmax_scale, **extra))
    return {"value": round(len(qs) / t, 2), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "cpu": _cpu_model(), "sample": f"{len(qs)} queries of the batch (64 heads each), median of 3, "
                                          "scaled linearly to queries per second"}


# ------------------------------------------------------------------------------------------- GPU arms
def _event():
    return torch.cuda.Event(enable_timing=True)


def bench_csa(dev, rank: int, world: int, steps: int, warmup: int, secondary: bool, batch_size: int = 64) -> dict:
    from csahca_b200 import extension as ext
    from csahca_b200 import partition as P
    from csahca_b200 import workloads as W

    lens_all = W.csa_request_lengths(batch=batch_size)
    shares = P.shard_requests_by_length(lens_all, world)
    batch = W.csa_batched(dev, batch=batch_size, requests=shares[rank])
    nbytes = W.csa_algorithmic_bytes(batch)
    q, k, v, lens, c, top_k = batch.q, batch.k, batch.v, batch.seq_lens, batch.chunk, batch.top_k
    torch.cuda.synchronize(dev)

    def step():
        sel = ext.select_topk_chunks(q, k, c, top_k, lens)
        return ext.csa_decode_forward_tiled(q, k, v, sel, c)

    for _ in range(max(3, warmup)):
        step()
    ev = [(_event(), _event(), _event()) for _ in range(steps)]
    _barrier(world)
    torch.cuda.synchronize(dev)
    with ClockSampler(dev.index) as clk:
        t_start, t_end = _event(), _event()
        t_start.record()
        for e0, e1, e2 in ev:
            e0.record()
            sel = ext.select_topk_chunks(q, k, c, top_k, lens)
            e1.record()
            ext.csa_decode_forward_tiled(q, k, v, sel, c)
            e2.record()
        t_end.record()
        torch.cuda.synchronize(dev)
        _barrier(world)
        # keep the sampler alive for at least a few samples
        time.sleep(max(0.0, 0.5 - t_start.elapsed_time(t_end) / 1e3))
    own_ms = t_start.elapsed_time(t_end)
    total_ms = _max_over_ranks(own_ms, dev, world)
    sel_ms = sum(e0.elapsed_time(e1) for e0, e1, _ in ev) / steps
    dec_ms = sum(e1.elapsed_time(e2) for _, e1, e2 in ev) / steps
    _barrier(world)

    # end to end through the public API: pinned host q in, host output out
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    for _ in range(3):
        q.copy_(q_host, non_blocking=True)
        out_host.copy_(step(), non_blocking=True)
    torch.cuda.synchronize(dev)
    _barrier(world)
    e_s, e_e = _event(), _event()
    e_s.record()
    for _ in range(steps):
        q.copy_(q_host, non_blocking=True)
        out_host.copy_(step(), non_blocking=True)
    e_e.record()
    torch.cuda.synchronize(dev)
    e2e_ms = _max_over_ranks(e_s.elapsed_time(e_e), dev, world)

    hbm, peak_kind = _peaks()
    achieved = nbytes["scorer"] / (sel_ms / 1e3) / 1e9
    res = {
        "total_ms": total_ms, "own_ms": own_ms, "steps": steps, "select_ms": sel_ms, "decode_ms": dec_ms,
        "e2e_ms": e2e_ms, "clocks": clk.summary(), "requests": len(shares[rank]),
        "imbalance": round(P.imbalance(lens_all, shares), 4),
        "h2d": q_host.numel() * q_host.element_size(), "d2h": out_host.numel() * out_host.element_size(),
        "roofline": {"bound": "hbm", "kernel": "csa_select (chunk scorer + top-k)",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "peak_source": f"{peak_kind} hbm_gbs",
                     "traffic": round(NCU_TRAFFIC["csa_select"] * nbytes["scorer"]),
                     "traffic_source": "ncu dram__bytes_read+write at batch 4, scaled by valid K bytes",
                     "algorithmic_bytes": nbytes["scorer"]},
        "decode_kernel": {"achieved_gbs": round(nbytes["decode"] / (dec_ms / 1e3) / 1e9, 1),
                          "frac": round(nbytes["decode"] / (dec_ms / 1e3) / 1e9 / hbm, 4),
                          "algorithmic_bytes": nbytes["decode"]},
        "step_gbs": round(nbytes["step"] / (own_ms / steps / 1e3) / 1e9, 1),
    }
    cached_line = {}
    if secondary:
        # The same config-2 step with the chunk-sum cache: fold each
        # request's newest K row into the cache, select on the cache, decode.
        sums = ext.chunk_sums_build(k, c)
        pos = (lens - 1).clamp(min=0)

        def cached_step():
            ext.chunk_sums_append(k, sums, pos, c)
            sel_c = ext.select_topk_chunks_from_sums(q, sums, top_k, lens, chunk_size=c)
            return ext.csa_decode_forward_tiled(q, k, v, sel_c, c)

        ms_c = _time_flushed(cached_step, dev, iters=50)
        cached_line = {"csa_cfg2 step with the chunk-sum cache (config 2, same batch)": {
            "us_per_step": round(ms_c * 1e3, 1), "tokens_per_s": round(batch_size / (ms_c / 1e3), 1),
            "cache_bytes": sums.numel() * 4,
            "note": "scorer reads the fp32 chunk sums (1/32 of K) instead of K; not the headline workload"}}
        del sums

    del batch, q, k, v
    torch.cuda.empty_cache()
    if secondary:
        res["secondary"] = bench_secondary(dev, hbm)
        res["secondary"].update(cached_line)
    return res


_FLUSH: dict = {}


def _time_flushed(fn, dev, iters=50, warm=5) -> float:
    """Mean device time of ``fn`` with L2 flushed before every timed call (a
    256 MB write between iterations; only ``fn`` lies inside the events)."""
    buf = _FLUSH.get(dev)
    if buf is None:
        buf = _FLUSH[dev] = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(warm):
        fn()
    evs = []
    for _ in range(iters):
        # L2 flush first, then keep the GPU busy (~0.5 ms spin) while the host
        # enqueues the events and the call, so host-side overhead of short
        # calls (argument checks, ctypes) does not leak into the events.
        buf.fill_(1)
        torch.cuda._sleep(1_000_000)
        a, b = _event(), _event()
        a.record()
        fn()
        b.record()
        evs.append((a, b))
    torch.cuda.synchronize(dev)
    return sum(a.elapsed_time(b) for a, b in evs) / iters


MINI_BLOCK_BYTES = {"weights": 2 * 1024 * 1024 * 2 + 2 * 1024 * 2048 * 2,   # q/out + up/down projections, bf16
                    "attention": 8 * 512 * 128 * 2 * 2 + 8 * 8 * 4 + 3 * 8 * 128 * 2,
                    "scorer": 8 * 32768 * 128 * 2}


def bench_mini_block(dev) -> dict:
    """Config 3: mini decode block (d_model 1024 = 8 x 128, seq 32768, c64 k8,
    MLP ratio 2.0, bf16, batch 1), ms per token, L2 flushed before each step."""
    from csahca_b200 import extension as ext
    from csahca_b200.model_inference import DecodeStepGraph, MiniCSADecodeBlock

    torch.manual_seed(0)
    res = {}
    hbm, _ = _peaks()
    g = torch.Generator(device=dev).manual_seed(0)
    hidden = torch.randn(1, 1024, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(1, 8, 32768, 128, generator=g, device=dev, dtype=torch.bfloat16)
    v = torch.randn(1, 8, 32768, 128, generator=g, device=dev, dtype=torch.bfloat16)
    kw = dict(backend="cuda-csa-tiled", chunk_size=64, top_k=8)
    for variant in ("reference", "rmsnorm_silu"):
        blk = MiniCSADecodeBlock(heads=8, head_dim=128, dtype=torch.bfloat16, device=dev, mlp_ratio=2.0,
                                 variant=variant).eval()
        if variant == "rmsnorm_silu":
            for lin in (blk.q_proj, blk.out_proj, blk.up_proj, blk.down_proj):
                torch.nn.init.normal_(lin.weight, std=0.02)
        with torch.no_grad():
            sel = ext.select_topk_chunks(blk.q_proj(hidden).view(1, 8, 128), k, 64, 8)
            for mode, chunks in (("precomputed", sel), ("dynamic", None)):
                eager = _time_flushed(lambda: blk(hidden, k, v, chunks, **kw), dev, iters=100)
                graph = DecodeStepGraph(blk, hidden, k, v, chunks, **kw)
                graphed = _time_flushed(lambda: graph.step(hidden), dev, iters=100)
                nb = MINI_BLOCK_BYTES["weights"] + MINI_BLOCK_BYTES["attention"] + \
                    (MINI_BLOCK_BYTES["scorer"] if mode == "dynamic" else 0)
                res[f"{variant}/{mode}"] = {"ms_per_token_eager": round(eager, 4),
                                            "ms_per_token_graph": round(graphed, 4),
                                            "algorithmic_bytes": nb,
                                            "hbm_frac_graph": round(nb / (graphed / 1e3) / 1e9 / hbm, 4)}
        if variant == "reference":
            res["cpu_baseline"] = cpu_mini_block(blk, hidden, k, v)
    return res


def bench_splitkv(dev, rank: int, world: int, steps: int, warmup: int) -> dict:
    """One config-5 request (H64, 65536 context, 512 main + 64 C4 slots) decoded
    with its slots split across the ranks: per-shard partial kernel, NCCL
    all-gather of (o, lse), combine kernel.  Every rank holds the full caches.
    Device time per step, max over ranks; L2 flushed before every step."""
    from csahca_b200 import workloads as W
    from csahca_b200.split_kv import dsv4_split_kv_decode

    b = W.dsv4_cache(dev, num_queries=1, heads=64, context=65536, ratio=4, n_main=512, n_extra=64, seed=7)
    fn = lambda: dsv4_split_kv_decode(  # noqa: E731
        b.q, b.cache, b.token_indices, b.topk_lengths, b.extra_cache, b.extra_token_indices, b.extra_topk_lengths,
        b.attn_sink, b.page_size, b.extra_page_size, b.softmax_scale)
    _barrier(world)
    ms = _max_over_ranks(_time_flushed(fn, dev, iters=steps, warm=warmup), dev, world)
    return {"workload": "dsv4_splitkv (config 5 C4, one request, H64, 512 + 64 slots)", "n_gpus": world,
            "us_per_step": round(ms * 1e3, 2), "steps": steps, "warmup": warmup,
            "collective": "all_gather (o, lse) over NCCL" if world > 1 else "none",
            "note": "latency-bound by design: one query's work is split, the exchange is one all-gather"}


DSV4_CASES = {
    "dsv4_c0 (config 4: Q128 H64 window 128, ctx 2048-16384)":
        dict(num_queries=128, heads=64, context=(2048, 16384), ratio=0, window=128),
    "dsv4_c4 (config 5: Q256 H64 ctx 65536, 512 + 64 C4 slots)":
        dict(num_queries=256, heads=64, context=65536, ratio=4, n_main=512, n_extra=64),
    "dsv4_c128 (config 5: Q256 H64 ctx 65536, 512 + 64 C128 slots)":
        dict(num_queries=256, heads=64, context=65536, ratio=128, n_main=512, n_extra=64),
    "dsv4_c4_q1 (config 5 shape, one query: latency; the slots are split over the SMs)":
        dict(num_queries=1, heads=64, context=65536, ratio=4, n_main=512, n_extra=64),
}


def _dsv4_fn(b):
    from csahca_b200 import extension as ext

    if b.extra_cache is not None:
        return lambda: ext.dsv4_sparse_decode_forward(
            b.q, b.cache, b.token_indices, b.topk_lengths, b.extra_cache, b.extra_token_indices,
            b.extra_topk_lengths, b.attn_sink, b.page_size, b.extra_page_size, b.softmax_scale)
    return lambda: ext.dsv4_swa_decode_forward(
        b.q, b.cache, b.token_indices, b.topk_lengths, b.attn_sink, b.page_size, b.softmax_scale)


def _dsv4_figures(b, ms: float, hbm: float) -> dict:
    from csahca_b200 import workloads as W

    nb = W.dsv4_algorithmic_bytes(b)
    slots = b.token_indices.shape[1] + (0 if b.extra_token_indices is None else b.extra_token_indices.shape[1])
    flops = 4 * b.q.shape[0] * b.q.shape[1] * slots * 512
    return {"us_per_step": round(ms * 1e3, 2), "tokens_per_s": round(b.q.shape[0] / (ms / 1e3), 1),
            "achieved_gbs": round(nb / (ms / 1e3) / 1e9, 1), "hbm_frac": round(nb / (ms / 1e3) / 1e9 / hbm, 4),
            "tensor_tflops": round(flops / (ms / 1e3) / 1e12, 1), "algorithmic_bytes": nb}


def bench_dsv4_case(dev, hbm: float, kw: dict, iters: int = 50, warm: int = 5, cpu: bool = False) -> dict:
    from csahca_b200 import workloads as W

    b = W.dsv4_cache(dev, **kw)
    ms = _time_flushed(_dsv4_fn(b), dev, iters=iters, warm=warm)
    res = _dsv4_figures(b, ms, hbm)
    if cpu:
        res["cpu_baseline"] = cpu_dsv4(b)
    del b
    torch.cuda.empty_cache()
    return res


def bench_indexer(dev, hbm: float, nq: int = 256, n: int = 16384, top_k: int = 64) -> dict:
    """DSV4 compressed-slot indexer at config 5's shape: 256 queries, the 16384
    C4 slots of a 65536 context, 64 indexer heads of dim 128, top-64."""
    from csahca_b200 import extension as ext
    from oracle import indexer

    g = torch.Generator(device=dev).manual_seed(5)
    q = torch.randn(nq, 64, 128, generator=g, device=dev).to(torch.bfloat16)
    w = torch.randn(nq, 64, generator=g, device=dev) * 0.1
    keys = torch.randn(nq, n, 128, generator=g, device=dev, dtype=torch.bfloat16)
    ms = _time_flushed(lambda: ext.dsv4_indexer_topk(q, w, keys, top_k), dev, iters=30)
    nb = keys.numel() * 2 + q.numel() * 2 + w.numel() * 4 + nq * top_k * 4
    flops = 2 * nq * n * 64 * 128
    s = 2  # CPU sample: queries
    qh, wh, kh = _host(q[:s]), w[:s].cpu().numpy(), _host(keys[:s])
    t = _median_time(lambda: indexer.indexer_topk(qh, wh, kh, top_k))
    res = {"us_per_step": round(ms * 1e3, 2), "tokens_per_s": round(nq / (ms / 1e3), 1),
           "achieved_gbs": round(nb / (ms / 1e3) / 1e9, 1), "hbm_frac": round(nb / (ms / 1e3) / 1e9 / hbm, 4),
           "tensor_tflops": round(flops / (ms / 1e3) / 1e12, 1), "algorithmic_bytes": nb,
           "cpu_baseline": {"value": round(s / t, 2), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                            "cpu": _cpu_model(), "sample": f"{s} queries (numpy restatement of the published "
                                                          "indexer score + top-k), median of 3, scaled linearly"}}
    del q, w, keys
    torch.cuda.empty_cache()
    return res


def bench_secondary(dev, hbm: float) -> dict:
    from csahca_b200 import extension as ext

    out = {}
    out["dsv4_indexer (config 5 shape: Q256, 16384 C4 slots, 64 x 128 indexer heads, top-64)"] = \
        bench_indexer(dev, hbm)
    for name, kw in DSV4_CASES.items():
        out[name] = bench_dsv4_case(dev, hbm, kw, cpu="q1" not in name)
    # config 1: B1 H8 S32768 D128 c64 k8, one dynamic step
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(1, 8, 128, generator=g, device=dev, dtype=torch.bfloat16)
    k = torch.randn(1, 8, 32768, 128, generator=g, device=dev, dtype=torch.bfloat16)
    v = torch.randn(1, 8, 32768, 128, generator=g, device=dev, dtype=torch.bfloat16)
    ms = _time_flushed(lambda: ext.csa_decode_step(q, k, v, 64, 8), dev, iters=200)
    sel = ext.select_topk_chunks(q, k, 64, 8)
    ms_dec = _time_flushed(lambda: ext.csa_decode_forward_tiled(q, k, v, sel, 64, 8), dev, iters=200)
    dec_bytes = 8 * 512 * 128 * 2 * 2 + 8 * 8 * 4 + 2 * 8 * 128 * 2
    step_bytes = 8 * 32768 * 128 * 2 + dec_bytes
    name = "csa_cfg1 (config 1: B1 H8 S32768 k8, L2 flushed per step)"
    out[name] = {
        "us_per_step_dynamic": round(ms * 1e3, 2), "us_decode_precomputed": round(ms_dec * 1e3, 2),
        "tokens_per_s_dynamic": round(1.0 / (ms / 1e3), 1),
        "algorithmic_bytes_dynamic": step_bytes, "hbm_frac_dynamic": round(step_bytes / (ms / 1e3) / 1e9 / hbm, 4),
        "algorithmic_bytes_decode": dec_bytes, "hbm_frac_decode": round(dec_bytes / (ms_dec / 1e3) / 1e9 / hbm, 4),
        "decode_gbs_selected_kv": round(8 * 512 * 128 * 2 * 2 / (ms_dec / 1e3) / 1e9, 1)}
    # the same step with the chunk-sum cache: append this step's K row, select on the sums, decode
    sums = ext.chunk_sums_build(k, 64)
    pos = torch.tensor([32767], dtype=torch.int32, device=dev)

    def cached_step():
        ext.chunk_sums_append(k, sums, pos, 64)
        sel_c = ext.select_topk_chunks_from_sums(q, sums, 8, chunk_size=64)
        return ext.csa_decode_forward_tiled(q, k, v, sel_c, 64, 8)

    ms_cached = _time_flushed(cached_step, dev, iters=200)
    out[name]["us_per_step_dynamic_chunk_sum_cache"] = round(ms_cached * 1e3, 2)
    out[name]["cpu_baseline"] = cpu_cfg1(q, k, v)
    del sums, q, k, v
    torch.cuda.empty_cache()
    out["mini_block (config 3: d1024 H8 S32768 c64 k8 mlp 2.0, ms/token, L2 flushed)"] = bench_mini_block(dev)
    return out


# ------------------------------------------------------------------------------------------- sharded arms
def bench_dsv4_sharded(dev, rank: int, world: int, workload: str, steps: int, warmup: int, queries: int = 0,
                       context: int = 0) -> dict:
    """DSV4 batch split by query over the ranks (Q/N each, no collective): every
    rank builds and decodes only its queries; step time = max over ranks."""
    from csahca_b200 import partition as P
    from csahca_b200 import workloads as W

    kw = dict(next(v for k, v in DSV4_CASES.items() if k.startswith(workload + " ")))
    if queries:
        kw["num_queries"] = queries
    if context and kw["ratio"]:
        kw["context"] = context
    mine = P.shard_queries(kw["num_queries"], rank, world)
    b = W.dsv4_cache(dev, queries=mine, **kw)
    fn = _dsv4_fn(b)
    _barrier(world)
    with ClockSampler(dev.index) as clk:
        ms_own = _time_flushed(fn, dev, iters=steps, warm=max(3, warmup))
    ms = _max_over_ranks(ms_own, dev, world)
    hbm, _ = _peaks()
    fig = _dsv4_figures(b, ms_own, hbm)
    # end to end: q in from pinned host memory, output back, each step
    q_host = b.q.cpu().pin_memory()
    out_host = torch.empty(b.q.shape, dtype=b.q.dtype).pin_memory()

    def e2e_step():
        b.q.copy_(q_host, non_blocking=True)
        out_host.copy_(fn(), non_blocking=True)

    e2e_ms = _max_over_ranks(_time_flushed(e2e_step, dev, iters=steps, warm=3), dev, world)
    return {"ms": ms, "e2e_ms": e2e_ms, "kw": kw, "own": fig, "clocks": clk.summary(), "queries": len(mine),
            "h2d": q_host.numel() * 2, "d2h": out_host.numel() * 2}


def bench_indexer_sharded(dev, rank: int, world: int, steps: int, warmup: int, queries: int = 0) -> dict:
    """DSV4 indexer (score + top-64 over 16384 C4 slots, config 5's shape) split
    by query over the ranks, no collective; step time = max over ranks."""
    from csahca_b200 import extension as ext
    from csahca_b200 import partition as P

    nq_total, n, top_k = queries or 256, 16384, 64
    mine = P.shard_queries(nq_total, rank, world)
    nq = len(mine)
    g = torch.Generator(device=dev).manual_seed(5 + rank)
    q = torch.randn(nq, 64, 128, generator=g, device=dev).to(torch.bfloat16)
    w = torch.randn(nq, 64, generator=g, device=dev) * 0.1
    keys = torch.randn(nq, n, 128, generator=g, device=dev, dtype=torch.bfloat16)
    _barrier(world)
    with ClockSampler(dev.index) as clk:
        ms_own = _time_flushed(lambda: ext.dsv4_indexer_topk(q, w, keys, top_k), dev, iters=steps,
                               warm=max(3, warmup))
    nb = keys.numel() * 2 + q.numel() * 2 + w.numel() * 4 + nq * top_k * 4
    return {"ms": _max_over_ranks(ms_own, dev, world), "clocks": clk.summary(), "queries": nq,
            "nq_total": nq_total, "achieved_gbs": round(nb / (ms_own / 1e3) / 1e9, 1),
            "hbm_frac": round(nb / (ms_own / 1e3) / 1e9 / _peaks()[0], 4), "algorithmic_bytes": nb}


def bench_cfg1_sharded(dev, rank: int, world: int, steps: int, warmup: int) -> dict:
    """Config 1 (one request, 8 heads) split by head: rank r scores, selects and
    decodes heads [8r/N, 8(r+1)/N).  L2 flushed before every step."""
    from csahca_b200 import extension as ext
    from csahca_b200 import partition as P

    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(1, 8, 128, generator=g, device=dev, dtype=torch.bfloat16)
    k = torch.randn(1, 8, 32768, 128, generator=g, device=dev, dtype=torch.bfloat16)
    v = torch.randn(1, 8, 32768, 128, generator=g, device=dev, dtype=torch.bfloat16)
    lo, hi = P.shard_heads(8, rank, world)
    q, k, v = (t[:, lo:hi].contiguous() for t in (q, k, v))
    torch.cuda.empty_cache()
    _barrier(world)
    with ClockSampler(dev.index) as clk:
        ms_own = _time_flushed(lambda: ext.csa_decode_step(q, k, v, 64, 8), dev, iters=steps, warm=max(3, warmup))
    return {"ms": _max_over_ranks(ms_own, dev, world), "clocks": clk.summary(), "heads": hi - lo}


def _barrier(world: int) -> None:
    if world > 1:
        torch.distributed.barrier()


def _max_over_ranks(x: float, dev, world: int) -> float:
    if world <= 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------------------- main
def _cpu_workers(cores: int, requested: int) -> int:
    return max(1, min(cores, requested))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--cpu-requests", type=int, default=0,
                    help="config-2 requests in one CPU sample (default: one per host core, at most 16)")
    ap.add_argument("--workload", choices=["csa_batched", "csa_cfg1", "dsv4_c0", "dsv4_c4", "dsv4_c128",
                                           "dsv4_splitkv", "dsv4_indexer"], default="csa_batched",
                    help="csa_cfg1: config 1 split by head; dsv4_c*: that DSV4 batch split by query; "
                         "dsv4_splitkv: one config-5 request (C4) split across the ranks with an NCCL all-gather; "
                         "dsv4_indexer: the config-5 indexer (score + top-64) split by query")
    ap.add_argument("--batch", type=int, default=64, help="csa_batched: override the batch (profiling only)")
    ap.add_argument("--queries", type=int, default=0, help="dsv4_*: override the number of queries")
    ap.add_argument("--context", type=int, default=0, help="dsv4_c4/c128: override the per-request context")
    a = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cores = os.cpu_count() or 1
    cpu_requests = a.cpu_requests or min(cores, 16)

    if a.impl == "reference":
        if rank != 0:
            return 0
        workers = _cpu_workers(cores, cpu_requests)
        sample = make_cpu_sample(cpu_requests)
        steps = max(1, a.steps)
        for _ in range(max(0, min(a.warmup, 3))):
            time_cpu_oracle(sample, workers, repeats=1)
        value, times = time_cpu_oracle(sample, workers, repeats=steps)
        line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "impl": "reference", "n_gpus": a.gpus,
                "steps": steps, "warmup": a.warmup, "ms_per_step": round(1e3 * float(np.median(times)), 2),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded, config-2 distributions)", "config": CONFIG,
                "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": workers, "kind": "port",
                                 "cpu": _cpu_model(),
                                 "sample": f"{len(sample)} config-2 requests x 32 heads per step (numpy port of "
                                           "reference.py select_topk_chunks + csa_reference), one process per "
                                           "request, BLAS one thread each; median over steps"},
                "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    if world > 1:
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    try:
        return _run(a, dev, rank, world, cores, cpu_requests)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


def _run(a, dev, rank: int, world: int, cores: int, cpu_requests: int) -> int:
    common = {"n_gpus": world, "steps": a.steps, "warmup": a.warmup, "higher_is_better": True,
              "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
              "data": "synthetic (seeded BASELINE distributions; no dataset exists for this path)"}
    if a.workload == "dsv4_splitkv":
        res = bench_splitkv(dev, rank, world, a.steps, max(3, a.warmup))
        if rank == 0:
            print(json.dumps(res), flush=True)
        return 0
    if a.workload == "csa_cfg1":
        r = bench_cfg1_sharded(dev, rank, world, a.steps, a.warmup)
        if rank == 0:
            ms = r["ms"]
            print(json.dumps({"metric": "CSA decode throughput (score+top-k+attention), config 1",
                              "value": round(1.0 / (ms / 1e3), 1), "unit": UNIT, **common,
                              "ms_per_step": round(ms, 5), "us_per_step": round(ms * 1e3, 2),
                              "config": {"workload": "csa_cfg1 (BASELINE config 1: B1 H8 S32768 D128 c64 k8)",
                                         "parallelism": f"head-sharded over {world} GPUs, no collective",
                                         "heads_per_rank_0": r["heads"], "l2": "flushed before every step"},
                              "gpu_launches": 2 * a.steps, "clocks": r["clocks"]}), flush=True)
        return 0
    if a.workload == "dsv4_indexer":
        r = bench_indexer_sharded(dev, rank, world, a.steps, a.warmup, a.queries)
        if rank == 0:
            ms = r["ms"]
            print(json.dumps({"metric": "DSV4 indexer throughput (score + top-64), config 5 shape",
                              "value": round(r["nq_total"] / (ms / 1e3), 1), "unit": UNIT, **common,
                              "ms_per_step": round(ms, 5), "us_per_step": round(ms * 1e3, 2),
                              "config": {"workload": f"dsv4_indexer (Q{r['nq_total']}, 16384 C4 slots, "
                                                     "64 x 128 indexer heads, top-64)",
                                         "parallelism": f"query-sharded over {world} GPUs, no collective",
                                         "l2": "flushed before every step"},
                              "roofline": {"bound": "hbm", "kernel": "indexer_score_kernel + indexer_topk_kernel",
                                           "achieved": r["achieved_gbs"], "peak": _peaks()[0], "unit": "GB/s",
                                           "frac": r["hbm_frac"], "traffic": None},
                              "gpu_launches": 2 * a.steps, "clocks": r["clocks"]}), flush=True)
        return 0
    if a.workload != "csa_batched":
        r = bench_dsv4_sharded(dev, rank, world, a.workload, a.steps, a.warmup, a.queries, a.context)
        if rank == 0:
            ms, nq = r["ms"], r["kw"]["num_queries"]
            own = r["own"]
            print(json.dumps({"metric": f"DSV4 batched decode throughput, {a.workload}", "value":
                              round(nq / (ms / 1e3), 1), "unit": UNIT, **common, "ms_per_step": round(ms, 5),
                              "us_per_step": round(ms * 1e3, 2),
                              "config": {"workload": a.workload, **{k: str(v) for k, v in r["kw"].items()},
                                         "parallelism": f"query-sharded over {world} GPUs, no collective",
                                         "l2": "flushed before every step"},
                              "rank0": {"queries": r["queries"], **own},
                              "roofline": {"bound": "hbm", "kernel": "dsv4_decode", "achieved": own["achieved_gbs"],
                                           "peak": _peaks()[0], "unit": "GB/s", "frac": own["hbm_frac"],
                                           "traffic": None},
                              "e2e": {"value": round(nq / (r["e2e_ms"] / 1e3), 1), "unit": UNIT,
                                      "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"]},
                              "clocks": r["clocks"]}), flush=True)
        return 0

    r = bench_csa(dev, rank, world, a.steps, a.warmup, secondary=(world == 1 and not a.no_secondary),
                  batch_size=a.batch)
    if rank == 0:
        ms = r["total_ms"] / a.steps
        value = a.batch / (ms / 1e3)
        e2e_ms = r["e2e_ms"] / a.steps
        line = {"metric": METRIC, "value": round(value, 1), "unit": UNIT, **common,
                "ms_per_step": round(ms, 4), "us_per_step": round(ms * 1e3, 1),
                "config": dict(CONFIG, batch=a.batch,
                               parallelism=f"request-sharded over {world} GPUs (greedy by sum of context "
                                           f"lengths, imbalance {r['imbalance']}), no collective"),
                "gpu_launches": 2 * a.steps,
                "rank0": {"requests": r["requests"], "kernel_ms": {"csa_select": round(r["select_ms"], 4),
                                                                   "csa_decode": round(r["decode_ms"], 4)}},
                "kernel_ms": {"csa_select": round(r["select_ms"], 4), "csa_decode": round(r["decode_ms"], 4)},
                "step_achieved_gbs": r["step_gbs"], "roofline": r["roofline"], "decode_kernel": r["decode_kernel"],
                "e2e": {"value": round(a.batch / (e2e_ms / 1e3), 1), "unit": UNIT,
                        "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"]},
                "clocks": r["clocks"]}
        if "secondary" in r:
            line["secondary"] = r["secondary"]
        if world == 1:
            workers = _cpu_workers(cores, cpu_requests)
            sample = make_cpu_sample(cpu_requests)
            cpu_v, _ = time_cpu_oracle(sample, workers, repeats=3)
            line["cpu_baseline"] = {"value": round(cpu_v, 3), "unit": UNIT, "cores": workers, "kind": "port",
                                    "cpu": _cpu_model(),
                                    "sample": f"{len(sample)} config-2 requests x 32 heads (numpy port of "
                                              "select_topk_chunks + csa_reference), one process per request, "
                                              "median of 3"}
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
