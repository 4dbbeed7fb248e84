"""Seeded synthetic inputs for the benchmark configurations (device-side setup code).

No dataset is involved anywhere in the reference's benchmarks: every input is
seeded random data with the shapes and distributions of BASELINE.json's configs.

* ``csa_batched``   config 2: B=64 requests, H=32, D=128, per-request context
                    uniform over multiples of 64 in [4096, 32768] (stored padded
                    to 32768), K = N(0,1) + a per-chunk N(0, 0.5) offset, V = N(0,1).
* ``dsv4_cache``    configs 4/5: DSV4 paged FP8 caches (448 e4m3 + 64 bf16 dims,
                    UE8M0 scale per 64 dims, hybrid_attention/dsv4_correctness.py:24-59)
                    behind a seeded permutation of physical pages; C4/C128
                    compressed caches hold the re-quantised mean of 4 / 128 raw
                    latents.

``pack_tokens_torch`` is the packer written with torch ops so it runs on the
GPU; its bytes equal the reference packer's (checked against the CPU oracle).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

DIM_NOPE, DIM_ROPE, HEAD_DIM = 448, 64, 512
ROW_BYTES, SCALE_BYTES = 576, 8


def bytes_per_page(page_size: int) -> int:
    raw = page_size * (ROW_BYTES + SCALE_BYTES)
    return ((raw + ROW_BYTES - 1) // ROW_BYTES) * ROW_BYTES


# ------------------------------------------------------------------------------------------------ CSA
@dataclass
class CsaBatch:
    q: torch.Tensor          # [B,H,D] bf16
    k: torch.Tensor          # [B,H,S,D] bf16
    v: torch.Tensor          # [B,H,S,D] bf16
    seq_lens: torch.Tensor   # [B] int32, multiples of chunk
    chunk: int
    top_k: int
    request_ids: list[int] | None = None  # which requests of the full batch these rows are


def _request_generator(device, seed: int, index: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1_000_003 + index + 1)
    return g


def csa_request_lengths(*, batch=64, seq_len=32768, chunk=64, min_len=4096, seed=0) -> list[int]:
    """Per-request context lengths of the full batch (uniform over multiples of
    ``chunk`` in [min_len, seq_len]); host-side, so every rank agrees on them."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randint(min_len // chunk, seq_len // chunk + 1, (batch,), generator=g) * chunk).tolist()


def csa_batched(device, *, batch=64, heads=32, seq_len=32768, head_dim=128, chunk=64, top_k=16,
                min_len=4096, seed=0, dtype=torch.bfloat16, requests=None) -> CsaBatch:
    """Config 2's batch, or only the rows ``requests`` of it (a rank's share).

    Every request draws its q, K and V from its own generator, so a request's
    data is the same whichever subset of the batch is materialised."""
    lens_all = csa_request_lengths(batch=batch, seq_len=seq_len, chunk=chunk, min_len=min_len, seed=seed)
    ids = list(range(batch)) if requests is None else [int(r) for r in requests]
    n = len(ids)
    q = torch.empty(n, heads, head_dim, device=device, dtype=dtype)
    k = torch.empty(n, heads, seq_len, head_dim, device=device, dtype=dtype)
    v = torch.empty_like(k)
    for i, r in enumerate(ids):  # per request, to bound temporaries
        g = _request_generator(device, seed, r)
        q[i].copy_(torch.randn(heads, head_dim, generator=g, device=device, dtype=dtype))
        kb = torch.randn(heads, seq_len // chunk, chunk, head_dim, generator=g, device=device, dtype=torch.float32)
        kb += torch.randn(heads, seq_len // chunk, 1, 1, generator=g, device=device) * 0.5
        k[i].copy_(kb.view(heads, seq_len, head_dim))
        del kb
        v[i].copy_(torch.randn(heads, seq_len, head_dim, generator=g, device=device, dtype=dtype))
    lens = torch.tensor([lens_all[r] for r in ids], dtype=torch.int32, device=device)
    return CsaBatch(q, k, v, lens, chunk, top_k, ids)


def csa_algorithmic_bytes(batch: CsaBatch) -> dict[str, int]:
    """Bytes a step must move at minimum: the scorer reads every valid K row once;
    the decode reads the selected K and V rows; plus q, indices and outputs."""
    b, h, _, d = batch.k.shape
    es = batch.k.element_size()
    valid_tokens = int(batch.seq_lens.sum().item())
    q_bytes = b * h * d * es
    idx_bytes = b * h * batch.top_k * 4
    scorer = valid_tokens * h * d * es + q_bytes + idx_bytes
    decode = 2 * b * h * batch.top_k * batch.chunk * d * es + q_bytes + idx_bytes + q_bytes
    return {"scorer": scorer, "decode": decode, "step": scorer + decode - q_bytes - idx_bytes}


# ------------------------------------------------------------------------------------------------ DSV4
def pack_tokens_torch(tokens_bf16: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantise ``[T,512]`` bf16 -> (data rows uint8 [T,576], scale bytes uint8 [T,8]).

    Same arithmetic as hybrid_attention/dsv4_correctness.py:43-57: per 64-dim
    tile, scale = 2^ceil(log2(max|x| / 448)), e4m3 = clamp(x / scale), UE8M0 byte
    = exponent + 127.
    """
    t = tokens_bf16.shape[0]
    nope = tokens_bf16[:, :DIM_NOPE].float().view(t, 7, 64)
    max_abs = nope.abs().amax(dim=-1).clamp_min(1e-8)
    ratio = max_abs / 448.0
    exponent = torch.ceil(torch.log2(ratio.double())).to(torch.int64)
    scale_u8 = (exponent + 127).clamp(0, 255).to(torch.uint8)
    scale = torch.ldexp(torch.ones_like(max_abs), exponent.to(torch.float32))
    codes = (nope / scale[..., None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8).view(t, DIM_NOPE)
    rope = tokens_bf16[:, DIM_NOPE:].contiguous().view(torch.uint8).view(t, 2 * DIM_ROPE)
    data = torch.cat([codes, rope], dim=1)
    scales = torch.cat([scale_u8, torch.zeros(t, 1, dtype=torch.uint8, device=tokens_bf16.device)], dim=1)
    return data, scales


def write_rows(cache: torch.Tensor, page_size: int, locs: torch.Tensor, data: torch.Tensor, scales: torch.Tensor):
    """Scatter packed rows into ``cache [pages, bytes_per_page]`` at absolute slots ``locs``."""
    rows = cache[:, : page_size * ROW_BYTES].unflatten(1, (page_size, ROW_BYTES))
    base = page_size * ROW_BYTES
    srows = cache[:, base : base + page_size * SCALE_BYTES].unflatten(1, (page_size, SCALE_BYTES))
    page, slot = locs // page_size, locs % page_size
    rows[page, slot] = data
    srows[page, slot] = scales


@dataclass
class Dsv4Batch:
    q: torch.Tensor                 # [Q,H,512] bf16
    cache: torch.Tensor             # [pages, bpp] uint8
    page_size: int
    token_indices: torch.Tensor     # [Q, n_main] int32
    topk_lengths: torch.Tensor      # [Q] int32
    extra_cache: torch.Tensor | None
    extra_page_size: int
    extra_token_indices: torch.Tensor | None
    extra_topk_lengths: torch.Tensor | None
    attn_sink: torch.Tensor         # [H] fp32
    softmax_scale: float
    query_ids: list[int] | None = None  # which requests of the full batch these rows are


def dsv4_cache(device, *, num_queries=256, heads=64, context=65536, page_size=64, n_main=512, ratio=4,
               n_extra=64, window=None, seed=0, queries=None) -> Dsv4Batch:
    """Config 5 (ratio 4 / 128, ``n_main`` sampled slots + ``n_extra`` compressed slots)
    or config 4 (ratio 0: the last ``window`` positions of a per-request context in
    ``context`` = [2048, 16384]).

    ``queries`` selects a subset of the ``num_queries`` requests (a rank's
    share).  Context lengths and the sink come from one host generator and every
    request's q, latents and slot choices from its own, so a request decodes to
    the same output whichever subset is built; only the physical page order
    (a seeded permutation over the pages built) differs."""
    master = torch.Generator().manual_seed(seed)
    if ratio == 0:
        lo, hi = context if isinstance(context, tuple) else (context, context)
        ctx_all = torch.randint(lo, hi + 1, (num_queries,), generator=master).tolist()
    else:
        ctx_all = [int(context)] * num_queries
    sink = torch.randn(heads, generator=master, dtype=torch.float32).to(device)
    ids = list(range(num_queries)) if queries is None else [int(r) for r in queries]
    nq = len(ids)
    ctx_host = [ctx_all[r] for r in ids]
    pages_host = [(L + page_size - 1) // page_size for L in ctx_host]
    total_pages = sum(pages_host)
    first_host = [sum(pages_host[:i]) for i in range(nq)]
    gp = torch.Generator(device=device)
    gp.manual_seed(seed * 7919 + 17)
    perm = torch.randperm(max(total_pages, 1), generator=gp, device=device)
    cache = torch.zeros(max(total_pages, 1), bytes_per_page(page_size), dtype=torch.uint8, device=device)
    xp = 0
    if ratio:
        xp = max(1, page_size // ratio)
        xtok_per_req = int(context) // ratio
        xpages_per_req = (xtok_per_req + xp - 1) // xp
        xcache = torch.zeros(max(nq, 1) * xpages_per_req, bytes_per_page(xp), dtype=torch.uint8, device=device)
        xperm = torch.randperm(max(nq, 1) * xpages_per_req, generator=gp, device=device)
    q = torch.empty(nq, heads, HEAD_DIM, device=device, dtype=torch.bfloat16)
    idx = torch.empty(nq, n_main if ratio else (window or 128), dtype=torch.int32, device=device)
    xidx = torch.empty(nq, n_extra, dtype=torch.int32, device=device) if ratio else None
    for i, r in enumerate(ids):
        g = _request_generator(device, seed, r)
        q[i].copy_(torch.randn(heads, HEAD_DIM, generator=g, device=device, dtype=torch.bfloat16))
        L = ctx_host[i]
        raw = torch.randn(L, HEAD_DIM, generator=g, device=device, dtype=torch.bfloat16)
        pos = torch.arange(L, device=device)
        locs = perm[first_host[i] + pos // page_size] * page_size + pos % page_size
        data, sc = pack_tokens_torch(raw)
        write_rows(cache, page_size, locs, data, sc)
        if ratio:
            sel = torch.randperm(L, generator=g, device=device)[:n_main]
            idx[i] = locs[sel].to(torch.int32)
            comp = raw[: (L // ratio) * ratio].float().view(-1, ratio, HEAD_DIM).mean(1).to(torch.bfloat16)
            xpos = torch.arange(comp.shape[0], device=device)
            xlocs = xperm[i * xpages_per_req + xpos // xp] * xp + xpos % xp
            xd, xs = pack_tokens_torch(comp)
            write_rows(xcache, xp, xlocs, xd, xs)
            xsel = torch.randperm(comp.shape[0], generator=g, device=device)[:n_extra]
            xidx[i] = xlocs[xsel].to(torch.int32)
        else:
            w = idx.shape[1]
            lastp = torch.arange(max(0, L - w), L, device=device)
            row = torch.full((w,), -1, dtype=torch.int32, device=device)
            row[: lastp.numel()] = locs[lastp].to(torch.int32)
            idx[i] = row
    lens = torch.full((nq,), idx.shape[1], dtype=torch.int32, device=device)
    return Dsv4Batch(q, cache, page_size, idx, lens, xcache if ratio else None, xp, xidx,
                     torch.full((nq,), n_extra, dtype=torch.int32, device=device) if ratio else None,
                     sink, 1.0 / math.sqrt(HEAD_DIM), ids)


def dsv4_algorithmic_bytes(b: Dsv4Batch) -> int:
    """Selected rows (576 data + 8 scale bytes each) + indices + lengths + q + out + sink."""
    nq = b.q.shape[0]
    slots = int((b.token_indices >= 0).sum().item())
    idx_bytes = b.token_indices.numel() * 4 + nq * 4
    if b.extra_token_indices is not None:
        slots += int((b.extra_token_indices >= 0).sum().item())
        idx_bytes += b.extra_token_indices.numel() * 4 + nq * 4
    qo = 2 * b.q.numel() * b.q.element_size()
    return slots * (ROW_BYTES + SCALE_BYTES) + idx_bytes + qo + b.attn_sink.numel() * 4
