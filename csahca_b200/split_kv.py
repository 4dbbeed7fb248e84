"""Split-KV DSV4 decode of long requests across GPUs.

One process per GPU.  Every rank holds the request's paged caches (or the pages
its slots point to) and the same index lists; rank r of G decodes a contiguous
range of the main slots and of the extra slots (``shard_slots``), producing an
fp32 output normalised by its own softmax sum and its log-sum-exp
(``dsv4_decode_partial``; the kernel slices the lists itself).  The (o, lse) pairs are all-gathered over the process
group (NCCL over NVLink on a B200 node) and every rank merges them locally
(``dsv4_combine_partials``), the sink counted once.  The merge rule is the
reference's split merge (csrc/dsv4_attention.cu:273-335); the reference runs
the split inside one GPU only.

The all-gather moves Q*H*(512+1)*4 bytes per rank (131 KB for one query with
64 heads): one exchange step per decode, latency-bound.
"""

from __future__ import annotations

import functools
from typing import Callable

import torch
import torch.distributed as dist

from . import _native as N
from .hybrid_attention_cuda import _check, _dsv4_common, _extra_checks

DSV4_HEAD_DIM = 512
MAX_SHARDS = 64  # csahca_dsv4_combine_partials merges at most this many shards


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous slot range ``[lo, hi)`` of rank ``rank`` out of ``n`` slots."""
    return (n * rank) // world, (n * (rank + 1)) // world


def shard_slots(token_indices: torch.Tensor, topk_lengths: torch.Tensor | None, rank: int,
                world: int) -> tuple[torch.Tensor, torch.Tensor]:
    """This rank's slice of an index list and the matching per-query lengths.

    A query's valid slots are its first ``clamp(length, 0, slots)``; the shard
    ``[lo, hi)`` keeps ``clamp(length - lo, 0, hi - lo)`` of them.
    """
    n = token_indices.shape[1]
    lo, hi = shard_range(n, rank, world)
    idx = token_indices[:, lo:hi].contiguous()
    if topk_lengths is None:
        full = torch.full((token_indices.shape[0],), n, dtype=torch.int32, device=token_indices.device)
    else:
        full = topk_lengths.to(torch.int32).clamp(0, n)
    lens = (full - lo).clamp(0, hi - lo).to(torch.int32).contiguous()
    return idx, lens


@functools.lru_cache(maxsize=None)
def _sm_count(device_index: int) -> int:
    return torch.cuda.get_device_properties(device_index).multi_processor_count


def auto_local_splits(num_queries: int, slots: int, device: torch.device) -> int:
    """Shards per GPU so that about one CTA per SM has work, at least 64 slots each."""
    sms = _sm_count(device.index if device.index is not None else torch.cuda.current_device()) \
        if device.type == "cuda" else 1
    return max(1, min(sms // max(1, num_queries), slots // 64))


def dsv4_decode_partial(q, paged_k_cache_u8, token_indices, topk_lengths, extra_paged_k_cache_u8,
                        extra_token_indices, extra_topk_lengths, page_size: int, extra_page_size: int,
                        softmax_scale: float, shard0: int = 0, shards: int = 1,
                        shards_total: int = 1) -> tuple[torch.Tensor, torch.Tensor]:
    """Shards ``shard0 .. shard0+shards-1`` of ``shards_total`` (equal ranges of
    every query's main and extra slot lists, sliced inside the kernel) in one
    launch: ``(o fp32 [shards,Q,H,512], lse fp32 [shards,Q,H])``."""
    # The same argument checks as the reference-facing entries (device,
    # contiguity, int32 indices and lengths, page layout): a pointer the kernel
    # cannot use must fail here, before any launch.
    _dsv4_common(q, paged_k_cache_u8, token_indices, topk_lengths, None, page_size, tiled=True)
    x, xi, xl = extra_paged_k_cache_u8, extra_token_indices, extra_topk_lengths
    has_extra = x is not None and xi is not None and x.numel() > 0 and xi.numel() > 0
    if has_extra:
        _extra_checks(x, xi, xl, q.shape[0], extra_page_size, tiled=True)
    _check(1 <= shards and 0 <= shard0 and shard0 + shards <= shards_total <= MAX_SHARDS,
           f"shards must satisfy 0 <= shard0 < shard0 + shards <= shards_total <= {MAX_SHARDS}")
    lib = N.lib()
    nq, heads, _ = q.shape
    o = torch.empty((shards, nq, heads, DSV4_HEAD_DIM), dtype=torch.float32, device=q.device)
    lse = torch.empty((shards, nq, heads), dtype=torch.float32, device=q.device)
    if nq == 0 or heads == 0:
        return o, lse
    with torch.cuda.device(q.device):
        N.check(lib.csahca_dsv4_decode_partial(
            q.contiguous().data_ptr(), N.DTYPE_CODE[q.dtype], nq, heads,
            paged_k_cache_u8.data_ptr(), paged_k_cache_u8.shape[0], paged_k_cache_u8.shape[1], int(page_size),
            token_indices.data_ptr() if token_indices.numel() else None, token_indices.shape[1],
            N.ptr(topk_lengths),
            x.data_ptr() if has_extra else None, x.shape[0] if has_extra else 0, x.shape[1] if has_extra else 0,
            int(extra_page_size) if has_extra else 1, xi.data_ptr() if has_extra else None,
            xi.shape[1] if has_extra else 0, N.ptr(xl) if has_extra else None,
            float(softmax_scale), int(shard0), int(shards), int(shards_total), o.data_ptr(), lse.data_ptr(),
            N.stream_handle(q.device)))
    return o, lse


def dsv4_combine_partials(o_parts: torch.Tensor, lse_parts: torch.Tensor, attn_sink: torch.Tensor | None,
                          out_dtype: torch.dtype) -> torch.Tensor:
    """Merge ``[G,Q,H,512]`` / ``[G,Q,H]`` shards into ``[Q,H,512]`` of ``out_dtype``."""
    _check(o_parts.is_cuda and lse_parts.is_cuda, "o_parts and lse_parts must be CUDA tensors")
    _check(o_parts.dtype == torch.float32 and lse_parts.dtype == torch.float32,
           "o_parts and lse_parts must be float32")
    _check(o_parts.dim() == 4 and o_parts.shape[3] == DSV4_HEAD_DIM, "o_parts must be [shards, Q, H, 512]")
    _check(tuple(lse_parts.shape) == tuple(o_parts.shape[:3]), "lse_parts must be [shards, Q, H]")
    _check(1 <= o_parts.shape[0] <= MAX_SHARDS, f"between 1 and {MAX_SHARDS} shards")
    _check(attn_sink is None or attn_sink.numel() in (0, o_parts.shape[2]), "attn_sink must have one value per head")
    _check(attn_sink is None or attn_sink.device == o_parts.device, "attn_sink must be on the device of o_parts")
    lib = N.lib()
    g, nq, heads, _ = o_parts.shape
    out = torch.empty((nq, heads, DSV4_HEAD_DIM), dtype=out_dtype, device=o_parts.device)
    sink = None if attn_sink is None or attn_sink.numel() == 0 else attn_sink.to(torch.float32).contiguous()
    with torch.cuda.device(o_parts.device):
        N.check(lib.csahca_dsv4_combine_partials(
            o_parts.contiguous().data_ptr(), lse_parts.contiguous().data_ptr(), g, nq, heads, N.ptr(sink),
            out.data_ptr(), N.DTYPE_CODE[out_dtype], N.stream_handle(o_parts.device)))
    return out


def dsv4_split_kv_decode(q, paged_k_cache_u8, token_indices, topk_lengths, extra_paged_k_cache_u8,
                         extra_token_indices, extra_topk_lengths, attn_sink, page_size: int, extra_page_size: int,
                         softmax_scale: float, *, group=None, local_splits: int | None = None,
                         partial_fn: Callable | None = None, combine_fn: Callable | None = None) -> torch.Tensor:
    """DSV4 decode with the slot lists split across the ranks of ``group``.

    Every rank passes the same arguments and gets the full output.  With no
    initialised process group (or a group of one) only the local split applies.
    Each rank further splits its range into ``local_splits`` shards (default:
    enough to give every SM work) that one partial launch decodes side by side,
    so a single long request spreads over the GPU's SMs too.
    ``partial_fn`` / ``combine_fn`` replace the GPU kernels (the CPU tests run
    the host logic and the collective with the numpy oracle in their place);
    ``partial_fn`` has the signature of ``dsv4_decode_partial``.
    """
    partial_fn = partial_fn or dsv4_decode_partial
    combine_fn = combine_fn or dsv4_combine_partials
    distributed = dist.is_available() and dist.is_initialized()
    world = dist.get_world_size(group) if distributed else 1
    rank = dist.get_rank(group) if distributed else 0
    if local_splits is None:
        local_splits = auto_local_splits(q.shape[0], token_indices.shape[1] // world, q.device)
        local_splits = min(local_splits, MAX_SHARDS // world)  # the combine merges at most MAX_SHARDS shards
    local_splits = max(1, int(local_splits))
    if world * local_splits > MAX_SHARDS:
        raise ValueError(f"at most {MAX_SHARDS} shards in total (world x local_splits)")
    has_extra = (extra_paged_k_cache_u8 is not None and extra_token_indices is not None
                 and extra_token_indices.numel() > 0)
    o, lse = partial_fn(q, paged_k_cache_u8, token_indices, topk_lengths,
                        extra_paged_k_cache_u8 if has_extra else None, extra_token_indices if has_extra else None,
                        extra_topk_lengths if has_extra else None, page_size, extra_page_size, softmax_scale,
                        rank * local_splits, local_splits, world * local_splits)
    if world > 1:
        o_all = torch.empty((world * o.shape[0],) + tuple(o.shape[1:]), dtype=o.dtype, device=o.device)
        lse_all = torch.empty((world * lse.shape[0],) + tuple(lse.shape[1:]), dtype=lse.dtype, device=lse.device)
        dist.all_gather_into_tensor(o_all, o.contiguous(), group=group)
        dist.all_gather_into_tensor(lse_all, lse.contiguous(), group=group)
    else:
        o_all, lse_all = o, lse
    return combine_fn(o_all, lse_all, attn_sink, q.dtype)
