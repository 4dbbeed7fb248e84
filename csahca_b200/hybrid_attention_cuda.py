"""Drop-in for the reference's native module ``hybrid_attention_cuda``.

Same five functions, argument order, dtypes and error messages as the pybind
module built from csrc/bindings.cpp:158-164, with the argument checks of the
reference host code (csrc/csa_attention.cu:330-452, csrc/dsv4_attention.cu:585-909)
raised as ``RuntimeError`` like ``TORCH_CHECK``.  Every op allocates and
returns a new output (``torch.empty_like(q)``), runs on the current CUDA stream
and does not synchronise, as the reference ops do.  Compute goes through the
C ABI of ``libcsahca_b200.so``; there is no fallback.

The reference's ``tile_size`` arguments are accepted and ignored: they only
tune the reference's split, and results do not depend on them.
"""

from __future__ import annotations

import os

import torch

from . import _native as N

__all__ = [
    "csa_decode_forward",
    "csa_decode_forward_tiled",
    "dsv4_swa_decode_forward",
    "dsv4_sparse_decode_forward",
    "dsv4_decode_forward_tiled",
]

_FLOAT_DTYPES = (torch.float32, torch.float16, torch.bfloat16)
DSV4_HEAD_DIM = 512
DSV4_TOKEN_BYTES = 584  # 576 data bytes + 8 scale bytes


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


# ----------------------------------------------------------------------------------------------- CSA
def _csa_checks(q, k_cache, v_cache, chunk_indices, chunk_size: int, tiled: bool) -> None:
    # csrc/bindings.cpp:60-62, 74-76
    if not (q.is_cuda and k_cache.is_cuda and v_cache.is_cuda and chunk_indices.is_cuda):
        _check(False, "all tensors must be CUDA tensors")
    # csrc/csa_attention.cu:336-365 (v1) and :393-423 (tiled)
    _check(q.is_contiguous(), "q must be contiguous")
    _check(k_cache.is_contiguous(), "k_cache must be contiguous")
    _check(v_cache.is_contiguous(), "v_cache must be contiguous")
    _check(chunk_indices.is_contiguous(), "chunk_indices must be contiguous")
    _check(q.dim() == 3, "q must be [batch, heads, head_dim]")
    _check(k_cache.dim() == 4, "k_cache must be [batch, heads, seq, head_dim]")
    _check(v_cache.shape == k_cache.shape, "v_cache must match k_cache shape")
    _check(chunk_indices.dim() == 3, "chunk_indices must be [batch, heads, top_k]")
    _check(q.dtype == k_cache.dtype, "q and k_cache dtype must match")
    _check(q.dtype == v_cache.dtype, "q and v_cache dtype must match")
    _check(chunk_indices.dtype in (torch.int32, torch.int64), "chunk_indices must be int32 or int64")
    b, h, d = q.shape
    _check(k_cache.shape[0] == b and k_cache.shape[1] == h and k_cache.shape[3] == d, "KV cache shape must match q")
    _check(chunk_indices.shape[0] == b and chunk_indices.shape[1] == h,
           "chunk_indices batch/head dimensions must match q")
    _check(chunk_size > 0, "chunk_size must be positive")
    _check(d <= 1024, f"head_dim > 1024 is not supported by the {'tiled' if tiled else 'v1'} kernel")
    _check(q.dtype in _FLOAT_DTYPES, f"\"csa_decode_forward_cuda\" not implemented for '{q.dtype}'")


def _csa_decode(q, k_cache, v_cache, chunk_indices, chunk_size: int) -> torch.Tensor:
    lib = N.lib()
    out = torch.empty_like(q)
    b, h, d = q.shape
    s = k_cache.shape[2]
    top_k = chunk_indices.shape[2]
    with torch.cuda.device(q.device):
        ws = N.workspaces.get(q.device, lib.csahca_csa_decode_workspace_size(b, h, d, top_k, chunk_size), "csa_decode")
        N.check(lib.csahca_csa_decode(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), chunk_indices.data_ptr(),
            N.INDEX_CODE[chunk_indices.dtype], N.DTYPE_CODE[q.dtype], b, h, s, d, top_k, int(chunk_size),
            out.data_ptr(), ws.data_ptr(), ws.numel(), N.stream_handle(q.device)))
    return out


def csa_decode_forward(q, k_cache, v_cache, chunk_indices, chunk_size: int) -> torch.Tensor:
    """CSA decode over selected chunks (reference symbol, csrc/bindings.cpp:54-64)."""
    _csa_checks(q, k_cache, v_cache, chunk_indices, chunk_size, tiled=False)
    return _csa_decode(q, k_cache, v_cache, chunk_indices, int(chunk_size))


def csa_decode_forward_tiled(q, k_cache, v_cache, chunk_indices, chunk_size: int, tile_size: int) -> torch.Tensor:
    """Split-K CSA decode (reference symbol, csrc/bindings.cpp:66-77); ``tile_size`` is validated, then unused."""
    _csa_checks(q, k_cache, v_cache, chunk_indices, chunk_size, tiled=True)
    _check(tile_size > 0, "tile_size must be positive")
    return _csa_decode(q, k_cache, v_cache, chunk_indices, int(chunk_size))


# ---------------------------------------------------------------------------------------------- DSV4
def _dsv4_auto_shards(q, token_indices, xidx) -> int:
    """Shards per query for a DSV4 launch: 1 while the queries alone keep at
    least half of the SMs busy or a query has fewer than 256 slots; otherwise
    enough 64-slot shards to cover the SMs (at most 64).
    ``CSAHCA_DSV4_SPLIT=0`` turns splitting off."""
    if os.environ.get("CSAHCA_DSV4_SPLIT", "1").strip().lower() in {"0", "false", "no", "off"}:
        return 1
    from .split_kv import MAX_SHARDS, _sm_count

    items = q.shape[0] * ((q.shape[1] + 63) // 64)
    sms = _sm_count(q.device.index if q.device.index is not None else torch.cuda.current_device())
    if 2 * items > sms:
        return 1
    slots = token_indices.shape[1] + (xidx.shape[1] if xidx is not None else 0)
    if slots < 4 * 64:
        # Up to three 64-slot blocks per query: a split shortens each CTA's
        # chain by at most two blocks, less than the merge costs (config 4's
        # 128-slot window: 23 us unsplit at 128 queries, 39 us split at 64).
        return 1
    return max(1, min(sms // items, slots // 64, MAX_SHARDS))


def _launch_dsv4(q, cache, token_indices, topk_lengths, xcache, xidx, xlens, sink, page_size, xpage_size,
                 softmax_scale) -> torch.Tensor:
    lib = N.lib()
    nq, heads, _ = q.shape
    if nq == 0 or heads == 0:
        return torch.empty_like(q)
    has_extra = xcache is not None and xidx is not None and xcache.numel() > 0 and xidx.numel() > 0
    shards = _dsv4_auto_shards(q, token_indices, xidx if has_extra else None)
    if shards > 1:
        # Few queries: split every query's slot lists over several CTAs (the
        # reference's tiled path splits the same way) and merge the shards.
        from .split_kv import dsv4_combine_partials, dsv4_decode_partial

        o, lse = dsv4_decode_partial(q, cache, token_indices, topk_lengths, xcache if has_extra else None,
                                     xidx if has_extra else None, xlens if has_extra else None, page_size,
                                     xpage_size, softmax_scale, 0, shards, shards)
        return dsv4_combine_partials(o, lse, sink, q.dtype)
    out = torch.empty_like(q)
    lens_ptr = topk_lengths.data_ptr() if topk_lengths is not None and topk_lengths.numel() > 0 else None
    sink_ptr = sink.data_ptr() if sink is not None and sink.numel() > 0 else None
    xl_ptr = xlens.data_ptr() if has_extra and xlens is not None and xlens.numel() > 0 else None
    with torch.cuda.device(q.device):
        N.check(lib.csahca_dsv4_decode(
            q.data_ptr(), N.DTYPE_CODE[q.dtype], nq, heads,
            cache.data_ptr(), cache.shape[0], cache.shape[1], int(page_size),
            token_indices.data_ptr() if token_indices.numel() else None, token_indices.shape[1], lens_ptr,
            xcache.data_ptr() if has_extra else None, xcache.shape[0] if has_extra else 0,
            xcache.shape[1] if has_extra else 0, int(xpage_size) if has_extra else 1,
            xidx.data_ptr() if has_extra else None, xidx.shape[1] if has_extra else 0, xl_ptr,
            sink_ptr, float(softmax_scale), out.data_ptr(), N.stream_handle(q.device)))
    return out


def _dsv4_common(q, cache, token_indices, topk_lengths, attn_sink, page_size, tiled: bool) -> None:
    _check(q.is_cuda, "q must be CUDA")
    _check(cache.is_cuda, "paged_k_cache_u8 must be CUDA")
    _check(token_indices.is_cuda, "token_indices must be CUDA")
    _check(topk_lengths is None or topk_lengths.is_cuda, "topk_lengths must be CUDA when defined")
    _check(attn_sink is None or attn_sink.is_cuda, "attn_sink must be CUDA when defined")
    _check(q.is_contiguous(), "q must be contiguous")
    _check(cache.is_contiguous(), "paged_k_cache_u8 must be contiguous")
    _check(token_indices.is_contiguous(), "token_indices must be contiguous")
    _check(topk_lengths is None or topk_lengths.is_contiguous(), "topk_lengths must be contiguous")
    _check(attn_sink is None or attn_sink.is_contiguous(), "attn_sink must be contiguous")
    _check(q.dim() == 3, "q must be [num_queries, heads, 512]")
    _check(q.shape[2] == DSV4_HEAD_DIM, "q head_dim must be 512 for DSV4")
    _check(cache.dim() == 2, "paged_k_cache_u8 must be [num_pages, bytes_per_page]")
    _check(cache.dtype == torch.uint8, "paged_k_cache_u8 must be uint8")
    _check(token_indices.dim() == 2, "token_indices must be [num_queries, topk_slots]")
    _check(token_indices.dtype == torch.int32, "token_indices must be int32")
    _check(topk_lengths is None or topk_lengths.dtype == torch.int32, "topk_lengths must be int32 when defined")
    _check(attn_sink is None or attn_sink.dtype == torch.float32, "attn_sink must be float32 when defined")
    _check(page_size > 0, "page_size must be positive")
    nq, heads = q.shape[0], q.shape[1]
    _check(token_indices.shape[0] == nq, "token_indices query dimension must match q")
    if tiled:
        _check(topk_lengths is None or topk_lengths.numel() in (0, nq), "topk_lengths must have one value per query")
        _check(attn_sink is None or attn_sink.numel() in (0, heads), "attn_sink must have one value per head")
    else:
        _check(topk_lengths is None or topk_lengths.numel() == nq, "topk_lengths must have one value per query")
        _check(attn_sink is None or attn_sink.numel() == heads, "attn_sink must have one value per head")
    _check(cache.shape[1] >= page_size * DSV4_TOKEN_BYTES, "bytes_per_page is too small for DSV4 page layout")
    _check(q.dtype in _FLOAT_DTYPES, f"\"dsv4_decode_forward_cuda\" not implemented for '{q.dtype}'")


def _extra_checks(x, xi, xl, nq: int, extra_page_size: int, tiled: bool) -> None:
    _check(x.is_cuda, "extra_paged_k_cache_u8 must be CUDA")
    _check(xi.is_cuda, "extra_token_indices must be CUDA")
    _check(xl is None or xl.is_cuda, "extra_topk_lengths must be CUDA when defined")
    _check(x.is_contiguous(), "extra_paged_k_cache_u8 must be contiguous")
    _check(xi.is_contiguous(), "extra_token_indices must be contiguous")
    _check(xl is None or xl.is_contiguous(), "extra_topk_lengths must be contiguous")
    _check(x.dim() == 2, "extra_paged_k_cache_u8 must be [num_pages, bytes_per_page]")
    _check(x.dtype == torch.uint8, "extra_paged_k_cache_u8 must be uint8")
    _check(xi.dim() == 2, "extra_token_indices must be [num_queries, extra_topk_slots]")
    _check(xi.dtype == torch.int32, "extra_token_indices must be int32")
    if tiled:
        _check(xl is None or xl.numel() == 0 or xl.dtype == torch.int32, "extra_topk_lengths must be int32 when defined")
    else:
        _check(xl is None or xl.dtype == torch.int32, "extra_topk_lengths must be int32 when defined")
    _check(extra_page_size > 0, "extra_page_size must be positive")
    _check(xi.shape[0] == nq, "extra_token_indices query dimension must match q")
    if tiled:
        _check(xl is None or xl.numel() in (0, nq), "extra_topk_lengths must have one value per query")
    else:
        _check(xl is None or xl.numel() == nq, "extra_topk_lengths must have one value per query")
    _check(x.shape[1] >= extra_page_size * DSV4_TOKEN_BYTES, "extra_bytes_per_page is too small for DSV4 page layout")


def dsv4_swa_decode_forward(q, paged_k_cache_u8, token_indices, topk_lengths, attn_sink, page_size: int,
                            softmax_scale: float) -> torch.Tensor:
    """DSV4 SWA decode (reference symbol, csrc/bindings.cpp:79-92; checks dsv4_attention.cu:593-625)."""
    if not (q.is_cuda and paged_k_cache_u8.is_cuda and token_indices.is_cuda):
        _check(False, "q, paged_k_cache_u8, and token_indices must be CUDA tensors")
    _dsv4_common(q, paged_k_cache_u8, token_indices, topk_lengths, attn_sink, page_size, tiled=False)
    return _launch_dsv4(q, paged_k_cache_u8, token_indices, topk_lengths, None, None, None, attn_sink, page_size,
                        1, softmax_scale)


def dsv4_sparse_decode_forward(q, paged_k_cache_u8, token_indices, topk_lengths, extra_paged_k_cache_u8,
                               extra_token_indices, extra_topk_lengths, attn_sink, page_size: int,
                               extra_page_size: int, softmax_scale: float) -> torch.Tensor:
    """DSV4 SWA + C4/C128 decode (reference symbol, csrc/bindings.cpp:94-125; checks dsv4_attention.cu:671-728)."""
    if not (q.is_cuda and paged_k_cache_u8.is_cuda and token_indices.is_cuda and extra_paged_k_cache_u8.is_cuda
            and extra_token_indices.is_cuda):
        _check(False, "q, paged_k_cache_u8, token_indices, extra_paged_k_cache_u8, and extra_token_indices "
                      "must be CUDA tensors")
    _dsv4_common(q, paged_k_cache_u8, token_indices, topk_lengths, attn_sink, page_size, tiled=False)
    _extra_checks(extra_paged_k_cache_u8, extra_token_indices, extra_topk_lengths, q.shape[0], extra_page_size,
                  tiled=False)
    return _launch_dsv4(q, paged_k_cache_u8, token_indices, topk_lengths, extra_paged_k_cache_u8,
                        extra_token_indices, extra_topk_lengths, attn_sink, page_size, extra_page_size,
                        softmax_scale)


def dsv4_decode_forward_tiled(q, paged_k_cache_u8, token_indices, topk_lengths, extra_paged_k_cache_u8,
                              extra_token_indices, extra_topk_lengths, attn_sink, page_size: int,
                              extra_page_size: int, tile_size: int, softmax_scale: float) -> torch.Tensor:
    """Default DSV4 entry (reference symbol, csrc/bindings.cpp:127-156; checks dsv4_attention.cu:775-848).

    The extra cache is used when both it and its indices are non-empty; empty
    lengths / sink tensors mean "absent", as in the reference.
    """
    if not (q.is_cuda and paged_k_cache_u8.is_cuda and token_indices.is_cuda):
        _check(False, "q, paged_k_cache_u8, and token_indices must be CUDA tensors")
    _dsv4_common(q, paged_k_cache_u8, token_indices, topk_lengths, attn_sink, page_size, tiled=True)
    _check(paged_k_cache_u8.shape[1] % 4 == 0,
           "tiled DSV4 kernel requires bytes_per_page divisible by 4 for vectorized loads")
    x, xi, xl = extra_paged_k_cache_u8, extra_token_indices, extra_topk_lengths
    has_extra = x is not None and x.numel() > 0 and xi is not None and xi.numel() > 0
    if has_extra:
        _extra_checks(x, xi, xl, q.shape[0], extra_page_size, tiled=True)
        _check(x.shape[1] % 4 == 0,
               "tiled DSV4 kernel requires extra_bytes_per_page divisible by 4 for vectorized loads")
    else:
        x = xi = xl = None
    return _launch_dsv4(q, paged_k_cache_u8, token_indices, topk_lengths, x, xi, xl, attn_sink, page_size,
                        extra_page_size, softmax_scale)
