"""Operator surface of the CSA / DSV4 decode path.

Mirrors hybrid_attention/extension.py of the reference (same function names,
arguments, input normalisation and environment switches), backed by the sm_100a
kernels of ``libcsahca_b200.so``:

* ``csa_decode_forward`` / ``csa_decode_forward_tiled``  (extension.py:48-81)
* ``dsv4_swa_decode_forward`` / ``dsv4_sparse_decode_forward`` (extension.py:98-197),
  routed to ``dsv4_decode_forward_tiled`` unless ``CSAHCA_DSV4_TILED`` is off,
  exactly as the reference routes them (extension.py:84-95)
* ``select_topk_chunks`` — the chunk scorer of hybrid_attention/reference.py:48-56
  as one GPU kernel (the reference runs it as torch ops), plus ``seq_lens`` for
  ragged batches
* ``csa_decode_step`` — score, select and decode in one call (the dynamic-selection
  step of hybrid_attention/model_inference.py:52-69)

``load_cuda_extension()`` returns the drop-in ``hybrid_attention_cuda`` module.
"""

from __future__ import annotations

import math
import os
from types import ModuleType

import torch

from . import _native as N
from . import hybrid_attention_cuda as _module


def load_cuda_extension() -> ModuleType:
    """The native module (the reference's loader, extension.py:13-45, imports ``hybrid_attention_cuda``)."""
    N.lib()  # fail loudly if the kernels are not built
    return _module


def csa_decode_forward(q, k_cache, v_cache, selected_chunks, chunk_size: int) -> torch.Tensor:
    module = load_cuda_extension()
    return module.csa_decode_forward(q.contiguous(), k_cache.contiguous(), v_cache.contiguous(),
                                     selected_chunks.contiguous(), int(chunk_size))


def csa_decode_forward_tiled(q, k_cache, v_cache, selected_chunks, chunk_size: int, tile_size: int = 8) -> torch.Tensor:
    module = load_cuda_extension()
    return module.csa_decode_forward_tiled(q.contiguous(), k_cache.contiguous(), v_cache.contiguous(),
                                           selected_chunks.contiguous(), int(chunk_size), int(tile_size))


def _dsv4_tiled_enabled(module: ModuleType) -> bool:
    if os.environ.get("CSAHCA_DSV4_TILED", "1").strip().lower() in {"", "0", "false", "no", "off"}:
        return False
    return hasattr(module, "dsv4_decode_forward_tiled")


def _dsv4_tile_size() -> int:
    try:
        return int(os.environ.get("CSAHCA_DSV4_TILE_SIZE", "0"))
    except ValueError:
        return 0


def dsv4_swa_decode_forward(q, paged_k_cache, token_indices, topk_lengths, attn_sink, page_size: int,
                            softmax_scale: float) -> torch.Tensor:
    """DSV4 decode over the SWA (compress_ratio=0) paged FP8 cache; the cache may be a uint8 or float8 view."""
    module = load_cuda_extension()
    cache_u8 = paged_k_cache.contiguous().view(torch.uint8)
    if topk_lengths is None:
        topk_lengths = torch.empty(0, dtype=torch.int32, device=q.device)
    if attn_sink is None:
        attn_sink = torch.empty(0, dtype=torch.float32, device=q.device)
    if _dsv4_tiled_enabled(module):
        return module.dsv4_decode_forward_tiled(
            q.contiguous(), cache_u8, token_indices.contiguous().to(torch.int32),
            topk_lengths.contiguous().to(torch.int32),
            torch.empty((0, 0), dtype=torch.uint8, device=q.device),
            torch.empty((0, 0), dtype=torch.int32, device=q.device),
            torch.empty(0, dtype=torch.int32, device=q.device),
            attn_sink.contiguous().to(torch.float32), int(page_size), 1, _dsv4_tile_size(), float(softmax_scale))
    return module.dsv4_swa_decode_forward(
        q.contiguous(), cache_u8, token_indices.contiguous().to(torch.int32),
        topk_lengths.contiguous().to(torch.int32), attn_sink.contiguous().to(torch.float32),
        int(page_size), float(softmax_scale))


def dsv4_sparse_decode_forward(q, paged_k_cache, token_indices, topk_lengths, extra_paged_k_cache,
                               extra_token_indices, extra_topk_lengths, attn_sink, page_size: int,
                               extra_page_size: int, softmax_scale: float) -> torch.Tensor:
    """DSV4 decode over the SWA cache plus the C4/C128 compressed cache."""
    module = load_cuda_extension()
    cache_u8 = paged_k_cache.contiguous().view(torch.uint8)
    extra_cache_u8 = extra_paged_k_cache.contiguous().view(torch.uint8)
    if topk_lengths is None:
        topk_lengths = torch.empty(0, dtype=torch.int32, device=q.device)
    if extra_topk_lengths is None:
        extra_topk_lengths = torch.empty(0, dtype=torch.int32, device=q.device)
    if attn_sink is None:
        attn_sink = torch.empty(0, dtype=torch.float32, device=q.device)
    args = (q.contiguous(), cache_u8, token_indices.contiguous().to(torch.int32),
            topk_lengths.contiguous().to(torch.int32), extra_cache_u8,
            extra_token_indices.contiguous().to(torch.int32), extra_topk_lengths.contiguous().to(torch.int32),
            attn_sink.contiguous().to(torch.float32), int(page_size), int(extra_page_size))
    if _dsv4_tiled_enabled(module):
        return module.dsv4_decode_forward_tiled(*args, _dsv4_tile_size(), float(softmax_scale))
    return module.dsv4_sparse_decode_forward(*args, float(softmax_scale))


# ------------------------------------------------------------------------------------------ chunk scorer
def select_topk_chunks(q: torch.Tensor, k_cache: torch.Tensor, chunk_size: int, top_k: int,
                       seq_lens: torch.Tensor | None = None) -> torch.Tensor:
    """Top-k chunks by ``q . mean(K_chunk) / sqrt(D)`` on the GPU (hybrid_attention/reference.py:48-56).

    Returns int32 ``[B, H, min(top_k, S // chunk_size)]``, largest score first;
    equal scores are ordered by lower chunk index.  ``seq_lens`` (int32 ``[B]``,
    multiples of ``chunk_size``) restricts request b to its first
    ``seq_lens[b]`` tokens; slots beyond its chunk count are -1.
    """
    if q.ndim != 3:
        raise ValueError(f"q must be [batch, heads, head_dim], got {tuple(q.shape)}")
    if k_cache.ndim != 4:
        raise ValueError("k_cache and v_cache must be [batch, heads, seq, head_dim]")
    if q.shape[0] != k_cache.shape[0] or q.shape[1] != k_cache.shape[1]:
        raise ValueError("q and KV cache batch/head dimensions must match")
    if q.shape[2] != k_cache.shape[3]:
        raise ValueError("q head_dim must match KV head_dim")
    if k_cache.shape[2] % chunk_size != 0:
        raise ValueError("seq length must be divisible by chunk_size")
    if q.dtype != k_cache.dtype:
        raise ValueError("q and k_cache dtype must match")
    if not (q.is_cuda and k_cache.is_cuda):
        raise RuntimeError("select_topk_chunks: q and k_cache must be CUDA tensors")
    lib = N.lib()
    q = q.contiguous()
    k_cache = k_cache.contiguous()
    b, h, s, d = k_cache.shape
    kout = min(int(top_k), s // chunk_size)
    out = torch.empty((b, h, kout), dtype=torch.int32, device=q.device)
    if seq_lens is not None:
        seq_lens = seq_lens.to(device=q.device, dtype=torch.int32).contiguous()
        if seq_lens.numel() != b:
            raise ValueError("seq_lens must have one value per batch entry")
    with torch.cuda.device(q.device):
        ws = N.workspaces.get(q.device, lib.csahca_csa_select_topk_workspace_size(b, h, s, chunk_size), "csa_select")
        N.check(lib.csahca_csa_select_topk(
            q.data_ptr(), k_cache.data_ptr(), N.ptr(seq_lens), N.DTYPE_CODE[q.dtype], b, h, s, d, int(chunk_size),
            int(top_k), out.data_ptr(), ws.data_ptr(), ws.numel(), N.stream_handle(q.device)))
    return out


# ------------------------------------------------------------------------------------ chunk-sum cache
def chunk_sums_build(k_cache: torch.Tensor, chunk_size: int) -> torch.Tensor:
    """fp32 chunk sums ``[B, H, S // chunk_size, D]`` of ``k_cache`` (the cache
    that replaces the scorer's full read of K during decoding)."""
    lib = N.lib()
    k_cache = k_cache.contiguous()
    b, h, s, d = k_cache.shape
    sums = torch.empty((b, h, s // chunk_size, d), dtype=torch.float32, device=k_cache.device)
    with torch.cuda.device(k_cache.device):
        N.check(lib.csahca_csa_chunk_sums_build(k_cache.data_ptr(), N.DTYPE_CODE[k_cache.dtype], b, h, s, d,
                                                int(chunk_size), sums.data_ptr(), N.stream_handle(k_cache.device)))
    return sums


def chunk_sums_append(k_cache: torch.Tensor, sums: torch.Tensor, positions: torch.Tensor, chunk_size: int) -> None:
    """Fold the K row each request just wrote (``positions``: int32 ``[B]``) into ``sums`` in place."""
    lib = N.lib()
    b, h, s, d = k_cache.shape
    positions = positions.to(device=k_cache.device, dtype=torch.int32).contiguous()
    with torch.cuda.device(k_cache.device):
        N.check(lib.csahca_csa_chunk_sums_append(k_cache.data_ptr(), N.DTYPE_CODE[k_cache.dtype], b, h, s, d,
                                                 int(chunk_size), positions.data_ptr(), sums.data_ptr(),
                                                 N.stream_handle(k_cache.device)))


def select_topk_chunks_from_sums(q: torch.Tensor, sums: torch.Tensor, top_k: int,
                                 seq_lens: torch.Tensor | None = None, chunk_size: int = 64) -> torch.Tensor:
    """``select_topk_chunks`` on the chunk-sum cache ``[B, H, C, D]`` fp32: the
    same indices (up to fp32 rounding of near-equal scores) from C*D*4 bytes per
    row instead of all of K.  ``seq_lens`` is in tokens, as for ``select_topk_chunks``."""
    if q.ndim != 3 or sums.ndim != 4 or q.shape[:2] != sums.shape[:2] or q.shape[2] != sums.shape[3]:
        raise ValueError("q must be [B,H,D] and sums [B,H,C,D]")
    if sums.dtype != torch.float32:
        raise ValueError("sums must be float32")
    lib = N.lib()
    q = q.contiguous()
    sums = sums.contiguous()
    b, h, c, d = sums.shape
    kout = min(int(top_k), c)
    out = torch.empty((b, h, kout), dtype=torch.int32, device=q.device)
    if seq_lens is not None:
        seq_lens = seq_lens.to(device=q.device, dtype=torch.int32).contiguous()
    with torch.cuda.device(q.device):
        ws = N.workspaces.get(q.device, lib.csahca_csa_select_topk_workspace_size(b, h, c * chunk_size, chunk_size),
                              "csa_select")
        N.check(lib.csahca_csa_select_topk_from_sums(
            q.data_ptr(), N.DTYPE_CODE[q.dtype], sums.data_ptr(), N.ptr(seq_lens), b, h, c, d, int(chunk_size),
            int(top_k), out.data_ptr(), ws.data_ptr(), ws.numel(), N.stream_handle(q.device)))
    return out


def csa_decode_step(q, k_cache, v_cache, chunk_size: int, top_k: int,
                    seq_lens: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """One dynamic-selection CSA decode step: ``(output [B,H,D], selected chunks [B,H,k])``."""
    selected = select_topk_chunks(q, k_cache, chunk_size, top_k, seq_lens)
    return csa_decode_forward_tiled(q, k_cache, v_cache, selected, chunk_size), selected


def dsv4_indexer_topk(q_idx: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor, top_k: int,
                      key_lens: torch.Tensor | None = None) -> torch.Tensor:
    """Compressed-slot indices for the DSV4 decode, selected on the GPU.

    Per query t the index score of key slot s is
    ``sum_j weights[t, j] * relu(q_idx[t, j] . keys[t, s])`` (the lightning
    indexer of the DeepSeek-V3.2 report); returns int32 ``[Q, min(top_k, N)]``
    slot positions, largest score first, equal scores by lower slot, -1 past
    ``key_lens[t]``.  ``q_idx`` bf16 ``[Q, 64, 128]``, ``weights`` fp32 ``[Q, 64]``,
    ``keys`` bf16 ``[Q, N, 128]``.  The reference receives these indices from
    its caller (integrations/sglang_dsv4/csahca_sglang_dsv4_patch/patch.py:336-341).
    """
    if q_idx.ndim != 3 or keys.ndim != 3 or weights.ndim != 2:
        raise ValueError("q_idx must be [Q,H,D], weights [Q,H], keys [Q,N,D]")
    if q_idx.shape[0] != keys.shape[0] or q_idx.shape[2] != keys.shape[2] or weights.shape != q_idx.shape[:2]:
        raise ValueError("q_idx, weights and keys dimensions must match")
    if q_idx.dtype != torch.bfloat16 or keys.dtype != torch.bfloat16:
        raise ValueError("q_idx and keys must be bfloat16")
    if not (q_idx.is_cuda and keys.is_cuda and weights.is_cuda):
        raise RuntimeError("dsv4_indexer_topk: tensors must be CUDA tensors")
    lib = N.lib()
    q_idx, keys = q_idx.contiguous(), keys.contiguous()
    weights = weights.to(torch.float32).contiguous()
    nq, heads, d = q_idx.shape
    n = keys.shape[1]
    out = torch.empty((nq, min(int(top_k), n)), dtype=torch.int32, device=q_idx.device)
    if key_lens is not None:
        key_lens = key_lens.to(device=q_idx.device, dtype=torch.int32).contiguous()
        if key_lens.numel() != nq:
            raise ValueError("key_lens must have one value per query")
    with torch.cuda.device(q_idx.device):
        ws = N.workspaces.get(q_idx.device, lib.csahca_dsv4_indexer_workspace_size(nq, n), "dsv4_indexer")
        N.check(lib.csahca_dsv4_indexer_topk(
            q_idx.data_ptr(), weights.data_ptr(), keys.data_ptr(), N.ptr(key_lens), nq, heads, n, d, int(top_k),
            out.data_ptr(), ws.data_ptr(), ws.numel(), N.stream_handle(q_idx.device)))
    return out


def default_dsv4_softmax_scale() -> float:
    return 1.0 / math.sqrt(512)
