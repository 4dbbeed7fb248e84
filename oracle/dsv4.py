"""CPU restatement of CSAHCA's DeepSeek-V4 paged FP8 cache and decode oracle
(TEST INFRASTRUCTURE ONLY: only `tests/`, `__graft_entry__.smoke()` and
`bench.py`'s CPU-baseline legs may use it).

Follows hybrid_attention/dsv4_correctness.py:

* layout constants      :10-16   (448 e4m3 "nope" dims + 64 bf16 "rope" dims;
                                  one UE8M0 scale byte per 64 nope dims, 7 + 1 pad)
* ``bytes_per_page``    :19-21
* ``pack_dsv4_cache``   :24-59   (vectorised here; byte-identical output)
* ``dequant_dsv4_cache``:62-88   (nope = e4m3 * 2^(s-127) in fp32, rounded to bf16)
* ``reference_attention``:91-141 (fp32 softmax with the sink as a zero-valued
                                  virtual token; lengths clamped to [0, slots];
                                  negative slots skipped)
* ``partial_attention`` / ``combine_partials``: the same decode split over
  shards of the slot list and merged by log-sum-exp, the sink entering once
  (the merge rule of csrc/dsv4_attention.cu:273-335)

The slot-validity rules match csrc/dsv4_attention.cu:185-225.
"""

from __future__ import annotations

import math

import numpy as np

from .numerics import E4M3_TO_F32, FP8_E4M3_MAX, bf16_to_f32, f32_to_bf16, f32_to_e4m3, from_f32, to_f32

DIM_NOPE = 448
DIM_ROPE = 64
HEAD_DIM = DIM_NOPE + DIM_ROPE
SCALE_TILE = 64
NUM_SCALE_TILES = DIM_NOPE // SCALE_TILE
NOPE_ROPE_BYTES = DIM_NOPE + DIM_ROPE * 2  # 576
SCALE_BYTES_PER_TOKEN = NUM_SCALE_TILES + 1  # 8
TOKEN_BYTES = NOPE_ROPE_BYTES + SCALE_BYTES_PER_TOKEN  # 584


def bytes_per_page(page_size: int) -> int:
    raw = page_size * TOKEN_BYTES
    return ((raw + NOPE_ROPE_BYTES - 1) // NOPE_ROPE_BYTES) * NOPE_ROPE_BYTES


def quantize_tokens(k_tokens_bf16: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Per-token quantisation of ``[T,512]`` bf16 bits -> (e4m3 [T,448], scale u8 [T,7], rope bits [T,64])."""
    t = k_tokens_bf16.shape[0]
    nope = bf16_to_f32(k_tokens_bf16[:, :DIM_NOPE]).reshape(t, NUM_SCALE_TILES, SCALE_TILE)
    max_abs = np.maximum(np.abs(nope).max(axis=-1), np.float32(1e-8)).astype(np.float32)
    ratio = (max_abs / np.float32(FP8_E4M3_MAX)).astype(np.float32)
    exponent = np.ceil(np.log2(ratio.astype(np.float64))).astype(np.int64)
    scale_u8 = np.clip(exponent + 127, 0, 255).astype(np.uint8)
    scale = np.ldexp(np.float32(1.0), exponent).astype(np.float32)
    vals = np.clip(nope / scale[..., None], -FP8_E4M3_MAX, FP8_E4M3_MAX).astype(np.float32)
    codes = f32_to_e4m3(vals).reshape(t, DIM_NOPE)
    rope = np.ascontiguousarray(k_tokens_bf16[:, DIM_NOPE:], dtype=np.uint16)
    return codes, scale_u8, rope


def pack_dsv4_cache(k_tokens_bf16: np.ndarray, *, page_size: int) -> np.ndarray:
    """Pack ``[T,512]`` bf16 bits into ``[pages, bytes_per_page]`` uint8 (dsv4_correctness.py:24-59)."""
    t = k_tokens_bf16.shape[0]
    num_pages = (t + page_size - 1) // page_size
    bpp = bytes_per_page(page_size)
    cache = np.zeros((num_pages, bpp), dtype=np.uint8)
    if t == 0:
        return cache
    codes, scale_u8, rope = quantize_tokens(k_tokens_bf16)
    loc = np.arange(t)
    page = loc // page_size
    in_page = loc % page_size
    data = np.concatenate([codes, rope.view(np.uint8).reshape(t, DIM_ROPE * 2)], axis=1)
    data_cols = in_page[:, None] * NOPE_ROPE_BYTES + np.arange(NOPE_ROPE_BYTES)[None, :]
    cache[page[:, None], data_cols] = data
    scale_cols = page_size * NOPE_ROPE_BYTES + in_page[:, None] * SCALE_BYTES_PER_TOKEN + np.arange(NUM_SCALE_TILES)[None, :]
    cache[page[:, None], scale_cols] = scale_u8
    return cache


def pack_tokens_at(cache: np.ndarray, locs: np.ndarray, k_tokens_bf16: np.ndarray, *, page_size: int) -> None:
    """Write tokens into an existing cache at absolute slot indices ``locs`` (same bytes as the packer)."""
    codes, scale_u8, rope = quantize_tokens(k_tokens_bf16)
    t = locs.shape[0]
    page = locs // page_size
    in_page = locs % page_size
    data = np.concatenate([codes, rope.view(np.uint8).reshape(t, DIM_ROPE * 2)], axis=1)
    cache[page[:, None], in_page[:, None] * NOPE_ROPE_BYTES + np.arange(NOPE_ROPE_BYTES)[None, :]] = data
    cols = page_size * NOPE_ROPE_BYTES + in_page[:, None] * SCALE_BYTES_PER_TOKEN + np.arange(SCALE_BYTES_PER_TOKEN)[None, :]
    cache[page[:, None], cols] = np.concatenate([scale_u8, np.zeros((t, 1), np.uint8)], axis=1)


def dequant_dsv4_cache(cache: np.ndarray, token_indices: np.ndarray, *, page_size: int) -> np.ndarray:
    """Rows at absolute slot indices -> bf16 bits ``[..., 512]`` (dsv4_correctness.py:62-88)."""
    bpp = cache.shape[1]
    flat = cache.reshape(-1)
    loc = np.asarray(token_indices, dtype=np.int64).reshape(-1)
    page = loc // page_size
    in_page = loc % page_size
    data_base = page * bpp + in_page * NOPE_ROPE_BYTES
    scale_base = page * bpp + page_size * NOPE_ROPE_BYTES + in_page * SCALE_BYTES_PER_TOKEN
    nope = E4M3_TO_F32[flat[data_base[:, None] + np.arange(DIM_NOPE)[None, :]]]
    s = flat[scale_base[:, None] + np.arange(NUM_SCALE_TILES)[None, :]].astype(np.int64) - 127
    scale = np.ldexp(np.float32(1.0), s).astype(np.float32)
    nope = (nope * np.repeat(scale, SCALE_TILE, axis=1)).astype(np.float32)
    rope_bytes = flat[(data_base + DIM_NOPE)[:, None] + np.arange(DIM_ROPE * 2)[None, :]]
    rope = np.ascontiguousarray(rope_bytes).view(np.uint16).reshape(-1, DIM_ROPE)
    out = np.concatenate([f32_to_bf16(nope), rope], axis=1)
    return out.reshape(*np.shape(token_indices), HEAD_DIM)


def _valid_slots(indices: np.ndarray, length: int | None) -> np.ndarray:
    n = indices.shape[0]
    valid = n if length is None else max(0, min(int(length), n))
    s = indices[:valid]
    return s[s >= 0]


def reference_attention(
    q: np.ndarray,
    q_dtype: str,
    cache: np.ndarray,
    token_indices: np.ndarray,
    topk_lengths: np.ndarray | None,
    attn_sink: np.ndarray | None,
    *,
    page_size: int,
    softmax_scale: float,
    extra_cache: np.ndarray | None = None,
    extra_token_indices: np.ndarray | None = None,
    extra_topk_lengths: np.ndarray | None = None,
    extra_page_size: int | None = None,
) -> np.ndarray:
    """fp32 sink-softmax decode over the valid slots (dsv4_correctness.py:91-141).

    Returns the output in q's storage form ``[Q,H,512]``.
    """
    nq, heads, _ = q.shape
    qf = to_f32(q, q_dtype)
    scale = np.float32(softmax_scale)
    out = np.zeros((nq, heads, HEAD_DIM), dtype=np.float32)
    for qi in range(nq):
        main = _valid_slots(token_indices[qi], None if topk_lengths is None else topk_lengths[qi])
        rows = [dequant_dsv4_cache(cache, main, page_size=page_size)] if main.size else []
        if extra_cache is not None and extra_token_indices is not None and extra_token_indices.shape[1] > 0:
            if extra_page_size is None:
                raise ValueError("extra_page_size is required with extra_cache")
            xs = _valid_slots(
                extra_token_indices[qi], None if extra_topk_lengths is None else extra_topk_lengths[qi]
            )
            if xs.size:
                rows.append(dequant_dsv4_cache(extra_cache, xs, page_size=extra_page_size))
        kv = bf16_to_f32(np.concatenate(rows, axis=0)) if rows else np.zeros((0, HEAD_DIM), np.float32)
        scores = (kv @ qf[qi].T).astype(np.float32) * scale  # [N, H]
        if attn_sink is not None:
            sink = np.asarray(attn_sink, dtype=np.float32)[None, :]
            scores = np.concatenate([sink, scores], axis=0)
            kv = np.concatenate([np.zeros((1, HEAD_DIM), np.float32), kv], axis=0)
        if scores.shape[0] == 0:
            continue
        m = scores.max(axis=0, keepdims=True)
        e = np.exp(scores - m, dtype=np.float32)
        p = (e / e.sum(axis=0, keepdims=True, dtype=np.float32)).astype(np.float32)
        out[qi] = p.T @ kv
    return from_f32(out, q_dtype)


def default_softmax_scale() -> float:
    return 1.0 / math.sqrt(HEAD_DIM)


def partial_attention(
    q: np.ndarray,
    q_dtype: str,
    cache: np.ndarray,
    token_indices: np.ndarray,
    topk_lengths: np.ndarray | None,
    *,
    page_size: int,
    softmax_scale: float,
    extra_cache: np.ndarray | None = None,
    extra_token_indices: np.ndarray | None = None,
    extra_topk_lengths: np.ndarray | None = None,
    extra_page_size: int | None = None,
) -> tuple[np.ndarray, np.ndarray]:
    """One shard of a split-KV decode: softmax over this shard's valid slots only,
    no sink.  Returns ``(o, lse)``: fp32 ``[Q,H,512]`` normalised by the shard's
    own sum, and fp32 ``[Q,H]`` = log2 of that sum plus the max score in log2
    units (``-inf`` for a shard with no valid slot, whose ``o`` is zero)."""
    nq, heads, _ = q.shape
    qf = to_f32(q, q_dtype)
    scale = np.float32(softmax_scale)
    o = np.zeros((nq, heads, HEAD_DIM), np.float32)
    lse = np.full((nq, heads), -np.inf, np.float32)
    for qi in range(nq):
        main = _valid_slots(token_indices[qi], None if topk_lengths is None else topk_lengths[qi])
        rows = [dequant_dsv4_cache(cache, main, page_size=page_size)] if main.size else []
        if extra_cache is not None and extra_token_indices is not None and extra_token_indices.shape[1] > 0:
            xs = _valid_slots(extra_token_indices[qi], None if extra_topk_lengths is None else extra_topk_lengths[qi])
            if xs.size:
                rows.append(dequant_dsv4_cache(extra_cache, xs, page_size=extra_page_size))
        if not rows:
            continue
        kv = bf16_to_f32(np.concatenate(rows, axis=0))
        scores = (kv @ qf[qi].T).astype(np.float32) * scale  # [N, H]
        m = scores.max(axis=0)
        e = np.exp(scores - m[None, :], dtype=np.float32)
        s = e.sum(axis=0, dtype=np.float32)
        o[qi] = (e / s[None, :]).T @ kv
        lse[qi] = (np.log2(s) + m * np.float32(math.log2(math.e))).astype(np.float32)
    return o, lse


def combine_partials(o_parts: np.ndarray, lse_parts: np.ndarray, attn_sink: np.ndarray | None,
                     q_dtype: str) -> np.ndarray:
    """Merge shard outputs ``[G,Q,H,512]`` / ``[G,Q,H]`` into the full decode,
    the sink entering once as a zero-valued token (dsv4_attention.cu:292-299)."""
    lse = lse_parts.astype(np.float64)
    m = lse.max(axis=0)
    if attn_sink is not None:
        sk = np.asarray(attn_sink, np.float64)[None, :] * math.log2(math.e)
        m = np.maximum(m, sk)
    with np.errstate(invalid="ignore"):
        w = np.where(np.isfinite(lse), np.exp2(lse - m[None]), 0.0)
    total = w.sum(axis=0)
    if attn_sink is not None:
        total = total + np.where(np.isfinite(m), np.exp2(sk - m), 0.0)
    out = (w[..., None] * o_parts).sum(axis=0) / np.where(total > 0, total, 1.0)[..., None]
    out = np.where((total > 0)[..., None], out, 0.0)
    return from_f32(out.astype(np.float32), q_dtype)
