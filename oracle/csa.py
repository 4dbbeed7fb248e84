"""CPU restatement of CSAHCA's compressed-sparse-attention math (TEST INFRASTRUCTURE ONLY).

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline legs may
use this module; the product path never does.

Each function restates one function of hybrid_attention/reference.py in numpy:

* ``chunk_mean``            reference.py:40-45
* ``select_topk_chunks``    reference.py:48-56 (ties: lower chunk index first; the
                            reference's ``torch.topk`` makes no tie promise)
* ``gather_chunk_tokens``   reference.py:59-66
* ``full_decode_attention`` reference.py:31-37 (fp32 scores, fp32 softmax, probs
                            rounded to the value dtype before the PV product, output
                            rounded to the value dtype)
* ``csa_reference``         reference.py:69-84

Tensors are numpy arrays in their storage form: bf16 as uint16 bit patterns,
f16 as float16, f32 as float32 (see ``oracle.numerics``).  ``dtype`` names the
storage type ("bf16" | "f16" | "f32").
"""

from __future__ import annotations

import math

import numpy as np

from .numerics import from_f32, round_to_dtype, to_f32


def chunk_mean(cache: np.ndarray, chunk_size: int, dtype: str) -> np.ndarray:
    """fp32 mean of each run of ``chunk_size`` tokens: ``[B,H,S,D] -> [B,H,S/c,D]``."""
    b, h, s, d = cache.shape
    if s % chunk_size != 0:
        raise ValueError("seq length must be divisible by chunk_size")
    x = to_f32(cache, dtype).reshape(b, h, s // chunk_size, chunk_size, d)
    return (x.sum(axis=3, dtype=np.float32) / np.float32(chunk_size)).astype(np.float32)


def chunk_scores(q: np.ndarray, k_cache: np.ndarray, chunk_size: int, dtype: str) -> np.ndarray:
    """Scaled chunk scores ``q . mean(K_chunk) / sqrt(D)`` in fp32: ``[B,H,C]``."""
    means = chunk_mean(k_cache, chunk_size, dtype)
    qf = to_f32(q, dtype)
    scale = np.float32(1.0 / math.sqrt(q.shape[-1]))
    return (np.einsum("bhd,bhcd->bhc", qf, means, dtype=np.float32) * scale).astype(np.float32)


def topk_lower_index(scores: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest values along the last axis, largest first,
    equal values ordered by lower index."""
    order = np.argsort(-scores, axis=-1, kind="stable")
    return order[..., :k].astype(np.int32)


def select_topk_chunks(q: np.ndarray, k_cache: np.ndarray, chunk_size: int, top_k: int, dtype: str) -> np.ndarray:
    """int32 ``[B,H,min(top_k, S/c)]`` chunk indices (reference.py:48-56)."""
    scores = chunk_scores(q, k_cache, chunk_size, dtype)
    k = min(top_k, scores.shape[-1])
    return topk_lower_index(scores, k)


def select_topk_chunks_ragged(
    q: np.ndarray, k_cache: np.ndarray, seq_lens: np.ndarray, chunk_size: int, top_k: int, dtype: str
) -> np.ndarray:
    """Per-request selection over each request's own unpadded prefix.

    Request b only sees its first ``seq_lens[b]`` tokens (a multiple of
    ``chunk_size``), exactly as running ``select_topk_chunks`` on the slice
    ``k_cache[b:b+1, :, :seq_lens[b]]``.  Slots beyond the request's chunk count
    are -1 so the output keeps one shape ``[B,H,min(top_k, S/c)]``.
    """
    b, h, s, _ = k_cache.shape
    kmax = min(top_k, s // chunk_size)
    out = np.full((b, h, kmax), -1, dtype=np.int32)
    for bi in range(b):
        length = int(seq_lens[bi])
        if length % chunk_size != 0:
            raise ValueError("seq length must be divisible by chunk_size")
        if length == 0:
            continue
        idx = select_topk_chunks(q[bi : bi + 1], k_cache[bi : bi + 1, :, :length], chunk_size, top_k, dtype)
        out[bi, :, : idx.shape[-1]] = idx[0]
    return out


def gather_chunk_tokens(cache: np.ndarray, selected_chunks: np.ndarray, chunk_size: int) -> np.ndarray:
    """Rows of the selected chunks, in slot order: ``[B,H,k*c,D]`` (reference.py:59-66)."""
    b, h, _, d = cache.shape
    offsets = np.arange(chunk_size, dtype=np.int64)
    tok = (selected_chunks.astype(np.int64)[..., None] * chunk_size + offsets).reshape(b, h, -1)
    return np.take_along_axis(cache, tok[..., None].repeat(d, axis=-1), axis=2)


def full_decode_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, dtype: str) -> np.ndarray:
    """Single-token decode attention (reference.py:31-37); returns storage-form output."""
    scale = np.float32(1.0 / math.sqrt(q.shape[-1]))
    scores = np.einsum("bhd,bhsd->bhs", to_f32(q, dtype), to_f32(k, dtype), dtype=np.float32) * scale
    m = scores.max(axis=-1, keepdims=True)
    e = np.exp(scores - m, dtype=np.float32)
    probs = (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    probs = round_to_dtype(probs, dtype)
    out = np.einsum("bhs,bhsd->bhd", probs, to_f32(v, dtype), dtype=np.float32)
    return from_f32(out, dtype)


def csa_reference(
    q: np.ndarray,
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    *,
    chunk_size: int,
    top_k: int,
    dtype: str,
    selected_chunks: np.ndarray | None = None,
) -> np.ndarray:
    """CSA decode over the selected chunks (reference.py:69-84)."""
    if selected_chunks is None:
        selected_chunks = select_topk_chunks(q, k_cache, chunk_size, top_k, dtype)
    ks = gather_chunk_tokens(k_cache, selected_chunks, chunk_size)
    vs = gather_chunk_tokens(v_cache, selected_chunks, chunk_size)
    return full_decode_attention(q, ks, vs, dtype)


def csa_decode_skipping(
    q: np.ndarray,
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    selected_chunks: np.ndarray,
    chunk_size: int,
    dtype: str,
) -> np.ndarray:
    """The CUDA op's contract for selections the torch reference cannot express.

    csrc/csa_attention.cu:47-57 and :180-186 skip slots whose chunk index is
    negative and tokens at or beyond ``seq_len``; an (b,h) with no token left
    yields zeros (:88).  Softmax runs in fp32 over the surviving tokens; the
    probabilities are NOT rounded (the kernels never round them), the output is
    rounded to the storage dtype.
    """
    b, h, s, d = k_cache.shape
    qf = to_f32(q, dtype)
    kf = to_f32(k_cache, dtype)
    vf = to_f32(v_cache, dtype)
    scale = np.float32(1.0 / math.sqrt(d))
    out = np.zeros((b, h, d), dtype=np.float32)
    for bi in range(b):
        for hi in range(h):
            toks = []
            for c in selected_chunks[bi, hi].tolist():
                if c < 0:
                    continue
                start = int(c) * chunk_size
                toks.extend(t for t in range(start, start + chunk_size) if t < s)
            if not toks:
                continue
            t = np.asarray(toks)
            sc = (kf[bi, hi, t] @ qf[bi, hi]).astype(np.float32) * scale
            e = np.exp(sc - sc.max(), dtype=np.float32)
            p = e / e.sum(dtype=np.float32)
            out[bi, hi] = p @ vf[bi, hi, t]
    return from_f32(out, dtype)
