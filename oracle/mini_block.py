"""CPU restatement of the mini decode block (TEST INFRASTRUCTURE ONLY).

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline legs may
use this module; the product path never does.

Restates ``MiniCSADecodeBlock.forward`` of hybrid_attention/model_inference.py:38-76
in numpy for the "cuda-csa" / "torch-csa" backends (they compute the same
function): ``q = q_proj(hidden)``, optional dynamic selection
(reference.py:48-56), CSA attention (reference.py:69-84), then
``hidden + 0.01 * (out_proj(attn) + down_proj(gelu(up_proj(hidden))))``.
Every torch op of the reference returns its input dtype, so each intermediate is
rounded to ``dtype`` here (GEMV products accumulate in fp32; GELU is the exact
erf form, torch's default).
"""

from __future__ import annotations

import math

import numpy as np

from . import csa
from .numerics import from_f32, to_f32


def _r(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 values to ``dtype`` and back to fp32."""
    return to_f32(from_f32(np.asarray(x, np.float32), dtype), dtype)


def _linear(x: np.ndarray, w: np.ndarray, dtype: str) -> np.ndarray:
    return _r(x.astype(np.float32) @ w.astype(np.float32).T, dtype)


def _gelu(x: np.ndarray) -> np.ndarray:
    erf = np.vectorize(math.erf, otypes=[np.float64])
    return (0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))).astype(np.float32)


def block_forward(hidden, k_cache, v_cache, w_q, w_o, w_up, w_down, *, chunk_size: int, top_k: int,
                  dtype: str, selected_chunks=None, q_override=None):
    """One decode step.  Arrays are in storage form (``oracle.numerics``);
    weights are ``[out, in]`` like ``nn.Linear``.  ``w_up``/``w_down`` may be
    None (mlp_ratio 0).  ``q_override`` (fp32 values already rounded to
    ``dtype``, ``[B,H,D]``) replaces the q projection when the caller wants the
    selection taken on a given q.  Returns ``(new_hidden, selected_chunks)``."""
    b, h, s, d = k_cache.shape
    hid = to_f32(hidden, dtype)
    wq, wo = to_f32(w_q, dtype), to_f32(w_o, dtype)
    q = _linear(hid, wq, dtype).reshape(b, h, d) if q_override is None else q_override
    q_store = from_f32(q, dtype)
    if selected_chunks is None:
        selected_chunks = csa.select_topk_chunks(q_store, k_cache, chunk_size, top_k, dtype)
    attn = csa.csa_reference(q_store, k_cache, v_cache, chunk_size=chunk_size, top_k=selected_chunks.shape[-1],
                             dtype=dtype, selected_chunks=selected_chunks)
    out = _linear(to_f32(attn, dtype).reshape(b, h * d), wo, dtype)
    if w_up is not None:
        up = _linear(hid, to_f32(w_up, dtype), dtype)
        mlp = _linear(_r(_gelu(up), dtype), to_f32(w_down, dtype), dtype)
        out = _r(out + mlp, dtype)
    new = _r(hid + _r(np.float32(0.01) * out, dtype), dtype)
    return from_f32(new, dtype), selected_chunks
