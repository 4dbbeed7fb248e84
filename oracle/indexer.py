"""CPU restatement of the DSV4 compressed-slot indexer (TEST INFRASTRUCTURE ONLY).

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline legs may
use this module; the product path never does.

The reference has no indexer of its own: its DSV4 decode receives the
compressed-slot indices from its caller
(integrations/sglang_dsv4/csahca_sglang_dsv4_patch/patch.py:336-341) and lists an
on-device indexer as future work (docs/dsv4_abi_status.md:111-119).  This file
restates the published definition the GPU kernel implements, the lightning
indexer of the DeepSeek-V3.2 technical report ("DeepSeek Sparse Attention"):

    I[t, s] = sum_j w[t, j] * ReLU(q[t, j, :] . k[s, :])

followed by the top-k slots of I[t, :] (largest first; equal scores by lower
slot, as the CSA selection orders them; -1 past the query's valid slots).
Parity is therefore anchored on this definition, not on reference outputs.
Dot products and the weighted sum are fp32 on bf16 inputs.
"""

from __future__ import annotations

import numpy as np

from .csa import topk_lower_index
from .numerics import to_f32


def index_scores(q: np.ndarray, w: np.ndarray, keys: np.ndarray) -> np.ndarray:
    """fp32 ``[Q, N]`` index scores; ``q`` bf16 bits ``[Q, H, D]``, ``w`` fp32
    ``[Q, H]``, ``keys`` bf16 bits ``[Q, N, D]``."""
    qf = to_f32(q, "bf16")
    kf = to_f32(keys, "bf16")
    dots = np.einsum("qhd,qnd->qnh", qf, kf, dtype=np.float32)
    return np.einsum("qnh,qh->qn", np.maximum(dots, 0.0), w.astype(np.float32), dtype=np.float32)


def indexer_topk(q: np.ndarray, w: np.ndarray, keys: np.ndarray, top_k: int,
                 key_lens: np.ndarray | None = None) -> np.ndarray:
    """int32 ``[Q, min(top_k, N)]`` selected slots (-1 past each query's valid count)."""
    nq, n = keys.shape[0], keys.shape[1]
    k = min(top_k, n)
    scores = index_scores(q, w, keys)
    out = np.full((nq, k), -1, np.int32)
    for t in range(nq):
        valid = n if key_lens is None else max(0, min(int(key_lens[t]), n))
        if valid:
            sel = topk_lower_index(scores[t, :valid], min(k, valid))
            out[t, : sel.shape[0]] = sel
    return out
