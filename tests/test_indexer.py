"""DSV4 compressed-slot indexer (lightning-indexer score + top-k) on the GPU
against the CPU restatement of its published definition.

Contract: selected slots bit-exact wherever the oracle's k-th and (k+1)-th
scores (and every adjacent pair above them) are separated by more than fp32
rounding of a differently ordered sum; where they are not, the scores of the
selected slots agree.  Parity is anchored on the published definition (the
reference has no indexer of its own).
"""

import numpy as np
import pytest
import torch

from helpers import to_torch
from oracle import indexer
from oracle.numerics import from_f32


def _case(seed, nq, n, heads=64, d=128):
    rng = np.random.default_rng(seed)
    q = from_f32(rng.standard_normal((nq, heads, d)).astype(np.float32), "bf16")
    keys = from_f32(rng.standard_normal((nq, n, d)).astype(np.float32), "bf16")
    w = (rng.standard_normal((nq, heads)) * 0.1).astype(np.float32)
    return q, w, keys


def test_oracle_definition_small():
    """The oracle equals the formula evaluated term by term."""
    q, w, keys = _case(1, 2, 9, heads=3, d=4)
    from oracle.numerics import to_f32

    qf, kf = to_f32(q, "bf16"), to_f32(keys, "bf16")
    want = np.zeros((2, 9), np.float64)
    for t in range(2):
        for s in range(9):
            want[t, s] = sum(w[t, j] * max(0.0, float(qf[t, j] @ kf[t, s])) for j in range(3))
    np.testing.assert_allclose(indexer.index_scores(q, w, keys), want, rtol=1e-5, atol=1e-6)
    sel = indexer.indexer_topk(q, w, keys, 4, key_lens=np.array([9, 2], np.int32))
    assert sel.shape == (2, 4) and (sel[1, 2:] == -1).all()
    assert list(sel[0]) == list(np.argsort(-want[0], kind="stable")[:4])


def _check(sel, q, w, keys, top_k, lens):
    """Every output position whose oracle score is separated from both
    neighbours in the sorted order must hold the oracle's slot; elsewhere the
    selected slots' scores must agree.  Returns the share of separated positions."""
    ref = indexer.indexer_topk(q, w, keys, top_k, lens)
    scores = indexer.index_scores(q, w, keys)
    separated = total = 0
    for t in range(sel.shape[0]):
        valid = keys.shape[1] if lens is None else int(min(max(lens[t], 0), keys.shape[1]))
        k = min(top_k, valid)
        np.testing.assert_array_equal(sel[t, k:], -1)
        if k == 0:
            continue
        srt = -np.sort(-scores[t, :valid])[: k + 1]
        tol = 1e-5 * np.abs(srt).clip(1e-3)
        gap_after = np.append(srt[:-1] - srt[1:], np.inf)[:k]  # position i vs i+1
        gap_before = np.insert(srt[:-1] - srt[1:], 0, np.inf)[:k]  # position i vs i-1
        iso = (gap_after > tol[:k]) & (gap_before > tol[:k])
        np.testing.assert_array_equal(sel[t, :k][iso], ref[t, :k][iso], err_msg=f"query {t}")
        np.testing.assert_allclose(scores[t, sel[t, :k]], scores[t, ref[t, :k]], rtol=1e-5, atol=1e-5)
        separated += int(iso.sum())
        total += k
    return separated / max(total, 1)


@pytest.mark.gpu
@pytest.mark.parametrize("nq,n,top_k,ragged", [(4, 16384, 64, False), (3, 1000, 16, True), (5, 130, 200, True),
                                                (2, 128, 8, False), (6, 2049, 512, True)])
def test_indexer_matches_oracle(cuda, nq, n, top_k, ragged):
    from csahca_b200 import extension as ext

    q, w, keys = _case(nq * 7 + n, nq, n)
    lens = None
    if ragged:
        lens = np.random.default_rng(n).integers(0, n + 1, nq).astype(np.int32)
        lens[0] = n
        if nq > 2:
            lens[1] = 0
    for _ in range(2):  # the workspace is reused as is
        sel = ext.dsv4_indexer_topk(to_torch(q, "bf16", cuda), torch.from_numpy(w).to(cuda),
                                    to_torch(keys, "bf16", cuda), top_k,
                                    None if lens is None else torch.from_numpy(lens).to(cuda)).cpu().numpy()
        assert _check(sel, q, w, keys, top_k, lens) > 0.9


@pytest.mark.gpu
@pytest.mark.parametrize("nq,n,top_k", [(3, 16384, 512), (2, 16384, 64), (2, 20000, 64), (2, 49152, 100),
                                        (1, 50000, 32), (2, 3000, 600), (2, 700, 700)])
def test_indexer_ties_exact(cuda, nq, n, top_k):
    """Scores that are small integers (exact in fp32 whatever the summation
    order) with heavy ties: the selection must equal the oracle's bit for bit,
    equal scores ordered by the lower slot.  Covers the radix path (its index
    digits are reached only through ties) up to its 49152-slot limit and the
    per-round fallback (more slots, or top_k above 512)."""
    from csahca_b200 import extension as ext

    rng = np.random.default_rng(n + top_k)
    q32 = np.zeros((nq, 64, 128), np.float32)
    q32[:, :, 0] = 1.0
    k32 = np.zeros((nq, n, 128), np.float32)
    k32[:, :, 0] = rng.integers(-3, 4, (nq, n))
    k32[0] = 0.0  # query 0: every score equal
    q, keys = from_f32(q32, "bf16"), from_f32(k32, "bf16")
    w = rng.integers(1, 3, (nq, 64)).astype(np.float32)
    want = indexer.indexer_topk(q, w, keys, top_k)
    got = ext.dsv4_indexer_topk(to_torch(q, "bf16", cuda), torch.from_numpy(w).to(cuda),
                                to_torch(keys, "bf16", cuda), top_k).cpu().numpy()
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(got[0, :min(top_k, n)], np.arange(min(top_k, n)))


@pytest.mark.gpu
def test_indexer_bench_batch(cuda):
    """The bench's own full batch (config 5's shape: 256 queries x 16384 C4
    slots, generated exactly as ``bench.py --workload dsv4_indexer`` does,
    top-64): a spread of queries checked against the oracle with the same
    per-position contract."""
    from csahca_b200 import extension as ext
    from helpers import to_numpy

    g = torch.Generator(device=cuda).manual_seed(5)
    q = torch.randn(256, 64, 128, generator=g, device=cuda).to(torch.bfloat16)
    w = torch.randn(256, 64, generator=g, device=cuda) * 0.1
    keys = torch.randn(256, 16384, 128, generator=g, device=cuda, dtype=torch.bfloat16)
    sel = ext.dsv4_indexer_topk(q, w, keys, 64).cpu().numpy()
    pick = [0, 1, 37, 128, 147, 148, 200, 255]  # score-CTA tile shares cross query boundaries throughout
    share = _check(sel[pick], to_numpy(q[pick]), w[pick].cpu().numpy(), to_numpy(keys[pick]), 64, None)
    assert share > 0.9


@pytest.mark.gpu
def test_indexer_rejects_unsupported_shapes(cuda):
    from csahca_b200 import extension as ext

    q = torch.zeros(1, 32, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(RuntimeError, match="64 heads of dim 128"):
        ext.dsv4_indexer_topk(q, torch.zeros(1, 32, device=cuda), torch.zeros(1, 8, 128, dtype=torch.bfloat16,
                                                                              device=cuda), 4)


def test_indexer_validates_before_any_launch():
    """Shape, dtype and device errors are raised in Python, before the library runs."""
    from csahca_b200 import extension as ext

    q = torch.zeros(2, 64, 128, dtype=torch.bfloat16)
    w = torch.zeros(2, 64)
    keys = torch.zeros(2, 300, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="must be CUDA tensors"):
        ext.dsv4_indexer_topk(q, w, keys, 8)
    with pytest.raises(ValueError, match="bfloat16"):
        ext.dsv4_indexer_topk(q.float(), w, keys, 8)
    with pytest.raises(ValueError, match="dimensions must match"):
        ext.dsv4_indexer_topk(q, w[:1], keys, 8)
