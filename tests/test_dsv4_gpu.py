"""DSV4 paged-FP8 decode on the GPU against the CPU oracle.

Contract: outputs within 2e-2 absolute / 1e-2 relative of the fp32 oracle
(hybrid_attention/dsv4_correctness.py:91-141) for bf16 q; the same bound is
used for fp16 / fp32 q.
"""

import math

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from helpers import to_torch
from oracle import dsv4
from oracle.numerics import from_f32, to_f32

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2
SCALE = 1.0 / math.sqrt(512)


def _ext():
    from csahca_b200 import extension

    return extension


def _t(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


@pytest.mark.parametrize("name", ["dsv4_c0", "dsv4_c4", "dsv4_c128", "dsv4_c0_f32q"])
@pytest.mark.parametrize("sink", [True, False])
@pytest.mark.parametrize("tiled", ["1", "0"])
@pytest.mark.parametrize("split", ["1", "0"])
def test_golden_cases(cuda, name, sink, tiled, split, monkeypatch):
    """``split``: few queries are split over several CTAs and merged (default)
    or decoded one CTA per query (CSAHCA_DSV4_SPLIT=0)."""
    if tiled == "0" and not sink:
        pytest.skip("the reference's non-tiled entries reject an absent sink (empty tensor, numel != heads)")
    monkeypatch.setenv("CSAHCA_DSV4_TILED", tiled)
    monkeypatch.setenv("CSAHCA_DSV4_SPLIT", split)
    z = np.load(GOLDEN / f"{name}.npz")
    dt = str(z["dtype"])
    page = int(z["meta"][4])
    q = to_torch(z["q"], dt, cuda)
    cache = _t(z["cache"], cuda)
    ti, tl = _t(z["token_indices"], cuda), _t(z["topk_lengths"], cuda)
    sk = _t(z["attn_sink"], cuda) if sink else None
    ext = _ext()
    if "x_cache" in z:
        out = ext.dsv4_sparse_decode_forward(q, cache, ti, tl, _t(z["x_cache"], cuda), _t(z["x_idx"], cuda),
                                             _t(z["x_len"], cuda), sk, page, int(z["extra_page_size"]),
                                             float(z["softmax_scale"]))
    else:
        out = ext.dsv4_swa_decode_forward(q, cache, ti, tl, sk, page, float(z["softmax_scale"]))
    ref = z["out"] if sink else z["out_nosink"]
    np.testing.assert_allclose(out.float().cpu().numpy(), to_f32(ref, dt), atol=ATOL, rtol=RTOL)


def _case(seed, nq, heads, ntok, nmain, page, *, xtok=0, nextra=0, xpage=1, qdtype="bf16", lens=True,
          neg_frac=0.0):
    rng = np.random.default_rng(seed)
    toks = from_f32(rng.standard_normal((ntok, 512)).astype(np.float32), "bf16")
    cache = dsv4.pack_dsv4_cache(toks, page_size=page)
    idx = rng.integers(0, ntok, size=(nq, nmain)).astype(np.int32)
    if neg_frac:
        idx[rng.random(idx.shape) < neg_frac] = -1
    tl = rng.integers(0, nmain + 3, size=nq).astype(np.int32) if lens else None
    c = dict(q=from_f32(rng.standard_normal((nq, heads, 512)).astype(np.float32), qdtype), cache=cache, idx=idx,
             tl=tl, sink=rng.standard_normal(heads).astype(np.float32), page=page, qdtype=qdtype)
    if xtok:
        xt = from_f32((rng.standard_normal((xtok, 512)) * 0.5).astype(np.float32), "bf16")
        c.update(xcache=dsv4.pack_dsv4_cache(xt, page_size=xpage), xpage=xpage,
                 xidx=rng.integers(-1, xtok, size=(nq, nextra)).astype(np.int32),
                 xl=rng.integers(0, nextra + 1, size=nq).astype(np.int32))
    return c


def _run(c, cuda, sink=True):
    q = to_torch(c["q"], c["qdtype"], cuda)
    args = [q, _t(c["cache"], cuda), _t(c["idx"], cuda), None if c["tl"] is None else _t(c["tl"], cuda)]
    sk = _t(c["sink"], cuda) if sink else None
    if "xcache" in c:
        return _ext().dsv4_sparse_decode_forward(*args, _t(c["xcache"], cuda), _t(c["xidx"], cuda),
                                                 _t(c["xl"], cuda), sk, c["page"], c["xpage"], SCALE)
    return _ext().dsv4_swa_decode_forward(*args, sk, c["page"], SCALE)


def _ref(c, sink=True, rows=None):
    rows = slice(None) if rows is None else rows
    kw = {}
    if "xcache" in c:
        kw = dict(extra_cache=c["xcache"], extra_token_indices=c["xidx"][rows], extra_topk_lengths=c["xl"][rows],
                  extra_page_size=c["xpage"])
    return dsv4.reference_attention(c["q"][rows], c["qdtype"], c["cache"], c["idx"][rows],
                                    None if c["tl"] is None else c["tl"][rows], c["sink"] if sink else None,
                                    page_size=c["page"], softmax_scale=SCALE, **kw)


def _check(out, ref, qdtype, rows=None):
    o = out.float().cpu().numpy()
    if rows is not None:
        o = o[rows]
    np.testing.assert_allclose(o, to_f32(ref, qdtype), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("heads", [8, 16, 64, 96, 128])
@pytest.mark.parametrize("split", ["1", "0"])
def test_head_counts(cuda, heads, split, monkeypatch):
    monkeypatch.setenv("CSAHCA_DSV4_SPLIT", split)
    c = _case(1, 5, heads, 700, 300, 64, neg_frac=0.1)  # >= 256 slots: the split path is taken
    _check(_run(c, cuda), _ref(c), "bf16")


@pytest.mark.parametrize("qdtype", ["f16", "f32"])
def test_q_dtypes(cuda, qdtype):
    c = _case(2, 4, 64, 500, 150, 64, qdtype=qdtype)
    _check(_run(c, cuda), _ref(c), qdtype)


@pytest.mark.parametrize("sink", [True, False])
def test_extra_cache_many_blocks(cuda, sink):
    """5 blocks of 128 slots per query (main 512 + extra 64) across both caches."""
    c = _case(3, 6, 64, 2048, 512, 64, xtok=256, nextra=64, xpage=16, neg_frac=0.05)
    c["tl"][:] = 512
    _check(_run(c, cuda, sink), _ref(c, sink), "bf16")


def test_lengths_absent_and_empty_queries(cuda):
    c = _case(4, 6, 64, 300, 40, 64, lens=False)
    _check(_run(c, cuda), _ref(c), "bf16")
    c = _case(5, 4, 64, 300, 40, 64)
    c["tl"][:] = [0, 40, -3, 1]
    c["idx"][1, :] = -1
    out = _run(c, cuda)
    _check(out, _ref(c), "bf16")
    assert (out[0] == 0).all() and (out[1] == 0).all() and (out[2] == 0).all()


def test_online_softmax_rebase(cuda):
    """Later blocks score far higher than earlier ones, forcing the running-max re-base of O."""
    rng = np.random.default_rng(6)
    nq, heads, nmain = 2, 64, 640
    base = rng.standard_normal((nmain, 512)).astype(np.float32)
    ramp = np.repeat(np.linspace(0.2, 4.0, 5), 128)[:, None].astype(np.float32)
    q = rng.standard_normal((nq, heads, 512)).astype(np.float32)
    toks = base * ramp + np.sign(q[0].mean(0))[None, :] * ramp * 0.5
    cache = dsv4.pack_dsv4_cache(from_f32(toks, "bf16"), page_size=64)
    c = dict(q=from_f32(q, "bf16"), cache=cache, idx=np.tile(np.arange(nmain, dtype=np.int32), (nq, 1)),
             tl=np.full(nq, nmain, np.int32), sink=rng.standard_normal(heads).astype(np.float32), page=64,
             qdtype="bf16")
    _check(_run(c, cuda), _ref(c), "bf16")


def test_page_table_permutation_and_page_sizes(cuda):
    """Absolute slot indices through a permuted page table; C128-style page_size 1 extra cache."""
    rng = np.random.default_rng(7)
    page, ntok = 64, 64 * 12
    perm = rng.permutation(12)
    toks = from_f32(rng.standard_normal((ntok, 512)).astype(np.float32), "bf16")
    cache = np.zeros((12, dsv4.bytes_per_page(page)), np.uint8)
    logical = np.arange(ntok)
    locs = perm[logical // page] * page + logical % page
    dsv4.pack_tokens_at(cache, locs, toks, page_size=page)
    nq = 3
    idx = locs[rng.integers(0, ntok, size=(nq, 128))].astype(np.int32)
    xt = from_f32(rng.standard_normal((32, 512)).astype(np.float32), "bf16")
    c = dict(q=from_f32(rng.standard_normal((nq, 64, 512)).astype(np.float32), "bf16"), cache=cache, idx=idx,
             tl=np.full(nq, 128, np.int32), sink=rng.standard_normal(64).astype(np.float32), page=page,
             qdtype="bf16", xcache=dsv4.pack_dsv4_cache(xt, page_size=1), xpage=1,
             xidx=rng.integers(0, 32, size=(nq, 16)).astype(np.int32), xl=np.full(nq, 16, np.int32))
    _check(_run(c, cuda), _ref(c), "bf16")


def test_out_of_range_slot_is_skipped_and_flagged(cuda):
    from csahca_b200 import _native

    _native.read_device_error()
    c = _case(8, 2, 64, 256, 16, 64)
    c["tl"][:] = 16
    c["idx"][0, 3] = 10_000_000
    out = _run(c, cuda)
    assert _native.read_device_error() == 2
    c2 = dict(c)
    c2["idx"] = c["idx"].copy()
    c2["idx"][0, 3] = -1
    _check(out, _ref(c2), "bf16")


def test_large_batch_subset(cuda):
    """256 queries x 64 heads (the config-5 batch) over a shared cache; 8 queries checked."""
    c = _case(9, 256, 64, 4096, 512, 64, xtok=1024, nextra=64, xpage=16)
    c["tl"][:] = 512
    out = _run(c, cuda)
    rows = np.array([0, 1, 77, 128, 200, 253, 254, 255])
    _check(out, _ref(c, rows=rows), "bf16", rows=rows)
    out2 = _run(c, cuda)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


def test_capturable_in_cuda_graph(cuda):
    c = _case(10, 16, 64, 1024, 256, 64)
    ref = _run(c, cuda)
    torch.cuda.synchronize()
    q = to_torch(c["q"], "bf16", cuda)
    cache, idx, tl, sk = _t(c["cache"], cuda), _t(c["idx"], cuda), _t(c["tl"], cuda), _t(c["sink"], cuda)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = _ext().dsv4_swa_decode_forward(q, cache, idx, tl, sk, 64, SCALE)
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("split", ["1", "0"])
def test_extra_slots_only_and_empty_main(cuda, split, monkeypatch):
    """Queries whose main list is empty (length 0 or all -1) but whose compressed
    list is not, next to queries with both lists empty."""
    monkeypatch.setenv("CSAHCA_DSV4_SPLIT", split)
    c = _case(6, 5, 64, 400, 96, 64, xtok=300, nextra=40, xpage=16)
    c["tl"][:] = [0, 96, 0, 5, 0]
    c["idx"][2, :] = -1
    c["xl"][:] = [40, 0, 17, 0, 0]
    out = _run(c, cuda)
    _check(out, _ref(c), "bf16")
    assert (out[4] == 0).all()
