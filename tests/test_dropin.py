"""The drop-in, shown end to end: the reference's own Python layer
(``hybrid_attention.extension`` and ``hybrid_attention.model_inference``,
unmodified) running on this package's kernels.

The reference imports its native module as ``import hybrid_attention_cuda``
(hybrid_attention/extension.py:13-45).  Registering
``csahca_b200.hybrid_attention_cuda`` under that name, as a deployment would,
routes every op of the reference's wrappers through our C ABI.

The reference package is looked up where the reference arm installs it
(``baseline/_ref``, a pip install of the reference with its compiled module
removed) or at ``$CSAHCA_REFERENCE_PATH``; the tests skip when it is absent.
Also: the argument-check messages of the drop-in on CUDA tensors (shape, dtype
and size mismatches), which must equal the reference's TORCH_CHECK texts.
"""

from __future__ import annotations

import importlib
import math
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import GOLDEN, ROOT
from helpers import to_torch
from oracle.numerics import to_f32

ATOL, RTOL = 2e-2, 1e-2


def _reference_root() -> Path | None:
    for cand in (os.environ.get("CSAHCA_REFERENCE_PATH"), str(ROOT / "baseline" / "_ref")):
        if cand and (Path(cand) / "hybrid_attention" / "extension.py").exists():
            return Path(cand)
    return None


@pytest.fixture
def reference(monkeypatch):
    """The reference's ``hybrid_attention`` package with ``hybrid_attention_cuda``
    aliased to this package's drop-in module."""
    root = _reference_root()
    if root is None:
        pytest.skip("reference Python package not installed (baseline/_ref)")
    from csahca_b200 import hybrid_attention_cuda as ours

    monkeypatch.setitem(sys.modules, "hybrid_attention_cuda", ours)
    monkeypatch.syspath_prepend(str(root))
    for name in [n for n in sys.modules if n == "hybrid_attention" or n.startswith("hybrid_attention.")]:
        monkeypatch.delitem(sys.modules, name)
    ext = importlib.import_module("hybrid_attention.extension")
    mi = importlib.import_module("hybrid_attention.model_inference")
    assert Path(ext.__file__).resolve().is_relative_to(root.resolve())
    ext._CUDA_MODULE = None
    return ext, mi, ours


def test_reference_wrappers_load_our_module_and_keep_its_errors(reference):
    """CPU: the reference loader returns our module, sees the tiled DSV4 entry,
    and its wrappers surface our (= the reference's) error messages."""
    ext, _, ours = reference
    assert ext.load_cuda_extension() is ours
    assert ext._dsv4_tiled_enabled(ours)
    q = torch.zeros(1, 2, 64, dtype=torch.bfloat16)
    kv = torch.zeros(1, 2, 128, 64, dtype=torch.bfloat16)
    idx = torch.zeros(1, 2, 1, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="all tensors must be CUDA tensors"):
        ext.csa_decode_forward_tiled(q, kv, kv, idx, 64)
    with pytest.raises(RuntimeError, match="all tensors must be CUDA tensors"):
        ext.csa_decode_forward(q, kv, kv, idx, 64)
    qd = torch.zeros(1, 8, 512, dtype=torch.bfloat16)
    cache = torch.zeros(1, 37440, dtype=torch.uint8)
    ti = torch.zeros(1, 4, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="q, paged_k_cache_u8, and token_indices must be CUDA tensors"):
        ext.dsv4_swa_decode_forward(qd, cache, ti, None, None, 64, 1 / math.sqrt(512))


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["csa_bf16_small", "csa_f16_small"])
def test_reference_csa_wrappers_on_our_kernels(cuda, reference, name):
    ext, _, _ = reference
    z = np.load(GOLDEN / f"{name}.npz")
    dt = str(z["dtype"])
    c = int(z["meta"][4])
    q, kc, vc = (to_torch(z[n], dt, cuda) for n in ("q", "k", "v"))
    sel = torch.from_numpy(z["selected"]).to(cuda)
    for out in (ext.csa_decode_forward(q, kc, vc, sel, c), ext.csa_decode_forward_tiled(q, kc, vc, sel.long(), c)):
        np.testing.assert_allclose(out.float().cpu().numpy(), to_f32(z["out"], dt), atol=ATOL, rtol=RTOL)


@pytest.mark.gpu
@pytest.mark.parametrize("tiled", ["1", "0"])
def test_reference_dsv4_wrappers_on_our_kernels(cuda, reference, monkeypatch, tiled):
    ext, _, _ = reference
    monkeypatch.setenv("CSAHCA_DSV4_TILED", tiled)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    z = np.load(GOLDEN / "dsv4_c4.npz")
    q = to_torch(z["q"], "bf16", cuda)
    # The reference wrapper accepts a float8 view of the cache bytes too.
    cache = t(z["cache"]).view(torch.float8_e4m3fn)
    out = ext.dsv4_sparse_decode_forward(q, cache, t(z["token_indices"]).long(), t(z["topk_lengths"]),
                                         t(z["x_cache"]), t(z["x_idx"]), t(z["x_len"]), t(z["attn_sink"]),
                                         int(z["meta"][4]), int(z["extra_page_size"]), float(z["softmax_scale"]))
    np.testing.assert_allclose(out.float().cpu().numpy(), to_f32(z["out"], "bf16"), atol=ATOL, rtol=RTOL)
    z0 = np.load(GOLDEN / "dsv4_c0.npz")
    out0 = ext.dsv4_swa_decode_forward(to_torch(z0["q"], "bf16", cuda), t(z0["cache"]), t(z0["token_indices"]),
                                       t(z0["topk_lengths"]), t(z0["attn_sink"]), int(z0["meta"][4]),
                                       float(z0["softmax_scale"]))
    np.testing.assert_allclose(out0.float().cpu().numpy(), to_f32(z0["out"], "bf16"), atol=ATOL, rtol=RTOL)


@pytest.mark.gpu
@pytest.mark.parametrize("backend", ["cuda-csa", "cuda-csa-tiled"])
def test_reference_mini_block_on_our_kernels(cuda, reference, backend):
    """The reference's MiniCSADecodeBlock (its own selection in torch, its own
    projections) with the attention on our kernels, against the outputs the
    reference produced with its own torch path."""
    _, mi, _ = reference
    z = np.load(GOLDEN / "mini_block.npz")
    heads, head_dim, seq_len, chunk, top_k, steps = (int(x) for x in z["meta"])
    bf = lambda a: torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16).to(cuda)  # noqa: E731
    blk = mi.MiniCSADecodeBlock(heads=heads, head_dim=head_dim, dtype=torch.bfloat16, device=cuda,
                                mlp_ratio=2.0).eval()
    with torch.no_grad():
        blk.q_proj.weight.copy_(bf(z["w_q"]))
        blk.out_proj.weight.copy_(bf(z["w_o"]))
        blk.up_proj.weight.copy_(bf(z["w_up"]))
        blk.down_proj.weight.copy_(bf(z["w_down"]))
        h, k, v = bf(z["hidden"]), bf(z["k"]), bf(z["v"])
        for i in range(steps):
            h = blk(h, k, v, None, backend=backend, chunk_size=chunk, top_k=top_k, tile_size=8)
            np.testing.assert_allclose(h.float().cpu().numpy(), to_f32(z["outs"][i], "bf16"), atol=ATOL, rtol=RTOL)


# --------------------------------------------------------------------------- error contract on CUDA tensors
@pytest.mark.gpu
def test_csa_checks_on_cuda_tensors(cuda):
    from csahca_b200 import hybrid_attention_cuda as m

    q = torch.zeros(2, 4, 64, device=cuda, dtype=torch.bfloat16)
    kv = torch.zeros(2, 4, 256, 64, device=cuda, dtype=torch.bfloat16)
    idx = torch.zeros(2, 4, 3, device=cuda, dtype=torch.int32)
    cases = [
        ((q, kv[:, :3].contiguous(), kv[:, :3].contiguous(), idx, 64), "KV cache shape must match q"),
        ((q, kv, kv[..., :32].contiguous(), idx, 64), "v_cache must match k_cache shape"),
        ((q, kv, kv, idx.float(), 64), "chunk_indices must be int32 or int64"),
        ((q, kv.float(), kv, idx, 64), "q and k_cache dtype must match"),
        ((q, kv, kv, idx[:1].contiguous(), 64), "chunk_indices batch/head dimensions must match q"),
        ((q, kv, kv, idx, 0), "chunk_size must be positive"),
        ((q[0], kv, kv, idx, 64), r"q must be \[batch, heads, head_dim\]"),
        ((q, kv.transpose(2, 3), kv, idx, 64), "k_cache must be contiguous"),
        ((q.to(torch.int32), kv.to(torch.int32), kv.to(torch.int32), idx, 64), "not implemented for"),
    ]
    for args, msg in cases:
        with pytest.raises(RuntimeError, match=msg):
            m.csa_decode_forward(*args)
    with pytest.raises(RuntimeError, match="tile_size must be positive"):
        m.csa_decode_forward_tiled(q, kv, kv, idx, 64, 0)
    with pytest.raises(RuntimeError, match="all tensors must be CUDA tensors"):
        m.csa_decode_forward_tiled(q, kv, kv, idx.cpu(), 64, 8)


@pytest.mark.gpu
def test_dsv4_checks_on_cuda_tensors(cuda):
    from csahca_b200 import hybrid_attention_cuda as m

    z = np.load(GOLDEN / "dsv4_c4.npz")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    q = to_torch(z["q"], "bf16", cuda)
    cache, ti, tl, sink = t(z["cache"]), t(z["token_indices"]), t(z["topk_lengths"]), t(z["attn_sink"])
    xc, xi, xl = t(z["x_cache"]), t(z["x_idx"]), t(z["x_len"])
    page, xpage, scale = int(z["meta"][4]), int(z["extra_page_size"]), float(z["softmax_scale"])
    swa = lambda *a: m.dsv4_swa_decode_forward(*a)  # noqa: E731
    cases = [
        (lambda: swa(q, cache[:, :100].contiguous(), ti, tl, sink, page, scale),
         "bytes_per_page is too small for DSV4 page layout"),
        (lambda: swa(q[..., :256].contiguous(), cache, ti, tl, sink, page, scale), "q head_dim must be 512 for DSV4"),
        (lambda: swa(q, cache, ti.long(), tl, sink, page, scale), "token_indices must be int32"),
        (lambda: swa(q, cache.view(torch.int8), ti, tl, sink, page, scale), "paged_k_cache_u8 must be uint8"),
        (lambda: swa(q, cache, ti, tl[:1].contiguous(), sink, page, scale), "topk_lengths must have one value per query"),
        (lambda: swa(q, cache, ti, tl, sink[:3].contiguous(), page, scale), "attn_sink must have one value per head"),
        (lambda: swa(q, cache, ti[:1].contiguous(), tl, sink, page, scale),
         "token_indices query dimension must match q"),
        (lambda: swa(q, cache.flatten(), ti, tl, sink, page, scale),
         r"paged_k_cache_u8 must be \[num_pages, bytes_per_page\]"),
        (lambda: swa(q, cache, ti, tl, sink, 0, scale), "page_size must be positive"),
        (lambda: m.dsv4_sparse_decode_forward(q, cache, ti, tl, xc[:, :64].contiguous(), xi, xl, sink, page, xpage,
                                              scale), "extra_bytes_per_page is too small for DSV4 page layout"),
        (lambda: m.dsv4_sparse_decode_forward(q, cache, ti, tl, xc, xi.long(), xl, sink, page, xpage, scale),
         "extra_token_indices must be int32"),
        (lambda: m.dsv4_decode_forward_tiled(q, torch.zeros(4, page * 584 + 2, dtype=torch.uint8, device=cuda), ti,
                                             tl, xc, xi, xl, sink, page, xpage, 0, scale),
         "tiled DSV4 kernel requires bytes_per_page divisible by 4"),
    ]
    for fn, msg in cases:
        with pytest.raises(RuntimeError, match=msg):
            fn()
