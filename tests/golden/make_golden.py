"""Generate golden vectors for the oracle from the reference's own PyTorch code.

Run in a container that has the reference checkout (default: a ``reference``
directory beside this repository; override with ``CSAHCA_REFERENCE``):

    python tests/golden/make_golden.py

It imports hybrid_attention.reference and hybrid_attention.dsv4_correctness from
that checkout, runs them on CPU with fixed seeds, and writes ``*.npz`` files next
to this script.  bf16 tensors are stored as uint16 bit patterns.  The fixtures
are committed; the GPU box never needs the reference.
"""

from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("CSAHCA_REFERENCE", str(HERE.parents[2] / "reference")))
sys.path.insert(0, str(REF))

from hybrid_attention import dsv4_correctness as D  # noqa: E402
from hybrid_attention.reference import csa_reference, make_synthetic_case, select_topk_chunks  # noqa: E402


def store(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float8_e4m3fn:
        return t.contiguous().view(torch.uint8).numpy()
    return t.contiguous().numpy()


DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def csa_case(name, *, batch, heads, seq_len, head_dim, chunk, top_k, dtype, seed, keep_inputs=True):
    c = make_synthetic_case(batch=batch, heads=heads, seq_len=seq_len, head_dim=head_dim, chunk_size=chunk,
                            top_k=top_k, dtype=DT[dtype], device="cpu", seed=seed)
    sel = select_topk_chunks(c.q, c.k_cache, chunk, top_k)
    out = csa_reference(c.q, c.k_cache, c.v_cache, chunk_size=chunk, top_k=top_k, selected_chunks=sel)
    arrs = dict(selected=sel.numpy(), out=store(out),
                meta=np.array([batch, heads, seq_len, head_dim, chunk, top_k, seed]),
                dtype=np.array(dtype), k_checksum=np.float64(c.k_cache.double().sum().item()))
    if keep_inputs:
        arrs.update(q=store(c.q), k=store(c.k_cache), v=store(c.v_cache))
    np.savez_compressed(HERE / f"{name}.npz", **arrs)
    print("wrote", name)


def dsv4_case(name, *, num_queries, heads, num_tokens, top_k, page_size, ratio, extra_tokens, extra_top_k, seed,
              dtype="bf16"):
    """Same generator order as dsv4_correctness.main (dsv4_correctness.py:162-227)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    q = torch.randn(num_queries, heads, D.HEAD_DIM, dtype=DT[dtype], generator=g)
    k_tokens = torch.randn(num_tokens, D.HEAD_DIM, dtype=torch.bfloat16, generator=g)
    cache = D.pack_dsv4_cache(k_tokens, page_size=page_size)
    token_indices = torch.randint(0, num_tokens, (num_queries, top_k), dtype=torch.int32, generator=g)
    topk_lengths = torch.randint(max(1, top_k // 2), top_k + 1, (num_queries,), dtype=torch.int32, generator=g)
    attn_sink = torch.randn(heads, dtype=torch.float32, generator=g)
    scale = 1.0 / math.sqrt(D.HEAD_DIM)
    arrs = dict(q=store(q), k_tokens=store(k_tokens), cache=cache.numpy(), token_indices=token_indices.numpy(),
                topk_lengths=topk_lengths.numpy(), attn_sink=attn_sink.numpy(), dtype=np.array(dtype),
                meta=np.array([num_queries, heads, num_tokens, top_k, page_size, ratio, extra_tokens, extra_top_k, seed]),
                softmax_scale=np.float64(scale))
    kw = {}
    if ratio:
        extra_page_size = page_size // ratio
        x_tokens = torch.randn(extra_tokens, D.HEAD_DIM, dtype=torch.bfloat16, generator=g)
        x_cache = D.pack_dsv4_cache(x_tokens, page_size=extra_page_size)
        x_idx = torch.randint(0, extra_tokens, (num_queries, extra_top_k), dtype=torch.int32, generator=g)
        if extra_top_k >= 4:
            x_idx[:, -2:] = -1
        x_len = torch.randint(max(1, extra_top_k // 2), extra_top_k + 1, (num_queries,), dtype=torch.int32, generator=g)
        kw = dict(extra_cache=x_cache, extra_token_indices=x_idx, extra_topk_lengths=x_len,
                  extra_page_size=extra_page_size)
        arrs.update(x_tokens=store(x_tokens), x_cache=x_cache.numpy(), x_idx=x_idx.numpy(), x_len=x_len.numpy(),
                    extra_page_size=np.int64(extra_page_size))
    out = D.reference_attention(q, cache, token_indices, topk_lengths, attn_sink, page_size=page_size,
                                softmax_scale=scale, **kw)
    out_nosink = D.reference_attention(q, cache, token_indices, topk_lengths, None, page_size=page_size,
                                       softmax_scale=scale, **kw)
    arrs.update(out=store(out), out_nosink=store(out_nosink))
    np.savez_compressed(HERE / f"{name}.npz", **arrs)
    print("wrote", name)


def mini_block_case(name, *, heads, head_dim, seq_len, chunk, top_k, mlp_ratio, seed, steps):
    """``steps`` dynamic-selection decode steps of the reference block
    (model_inference.py MiniCSADecodeBlock, backend "torch-csa") on CPU in bf16."""
    from hybrid_attention.model_inference import MiniCSADecodeBlock

    torch.manual_seed(seed)
    blk = MiniCSADecodeBlock(heads=heads, head_dim=head_dim, dtype=torch.bfloat16, device=torch.device("cpu"),
                             mlp_ratio=mlp_ratio).eval()
    g = torch.Generator().manual_seed(seed + 1)
    hd = heads * head_dim
    hidden = torch.randn(1, hd, generator=g).to(torch.bfloat16)
    k = torch.randn(1, heads, seq_len, head_dim, generator=g).to(torch.bfloat16)
    v = torch.randn(1, heads, seq_len, head_dim, generator=g).to(torch.bfloat16)
    outs = []
    h = hidden
    with torch.no_grad():
        for _ in range(steps):
            h = blk(h, k, v, None, backend="torch-csa", chunk_size=chunk, top_k=top_k, tile_size=8)
            outs.append(store(h))
    arrs = dict(hidden=store(hidden), k=store(k), v=store(v), w_q=store(blk.q_proj.weight),
                w_o=store(blk.out_proj.weight), w_up=store(blk.up_proj.weight), w_down=store(blk.down_proj.weight),
                outs=np.stack(outs), meta=np.array([heads, head_dim, seq_len, chunk, top_k, steps]),
                mlp_ratio=np.float64(mlp_ratio))
    np.savez_compressed(HERE / f"{name}.npz", **arrs)
    print("wrote", name)


def main() -> None:
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    csa_case("csa_bf16_small", batch=1, heads=2, seq_len=512, head_dim=128, chunk=64, top_k=4, dtype="bf16", seed=0)
    csa_case("csa_f16_small", batch=1, heads=2, seq_len=256, head_dim=64, chunk=32, top_k=3, dtype="f16", seed=1)
    csa_case("csa_f32_small", batch=2, heads=1, seq_len=256, head_dim=128, chunk=64, top_k=2, dtype="f32", seed=2)
    # Config 1 at full size; inputs are regenerated from the seed by the tests.
    csa_case("csa_cfg1", batch=1, heads=8, seq_len=32768, head_dim=128, chunk=64, top_k=8, dtype="bf16", seed=0,
             keep_inputs=False)
    dsv4_case("dsv4_c0", num_queries=3, heads=8, num_tokens=256, top_k=32, page_size=64, ratio=0,
              extra_tokens=0, extra_top_k=0, seed=0)
    dsv4_case("dsv4_c4", num_queries=3, heads=8, num_tokens=256, top_k=32, page_size=64, ratio=4,
              extra_tokens=256, extra_top_k=16, seed=1)
    dsv4_case("dsv4_c128", num_queries=2, heads=16, num_tokens=192, top_k=24, page_size=128, ratio=128,
              extra_tokens=64, extra_top_k=8, seed=2)
    dsv4_case("dsv4_c0_f32q", num_queries=2, heads=8, num_tokens=128, top_k=16, page_size=64, ratio=0,
              extra_tokens=0, extra_top_k=0, seed=3, dtype="f32")
    mini_block_case("mini_block", heads=2, head_dim=64, seq_len=1024, chunk=64, top_k=4, mlp_ratio=2.0, seed=0,
                    steps=3)


if __name__ == "__main__":
    main()
