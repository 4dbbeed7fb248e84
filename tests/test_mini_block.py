"""Mini decode block (hybrid_attention/model_inference.py:14-76): the CPU
restatement against the reference's own outputs, and the B200 block against
both (GPU)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import mini_block
from oracle.numerics import to_f32

ATOL, RTOL = 2e-2, 1e-2


def _golden():
    z = np.load(GOLDEN / "mini_block.npz")
    heads, head_dim, seq_len, chunk, top_k, steps = (int(x) for x in z["meta"])
    return z, heads, head_dim, seq_len, chunk, top_k, steps


def test_oracle_block_matches_reference_outputs():
    z, heads, head_dim, seq_len, chunk, top_k, steps = _golden()
    h = z["hidden"]
    for i in range(steps):
        h, _ = mini_block.block_forward(h, z["k"], z["v"], z["w_q"], z["w_o"], z["w_up"], z["w_down"],
                                        chunk_size=chunk, top_k=top_k, dtype="bf16")
        np.testing.assert_allclose(to_f32(h, "bf16"), to_f32(z["outs"][i], "bf16"), atol=ATOL, rtol=RTOL)


@pytest.mark.gpu
@pytest.mark.parametrize("backend", ["cuda-csa", "cuda-csa-tiled"])
def test_b200_block_matches_reference_outputs(cuda, backend):
    from csahca_b200.model_inference import MiniCSADecodeBlock, run_decode

    z, heads, head_dim, seq_len, chunk, top_k, steps = _golden()
    bf = lambda a: torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16).to(cuda)  # noqa: E731
    blk = MiniCSADecodeBlock(heads=heads, head_dim=head_dim, dtype=torch.bfloat16, device=cuda, mlp_ratio=2.0).eval()
    with torch.no_grad():
        blk.q_proj.weight.copy_(bf(z["w_q"]))
        blk.out_proj.weight.copy_(bf(z["w_o"]))
        blk.up_proj.weight.copy_(bf(z["w_up"]))
        blk.down_proj.weight.copy_(bf(z["w_down"]))
        h = bf(z["hidden"])
        k, v = bf(z["k"]), bf(z["v"])
        for i in range(steps):
            h = run_decode(blk, h, k, v, None, backend=backend, chunk_size=chunk, top_k=top_k, steps=1)
            np.testing.assert_allclose(h.float().cpu().numpy(), to_f32(z["outs"][i], "bf16"), atol=ATOL, rtol=RTOL)


@pytest.mark.gpu
def test_b200_block_selection_and_graph_step(cuda):
    """Dynamic selection on the GPU scorer equals the oracle's on the same q;
    the CUDA-graph step equals the eager step."""
    from csahca_b200 import extension as ext
    from csahca_b200.model_inference import DecodeStepGraph, MiniCSADecodeBlock
    from oracle import csa
    from oracle.numerics import from_f32

    torch.manual_seed(3)
    heads, head_dim, seq_len, chunk, top_k = 8, 128, 8192, 64, 8
    blk = MiniCSADecodeBlock(heads=heads, head_dim=head_dim, dtype=torch.bfloat16, device=cuda, mlp_ratio=2.0,
                             variant="rmsnorm_silu").eval()
    g = torch.Generator(device=cuda).manual_seed(4)
    hidden = torch.randn(1, heads * head_dim, device=cuda, generator=g).to(torch.bfloat16)
    k = torch.randn(1, heads, seq_len, head_dim, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(1, heads, seq_len, head_dim, device=cuda, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        q = blk.q_proj(hidden).view(1, heads, head_dim)
        sel = ext.select_topk_chunks(q, k, chunk, top_k)
        qn = q.float().cpu().numpy()
        kn = from_f32(k.float().cpu().numpy(), "bf16")
        np.testing.assert_array_equal(sel.cpu().numpy(),
                                      csa.select_topk_chunks(from_f32(qn, "bf16"), kn, chunk, top_k, "bf16"))
        kw = dict(backend="cuda-csa-tiled", chunk_size=chunk, top_k=top_k)
        eager = blk(hidden, k, v, None, **kw)
        graph = DecodeStepGraph(blk, hidden, k, v, None, **kw)
        out = graph.step(hidden)
        torch.testing.assert_close(out, eager, atol=0, rtol=0)
        out2 = graph.step(out.clone())
        torch.testing.assert_close(out2, blk(eager, k, v, None, **kw), atol=0, rtol=0)


def test_block_rejects_the_reference_torch_backends():
    """The reference's torch-full / torch-csa backends are its oracle and have no
    counterpart here: asking for them fails before any kernel runs."""
    from csahca_b200.model_inference import MiniCSADecodeBlock

    blk = MiniCSADecodeBlock(heads=2, head_dim=64, dtype=torch.float32, device=torch.device("cpu"), mlp_ratio=2.0)
    h = torch.zeros(1, 128)
    kv = torch.zeros(1, 2, 128, 64)
    for backend in ("torch-full", "torch-csa"):
        with pytest.raises(ValueError, match="unknown backend"):
            blk(h, kv, kv, None, backend=backend, chunk_size=64, top_k=2)
    with pytest.raises(ValueError, match="unknown variant"):
        MiniCSADecodeBlock(heads=2, head_dim=64, dtype=torch.float32, device=torch.device("cpu"), mlp_ratio=0.0,
                           variant="other")
