"""Mini hybrid decode block on the B200 kernels.

Mirrors ``MiniCSADecodeBlock`` of hybrid_attention/model_inference.py:14-76
(same constructor, parameter names, forward signature and residual form
``hidden + 0.01 * (out_proj(attn) + down_proj(gelu(up_proj(hidden))))``), with
the attention and the dynamic chunk selection running on this package's sm_100a
kernels.  The projections are plain library GEMVs (torch / cuBLAS).

Backends: ``"cuda-csa"`` and ``"cuda-csa-tiled"`` as in the reference
(model_inference.py:60-63).  The reference's ``"torch-full"`` / ``"torch-csa"``
backends are its CPU/torch oracle and have no counterpart here: asking for
them raises ``ValueError``.

``variant="rmsnorm_silu"`` is the block BASELINE config 3 describes (RMSNorm
in front of a SiLU MLP); the default ``"reference"`` is the reference's own
GELU block without a norm, which is what parity is checked against.

``DecodeStepGraph`` captures one whole decode step (q projection, chunk
selection, decode, output projection and MLP) in a CUDA graph, so a step costs
one graph launch instead of a dozen kernel launches.
"""

from __future__ import annotations

import torch
from torch import nn

from . import extension as ext

BACKENDS = ("cuda-csa", "cuda-csa-tiled")
VARIANTS = ("reference", "rmsnorm_silu")


class MiniCSADecodeBlock(nn.Module):
    """Tiny decode block that routes its attention through the B200 CSA kernels."""

    def __init__(self, *, heads: int, head_dim: int, dtype: torch.dtype, device: torch.device,
                 mlp_ratio: float, variant: str = "reference") -> None:
        super().__init__()
        if variant not in VARIANTS:
            raise ValueError(f"unknown variant: {variant}")
        self.heads = heads
        self.head_dim = head_dim
        self.hidden_dim = heads * head_dim
        self.variant = variant
        self.q_proj = nn.Linear(self.hidden_dim, self.hidden_dim, bias=False, device=device, dtype=dtype)
        self.out_proj = nn.Linear(self.hidden_dim, self.hidden_dim, bias=False, device=device, dtype=dtype)
        mlp_dim = int(self.hidden_dim * mlp_ratio)
        self.use_mlp = mlp_dim > 0
        if self.use_mlp:
            self.up_proj = nn.Linear(self.hidden_dim, mlp_dim, bias=False, device=device, dtype=dtype)
            self.down_proj = nn.Linear(mlp_dim, self.hidden_dim, bias=False, device=device, dtype=dtype)
        if variant == "rmsnorm_silu":
            self.norm = nn.RMSNorm(self.hidden_dim, eps=1e-6, device=device, dtype=dtype)

    def _mlp(self, hidden: torch.Tensor) -> torch.Tensor:
        if self.variant == "rmsnorm_silu":
            return self.down_proj(torch.nn.functional.silu(self.up_proj(self.norm(hidden))))
        return self.down_proj(torch.nn.functional.gelu(self.up_proj(hidden)))

    def forward(self, hidden: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                selected_chunks: torch.Tensor | None, *, backend: str, chunk_size: int, top_k: int,
                tile_size: int = 8) -> torch.Tensor:
        if backend not in BACKENDS:
            raise ValueError(f"unknown backend: {backend} (this block runs {', '.join(BACKENDS)})")
        batch = hidden.shape[0]
        q = self.q_proj(hidden).view(batch, self.heads, self.head_dim)
        if selected_chunks is None:  # dynamic selection (model_inference.py:52-53), on the GPU scorer
            selected_chunks = ext.select_topk_chunks(q, k_cache, chunk_size, top_k)
        if backend == "cuda-csa":
            attn = ext.csa_decode_forward(q, k_cache, v_cache, selected_chunks, chunk_size)
        else:
            attn = ext.csa_decode_forward_tiled(q, k_cache, v_cache, selected_chunks, chunk_size, tile_size)
        out = self.out_proj(attn.reshape(batch, self.hidden_dim))
        if self.use_mlp:
            out = out + self._mlp(hidden)
        return hidden + 0.01 * out


def run_decode(block: MiniCSADecodeBlock, hidden: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
               selected_chunks: torch.Tensor | None, *, backend: str, chunk_size: int, top_k: int,
               steps: int, tile_size: int = 8) -> torch.Tensor:
    """``steps`` decode steps feeding each output back as the next input
    (model_inference.py:118-138); ``selected_chunks=None`` selects every step."""
    for _ in range(steps):
        hidden = block(hidden, k_cache, v_cache, selected_chunks, backend=backend, chunk_size=chunk_size,
                       top_k=top_k, tile_size=tile_size)
    return hidden


class DecodeStepGraph:
    """One decode step of ``block`` captured in a CUDA graph.

    ``step(hidden)`` copies ``hidden`` into the graph's static input, replays the
    graph and returns the static output (overwritten by the next step).  The
    caches and the selection mode are fixed at capture time.
    """

    def __init__(self, block: MiniCSADecodeBlock, hidden: torch.Tensor, k_cache: torch.Tensor,
                 v_cache: torch.Tensor, selected_chunks: torch.Tensor | None, *, backend: str, chunk_size: int,
                 top_k: int, tile_size: int = 8) -> None:
        self._static_in = hidden.clone()
        kw = dict(backend=backend, chunk_size=chunk_size, top_k=top_k, tile_size=tile_size)
        stream = torch.cuda.Stream(device=hidden.device)
        stream.wait_stream(torch.cuda.current_stream(hidden.device))
        with torch.no_grad(), torch.cuda.stream(stream):
            for _ in range(2):  # warm-up on the capture stream: workspaces are allocated outside the graph
                block(self._static_in, k_cache, v_cache, selected_chunks, **kw)
            torch.cuda.current_stream(hidden.device).synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=stream):
                self._static_out = block(self._static_in, k_cache, v_cache, selected_chunks, **kw)
        torch.cuda.current_stream(hidden.device).wait_stream(stream)

    def step(self, hidden: torch.Tensor) -> torch.Tensor:
        self._static_in.copy_(hidden)
        self.graph.replay()
        return self._static_out
