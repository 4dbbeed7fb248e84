"""Chunk-sum cache for the CSA scorer: build / append against torch fp32 sums,
and selection on the cache against the oracle's selection on K."""

import numpy as np
import pytest
import torch

from helpers import to_numpy
from oracle import csa

pytestmark = pytest.mark.gpu


def _ext():
    from csahca_b200 import extension

    return extension


@pytest.mark.parametrize("dtype,b,h", [(torch.bfloat16, 3, 4), (torch.float16, 3, 4), (torch.float32, 3, 4),
                                       (torch.bfloat16, 3, 50)])
def test_build_matches_torch_and_selection_matches_oracle(cuda, dtype, b, h):
    """Few rows (512-thread CTAs) and 150 rows (256-thread CTAs, three per SM)."""
    g = torch.Generator(device=cuda).manual_seed(11)
    s, d, c, k = 64 * 96, 128, 64, 8
    base = torch.randn(b, h, s // c, 1, 1, generator=g, device=cuda) * 0.5
    kc = (torch.randn(b, h, s // c, c, d, generator=g, device=cuda) + base).reshape(b, h, s, d).to(dtype)
    q = torch.randn(b, h, d, generator=g, device=cuda).to(dtype)
    ext = _ext()
    sums = ext.chunk_sums_build(kc, c)
    ref = kc.float().reshape(b, h, s // c, c, d).sum(3)
    torch.testing.assert_close(sums, ref, atol=1e-3, rtol=1e-5)
    lens = torch.tensor([s, 64 * 40, 64 * 7], dtype=torch.int32, device=cuda)[:b]
    sel = ext.select_topk_chunks_from_sums(q, sums, k, lens, chunk_size=c).cpu().numpy()
    dt = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[dtype]
    want = csa.select_topk_chunks_ragged(to_numpy(q), to_numpy(kc), lens.cpu().numpy(), c, k, dt)
    np.testing.assert_array_equal(sel, want)


def test_append_tracks_a_growing_cache(cuda):
    g = torch.Generator(device=cuda).manual_seed(12)
    b, h, s, d, c = 2, 3, 64 * 8, 64, 64
    kc = torch.randn(b, h, s, d, generator=g, device=cuda).to(torch.bfloat16)
    lens = [100, 256]
    for i, n in enumerate(lens):
        kc[i, :, n:] = 0
    ext = _ext()
    sums = ext.chunk_sums_build(kc, c)
    pos = torch.tensor(lens, dtype=torch.int32, device=cuda)
    for _ in range(70):  # crosses chunk boundaries for both requests
        for i in range(b):
            kc[i, :, int(pos[i])] = torch.randn(h, d, generator=g, device=cuda).to(torch.bfloat16)
        ext.chunk_sums_append(kc, sums, pos, c)
        pos += 1
    torch.testing.assert_close(sums, ext.chunk_sums_build(kc, c), atol=1e-3, rtol=1e-5)
    # positions outside the cache are ignored
    before = sums.clone()
    ext.chunk_sums_append(kc, sums, torch.tensor([-1, s], dtype=torch.int32, device=cuda), c)
    torch.testing.assert_close(sums, before, atol=0, rtol=0)
