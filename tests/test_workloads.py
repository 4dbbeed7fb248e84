"""The device-side workload generators match the oracle's layout (run on CPU)."""

import numpy as np
import torch

from csahca_b200 import workloads as W
from oracle import dsv4


def test_torch_packer_is_byte_identical_to_oracle():
    g = torch.Generator().manual_seed(0)
    toks = torch.randn(300, 512, generator=g, dtype=torch.bfloat16) * 3
    toks[5] = 0
    data, scales = W.pack_tokens_torch(toks)
    cache = torch.zeros(5, W.bytes_per_page(64), dtype=torch.uint8)
    W.write_rows(cache, 64, torch.arange(300), data, scales)
    ref = dsv4.pack_dsv4_cache(toks.view(torch.int16).numpy().view(np.uint16), page_size=64)
    np.testing.assert_array_equal(cache.numpy(), ref)


def test_dsv4_cache_generator_rows_dequantise_back():
    b = W.dsv4_cache("cpu", num_queries=3, heads=8, context=256, page_size=16, n_main=32, ratio=4, n_extra=8)
    assert b.cache.shape[1] == W.bytes_per_page(16)
    assert (b.token_indices >= 0).all() and b.extra_token_indices.shape == (3, 8)
    rows = dsv4.dequant_dsv4_cache(b.cache.numpy(), b.token_indices.numpy(), page_size=16)
    assert rows.shape == (3, 32, 512) and np.isfinite(rows.view(np.uint16).astype(np.float32)).all()
    c0 = W.dsv4_cache("cpu", num_queries=2, heads=8, context=(200, 300), page_size=64, ratio=0, window=128)
    assert c0.token_indices.shape == (2, 128) and c0.extra_cache is None


def test_csa_batch_shapes_and_bytes():
    b = W.csa_batched("cpu", batch=2, heads=2, seq_len=512, head_dim=64, chunk=64, top_k=4, min_len=128)
    assert b.k.shape == (2, 2, 512, 64) and (b.seq_lens % 64 == 0).all() and (b.seq_lens >= 128).all()
    nb = W.csa_algorithmic_bytes(b)
    assert nb["scorer"] >= int(b.seq_lens.sum()) * 2 * 64 * 2


def test_request_subsets_reproduce_the_full_batch_rows():
    """A rank that builds only its share of a batch gets the same rows as the
    full build (per-request generators), so a sharded run decodes the same job."""
    kw = dict(batch=5, heads=2, seq_len=256, head_dim=32, chunk=64, top_k=2, min_len=64, seed=3)
    full = W.csa_batched("cpu", **kw)
    part = W.csa_batched("cpu", requests=[4, 1], **kw)
    assert part.request_ids == [4, 1]
    for i, r in enumerate([4, 1]):
        assert torch.equal(part.q[i], full.q[r]) and torch.equal(part.k[i], full.k[r])
        assert torch.equal(part.v[i], full.v[r]) and int(part.seq_lens[i]) == int(full.seq_lens[r])
    dk = dict(num_queries=4, heads=8, context=256, page_size=16, n_main=32, ratio=4, n_extra=8, seed=2)
    fd = W.dsv4_cache("cpu", **dk)
    pd = W.dsv4_cache("cpu", queries=[2, 3], **dk)
    for i, r in enumerate([2, 3]):
        assert torch.equal(pd.q[i], fd.q[r])
        a = dsv4.dequant_dsv4_cache(pd.cache.numpy(), pd.token_indices[i].numpy(), page_size=16)
        b = dsv4.dequant_dsv4_cache(fd.cache.numpy(), fd.token_indices[r].numpy(), page_size=16)
        np.testing.assert_array_equal(a, b)
        a = dsv4.dequant_dsv4_cache(pd.extra_cache.numpy(), pd.extra_token_indices[i].numpy(), page_size=4)
        b = dsv4.dequant_dsv4_cache(fd.extra_cache.numpy(), fd.extra_token_indices[r].numpy(), page_size=4)
        np.testing.assert_array_equal(a, b)
