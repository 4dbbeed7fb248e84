"""Request / head / query partitioning of batched decodes over ranks.

CPU: the greedy length split balances config 2's batch; two gloo ranks each
decode their share with the oracle standing in for the kernels, the shares are
reassembled with ``gather_rows``, and the result equals the one-rank decode of
the whole batch (CSA by request and by head, DSV4 by query)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from csahca_b200 import partition as P
from csahca_b200 import workloads as W
from helpers import to_numpy
from oracle import csa, dsv4
from oracle.numerics import to_f32


def test_length_split_covers_every_request_once_and_balances_config2():
    lens = W.csa_request_lengths(batch=64, seq_len=32768, chunk=64, min_len=4096, seed=0)
    for world in (1, 2, 3, 4, 8):
        shares = P.shard_requests_by_length(lens, world)
        assert sorted(i for s in shares for i in s) == list(range(64))
        assert P.imbalance(lens, shares) < 1.03, (world, P.imbalance(lens, shares))
    assert P.shard_requests_by_length([5, 5, 5], 2) == [[0, 2], [1]]
    assert P.shard_requests_by_length([1, 2], 4) == [[1], [0], [], []]


def test_head_and_query_ranges_tile_the_whole():
    for n, world in ((8, 8), (8, 3), (256, 8), (128, 5)):
        got = [P.shard_range(n, r, world) for r in range(world)]
        assert got[0][0] == 0 and got[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
        assert max(h - lo for lo, h in got) - min(h - lo for lo, h in got) <= 1
    assert P.shard_queries(10, 1, 4) == [2, 3, 4]


CSA_KW = dict(batch=5, heads=3, seq_len=512, head_dim=64, chunk=64, top_k=3, min_len=128, seed=11)
DSV4_KW = dict(num_queries=5, heads=8, context=512, page_size=16, n_main=24, ratio=4, n_extra=6, seed=5)


def _csa_oracle(b: W.CsaBatch) -> np.ndarray:
    qn, kn, vn = (to_numpy(t) for t in (b.q, b.k, b.v))
    lens = b.seq_lens.numpy()
    sel = csa.select_topk_chunks_ragged(qn, kn, lens, b.chunk, b.top_k, "bf16")
    return to_f32(csa.csa_decode_skipping(qn, kn, vn, sel, b.chunk, "bf16"), "bf16")


def _dsv4_oracle(b: W.Dsv4Batch) -> np.ndarray:
    return to_f32(dsv4.reference_attention(
        to_numpy(b.q), "bf16", b.cache.numpy(), b.token_indices.numpy(), b.topk_lengths.numpy(),
        b.attn_sink.numpy(), page_size=b.page_size, softmax_scale=b.softmax_scale, extra_cache=b.extra_cache.numpy(),
        extra_token_indices=b.extra_token_indices.numpy(), extra_topk_lengths=b.extra_topk_lengths.numpy(),
        extra_page_size=b.extra_page_size), "bf16")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    # CSA, by request: this rank builds and decodes only its share
    lens = W.csa_request_lengths(batch=CSA_KW["batch"], seq_len=CSA_KW["seq_len"], chunk=CSA_KW["chunk"],
                                 min_len=CSA_KW["min_len"], seed=CSA_KW["seed"])
    mine = P.shard_requests_by_length(lens, world)[rank]
    share = W.csa_batched("cpu", requests=mine, **CSA_KW)
    by_req = P.gather_rows(torch.from_numpy(_csa_oracle(share)), mine, CSA_KW["batch"])
    # CSA, by head (one request): heads [lo, hi) of q, K and V
    one = W.csa_batched("cpu", requests=[0], **CSA_KW)
    lo, hi = P.shard_heads(CSA_KW["heads"], rank, world)
    sl = W.CsaBatch(one.q[:, lo:hi].contiguous(), one.k[:, lo:hi].contiguous(), one.v[:, lo:hi].contiguous(),
                    one.seq_lens, one.chunk, one.top_k)
    by_head = P.gather_rows(torch.from_numpy(_csa_oracle(sl)[0]), list(range(lo, hi)), CSA_KW["heads"])
    # DSV4, by query
    qs = P.shard_queries(DSV4_KW["num_queries"], rank, world)
    by_query = P.gather_rows(torch.from_numpy(_dsv4_oracle(W.dsv4_cache("cpu", queries=qs, **DSV4_KW))), qs,
                             DSV4_KW["num_queries"])
    np.savez(f"{out_path}.{rank}.npz", by_req=by_req.numpy(), by_head=by_head.numpy(), by_query=by_query.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_reassemble_the_one_rank_decode(tmp_path):
    world, port = 2, _free_port()
    mp.start_processes(_rank, args=(world, port, str(tmp_path / "out")), nprocs=world, start_method="spawn")
    full_csa = _csa_oracle(W.csa_batched("cpu", **CSA_KW))
    full_dsv4 = _dsv4_oracle(W.dsv4_cache("cpu", **DSV4_KW))
    for r in range(world):
        z = np.load(tmp_path / f"out.{r}.npz")
        np.testing.assert_array_equal(z["by_req"], full_csa)
        np.testing.assert_array_equal(z["by_head"], full_csa[0])
        np.testing.assert_array_equal(z["by_query"], full_dsv4)
