"""Split-KV DSV4 decode of one long request across ranks.

CPU: the shard-and-merge math of the oracle equals the one-shard oracle, and
the host logic plus the all-gather run as two gloo ranks (the numpy oracle
stands in for the kernels).  GPU: the partial and combine kernels against the
one-shard kernel and the oracle."""

from __future__ import annotations

import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import GOLDEN
from oracle import dsv4
from oracle.numerics import to_f32

ATOL, RTOL = 2e-2, 1e-2


def _golden():
    z = np.load(GOLDEN / "dsv4_c4.npz")
    return dict(q=z["q"], cache=z["cache"], idx=z["token_indices"], tl=z["topk_lengths"], sink=z["attn_sink"],
                page=int(z["meta"][4]), xcache=z["x_cache"], xidx=z["x_idx"], xl=z["x_len"],
                xpage=int(z["extra_page_size"]), scale=float(z["softmax_scale"]), out=z["out"])


def _oracle_partial(c, rank, world):
    from csahca_b200.split_kv import shard_slots

    idx, tl = shard_slots(torch.from_numpy(c["idx"]), torch.from_numpy(c["tl"]), rank, world)
    xidx, xl = shard_slots(torch.from_numpy(c["xidx"]), torch.from_numpy(c["xl"]), rank, world)
    return dsv4.partial_attention(c["q"], "bf16", c["cache"], idx.numpy(), tl.numpy(), page_size=c["page"],
                                  softmax_scale=c["scale"], extra_cache=c["xcache"], extra_token_indices=xidx.numpy(),
                                  extra_topk_lengths=xl.numpy(), extra_page_size=c["xpage"])


@pytest.mark.parametrize("world", [1, 2, 3, 5])
def test_oracle_shards_merge_to_full_decode(world):
    c = _golden()
    parts = [_oracle_partial(c, r, world) for r in range(world)]
    out = dsv4.combine_partials(np.stack([p[0] for p in parts]), np.stack([p[1] for p in parts]), c["sink"], "bf16")
    np.testing.assert_allclose(to_f32(out, "bf16"), to_f32(c["out"], "bf16"), atol=ATOL, rtol=RTOL)


def test_shard_slots_lengths():
    from csahca_b200.split_kv import shard_slots

    idx = torch.arange(20, dtype=torch.int32).reshape(2, 10)
    tl = torch.tensor([7, 0], dtype=torch.int32)
    got = [shard_slots(idx, tl, r, 3) for r in range(3)]
    assert [g[0].shape[1] for g in got] == [3, 3, 4]
    assert [g[1].tolist() for g in got] == [[3, 0], [3, 0], [1, 0]]
    _, full = shard_slots(idx, None, 2, 3)
    assert full.tolist() == [4, 4]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from csahca_b200.split_kv import dsv4_split_kv_decode

    c = _golden()
    t = torch.from_numpy

    def partial_fn(q, cache, idx, lens, xcache, xidx, xlens, page, xpage, scale, shard0, shards, total):
        from csahca_b200.split_kv import shard_slots

        os_, ls_ = [], []
        for sh in range(shard0, shard0 + shards):
            i, li = shard_slots(idx, lens, sh, total)
            xi, xli = shard_slots(xidx, xlens, sh, total)
            o, lse = dsv4.partial_attention(q.numpy(), "bf16", cache.numpy(), i.numpy(), li.numpy(),
                                            page_size=page, softmax_scale=scale, extra_cache=xcache.numpy(),
                                            extra_token_indices=xi.numpy(), extra_topk_lengths=xli.numpy(),
                                            extra_page_size=xpage)
            os_.append(o)
            ls_.append(lse)
        return t(np.stack(os_)), t(np.stack(ls_))

    def combine_fn(o_all, lse_all, sink, dtype):
        return t(dsv4.combine_partials(o_all.numpy(), lse_all.numpy(), sink.numpy(), "bf16").astype(np.int16))

    out = dsv4_split_kv_decode(t(c["q"].astype(np.int16)), t(c["cache"]), t(c["idx"]), t(c["tl"]), t(c["xcache"]),
                               t(c["xidx"]), t(c["xl"]), t(c["sink"]), c["page"], c["xpage"], c["scale"],
                               partial_fn=partial_fn, combine_fn=combine_fn)
    np.save(f"{result_path}.{rank}.npy", out.numpy().view(np.uint16))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_gather_and_merge(tmp_path):
    world, port = 2, _free_port()
    mp.start_processes(_gloo_rank, args=(world, port, str(tmp_path / "out")), nprocs=world, start_method="spawn")
    c = _golden()
    for r in range(world):
        out = np.load(tmp_path / f"out.{r}.npy")
        np.testing.assert_allclose(to_f32(out, "bf16"), to_f32(c["out"], "bf16"), atol=ATOL, rtol=RTOL)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [1, 2, 4, 7])
def test_gpu_partials_merge_to_full_decode(cuda, world):
    from csahca_b200 import extension as ext
    from csahca_b200.split_kv import dsv4_combine_partials, dsv4_decode_partial, shard_slots
    from helpers import to_torch

    rng = np.random.default_rng(world)
    ntok, nq, heads, nmain, nextra, page, xpage = 3000, 3, 64, 700, 90, 64, 16
    from oracle.numerics import from_f32
    toks = from_f32(rng.standard_normal((ntok, 512)).astype(np.float32), "bf16")
    xt = from_f32((rng.standard_normal((800, 512)) * 0.5).astype(np.float32), "bf16")
    c = dict(q=from_f32(rng.standard_normal((nq, heads, 512)).astype(np.float32), "bf16"),
             cache=dsv4.pack_dsv4_cache(toks, page_size=page), idx=rng.integers(-1, ntok, (nq, nmain)).astype(np.int32),
             tl=np.array([nmain, 333, 0], np.int32), xcache=dsv4.pack_dsv4_cache(xt, page_size=xpage),
             xidx=rng.integers(0, 800, (nq, nextra)).astype(np.int32), xl=np.array([nextra, 5, 0], np.int32),
             sink=rng.standard_normal(heads).astype(np.float32))
    d = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    q = to_torch(c["q"], "bf16", cuda)
    scale = 1.0 / math.sqrt(512)
    args = (q, d(c["cache"]), d(c["idx"]), d(c["tl"]), d(c["xcache"]), d(c["xidx"]), d(c["xl"]), page, xpage, scale)
    parts = [dsv4_decode_partial(*args, r, 1, world) for r in range(world)]  # one shard per "rank"
    o_all, lse_all = dsv4_decode_partial(*args, 0, world, world)  # all shards in one launch
    torch.testing.assert_close(o_all, torch.cat([p[0] for p in parts]), atol=0, rtol=0)
    torch.testing.assert_close(lse_all, torch.cat([p[1] for p in parts]), atol=0, rtol=0)
    # the kernel's shard against the oracle's shard (host slicing)
    for r in range(world):
        idx, tl = shard_slots(torch.from_numpy(c["idx"]), torch.from_numpy(c["tl"]), r, world)
        xidx, xl = shard_slots(torch.from_numpy(c["xidx"]), torch.from_numpy(c["xl"]), r, world)
        o_ref, lse_ref = dsv4.partial_attention(c["q"], "bf16", c["cache"], idx.numpy(), tl.numpy(), page_size=page,
                                                softmax_scale=scale, extra_cache=c["xcache"],
                                                extra_token_indices=xidx.numpy(), extra_topk_lengths=xl.numpy(),
                                                extra_page_size=xpage)
        np.testing.assert_allclose(parts[r][0][0].cpu().numpy(), o_ref, atol=ATOL, rtol=RTOL)
        fin = np.isfinite(lse_ref)
        np.testing.assert_array_equal(np.isfinite(parts[r][1][0].cpu().numpy()), fin)
        np.testing.assert_allclose(parts[r][1][0].cpu().numpy()[fin], lse_ref[fin], atol=1e-3, rtol=1e-4)
    out = dsv4_combine_partials(o_all, lse_all, d(c["sink"]), torch.bfloat16)
    full = ext.dsv4_sparse_decode_forward(q, d(c["cache"]), d(c["idx"]), d(c["tl"]), d(c["xcache"]), d(c["xidx"]),
                                          d(c["xl"]), d(c["sink"]), page, xpage, scale)
    ref = dsv4.reference_attention(c["q"], "bf16", c["cache"], c["idx"], c["tl"], c["sink"], page_size=page,
                                   softmax_scale=scale, extra_cache=c["xcache"], extra_token_indices=c["xidx"],
                                   extra_topk_lengths=c["xl"], extra_page_size=xpage)
    np.testing.assert_allclose(out.float().cpu().numpy(), to_f32(ref, "bf16"), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(out.float(), full.float(), atol=ATOL, rtol=RTOL)


def _nccl_rank(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    from csahca_b200 import extension as ext
    from csahca_b200.split_kv import dsv4_split_kv_decode
    from helpers import to_torch

    c = _golden()
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    q = to_torch(c["q"], "bf16", dev)
    args = (q, d(c["cache"]), d(c["idx"]), d(c["tl"]), d(c["xcache"]), d(c["xidx"]), d(c["xl"]), d(c["sink"]),
            c["page"], c["xpage"], c["scale"])
    out = dsv4_split_kv_decode(*args)
    full = ext.dsv4_sparse_decode_forward(*args)
    np.save(f"{result_path}.{rank}.npy", np.stack([out.float().cpu().numpy(), full.float().cpu().numpy()]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.gpu
def test_two_nccl_ranks(cuda, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, port = 2, _free_port()
    mp.start_processes(_nccl_rank, args=(world, port, str(tmp_path / "out")), nprocs=world, start_method="spawn")
    c = _golden()
    for r in range(world):
        out, full = np.load(tmp_path / f"out.{r}.npy")
        np.testing.assert_allclose(out, to_f32(c["out"], "bf16"), atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(out, full, atol=ATOL, rtol=RTOL)


@pytest.mark.gpu
@pytest.mark.parametrize("local_splits", [None, 1, 3, 8])
def test_one_gpu_local_splits(cuda, local_splits):
    from csahca_b200.split_kv import dsv4_split_kv_decode
    from helpers import to_torch

    c = _golden()
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    out = dsv4_split_kv_decode(to_torch(c["q"], "bf16", cuda), d(c["cache"]), d(c["idx"]), d(c["tl"]),
                               d(c["xcache"]), d(c["xidx"]), d(c["xl"]), d(c["sink"]), c["page"], c["xpage"],
                               c["scale"], local_splits=local_splits)
    np.testing.assert_allclose(out.float().cpu().numpy(), to_f32(c["out"], "bf16"), atol=ATOL, rtol=RTOL)


def test_partial_and_combine_validate_before_any_launch():
    """CPU-resident tensors, int64 index lists and mis-shaped partials raise
    RuntimeError in the Python layer, before the library is touched."""
    from csahca_b200.split_kv import dsv4_combine_partials, dsv4_decode_partial

    c = _golden()
    q = torch.from_numpy(c["q"].view(np.int16)).view(torch.bfloat16)
    cache = torch.from_numpy(c["cache"])
    idx, tl = torch.from_numpy(c["idx"]), torch.from_numpy(c["tl"])
    with pytest.raises(RuntimeError, match="q must be CUDA"):
        dsv4_decode_partial(q, cache, idx, tl, None, None, None, c["page"], 1, c["scale"])
    with pytest.raises(RuntimeError, match="q must be CUDA"):
        dsv4_decode_partial(q, cache, idx.to(torch.int64), tl, None, None, None, c["page"], 1, c["scale"])
    with pytest.raises(RuntimeError, match="must be CUDA tensors"):
        dsv4_combine_partials(torch.zeros(2, 1, 4, 512), torch.zeros(2, 1, 4), None, torch.bfloat16)


@pytest.mark.gpu
def test_partial_rejects_int64_and_cpu_indices_on_gpu(cuda):
    from csahca_b200.split_kv import dsv4_combine_partials, dsv4_decode_partial

    c = _golden()
    q = torch.from_numpy(c["q"].view(np.int16)).view(torch.bfloat16).to(cuda)
    cache = torch.from_numpy(c["cache"]).to(cuda)
    idx, tl = torch.from_numpy(c["idx"]).to(cuda), torch.from_numpy(c["tl"]).to(cuda)
    args = (c["page"], 1, c["scale"])
    with pytest.raises(RuntimeError, match="token_indices must be int32"):
        dsv4_decode_partial(q, cache, idx.to(torch.int64), tl, None, None, None, *args)
    with pytest.raises(RuntimeError, match="token_indices must be CUDA"):
        dsv4_decode_partial(q, cache, idx.cpu(), tl, None, None, None, *args)
    with pytest.raises(RuntimeError, match="topk_lengths must be int32"):
        dsv4_decode_partial(q, cache, idx, tl.to(torch.int64), None, None, None, *args)
    with pytest.raises(RuntimeError, match="token_indices must be contiguous"):
        dsv4_decode_partial(q, cache, idx.t().contiguous().t(), tl, None, None, None, *args)
    with pytest.raises(RuntimeError, match="shards must satisfy"):
        dsv4_decode_partial(q, cache, idx, tl, None, None, None, *args, shard0=3, shards=2, shards_total=4)
    o = torch.zeros(2, q.shape[0], q.shape[1], 512, device=cuda)
    with pytest.raises(RuntimeError, match="lse_parts must be"):
        dsv4_combine_partials(o, torch.zeros(2, q.shape[0], 3, device=cuda), None, torch.bfloat16)
