"""CSA scorer + decode on the GPU against the CPU oracle.

Contract: selected chunk indices bit-exact; outputs within
2e-2 absolute / 1e-2 relative for bf16 (fp16 / fp32 get the same bound).
"""

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from helpers import to_numpy, to_torch
from oracle import csa
from oracle.numerics import from_f32, to_f32

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def _ext():
    from csahca_b200 import extension

    return extension


def _check_out(got, ref, dtype):
    np.testing.assert_allclose(got.float().cpu().numpy(), to_f32(ref, dtype), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("name", ["csa_bf16_small", "csa_f16_small", "csa_f32_small"])
@pytest.mark.parametrize("entry", ["v1", "tiled"])
def test_golden_cases(cuda, name, entry):
    z = np.load(GOLDEN / f"{name}.npz")
    dt = str(z["dtype"])
    _, _, _, _, c, k, _ = (int(x) for x in z["meta"])
    q, kc, vc = (to_torch(z[n], dt, cuda) for n in ("q", "k", "v"))
    ext = _ext()
    sel = ext.select_topk_chunks(q, kc, c, k)
    np.testing.assert_array_equal(sel.cpu().numpy(), z["selected"])
    if entry == "v1":
        out = ext.csa_decode_forward(q, kc, vc, sel, c)
    else:
        out = ext.csa_decode_forward_tiled(q, kc, vc, sel, c, 8)
    _check_out(out, z["out"], dt)


def test_config1_full_size(cuda):
    """B1 H8 S32768 D128 c64 k8 bf16 with the reference's seeded inputs."""
    z = np.load(GOLDEN / "csa_cfg1.npz")
    b, h, s, d, c, k, seed = (int(x) for x in z["meta"])
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    q = torch.randn(b, h, d, dtype=torch.bfloat16, generator=g).to(cuda)
    kc = torch.randn(b, h, s, d, dtype=torch.bfloat16, generator=g).to(cuda)
    vc = torch.randn(b, h, s, d, dtype=torch.bfloat16, generator=g).to(cuda)
    out, sel = _ext().csa_decode_step(q, kc, vc, c, k)
    np.testing.assert_array_equal(sel.cpu().numpy(), z["selected"])
    _check_out(out, z["out"], "bf16")


def _ragged_case(seed, b, h, s, d, c, dtype="bf16"):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((b, h, d)).astype(np.float32)
    k = rng.standard_normal((b, h, s, d)).astype(np.float32)
    k += np.repeat(rng.normal(0, 0.5, (b, h, s // c, 1)).astype(np.float32), c, axis=2)
    v = rng.standard_normal((b, h, s, d)).astype(np.float32)
    lens = (rng.integers(s // (8 * c), s // c + 1, size=b) * c).astype(np.int32)
    return from_f32(q, dtype), from_f32(k, dtype), from_f32(v, dtype), lens


def _assert_tie_free(qn, kn, lens, c, k, dtype):
    for bi in range(qn.shape[0]):
        sc = csa.chunk_scores(qn[bi:bi + 1], kn[bi:bi + 1, :, : lens[bi]], c, dtype)[0]
        srt = -np.sort(-sc, axis=-1)
        if srt.shape[-1] > k:
            gap = srt[:, k - 1] - srt[:, k]
            assert (gap > 1e-5 * np.abs(srt[:, k - 1]).clip(1e-3)).all(), "near-tie in the seeded data"


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_ragged_batch_selection_and_decode(cuda, dtype):
    b, h, s, d, c, k = 6, 4, 4096, 128, 64, 16
    qn, kn, vn, lens = _ragged_case(3, b, h, s, d, c, dtype)
    _assert_tie_free(qn, kn, lens, c, k, dtype)
    ref_sel = csa.select_topk_chunks_ragged(qn, kn, lens, c, k, dtype)
    q, kc, vc = (to_torch(x, dtype, cuda) for x in (qn, kn, vn))
    out, sel = _ext().csa_decode_step(q, kc, vc, c, k, seq_lens=torch.from_numpy(lens).to(cuda))
    np.testing.assert_array_equal(sel.cpu().numpy(), ref_sel)
    _check_out(out, csa.csa_decode_skipping(qn, kn, vn, ref_sel, c, dtype), dtype)


@pytest.mark.parametrize("d", [32, 64, 256, 512])
def test_head_dims(cuda, d):
    rng = np.random.default_rng(d)
    b, h, s, c, k = 2, 3, 1024, 64, 5
    qn, kn, vn = (from_f32(rng.standard_normal(sh).astype(np.float32), "bf16")
                  for sh in [(b, h, d), (b, h, s, d), (b, h, s, d)])
    q, kc, vc = (to_torch(x, "bf16", cuda) for x in (qn, kn, vn))
    ext = _ext()
    sel = ext.select_topk_chunks(q, kc, c, k)
    np.testing.assert_array_equal(sel.cpu().numpy(), csa.select_topk_chunks(qn, kn, c, k, "bf16"))
    out = ext.csa_decode_forward_tiled(q, kc, vc, sel, c)
    _check_out(out, csa.csa_reference(qn, kn, vn, chunk_size=c, top_k=k, dtype="bf16",
                                      selected_chunks=sel.cpu().numpy()), "bf16")


@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
def test_decode_skips_negative_and_out_of_range(cuda, index_dtype):
    """Negative chunk slots and tokens >= seq_len are skipped (csa_attention.cu:176-184)."""
    rng = np.random.default_rng(11)
    b, h, s, d, c = 2, 4, 1000, 128, 64  # s not a multiple of c: the last chunk is partial
    qn, kn, vn = (from_f32(rng.standard_normal(sh).astype(np.float32), "bf16")
                  for sh in [(b, h, d), (b, h, s, d), (b, h, s, d)])
    sel = np.array([[[0, -1, 15, 3], [15, 15, -1, -1], [-1, -1, -1, -1], [2, 7, 40, 1]],
                    [[14, 13, 12, 11], [-5, 0, 1, 2], [15, 0, 3, -1], [9, 9, 9, 9]]], dtype=np.int64)
    q, kc, vc = (to_torch(x, "bf16", cuda) for x in (qn, kn, vn))
    idx = torch.from_numpy(sel).to(device=cuda, dtype=index_dtype)
    out = _ext().csa_decode_forward(q, kc, vc, idx, c)
    _check_out(out, csa.csa_decode_skipping(qn, kn, vn, sel, c, "bf16"), "bf16")
    assert (out[0, 2] == 0).all()


@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
def test_decode_skips_chunks_past_the_end(cuda, index_dtype):
    """Chunk indices from ceil(seq_len/chunk) up to 2^30 (and beyond, for int64)
    select no token; c * chunk must not wrap into a valid-looking offset."""
    rng = np.random.default_rng(12)
    b, h, s, d, c = 1, 3, 1000, 128, 64
    qn, kn, vn = (from_f32(rng.standard_normal(sh).astype(np.float32), "bf16")
                  for sh in [(b, h, d), (b, h, s, d), (b, h, s, d)])
    big = [16, 17, 2**25, 2**26 + 3, 2**30 - 1, 2**30]
    if index_dtype == torch.int64:
        big += [2**31, 2**40]
    else:
        big += [2**31 - 1, 2**31 - 64]
    sel = np.array([[[5] + big[:3], big[3:7], [15, big[7], 0, big[0]]]], dtype=np.int64)
    q, kc, vc = (to_torch(x, "bf16", cuda) for x in (qn, kn, vn))
    idx = torch.from_numpy(sel).to(device=cuda, dtype=index_dtype)
    out = _ext().csa_decode_forward_tiled(q, kc, vc, idx, c, 8)
    _check_out(out, csa.csa_decode_skipping(qn, kn, vn, sel, c, "bf16"), "bf16")
    assert (out[0, 1] == 0).all()


@pytest.mark.parametrize("b,h,top_k", [(1, 2, 32), (1, 1, 3), (16, 32, 16), (64, 32, 16), (8, 32, 32), (64, 32, 32)])
def test_split_and_merge_paths(cuda, b, h, top_k):
    """Row splits with the in-kernel last-CTA combine, repeated to exercise the workspace reset."""
    s, d, c = 2048, 128, 64
    g = torch.Generator(device=cuda)
    g.manual_seed(b * 100 + top_k)
    q = torch.randn(b, h, d, device=cuda, generator=g).to(torch.bfloat16)
    kc = torch.randn(b, h, s, d, device=cuda, generator=g).to(torch.bfloat16)
    vc = torch.randn(b, h, s, d, device=cuda, generator=g).to(torch.bfloat16)
    idx = torch.argsort(torch.rand(b, h, s // c, device=cuda, generator=g), dim=-1)[..., :top_k].to(torch.int32)
    ext = _ext()
    o1 = ext.csa_decode_forward_tiled(q, kc, vc, idx, c)
    o2 = ext.csa_decode_forward_tiled(q, kc, vc, idx, c)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    rows = slice(0, min(b, 3))
    qn, kn, vn, sel = (to_numpy(t[rows]) for t in (q, kc, vc, idx))
    ref = csa.csa_reference(qn, kn, vn, chunk_size=c, top_k=top_k, dtype="bf16", selected_chunks=sel)
    _check_out(o1[rows], ref, "bf16")


def test_topk_larger_than_chunks_and_empty_requests(cuda):
    rng = np.random.default_rng(5)
    b, h, s, d, c = 3, 2, 512, 64, 64
    qn = from_f32(rng.standard_normal((b, h, d)).astype(np.float32), "bf16")
    kn = from_f32(rng.standard_normal((b, h, s, d)).astype(np.float32), "bf16")
    q, kc = (to_torch(x, "bf16", cuda) for x in (qn, kn))
    ext = _ext()
    sel = ext.select_topk_chunks(q, kc, c, 100)
    assert sel.shape == (b, h, 8)
    np.testing.assert_array_equal(sel.cpu().numpy(), csa.select_topk_chunks(qn, kn, c, 100, "bf16"))
    lens = np.array([512, 0, 192], np.int32)
    sel = ext.select_topk_chunks(q, kc, c, 4, seq_lens=torch.from_numpy(lens).to(cuda))
    np.testing.assert_array_equal(sel.cpu().numpy(), csa.select_topk_chunks_ragged(qn, kn, lens, c, 4, "bf16"))


@pytest.mark.parametrize("c,d,dtype", [(1, 128, "bf16"), (3, 64, "f16"), (48, 128, "bf16"), (32, 128, "f32"),
                                         (128, 64, "bf16"), (128, 32, "f32")])
def test_chunk_sizes_and_unit_sizes(cuda, c, d, dtype):
    """Odd chunk sizes (partial token steps), chunks that exactly fill a staging
    slot, and enough rows that the scorer uses its largest ticket units."""
    rng = np.random.default_rng(c * 7 + d)
    n_chunks = 160 if c <= 48 else 40
    b, h, s, k = 5, 40, c * n_chunks, 9
    qn = from_f32(rng.standard_normal((b, h, d)).astype(np.float32), dtype)
    kn = from_f32(rng.standard_normal((b, h, s, d)).astype(np.float32), dtype)
    lens = (rng.integers(0, n_chunks + 1, b) * c).astype(np.int32)
    q, kc = (to_torch(x, dtype, cuda) for x in (qn, kn))
    sel = _ext().select_topk_chunks(q, kc, c, k, seq_lens=torch.from_numpy(lens).to(cuda)).cpu().numpy()
    ref = csa.select_topk_chunks_ragged(qn, kn, lens, c, k, dtype)
    np.testing.assert_array_equal(sel < 0, ref < 0)
    # A row whose top k+1 oracle scores are all separated by more than fp32
    # rounding of a differently ordered sum must match exactly.  In a row with
    # such a near-tie only the near-tied chunks may trade places, so the scores
    # at every selected position must still agree.
    exact_rows = 0
    for bi in range(b):
        if lens[bi] == 0:
            continue
        sc = csa.chunk_scores(qn[bi:bi + 1], kn[bi:bi + 1, :, : lens[bi]], c, dtype)[0]
        got = np.take_along_axis(sc, np.maximum(sel[bi], 0), -1)
        want = np.take_along_axis(sc, np.maximum(ref[bi], 0), -1)
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
        srt = -np.sort(-sc, axis=-1)[:, : k + 1]
        gaps = srt[:, :-1] - srt[:, 1:]
        tie_free = (gaps > 1e-5 * np.abs(srt[:, :-1]).clip(1e-3)).all(axis=-1)
        np.testing.assert_array_equal(sel[bi][tie_free], ref[bi][tie_free])
        exact_rows += int(tie_free.sum())
    assert exact_rows >= 0.9 * h * int((lens > 0).sum()), exact_rows


def test_many_chunks_global_topk_path(cuda):
    """More chunks than the register top-k path holds (> 4096): the global-memory scan."""
    rng = np.random.default_rng(9)
    b, h, s, d, c, k = 1, 2, 5000 * 16, 32, 16, 7
    qn = from_f32(rng.standard_normal((b, h, d)).astype(np.float32), "bf16")
    kn = from_f32(rng.standard_normal((b, h, s, d)).astype(np.float32), "bf16")
    q, kc = (to_torch(x, "bf16", cuda) for x in (qn, kn))
    sel = _ext().select_topk_chunks(q, kc, c, k)
    np.testing.assert_array_equal(sel.cpu().numpy(), csa.select_topk_chunks(qn, kn, c, k, "bf16"))


def test_equal_scores_break_ties_by_lower_index(cuda):
    b, h, s, d, c = 1, 1, 64 * 40, 64, 64
    kn = np.zeros((b, h, s, d), np.float32)
    for ch in (7, 30, 3):
        kn[0, 0, 64 * ch:64 * (ch + 1)] = 1.0
    q = to_torch(from_f32(np.ones((b, h, d), np.float32), "bf16"), "bf16", cuda)
    sel = _ext().select_topk_chunks(q, to_torch(from_f32(kn, "bf16"), "bf16", cuda), c, 5)
    assert sel[0, 0].tolist() == [3, 7, 30, 0, 1]


def test_capturable_in_cuda_graph(cuda):
    rng = np.random.default_rng(2)
    b, h, s, d, c, k = 4, 8, 2048, 128, 64, 8
    qn, kn, vn = (from_f32(rng.standard_normal(sh).astype(np.float32), "bf16")
                  for sh in [(b, h, d), (b, h, s, d), (b, h, s, d)])
    q, kc, vc = (to_torch(x, "bf16", cuda) for x in (qn, kn, vn))
    ext = _ext()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        ref_out, ref_sel = ext.csa_decode_step(q, kc, vc, c, k)  # warm-up allocates the workspaces
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        out, sel = ext.csa_decode_step(q, kc, vc, c, k)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(sel, ref_sel)
    assert torch.equal(out, ref_out)


def test_workspace_left_zero_across_shapes(cuda):
    """Every scorer call leaves its scratch all-zero, so a later call whose arrival
    counters fall where an earlier call kept scores starts clean; the decode
    clears its own counters, so its scratch may hold anything."""
    from csahca_b200 import _native

    ext = _ext()
    rng = np.random.default_rng(21)
    shapes = [(1, 2, 64 * 600, 64, 64, 9), (6, 40, 64 * 20, 128, 64, 4), (1, 1, 16 * 5000, 32, 16, 3),
              (8, 32, 64 * 12, 128, 64, 16)]
    for b, h, s, d, c, k in shapes:
        qn = from_f32(rng.standard_normal((b, h, d)).astype(np.float32), "bf16")
        kn = from_f32(rng.standard_normal((b, h, s, d)).astype(np.float32), "bf16")
        q, kc = (to_torch(x, "bf16", cuda) for x in (qn, kn))
        sel = ext.select_topk_chunks(q, kc, c, k)
        np.testing.assert_array_equal(sel.cpu().numpy(), csa.select_topk_chunks(qn, kn, c, k, "bf16"))
        for key, buf in _native.workspaces._bufs.items():
            if key[0] == "csa_decode":
                buf.fill_(0xA5)
        out = ext.csa_decode_forward_tiled(q, kc, kc, sel, c)
        _check_out(out, csa.csa_reference(qn, kn, kn, chunk_size=c, top_k=k, dtype="bf16",
                                          selected_chunks=sel.cpu().numpy()), "bf16")
        torch.cuda.synchronize()
        for key, buf in _native.workspaces._bufs.items():
            if key[0] == "csa_select":
                assert int(torch.count_nonzero(buf)) == 0, (key, (b, h, s, d, c, k))
