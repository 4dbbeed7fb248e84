"""The C-ABI library and the host-side mirror, without a GPU."""

import ctypes
import re

import pytest
import torch

from conftest import ROOT


def _header_functions():
    text = (ROOT / "include" / "csahca_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(csahca_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from csahca_b200 import _native

    lib = _native.lib()
    names = _header_functions()
    assert len(names) >= 8
    for name in names:
        assert hasattr(lib, name), name
    assert b"sm_100a" in lib.csahca_version()


def test_argument_errors_need_no_gpu():
    from csahca_b200 import _native as N

    lib = N.lib()
    assert lib.csahca_csa_select_topk(None, None, None, 2, 1, 1, 64, 128, 0, 4, None, None, 0, None) == 1
    assert b"chunk_size must be positive" in lib.csahca_last_error()
    assert lib.csahca_csa_select_topk(None, None, None, 2, 1, 1, 65, 128, 64, 4, None, None, 0, None) == 1
    assert b"divisible" in lib.csahca_last_error()
    assert lib.csahca_csa_decode(None, None, None, None, 5, 2, 1, 1, 64, 128, 4, 64, None, None, 0, None) == 1
    assert b"int32 or int64" in lib.csahca_last_error()
    assert lib.csahca_dsv4_decode(None, 2, 1, 64, None, 1, 100, 64, None, 8, None, None, 0, 0, 0, None, 0, None,
                                  None, ctypes.c_float(0.1), None, None) == 1
    assert b"bytes_per_page is too small" in lib.csahca_last_error()
    with pytest.raises(TypeError):
        lib.csahca_csa_select_topk(1, 2, 3)
    # split-KV entries
    assert lib.csahca_dsv4_decode_partial(None, 2, 1, 64, None, 1, 37440, 64, None, 8, None, None, 0, 0, 0, None,
                                          0, None, ctypes.c_float(0.1), 2, 1, 2, None, None, None) == 1
    assert b"o_partial and lse_partial are required" in lib.csahca_last_error()
    buf = ctypes.create_string_buffer(64)
    assert lib.csahca_dsv4_decode_partial(None, 2, 1, 64, None, 1, 37440, 64, None, 8, None, None, 0, 0, 0, None,
                                          0, None, ctypes.c_float(0.1), 2, 1, 2, buf, buf, None) == 1
    assert b"invalid shard range" in lib.csahca_last_error()
    assert lib.csahca_dsv4_combine_partials(None, None, 0, 1, 64, None, None, 2, None) == 1
    assert b"parts must be in [1, 64]" in lib.csahca_last_error()
    # chunk-sum cache entries
    assert lib.csahca_csa_chunk_sums_build(None, 2, 1, 1, 100, 128, 64, None, None) == 1
    assert b"divisible" in lib.csahca_last_error()
    assert lib.csahca_csa_chunk_sums_append(None, 2, 1, 1, 128, 128, 64, None, None, None) == 1
    assert b"positions is required" in lib.csahca_last_error()
    assert lib.csahca_csa_select_topk_from_sums(None, 2, None, None, 1, 1, 8, 128, 64, 0, None, None, 0, None) == 1
    assert b"top_k must be positive" in lib.csahca_last_error()


def test_workspace_sizes():
    from csahca_b200 import _native as N

    lib = N.lib()
    # 256 ticket bytes + counters + one fp32 score per chunk
    assert lib.csahca_csa_select_topk_workspace_size(64, 32, 32768, 64) == 256 + 8192 + 64 * 32 * 512 * 4
    assert lib.csahca_csa_decode_workspace_size(1, 8, 128, 8, 64) >= 256


def test_reference_error_messages_on_cpu_tensors():
    from csahca_b200 import hybrid_attention_cuda as m

    q = torch.zeros(1, 2, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 2, 256, 128, dtype=torch.bfloat16)
    idx = torch.zeros(1, 2, 2, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="all tensors must be CUDA tensors"):
        m.csa_decode_forward(q, k, k, idx, 64)
    with pytest.raises(RuntimeError, match="all tensors must be CUDA tensors"):
        m.csa_decode_forward_tiled(q, k, k, idx, 64, 8)
    qd = torch.zeros(1, 8, 512, dtype=torch.bfloat16)
    cache = torch.zeros(4, 37440, dtype=torch.uint8)
    ti = torch.zeros(1, 4, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="q, paged_k_cache_u8, and token_indices must be CUDA tensors"):
        m.dsv4_decode_forward_tiled(qd, cache, ti, None, None, None, None, None, 64, 1, 0, 0.04)
    with pytest.raises(RuntimeError, match="extra_token_indices must be CUDA tensors"):
        m.dsv4_sparse_decode_forward(qd, cache, ti, None, cache, ti, None, None, 64, 16, 0.04)


def test_extension_surface_matches_reference_names():
    from csahca_b200 import extension, hybrid_attention_cuda

    for name in ["load_cuda_extension", "csa_decode_forward", "csa_decode_forward_tiled",
                 "dsv4_swa_decode_forward", "dsv4_sparse_decode_forward", "_dsv4_tiled_enabled", "_dsv4_tile_size"]:
        assert callable(getattr(extension, name)), name
    for name in ["csa_decode_forward", "csa_decode_forward_tiled", "dsv4_swa_decode_forward",
                 "dsv4_sparse_decode_forward", "dsv4_decode_forward_tiled"]:
        assert callable(getattr(hybrid_attention_cuda, name)), name
    assert extension.load_cuda_extension() is hybrid_attention_cuda


def test_tiled_switch_env(monkeypatch):
    from csahca_b200 import extension, hybrid_attention_cuda

    monkeypatch.setenv("CSAHCA_DSV4_TILED", "0")
    assert not extension._dsv4_tiled_enabled(hybrid_attention_cuda)
    monkeypatch.setenv("CSAHCA_DSV4_TILED", "1")
    assert extension._dsv4_tiled_enabled(hybrid_attention_cuda)
    monkeypatch.setenv("CSAHCA_DSV4_TILE_SIZE", "junk")
    assert extension._dsv4_tile_size() == 0
