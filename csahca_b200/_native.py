"""ctypes binding of ``libcsahca_b200.so`` (the C ABI declared in include/csahca_b200.h).

The library is the only compute path.  Loading fails loudly (RuntimeError) when
it has not been built; there is no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libcsahca_b200.so"

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
INDEX_CODE = {torch.int32: 0, torch.int64: 1}

_lib: ctypes.CDLL | None = None
_lock = threading.Lock()

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_sz = ctypes.c_size_t


def _declare(lib: ctypes.CDLL) -> None:
    lib.csahca_last_error.restype = ctypes.c_char_p
    lib.csahca_last_error.argtypes = []
    lib.csahca_version.restype = ctypes.c_char_p
    lib.csahca_version.argtypes = []
    lib.csahca_read_device_error.restype = _int
    lib.csahca_read_device_error.argtypes = [ctypes.POINTER(_int)]

    lib.csahca_csa_select_topk_workspace_size.restype = _sz
    lib.csahca_csa_select_topk_workspace_size.argtypes = [_i64, _i64, _i64, _i64]
    lib.csahca_csa_select_topk.restype = _int
    lib.csahca_csa_select_topk.argtypes = [_vp, _vp, _vp, _int, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _sz, _vp]

    lib.csahca_csa_chunk_sums_build.restype = _int
    lib.csahca_csa_chunk_sums_build.argtypes = [_vp, _int, _i64, _i64, _i64, _i64, _i64, _vp, _vp]
    lib.csahca_csa_select_topk_from_sums.restype = _int
    lib.csahca_csa_select_topk_from_sums.argtypes = [_vp, _int, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp,
                                                     _vp, _sz, _vp]
    lib.csahca_csa_chunk_sums_append.restype = _int
    lib.csahca_csa_chunk_sums_append.argtypes = [_vp, _int, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp]

    lib.csahca_csa_decode_workspace_size.restype = _sz
    lib.csahca_csa_decode_workspace_size.argtypes = [_i64, _i64, _i64, _i64, _i64]
    lib.csahca_csa_decode.restype = _int
    lib.csahca_csa_decode.argtypes = [_vp, _vp, _vp, _vp, _int, _int, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp,
                                      _sz, _vp]

    lib.csahca_dsv4_indexer_workspace_size.restype = _sz
    lib.csahca_dsv4_indexer_workspace_size.argtypes = [_i64, _i64]
    lib.csahca_dsv4_indexer_topk.restype = _int
    lib.csahca_dsv4_indexer_topk.argtypes = [_vp, _vp, _vp, _vp] + [_i64] * 5 + [_vp, _vp, _sz, _vp]

    lib.csahca_dsv4_decode.restype = _int
    lib.csahca_dsv4_decode.argtypes = [
        _vp, _int, _i64, _i64,          # q, q_dtype, num_queries, heads
        _vp, _i64, _i64, _i64,          # cache, num_pages, bytes_per_page, page_size
        _vp, _i64, _vp,                 # token_indices, topk_slots, topk_lengths
        _vp, _i64, _i64, _i64,          # extra cache, pages, bytes_per_page, page_size
        _vp, _i64, _vp,                 # extra indices, extra slots, extra lengths
        _vp, ctypes.c_float, _vp, _vp,  # sink, scale, out, stream
    ]
    lib.csahca_dsv4_decode_partial.restype = _int
    lib.csahca_dsv4_decode_partial.argtypes = [
        _vp, _int, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _vp,
        _vp, _i64, _i64, _i64, _vp, _i64, _vp,
        ctypes.c_float, _i64, _i64, _i64, _vp, _vp, _vp,  # scale, shard0, shards, total, o, lse, stream
    ]
    lib.csahca_dsv4_combine_partials.restype = _int
    lib.csahca_dsv4_combine_partials.argtypes = [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _int, _vp]


def lib() -> ctypes.CDLL:
    """The loaded native library (built in-tree by ``python -m csahca_b200.build``)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = Path(os.environ.get("CSAHCA_B200_LIB", str(LIB_PATH)))
            if not path.exists():
                raise RuntimeError(
                    f"csahca_b200 native library not found at {path}; build it with `python -m csahca_b200.build`"
                )
            handle = ctypes.CDLL(str(path))
            _declare(handle)
            _lib = handle
    return _lib


def check(status: int) -> None:
    if status != 0:
        msg = lib().csahca_last_error().decode(errors="replace")
        raise RuntimeError(msg)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def read_device_error() -> int:
    """Reads and clears the current device's kernel error word (synchronises)."""
    code = _int(0)
    check(lib().csahca_read_device_error(ctypes.byref(code)))
    return int(code.value)


class WorkspacePool:
    """Zero-initialised scratch buffers, one per (op, device, stream).

    The kernels that use scratch leave their zero-initialised regions at zero
    when they finish, so a buffer is zeroed once when it is (re)allocated and
    then reused by every call of the same op on the same stream; calls on one
    stream never overlap on the GPU.  Allocate (warm up) before capturing a
    CUDA graph so the buffer lives outside the graph's memory pool.
    """

    def __init__(self) -> None:
        self._bufs: dict[tuple[str, int, int], torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device, nbytes: int, tag: str) -> torch.Tensor:
        index = device.index if device.index is not None else torch.cuda.current_device()
        key = (tag, index, stream_handle(device))
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 1 << 16)
                if buf is not None:
                    size = max(size, 2 * buf.numel())
                buf = torch.zeros(size, dtype=torch.uint8, device=device)
                self._bufs[key] = buf
            return buf


workspaces = WorkspacePool()
