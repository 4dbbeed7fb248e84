"""The allocation-free CSA decode entry point, called through the C ABI.

``csahca_csa_decode_noalloc`` serves callers that cannot allocate device memory
when they call us (a server that reserved all HBM up front, a latency-critical
loop that must not hit cudaMalloc's implicit synchronisation, a foreign-language
binding without a device allocator).  It keeps its scratch in a fixed array
inside the library.  This file is collected last on purpose, so that a run
that stops at the first failure has run every other test already; it also
passes when run alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle.numerics import to_f32

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2  # the bound every other CSA parity test uses


def _entry():
    from csahca_b200 import _native as N

    lib = N.lib()
    fn = lib.csahca_csa_decode_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int, ctypes.c_int] + [ctypes.c_int64] * 6 + [ctypes.c_void_p] * 2
    lib.csahca_csa_decode_noalloc_max_scratch_bytes.restype = ctypes.c_size_t
    return N, lib, fn


def _call(N, fn, q, k, v, idx, chunk, out):
    b, h, d = q.shape
    return fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), idx.data_ptr(), N.INDEX_CODE[idx.dtype],
              N.DTYPE_CODE[q.dtype], b, h, k.shape[2], d, idx.shape[2], chunk, out.data_ptr(),
              N.stream_handle(q.device))


# (16,32,16) and (2,8,8) combine inside a thread-block cluster and touch no
# scratch.  (1,2,32) splits each row into 32 single-chunk CTAs and (64,32,32)
# gives 2048 rows x 2 units: both combine through the scratch array (arrival
# counters + fp32 partials), which is what this entry point exists for.
@pytest.mark.parametrize("b,h,top_k", [(16, 32, 16), (2, 8, 8), (1, 2, 32), (64, 32, 32)])
def test_noalloc_matches_workspace_entry_two_calls_in_a_row(cuda, b, h, top_k):
    from csahca_b200 import hybrid_attention_cuda as m
    from helpers import to_numpy
    from oracle import csa

    N, lib, fn = _entry()
    s, d, c = 2048, 128, 64
    g = torch.Generator(device=cuda).manual_seed(7 + b + top_k)
    q = torch.randn(b, h, d, device=cuda, generator=g).to(torch.bfloat16)
    k = torch.randn(b, h, s, d, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(b, h, s, d, device=cuda, generator=g).to(torch.bfloat16)
    idx = torch.argsort(torch.rand(b, h, s // c, device=cuda, generator=g), dim=-1)[..., :top_k].to(torch.int32)
    ref = m.csa_decode_forward_tiled(q, k, v, idx, c, 8)
    rows = slice(0, min(b, 2))
    want = csa.csa_reference(*(to_numpy(t[rows]) for t in (q, k, v)), chunk_size=c, top_k=top_k, dtype="bf16",
                             selected_chunks=to_numpy(idx[rows]))
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        assert _call(N, fn, q, k, v, idx, c, out) == 0, lib.csahca_last_error()
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.float().cpu().numpy(), ref.float().cpu().numpy(), atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(out[rows].float().cpu().numpy(), to_f32(want, "bf16"), atol=ATOL, rtol=RTOL)


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    N, lib, fn = _entry()
    cap = lib.csahca_csa_decode_noalloc_max_scratch_bytes()
    assert cap == 8 << 20
    q = torch.zeros(1, 1, 128, device=cuda, dtype=torch.bfloat16)
    # 65536 x 64 rows split 16 ways need far more than 8 MiB of partials: rejected before any launch
    rc = fn(q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), 0, 2, 65536, 64, 1024, 128, 64, 64,
            q.data_ptr(), N.stream_handle(cuda))
    assert rc == 1
    assert b"8 MiB" in lib.csahca_last_error()
