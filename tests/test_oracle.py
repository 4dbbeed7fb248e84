"""The CPU oracle against golden vectors produced by the reference itself.

Fixtures: tests/golden/*.npz, written by tests/golden/make_golden.py from
hybrid_attention/reference.py and hybrid_attention/dsv4_correctness.py.
"""

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import csa, dsv4
from oracle.numerics import bf16_to_f32, e4m3_to_f32, f32_to_bf16, f32_to_e4m3, to_f32


def _load(name):
    return np.load(GOLDEN / f"{name}.npz")


@pytest.mark.parametrize("name", ["csa_bf16_small", "csa_f16_small", "csa_f32_small"])
def test_csa_oracle_matches_reference(name):
    z = _load(name)
    dt = str(z["dtype"])
    _, _, _, _, c, k, _ = (int(x) for x in z["meta"])
    sel = csa.select_topk_chunks(z["q"], z["k"], c, k, dt)
    np.testing.assert_array_equal(sel, z["selected"])
    out = csa.csa_reference(z["q"], z["k"], z["v"], chunk_size=c, top_k=k, dtype=dt, selected_chunks=z["selected"])
    np.testing.assert_allclose(to_f32(out, dt), to_f32(z["out"], dt), atol=1e-6, rtol=0)


def test_csa_oracle_config1_full_size():
    """Config 1 (B1 H8 S32768 D128 c64 k8 bf16): inputs regenerated from the reference's seeded generator."""
    z = _load("csa_cfg1")
    b, h, s, d, c, k, seed = (int(x) for x in z["meta"])
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    q = torch.randn(b, h, d, dtype=torch.bfloat16, generator=g)
    kc = torch.randn(b, h, s, d, dtype=torch.bfloat16, generator=g)
    vc = torch.randn(b, h, s, d, dtype=torch.bfloat16, generator=g)
    assert float(kc.double().sum()) == pytest.approx(float(z["k_checksum"]), rel=0, abs=1e-6)
    qn, kn, vn = (t.view(torch.int16).numpy().view(np.uint16) for t in (q, kc, vc))
    sel = csa.select_topk_chunks(qn, kn, c, k, "bf16")
    np.testing.assert_array_equal(sel, z["selected"])
    out = csa.csa_reference(qn, kn, vn, chunk_size=c, top_k=k, dtype="bf16", selected_chunks=sel)
    np.testing.assert_allclose(bf16_to_f32(out), bf16_to_f32(z["out"]), atol=2e-3, rtol=0)


@pytest.mark.parametrize("name", ["dsv4_c0", "dsv4_c4", "dsv4_c128", "dsv4_c0_f32q"])
def test_dsv4_packer_is_byte_identical(name):
    z = _load(name)
    page = int(z["meta"][4])
    np.testing.assert_array_equal(dsv4.pack_dsv4_cache(z["k_tokens"], page_size=page), z["cache"])
    if "x_cache" in z:
        np.testing.assert_array_equal(
            dsv4.pack_dsv4_cache(z["x_tokens"], page_size=int(z["extra_page_size"])), z["x_cache"])


@pytest.mark.parametrize("name", ["dsv4_c0", "dsv4_c4", "dsv4_c128", "dsv4_c0_f32q"])
@pytest.mark.parametrize("sink", [True, False])
def test_dsv4_oracle_matches_reference(name, sink):
    z = _load(name)
    dt = str(z["dtype"])
    page = int(z["meta"][4])
    kw = {}
    if "x_cache" in z:
        kw = dict(extra_cache=z["x_cache"], extra_token_indices=z["x_idx"], extra_topk_lengths=z["x_len"],
                  extra_page_size=int(z["extra_page_size"]))
    out = dsv4.reference_attention(z["q"], dt, z["cache"], z["token_indices"], z["topk_lengths"],
                                   z["attn_sink"] if sink else None, page_size=page,
                                   softmax_scale=float(z["softmax_scale"]), **kw)
    ref = z["out"] if sink else z["out_nosink"]
    # one output ulp of the storage dtype (fp32 accumulation order differs from torch.mv)
    tol = 4e-3 if dt == "bf16" else 1e-5
    np.testing.assert_allclose(to_f32(out, dt), to_f32(ref, dt), atol=tol, rtol=tol)


def test_numerics_match_torch_casts():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 50,
                        np.array([0.0, -0.0, 448.0, -448.0, 1e-9, -1e-9, 2 ** -9, 2 ** -10], np.float32)])
    x = np.clip(x, -448, 448).astype(np.float32)
    ref8 = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(f32_to_e4m3(x), ref8)
    np.testing.assert_array_equal(e4m3_to_f32(ref8), torch.from_numpy(ref8).view(torch.float8_e4m3fn).float().numpy())
    refb = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(f32_to_bf16(x), refb)


def test_ragged_selection_equals_per_request_slices():
    rng = np.random.default_rng(1)
    q = f32_to_bf16(rng.standard_normal((3, 2, 64)).astype(np.float32))
    k = f32_to_bf16(rng.standard_normal((3, 2, 512, 64)).astype(np.float32))
    lens = np.array([512, 128, 0], np.int32)
    sel = csa.select_topk_chunks_ragged(q, k, lens, 32, 6, "bf16")
    assert sel.shape == (3, 2, 6)
    np.testing.assert_array_equal(sel[0], csa.select_topk_chunks(q[:1], k[:1], 32, 6, "bf16")[0])
    np.testing.assert_array_equal(sel[1, :, :4], csa.select_topk_chunks(q[1:2], k[1:2, :, :128], 32, 6, "bf16")[0])
    assert (sel[1, :, 4:] == -1).all() and (sel[2] == -1).all()
