"""CPU: the oracle against the golden vectors and known identities.

The golden vectors come from an independent numpy restatement of the same
reference shaders (tests/golden/make_golden.py); the reference itself ships
none for this path, so parity is unpinned by reference tests.
"""
import numpy as np
import pytest

import oracle as O
from conftest import load_golden


def test_round_f16_matches_ieee():
    rng = np.random.default_rng(5)
    vals = np.concatenate([
        rng.standard_normal(2000).astype(np.float32) * 10,
        rng.standard_normal(500).astype(np.float32) * 1e-5,   # half subnormals
        np.array([65504, 65519, 65520, 1e6, -1e6, 0.0, -0.0, 6.1e-5, 5.96e-8, 2.9e-8],
                 np.float32),
    ])
    want = vals.astype(np.float16).astype(np.float32)
    got = np.array([O.round_f16(float(x)) for x in vals], np.float32)
    np.testing.assert_array_equal(got, want)


def test_round_bf16_rne():
    import torch
    rng = np.random.default_rng(6)
    vals = rng.standard_normal(3000).astype(np.float32) * 100
    want = torch.from_numpy(vals).to(torch.bfloat16).float().numpy()
    got = np.array([O.round_bf16(float(x)) for x in vals], np.float32)
    np.testing.assert_array_equal(got, want)


def test_head_norm_golden(manifest):
    m = manifest["head_norm"]
    p = m["params"]
    x = load_golden(m["x"])
    O.batch_head_norm(x, load_golden(m["gain"]), p["H"], p["D"], p["S"], p["eps"])
    np.testing.assert_allclose(x, load_golden(m["out"]), rtol=0, atol=2e-6)


def test_head_norm_matches_reference_test_cpu_rmsnorm(manifest):
    """batch_head_norm equals the reference test suite's own CPU RMSNorm
    (test/mesh_encoder_test.c3:81-92, restated in the fixture generator) per
    (token, head) row, to fp32 rounding (the shader sums the squares as a
    256-lane tree, the test in order)."""
    m = manifest["head_norm"]
    p = m["params"]
    x = load_golden(m["x"])
    O.batch_head_norm(x, load_golden(m["gain"]), p["H"], p["D"], p["S"], p["eps"])
    want = load_golden(manifest["cpu_rmsnorm_head_norm"]["out"])
    np.testing.assert_allclose(x, want, rtol=0, atol=2e-6)


@pytest.mark.parametrize("direction", [0, 1])
def test_transpose_golden(manifest, direction):
    m = manifest["transpose"]
    p = m["params"]
    got = O.transpose_heads(load_golden(m["x"]), p["S"], p["H"], p["D"], direction)
    np.testing.assert_array_equal(got.reshape(-1), load_golden(m[f"out{direction}"]).reshape(-1))


@pytest.mark.parametrize("name", ["rope_flux1", "rope_flux2", "rope_zimage"])
def test_rope_tables_golden(manifest, name):
    m = manifest[name]
    pos = load_golden(m["pos"]).astype(np.int32)
    c, s = O.rope_tables(pos, m["params"]["axes"], m["params"]["theta"])
    np.testing.assert_allclose(c, load_golden(m["cos"]), rtol=0, atol=1e-6)
    np.testing.assert_allclose(s, load_golden(m["sin"]), rtol=0, atol=1e-6)
    # The reference's own table test (test/zimage_component_test.c3:237-251)
    # checks cos^2 + sin^2 == 1.
    np.testing.assert_allclose(c * c + s * s, 1.0, atol=1e-6)


def test_rope_identity_rows():
    """Position 0 on every axis is the identity rotation (dit.c3:660-666)."""
    c, s = O.rope_tables(np.zeros((4, 3), np.int32), (16, 56, 56), 10000.0)
    assert np.all(c == 1.0) and np.all(s == 0.0)


def test_mrope_golden(manifest):
    m = manifest["mrope"]
    p = m["params"]
    x = load_golden(m["x"])
    O.mrope(x, load_golden(m["cos"]), load_golden(m["sin"]), p["S"], p["H"])
    np.testing.assert_allclose(x, load_golden(m["out"]), rtol=0, atol=1e-6)


def test_fa2_golden(manifest):
    m = manifest["fa2"]
    p = m["params"]
    got = O.flash_attention_v2(load_golden(m["q"]), load_golden(m["k"]), load_golden(m["v"]),
                               p["D"], p["H"], p["S"], p["scale"])
    np.testing.assert_allclose(got, load_golden(m["out"]), rtol=0, atol=2e-6)


def test_spatial_golden(manifest):
    m = manifest["spatial"]
    p = m["params"]
    got = O.spatial_attention(load_golden(m["q"]), load_golden(m["k"]), load_golden(m["v"]),
                              p["D"], p["H"], p["S"], p["scale"])
    np.testing.assert_allclose(got, load_golden(m["out"]), rtol=0, atol=2e-6)


def test_vae_golden(manifest):
    """orc_vae_attention against the independent numpy restatement of
    vae_attention (two heads in [S, C], 4100 keys across the shader's
    4096-key tile boundary)."""
    m = manifest["vae"]
    p = m["params"]
    got = O.vae_attention(load_golden(m["q"]), load_golden(m["k"]), load_golden(m["v"]),
                          p["D"], p["H"], p["S"], p["scale"])
    np.testing.assert_allclose(got, load_golden(m["out"]), rtol=0, atol=2e-6)


def test_vae_is_exact_fp32_and_row_subsets():
    """The shader's tiled fp32 softmax agrees with fp64 attention within 1e-5
    at D = 512, and a row range computes exactly those rows."""
    rng = np.random.default_rng(14)
    S, D = 150, 512
    q, k, v = (rng.standard_normal((S, D), dtype=np.float32) for _ in range(3))
    sc = D ** -0.5
    out = O.vae_attention(q, k, v, D, 1, S, sc)
    ex = O.attention_f64(q[None], k[None], v[None], D, 1, S, sc)[0]
    assert np.abs(out - ex).max() < 1e-5
    part = O.vae_attention(q, k, v, D, 1, S, sc, rows=(40, 90))
    np.testing.assert_array_equal(part[40:90], out[40:90])
    assert np.all(part[:40] == 0) and np.all(part[90:] == 0)


def test_exact_path_matches_reference_test_cpu_attention(manifest):
    """The reference's own CPU attention (test/mesh_encoder_test.c3:95-135,
    restated in tests/golden/make_golden.py) on the spatial fixture's inputs
    equals the oracle's spatial_attention to fp32 rounding."""
    m = manifest["spatial"]
    p = m["params"]
    got = O.spatial_attention(load_golden(m["q"]), load_golden(m["k"]), load_golden(m["v"]),
                              p["D"], p["H"], p["S"], p["scale"])
    want = load_golden(manifest["cpu_attention_spatial"]["out"])
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-6)


def test_fa2_within_reference_test_tolerance(manifest):
    """The oracle's flash_attention_v2 (fp16 operands) stays within the
    tolerance the reference's own test gives its FA2-style shader against
    cpu_attention (expect_close(..., 1e-3f), test/mesh_encoder_test.c3:322,
    :361) on the fa2 fixture's inputs (ragged S = 45, D = 128)."""
    m = manifest["fa2"]
    p = m["params"]
    got = O.flash_attention_v2(load_golden(m["q"]), load_golden(m["k"]), load_golden(m["v"]),
                               p["D"], p["H"], p["S"], p["scale"])
    want = load_golden(manifest["cpu_attention_fa2"]["out"])
    want = want.transpose(1, 0, 2).reshape(p["S"], p["H"] * p["D"])
    assert np.abs(got - want).max() <= 1e-3


def test_split_qkv_golden(manifest):
    m = manifest["split_qkv"]
    p = m["params"]
    q, k, v = O.split_qkv(load_golden(m["qkv"]), p["dim"], p["n_rows"])
    np.testing.assert_array_equal(q, load_golden(m["q"]))
    np.testing.assert_array_equal(k, load_golden(m["k"]))
    np.testing.assert_array_equal(v, load_golden(m["v"]))


def test_block_golden(manifest):
    m = manifest["block_flux"]
    p = m["params"]
    got = O.attention_block(load_golden(m["q"]), load_golden(m["k"]), load_golden(m["v"]),
                            p["H"], p["D"], p["scale"], eps=p["eps"],
                            q_gain=load_golden(m["q_gain"]), k_gain=load_golden(m["k_gain"]),
                            split_row=p["split"], cos=load_golden(m["cos"]),
                            sin=load_golden(m["sin"]))
    np.testing.assert_allclose(got, load_golden(m["out"]), rtol=0, atol=5e-6)


def test_fa2_vs_f64_error_budget():
    """The reference's fp16 operand rounding stays well inside the 2e-3 bar
    against exact fp64 attention; this is the budget the B200 path shares."""
    rng = np.random.default_rng(11)
    H, S, D = 2, 300, 128
    q = rng.standard_normal((H, S, D), dtype=np.float32)
    k = rng.standard_normal((H, S, D), dtype=np.float32)
    v = rng.standard_normal((H, S, D), dtype=np.float32)
    sc = 1 / np.sqrt(128)
    fa = O.flash_attention_v2(q, k, v, D, H, S, sc).reshape(S, H, D).transpose(1, 0, 2)
    ex = O.attention_f64(q, k, v, D, H, S, sc)
    err = np.abs(fa - ex)
    assert err.max() < 2e-3 and err.mean() < 2e-4


def test_spatial_is_exact_fp32():
    rng = np.random.default_rng(12)
    H, S, D = 2, 200, 64
    q = rng.standard_normal((H, S, D), dtype=np.float32)
    k = rng.standard_normal((H, S, D), dtype=np.float32)
    v = rng.standard_normal((H, S, D), dtype=np.float32)
    sp = O.spatial_attention(q, k, v, D, H, S, 0.125)
    ex = O.attention_f64(q, k, v, D, H, S, 0.125)
    assert np.abs(sp - ex).max() < 1e-5


def test_row_subsets_match_full():
    rng = np.random.default_rng(13)
    H, S, D = 2, 70, 128
    q = rng.standard_normal((H, S, D), dtype=np.float32)
    full = O.flash_attention_v2(q, q, q, D, H, S, 0.1)
    part = O.flash_attention_v2(q, q, q, D, H, S, 0.1, qb_range=(1, 3))
    np.testing.assert_array_equal(part[16:48], full[16:48])
    assert np.all(part[:16] == 0) and np.all(part[48:] == 0)
