"""The oracle against golden vectors produced by the reference (CPU only).

Pins every oracle function used as a checker by the GPU parity tests.
"""
import math

import numpy as np
import pytest

import inputs as gi
from oracle import tq_oracle as O

GOLD = "tests/golden/"


@pytest.fixture(scope="module")
def books():
    z = np.load(GOLD + "codebooks.npz")
    return {(d, b): (z[f"c{d}_{b}"], z[f"b{d}_{b}"]) for d in gi.CODEBOOK_DIMS
            for b in range(1, 9)}


@pytest.mark.parametrize("d,b", [(32, 1), (64, 3), (128, 2), (128, 4), (128, 8), (256, 5)])
def test_lloyd_max_bit_exact(books, d, b):
    c, bd = O.solve_lloyd_max(d, b)
    assert np.array_equal(c, books[(d, b)][0])
    assert np.array_equal(bd, books[(d, b)][1])


def test_codebook_properties(books):
    # reference tests: test_inference.py:26-48
    c, bd = books[(128, 4)]
    assert c.shape == (16,) and bd.shape == (15,)
    assert np.all(np.diff(c) > 0) and np.all(np.diff(bd) > 0)
    rng = np.random.Generator(np.random.PCG64(0))
    x = (rng.standard_normal(10000) / math.sqrt(128)).astype(np.float32)
    xh = c[np.abs(x[:, None] - c[None]).argmin(-1)]
    assert ((x - xh) ** 2).mean() < (1 / 128) * 2 ** -8 * math.pi ** 2 / 3 * 4


def test_rotation_bit_exact():
    z = np.load(GOLD + "rotations.npz")
    for d, s in gi.ROTATION_CASES:
        R = O.rotation_matrix(d, s)
        assert np.array_equal(R, z[f"R{d}_{s}"]), (d, s)
        assert np.allclose(R @ R.T, np.eye(d), atol=1e-5)


def test_bucketize_edges_bit_exact(books):
    z = np.load(GOLD + "quantize_edges.npz")
    for d, b in gi.EDGE_CASES:
        y = z[f"y{d}_{b}"]
        assert np.array_equal(O.bucketize(y, books[(d, b)][1]), z[f"idx{d}_{b}"]), (d, b)


def _unpack_nibbles(p, shape):
    a = np.empty(p.size * 2, np.uint8)
    a[0::2] = p & 15
    a[1::2] = p >> 4
    return a[: int(np.prod(shape))].reshape(shape)


def test_config1_pipeline(books):
    z = np.load(GOLD + "config1.npz")
    k, v, q = gi.config1_inputs()
    np.testing.assert_allclose(z["input_checksum"],
                               [k.sum(dtype=np.float64), v.sum(dtype=np.float64),
                                q.sum(dtype=np.float64)], rtol=0, atol=0)
    c = O.TurboQuantCache(1, 64, 3, 3, residual_window=0, protected_layers=0,
                          dtype="float32", codebooks=books)
    fk, fv = c.update(k, v, 0)
    st = c.stores[0]
    shape = tuple(z["idx_shape"])
    assert np.array_equal(np.stack(st.k_idx), _unpack_nibbles(z["k_idx_packed"], shape))
    assert np.array_equal(np.stack(st.v_idx), _unpack_nibbles(z["v_idx_packed"], shape))
    assert np.array_equal(np.stack(st.k_norm), z["k_norm"])
    assert np.array_equal(np.stack(st.v_norm), z["v_norm"])
    # quantising the reference's own rotated tensor is bit-exact
    cb3 = books[(64, 3)][1]
    assert np.array_equal(O.bucketize(z["yk_sub"], cb3), np.stack(st.k_idx)[:64])
    assert np.array_equal(O.bucketize(z["yv_sub"], cb3), np.stack(st.v_idx)[:64])
    np.testing.assert_allclose(fk[:, :, :64], z["fk_sub"], atol=5e-5)
    np.testing.assert_allclose(fv[:, :, :64], z["fv_sub"], atol=5e-5)
    np.testing.assert_allclose(fk.sum(-1), z["fk_rowsum"], atol=5e-4)
    np.testing.assert_allclose((fv * fv).sum(-1), z["fv_rowsq"], rtol=1e-5)
    o = O.sdpa(q, fk, fv)
    np.testing.assert_allclose(o, z["out_tq"], atol=1e-4)
    np.testing.assert_allclose(O.sdpa(q, k, v), z["out_fp32"], atol=1e-4)


def test_incremental_window_and_protected(books):
    z = np.load(GOLD + "incremental.npz")
    s = gi.INCREMENTAL
    c = O.TurboQuantCache(s["num_layers"], s["D"], s["key_bits"], s["value_bits"],
                          residual_window=s["residual_window"],
                          protected_layers=s["protected_layers"], dtype="float32",
                          codebooks=books)
    for layer in s["layers"]:
        chunks = gi.incremental_inputs(layer)
        for step, (kc, vc) in enumerate(chunks):
            ok, ov = c.update(kc, vc, layer)
            if f"L{layer}_s{step}_k" in z.files:
                np.testing.assert_allclose(ok, z[f"L{layer}_s{step}_k"], atol=5e-5)
                np.testing.assert_allclose(ov, z[f"L{layer}_s{step}_v"], atol=5e-5)
            else:
                np.testing.assert_allclose(ok.sum(-1), z[f"L{layer}_s{step}_krow"], atol=5e-4)
        st = c.stores[layer]
        assert [st.key_bits, st.value_bits] == list(z[f"L{layer}_bits"])
        assert st.comp_tokens == int(z[f"L{layer}_comp"][0])
        assert np.array_equal(np.stack(st.k_idx), z[f"L{layer}_k_idx"])
        assert np.array_equal(np.stack(st.v_idx), z[f"L{layer}_v_idx"])


def test_bf16_case(books):
    z = np.load(GOLD + "bf16_case.npz")
    s = gi.BF16_CASE
    k, v, q = gi.bf16_case_inputs()
    c = O.TurboQuantCache(1, s["D"], s["key_bits"], s["value_bits"], residual_window=0,
                          protected_layers=0, dtype="bfloat16", codebooks=books)
    fk, fv = c.update(k, v, 0)
    st = c.stores[0]
    ki = np.stack(st.k_idx)
    assert (ki == z["k_idx"]).mean() > 0.9999
    assert np.array_equal(np.stack(st.k_norm), z["k_norm"])
    rk = (z["fk_bits"].astype(np.uint32) << 16).view(np.float32)
    # dequantised values are the same bf16 number or one bf16 ulp apart
    assert np.abs(fk - rk).max() <= 2 ** -7 * np.abs(rk).max()
    o = O.sdpa(q, fk, fv, out_dtype="bfloat16")
    np.testing.assert_allclose(o, z["out_tq"], atol=2e-2)


# ---------------------------------------------------------------------------
# build-defined parts: packing round trips, QJL properties
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("D", [32, 64, 128, 256])
def test_orders_are_permutations(D):
    for order in (O.k_order(D), O.v_order(D)):
        assert sorted(order.tolist()) == list(range(D))
    assert sorted(O.qjl_bit_positions(D).tolist()) == list(range(D))


@pytest.mark.parametrize("D,kb,vb,qjl", [(128, 4, 2, True), (128, 3, 3, False),
                                         (64, 3, 3, True), (32, 6, 4, False),
                                         (64, 5, 5, True), (128, 8, 8, False)])
def test_pages_round_trip(D, kb, vb, qjl):
    rng = np.random.Generator(np.random.PCG64(D * 100 + kb * 10 + vb))
    S, T = 3, 150
    geom = O.PageGeom(D, kb, vb, qjl)
    ki = rng.integers(0, 2 ** kb, (S, T, D)).astype(np.int16)
    vi = rng.integers(0, 2 ** vb, (S, T, D)).astype(np.int16)
    kn = rng.random((S, T)).astype(np.float16)
    vn = rng.random((S, T)).astype(np.float16)
    qb = rng.integers(0, 2, (S, T, D)).astype(np.uint8) if qjl else None
    gm = rng.random((S, T)).astype(np.float16) if qjl else None
    pages = O.build_pages(geom, ki, vi, kn, vn, qb, gm)
    assert pages.shape == (S, 3, geom.page_bytes)
    assert geom.page_bytes % 16 == 0
    back = O.parse_pages(geom, pages, T)
    assert np.array_equal(back["k_idx"], ki) and np.array_equal(back["v_idx"], vi)
    assert np.array_equal(back["k_norm"], kn) and np.array_equal(back["v_norm"], vn)
    if qjl:
        assert np.array_equal(back["qbits"], qb) and np.array_equal(back["gamma"], gm)


def test_page_bytes_formula():
    # 118 B per token-head for K4+QJL / V2 at D=128 (packed-KV bytes of the
    # Mixtral decode workload) and for K3+QJL / V3
    assert O.PageGeom(128, 4, 2, True).bytes_per_token() == 118
    assert O.PageGeom(128, 3, 3, True).bytes_per_token() == 118
    assert O.PageGeom(128, 3, 3, False).bytes_per_token() == 100
    assert O.PageGeom(64, 3, 3, False).bytes_per_token() == 52


def test_codes_attention_matches_dense_sdpa(books):
    """Attention evaluated from codes in the rotated basis equals SDPA over the
    dequantised K/V (no QJL, no window)."""
    rng = np.random.Generator(np.random.PCG64(3))
    B, Hkv, g, T, D = 2, 2, 4, 70, 64
    kc, kb = books[(D, 4)]
    vc, vb = books[(D, 2)]
    R = O.rotation_matrix(D, 42)
    k = rng.standard_normal((B, Hkv, T, D)).astype(np.float32)
    v = rng.standard_normal((B, Hkv, T, D)).astype(np.float32)
    q = rng.standard_normal((B, Hkv * g, D)).astype(np.float32)
    ki, kn, _ = O.compress(k.reshape(B * Hkv, T, D), R, kb)
    vi, vn, _ = O.compress(v.reshape(B * Hkv, T, D), R, vb)
    o1 = O.decode_attention_codes(q, ki, vi, kn, vn, kc, vc, R)
    fk = O.decode_range(ki, kn, kc, R).reshape(B, Hkv, T, D)
    fv = O.decode_range(vi, vn, vc, R).reshape(B, Hkv, T, D)
    o2 = O.sdpa(q[:, :, None], fk, fv)[:, :, 0]
    np.testing.assert_allclose(o1, o2, atol=2e-5)


def test_qjl_estimator_unbiased(books):
    """E over sketch matrices of the QJL-corrected score equals <q, k>."""
    rng = np.random.Generator(np.random.PCG64(11))
    D = 64
    kc, kb = books[(D, 2)]
    R = O.rotation_matrix(D, 42)
    k = rng.standard_normal((1, D)).astype(np.float32)
    q = rng.standard_normal(D).astype(np.float32)
    ki, kn, y = O.compress(k, R, kb)
    exact = float(q @ k[0])
    mse_only = float(kn[0]) * float((q @ R.T) @ kc[ki[0].astype(np.int64)])
    est = []
    for s in range(400):
        S = rng.standard_normal((D, D)).astype(np.float32)
        bits, gam = O.qjl_sketch(y, ki, kc, kn.astype(np.float32), S)
        qr = (q @ R.T).astype(np.float64)
        corr = O.qjl_alpha(D) * float(gam[0]) * float((S.astype(np.float64) @ qr) @ (2.0 * bits[0] - 1))
        est.append(mse_only + corr)
    est = np.array(est)
    se = est.std() / math.sqrt(len(est))
    assert abs(est.mean() - exact) < 4 * se + 1e-3
    assert abs(est.mean() - exact) < abs(mse_only - exact) + 4 * se
