"""GPU parity: the CUDA kernels (through the C ABI) against the oracle and the
reference's golden vectors.

Tolerances:
  * codes from tq_quantize_rotated: bit-exact (same rotated fp32 input)
  * codes from the fused append: >= 99.99 % identical to the oracle; every
    mismatch sits within 1e-5 of a boundary (the rotation is an fp32 dot
    product whose rounding differs from a CPU BLAS sgemm)
  * dequantised K/V and attention outputs vs the reference: max-abs <= 1e-2
    and cosine >= 0.999 (the reference rounds dequantised K/V to bf16)
  * decode attention vs the oracle evaluated on the kernel's own codes:
    cosine >= 0.9999 and max-abs <= 2e-3 * max|o| (fp16 MMA operands)
"""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import inputs as gi
from bhaskera_col_b200.inference import TurboQuantKVCache, ops
from bhaskera_col_b200.inference.kv_cache import (FastLloydMaxCodebook, _generate_qjl_matrix,
                                                  _generate_rotation_matrix)
from oracle import tq_oracle as O

pytestmark = pytest.mark.gpu
GOLD = "tests/golden/"
DEV = torch.device("cuda:0")


@pytest.fixture(scope="module")
def books():
    z = np.load(GOLD + "codebooks.npz")
    return {(d, b): (z[f"c{d}_{b}"], z[f"b{d}_{b}"]) for d in gi.CODEBOOK_DIMS
            for b in range(1, 9)}


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def make_tables(D, kb, vb, qjl, seed=42):
    kc = FastLloydMaxCodebook.get(D, kb, DEV)
    vc = FastLloydMaxCodebook.get(D, vb, DEV)
    R = _generate_rotation_matrix(D, seed, DEV).contiguous()
    S = _generate_qjl_matrix(D, seed, DEV).contiguous() if qjl else None
    return ops.LayerTables(D, kb, vb, qjl, kc.centroids, kc.boundaries, vc.centroids,
                           vc.boundaries, R, S)


def rand_kv(shape, seed, dtype=torch.bfloat16, outliers=2):
    rng = np.random.Generator(np.random.PCG64(seed))
    x = gi.outlier_normal(rng, shape, outliers, 8.0)
    return torch.from_numpy(x).to(dtype)


def new_pages(S, T, tables):
    P = -(-T // 64)
    pb = ops.page_bytes(tables.head_dim, tables.key_bits, tables.value_bits, tables.qjl)
    return torch.zeros((S, P, pb), dtype=torch.uint8, device=DEV)


def parse(tables, pages, T):
    geom = O.PageGeom(tables.head_dim, tables.key_bits, tables.value_bits, tables.qjl)
    return geom, O.parse_pages(geom, pages.cpu().numpy(), T)


# ----------------------------------------------------------------- quantiser
def test_quantize_rotated_golden_edges(books):
    z = np.load(GOLD + "quantize_edges.npz")
    for d, b in gi.EDGE_CASES:
        y = torch.from_numpy(z[f"y{d}_{b}"]).to(DEV)
        bd = torch.from_numpy(books[(d, b)][1]).to(DEV)
        got = ops.quantize_rotated(y, bd).cpu().numpy()
        assert np.array_equal(got, z[f"idx{d}_{b}"]), (d, b)


def test_quantize_rotated_golden_config1(books):
    z = np.load(GOLD + "config1.npz")
    bd = torch.from_numpy(books[(64, 3)][1]).to(DEV)
    shape = tuple(z["idx_shape"])
    a = np.empty(z["k_idx_packed"].size * 2, np.uint8)
    a[0::2], a[1::2] = z["k_idx_packed"] & 15, z["k_idx_packed"] >> 4
    kidx = a[: int(np.prod(shape))].reshape(shape)
    got = ops.quantize_rotated(torch.from_numpy(z["yk_sub"]).to(DEV), bd).cpu().numpy()
    assert np.array_equal(got, kidx[:64])


def test_quantize_rotated_matches_bucketize_large():
    g = torch.Generator(device=DEV)
    g.manual_seed(5)
    y = torch.randn(3_000_001, device=DEV, generator=g) / 8.0
    for bits in (1, 3, 4, 8):
        bd = FastLloydMaxCodebook.get(64, bits, DEV).boundaries
        assert torch.equal(ops.quantize_rotated(y, bd).long(), torch.bucketize(y, bd))


# ------------------------------------------------------------------- append
APPEND_CASES = [(128, 4, 2, True, torch.bfloat16), (128, 3, 3, False, torch.float16),
                (64, 3, 3, False, torch.float32), (64, 4, 2, True, torch.bfloat16),
                (32, 6, 4, True, torch.float32), (128, 8, 8, False, torch.bfloat16),
                (128, 5, 5, True, torch.bfloat16)]


@pytest.mark.parametrize("D,kb,vb,qjl,dtype", APPEND_CASES)
def test_append_matches_oracle(D, kb, vb, qjl, dtype):
    B, H, T1, T2 = 2, 3, 100, 37
    t = make_tables(D, kb, vb, qjl)
    k = rand_kv((B, H, T1 + T2, D), 1, dtype)
    v = rand_kv((B, H, T1 + T2, D), 2, dtype)
    pages = new_pages(B * H, T1 + T2, t)
    kd, vd = k.to(DEV), v.to(DEV)
    ops.append(t, pages, kd[:, :, :T1], vd[:, :, :T1], 0)
    # second chunk from a transposed (non-contiguous) view: strides honoured
    k2 = kd[:, :, T1:].transpose(1, 2).contiguous().transpose(1, 2)
    ops.append(t, pages, k2, vd[:, :, T1:], T1)
    torch.cuda.synchronize()
    geom, got = parse(t, pages, T1 + T2)
    # byte-exact layout: re-packing the parsed fields reproduces the pages
    rebuilt = O.build_pages(geom, got["k_idx"], got["v_idx"], got["k_norm"], got["v_norm"],
                            got.get("qbits"), got.get("gamma"))
    assert np.array_equal(rebuilt, pages.cpu().numpy())

    R = t.rot.cpu().numpy()
    kc, kb_ = t.k_centroids.cpu().numpy(), t.k_boundaries.cpu().numpy()
    vb_ = t.v_boundaries.cpu().numpy()
    kx = k.float().numpy().reshape(B * H, T1 + T2, D)
    vx = v.float().numpy().reshape(B * H, T1 + T2, D)
    ki, kn, ky = O.compress(kx, R, kb_)
    vi, vn, vy = O.compress(vx, R, vb_)
    for got_i, want_i, y, bd in ((got["k_idx"], ki, ky, kb_), (got["v_idx"], vi, vy, vb_)):
        agree = (got_i == want_i)
        assert agree.mean() >= 0.9999, agree.mean()
        if not agree.all():   # mismatches only at boundaries
            dist = np.abs(y[~agree][:, None] - bd[None, :]).min(-1)
            assert dist.max() < 1e-5
    assert (got["k_norm"] == kn).mean() >= 0.999
    assert (got["v_norm"] == vn).mean() >= 0.999
    np.testing.assert_allclose(got["k_norm"].astype(np.float32), kn.astype(np.float32),
                               rtol=1e-3)
    if qjl:
        S = _generate_qjl_matrix(D, 42).numpy()
        bits, gam = O.qjl_sketch(ky, got["k_idx"], kc, kn.astype(np.float32), S)
        assert (got["qbits"] == bits).mean() >= 0.999
        np.testing.assert_allclose(got["gamma"].astype(np.float32), gam.astype(np.float32),
                                   rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize("D,kb,vb", [(128, 4, 2), (64, 3, 3), (32, 6, 4)])
def test_dequantize_matches_oracle(D, kb, vb):
    B, H, T = 2, 2, 130
    t = make_tables(D, kb, vb, False)
    k, v = rand_kv((B, H, T, D), 3), rand_kv((B, H, T, D), 4)
    pages = new_pages(B * H, T, t)
    ops.append(t, pages, k.to(DEV), v.to(DEV), 0)
    ko = torch.empty((B, H, T - 5, D), dtype=torch.float32, device=DEV)
    vo = torch.empty_like(ko)
    ops.dequantize(t, pages, 5, T, ko, vo)
    torch.cuda.synchronize()
    _, got = parse(t, pages, T)
    R = t.rot.cpu().numpy()
    wk = O.decode_range(got["k_idx"], got["k_norm"], t.k_centroids.cpu().numpy(), R)
    wv = O.decode_range(got["v_idx"], got["v_norm"], t.v_centroids.cpu().numpy(), R)
    np.testing.assert_allclose(ko.cpu().numpy().reshape(B * H, T - 5, D), wk[:, 5:],
                               atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(vo.cpu().numpy().reshape(B * H, T - 5, D), wv[:, 5:],
                               atol=1e-5, rtol=1e-5)


# ------------------------------------------------------------ decode kernel
DECODE_CASES = [
    # D, kb, vb, qjl, B, Hkv, g, T, W
    (128, 4, 2, True, 2, 2, 4, 300, 0),
    (128, 4, 2, False, 2, 2, 4, 300, 0),
    (128, 3, 3, False, 1, 2, 5, 1000, 0),
    (128, 3, 3, True, 1, 1, 5, 64, 0),
    (128, 2, 2, False, 3, 1, 1, 65, 0),
    (128, 4, 4, False, 1, 2, 16, 130, 0),
    (128, 4, 4, True, 2, 2, 4, 200, 5),
    (128, 6, 4, True, 1, 2, 8, 200, 7),
    (128, 5, 5, False, 2, 1, 3, 17, 16),
    (128, 8, 8, False, 1, 1, 2, 90, 0),
    (64, 3, 3, False, 1, 4, 4, 512, 0),
    (64, 4, 2, True, 2, 1, 71, 150, 5),
    (32, 4, 2, False, 1, 2, 2, 40, 8),
    (32, 6, 4, True, 1, 2, 1, 1, 0),
    (128, 4, 2, False, 1, 2, 4, 0, 9),
]


@pytest.mark.parametrize("D,kb,vb,qjl,B,Hkv,g,T,W", DECODE_CASES)
def test_decode_matches_oracle(D, kb, vb, qjl, B, Hkv, g, T, W):
    t = make_tables(D, kb, vb, qjl)
    S = B * Hkv
    k, v = rand_kv((B, Hkv, max(T, 1), D), 5), rand_kv((B, Hkv, max(T, 1), D), 6)
    pages = new_pages(S, max(T, 64), t)
    if T:
        ops.append(t, pages, k[:, :, :T].to(DEV), v[:, :, :T].to(DEV), 0)
    q = rand_kv((B, Hkv * g, 1, D), 7, outliers=0)
    wk = rand_kv((B, Hkv, W, D), 8) if W else None
    wv = rand_kv((B, Hkv, W, D), 9) if W else None
    out = ops.decode_attention(t, pages, q.to(DEV), T,
                               wk.to(DEV) if W else None, wv.to(DEV) if W else None)
    ws_ok = torch.cuda.synchronize() is None
    assert ws_ok
    _, got = parse(t, pages, T)
    Smat = _generate_qjl_matrix(D, 42).numpy() if qjl else None
    want = O.decode_attention_codes(
        q[:, :, 0].float().numpy(), got["k_idx"], got["v_idx"], got["k_norm"], got["v_norm"],
        t.k_centroids.cpu().numpy(), t.v_centroids.cpu().numpy(), t.rot.cpu().numpy(),
        qbits=got.get("qbits"), gamma=got.get("gamma"), S=Smat, T=T,
        window_k=wk.float().numpy() if W else None, window_v=wv.float().numpy() if W else None)
    o = out[:, :, 0].float().cpu().numpy()
    bf = 2 ** -8 * np.abs(want).max()          # output is bf16
    assert np.abs(o - want).max() <= 2e-3 * np.abs(want).max() + bf
    assert cosine(o, want) >= 0.9999


@pytest.mark.parametrize("D,kb,vb,qjl,W", [(128, 4, 2, True, 0), (128, 4, 2, False, 7),
                                            (128, 3, 3, False, 0), (64, 4, 4, False, 5)])
def test_decode_left_padding_matches_oracle(D, kb, vb, qjl, W):
    """kv_start: each row's keys before its first real position (packed and
    window alike) take no weight; a row with nothing left returns zeros."""
    B, Hkv, g, T = 4, 2, 4, 300
    t = make_tables(D, kb, vb, qjl)
    k, v = rand_kv((B, Hkv, T, D), 61), rand_kv((B, Hkv, T, D), 62)
    pages = new_pages(B * Hkv, T, t)
    ops.append(t, pages, k.to(DEV), v.to(DEV), 0)
    q = rand_kv((B, Hkv * g, 1, D), 63, outliers=0)
    wk = rand_kv((B, Hkv, W, D), 64) if W else None
    wv = rand_kv((B, Hkv, W, D), 65) if W else None
    start = [0, 37, 299, T + W]                 # the last row: everything is padding
    ks = torch.tensor(start, dtype=torch.int32, device=DEV)
    ws = ops.DecodeWorkspace()
    out = ops.decode_attention(t, pages, q.to(DEV), T, wk.to(DEV) if W else None,
                               wv.to(DEV) if W else None, workspace=ws, kv_start=ks)
    torch.cuda.synchronize()
    assert ws.status() == 0
    _, got = parse(t, pages, T)
    Smat = _generate_qjl_matrix(D, 42).numpy() if qjl else None
    want = O.decode_attention_codes(
        q[:, :, 0].float().numpy(), got["k_idx"], got["v_idx"], got["k_norm"], got["v_norm"],
        t.k_centroids.cpu().numpy(), t.v_centroids.cpu().numpy(), t.rot.cpu().numpy(),
        qbits=got.get("qbits"), gamma=got.get("gamma"), S=Smat, T=T,
        window_k=wk.float().numpy() if W else None, window_v=wv.float().numpy() if W else None,
        kv_start=start)
    o = out[:, :, 0].float().cpu().numpy()
    assert np.abs(o[3]).max() == 0.0
    bf = 2 ** -8 * np.abs(want).max()
    assert np.abs(o - want).max() <= 2e-3 * np.abs(want).max() + bf
    assert cosine(o[:3], want[:3]) >= 0.9999


def test_decode_no_device_errors_and_split_independence():
    """Results do not depend on how the page space is split across CTAs."""
    D, B, Hkv, g, T = 128, 2, 4, 4, 2000
    t = make_tables(D, 4, 2, True)
    pages = new_pages(B * Hkv, T, t)
    ops.append(t, pages, rand_kv((B, Hkv, T, D), 10).to(DEV),
               rand_kv((B, Hkv, T, D), 11).to(DEV), 0)
    q = rand_kv((B, Hkv * g, 1, D), 12, outliers=0).to(DEV)
    ws = ops.DecodeWorkspace()
    outs = [ops.decode_attention(t, pages, q, T, workspace=ws, num_ctas=n).float()
            for n in (1, 7, 64, 0)]
    for o in outs[1:]:
        assert torch.allclose(o, outs[0], atol=2e-2 * outs[0].abs().max().item())
    assert ws.status() == 0


# ------------------------------------------------ cache API vs the reference
def test_config1_end_to_end():
    """B1 Hq16 Hkv4 D64 T512, fp32, K3/V3: dense update() output and the fused
    attend() output against the reference's own path."""
    z = np.load(GOLD + "config1.npz")
    k, v, q = gi.config1_inputs()
    cache = TurboQuantKVCache(num_layers=1, batch_size=1, num_heads=4, head_dim=64,
                              key_bits=3, value_bits=3, residual_window=0,
                              protected_layers=0, dtype=torch.float32, device=DEV,
                              max_seq_len=512)
    fk, fv = cache.update(torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV), 0)
    fk, fv = fk.cpu().numpy(), fv.cpu().numpy()
    assert np.abs(fk[:, :, :64] - z["fk_sub"]).max() <= 1e-2
    assert cosine(fk[:, :, :64], z["fk_sub"]) >= 0.999
    assert np.abs(fk.sum(-1) - z["fk_rowsum"]).max() <= 5e-2
    assert np.abs((fv * fv).sum(-1) - z["fv_rowsq"]).max() <= 1e-2 * np.abs(z["fv_rowsq"]).max()
    o = cache.attend(torch.from_numpy(q).to(DEV), 0).cpu().numpy()
    assert np.abs(o - z["out_tq"]).max() <= 1e-2 * max(1.0, np.abs(z["out_tq"]).max())
    assert cosine(o, z["out_tq"]) >= 0.999
    od = F.scaled_dot_product_attention(torch.from_numpy(q), torch.from_numpy(fk),
                                        torch.from_numpy(fv), enable_gqa=True).numpy()
    assert cosine(od, z["out_tq"]) >= 0.9999
    assert cache.device_status() == 0


def test_incremental_window_protected_vs_reference():
    z = np.load(GOLD + "incremental.npz")
    s = gi.INCREMENTAL
    cache = TurboQuantKVCache(num_layers=s["num_layers"], batch_size=s["B"], num_heads=s["H"],
                              head_dim=s["D"], key_bits=s["key_bits"],
                              value_bits=s["value_bits"], residual_window=s["residual_window"],
                              protected_layers=s["protected_layers"], dtype=torch.float32,
                              device=DEV, max_seq_len=s["max_seq_len"])
    for layer in s["layers"]:
        chunks = gi.incremental_inputs(layer)
        for step, (kc, vc) in enumerate(chunks):
            ok, ov = cache.update(torch.from_numpy(kc).to(DEV), torch.from_numpy(vc).to(DEV),
                                  layer)
            ok, ov = ok.cpu().numpy(), ov.cpu().numpy()
            if f"L{layer}_s{step}_k" in z.files:
                ref_k, ref_v = z[f"L{layer}_s{step}_k"], z[f"L{layer}_s{step}_v"]
                assert ok.shape == ref_k.shape
                assert np.abs(ok - ref_k).max() <= 1e-2 and cosine(ok, ref_k) >= 0.999
                assert np.abs(ov - ref_v).max() <= 1e-2 and cosine(ov, ref_v) >= 0.999
            else:
                assert np.abs(ok.sum(-1) - z[f"L{layer}_s{step}_krow"]).max() <= 5e-2
        st = cache._stores[layer]
        assert [st.key_bits, st.value_bits] == list(z[f"L{layer}_bits"])
        assert st._comp_ptr == int(z[f"L{layer}_comp"][0])
    stats = cache.compression_stats()
    assert set(stats) == {"tq_mb", "bf16_mb", "compression_ratio", "seq_len"}
    assert stats["seq_len"] == s["prefill"] + s["decode_steps"]
    cache.reset()
    assert cache.seq_len == 0


def test_bf16_case_vs_reference():
    z = np.load(GOLD + "bf16_case.npz")
    s = gi.BF16_CASE
    k, v, q = gi.bf16_case_inputs()
    cache = TurboQuantKVCache(num_layers=1, batch_size=s["B"], num_heads=s["Hkv"],
                              head_dim=s["D"], key_bits=s["key_bits"],
                              value_bits=s["value_bits"], residual_window=0,
                              protected_layers=0, dtype=torch.bfloat16, device=DEV,
                              max_seq_len=s["T"])
    fk, fv = cache.update(torch.from_numpy(k).to(DEV, torch.bfloat16),
                          torch.from_numpy(v).to(DEV, torch.bfloat16), 0)
    rk = (z["fk_bits"].astype(np.uint32) << 16).view(np.float32)
    rv = (z["fv_bits"].astype(np.uint32) << 16).view(np.float32)
    fk, fv = fk.float().cpu().numpy(), fv.float().cpu().numpy()
    assert np.abs(fk - rk).max() <= 1e-2 * max(1.0, np.abs(rk).max())
    assert cosine(fk, rk) >= 0.999 and cosine(fv, rv) >= 0.999
    qd = torch.from_numpy(q).to(DEV, torch.bfloat16)
    o = cache.attend(qd, 0).float().cpu().numpy()
    assert np.abs(o - z["out_tq"]).max() <= 1e-2 * max(1.0, np.abs(z["out_tq"]).max())
    assert cosine(o, z["out_tq"]) >= 0.999


@pytest.mark.parametrize("rw", [0, 16])
def test_fused_attend_equals_sdpa_on_dense(rw):
    B, Hkv, g, T, D = 4, 8, 4, 1000, 128
    cache = TurboQuantKVCache(num_layers=2, batch_size=B, num_heads=Hkv, head_dim=D,
                              key_bits=4, value_bits=2, residual_window=rw,
                              protected_layers=0, dtype=torch.bfloat16, device=DEV,
                              max_seq_len=T)
    k, v = rand_kv((B, Hkv, T, D), 20).to(DEV), rand_kv((B, Hkv, T, D), 21).to(DEV)
    fk, fv = cache.update(k[:, :, :-3], v[:, :, :-3], 1)
    for i in range(3, 0, -1):   # decode steps
        fk, fv = cache.update(k[:, :, -i:T - i + 1], v[:, :, -i:T - i + 1], 1)
    assert fk.shape[2] == T
    q = rand_kv((B, Hkv * g, 1, D), 22, outliers=0).to(DEV)
    want = F.scaled_dot_product_attention(q.float(), fk.float(), fv.float(), enable_gqa=True)
    got = cache.attend(q, 1).float()
    assert cosine(got.cpu(), want.cpu()) >= 0.999
    assert (got - want).abs().max().item() <= 1e-2 * max(1.0, want.abs().max().item())


def test_full_size_mixtral_decode_property():
    """Mixtral decode shapes (B16, Hq32, Hkv8, D128, T8192, K4/V2): the fused
    kernel equals dense SDPA over the kernel's own dequantised K/V."""
    B, Hkv, g, T, D = 16, 8, 4, 8192, 128
    t = make_tables(D, 4, 2, False)
    pages = new_pages(B * Hkv, T, t)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(0)
    for c0 in range(0, T, 2048):
        kk = torch.randn((B, Hkv, 2048, D), device=DEV, generator=gen).to(torch.bfloat16)
        vv = torch.randn((B, Hkv, 2048, D), device=DEV, generator=gen).to(torch.bfloat16)
        ops.append(t, pages, kk, vv, c0)
    q = torch.randn((B, Hkv * g, 1, D), device=DEV, generator=gen).to(torch.bfloat16)
    got = ops.decode_attention(t, pages, q, T).float()
    dk = torch.empty((B, Hkv, T, D), dtype=torch.float32, device=DEV)
    dv = torch.empty_like(dk)
    ops.dequantize(t, pages, 0, T, dk, dv)
    want = F.scaled_dot_product_attention(q.float(), dk, dv, enable_gqa=True)
    assert cosine(got.cpu(), want.cpu()) >= 0.9995
    assert (got - want).abs().max().item() <= 1e-2


def test_full_size_headline_decode_step_matches_oracle():
    """The headline configuration exactly as bench.py runs it: B16, Hq32/Hkv8,
    D128, 8192 tokens, K4 + QJL / V2, bf16 K/V ~ N(0,1) with 2 of 128 channels
    x8, the last token stored by the fused decode step.  Rows 0, 7 and 15 (24
    streams) are compared with the oracle evaluated on the kernel's own codes
    and QJL bits, at the small cases' tolerance."""
    B, Hkv, g, T, D = 16, 8, 4, 8192, 128
    t = make_tables(D, 4, 2, True)
    pages = new_pages(B * Hkv, T, t)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(3)
    sc = torch.ones(D, device=DEV)
    sc[torch.randperm(D, generator=torch.Generator().manual_seed(7))[:2].to(DEV)] = 8.0
    for c0 in range(0, T, 2048):
        n = min(2048, T - 1 - c0)
        kk = (torch.randn((B, Hkv, n, D), device=DEV, generator=gen) * sc).to(torch.bfloat16)
        vv = (torch.randn((B, Hkv, n, D), device=DEV, generator=gen) * sc).to(torch.bfloat16)
        ops.append(t, pages, kk, vv, c0)
    k1 = (torch.randn((B, Hkv, 1, D), device=DEV, generator=gen) * sc).to(torch.bfloat16)
    v1 = (torch.randn((B, Hkv, 1, D), device=DEV, generator=gen) * sc).to(torch.bfloat16)
    q = (torch.randn((B, Hkv * g, 1, D), device=DEV, generator=gen) * sc).to(torch.bfloat16)
    ws = ops.DecodeWorkspace()
    out = ops.decode_step(t, pages, k1, v1, T - 1, q, workspace=ws)
    torch.cuda.synchronize()
    assert ws.status() == 0
    rows = [0, 7, 15]
    streams = [b * Hkv + h for b in rows for h in range(Hkv)]
    _, got = parse(t, pages[streams], T)
    Smat = _generate_qjl_matrix(D, 42).numpy()
    want = O.decode_attention_codes(
        q[rows, :, 0].float().cpu().numpy(), got["k_idx"], got["v_idx"], got["k_norm"],
        got["v_norm"], t.k_centroids.cpu().numpy(), t.v_centroids.cpu().numpy(),
        t.rot.cpu().numpy(), qbits=got["qbits"], gamma=got["gamma"], S=Smat, T=T)
    o = out[rows, :, 0].float().cpu().numpy()
    bf = 2 ** -8 * np.abs(want).max()          # output is bf16
    assert np.abs(o - want).max() <= 2e-3 * np.abs(want).max() + bf
    assert cosine(o, want) >= 0.9999


# ------------------------------------------------------- fused decode step
@pytest.mark.parametrize("D,kb,vb,qjl,B,Hkv,g,T,W", [
    (128, 4, 2, True, 2, 4, 4, 300, 0), (128, 3, 3, False, 1, 2, 5, 64, 0),
    (64, 4, 2, True, 1, 2, 8, 17, 6), (128, 6, 4, True, 1, 1, 16, 129, 0),
    (32, 4, 2, False, 2, 1, 3, 0, 0)])
def test_decode_step_equals_append_then_attend(D, kb, vb, qjl, B, Hkv, g, T, W):
    """tq_decode_step writes the same page bytes as tq_append and returns the
    same output as tq_decode_attn over tokens [0, T + 1)."""
    t = make_tables(D, kb, vb, qjl)
    k, v = rand_kv((B, Hkv, T + 1, D), 30).to(DEV), rand_kv((B, Hkv, T + 1, D), 31).to(DEV)
    q = rand_kv((B, Hkv * g, 1, D), 32, outliers=0).to(DEV)
    wk = rand_kv((B, Hkv, W, D), 33).to(DEV) if W else None
    wv = rand_kv((B, Hkv, W, D), 34).to(DEV) if W else None
    pa, pb = new_pages(B * Hkv, T + 1, t), new_pages(B * Hkv, T + 1, t)
    if T:
        ops.append(t, pa, k[:, :, :T], v[:, :, :T], 0)
        ops.append(t, pb, k[:, :, :T], v[:, :, :T], 0)
    ops.append(t, pa, k[:, :, T:], v[:, :, T:], T)
    want = ops.decode_attention(t, pa, q, T + 1, wk, wv)
    got = ops.decode_step(t, pb, k[:, :, T:], v[:, :, T:], T, q, wk, wv)
    torch.cuda.synchronize()
    assert torch.equal(pa, pb)
    assert torch.equal(got, want)


@pytest.mark.parametrize("rw", [0, 4])
def test_cache_decode_matches_store_then_attend(rw):
    B, Hkv, g, T, D = 2, 4, 4, 150, 128
    kw = dict(num_layers=1, batch_size=B, num_heads=Hkv, head_dim=D, key_bits=4, value_bits=2,
              residual_window=rw, protected_layers=0, dtype=torch.bfloat16, device=DEV,
              max_seq_len=T + 8, qjl=True)
    c1, c2 = TurboQuantKVCache(**kw), TurboQuantKVCache(**kw)
    k, v = rand_kv((B, Hkv, T + 5, D), 40).to(DEV), rand_kv((B, Hkv, T + 5, D), 41).to(DEV)
    c1.append(k[:, :, :T], v[:, :, :T], 0)
    c2.append(k[:, :, :T], v[:, :, :T], 0)
    for i in range(5):
        q = rand_kv((B, Hkv * g, 1, D), 50 + i, outliers=0).to(DEV)
        kt, vt = k[:, :, T + i:T + i + 1], v[:, :, T + i:T + i + 1]
        got = c1.decode(q, kt, vt, 0)
        c2.append(kt, vt, 0)
        want = c2.attend(q, 0)
        assert torch.equal(got, want), i
    assert torch.equal(c1._stores[0]._pages, c2._stores[0]._pages)
    assert c1.device_status() == 0
