"""GPU parity of the tensor-core append (tcgen05 rotation, head_dim 128, with
and without the QJL sketch).

The kernel computes y = x R^T as three exact bf16 x bf16 products (R split
into hi/mid/lo bf16 terms) summed in fp32, and takes the norm as ||y||.  Its
rounding therefore differs from the reference's fp32 matmul, so the bar is the
one the CUDA-core append meets (kv_cache.py:382-398 restated in
oracle/tq_oracle.py:compress):
  * codes >= 99.99 % identical to the oracle, every mismatch within 1e-5 of a
    boundary;
  * fp16 norms >= 99.9 % identical, all within rtol 1e-3;
  * the pages re-pack byte for byte from their parsed fields (layout exact);
  * against the CUDA-core kernel on the same inputs: codes >= 99.99 %
    identical, norms >= 99.9 % identical.
With the QJL sketch (z = S r on the tensor cores, r in bf16 hi + lo terms):
sign bits >= 99.9 % identical to the oracle's sketch of the kernel's own
codes, and gamma within rtol 1e-2, as for the CUDA-core kernel.
"""
import numpy as np
import pytest
import torch

from bhaskera_col_b200.inference import ops
from oracle import tq_oracle as O
from test_gpu_parity import DEV, make_tables, new_pages, parse, rand_kv

pytestmark = pytest.mark.gpu

TC_BITS = [(4, 2), (3, 3), (2, 2), (8, 8), (1, 1), (5, 5), (6, 4), (7, 7), (4, 4)]


def _check_codes(got, want, y, bd):
    agree = got == want
    assert agree.mean() >= 0.9999, agree.mean()
    if not agree.all():
        dist = np.abs(y[~agree][:, None] - bd[None, :]).min(-1)
        assert dist.max() < 1e-5, dist.max()


def _check_vs_oracle(t, pages, k, v):
    B, H, T, D = k.shape
    geom, got = parse(t, pages, T)
    rebuilt = O.build_pages(geom, got["k_idx"], got["v_idx"], got["k_norm"], got["v_norm"],
                            got.get("qbits"), got.get("gamma"))
    assert np.array_equal(rebuilt, pages.cpu().numpy())
    R = t.rot.cpu().numpy()
    for x, key, bnd in ((k, "k", t.k_boundaries), (v, "v", t.v_boundaries)):
        bd = bnd.cpu().numpy()
        xs = x.float().numpy().reshape(B * H, T, D)
        idx, nrm, y = O.compress(xs, R, bd)
        _check_codes(got[key + "_idx"], idx, y, bd)
        assert (got[key + "_norm"] == nrm).mean() >= 0.999
        np.testing.assert_allclose(got[key + "_norm"].astype(np.float32),
                                   nrm.astype(np.float32), rtol=1e-3)
        if key == "k" and t.qjl:
            S = t.qjl_mat.cpu().numpy()
            bits, gam = O.qjl_sketch(y, got["k_idx"], t.k_centroids.cpu().numpy(),
                                     nrm.astype(np.float32), S)
            assert (got["qbits"] == bits).mean() >= 0.999, (got["qbits"] == bits).mean()
            np.testing.assert_allclose(got["gamma"].astype(np.float32), gam.astype(np.float32),
                                       rtol=1e-2, atol=1e-3)


TC_CASES = [(kb, vb, False) for kb, vb in TC_BITS] + [(4, 2, True), (3, 3, True), (2, 2, True),
                                                       (5, 5, True), (8, 8, True), (1, 1, True)]


@pytest.mark.parametrize("kb,vb,qjl", TC_CASES)
def test_tensor_core_append_matches_oracle(kb, vb, qjl):
    B, H, T1, T2, D = 2, 3, 300, 170, 128
    t = make_tables(D, kb, vb, qjl)
    k = rand_kv((B, H, T1 + T2, D), 11)
    v = rand_kv((B, H, T1 + T2, D), 12)
    k[:, :, 5] = 0                                   # zero vectors
    v[:, 1, 9] = 0
    k[:, :, 6] = (k[:, :, 6].float() * 1e-9).bfloat16()   # norms below the 1e-8 clamp
    pages = new_pages(B * H, T1 + T2, t)
    kd, vd = k.to(DEV), v.to(DEV)
    # first chunk: partial 128-token tiles; second: a strided view starting
    # mid-page (pos = 300 is not a multiple of 64)
    k2 = kd[:, :, T1:].transpose(1, 2).contiguous().transpose(1, 2)
    assert ops.append_uses_tensor_cores(t, kd[:, :, :T1], vd[:, :, :T1])
    assert ops.append_uses_tensor_cores(t, k2, vd[:, :, T1:])
    ops.append(t, pages, kd[:, :, :T1], vd[:, :, :T1], 0)
    ops.append(t, pages, k2, vd[:, :, T1:], T1)
    torch.cuda.synchronize()
    assert ops.device_status(DEV) == 0
    _check_vs_oracle(t, pages, k, v)


def test_tensor_core_path_selection():
    t = make_tables(128, 4, 2, False)
    x = torch.zeros((1, 2, 64, 128), dtype=torch.bfloat16, device=DEV)
    assert ops.append_uses_tensor_cores(t, x, x)
    assert not ops.append_uses_tensor_cores(t, x[:, :, :16], x[:, :, :16])      # < 32 tokens
    assert not ops.append_uses_tensor_cores(t, x.half(), x.half())              # fp16 input
    assert ops.append_uses_tensor_cores(make_tables(128, 4, 2, True), x, x)      # QJL sketch
    q = make_tables(128, 4, 2, True)             # an S that is not exactly bf16 keeps
    custom = ops.LayerTables(128, 4, 2, True, q.k_centroids, q.k_boundaries, q.v_centroids,
                             q.v_boundaries, q.rot, q.qjl_mat + 1e-3)   # the CUDA-core sketch
    assert custom.qjl_bf16 is None
    assert not ops.append_uses_tensor_cores(custom, x, x)
    assert not ops.append_uses_tensor_cores(make_tables(64, 4, 2, False), x[..., :64],
                                            x[..., :64])


def _core_tables(t):
    """Same tables without the bf16 split: forces the CUDA-core kernel."""
    c = ops.LayerTables(t.head_dim, t.key_bits, t.value_bits, t.qjl, t.k_centroids,
                        t.k_boundaries, t.v_centroids, t.v_boundaries, t.rot, t.qjl_mat)
    c.rot_bf16x3 = None
    c.qjl_bf16 = None
    return c


@pytest.mark.parametrize("bits,qjl", [(4, False), (3, False), (4, True), (3, True)])
def test_tensor_core_append_equals_core_kernel_full_size(bits, qjl):
    """Prefill of 8 x 8 streams x 4096 tokens (the append benchmark's layer)."""
    B, H, T, D = 8, 8, 4096, 128
    t = make_tables(D, bits, bits, qjl)
    tc_ = _core_tables(t)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(5)
    sc = torch.exp(torch.empty(D, device=DEV).uniform_(-2.3, 2.3, generator=gen))
    k = (torch.randn((B, H, T, D), device=DEV, generator=gen) * sc).bfloat16()
    v = (torch.randn((B, H, T, D), device=DEV, generator=gen) * sc).bfloat16()
    assert ops.append_uses_tensor_cores(t, k, v)
    assert not ops.append_uses_tensor_cores(tc_, k, v)
    p_tc, p_core = new_pages(B * H, T, t), new_pages(B * H, T, t)
    ops.append(t, p_tc, k, v, 0)
    ops.append(tc_, p_core, k, v, 0)
    torch.cuda.synchronize()
    assert ops.device_status(DEV) == 0
    geom, a = parse(t, p_tc, T)
    _, b = parse(t, p_core, T)
    rebuilt = O.build_pages(geom, a["k_idx"], a["v_idx"], a["k_norm"], a["v_norm"],
                            a.get("qbits"), a.get("gamma"))
    assert np.array_equal(rebuilt, p_tc.cpu().numpy())
    if qjl:
        assert (a["qbits"] == b["qbits"]).mean() >= 0.999
        np.testing.assert_allclose(a["gamma"].astype(np.float32), b["gamma"].astype(np.float32),
                                   rtol=1e-2, atol=1e-3)
    for key in ("k_idx", "v_idx"):
        assert (a[key] == b[key]).mean() >= 0.9999
        assert np.abs(a[key].astype(np.int32) - b[key].astype(np.int32)).max() <= 1
    for key in ("k_norm", "v_norm"):
        assert (a[key] == b[key]).mean() >= 0.999
        np.testing.assert_allclose(a[key].astype(np.float32), b[key].astype(np.float32),
                                   rtol=1e-3)
