"""tq_init_tables (tables from host arrays, for callers without PyTorch) builds
the same bytes as the Python LayerTables, and the kernels give identical
results with either."""
import ctypes

import pytest
import torch

from bhaskera_col_b200 import _lib
from bhaskera_col_b200.inference import ops
from test_gpu_parity import DEV, make_tables, new_pages, rand_kv

pytestmark = pytest.mark.gpu


def _c_tables(t: ops.LayerTables):
    """The layer's tables built by tq_init_tables from host copies."""
    lib = _lib.load()
    g = t.geom()
    n = lib.tq_tables_bytes(ctypes.byref(g))
    buf = torch.empty(n + 256, dtype=torch.uint8, device=DEV)
    off = (-buf.data_ptr()) % 256
    host = {k: getattr(t, k).detach().float().cpu().contiguous().numpy()
            for k in ("k_centroids", "k_boundaries", "v_centroids", "v_boundaries", "rot")}
    S = t.qjl_mat.cpu().contiguous().numpy() if t.qjl else None

    def ptr(a):
        return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None

    ct = _lib.Tables()
    _lib.check("tq_init_tables", lib.tq_init_tables(
        ctypes.byref(g), ptr(host["k_centroids"]), ptr(host["k_boundaries"]),
        ptr(host["v_centroids"]), ptr(host["v_boundaries"]), ptr(host["rot"]), ptr(S),
        buf.data_ptr() + off, n, ctypes.byref(ct), torch.cuda.current_stream(DEV).cuda_stream))
    return ct, buf


class _Raw:
    """A uint8 view of raw device memory (for torch.as_tensor)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3}


def _dev_bytes(ptr, nbytes):
    return torch.as_tensor(_Raw(ptr, nbytes), device=DEV).clone()


@pytest.mark.parametrize("D,kb,vb,qjl", [(128, 4, 2, True), (128, 3, 3, False), (64, 4, 2, True)])
def test_init_tables_matches_python_tables(D, kb, vb, qjl):
    t = make_tables(D, kb, vb, qjl)
    ct, _buf = _c_tables(t)
    pairs = [("k_centroids", t.k_centroids), ("k_boundaries", t.k_boundaries),
             ("v_centroids", t.v_centroids), ("v_boundaries", t.v_boundaries),
             ("rot", t.rot), ("rot_t", t.rot_t), ("rot_f16", t.rot_f16)]
    if qjl:
        pairs += [("qjl", t.qjl_mat), ("qjl_t", t.qjl_t)]
    if D == 128:
        pairs += [("rot_bf16x3", t.rot_bf16x3)]
    if D == 128 and qjl:
        pairs += [("qjl_bf16", t.qjl_bf16)]     # S in bf16, K quad order, for the sketch
    for name, ref in pairs:
        ref = ref.contiguous()
        got = _dev_bytes(getattr(ct, name), ref.numel() * ref.element_size())
        assert torch.equal(got, ref.view(torch.uint8).flatten()), name
    if D != 128:
        assert not ct.rot_bf16x3
    if D != 128 or not qjl:
        assert not ct.qjl_bf16


def test_kernels_identical_with_c_tables():
    D, B, Hkv, g, T = 128, 2, 2, 4, 300
    t = make_tables(D, 4, 2, True)
    ct, _buf = _c_tables(t)
    k, v = rand_kv((B, Hkv, T, D), 90).to(DEV), rand_kv((B, Hkv, T, D), 91).to(DEV)
    q = rand_kv((B, Hkv * g, 1, D), 92, outliers=0).to(DEV)
    pa, pb = new_pages(B * Hkv, T, t), new_pages(B * Hkv, T, t)
    ops.append(t, pa, k, v, 0)
    want = ops.decode_attention(t, pa, q, T)
    t.__dict__["_ctab"] = ct                 # the same LayerTables, C-built descriptor
    ops.append(t, pb, k, v, 0)
    got = ops.decode_attention(t, pb, q, T)
    torch.cuda.synchronize()
    assert torch.equal(pa, pb)
    assert torch.equal(got, want)
