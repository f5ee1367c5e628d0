"""The C-ABI library: loads without a GPU, exports every declared symbol, and
rejects bad arguments before touching the device (CPU only)."""
import ctypes
import os
import re

import pytest

from bhaskera_col_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "tq_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tq_[a-z_]+)\s*\(", src)))


def test_header_declares_the_binding_list():
    assert declared_functions() == sorted(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.tq_version() == 1


def _geom(D=128, kb=4, vb=2, q=1):
    return _lib.Geom(D, kb, vb, q)


def test_invalid_geometry_rejected():
    lib = _lib.load()
    assert lib.tq_page_bytes(ctypes.byref(_geom(D=48))) == -1
    assert "multiple of 32" in _lib.last_error()
    assert lib.tq_page_bytes(ctypes.byref(_geom(kb=9))) == -1
    assert "bit widths" in _lib.last_error()


def test_append_argument_validation():
    lib = _lib.load()
    g = _geom()
    t = _lib.Tables()                       # NULL tables
    c = _lib.Cache()
    k = _lib.Tensor4()
    rc = lib.tq_append(ctypes.byref(g), ctypes.byref(t), ctypes.byref(c), ctypes.byref(k),
                       ctypes.byref(k), 0, None)
    assert rc == _lib.TQ_ERR_INVALID
    assert "NULL" in _lib.last_error()
    # all pointers non-null, but k/v disagree with the cache's stream count
    t = _lib.Tables(*([16] * 10))
    c = _lib.Cache(1024, 3, 4)
    k = _lib.Tensor4(16, _lib.TQ_BF16, (ctypes.c_int64 * 4)(1, 2, 5, 128),
                     (ctypes.c_int64 * 4)(1280, 640, 128, 1))
    rc = lib.tq_append(ctypes.byref(g), ctypes.byref(t), ctypes.byref(c), ctypes.byref(k),
                       ctypes.byref(k), 0, None)
    assert rc == _lib.TQ_ERR_INVALID and "streams" in _lib.last_error()
    # capacity overflow: 4 pages * 64 tokens
    c = _lib.Cache(1024, 2, 4)
    rc = lib.tq_append(ctypes.byref(g), ctypes.byref(t), ctypes.byref(c), ctypes.byref(k),
                       ctypes.byref(k), 254, None)
    assert rc == _lib.TQ_ERR_INVALID and "capacity" in _lib.last_error()


def test_decode_argument_validation():
    lib = _lib.load()
    g = _geom()
    t = _lib.Tables(*([16] * 10))
    c = _lib.Cache(1024, 8, 4)
    q = _lib.Tensor4(16, _lib.TQ_BF16, (ctypes.c_int64 * 4)(2, 6, 1, 128),
                     (ctypes.c_int64 * 4)(768, 128, 128, 1))
    a = _lib.DecodeArgs()
    a.q = ctypes.pointer(q)
    a.out = ctypes.pointer(q)
    a.n_tokens = 10
    a.num_q_heads = 6                       # 6 query heads over 4 kv heads: invalid
    a.scale = 0.1
    rc = lib.tq_decode_attn(ctypes.byref(g), ctypes.byref(t), ctypes.byref(c),
                            ctypes.byref(a), None, 0, None)
    assert rc == _lib.TQ_ERR_INVALID and "multiple of Hkv" in _lib.last_error()
    q.shape[1] = 8
    a.num_q_heads = 8
    a.n_tokens = 10_000                     # beyond 4 pages
    rc = lib.tq_decode_attn(ctypes.byref(g), ctypes.byref(t), ctypes.byref(c),
                            ctypes.byref(a), None, 0, None)
    assert rc == _lib.TQ_ERR_INVALID and "capacity" in _lib.last_error()


def test_quantize_argument_validation():
    lib = _lib.load()
    rc = lib.tq_quantize_rotated(None, 10, None, 15, None, None)
    assert rc == _lib.TQ_ERR_INVALID
    rc = lib.tq_quantize_rotated(16, 10, 16, 300, 16, None)
    assert rc == _lib.TQ_ERR_INVALID


def test_block_table_validation():
    lib = _lib.load()
    g = _geom(q=0)
    t = _lib.Tables(*([16] * 10))
    k = _lib.Tensor4(16, _lib.TQ_BF16, (ctypes.c_int64 * 4)(1, 2, 5, 128),
                     (ctypes.c_int64 * 4)(1280, 640, 128, 1))
    bad = [_lib.Cache(1024, 2, 4, 1024, 3, 16),      # stride below pages_per_stream
           _lib.Cache(1024, 2, 4, 1024, 4, 0),       # empty pool
           _lib.Cache(1024, 2, 4, 1026, 4, 16)]      # misaligned table
    for c in bad:
        rc = lib.tq_append(ctypes.byref(g), ctypes.byref(t), ctypes.byref(c), ctypes.byref(k),
                           ctypes.byref(k), 0, None)
        assert rc == _lib.TQ_ERR_INVALID and "block table" in _lib.last_error()


def test_paged_pages_holder():
    import torch
    from bhaskera_col_b200.inference import ops
    pool = torch.zeros((10, 64), dtype=torch.uint8)
    bt = torch.zeros((3, 6), dtype=torch.int32)[:, :4]
    pp = ops.PagedPages(pool, bt)
    assert pp.shape == (3, 4, 64) and not pp.is_cuda
    c = ops._cache_desc(pp)
    assert (c.streams, c.pages_per_stream, c.block_table_stride, c.num_blocks) == (3, 4, 6, 10)
    assert c.block_table == bt.data_ptr() and c.pages == pool.data_ptr()
    with pytest.raises(ValueError):
        ops.PagedPages(pool.float(), bt)
    with pytest.raises(ValueError):
        ops.PagedPages(pool, bt.long())
    with pytest.raises(ValueError):
        ops.PagedPages(pool, torch.zeros((4, 3), dtype=torch.int32).t())
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.append(None, pp, torch.zeros(1), torch.zeros(1), 0)


def test_init_tables_sizes_and_validation():
    lib = _lib.load()
    g = _geom(D=128, kb=4, vb=2, q=1)
    n = lib.tq_tables_bytes(ctypes.byref(g))
    # kc 64 B, kb 60, vc 16, vb 12 (each in a 256-byte slot), R, R^T, S, S^T
    # (64 KiB each), three bf16 terms x 2 orders (192 KiB), R fp16 (32 KiB),
    # S in bf16 for the tensor-core sketch (32 KiB)
    assert n == 4 * 256 + 4 * 65536 + 196608 + 32768 + 32768
    assert lib.tq_tables_bytes(ctypes.byref(_geom(D=48))) == 0
    t = _lib.Tables()
    host = (ctypes.c_float * (128 * 128))()
    rc = lib.tq_init_tables(ctypes.byref(g), host, host, host, host, host, None, 256, n,
                            ctypes.byref(t), None)
    assert rc == _lib.TQ_ERR_INVALID and "NULL" in _lib.last_error()     # qjl needs S
    rc = lib.tq_init_tables(ctypes.byref(g), host, host, host, host, host, host, 256, n - 1,
                            ctypes.byref(t), None)
    assert rc == _lib.TQ_ERR_INVALID and "device buffer" in _lib.last_error()
    rc = lib.tq_init_tables(ctypes.byref(g), host, host, host, host, host, host, 264, n,
                            ctypes.byref(t), None)
    assert rc == _lib.TQ_ERR_INVALID and "aligned" in _lib.last_error()


def test_seq_lens_validation():
    """Ragged decode arguments are checked on the host before any launch."""
    import torch
    from bhaskera_col_b200.inference import ops
    q = torch.zeros((3, 8, 1, 128), dtype=torch.bfloat16)
    for bad in (torch.zeros(3, dtype=torch.int64), torch.zeros((3, 1), dtype=torch.int32),
                torch.zeros(4, dtype=torch.int32)):
        with pytest.raises(ValueError, match="seq_lens"):
            ops._seq_lens_ptr(bad, q)
    assert ops._seq_lens_ptr(None, q) is None
    lib = _lib.load()
    g = _geom()
    t = _lib.Tables(*([16] * 10))
    c = _lib.Cache(1024, 8, 4)
    qt = _lib.Tensor4(16, _lib.TQ_BF16, (ctypes.c_int64 * 4)(2, 8, 1, 128),
                      (ctypes.c_int64 * 4)(1024, 128, 128, 1))
    a = _lib.DecodeArgs()
    a.q = ctypes.pointer(qt)
    a.out = ctypes.pointer(qt)
    a.n_tokens = 10
    a.num_q_heads = 8
    a.scale = 0.1
    a.seq_lens = 1026                        # not 4-byte aligned
    rc = lib.tq_decode_attn(ctypes.byref(g), ctypes.byref(t), ctypes.byref(c),
                            ctypes.byref(a), None, 0, None)
    assert rc == _lib.TQ_ERR_INVALID and "aligned" in _lib.last_error()
    a.seq_lens = 1024
    a.phases = _lib.PHASE_DECODE             # the page layout needs the prep phase
    rc = lib.tq_decode_attn(ctypes.byref(g), ctypes.byref(t), ctypes.byref(c),
                            ctypes.byref(a), None, 0, None)
    assert rc == _lib.TQ_ERR_INVALID and "query-preparation" in _lib.last_error()
