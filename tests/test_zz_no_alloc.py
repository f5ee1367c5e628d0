"""tq_decode_attn_noalloc: decode attention for callers that cannot allocate.

Some callers cannot call cudaMalloc (a serving runtime that owns all device
memory through its own pool, or code that must not allocate while serving),
so they cannot hand tq_decode_attn a workspace.  tq_decode_attn_noalloc keeps
that scratch in a fixed array inside the library.  This test calls it through
the C ABI twice in a row and checks each result against the workspace entry
point.  Both run the same kernels on the same inputs, so the outputs must be
bitwise equal.  After every call the array's status word must read 0 through
tq_noalloc_status.  A paged call with a planted out-of-pool block-table entry
must report TQ_DEV_BAD_BLOCK there.  A call needing more than the array holds
is refused, and so is a phase-split call.
"""
import ctypes

import numpy as np
import pytest
import torch

import inputs as gi
from bhaskera_col_b200 import _lib
from bhaskera_col_b200.inference import ops
from bhaskera_col_b200.inference.kv_cache import (FastLloydMaxCodebook, _generate_qjl_matrix,
                                                  _generate_rotation_matrix)

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _tables(D, kb, vb, qjl):
    kc = FastLloydMaxCodebook.get(D, kb, DEV)
    vc = FastLloydMaxCodebook.get(D, vb, DEV)
    R = _generate_rotation_matrix(D, 42, DEV)
    S = _generate_qjl_matrix(D, 42, DEV) if qjl else None
    return ops.LayerTables(D, kb, vb, qjl, kc.centroids, kc.boundaries, vc.centroids,
                           vc.boundaries, R, S)


def _bf16(shape, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    return torch.from_numpy(gi.outlier_normal(rng, shape, 2, 8.0)).to(DEV, torch.bfloat16)


def _noalloc(tables, pages, q, n_tokens, phases=0):
    lib = _lib.load()
    out = torch.empty_like(q)
    keep = []
    a = ops._decode_args(q, out, n_tokens, None, None, None, 0, phases, keep)
    g, t, c = tables.geom(), tables.ctables(), ops._cache_desc(pages)
    rc = lib.tq_decode_attn_noalloc(ctypes.byref(g), ctypes.byref(t), ctypes.byref(c),
                                    ctypes.byref(a), ops._stream(DEV))
    return rc, out


def _noalloc_status():
    st = ctypes.c_uint32(0)
    rc = _lib.load().tq_noalloc_status(ctypes.byref(st), ops._stream(DEV))
    assert rc in (_lib.TQ_OK, _lib.TQ_ERR_DEVICE), _lib.last_error()
    return int(st.value)


def _filled(D=128, B=2, Hkv=4, T=700):
    t = _tables(D, 4, 2, True)
    pages = torch.zeros((B * Hkv, -(-T // 64), ops.page_bytes(D, 4, 2, True)), dtype=torch.uint8,
                        device=DEV)
    ops.append(t, pages, _bf16((B, Hkv, T, D), 1), _bf16((B, Hkv, T, D), 2), 0)
    return t, pages


def test_noalloc_matches_workspace_entry_point_twice():
    B, Hkv, g, T, D = 2, 4, 4, 700, 128
    t, pages = _filled(D, B, Hkv, T)
    for call in range(2):
        q = _bf16((B, Hkv * g, 1, D), 10 + call)
        n = T - 37 * call                       # second call attends fewer tokens
        want = ops.decode_attention(t, pages, q, n)
        rc, got = _noalloc(t, pages, q, n)
        assert rc == _lib.TQ_OK, _lib.last_error()
        torch.cuda.synchronize()
        assert torch.equal(got, want), call
        assert _noalloc_status() == 0, call


def test_noalloc_reports_an_out_of_pool_block():
    B, Hkv, g, T, D = 2, 4, 4, 700, 128
    t, pages = _filled(D, B, Hkv, T)
    S, P, pb = pages.shape
    bt = torch.arange(S * P, dtype=torch.int32, device=DEV).view(S, P).clone()
    bt[1, 3] = -1                               # never dereferenced: page 0 is read instead
    paged = ops.PagedPages(pages.view(S * P, pb), bt)
    q = _bf16((B, Hkv * g, 1, D), 20)
    rc, _ = _noalloc(t, paged, q, T)
    assert rc == _lib.TQ_OK, _lib.last_error()
    assert _noalloc_status() & _lib.DEV_BAD_BLOCK
    assert _noalloc_status() == 0               # read and cleared
    # the next good call starts from a clear word and reports nothing
    bt[1, 3] = 3 + P
    rc, got = _noalloc(t, paged, q, T)
    assert rc == _lib.TQ_OK, _lib.last_error()
    assert _noalloc_status() == 0
    assert torch.equal(got, ops.decode_attention(t, pages, q, T))


def test_noalloc_refuses_calls_beyond_its_scratch():
    D = 128
    t = _tables(D, 4, 2, True)
    streams = 8192                               # query fragments alone exceed 8 MiB
    pages = torch.zeros((streams, 1, ops.page_bytes(D, 4, 2, True)), dtype=torch.uint8,
                        device=DEV)                 # a real cache of that size, all in bounds
    lib = _lib.load()
    c = ops._cache_desc(pages)
    q = torch.zeros((streams, 1, 1, D), dtype=torch.bfloat16, device=DEV)
    out = torch.empty_like(q)
    keep = []
    a = ops._decode_args(q, out, 1, None, None, None, 0, 0, keep)
    g, tt = t.geom(), t.ctables()
    rc = lib.tq_decode_attn_noalloc(ctypes.byref(g), ctypes.byref(tt), ctypes.byref(c),
                                    ctypes.byref(a), ops._stream(DEV))
    assert rc == _lib.TQ_ERR_WORKSPACE
    assert "8 MiB" in _lib.last_error()


def test_noalloc_refuses_a_phase_split_call():
    t, pages = _filled()
    q = _bf16((2, 16, 1, 128), 30)
    rc, _ = _noalloc(t, pages, q, 700, phases=_lib.PHASE_DECODE)
    assert rc == _lib.TQ_ERR_INVALID
    assert "phases" in _lib.last_error()
