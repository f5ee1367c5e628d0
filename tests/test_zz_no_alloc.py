"""tq_decode_attn_noalloc: decode attention for callers that cannot allocate.

Some callers cannot call cudaMalloc (a serving runtime that owns all device
memory through its own pool, or code that must not allocate while serving),
so they cannot hand tq_decode_attn a workspace.  tq_decode_attn_noalloc keeps
that scratch in a fixed array inside the library.  This test calls it through
the C ABI twice in a row and checks each result against the workspace entry
point, within the tolerance the decode tests use (max-abs <= 2e-3 * max|o|).
It also checks that a call needing more than the array holds is refused.
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


def _noalloc(tables, pages, q, n_tokens):
    lib = _lib.load()
    out = torch.empty_like(q)
    keep = []
    a = ops._decode_args(q, out, n_tokens, None, None, None, 0, 0, keep)
    g, t, c = tables.geom(), tables.ctables(), ops._cache_desc(pages)
    rc = lib.tq_decode_attn_noalloc(ctypes.byref(g), ctypes.byref(t), ctypes.byref(c),
                                    ctypes.byref(a), ops._stream(DEV))
    return rc, out


def test_noalloc_matches_workspace_entry_point_twice():
    D, B, Hkv, g, T = 128, 2, 4, 4, 700
    t = _tables(D, 4, 2, True)
    pages = torch.zeros((B * Hkv, -(-T // 64), ops.page_bytes(D, 4, 2, True)), dtype=torch.uint8,
                        device=DEV)
    ops.append(t, pages, _bf16((B, Hkv, T, D), 1), _bf16((B, Hkv, T, D), 2), 0)
    for call in range(2):
        q = _bf16((B, Hkv * g, 1, D), 10 + call)
        n = T - 37 * call                       # second call attends fewer tokens
        want = ops.decode_attention(t, pages, q, n)
        rc, got = _noalloc(t, pages, q, n)
        assert rc == _lib.TQ_OK, _lib.last_error()
        torch.cuda.synchronize()
        tol = 2e-3 * want.float().abs().max().item()
        assert torch.allclose(got.float(), want.float(), rtol=0.0, atol=tol), call


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
