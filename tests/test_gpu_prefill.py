"""GPU parity of the prefill attention (tq_prefill_attn) against the oracle.

The oracle is the reference's prefill semantics: SDPA (float64, causal, GQA
repeat) over the dequantised K/V x^ = n (c[idx] R) that update() returns at
residual_window 0 (kv_cache.py:422-439, 483-488), evaluated on the codes and
norms the kernel's own append stored.  The kernel rotates queries, attends
fp16 centroid values and un-rotates outputs with fp16 operands, so the bar is
cosine >= 0.9999 and max-abs <= 4e-3 * max|o| per case.
"""
import math

import numpy as np
import pytest
import torch

from bhaskera_col_b200.inference import TurboQuantKVCache, ops
from oracle import tq_oracle as O
from test_gpu_parity import DEV, cosine, make_tables, new_pages, parse, rand_kv

pytestmark = pytest.mark.gpu


def _dequant(t, pages, n):
    geom, got = parse(t, pages, n)
    R = t.rot.cpu().numpy()
    k = O.decode_range(got["k_idx"], got["k_norm"], t.k_centroids.cpu().numpy(), R)
    v = O.decode_range(got["v_idx"], got["v_norm"], t.v_centroids.cpu().numpy(), R)
    return k, v                                   # (S, n, D) float32


def _check(got, want, tol=4e-3):
    got = got.float().cpu().numpy()
    assert cosine(got, want) >= 0.9999, cosine(got, want)
    err = np.abs(got - want).max()
    assert err <= tol * np.abs(want).max(), (err, np.abs(want).max())


CASES = [
    # D, kb, vb, qjl, B, Hkv, g, n_tokens, Tq, causal
    (128, 4, 2, False, 2, 2, 4, 300, 300, True),     # whole prefill, ragged tiles
    (128, 4, 4, False, 1, 2, 4, 500, 200, True),     # a second chunk at positions 300..499
    (128, 3, 3, False, 2, 1, 5, 130, 130, True),     # GQA 5 (Qwen-style)
    (128, 8, 8, False, 1, 1, 2, 64, 64, False),      # non-causal, one page
    (128, 4, 2, True, 1, 2, 2, 200, 77, True),       # cache with a QJL sketch (not used)
    (64, 4, 2, False, 2, 2, 4, 257, 257, True),
    (64, 3, 3, False, 1, 1, 8, 100, 40, True),
]


@pytest.mark.parametrize("D,kb,vb,qjl,B,Hkv,g,n,Tq,causal", CASES)
def test_prefill_matches_oracle(D, kb, vb, qjl, B, Hkv, g, n, Tq, causal):
    t = make_tables(D, kb, vb, qjl)
    k = rand_kv((B, Hkv, n, D), 21)
    v = rand_kv((B, Hkv, n, D), 22)
    q = rand_kv((B, Hkv * g, Tq, D), 23)
    pages = new_pages(B * Hkv, n, t)
    ops.append(t, pages, k.to(DEV), v.to(DEV), 0)
    out = ops.prefill_attention(t, pages, q.to(DEV), n, causal=causal)
    torch.cuda.synchronize()
    assert ops.device_status(DEV) == 0
    kd, vd = _dequant(t, pages, n)
    want = O.sdpa(q.float().numpy(), kd.reshape(B, Hkv, n, D), vd.reshape(B, Hkv, n, D),
                  causal=causal)
    _check(out, want)


def test_prefill_last_row_equals_decode():
    """The last query of a prefill chunk attends exactly what a decode call sees."""
    D, B, Hkv, g, n = 128, 2, 2, 4, 333
    t = make_tables(D, 4, 2, False)
    pages = new_pages(B * Hkv, n, t)
    ops.append(t, pages, rand_kv((B, Hkv, n, D), 1).to(DEV), rand_kv((B, Hkv, n, D), 2).to(DEV), 0)
    q = rand_kv((B, Hkv * g, 16, D), 3).to(DEV)
    pf = ops.prefill_attention(t, pages, q, n)
    dec = ops.decode_attention(t, pages, q[:, :, -1:].contiguous(), n)
    torch.cuda.synchronize()
    want = dec.float().cpu().numpy()
    _check(pf[:, :, -1:], want, tol=4e-3)


def test_cache_prefill_api_and_window_rule():
    B, Hkv, Hq, D, T = 1, 2, 8, 128, 150
    cache = TurboQuantKVCache(num_layers=2, batch_size=B, num_heads=Hkv, head_dim=D,
                              residual_window=0, protected_layers=0, device=DEV, max_seq_len=64)
    k, v = rand_kv((B, Hkv, T, D), 4).to(DEV), rand_kv((B, Hkv, T, D), 5).to(DEV)
    q = rand_kv((B, Hq, T, D), 6).to(DEV)
    out = cache.prefill(q, k, v, 1)
    assert cache._stores[1].tokens == T          # stored, capacity grown past max_seq_len
    st = cache._stores[1]
    want = ops.prefill_attention(st.tables, st._pages, q, T)
    assert torch.equal(out, want)
    assert cache.device_status() == 0
    windowed = TurboQuantKVCache(num_layers=1, batch_size=B, num_heads=Hkv, head_dim=D,
                                 residual_window=8, protected_layers=0, device=DEV)
    with pytest.raises(ValueError):
        windowed.prefill(q, k, v, 0)


def test_prefill_full_size_sampled():
    """The prefill-attention workload of one layer (B8, Hq32, Hkv8, 4096 tokens,
    4-bit K/V, causal), checked against the oracle on sampled streams/rows."""
    D, B, Hkv, g, T = 128, 8, 8, 4, 4096
    t = make_tables(D, 4, 4, False)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(11)
    sc = torch.exp(torch.empty(D, device=DEV).uniform_(math.log(0.1), math.log(10.0), generator=gen))
    k = (torch.randn((B, Hkv, T, D), device=DEV, generator=gen) * sc).bfloat16()
    v = (torch.randn((B, Hkv, T, D), device=DEV, generator=gen) * sc).bfloat16()
    q = torch.randn((B, Hkv * g, T, D), device=DEV, generator=gen).bfloat16()
    pages = new_pages(B * Hkv, T, t)
    ops.append(t, pages, k, v, 0)
    out = ops.prefill_attention(t, pages, q, T)
    torch.cuda.synchronize()
    assert ops.device_status(DEV) == 0
    assert torch.isfinite(out.float()).all()
    rows = np.array([0, 1, 63, 64, 127, 128, 1000, 2047, 2048, 4095])
    for (b, h) in [(0, 0), (3, 17), (7, 31)]:
        s = b * Hkv + h // g
        sub_pages = pages[s:s + 1]
        kd, vd = _dequant(t, sub_pages, T)
        qs = q[b:b + 1, h:h + 1].float().cpu().numpy()
        want = O.sdpa(qs, kd.reshape(1, 1, T, D), vd.reshape(1, 1, T, D), causal=True)
        _check(out[b:b + 1, h:h + 1, rows], want[:, :, rows])
