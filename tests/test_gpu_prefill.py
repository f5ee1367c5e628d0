"""GPU parity of the prefill attention (tq_prefill_attn) against the oracle.

The oracle is the reference's prefill semantics: SDPA (float64, causal, GQA
repeat) over the dequantised K/V x^ = n (c[idx] R) that update() returns at
residual_window 0 (kv_cache.py:422-439, 483-488), evaluated on the codes and
norms the kernel's own append stored.  The kernel rotates queries, attends
fp16 centroid values and un-rotates outputs with fp16 operands, so the bar is
cosine >= 0.9999 and max-abs <= 4e-3 * max|o| per case, plus half a unit in
the last place of the output dtype at max|o| (the rounding of an exact result
to bf16 alone reaches 0.0156 at |o| = 6).
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


_MANTISSA = {torch.bfloat16: 8, torch.float16: 11, torch.float32: 24}


def _check(got, want, tol=4e-3):
    top = float(np.abs(want).max())
    half_ulp = 2.0 ** (math.floor(math.log2(top)) - _MANTISSA[got.dtype]) if top > 0 else 0.0
    got = got.float().cpu().numpy()
    assert cosine(got, want) >= 0.9999, cosine(got, want)
    err = np.abs(got - want).max()
    assert err <= tol * top + half_ulp, (err, top, half_ulp)


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


@pytest.mark.parametrize("engine", [0, 1])
@pytest.mark.parametrize("D,kb,vb,qjl,B,Hkv,g,n,Tq,causal", CASES)
def test_prefill_matches_oracle(D, kb, vb, qjl, B, Hkv, g, n, Tq, causal, engine):
    _run_case(D, kb, vb, qjl, B, Hkv, g, n, Tq, causal, engine)


def _run_case(D, kb, vb, qjl, B, Hkv, g, n, Tq, causal, engine, q_dtype=torch.bfloat16,
              transpose_q=False, key_growth=0.0, out_dtype=None):
    t = make_tables(D, kb, vb, qjl)
    k = rand_kv((B, Hkv, n, D), 21)
    if key_growth:
        k = (k.float() * (1.0 + key_growth * torch.arange(n).view(1, 1, n, 1))).bfloat16()
    v = rand_kv((B, Hkv, n, D), 22)
    q = rand_kv((B, Hkv * g, Tq, D), 23)
    pages = new_pages(B * Hkv, n, t)
    ops.append(t, pages, k.to(DEV), v.to(DEV), 0)
    qd = q.to(DEV, q_dtype)
    if transpose_q:            # (B, Tq, Hq, D) storage seen as (B, Hq, Tq, D)
        qd = qd.transpose(1, 2).contiguous().transpose(1, 2)
    out = None if out_dtype is None else torch.empty(qd.shape, dtype=out_dtype, device=DEV)
    out = ops.prefill_attention(t, pages, qd, n, causal=causal, engine=engine, out=out)
    torch.cuda.synchronize()
    assert ops.device_status(DEV) == 0
    kd, vd = _dequant(t, pages, n)
    want = O.sdpa(qd.float().cpu().numpy(), kd.reshape(B, Hkv, n, D),
                  vd.reshape(B, Hkv, n, D), causal=causal)
    _check(out, want)


TC_CASES = [
    # D, kb, vb, qjl, B, Hkv, g, n_tokens, Tq, causal
    (128, 4, 2, True, 1, 2, 4, 1000, 1000, True),    # 8 key tiles, odd page count
    (128, 2, 2, False, 1, 1, 1, 700, 300, True),     # MHA: 128 positions per CTA, chunk 400..699
    (128, 3, 4, False, 1, 1, 8, 390, 390, False),    # group 8: 16 positions per CTA, non-causal
    (128, 4, 3, False, 2, 1, 2, 129, 5, True),       # 5 queries, one key on the third page
    (128, 2, 4, False, 1, 2, 3, 256, 256, True),     # group 3: one head per CTA
    (128, 3, 2, False, 1, 1, 4, 64, 1, True),        # a single query
]


@pytest.mark.parametrize("engine", [2, 3])
@pytest.mark.parametrize("out_dtype", [None, torch.float32])
@pytest.mark.parametrize("D,kb,vb,qjl,B,Hkv,g,n,Tq,causal", TC_CASES)
def test_tensor_core_prefill_matches_oracle(D, kb, vb, qjl, B, Hkv, g, n, Tq, causal, out_dtype,
                                            engine):
    """Both tcgen05 kernels (engine 2: 128 query rows per CTA; 3: 256 rows, two
    query tiles sharing each decoded K/V tile), bf16 output (the query dtype)
    and fp32 output, where the comparison sees the kernel's own error without
    the output rounding."""
    assert ops.prefill_uses_tensor_cores(make_tables(D, kb, vb, qjl))
    _run_case(D, kb, vb, qjl, B, Hkv, g, n, Tq, causal, engine, out_dtype=out_dtype)


@pytest.mark.parametrize("engine", [2, 3])
@pytest.mark.parametrize("q_dtype,transpose_q", [(torch.float16, False), (torch.bfloat16, True),
                                                 (torch.float32, False)])
def test_tensor_core_prefill_query_layouts(q_dtype, transpose_q, engine):
    _run_case(128, 4, 2, False, 1, 2, 4, 300, 300, True, engine, q_dtype=q_dtype,
              transpose_q=transpose_q)


@pytest.mark.parametrize("engine", [0, 1, 2, 3])
def test_prefill_growing_scores(engine):
    """Key norms growing 5x along the sequence lift the running max by more
    than 8 (log2 units) over the tiles, so the tcgen05 kernel rescales its
    output accumulator in tensor memory (scores stay within the range where
    fp16 operands keep the 4e-3 bar)."""
    _run_case(128, 4, 4, False, 1, 1, 4, 900, 900, True, engine, key_growth=0.005)


def test_tensor_core_coverage():
    assert not ops.prefill_uses_tensor_cores(make_tables(64, 4, 2, False))
    assert not ops.prefill_uses_tensor_cores(make_tables(128, 8, 8, False))
    assert ops.prefill_uses_tensor_cores(make_tables(128, 4, 2, True))
    # protected layers of K4/V2 and K3/V3 (+2 bits): pair tables with fewer
    # than four copies per entry
    assert ops.prefill_uses_tensor_cores(make_tables(128, 6, 4, False))
    assert ops.prefill_uses_tensor_cores(make_tables(128, 5, 5, False))


@pytest.mark.parametrize("engine", [2, 3])
@pytest.mark.parametrize("kb,vb", [(6, 4), (5, 5), (6, 6), (5, 4)])
def test_prefill_protected_layer_bits_match_oracle(kb, vb, engine):
    """5- and 6-bit codes on the tcgen05 kernels (pair tables of 1024 / 4096
    entries, down to one copy per entry)."""
    _run_case(128, kb, vb, False, 2, 2, 4, 300, 300, True, engine)


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
    # with a residual window the newest tokens stay dense and enter exactly
    windowed = TurboQuantKVCache(num_layers=1, batch_size=B, num_heads=Hkv, head_dim=D,
                                 residual_window=8, protected_layers=0, device=DEV)
    got = windowed.prefill(q, k, v, 0)
    ws = windowed._stores[0]
    assert ws._comp_ptr == T - 8 and ws._win_k.shape[2] == 8
    want = ops.prefill_attention(ws.tables, ws._pages, q, T, window_k=k[:, :, T - 8:],
                                 window_v=v[:, :, T - 8:])
    assert torch.equal(got, want)
    assert windowed.device_status() == 0


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


WINDOW_CASES = [
    # kb, vb, n_packed, W, Tq, engine
    (4, 2, 300, 128, 300, 0),      # whole-prompt tail in the window (256-row kernel)
    (4, 2, 0, 100, 100, 0),        # prompt shorter than the window: no packed key
    (6, 4, 170, 128, 50, 2),       # protected layer bits, 128-row kernel, a later chunk
    (3, 3, 64, 33, 97, 3),         # ragged window, 256-row kernel
]


@pytest.mark.parametrize("kb,vb,npk,W,Tq,engine", WINDOW_CASES)
def test_prefill_window_and_left_padding_match_oracle(kb, vb, npk, W, Tq, engine):
    """Residual window (dense keys after the packed ones, attended exactly)
    and kv_start (left padding), against the oracle's SDPA over the
    dequantised packed keys followed by the exact window."""
    D, B, Hkv, g = 128, 3, 2, 4
    n = npk + W
    t = make_tables(D, kb, vb, False)
    pages = new_pages(B * Hkv, max(npk, 1), t)
    if npk:
        ops.append(t, pages, rand_kv((B, Hkv, npk, D), 71).to(DEV),
                   rand_kv((B, Hkv, npk, D), 72).to(DEV), 0)
    wk, wv = rand_kv((B, Hkv, W, D), 73), rand_kv((B, Hkv, W, D), 74)
    q = rand_kv((B, Hkv * g, Tq, D), 75)
    start = [0, min(n - 1, 45), min(n - 2, npk + 5)]
    ks = torch.tensor(start, dtype=torch.int32, device=DEV)
    out = ops.prefill_attention(t, pages, q.to(DEV), n, engine=engine, kv_start=ks,
                                window_k=wk.to(DEV), window_v=wv.to(DEV))
    torch.cuda.synchronize()
    assert ops.device_status(DEV) == 0
    if npk:
        kd, vd = _dequant(t, pages, npk)
        kall = np.concatenate([kd.reshape(B, Hkv, npk, D), wk.float().numpy()], 2)
        vall = np.concatenate([vd.reshape(B, Hkv, npk, D), wv.float().numpy()], 2)
    else:
        kall, vall = wk.float().numpy(), wv.float().numpy()
    want = O.sdpa(q.float().numpy(), kall, vall, causal=True, kv_start=start)
    _check(out, want)
