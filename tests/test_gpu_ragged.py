"""Ragged decode batches (continuous batching): every batch row has its own
token count (vLLM's seq_lens), on contiguous pages and behind block tables.

Row b of a ragged decode must give the oracle's attention over its own
tokens [0, seq_lens[b]) (decode_attention_codes, the reference's single-query
attention over the stored codes, kv_cache.py:445-490 with engine.py:389);
a ragged decode step must store row b's token at seq_lens[b] - 1 with the same
page bytes as tq_append there, and return the same output as that append
followed by the ragged decode.  Same bar as the uniform decode: max-abs within
2e-3 of max|o| plus the bf16 rounding, cosine >= 0.9999.
"""
import numpy as np
import pytest
import torch

from bhaskera_col_b200.inference import ops
from oracle import tq_oracle as O
from bhaskera_col_b200.inference.kv_cache import _generate_qjl_matrix
from test_gpu_parity import DEV, cosine, make_tables, new_pages, parse, rand_kv

pytestmark = pytest.mark.gpu


def _oracle_rows(t, pages, q, lens, Hkv, wk=None, wv=None):
    """The oracle per batch row over its own tokens; (B, Hq, D) float64."""
    B, Hq, _, D = q.shape
    Smat = _generate_qjl_matrix(D, 42).numpy() if t.qjl else None
    out = np.zeros((B, Hq, D))
    for b, T in enumerate(lens):
        W = wk.shape[2] if wk is not None else 0
        if T == 0 and W == 0:
            continue                                    # nothing to attend: output 0
        _, got = parse(t, pages[b * Hkv:(b + 1) * Hkv], max(T, 1))
        sub = lambda k: got.get(k)
        out[b] = O.decode_attention_codes(
            q[b:b + 1, :, 0].float().cpu().numpy(), sub("k_idx"), sub("v_idx"), sub("k_norm"),
            sub("v_norm"), t.k_centroids.cpu().numpy(), t.v_centroids.cpu().numpy(),
            t.rot.cpu().numpy(), qbits=sub("qbits"), gamma=sub("gamma"), S=Smat, T=T,
            window_k=wk[b:b + 1].float().cpu().numpy() if W else None,
            window_v=wv[b:b + 1].float().cpu().numpy() if W else None)[0]
    return out


def _close(o, want):
    o = o[:, :, 0].float().cpu().numpy()
    top = np.abs(want).max()
    assert np.abs(o - want).max() <= 2e-3 * top + 2 ** -8 * top
    if top > 0:
        assert cosine(o, want) >= 0.9999


CASES = [
    # D, kb, vb, qjl, Hkv, g, lens, W
    (128, 4, 2, True, 2, 4, [300, 17, 64, 129], 0),
    (128, 4, 2, False, 8, 4, [1000, 1, 65, 700, 0, 333], 0),     # an empty row
    (128, 3, 3, False, 2, 5, [250, 3], 4),                       # with a window
    (64, 4, 2, True, 1, 8, [40, 200, 128], 0),
    (32, 4, 2, False, 2, 2, [5, 80], 3),
]


@pytest.mark.parametrize("D,kb,vb,qjl,Hkv,g,lens,W", CASES)
def test_ragged_decode_matches_oracle(D, kb, vb, qjl, Hkv, g, lens, W):
    t = make_tables(D, kb, vb, qjl)
    B, n = len(lens), max(lens)
    k, v = rand_kv((B, Hkv, n, D), 60), rand_kv((B, Hkv, n, D), 61)
    pages = new_pages(B * Hkv, n, t)
    ops.append(t, pages, k.to(DEV), v.to(DEV), 0)       # tokens past a row's length are ignored
    q = rand_kv((B, Hkv * g, 1, D), 62, outliers=0).to(DEV)
    wk = rand_kv((B, Hkv, W, D), 63).to(DEV) if W else None
    wv = rand_kv((B, Hkv, W, D), 64).to(DEV) if W else None
    sl = torch.tensor(lens, dtype=torch.int32, device=DEV)
    ws = ops.DecodeWorkspace()
    outs = [ops.decode_attention(t, pages, q, n, wk, wv, workspace=ws, seq_lens=sl, num_ctas=c)
            for c in (0, 1, 7)]
    torch.cuda.synchronize()
    assert ws.status() == 0
    want = _oracle_rows(t, pages, q, lens, Hkv, wk, wv)
    for o in outs:
        _close(o, want)


def test_ragged_uniform_lengths_equal_uniform_decode():
    D, B, Hkv, g, T = 128, 3, 4, 4, 777
    t = make_tables(D, 4, 2, True)
    pages = new_pages(B * Hkv, T, t)
    ops.append(t, pages, rand_kv((B, Hkv, T, D), 65).to(DEV), rand_kv((B, Hkv, T, D), 66).to(DEV), 0)
    q = rand_kv((B, Hkv * g, 1, D), 67, outliers=0).to(DEV)
    ref = ops.decode_attention(t, pages, q, T).float()
    for lens in ([T] * B, [T + 50] * B):        # lengths above n_tokens are clamped to it
        sl = torch.tensor(lens, dtype=torch.int32, device=DEV)
        got = ops.decode_attention(t, pages, q, T, seq_lens=sl).float()
        assert torch.allclose(got, ref, atol=2e-2 * ref.abs().max().item())
        assert cosine(got.cpu().numpy(), ref.cpu().numpy()) >= 0.99999


@pytest.mark.parametrize("paged", [False, True])
def test_ragged_decode_step(paged):
    """Row b stores its token at lens[b] - 1: page bytes as tq_append there,
    output as append + ragged decode (same layout, so bit-identical)."""
    D, Hkv, g = 128, 4, 4
    t = make_tables(D, 4, 2, True)
    lens = [200, 1, 64, 0, 129]                # row 3 is empty: nothing stored
    B, n = len(lens), max(lens)
    k, v = rand_kv((B, Hkv, n, D), 70).to(DEV), rand_kv((B, Hkv, n, D), 71).to(DEV)
    kn, vn = rand_kv((B, Hkv, 1, D), 72).to(DEV), rand_kv((B, Hkv, 1, D), 73).to(DEV)
    q = rand_kv((B, Hkv * g, 1, D), 74, outliers=0).to(DEV)
    pa, pb = new_pages(B * Hkv, n, t), new_pages(B * Hkv, n, t)
    for p in (pa, pb):
        ops.append(t, p, k, v, 0)
    for b, L in enumerate(lens):               # the reference order: append, then attend
        if L:
            rows = slice(b * Hkv, (b + 1) * Hkv)
            ops.append(t, pa[rows], kn[b:b + 1], vn[b:b + 1], L - 1)
    sl = torch.tensor(lens, dtype=torch.int32, device=DEV)
    want = ops.decode_attention(t, pa, q, n, seq_lens=sl)
    if paged:
        S, P, pbytes = pb.shape
        perm = torch.randperm(S * P + 5, generator=torch.Generator().manual_seed(3))[:S * P]
        pool = torch.zeros((S * P + 5, pbytes), dtype=torch.uint8, device=DEV)
        bt = perm.to(torch.int32).view(S, P).to(DEV)
        pool[bt.long()] = pb
        target = ops.PagedPages(pool, bt)
    else:
        target = pb
    ws = ops.DecodeWorkspace()
    got = ops.decode_step(t, target, kn, vn, n - 1, q, workspace=ws, seq_lens=sl)
    torch.cuda.synchronize()
    assert ws.status() == 0
    after = target.pool[target.block_table.long()] if paged else target
    assert torch.equal(after, pa)
    assert torch.equal(got, want)
    _close(got, _oracle_rows(t, pa, q, lens, Hkv))


def test_ragged_many_streams_skewed():
    """1,280 streams (the stream search takes three rounds), one long row
    among short and empty ones, on a block-table pool."""
    D, Hkv, g = 128, 8, 2
    t = make_tables(D, 4, 2, False)
    rng = np.random.default_rng(5)
    lens = [int(x) for x in rng.integers(0, 40, 160)]
    lens[17] = 1500
    B, n = len(lens), max(lens)
    S = B * Hkv
    cont = new_pages(S, n, t)
    ops.append(t, cont, rand_kv((B, Hkv, 40, D), 80).to(DEV), rand_kv((B, Hkv, 40, D), 81).to(DEV), 0)
    long_rows = cont[17 * Hkv:18 * Hkv]
    ops.append(t, long_rows, rand_kv((1, Hkv, n - 40, D), 83).to(DEV),
               rand_kv((1, Hkv, n - 40, D), 84).to(DEV), 40)
    P = cont.shape[1]
    perm = torch.randperm(S * P, generator=torch.Generator().manual_seed(4)).to(torch.int32)
    bt = perm.view(S, P).to(DEV)
    pool = torch.empty((S * P, cont.shape[2]), dtype=torch.uint8, device=DEV)
    pool[bt.long()] = cont
    paged = ops.PagedPages(pool, bt)
    q = rand_kv((B, Hkv * g, 1, D), 82, outliers=0).to(DEV)
    sl = torch.tensor(lens, dtype=torch.int32, device=DEV)
    ws = ops.DecodeWorkspace()
    got = ops.decode_attention(t, paged, q, n, workspace=ws, seq_lens=sl)
    got_c = ops.decode_attention(t, cont, q, n, seq_lens=sl)
    torch.cuda.synchronize()
    assert ws.status() == 0
    assert torch.equal(got, got_c)
    _close(got, _oracle_rows(t, cont, q, lens, Hkv))
