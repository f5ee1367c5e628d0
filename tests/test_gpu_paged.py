"""Paged storage (block tables) gives bit-identical results to contiguous pages.

vLLM keeps KV in a pool of fixed-size blocks and gives each sequence a row of
block ids (vLLM's PagedAttention block table; the reference's vLLM backend,
bhaskera/vllm_plugin/backend.py, forwards to that layout).  Here logical page
p of stream s lives at pool[block_table[s, p]].  Every kernel that touches
pages (append on CUDA and tensor cores, dequantise, decode, the fused decode
step, prefill on all engines) must store the same bytes into the mapped pool
pages as into a contiguous (streams, pages, page_bytes) tensor, and return the
same outputs bit for bit.  An entry outside the pool must never be
dereferenced: the write is dropped, reads come from pool page 0, and the
status word reports TQ_DEV_BAD_BLOCK.
"""
import pytest
import torch

from bhaskera_col_b200 import _lib
from bhaskera_col_b200.inference import ops
from test_gpu_parity import DEV, make_tables, new_pages, rand_kv

pytestmark = pytest.mark.gpu


def _paged(S, P, pb, spare=3, pad=2, seed=0):
    """A shuffled pool with `spare` unused blocks and a table whose rows are
    `pad` entries wider than P (the extra entries point outside the pool and
    are never read)."""
    g = torch.Generator().manual_seed(seed)
    nblocks = S * P + spare
    perm = torch.randperm(nblocks, generator=g)[:S * P].to(torch.int32)
    full = torch.full((S, P + pad), 1 << 30, dtype=torch.int32)
    full[:, :P] = perm.view(S, P)
    bt = full.to(DEV)[:, :P]
    assert bt.stride(0) == P + pad
    pool = torch.zeros((nblocks, pb), dtype=torch.uint8, device=DEV)
    return ops.PagedPages(pool, bt)


def _gathered(pp: ops.PagedPages) -> torch.Tensor:
    return pp.pool[pp.block_table.long()]


def _unused_blocks_zero(pp: ops.PagedPages) -> bool:
    used = torch.zeros(pp.pool.shape[0], dtype=torch.bool, device=DEV)
    used[pp.block_table.long().flatten()] = True
    return not bool(pp.pool[~used].any())


CASES = [
    # D, kb, vb, qjl, dtype, B, Hkv, g, T, W
    (128, 4, 2, False, torch.bfloat16, 2, 2, 4, 300, 0),   # tensor-core append, tcgen05 prefill
    (128, 4, 4, False, torch.bfloat16, 1, 2, 8, 200, 5),
    (128, 4, 2, True, torch.bfloat16, 2, 2, 4, 300, 0),    # QJL sketch
    (128, 3, 3, False, torch.float16, 1, 3, 5, 257, 0),    # CUDA-core append
    (64, 3, 3, False, torch.bfloat16, 2, 1, 4, 150, 6),
]


@pytest.mark.parametrize("D,kb,vb,qjl,dtype,B,Hkv,g,T,W", CASES)
def test_paged_equals_contiguous(D, kb, vb, qjl, dtype, B, Hkv, g, T, W):
    t = make_tables(D, kb, vb, qjl)
    S = B * Hkv
    k = rand_kv((B, Hkv, T + 1, D), 40, dtype).to(DEV)
    v = rand_kv((B, Hkv, T + 1, D), 41, dtype).to(DEV)
    cont = new_pages(S, T + 1, t)
    P, pb = cont.shape[1], cont.shape[2]
    paged = _paged(S, P, pb)
    cut = 200 if T > 200 else T // 2       # the second chunk starts mid-page
    for pages in (cont, paged):
        ops.append(t, pages, k[:, :, :cut], v[:, :, :cut], 0)
        ops.append(t, pages, k[:, :, cut:T], v[:, :, cut:T], cut)
    torch.cuda.synchronize()
    assert ops.device_status(DEV) == 0
    assert torch.equal(_gathered(paged), cont)
    assert _unused_blocks_zero(paged)

    q = rand_kv((B, Hkv * g, 1, D), 42, outliers=0).to(DEV)
    wk = rand_kv((B, Hkv, W, D), 43).to(DEV) if W else None
    wv = rand_kv((B, Hkv, W, D), 44).to(DEV) if W else None
    ws_c, ws_p = ops.DecodeWorkspace(), ops.DecodeWorkspace()
    oc = ops.decode_attention(t, cont, q, T, wk, wv, workspace=ws_c)
    op = ops.decode_attention(t, paged, q, T, wk, wv, workspace=ws_p)
    torch.cuda.synchronize()
    assert torch.equal(oc, op)

    # the fused decode step appends token T through the table, then attends
    oc = ops.decode_step(t, cont, k[:, :, T:], v[:, :, T:], T, q, wk, wv, workspace=ws_c)
    op = ops.decode_step(t, paged, k[:, :, T:], v[:, :, T:], T, q, wk, wv, workspace=ws_p)
    torch.cuda.synchronize()
    assert ws_c.status() == 0 and ws_p.status() == 0
    assert torch.equal(oc, op)
    assert torch.equal(_gathered(paged), cont)

    n = T + 1
    qp = rand_kv((B, Hkv * g, n - 37, D), 45).to(DEV)
    engines = [0, 1] + ([2, 3] if ops.prefill_uses_tensor_cores(t) else [])
    for e in engines:
        pc = ops.prefill_attention(t, cont, qp, n, engine=e)
        pq = ops.prefill_attention(t, paged, qp, n, engine=e)
        torch.cuda.synchronize()
        assert torch.equal(pc, pq), e

    kc = torch.empty((B, Hkv, n - 37, D), dtype=torch.float32, device=DEV)
    vc = torch.empty_like(kc)
    kq, vq = torch.empty_like(kc), torch.empty_like(kc)
    ops.dequantize(t, cont, 37, n, kc, vc)
    ops.dequantize(t, paged, 37, n, kq, vq)
    torch.cuda.synchronize()
    assert torch.equal(kc, kq) and torch.equal(vc, vq)
    assert ops.device_status(DEV) == 0


def test_paged_bad_entries_flag_and_do_not_write():
    """Entries -1 and num_blocks are skipped on write, read as pool page 0,
    and every kernel reports TQ_DEV_BAD_BLOCK; the valid pages still match."""
    D, B, Hkv, g, T = 128, 1, 2, 4, 200
    t = make_tables(D, 4, 2, False)
    S = B * Hkv
    k = rand_kv((B, Hkv, T, D), 50).to(DEV)
    v = rand_kv((B, Hkv, T, D), 51).to(DEV)
    cont = new_pages(S, T, t)
    P, pb = cont.shape[1], cont.shape[2]
    paged = _paged(S, P, pb, spare=0)
    bt = paged.block_table
    bad = [(0, 3, -1), (1, 1, paged.pool.shape[0])]
    for s, p, val in bad:
        bt[s, p] = val
    ops.append(t, cont, k, v, 0)
    assert ops.device_status(DEV) == 0
    for tc in (True, False):                  # tensor-core and CUDA-core append
        paged.pool.zero_()
        kk, vv = (k, v) if tc else (k.half(), v.half())
        assert ops.append_uses_tensor_cores(t, kk, vv) == tc
        ops.append(t, paged, kk, vv, 0)
        torch.cuda.synchronize()
        assert ops.device_status(DEV) & _lib.DEV_BAD_BLOCK
        if tc:
            ok = torch.ones((S, P), dtype=torch.bool, device=DEV)
            for s, p, _ in bad:
                ok[s, p] = False
            safe = bt.clamp(0, paged.pool.shape[0] - 1).long()
            assert torch.equal(paged.pool[safe][ok], cont[ok])

    q = rand_kv((B, Hkv * g, 1, D), 52, outliers=0).to(DEV)
    ws = ops.DecodeWorkspace()
    out = ops.decode_attention(t, paged, q, T, workspace=ws)
    assert ws.status() & _lib.DEV_BAD_BLOCK
    assert torch.isfinite(out.float()).all()
    out = ops.decode_step(t, paged, k[:, :, :1], v[:, :, :1], 3 * 64, q, workspace=ws)
    assert ws.status() & _lib.DEV_BAD_BLOCK

    qp = rand_kv((B, Hkv * g, T, D), 53).to(DEV)
    for e in (1, 2, 3):
        ops.prefill_attention(t, paged, qp, T, engine=e)
        torch.cuda.synchronize()
        assert ops.device_status(DEV) & _lib.DEV_BAD_BLOCK, e
    kd = torch.empty((B, Hkv, T, D), dtype=torch.float32, device=DEV)
    ops.dequantize(t, paged, 0, T, kd, None)
    torch.cuda.synchronize()
    assert ops.device_status(DEV) & _lib.DEV_BAD_BLOCK
    # the context is healthy afterwards: a clean contiguous decode runs
    ops.decode_attention(t, cont, q, T, workspace=ws)
    assert ws.status() == 0
