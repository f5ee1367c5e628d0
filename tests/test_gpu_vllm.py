"""The vLLM paged path (TurboQuantPagedAttention) over a served batch schedule.

A small scheduler drives one layer through vLLM-shaped steps (flattened
tokens, query_start_loc, seq_lens, block tables of shuffled block ids): whole
prefills, a chunked prefill, mixed prefill + decode steps and decode-only
steps with ragged lengths.  Checks, per step:
  * outputs against the oracle: float64 causal attention (GQA) over the K/V
    dequantised from the codes the kernels stored (the reference's
    decompress, vllm_turboquant.py:218-230, then vLLM's attention), the same
    bar as the prefill and decode tests (cosine >= 0.9999, max-abs within
    4e-3 of max|o| plus half a bf16 ulp);
  * the pool pages, gathered through the block table, byte-identical to a
    contiguous cache fed the same tokens by tq_append (addressing is exact).
"""
import math

import numpy as np
import pytest
import torch

from bhaskera_col_b200.inference import ops
from bhaskera_col_b200.inference.vllm_turboquant import (PAGE_TOKENS, TurboQuantPagedAttention,
                                                         VLLMBatch, layer_bits)
from oracle import tq_oracle as O
from test_gpu_parity import DEV, cosine, rand_kv

pytestmark = pytest.mark.gpu


def _tokens(n, heads, D, seed, outliers=2):
    """(n, heads, D) token-major bf16 rows (the seeded generator works on (B, H, T, D))."""
    return rand_kv((1, heads, n, D), seed, outliers=outliers)[0].transpose(0, 1).contiguous()


class _Sched:
    """Requests with block lists, like vLLM's KV cache manager."""

    def __init__(self, layer: TurboQuantPagedAttention, seed=0):
        self.layer = layer
        g = torch.Generator().manual_seed(seed)
        self.free = torch.randperm(layer.num_blocks, generator=g).tolist()
        self.blocks, self.length = {}, {}
        self.k, self.v = {}, {}                      # raw tokens so far, (T, Hkv, D)
        self.ref = {}                                # contiguous pages per request

    def add(self, r):
        self.blocks[r], self.length[r] = [], 0
        D, H = self.layer.head_dim, self.layer.num_kv_heads
        self.k[r] = torch.zeros((0, H, D), dtype=torch.bfloat16)
        self.v[r] = torch.zeros((0, H, D), dtype=torch.bfloat16)

    def step(self, work, seed):
        """work: [(request, new tokens)], in batch order; returns the step's
        inputs and the layer output."""
        L = self.layer
        H, Hq, D = L.num_kv_heads, L.num_heads, L.head_dim
        qsl, sl, toks_k, toks_v = [0], [], [], []
        for i, (r, n) in enumerate(work):
            if r not in self.blocks:
                self.add(r)
            self.length[r] += n
            while len(self.blocks[r]) * L.block_size < self.length[r]:
                self.blocks[r].append(self.free.pop())
            qsl.append(qsl[-1] + n)
            sl.append(self.length[r])
            k = _tokens(n, H, D, seed + 2 * i)
            v = _tokens(n, H, D, seed + 2 * i + 1)
            self.k[r] = torch.cat([self.k[r], k])
            self.v[r] = torch.cat([self.v[r], v])
            toks_k.append(k)
            toks_v.append(v)
        N = qsl[-1]
        MB = max(len(self.blocks[r]) for r, _ in work) + 1     # a spare column, as vLLM pads
        bt = torch.zeros((len(work), MB), dtype=torch.int32)
        for i, (r, _) in enumerate(work):
            bt[i, :len(self.blocks[r])] = torch.tensor(self.blocks[r], dtype=torch.int32)
        batch = VLLMBatch(torch.tensor(qsl, dtype=torch.int32, device=DEV),
                          torch.tensor(sl, dtype=torch.int32, device=DEV), bt.to(DEV), N,
                          max(n for _, n in work))
        q = _tokens(N, Hq, D, seed + 999, outliers=0).to(DEV)
        key = torch.cat(toks_k).to(DEV)
        val = torch.cat(toks_v).to(DEV)
        out = L.forward(q, key, val, batch)
        # the same tokens through tq_append into contiguous per-request pages
        for (r, n), k, v in zip(work, toks_k, toks_v):
            if r not in self.ref:
                self.ref[r] = torch.zeros((H, 64, L.page_bytes), dtype=torch.uint8, device=DEV)
            ops.append(L.tables, self.ref[r], k.permute(1, 0, 2).unsqueeze(0).to(DEV),
                       v.permute(1, 0, 2).unsqueeze(0).to(DEV), self.length[r] - n)
        torch.cuda.synchronize()
        assert L.workspace.status() == 0
        assert ops.device_status(DEV) == 0
        return batch, q, out

    def pages_of(self, r):
        """The request's pages gathered from the pool, (Hkv, P, page_bytes)."""
        L = self.layer
        bt = torch.tensor([self.blocks[r]], dtype=torch.int32, device=DEV)
        st = L.stream_table(bt)
        return L.pool[st.long()]

    def check(self, work, batch, q, out):
        L = self.layer
        H, Hq, D = L.num_kv_heads, L.num_heads, L.head_dim
        g = Hq // H
        geom = O.PageGeom(D, L.key_bits, L.value_bits, False)
        R = L.tables.rot.cpu().numpy()
        qsl = batch.query_start_loc.tolist()
        for i, (r, n) in enumerate(work):
            T = self.length[r]
            got = self.pages_of(r)
            P = -(-T // PAGE_TOKENS)
            assert torch.equal(got[:, :P], self.ref[r][:, :P]), r
            f = O.parse_pages(geom, got.cpu().numpy(), T)
            kd = O.decode_range(f["k_idx"], f["k_norm"], L.tables.k_centroids.cpu().numpy(), R)
            vd = O.decode_range(f["v_idx"], f["v_norm"], L.tables.v_centroids.cpu().numpy(), R)
            qs = q[qsl[i]:qsl[i + 1]].double().cpu().numpy()          # (n, Hq, D)
            want = np.zeros((n, Hq, D))
            for h in range(Hq):
                kh, vh = kd[h // g].astype(np.float64), vd[h // g].astype(np.float64)
                s = qs[:, h] @ kh.T * L.scale                         # (n, T)
                pos = T - n + np.arange(n)
                s[np.arange(T)[None, :] > pos[:, None]] = -np.inf
                p = np.exp(s - s.max(1, keepdims=True))
                want[:, h] = (p / p.sum(1, keepdims=True)) @ vh
            o = out[qsl[i]:qsl[i + 1]].float().cpu().numpy()
            top = np.abs(want).max()
            half_ulp = 2.0 ** (math.floor(math.log2(top)) - 8)
            assert cosine(o, want) >= 0.9999, (r, cosine(o, want))
            assert np.abs(o - want).max() <= 4e-3 * top + half_ulp, r


@pytest.mark.parametrize("block_size,layer_idx", [(64, 5), (128, 0)])
def test_vllm_schedule_matches_oracle(block_size, layer_idx):
    layer = TurboQuantPagedAttention(layer_idx, 32, num_heads=8, num_kv_heads=2, head_dim=128,
                                     num_blocks=64, block_size=block_size, key_bits=4,
                                     value_bits=2, protected_layers=2, device=DEV)
    assert (layer.key_bits, layer.value_bits) == layer_bits(layer_idx, 32, 4, 2, 2)
    s = _Sched(layer, seed=block_size)
    plan = [
        [("A", 150), ("B", 70), ("C", 200)],          # prefills, C chunked
        [("A", 1), ("B", 1), ("C", 100)],             # two decodes + C's second chunk
        [("A", 1), ("B", 1), ("C", 1)],               # decode only, ragged
        [("C", 1), ("A", 1), ("B", 1)],               # another order
        [("A", 1), ("D", 64), ("B", 1), ("C", 1)],    # a new request in a decode batch
        [("D", 1), ("A", 1), ("B", 1), ("C", 1)],
    ]
    for i, work in enumerate(plan):
        batch, q, out = s.step(work, seed=100 * i)
        s.check(work, batch, q, out)
    assert layer.tokens_stored == sum(n for w in plan for _, n in w)


def test_vllm_decode_batch_is_one_call_without_host_sync():
    """A decode-only batch runs the fused store + ragged decode and never
    needs the host copies of seq_lens / query_start_loc."""
    layer = TurboQuantPagedAttention(3, 32, 8, 2, 128, 32, 64, device=DEV)
    s = _Sched(layer)
    s.step([("A", 100), ("B", 30)], seed=1)
    work = [("A", 1), ("B", 1)]
    batch, q, out = s.step(work, seed=2)
    assert batch.query_start_loc_cpu is None and batch.seq_lens_cpu is None
    s.check(work, batch, q, out)
