"""CPU baseline of the reference's TurboQuant path — TEST/BENCH INFRASTRUCTURE.

Only bench.py's cpu_baseline leg and ``--impl reference`` arm use this module.
It restates, with torch CPU ops (the reference's own framework, all host
threads), the work the reference does per layer per decode step
(aditya25058/Bhaskera_col src/bhaskera/inference/kv_cache.py):

  update(k, v) with residual_window = 0               kv_cache.py:445-490
    window = cat(window, new) in the model dtype       :461-466
    evict -> _compress_chunk: per-token loop of fp32 norm, normalise,
            rotate (u @ R^T), bucketize, store codes + fp16 norms  :355-399
    _decode_range of the evicted rows, cat onto the decoded history
                                                       :402-439
    return cat(decoded history, window)                :483-488
  then HF SDPA over the returned bf16 K/V with GQA     (engine.py:389)

and, for the prefill append, _compress_chunk over a whole chunk of tokens.
"""
from __future__ import annotations

import math
import os
import time
from typing import Tuple

import torch
import torch.nn.functional as F


def _rotation(d: int, seed: int) -> torch.Tensor:
    nt = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        g = torch.Generator(device="cpu")
        g.manual_seed(seed)
        Q, R = torch.linalg.qr(torch.randn(d, d, generator=g))
        s = torch.sign(torch.diag(R))
        s[s == 0] = 1.0
        return Q * s.unsqueeze(0)
    finally:
        torch.set_num_threads(nt)


class RefLayer:
    """State of one reference _LayerKVStore with its decoded bf16 history."""

    def __init__(self, B, H, D, T, key_bits, value_bits, kc, kb, vc, vb, seed=42,
                 dtype=torch.bfloat16, history=True):
        """``history``: start with a random decoded history of T tokens (a
        steady-state timing sample); False: start empty, with room for T + 64
        compressed tokens (the parity check against the reference's own
        outputs)."""
        self.B, self.H, self.D, self.dtype = B, H, D, dtype
        self.kc, self.kb, self.vc, self.vb = kc, kb, vc, vb
        self.R = _rotation(D, seed)
        cap = T + 64
        self.k_idx = torch.zeros(cap, B * H, D, dtype=torch.int16)
        self.v_idx = torch.zeros(cap, B * H, D, dtype=torch.int16)
        self.k_norm = torch.zeros(cap, B * H, dtype=torch.float16)
        self.v_norm = torch.zeros(cap, B * H, dtype=torch.float16)
        self.comp = T if history else 0
        g = torch.Generator(device="cpu")
        g.manual_seed(seed)
        # decoded history of T tokens (values only matter for timing)
        n = T if history else 0
        self.dec_k = torch.randn(B, H, n, D, generator=g).to(dtype)
        self.dec_v = torch.randn(B, H, n, D, generator=g).to(dtype)

    def _compress(self, k: torch.Tensor, v: torch.Tensor) -> None:
        B, H, T, D = k.shape
        kf = k.permute(2, 0, 1, 3).reshape(T, B * H, D)
        vf = v.permute(2, 0, 1, 3).reshape(T, B * H, D)
        for t in range(T):
            if self.comp >= self.k_idx.shape[0]:
                self.comp = 0           # bounded sample: reuse the row range
            for x, b, idx, nrm in ((kf[t], self.kb, self.k_idx, self.k_norm),
                                   (vf[t], self.vb, self.v_idx, self.v_norm)):
                x = x.float()
                n = x.norm(dim=-1)
                u = x / n.unsqueeze(-1).clamp(min=1e-8)
                y = u @ self.R.T
                idx[self.comp] = torch.bucketize(y.reshape(-1), b).reshape(y.shape).to(torch.int16)
                nrm[self.comp] = n.to(torch.float16)
            self.comp += 1
        r0 = self.comp - T
        dk = self._decode(self.k_idx[r0:self.comp], self.k_norm[r0:self.comp], self.kc, T)
        dv = self._decode(self.v_idx[r0:self.comp], self.v_norm[r0:self.comp], self.vc, T)
        self.dec_k = torch.cat([self.dec_k, dk], dim=2)
        self.dec_v = torch.cat([self.dec_v, dv], dim=2)

    def _decode(self, idx, nrm, c, T):
        x = (c[idx.long()] @ self.R) * nrm.float().unsqueeze(-1)
        return x.reshape(T, self.B, self.H, self.D).permute(1, 2, 0, 3).to(self.dtype)

    def decode_step(self, k, v, q) -> torch.Tensor:
        win_k, win_v = k.to(self.dtype), v.to(self.dtype)
        self._compress(win_k.float(), win_v.float())
        win_k, win_v = win_k[:, :, 1:], win_v[:, :, 1:]
        full_k = torch.cat([self.dec_k, win_k], dim=2)
        full_v = torch.cat([self.dec_v, win_v], dim=2)
        out = F.scaled_dot_product_attention(q, full_k, full_v, enable_gqa=True)
        # keep the history length fixed for a steady-state sample
        self.dec_k, self.dec_v = self.dec_k[:, :, 1:], self.dec_v[:, :, 1:]
        return out

    def append_chunk(self, k, v) -> None:
        self._compress(k.to(self.dtype).float(), v.to(self.dtype).float())
        T = k.shape[2]
        self.dec_k, self.dec_v = self.dec_k[:, :, T:], self.dec_v[:, :, T:]


def codebook(d: int, bits: int) -> Tuple[torch.Tensor, torch.Tensor]:
    from .tq_oracle import solve_lloyd_max
    c, b = solve_lloyd_max(d, bits)
    return torch.from_numpy(c), torch.from_numpy(b)


def time_decode(B, Hq, Hkv, D, T, key_bits, value_bits, steps=2, seed=0):
    """Seconds per layer per decode step of the reference CPU path."""
    kc, kb = codebook(D, key_bits)
    vc, vb = codebook(D, value_bits)
    layer = RefLayer(B, Hkv, D, T, key_bits, value_bits, kc, kb, vc, vb)
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    q = torch.randn(B, Hq, 1, D, generator=g).to(torch.bfloat16)
    times = []
    for i in range(steps + 1):
        k = torch.randn(B, Hkv, 1, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, Hkv, 1, D, generator=g).to(torch.bfloat16)
        t0 = time.perf_counter()
        layer.decode_step(k, v, q)
        if i:
            times.append(time.perf_counter() - t0)
    return sum(times) / len(times)


def time_append(B, H, D, T, bits, tokens=64, seed=0):
    """Seconds to append `tokens` tokens of one layer on the reference CPU path."""
    c, b = codebook(D, bits)
    layer = RefLayer(B, H, D, 1, bits, bits, c, b, c, b)
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    k = torch.randn(B, H, tokens, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, H, tokens, D, generator=g).to(torch.bfloat16)
    t0 = time.perf_counter()
    layer.append_chunk(k, v)
    return time.perf_counter() - t0


def host_threads() -> int:
    return torch.get_num_threads()


def use_all_host_threads() -> int:
    """Give torch every core this process may run on (a launcher such as
    torchrun sets OMP_NUM_THREADS=1 per rank); returns the thread count."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    torch.set_num_threads(max(1, n))
    return torch.get_num_threads()


def host_cores() -> int:
    return os.cpu_count() or 1
