"""TurboQuant KV cache on B200 — drop-in for bhaskera.inference.kv_cache.

Same module surface as the reference (aditya25058/Bhaskera_col
src/bhaskera/inference/kv_cache.py): ``BaseKVCache`` (a transformers
``Cache``), ``StaticKVCache``, ``FastLloydMaxCodebook``,
``_generate_rotation_matrix``, ``TurboQuantKVCache`` and ``build_kv_cache``,
with the same constructor arguments, ``update()`` contract, error behaviour
and ``compression_stats()`` keys.

What changes underneath: compressed tokens live in bit-packed 64-token pages
on the GPU (layout in include/tq_b200.h), written by one fused CUDA append
kernel (norm -> rotate -> bucketize -> pack -> optional QJL sketch).
``update()`` still returns dense (B, H, T, D) K/V in the model dtype for
stock HF attention; ``attend()`` runs the fused decode-attention kernel
straight off the packed pages and never materialises dense K/V.

There is no CPU path: constructing a TurboQuantKVCache on a non-CUDA device
raises.
"""
from __future__ import annotations

import logging
import math
from abc import abstractmethod
from typing import Any, Dict, List, Optional, Tuple

import torch

try:  # the reference subclasses transformers' Cache (kv_cache.py:46, 124)
    from transformers.cache_utils import Cache as _HFCache
except Exception:  # pragma: no cover - transformers is optional for the kernels
    _HFCache = object

from . import ops
from .lloyd_max import solve_lloyd_max

logger = logging.getLogger(__name__)

QJL_SEED_OFFSET = 1_000_003      # QJL sketch seed = rotation seed + this
PAGE_TOKENS = 64


# ---------------------------------------------------------------------------
# Rotation matrix (kv_cache.py:55-68)
# ---------------------------------------------------------------------------

def _generate_rotation_matrix(d: int, seed: int = 42,
                              device: torch.device = torch.device("cpu")) -> torch.Tensor:
    """Haar-random orthogonal (d, d) matrix from a seeded CPU Gaussian.

    QR of torch's seeded CPU normal stream with the columns' signs fixed by
    sign(diag(R)), zero signs -> +1 — the reference's construction.  QR runs
    on one CPU thread: LAPACK's threaded QR rounds differently with the
    thread count (1e-6 level), and the stored codes depend on every bit.
    """
    nt = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        gen = torch.Generator(device="cpu")
        gen.manual_seed(seed)
        G = torch.randn(d, d, generator=gen)
        Q, Rr = torch.linalg.qr(G)
        sgn = torch.sign(torch.diag(Rr))
        sgn[sgn == 0] = 1.0
        Q = Q * sgn.unsqueeze(0)
    finally:
        torch.set_num_threads(nt)
    return Q.to(device)


def _generate_qjl_matrix(d: int, rotation_seed: int,
                         device: torch.device = torch.device("cpu")) -> torch.Tensor:
    """(d, d) sketch matrix for the 1-bit QJL residual: i.i.d. N(0,1) draws
    rounded to bf16 (exact bf16 values, so the tensor-core append forms S r
    with a single S term; the rounding moves each entry by < 2^-9 of itself)."""
    gen = torch.Generator(device="cpu")
    gen.manual_seed(rotation_seed + QJL_SEED_OFFSET)
    return torch.randn(d, d, generator=gen).bfloat16().float().to(device)


# ---------------------------------------------------------------------------
# Codebook (kv_cache.py:75-117)
# ---------------------------------------------------------------------------

class FastLloydMaxCodebook:
    """Lloyd-Max codebook pinned to a device.  ``quantize`` is the bit-exact
    bucketize kernel (tq_quantize_rotated); CUDA tensors only."""

    _cache: Dict[tuple, "FastLloydMaxCodebook"] = {}
    _tables: Dict[tuple, Tuple[torch.Tensor, torch.Tensor]] = {}

    def __init__(self, d: int, bits: int, device: torch.device):
        self.d = d
        self.bits = bits
        self.n_levels = 2 ** bits
        self.device = torch.device(device)
        key = (d, bits)
        if key not in FastLloydMaxCodebook._tables:
            FastLloydMaxCodebook._tables[key] = solve_lloyd_max(d, bits)
        c, b = FastLloydMaxCodebook._tables[key]
        self.centroids = c.to(self.device)
        self.boundaries = b.to(self.device)

    @classmethod
    def get(cls, d: int, bits: int, device: torch.device) -> "FastLloydMaxCodebook":
        key = (d, bits, str(device))
        if key not in cls._cache:
            cls._cache[key] = cls(d, bits, device)
        return cls._cache[key]

    def quantize(self, x: torch.Tensor) -> torch.Tensor:
        """(..., d) fp32 -> (..., d) int16 codes: #{boundaries < x}."""
        return ops.quantize_rotated(x, self.boundaries)

    def dequantize(self, indices: torch.Tensor) -> torch.Tensor:
        return self.centroids[indices.long()]


# ---------------------------------------------------------------------------
# Base class (kv_cache.py:124-163)
# ---------------------------------------------------------------------------

class BaseKVCache(_HFCache):

    @abstractmethod
    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Optional[Dict[str, Any]] = None
               ) -> Tuple[torch.Tensor, torch.Tensor]: ...

    @abstractmethod
    def reset(self) -> None: ...

    def get_seq_length(self, layer_idx: Optional[int] = 0) -> int:
        return self.seq_len

    def get_mask_sizes(self, query_length: int, layer_idx: int = 0) -> Tuple[int, int]:
        """(kv_length, kv_offset) for transformers' mask builders: the stored
        tokens plus the query's.  transformers 5's default assumes per-layer
        cache objects and fails on this cache otherwise."""
        return self.get_seq_length(layer_idx) + query_length, 0

    @property
    @abstractmethod
    def seq_len(self) -> int: ...

    def memory_bytes(self) -> int:
        return 0

    def advance(self, n: int = 1) -> None:
        pass

    @property
    def layers(self) -> list:
        return [None] * getattr(self, "num_layers", 0)

    @property
    def is_compileable(self) -> bool:
        return False


# ---------------------------------------------------------------------------
# StaticKVCache (kv_cache.py:170-226)
# ---------------------------------------------------------------------------

class StaticKVCache(BaseKVCache):
    """Pre-allocated contiguous full-precision cache (no compression)."""

    def __init__(self, num_layers: int, batch_size: int, num_heads: int, head_dim: int,
                 max_seq_len: int, dtype: torch.dtype = torch.bfloat16,
                 device: torch.device = torch.device("cpu")):
        self.num_layers = num_layers
        self.batch_size = batch_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.max_seq_len = max_seq_len
        self.dtype = dtype
        self.device = device
        self._seq_len = 0
        shape = (batch_size, num_heads, max_seq_len, head_dim)
        self._keys = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        self._values = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        n = key_states.shape[2]
        end = self._seq_len + n
        if end > self.max_seq_len:
            raise ValueError(f"StaticKVCache overflow: cur={self._seq_len} + new={n} > "
                             f"max={self.max_seq_len}")
        self._keys[layer_idx][:, :, self._seq_len:end] = key_states.to(self.dtype)
        self._values[layer_idx][:, :, self._seq_len:end] = value_states.to(self.dtype)
        return self._keys[layer_idx][:, :, :end], self._values[layer_idx][:, :, :end]

    def advance(self, n: int = 1) -> None:
        self._seq_len += n

    def reset(self) -> None:
        for k, v in zip(self._keys, self._values):
            k.zero_()
            v.zero_()
        self._seq_len = 0

    @property
    def seq_len(self) -> int:
        return self._seq_len

    def memory_bytes(self) -> int:
        elem = self.batch_size * self.num_heads * self.max_seq_len * self.head_dim
        bpe = {torch.float32: 4, torch.float16: 2, torch.bfloat16: 2}.get(self.dtype, 2)
        return 2 * self.num_layers * elem * bpe


# ---------------------------------------------------------------------------
# Per-layer packed store
# ---------------------------------------------------------------------------

class _LayerKVStore:
    """One layer: packed pages on the GPU, a full-precision residual window of
    the newest tokens, and (only if ``store_and_get`` is used) a dense copy of
    the dequantised history for stock attention.

    Window semantics follow _LayerKVStore.store_and_get (kv_cache.py:445-490):
    new tokens join the window in the model dtype; the oldest
    ``len(window) - residual_window`` tokens are evicted into compressed
    storage.  Protected layers use +2 bits capped at 8 (kv_cache.py:290-291).
    """

    def __init__(self, head_dim: int, key_bits: int, value_bits: int, max_seq_len: int,
                 batch_size: int, num_heads: int, rotation_seed: int, device: torch.device,
                 dtype: torch.dtype, full_precision: bool = False, qjl: bool = False):
        self.head_dim = head_dim
        self.device = device
        self.dtype = dtype
        self.batch_size = batch_size
        self.num_heads = num_heads
        self.max_seq_len = max_seq_len
        self.key_bits = min(key_bits + 2, 8) if full_precision else key_bits
        self.value_bits = min(value_bits + 2, 8) if full_precision else value_bits
        self.rotation_seed = rotation_seed
        self.qjl = qjl
        self.k_cb = FastLloydMaxCodebook.get(head_dim, self.key_bits, device)
        self.v_cb = FastLloydMaxCodebook.get(head_dim, self.value_bits, device)
        self._R = _generate_rotation_matrix(head_dim, seed=rotation_seed, device=device)
        S = _generate_qjl_matrix(head_dim, rotation_seed, device) if qjl else None
        self.tables = ops.LayerTables(head_dim, self.key_bits, self.value_bits, qjl,
                                      self.k_cb.centroids, self.k_cb.boundaries,
                                      self.v_cb.centroids, self.v_cb.boundaries,
                                      self._R.contiguous().float(), S)
        self.page_bytes = ops.page_bytes(head_dim, self.key_bits, self.value_bits, qjl)
        self._pages: Optional[torch.Tensor] = None
        self._comp_ptr = 0
        self._win_k: Optional[torch.Tensor] = None
        self._win_v: Optional[torch.Tensor] = None
        self._dense_k: Optional[torch.Tensor] = None
        self._dense_v: Optional[torch.Tensor] = None
        self._dense_valid = 0
        self._allocated = False
        self.workspace = ops.DecodeWorkspace()
        # scratch of a windowed prefill (the rotated window); kept apart from the
        # decode workspace, whose first word is the decode status word
        self.prefill_workspace = ops.DecodeWorkspace()

    # -- storage -------------------------------------------------------------
    def _lazy_alloc(self, B: int, H: int) -> None:
        """Allocate from the first real tensor's B and H (kv_cache.py:323-339)."""
        if self._allocated:
            return
        self.batch_size, self.num_heads = B, H
        pages = -(-max(self.max_seq_len, 1) // PAGE_TOKENS)
        self._pages = torch.zeros((B * H, pages, self.page_bytes), dtype=torch.uint8,
                                  device=self.device)
        self._allocated = True

    @property
    def capacity(self) -> int:
        return 0 if self._pages is None else self._pages.shape[1] * PAGE_TOKENS

    def _ensure_capacity(self, n_tokens: int) -> None:
        """Grow by max(128 tokens, half the capacity) when full (kv_cache.py:369-376)."""
        while self._comp_ptr + n_tokens > self.capacity:
            extra_tok = max(128, self.capacity // 2)
            extra = -(-extra_tok // PAGE_TOKENS)
            old = self._pages
            new = torch.zeros((old.shape[0], old.shape[1] + extra, old.shape[2]),
                              dtype=torch.uint8, device=self.device)
            new[:, : old.shape[1]] = old
            self._pages = new

    def compress(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Append (B, H, T, D) tokens to the packed store."""
        T = k.shape[2]
        if T == 0:
            return
        self._ensure_capacity(T)
        ops.append(self.tables, self._pages, k, v, self._comp_ptr)
        self._comp_ptr += T

    def store(self, k: torch.Tensor, v: torch.Tensor, residual_window: int) -> None:
        B, H, _, D = k.shape
        self._lazy_alloc(B, H)
        k = k.to(self.dtype)
        v = v.to(self.dtype)
        if residual_window <= 0 and self._win_k is None:
            self.compress(k, v)
            return
        if self._win_k is None:
            self._win_k, self._win_v = k, v
        else:
            self._win_k = torch.cat([self._win_k, k], dim=2)
            self._win_v = torch.cat([self._win_v, v], dim=2)
        evict = self._win_k.shape[2] - residual_window
        if evict > 0:
            ek, ev = self._win_k[:, :, :evict], self._win_v[:, :, :evict]
            self._win_k = self._win_k[:, :, evict:]
            self._win_v = self._win_v[:, :, evict:]
            self.compress(ek, ev)

    # -- dense view for stock attention (kv_cache.py:483-488) -----------------
    def dense(self) -> Tuple[torch.Tensor, torch.Tensor]:
        B, H, D = self.batch_size, self.num_heads, self.head_dim
        W = 0 if self._win_k is None else self._win_k.shape[2]
        need = self._comp_ptr + W
        if self._dense_k is None or self._dense_k.shape[2] < need:
            cap = max(need, self.capacity, 1)
            nk = torch.empty((B, H, cap, D), dtype=self.dtype, device=self.device)
            nv = torch.empty_like(nk)
            if self._dense_k is not None and self._dense_valid:
                nk[:, :, : self._dense_valid] = self._dense_k[:, :, : self._dense_valid]
                nv[:, :, : self._dense_valid] = self._dense_v[:, :, : self._dense_valid]
            self._dense_k, self._dense_v = nk, nv
        if self._dense_valid < self._comp_ptr:
            t0, t1 = self._dense_valid, self._comp_ptr
            ops.dequantize(self.tables, self._pages, t0, t1,
                           self._dense_k[:, :, t0:t1], self._dense_v[:, :, t0:t1])
            self._dense_valid = t1
        if W:
            self._dense_k[:, :, self._comp_ptr:need] = self._win_k
            self._dense_v[:, :, self._comp_ptr:need] = self._win_v
        return self._dense_k[:, :, :need], self._dense_v[:, :, :need]

    def store_and_get(self, k, v, residual_window):
        self.store(k, v, residual_window)
        return self.dense()

    # -- fused decode attention ----------------------------------------------
    def attend(self, q: torch.Tensor, scale: Optional[float] = None,
               out: Optional[torch.Tensor] = None,
               kv_start: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Single-token attention of q (B, Hq, 1, D) over everything stored."""
        if not self._allocated:
            raise RuntimeError("attend() before any token was stored in this layer")
        return ops.decode_attention(self.tables, self._pages, q, self._comp_ptr,
                                    self._win_k, self._win_v, scale=scale, out=out,
                                    workspace=self.workspace, kv_start=kv_start)

    def decode(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, residual_window: int,
               scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
               gather=None, kv_start: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Store one new token and attend q to everything stored, in one fused
        call when exactly one token moves into packed storage this step.
        ``gather`` (a _lib.Gather, see head_parallel.SharedGather) fuses the
        multi-GPU output all-gather into that call."""
        B, H, T, D = k.shape
        self._lazy_alloc(B, H)
        k = k.to(self.dtype)
        v = v.to(self.dtype)
        W = 0 if self._win_k is None else self._win_k.shape[2]
        if gather is not None and not (T == 1 and residual_window <= 0 and W == 0):
            raise ValueError("the fused all-gather needs a single-token decode without a "
                             "residual window")
        if T == 1 and residual_window <= 0 and W == 0:
            self._ensure_capacity(1)
            out = ops.decode_step(self.tables, self._pages, k, v, self._comp_ptr, q, scale=scale,
                                  out=out, workspace=self.workspace, gather=gather,
                                  kv_start=kv_start)
            self._comp_ptr += 1
            return out
        if T == 1 and 0 < residual_window == W:
            # the oldest window token is evicted into packed storage
            ek, ev = self._win_k[:, :, :1], self._win_v[:, :, :1]
            wk = torch.cat([self._win_k[:, :, 1:], k], dim=2)
            wv = torch.cat([self._win_v[:, :, 1:], v], dim=2)
            self._ensure_capacity(1)
            out = ops.decode_step(self.tables, self._pages, ek, ev, self._comp_ptr, q,
                                  window_k=wk, window_v=wv, scale=scale, out=out,
                                  workspace=self.workspace, kv_start=kv_start)
            self._comp_ptr += 1
            self._win_k, self._win_v = wk, wv
            return out
        self.store(k, v, residual_window)
        return self.attend(q, scale=scale, out=out, kv_start=kv_start)

    def prefill(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, residual_window: int,
                scale: Optional[float] = None, causal: bool = True,
                out: Optional[torch.Tensor] = None,
                kv_start: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Store T new tokens (reference window semantics) and return the
        attention of q (B, Hq, T, D) at their positions over everything stored:
        the packed tokens straight off the pages, the residual window's tokens
        exactly.  ``kv_start`` (int32 (B,)): left padding per batch row."""
        self.store(k, v, residual_window)
        W = 0 if self._win_k is None else self._win_k.shape[2]
        return ops.prefill_attention(self.tables, self._pages, q, self._comp_ptr + W,
                                     scale=scale, causal=causal, out=out, kv_start=kv_start,
                                     window_k=self._win_k if W else None,
                                     window_v=self._win_v if W else None,
                                     workspace=self.prefill_workspace)

    def reset(self) -> None:
        self._comp_ptr = 0
        self._win_k = self._win_v = None
        self._dense_valid = 0
        if self._pages is not None:
            self._pages.zero_()

    @property
    def tokens(self) -> int:
        return self._comp_ptr + (0 if self._win_k is None else self._win_k.shape[2])

    def nbytes(self) -> int:
        b = 0 if self._pages is None else self._pages.numel()
        if self._win_k is not None:
            b += (self._win_k.numel() + self._win_v.numel()) * self._win_k.element_size()
        return b


# ---------------------------------------------------------------------------
# TurboQuantKVCache (kv_cache.py:516-624)
# ---------------------------------------------------------------------------

class TurboQuantKVCache(BaseKVCache):
    """TurboQuant V3 (MSE) KV cache with bit-packed GPU storage.

    Extra (build-only) keywords: ``qjl`` — also store a 1-bit QJL sketch of
    each key's quantisation residual; ``attend()`` then adds the unbiased
    residual inner-product estimate to every score.  ``fused_attention`` —
    ``update()`` stores nothing and returns the new K/V, for models whose
    attention is the registered "turboquant" function (hf_attention.py),
    which stores and attends straight off the packed pages.
    """

    def __init__(self, num_layers: int, batch_size: int, num_heads: int, head_dim: int,
                 key_bits: int = 4, value_bits: int = 2, residual_window: int = 128,
                 protected_layers: int = 2, dtype: torch.dtype = torch.bfloat16,
                 device: torch.device = torch.device("cpu"), max_seq_len: int = 2048,
                 qjl: bool = False, fused_attention: bool = False):
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("TurboQuantKVCache stores its pages on a CUDA device; "
                               f"got device={device} (there is no CPU path)")
        self.num_layers = num_layers
        self.batch_size = batch_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.key_bits = key_bits
        self.value_bits = value_bits
        self.residual_window = residual_window
        self.protected_layers = protected_layers
        self.dtype = dtype
        self.device = device
        self.qjl = qjl
        self.fused_attention = fused_attention
        self._seq_len = 0
        self._stores: List[_LayerKVStore] = []
        for i in range(num_layers):
            protected = i < protected_layers or i >= num_layers - protected_layers
            self._stores.append(_LayerKVStore(
                head_dim=head_dim, key_bits=key_bits, value_bits=value_bits,
                max_seq_len=max_seq_len, batch_size=batch_size, num_heads=num_heads,
                rotation_seed=42 + i * 13, device=device, dtype=dtype,
                full_precision=protected, qjl=qjl))
        logger.info("TurboQuantKVCache: %d layers, K%d/V%d bits, residual_window=%d, "
                    "%d protected layers at higher precision%s", num_layers, key_bits,
                    value_bits, residual_window, min(2 * protected_layers, num_layers),
                    ", QJL" if qjl else "")

    # -- HF Cache API ----------------------------------------------------------
    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Optional[Dict[str, Any]] = None
               ) -> Tuple[torch.Tensor, torch.Tensor]:
        if self.fused_attention:
            # the registered "turboquant" attention function stores and
            # attends in one call (hf_attention.py)
            from . import hf_attention
            hf_attention.set_current(self)
            return key_states, value_states
        return self._stores[layer_idx].store_and_get(key_states, value_states,
                                                     self.residual_window)

    # -- fused path --------------------------------------------------------------
    def append(self, key_states: torch.Tensor, value_states: torch.Tensor,
               layer_idx: int) -> None:
        """Store new tokens without materialising dense K/V."""
        self._stores[layer_idx].store(key_states, value_states, self.residual_window)

    def attend(self, query_states: torch.Tensor, layer_idx: int,
               scale: Optional[float] = None, out: Optional[torch.Tensor] = None
               ) -> torch.Tensor:
        """Decode attention of a single-token query (B, Hq, 1, D) over layer
        ``layer_idx``'s packed history and window (GQA: Hq % Hkv == 0)."""
        return self._stores[layer_idx].attend(query_states, scale=scale, out=out)

    def decode(self, query_states: torch.Tensor, key_states: torch.Tensor,
               value_states: torch.Tensor, layer_idx: int, scale: Optional[float] = None,
               out: Optional[torch.Tensor] = None, gather=None,
               kv_start: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One decode step of one layer: store the new token(s) (reference
        update() semantics, including the residual window) and return the
        attention of query_states (B, Hq, 1, D) over the whole cache, without
        materialising dense K/V.  ``kv_start`` (int32 (B,) on the device):
        each batch row's first attended position (left padding)."""
        return self._stores[layer_idx].decode(query_states, key_states, value_states,
                                              self.residual_window, scale=scale, out=out,
                                              gather=gather, kv_start=kv_start)

    def prefill(self, query_states: torch.Tensor, key_states: torch.Tensor,
                value_states: torch.Tensor, layer_idx: int, scale: Optional[float] = None,
                causal: bool = True, out: Optional[torch.Tensor] = None,
                kv_start: Optional[torch.Tensor] = None) -> torch.Tensor:
        """A prefill forward of one layer: store the T new tokens (residual
        window included) and return the causal attention of query_states
        (B, Hq, T, D) over the whole cache (the SDPA that follows update() in
        the reference), without dense K/V.  ``kv_start``: left padding."""
        return self._stores[layer_idx].prefill(query_states, key_states, value_states,
                                               self.residual_window, scale=scale,
                                               causal=causal, out=out, kv_start=kv_start)

    def device_status(self) -> int:
        """OR of the device status words of all layers and of the library's
        own status word (synchronises)."""
        st = 0
        for s in self._stores:
            st |= s.workspace.status()
        return st | ops.device_status(self.device)

    # -- bookkeeping -------------------------------------------------------------
    def advance(self, n: int = 1) -> None:
        self._seq_len += n

    def reset(self) -> None:
        for s in self._stores:
            s.reset()
        self._seq_len = 0

    @property
    def seq_len(self) -> int:
        # HF generate() never calls advance(); report the stored length then
        stored = self._stores[0].tokens if self._stores else 0
        return max(self._seq_len, stored)

    def memory_bytes(self) -> int:
        return sum(s.nbytes() for s in self._stores)

    def compression_stats(self) -> dict:
        """Keys of kv_cache.py:606-624; tq_mb counts the packed pages actually
        allocated plus the window (no dense copy is involved)."""
        tq_bytes = self.memory_bytes()
        seq = self.seq_len
        elem = self.batch_size * self.num_heads * seq * self.head_dim
        if self._stores and self._stores[0]._allocated:
            s = self._stores[0]
            elem = s.batch_size * s.num_heads * seq * self.head_dim
        bf16_bytes = 2 * 2 * self.num_layers * max(elem, 1)
        return {
            "tq_mb": tq_bytes / 1e6,
            "bf16_mb": bf16_bytes / 1e6,
            "compression_ratio": bf16_bytes / tq_bytes if tq_bytes > 0 else 0.0,
            "seq_len": seq,
        }


# ---------------------------------------------------------------------------
# Factory (kv_cache.py:631-659)
# ---------------------------------------------------------------------------

def build_kv_cache(strategy: str, num_layers: int, batch_size: int, num_heads: int,
                   head_dim: int, max_seq_len: int, dtype: torch.dtype,
                   device: torch.device, tq_cfg=None) -> Optional[BaseKVCache]:
    strategy = strategy.lower()
    if strategy == "none":
        return None
    if strategy == "static":
        return StaticKVCache(num_layers=num_layers, batch_size=batch_size, num_heads=num_heads,
                             head_dim=head_dim, max_seq_len=max_seq_len, dtype=dtype,
                             device=device)
    if strategy == "turboquant":
        if tq_cfg is None:
            raise ValueError("TurboQuantConfig required for strategy='turboquant'")
        return TurboQuantKVCache(
            num_layers=num_layers, batch_size=batch_size, num_heads=num_heads,
            head_dim=head_dim, key_bits=tq_cfg.key_bits, value_bits=tq_cfg.value_bits,
            residual_window=tq_cfg.residual_window, protected_layers=tq_cfg.protected_layers,
            dtype=dtype, device=device, max_seq_len=max_seq_len,
            qjl=bool(getattr(tq_cfg, "qjl", False)))
    raise ValueError(f"Unknown kv_cache strategy: '{strategy}'. Choose static/turboquant/none.")
