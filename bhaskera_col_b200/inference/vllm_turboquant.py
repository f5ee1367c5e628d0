"""vLLM integration: TurboQuant paged KV, attention computed from the packed pages.

The reference (vllm_turboquant.py:319-469) patches vLLM's Attention.forward,
compresses each decode step's K/V into a side buffer for memory accounting
only (vllm_turboquant.py:398-407) and still runs vLLM's own attention over the
full-precision paged cache.  Here the patched forward stores every token of
the batch into TurboQuant pages addressed through vLLM's own block table and
computes the attention from those pages with the fused kernels:

* a decode batch (one query token per request, any mix of context lengths)
  is ONE tq_decode_step: each request's new K/V is quantised into its page at
  seq_lens[r] - 1 and its query attends its own tokens, with the block table
  resolved inside the kernels (tq_cache.block_table) and the per-request
  lengths read on the device (tq_decode_args.seq_lens), so the call needs no
  host synchronisation;
* prefill and chunked-prefill requests append their new tokens at position
  seq_len - query_len and run the prefill attention over the packed context.

The compressor is the reference's vLLM one (vllm_turboquant.py:170-230): the
MSE codebooks without the QJL sketch, rotation seed 42 + 13 * layer
(vllm_turboquant.py:466), protected layers at min(bits + 2, 8)
(vllm_turboquant.py:459-461).

Page addressing.  A TurboQuant page holds 64 tokens of one KV head.  vLLM
block b (block_size tokens of every KV head) owns pages
(b * m + j) * Hkv + h, j < m = block_size / 64, of the layer's pool, so
logical page p of request r, head h is pool page
(block_table[r, p // m] * m + p % m) * Hkv + h.  block_size must be a
multiple of 64.
"""
from __future__ import annotations

import logging
import re
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch

from . import ops
from .kv_cache import FastLloydMaxCodebook, _generate_rotation_matrix

logger = logging.getLogger(__name__)

PAGE_TOKENS = 64


@dataclass
class VLLMBatch:
    """The fields of vLLM's attention metadata that the paged path reads.

    query_start_loc: int32 (R + 1,) on the device, token offsets of the
    requests in the flattened batch; seq_lens: int32 (R,) on the device,
    context length of each request including this step's tokens;
    block_table: int32 (R, max_blocks) on the device.  Host copies of the first
    two are needed only for batches holding a prefill (max_query_len > 1)."""

    query_start_loc: torch.Tensor
    seq_lens: torch.Tensor
    block_table: torch.Tensor
    num_actual_tokens: int
    max_query_len: int
    query_start_loc_cpu: Optional[List[int]] = None
    seq_lens_cpu: Optional[List[int]] = None

    @classmethod
    def from_metadata(cls, md) -> "VLLMBatch":
        """From a vLLM attention-metadata object (FlashAttentionMetadata and
        the backends shaped like it)."""
        bt = getattr(md, "block_table", None)
        if bt is None:
            bt = getattr(md, "block_table_tensor")
        qcpu = getattr(md, "query_start_loc_cpu", None)
        scpu = getattr(md, "seq_lens_cpu", None)
        return cls(md.query_start_loc, md.seq_lens, bt, int(md.num_actual_tokens),
                   int(md.max_query_len),
                   qcpu.tolist() if qcpu is not None else None,
                   scpu.tolist() if scpu is not None else None)

    def host_lists(self):
        if self.query_start_loc_cpu is None:
            self.query_start_loc_cpu = self.query_start_loc.tolist()
        if self.seq_lens_cpu is None:
            self.seq_lens_cpu = self.seq_lens.tolist()
        return self.query_start_loc_cpu, self.seq_lens_cpu


def layer_bits(layer_idx: int, num_layers: int, key_bits: int, value_bits: int,
               protected_layers: int):
    """(key_bits, value_bits) of a layer: the first and last
    ``protected_layers`` layers keep two more bits, capped at 8
    (vllm_turboquant.py:456-461)."""
    prot = layer_idx < protected_layers or layer_idx >= num_layers - protected_layers
    if prot:
        return min(key_bits + 2, 8), min(value_bits + 2, 8)
    return key_bits, value_bits


class TurboQuantPagedAttention:
    """One attention layer's packed paged KV and its attention over vLLM batches."""

    def __init__(self, layer_idx: int, num_layers: int, num_heads: int, num_kv_heads: int,
                 head_dim: int, num_blocks: int, block_size: int, key_bits: int = 4,
                 value_bits: int = 2, protected_layers: int = 2,
                 scale: Optional[float] = None, device: torch.device = torch.device("cuda")):
        if block_size % PAGE_TOKENS:
            raise ValueError(f"block_size {block_size} is not a multiple of {PAGE_TOKENS}")
        if num_heads % num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        self.layer_idx = layer_idx
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.num_blocks, self.block_size = num_blocks, block_size
        self.pages_per_block = block_size // PAGE_TOKENS
        self.scale = scale if scale is not None else head_dim ** -0.5
        self.device = torch.device(device)
        self.key_bits, self.value_bits = layer_bits(layer_idx, num_layers, key_bits,
                                                    value_bits, protected_layers)
        kc = FastLloydMaxCodebook.get(head_dim, self.key_bits, self.device)
        vc = FastLloydMaxCodebook.get(head_dim, self.value_bits, self.device)
        R = _generate_rotation_matrix(head_dim, seed=42 + 13 * layer_idx, device=self.device)
        self.tables = ops.LayerTables(head_dim, self.key_bits, self.value_bits, False,
                                      kc.centroids, kc.boundaries, vc.centroids, vc.boundaries,
                                      R.contiguous().float())
        self.page_bytes = ops.page_bytes(head_dim, self.key_bits, self.value_bits, False)
        self.pool = torch.zeros((num_blocks * self.pages_per_block * num_kv_heads,
                                 self.page_bytes), dtype=torch.uint8, device=self.device)
        self.workspace = ops.DecodeWorkspace()
        self.tokens_stored = 0
        self.decode_tokens = 0

    # -- addressing -----------------------------------------------------------
    def stream_table(self, block_table: torch.Tensor) -> torch.Tensor:
        """vLLM's (R, max_blocks) block table -> the (R * Hkv, pages) table of
        pool pages, stream r * Hkv + h."""
        R, MB = block_table.shape
        m, H = self.pages_per_block, self.num_kv_heads
        dev = block_table.device
        pages = block_table.to(torch.int64).unsqueeze(-1) * m + torch.arange(m, device=dev)
        st = pages.reshape(R, 1, MB * m) * H + torch.arange(H, device=dev).view(1, H, 1)
        return st.reshape(R * H, MB * m).to(torch.int32)

    def paged(self, stream_table: torch.Tensor) -> ops.PagedPages:
        return ops.PagedPages(self.pool, stream_table)

    # -- attention ------------------------------------------------------------
    def forward(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                batch: VLLMBatch, out: Optional[torch.Tensor] = None,
                stream_table: Optional[torch.Tensor] = None) -> torch.Tensor:
        """query (N, Hq, D), key / value (N, Hkv, D) in vLLM's flattened token
        order; stores the tokens, returns the (N, Hq, D) attention output."""
        if out is None:
            out = torch.empty_like(query)
        st = stream_table if stream_table is not None else self.stream_table(batch.block_table)
        H = self.num_kv_heads
        R = batch.seq_lens.shape[0]
        cap = st.shape[1] * PAGE_TOKENS
        self.tokens_stored += batch.num_actual_tokens
        if batch.max_query_len <= 1:
            # one token per request: a single fused store + ragged decode
            self._decode(query[:R], key[:R], value[:R], out[:R], batch.seq_lens, st, cap)
            self.decode_tokens += batch.num_actual_tokens
            return out
        qsl, sl = batch.host_lists()
        dec = [r for r in range(R) if qsl[r + 1] - qsl[r] == 1]
        if dec:
            tok = torch.tensor([qsl[r] for r in dec], dtype=torch.int64, device=query.device)
            rows = torch.tensor(dec, dtype=torch.int64, device=query.device)
            sub = st.view(R, H, -1).index_select(0, rows).reshape(len(dec) * H, -1)
            o = torch.empty((len(dec),) + tuple(query.shape[1:]), dtype=out.dtype,
                            device=out.device)
            self._decode(query.index_select(0, tok), key.index_select(0, tok),
                         value.index_select(0, tok), o, batch.seq_lens.index_select(0, rows),
                         sub, cap)
            out.index_copy_(0, tok, o)
            self.decode_tokens += len(dec)
        for r in range(R):
            qs, qe = qsl[r], qsl[r + 1]
            n = qe - qs
            if n <= 1:
                continue
            pages = self.paged(st[r * H:(r + 1) * H])
            ctx = sl[r] - n
            # (n, H, D) token-major rows seen as (1, H, n, D)
            ops.append(self.tables, pages, key[qs:qe].permute(1, 0, 2).unsqueeze(0),
                       value[qs:qe].permute(1, 0, 2).unsqueeze(0), ctx)
            ops.prefill_attention(self.tables, pages, query[qs:qe].permute(1, 0, 2).unsqueeze(0),
                                  sl[r], scale=self.scale, causal=True,
                                  out=out[qs:qe].permute(1, 0, 2).unsqueeze(0))
        return out

    def _decode(self, q, k, v, out, seq_lens, st, cap):
        ops.decode_step(self.tables, self.paged(st), k.unsqueeze(2), v.unsqueeze(2), cap - 1,
                        q.unsqueeze(2), scale=self.scale, out=out.unsqueeze(2),
                        workspace=self.workspace, seq_lens=seq_lens)

    def packed_bytes_per_token(self) -> float:
        """Bytes of packed storage per token (all KV heads, K and V)."""
        return self.page_bytes * self.num_kv_heads / PAGE_TOKENS


# ---------------------------------------------------------------------------
# vLLM attention monkey-patcher (the reference's API, vllm_turboquant.py:319-469)
# ---------------------------------------------------------------------------
def _vllm_attention_class():
    """vLLM's Attention layer class, wherever this vLLM version keeps it."""
    for mod, name in (("vllm.model_executor.layers.attention.attention", "Attention"),
                      ("vllm.attention.layer", "Attention"), ("vllm.attention", "Attention")):
        try:
            m = __import__(mod, fromlist=[name])
            return getattr(m, name)
        except (ImportError, AttributeError):
            continue
    raise RuntimeError("vLLM is not installed (no Attention layer found)")


def _layer_index(attn_self, fallback: int) -> int:
    idx = getattr(attn_self, "layer_idx", None)
    if idx is not None:
        return int(idx)
    m = re.findall(r"\.(\d+)\.", "." + str(getattr(attn_self, "layer_name", "")) + ".")
    return int(m[-1]) if m else fallback


def _forward_metadata(attn_self):
    """This layer's attention metadata of the running forward pass (None in
    vLLM's profiling and dummy runs)."""
    from vllm.forward_context import get_forward_context
    md = get_forward_context().attn_metadata
    if isinstance(md, dict):
        md = md.get(getattr(attn_self, "layer_name", None))
    elif isinstance(md, list):       # one dict per micro-batch
        md = md[0].get(getattr(attn_self, "layer_name", None)) if md else None
    return md


class VLLMTurboQuantPatcher:
    """Patches vLLM's Attention.forward so every layer stores its K/V as
    TurboQuant pages and attends from them (the reference's patch kept vLLM's
    own attention; vllm_turboquant.py:398-407).

    Usage (vLLM with enforce_eager=True and the model runner in-process, e.g.
    VLLM_ENABLE_V1_MULTIPROCESSING=0; block_size a multiple of 64)::

        patcher = VLLMTurboQuantPatcher(key_bits=4, value_bits=2,
                                        residual_window=128, protected_layers=2)
        patcher.patch()
        ... run vLLM ...
        patcher.unpatch()

    ``residual_window`` is kept for the reference's signature; as in the
    reference's vLLM path, every token is compressed.
    """

    def __init__(self, key_bits: int = 4, value_bits: int = 2, residual_window: int = 128,
                 protected_layers: int = 2, num_layers: Optional[int] = None,
                 num_blocks: Optional[int] = None, block_size: Optional[int] = None):
        self.key_bits = key_bits
        self.value_bits = value_bits
        self.residual_window = residual_window
        self.protected_layers = protected_layers
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self._original_forward = None
        self._cls = None
        self._patched = False
        self._layers: Dict[int, TurboQuantPagedAttention] = {}
        self._last_md = None
        self._last_table = None

    # -- patch / unpatch --------------------------------------------------------
    def patch(self) -> None:
        if self._patched:
            return
        cls = _vllm_attention_class()
        self._cls = cls
        self._original_forward = cls.forward
        patcher = self

        def _turboquant_forward(attn_self, query, key, value, *args, **kwargs):
            md = _forward_metadata(attn_self) if key is not None else None
            if md is None or not hasattr(md, "seq_lens"):
                return patcher._original_forward(attn_self, query, key, value, *args, **kwargs)
            return patcher.attend(attn_self, query, key, value, md)

        cls.forward = _turboquant_forward
        self._patched = True
        logger.info("[VLLMTurboQuantPatcher] patched vLLM Attention.forward (K%d/V%d)",
                    self.key_bits, self.value_bits)

    def unpatch(self) -> None:
        if not self._patched:
            return
        self._cls.forward = self._original_forward
        self._patched = False

    # -- the patched call ---------------------------------------------------------
    def attend(self, attn_self, query, key, value, md) -> torch.Tensor:
        H, Hkv = attn_self.num_heads, attn_self.num_kv_heads
        D = attn_self.head_size
        layer = self.layer_for(attn_self, query.device)
        if md is not self._last_md:          # one translation per step, shared by the layers
            self._last_md = md
            self._batch = VLLMBatch.from_metadata(md)
            self._last_table = layer.stream_table(self._batch.block_table)
        n = query.shape[0]
        out = torch.empty((n, H, D), dtype=query.dtype, device=query.device)
        if self._batch.num_actual_tokens < n:
            out[self._batch.num_actual_tokens:].zero_()    # padding tokens of a captured batch
        layer.forward(query.view(n, H, D), key.view(-1, Hkv, D), value.view(-1, Hkv, D),
                      self._batch, out=out, stream_table=self._last_table)
        return out.view(n, H * D)

    def layer_for(self, attn_self, device) -> TurboQuantPagedAttention:
        idx = _layer_index(attn_self, len(self._layers))
        layer = self._layers.get(idx)
        if layer is None:
            num_blocks, block_size = self._cache_geometry(attn_self)
            num_layers = self.num_layers or getattr(attn_self, "num_hidden_layers", None) or 32
            layer = TurboQuantPagedAttention(
                idx, num_layers, attn_self.num_heads, attn_self.num_kv_heads,
                attn_self.head_size, num_blocks, block_size, self.key_bits, self.value_bits,
                self.protected_layers, scale=getattr(attn_self, "scale", None)
                or getattr(getattr(attn_self, "impl", None), "scale", None), device=device)
            self._layers[idx] = layer
        return layer

    def _cache_geometry(self, attn_self):
        if self.num_blocks and self.block_size:
            return self.num_blocks, self.block_size
        # vLLM's own cache of the layer: (2, blocks, block_size, Hkv, D) for
        # FlashAttention, (blocks, 2, block_size, Hkv, D) for FlashInfer
        kv = getattr(attn_self, "kv_cache", None)
        if isinstance(kv, (list, tuple)) and kv:
            kv = kv[0]
        if isinstance(kv, torch.Tensor) and kv.dim() == 5 and \
                tuple(kv.shape[3:]) == (attn_self.num_kv_heads, attn_self.head_size):
            nb = kv.shape[1] if kv.shape[0] == 2 else kv.shape[0]
            return int(self.num_blocks or nb), int(self.block_size or kv.shape[2])
        from vllm.config import get_current_vllm_config
        cc = get_current_vllm_config().cache_config
        nb = self.num_blocks or cc.num_gpu_blocks
        bs = self.block_size or cc.block_size
        if not nb:
            raise RuntimeError("vLLM's block count is not known yet (pass num_blocks=)")
        return int(nb), int(bs)

    # -- accounting (the reference's API) ---------------------------------------
    def reset_buffers(self) -> None:
        for layer in self._layers.values():
            layer.pool.zero_()
            layer.tokens_stored = 0
            layer.decode_tokens = 0

    def compression_stats(self) -> dict:
        """Packed bytes of the stored tokens against bf16 K/V for them."""
        tq = sum(l.tokens_stored * l.packed_bytes_per_token() for l in self._layers.values())
        bf16 = sum(l.tokens_stored * l.num_kv_heads * l.head_dim * 2 * 2
                   for l in self._layers.values())
        n = max(len(self._layers), 1)
        return {"tq_mb": tq / 1e6, "bf16_mb": bf16 / 1e6,
                "compression_ratio": bf16 / tq if tq > 0 else 0.0,
                "decode_tokens": sum(l.decode_tokens for l in self._layers.values()) // n}
