"""transformers integration: an attention function that runs the fused kernels.

The reference passes its cache to a HF model as ``past_key_values`` and lets
HF attention run on the dense, dequantised K/V that ``update()`` returns
(engine.py:361-389; kv_cache.py:580-589).  Here the attention itself reads
the packed pages:

    from bhaskera_col_b200.inference import hf_attention
    hf_attention.register()                          # once per process
    model = AutoModelForCausalLM.from_config(cfg, attn_implementation="turboquant")
    cache = TurboQuantKVCache(..., residual_window=0, fused_attention=True)
    model(input_ids, past_key_values=cache, use_cache=True)

With ``fused_attention=True`` the cache's ``update()`` stores nothing and
hands the new K/V straight back; the registered attention function then
stores them and attends in one call: ``cache.decode`` for a single-token step
(append fused into the decode kernels), ``cache.prefill`` for a prompt chunk
(append, then the prefill-attention kernel, the residual window's tokens
entering exactly).  A padded batch (batched ``generate`` pads prompts on the
left) reaches the same kernels: the mask builder turns the 2-D padding mask
into each row's first real position on the device (no host synchronisation)
and the kernels give the padding keys no weight.  Only other masks (sliding
windows, custom mask functions, a 4-D mask from the caller) and, with a
residual window, layers whose bit widths have no tensor-core prefill kernel
store the tokens and run transformers' SDPA on the dense dequantised K/V,
which is exactly the reference's computation.

A padding mask must be left padding (zeros, then ones), the form
``generate`` produces for decoder-only models.

transformers calls the attention function of a layer right after that
layer's ``update()`` on the same thread, so the cache marks itself as the
thread's current fused cache in ``update()``.
"""
from __future__ import annotations

import threading
from typing import Optional

import torch

NAME = "turboquant"
_tls = threading.local()


def set_current(cache) -> None:
    """Called by a fused-mode cache's update(): the cache the next attention
    call on this thread belongs to."""
    _tls.cache = cache


def current():
    cache = getattr(_tls, "cache", None)
    if cache is None:
        raise RuntimeError("turboquant attention called without a TurboQuantKVCache in "
                           "fused_attention mode as past_key_values")
    return cache


def _left_pad(attention_mask) -> Optional[torch.Tensor]:
    """The per-row first real position the mask builder attached, or None."""
    if attention_mask is not None and getattr(attention_mask, "_tq_left_pad", False):
        return attention_mask
    return None


def turboquant_attention(module: torch.nn.Module, query: torch.Tensor, key: torch.Tensor,
                         value: torch.Tensor, attention_mask: Optional[torch.Tensor],
                         scaling: Optional[float] = None, dropout: float = 0.0, **kwargs):
    """HF attention-interface function: (B, Hq, T, D) query and the new
    (B, Hkv, T, D) K/V -> ((B, T, Hq, D) output, None)."""
    if dropout:
        raise ValueError("turboquant attention is inference-only (dropout must be 0)")
    from . import ops
    cache = current()
    layer = module.layer_idx
    T = query.shape[2]
    pad = _left_pad(attention_mask)
    if attention_mask is None or pad is not None:
        if T == 1:
            out = cache.decode(query, key, value, layer, scale=scaling, kv_start=pad)
            return out.transpose(1, 2).contiguous(), None
        store = cache._stores[layer]
        if cache.residual_window <= 0 or ops.prefill_uses_tensor_cores(store.tables):
            out = cache.prefill(query, key, value, layer, scale=scaling, causal=True,
                                kv_start=pad)
            return out.transpose(1, 2).contiguous(), None
    # reference path: store, then SDPA over the dense dequantised K/V
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    store = cache._stores[layer]
    store.store(key, value, cache.residual_window)
    k_all, v_all = store.dense()
    kv = k_all.shape[2]
    if attention_mask is None or pad is not None:
        # causal, aligned to the end: query i sits at position kv - T + i;
        # keys before a row's first real position are padding
        pos = torch.arange(kv, device=query.device)
        qpos = torch.arange(kv - T, kv, device=query.device)
        m = (pos[None, :] <= qpos[:, None])[None, None]
        if pad is not None:
            m = m & (pos[None, None, None, :] >= pad.long()[:, None, None, None])
        attention_mask = m
    return sdpa_attention_forward(module, query, k_all, v_all, attention_mask,
                                  dropout=0.0, scaling=scaling, **kwargs)


def turboquant_mask(batch_size: int, q_length: int, kv_length: int, q_offset: int = 0,
                    kv_offset: int = 0, mask_function=None, attention_mask=None,
                    local_size: Optional[int] = None, **kwargs):
    """Mask builder for the attention function.  A plain causal pattern needs
    no mask (the kernels take causality from token positions, also for a
    prompt chunk after cached tokens); with a 2-D left-padding mask it returns
    each row's first real position, kv_length - (real tokens), an int32 (B,)
    tensor computed on the device and marked for the attention function.
    Anything else gets SDPA's mask."""
    from transformers.masking_utils import causal_mask_function, sdpa_mask
    if mask_function is None:
        mask_function = causal_mask_function
    if local_size is None and mask_function is causal_mask_function and kv_offset == 0:
        if attention_mask is None:
            return None
        if attention_mask.dim() == 2:
            real = attention_mask[:, :kv_length].to(torch.int32).sum(-1, dtype=torch.int32)
            pad = (kv_length - real).to(torch.int32).contiguous()
            pad._tq_left_pad = True
            return pad
    return sdpa_mask(batch_size, q_length, kv_length, q_offset=q_offset, kv_offset=kv_offset,
                     mask_function=mask_function, attention_mask=attention_mask,
                     local_size=local_size, **kwargs)


def register(name: str = NAME) -> None:
    """Register the attention function and its mask builder under ``name``."""
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface
    AttentionInterface.register(name, turboquant_attention)
    AttentionMaskInterface.register(name, turboquant_mask)
