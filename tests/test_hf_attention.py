"""transformers wiring: the cache as past_key_values and the "turboquant"
attention function (hf_attention.py).

CPU tests: a tiny random Llama runs with the full-precision cache (the
reference fails there on transformers 5.5 for want of get_mask_sizes), and
the mask builder / registration logic.  GPU tests: the same model with a
TurboQuantKVCache, fused attention against the reference computation (update()
returning dense dequantised K/V, then SDPA), over a prompt in two chunks and
greedy decode steps.
"""
import pytest
import torch

from bhaskera_col_b200.inference import hf_attention
from bhaskera_col_b200.inference.kv_cache import StaticKVCache, TurboQuantKVCache

transformers = pytest.importorskip("transformers")
from transformers import LlamaConfig, LlamaForCausalLM  # noqa: E402


def _model(head_dim, impl, device="cpu", dtype=torch.float32):
    cfg = LlamaConfig(vocab_size=256, hidden_size=4 * head_dim, intermediate_size=512,
                      num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=head_dim, max_position_embeddings=1024)
    cfg._attn_implementation = impl
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).to(device=device, dtype=dtype).eval()


def test_static_cache_runs_hf_forward_and_decode():
    m = _model(64, "sdpa")
    ids = torch.randint(0, 256, (1, 12), generator=torch.Generator().manual_seed(1))
    cache = StaticKVCache(num_layers=3, batch_size=1, num_heads=2, head_dim=64, max_seq_len=64,
                          dtype=torch.float32)
    with torch.no_grad():
        out = m(ids, past_key_values=cache, use_cache=True).logits
        assert torch.allclose(out, m(ids).logits, atol=1e-5)
        cache.advance(12)
        nxt = ids[:, :1]
        step = m(nxt, past_key_values=cache, use_cache=True).logits
        full = m(torch.cat([ids, nxt], 1)).logits[:, -1:]
    assert torch.allclose(step, full, atol=1e-4)


def test_mask_builder():
    from transformers.masking_utils import causal_mask_function
    assert hf_attention.turboquant_mask(2, 1, 10, attention_mask=None) is None
    # a 2-D padding mask becomes each row's first real position, on the device
    pad = torch.ones(3, 10, dtype=torch.bool)
    pad[1, :3] = False
    pad[2, :9] = False
    m = hf_attention.turboquant_mask(3, 4, 10, q_offset=6, kv_offset=0,
                                     mask_function=causal_mask_function, attention_mask=pad,
                                     allow_is_causal_skip=False)
    assert m.dtype == torch.int32 and m.tolist() == [0, 3, 9]
    assert hf_attention._left_pad(m) is m
    assert hf_attention._left_pad(torch.zeros(3, dtype=torch.int32)) is None
    # other mask functions keep SDPA's mask
    from transformers.masking_utils import sliding_window_causal_mask_function
    other = hf_attention.turboquant_mask(3, 4, 10, q_offset=6,
                                         mask_function=sliding_window_causal_mask_function(4),
                                         attention_mask=pad, allow_is_causal_skip=False)
    assert other is not None and other.shape[-2:] == (4, 10)


def test_register_and_requires_a_fused_cache():
    hf_attention.register()
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    assert ALL_ATTENTION_FUNCTIONS["turboquant"] is hf_attention.turboquant_attention
    assert ALL_MASK_ATTENTION_FUNCTIONS["turboquant"] is hf_attention.turboquant_mask
    hf_attention._tls.cache = None
    with pytest.raises(RuntimeError):
        hf_attention.current()


def _run(model, cache, ids, chunks, steps, tokens=None):
    """Prompt in chunks, then greedy steps; `tokens` replays another run's
    choices so both runs see the same inputs."""
    outs, chosen = [], []
    pos = 0
    with torch.no_grad():
        for c in chunks:
            outs.append(model(ids[:, pos:pos + c], past_key_values=cache, use_cache=True).logits)
            pos += c
        tok = outs[-1][:, -1:].argmax(-1)
        for i in range(steps):
            tok = tokens[i] if tokens is not None else tok
            chosen.append(tok)
            lg = model(tok, past_key_values=cache, use_cache=True).logits
            outs.append(lg)
            tok = lg[:, -1:].argmax(-1)
    return outs, chosen


@pytest.mark.gpu
@pytest.mark.parametrize("window", [0, 16])
def test_fused_attention_matches_reference_path(window):
    dev = torch.device("cuda:0")
    hf_attention.register()
    ids = torch.randint(0, 256, (2, 150), generator=torch.Generator().manual_seed(2)).to(dev)

    def cache(fused):
        return TurboQuantKVCache(num_layers=3, batch_size=2, num_heads=2, head_dim=128,
                                 key_bits=4, value_bits=2, residual_window=window,
                                 protected_layers=1, device=dev, max_seq_len=64,
                                 fused_attention=fused)

    ref, toks = _run(_model(128, "sdpa", dev, torch.bfloat16), cache(False), ids, [100, 50], 6)
    got, _ = _run(_model(128, "turboquant", dev, torch.bfloat16), cache(True), ids, [100, 50], 6,
                  tokens=toks)
    for r, g in zip(ref, got):
        r, g = r.float(), g.float()
        cos = torch.nn.functional.cosine_similarity(r.flatten(), g.flatten(), dim=0).item()
        assert cos >= 0.999, cos
        assert (r - g).abs().max().item() <= 5e-2 * r.abs().max().item()


def _run_padded(model, cache, ids, mask, chunks, steps, tokens=None):
    """Left-padded prompts in chunks, then greedy steps, with the padding
    mask and position ids generate() would pass."""
    outs, chosen = [], []
    pos = 0
    B = ids.shape[0]
    with torch.no_grad():
        for c in chunks:
            m = mask[:, :pos + c]
            pid = (m.long().cumsum(-1) - 1).clamp(min=0)[:, pos:pos + c]
            outs.append(model(ids[:, pos:pos + c], attention_mask=m, position_ids=pid,
                              past_key_values=cache, use_cache=True).logits)
            pos += c
        tok = outs[-1][:, -1:].argmax(-1)
        for i in range(steps):
            tok = tokens[i] if tokens is not None else tok
            chosen.append(tok)
            mask = torch.cat([mask, torch.ones((B, 1), dtype=mask.dtype, device=mask.device)], 1)
            pid = (mask.long().sum(-1, keepdim=True) - 1)
            lg = model(tok, attention_mask=mask, position_ids=pid, past_key_values=cache,
                       use_cache=True).logits
            outs.append(lg)
            tok = lg[:, -1:].argmax(-1)
    return outs, chosen, mask


@pytest.mark.gpu
def test_padded_batch_with_residual_window_stays_fused(monkeypatch):
    """Four prompts of 150 / 97 / 40 / 128 tokens, left padded, at the
    reference's default residual_window=128 and a protected layer (K6/V4):
    prompt chunks and decode steps run the fused kernels only (transformers'
    SDPA fallback is made to fail), and the logits at real positions match the
    reference computation (update() + SDPA with the padding mask)."""
    dev = torch.device("cuda:0")
    hf_attention.register()
    lens = [150, 97, 40, 128]
    L = max(lens)
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, 256, (4, L), generator=g).to(dev)
    mask = torch.zeros((4, L), dtype=torch.long, device=dev)
    for b, n in enumerate(lens):
        mask[b, L - n:] = 1
        ids[b, :L - n] = 0

    def cache(fused):
        return TurboQuantKVCache(num_layers=3, batch_size=4, num_heads=2, head_dim=128,
                                 key_bits=4, value_bits=2, residual_window=128,
                                 protected_layers=1, device=dev, max_seq_len=64,
                                 fused_attention=fused)

    ref, toks, _ = _run_padded(_model(128, "sdpa", dev, torch.bfloat16), cache(False), ids, mask,
                               [100, 50], 6)
    import transformers.integrations.sdpa_attention as sa

    def no_sdpa(*a, **k):
        raise AssertionError("the fused run fell back to transformers' SDPA")

    monkeypatch.setattr(sa, "sdpa_attention_forward", no_sdpa)
    got, _, full = _run_padded(_model(128, "turboquant", dev, torch.bfloat16), cache(True), ids,
                               mask, [100, 50], 6, tokens=toks)
    # prompt chunks: compare real positions only; decode steps: every row
    real = [mask[:, :100].bool(), mask[:, 100:150].bool()] + [None] * 6
    for r, gg, sel in zip(ref, got, real):
        r, gg = r.float(), gg.float()
        if sel is not None:
            r, gg = r[sel], gg[sel]
        cos = torch.nn.functional.cosine_similarity(r.flatten(), gg.flatten(), dim=0).item()
        assert cos >= 0.999, cos
        assert (r - gg).abs().max().item() <= 5e-2 * r.abs().max().item()
