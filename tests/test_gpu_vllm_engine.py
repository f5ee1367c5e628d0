"""A live vLLM engine serving from TurboQuant pages (VLLMTurboQuantPatcher).

A small random-initialised Llama (4 layers, Hq 4 / Hkv 2, head_dim 128) is
served by vLLM in-process with eager execution, 64-token blocks, prefix
caching off and a 128-token step budget, so the 300-token prompt is prefilled
in chunks and decodes share steps with prefills.  With the patch on, every
layer stores its K/V as 8-bit TurboQuant pages and attends from them.

Checks: every layer took the patched path for every scheduled token; the
prompt log-probabilities match vLLM's own attention; and the log-probability
of each token the patched engine generated matches vLLM's own attention
scoring the same continuation (teacher forcing), so the decode path is
checked even where greedy choices could diverge.  Bar: mean |difference|
<= 0.02 nats and max <= 0.25 nats.  8-bit Lloyd-Max codes leave ~0.64 % RMS
error per K/V vector (distortion ~2.7 * 2^-16 of a unit Gaussian), which
four layers turn into a few hundredths of a nat at most; a page or order
mistake moves log-probabilities by whole nats.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engine(tmp_path_factory):
    vllm = pytest.importorskip("vllm")
    from transformers import LlamaConfig, LlamaForCausalLM
    os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
    path = tmp_path_factory.mktemp("tiny_llama")
    cfg = LlamaConfig(vocab_size=512, hidden_size=512, intermediate_size=1024,
                      num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
                      max_position_embeddings=2048, tie_word_embeddings=False)
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).to(torch.bfloat16)
    model.save_pretrained(str(path))
    llm = vllm.LLM(model=str(path), skip_tokenizer_init=True, enforce_eager=True,
                   block_size=64, enable_prefix_caching=False, gpu_memory_utilization=0.2,
                   num_gpu_blocks_override=256, max_model_len=1024,
                   max_num_batched_tokens=128, max_num_seqs=8, dtype="bfloat16", seed=0,
                   attention_backend="FLASH_ATTN")
    yield llm
    del llm


def _prompts():
    rng = np.random.default_rng(0)
    return [{"prompt_token_ids": rng.integers(1, 512, n).tolist()} for n in (100, 37, 300, 65)]


def _lp(entry, tok):
    return entry[tok].logprob


def _within(diffs):
    d = np.asarray(diffs)
    print(f"log-prob differences: mean {d.mean():.4f} max {d.max():.4f} over {d.size}")
    assert d.mean() <= 0.02 and d.max() <= 0.25, (d.mean(), d.max())


def test_vllm_engine_on_turboquant_pages(engine):
    from vllm import SamplingParams
    from bhaskera_col_b200.inference.vllm_turboquant import VLLMTurboQuantPatcher
    prompts = _prompts()
    gen_sp = SamplingParams(max_tokens=24, temperature=0.0, logprobs=0, prompt_logprobs=0,
                            detokenize=False)
    ref_prompt = engine.generate(prompts, gen_sp)            # vLLM's own attention

    patcher = VLLMTurboQuantPatcher(key_bits=8, value_bits=8, protected_layers=0, num_layers=4)
    patcher.patch()
    try:
        outs = engine.generate(prompts, gen_sp)
    finally:
        patcher.unpatch()

    n_prompt = sum(len(p["prompt_token_ids"]) for p in prompts)
    n_gen = [len(o.outputs[0].token_ids) for o in outs]
    assert all(n == 24 for n in n_gen)
    assert sorted(patcher._layers) == [0, 1, 2, 3]
    for layer in patcher._layers.values():
        # every prompt token and every generated token but the last was stored
        assert layer.tokens_stored == n_prompt + sum(n - 1 for n in n_gen)
        assert layer.workspace.status() == 0
    st = patcher.compression_stats()
    assert st["compression_ratio"] > 1.9 and st["decode_tokens"] > 0

    # prefill path: prompt log-probabilities against vLLM's attention
    diffs = []
    for o, r, p in zip(outs, ref_prompt, prompts):
        ids = p["prompt_token_ids"]
        for j in range(1, len(ids)):
            diffs.append(abs(_lp(o.prompt_logprobs[j], ids[j]) - _lp(r.prompt_logprobs[j], ids[j])))
    _within(diffs)

    # decode path: the patched engine's tokens scored by vLLM's attention
    forced = [{"prompt_token_ids": p["prompt_token_ids"] + list(o.outputs[0].token_ids)}
              for p, o in zip(prompts, outs)]
    tf = engine.generate(forced, SamplingParams(max_tokens=1, prompt_logprobs=0,
                                                detokenize=False))
    diffs = []
    for p, o, t in zip(prompts, outs, tf):
        n = len(p["prompt_token_ids"])
        for j, tok in enumerate(o.outputs[0].token_ids):
            diffs.append(abs(_lp(o.outputs[0].logprobs[j], tok) - _lp(t.prompt_logprobs[n + j], tok)))
    _within(diffs)
