"""Host logic of the vLLM paged path (CPU): bit widths of protected layers,
the block-table translation, reading vLLM's metadata, and patching vLLM's
Attention layer (no forward runs here)."""
from types import SimpleNamespace

import pytest
import torch

from bhaskera_col_b200.inference.vllm_turboquant import (TurboQuantPagedAttention,
                                                         VLLMBatch, VLLMTurboQuantPatcher,
                                                         layer_bits)


def test_layer_bits_follow_the_reference():
    # vllm_turboquant.py:456-461: first/last `protected_layers` layers +2 bits, capped at 8
    assert layer_bits(0, 32, 4, 2, 2) == (6, 4)
    assert layer_bits(1, 32, 4, 2, 2) == (6, 4)
    assert layer_bits(2, 32, 4, 2, 2) == (4, 2)
    assert layer_bits(30, 32, 4, 2, 2) == (6, 4)
    assert layer_bits(31, 32, 7, 8, 2) == (8, 8)
    assert layer_bits(0, 32, 4, 2, 0) == (4, 2)


@pytest.mark.parametrize("block_size", [64, 128, 256])
def test_stream_table_translation(block_size):
    cpu = torch.device("cpu")
    layer = TurboQuantPagedAttention(4, 32, 8, 2, 128, num_blocks=10, block_size=block_size,
                                     device=cpu)
    m = block_size // 64
    assert layer.pool.shape == (10 * m * 2, layer.page_bytes)
    vbt = torch.tensor([[3, 7, 0], [9, 1, 2]], dtype=torch.int32)
    st = layer.stream_table(vbt)
    assert st.dtype == torch.int32 and st.shape == (4, 3 * m)
    for r in range(2):
        for h in range(2):
            for p in range(3 * m):
                want = (int(vbt[r, p // m]) * m + p % m) * 2 + h
                assert int(st[r * 2 + h, p]) == want
    # every (block, page, head) has its own pool page
    full = layer.stream_table(torch.arange(10, dtype=torch.int32).view(1, 10))
    assert sorted(full.flatten().tolist()) == list(range(layer.pool.shape[0]))


def test_block_size_must_hold_whole_pages():
    with pytest.raises(ValueError, match="multiple of 64"):
        TurboQuantPagedAttention(0, 2, 8, 2, 128, 4, 16, device=torch.device("cpu"))


def test_batch_from_metadata():
    md = SimpleNamespace(query_start_loc=torch.tensor([0, 1, 5], dtype=torch.int32),
                         seq_lens=torch.tensor([10, 4], dtype=torch.int32),
                         block_table=torch.zeros((2, 3), dtype=torch.int32),
                         num_actual_tokens=5, max_query_len=4,
                         query_start_loc_cpu=torch.tensor([0, 1, 5]),
                         seq_lens_cpu=torch.tensor([10, 4]))
    b = VLLMBatch.from_metadata(md)
    assert b.num_actual_tokens == 5 and b.max_query_len == 4
    assert b.host_lists() == ([0, 1, 5], [10, 4])
    md2 = SimpleNamespace(query_start_loc=md.query_start_loc, seq_lens=md.seq_lens,
                          block_table_tensor=md.block_table, num_actual_tokens=5,
                          max_query_len=4)
    b2 = VLLMBatch.from_metadata(md2)
    assert b2.block_table is md.block_table and b2.host_lists() == ([0, 1, 5], [10, 4])


def test_patch_and_unpatch_vllm_attention():
    pytest.importorskip("vllm")
    from bhaskera_col_b200.inference.vllm_turboquant import _vllm_attention_class
    cls = _vllm_attention_class()
    before = cls.forward
    p = VLLMTurboQuantPatcher(key_bits=4, value_bits=2, residual_window=128, protected_layers=2)
    p.patch()
    try:
        assert cls.forward is not before
        p.patch()                               # idempotent
    finally:
        p.unpatch()
    assert cls.forward is before
    assert p.compression_stats() == {"tq_mb": 0.0, "bf16_mb": 0.0, "compression_ratio": 0.0,
                                     "decode_tokens": 0}
