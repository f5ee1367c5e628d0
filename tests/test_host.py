"""Host-side logic of the package (CPU only; no kernel launches)."""
import re

import numpy as np
import pytest
import torch
import yaml

import inputs as gi
from bhaskera_col_b200 import _lib
from bhaskera_col_b200.config import Config, TurboQuantConfig, load_config
from bhaskera_col_b200.inference import (LloydMaxCodebook, StaticKVCache, TurboQuantKVCache,
                                         _generate_rotation_matrix, build_kv_cache,
                                         solve_lloyd_max)
from bhaskera_col_b200.inference import ops
from oracle import tq_oracle as O

GOLD = "tests/golden/"


# --------------------------------------------------------------------- tables
@pytest.mark.parametrize("d", [32, 64, 128])
def test_solver_matches_reference_tables(d):
    z = np.load(GOLD + "codebooks.npz")
    for b in (1, 3, 4, 6):
        c, bd = solve_lloyd_max(d, b)
        assert np.array_equal(c.numpy(), z[f"c{d}_{b}"])
        assert np.array_equal(bd.numpy(), z[f"b{d}_{b}"])


def test_rotation_matches_reference_any_thread_count():
    z = np.load(GOLD + "rotations.npz")
    nt = torch.get_num_threads()
    try:
        for threads in (1, max(2, nt)):
            torch.set_num_threads(threads)
            for d, s in gi.ROTATION_CASES:
                assert np.array_equal(_generate_rotation_matrix(d, s).numpy(), z[f"R{d}_{s}"])
            assert torch.get_num_threads() == threads   # restored after QR
    finally:
        torch.set_num_threads(nt)


def test_legacy_codebook_api():
    cb = LloydMaxCodebook.get(128, 4)
    assert cb.centroids.shape == (16,) and cb.boundaries.shape == (15,)
    assert LloydMaxCodebook.get(128, 4) is cb
    assert LloydMaxCodebook.get(128, 2).n_levels == 4
    x = torch.randn(1000) / 128 ** 0.5
    assert cb.dequantize(cb.quantize(x)).shape == x.shape


# --------------------------------------------------------------------- config
def test_config_defaults():
    cfg = Config()
    assert cfg.inference.kv_cache == "static"
    assert cfg.inference.turboquant.key_bits == 4
    assert cfg.inference.turboquant.value_bits == 2
    assert cfg.inference.turboquant.residual_window == 128
    assert cfg.inference.turboquant.protected_layers == 2


def test_config_yaml_override(tmp_path):
    d = {"inference": {"max_new_tokens": 256, "kv_cache": "turboquant",
                       "turboquant": {"key_bits": 3, "residual_window": 64, "qjl": True}}}
    p = tmp_path / "t.yaml"
    p.write_text(yaml.dump(d))
    cfg = load_config(str(p))
    assert cfg.inference.max_new_tokens == 256
    assert cfg.inference.kv_cache == "turboquant"
    assert cfg.inference.turboquant.key_bits == 3
    assert cfg.inference.turboquant.residual_window == 64
    assert cfg.inference.turboquant.qjl is True
    assert cfg.inference.turboquant.value_bits == 2


# -------------------------------------------------------------------- factory
_BASE = dict(num_layers=2, batch_size=1, num_heads=4, head_dim=32, max_seq_len=128,
             dtype=torch.float32, device=torch.device("cpu"))


def test_factory_static_and_none():
    assert isinstance(build_kv_cache(strategy="static", tq_cfg=None, **_BASE), StaticKVCache)
    assert build_kv_cache(strategy="none", tq_cfg=None, **_BASE) is None


def test_factory_errors():
    with pytest.raises(ValueError):
        build_kv_cache(strategy="turboquant", tq_cfg=None, **_BASE)
    with pytest.raises(ValueError):
        build_kv_cache(strategy="invalid", tq_cfg=None, **_BASE)


def test_turboquant_refuses_cpu_device():
    with pytest.raises(RuntimeError, match="CUDA"):
        build_kv_cache(strategy="turboquant", tq_cfg=TurboQuantConfig(), **_BASE)


def test_static_cache_semantics():
    c = StaticKVCache(num_layers=4, batch_size=2, num_heads=8, head_dim=64, max_seq_len=512,
                      dtype=torch.float32)
    k = torch.randn(2, 8, 10, 64)
    fk, fv = c.update(k, torch.randn_like(k), 0)
    assert fk.shape == (2, 8, 10, 64)
    c.advance(5)
    c.reset()
    assert c.seq_len == 0
    c2 = StaticKVCache(num_layers=1, batch_size=2, num_heads=8, head_dim=64, max_seq_len=8,
                       dtype=torch.float32)
    with pytest.raises(ValueError, match="overflow"):
        c2.update(torch.randn(2, 8, 10, 64), torch.randn(2, 8, 10, 64), 0)


# --------------------------------------------------------------------- layout
@pytest.mark.parametrize("D,kb,vb,qjl", [(128, 4, 2, True), (128, 3, 3, False),
                                         (64, 3, 3, False), (32, 6, 4, True)])
def test_page_bytes_agree(D, kb, vb, qjl):
    want = O.PageGeom(D, kb, vb, qjl).page_bytes
    assert ops.page_bytes(D, kb, vb, qjl) == want
    lib = _lib.load()
    g = _lib.Geom(D, kb, vb, 1 if qjl else 0)
    assert lib.tq_page_bytes(g) == want
