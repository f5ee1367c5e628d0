"""Packed-cache file format (serialize.py): round trips, integrity checks,
and (GPU) bit-identical decoding after a save / restore."""
import io

import numpy as np
import pytest
import torch

from bhaskera_col_b200.inference import serialize as S
from oracle import tq_oracle as O


def _layers(rng, window):
    geom = O.PageGeom(64, 4, 2, True)
    out = []
    for i, tokens in enumerate([0, 1, 130]):
        S_, P = 6, max(1, -(-tokens // 64)) + 1          # spare page beyond the used ones
        k_idx = rng.integers(0, 16, (S_, tokens, 64))
        v_idx = rng.integers(0, 4, (S_, tokens, 64))
        kn = rng.standard_normal((S_, tokens)).astype(np.float16)
        vn = rng.standard_normal((S_, tokens)).astype(np.float16)
        qb = rng.integers(0, 2, (S_, tokens, 64)).astype(np.uint8)
        gm = rng.standard_normal((S_, tokens)).astype(np.float16)
        pages = np.zeros((S_, P, geom.page_bytes), np.uint8)
        if tokens:
            built = O.build_pages(geom, k_idx, v_idx, kn, vn, qb, gm)
            pages[:, :built.shape[1]] = built
        L = {"key_bits": 4, "value_bits": 2, "rotation_seed": 42 + 13 * i,
             "page_bytes": geom.page_bytes, "tokens": tokens, "pages": torch.from_numpy(pages)}
        if window:
            L["window_k"] = torch.randn(2, 3, window, 64).bfloat16()
            L["window_v"] = torch.randn(2, 3, window, 64).bfloat16()
        out.append(L)
    return out


META = {"num_layers": 3, "batch_size": 2, "num_heads": 3, "head_dim": 64, "key_bits": 4,
        "value_bits": 2, "residual_window": 0, "protected_layers": 0, "qjl": True,
        "dtype": "bfloat16"}


@pytest.mark.parametrize("window", [0, 5])
def test_round_trip(window):
    rng = np.random.default_rng(0)
    layers = _layers(rng, window)
    buf = io.BytesIO()
    S.write(buf, dict(META, residual_window=window), layers)
    raw = buf.getvalue()
    assert raw[:4] == b"TQKV"
    header, back = S.read(io.BytesIO(raw))
    assert header["version"] == 1 and header["page_tokens"] == 64
    for L, B in zip(layers, back):
        npg = -(-L["tokens"] // 64)
        assert B["tokens"] == L["tokens"] and B["pages"].shape[1] == npg
        assert torch.equal(B["pages"], L["pages"][:, :npg])
        assert B["pages_offset"] % 64 == 0
        if window:
            assert torch.equal(B["window_k"], L["window_k"])
            assert torch.equal(B["window_v"], L["window_v"])
        else:
            assert B["window_k"] is None


def test_integrity_checks():
    rng = np.random.default_rng(1)
    buf = io.BytesIO()
    S.write(buf, META, _layers(rng, 0))
    raw = bytearray(buf.getvalue())
    header, _ = S.read(io.BytesIO(bytes(raw)))
    off = header["layers"][2]["pages_offset"]
    bad = bytearray(raw)
    bad[off + 10] ^= 0xFF
    with pytest.raises(S.FormatError, match="checksum"):
        S.read(io.BytesIO(bytes(bad)))
    with pytest.raises(S.FormatError, match="magic"):
        S.read(io.BytesIO(b"XXXX" + bytes(raw[4:])))
    with pytest.raises(S.FormatError, match="bounds"):
        S.read(io.BytesIO(bytes(raw[:off + 100])))
    v2 = bytearray(raw)
    v2[4] = 2
    with pytest.raises(S.FormatError, match="version"):
        S.read(io.BytesIO(bytes(v2)))


def test_rejects_too_few_pages():
    rng = np.random.default_rng(2)
    layers = _layers(rng, 0)
    layers[2]["pages"] = layers[2]["pages"][:, :2]
    layers[2]["tokens"] = 200                       # needs 4 pages
    with pytest.raises(S.FormatError):
        S.write(io.BytesIO(), META, layers)


@pytest.mark.gpu
@pytest.mark.parametrize("window", [0, 16])
def test_restored_cache_decodes_identically(window):
    from bhaskera_col_b200.inference import TurboQuantKVCache
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    B, H, Hq, D, T = 2, 2, 8, 128, 200
    cache = TurboQuantKVCache(num_layers=3, batch_size=B, num_heads=H, head_dim=D, key_bits=4,
                              value_bits=2, residual_window=window, protected_layers=1,
                              device=dev, max_seq_len=64, qjl=True)
    for layer in range(3):
        cache.update(torch.randn(B, H, T, D, device=dev, generator=g).bfloat16(),
                     torch.randn(B, H, T, D, device=dev, generator=g).bfloat16(), layer)
    buf = io.BytesIO()
    S.save(cache, buf)
    buf.seek(0)
    restored = S.load(buf, dev)
    assert restored.seq_len == cache.seq_len
    for step in range(3):
        for layer in range(3):
            q = torch.randn(B, Hq, 1, D, device=dev, generator=g).bfloat16()
            k = torch.randn(B, H, 1, D, device=dev, generator=g).bfloat16()
            v = torch.randn(B, H, 1, D, device=dev, generator=g).bfloat16()
            a = cache.decode(q, k, v, layer)
            b = restored.decode(q, k, v, layer)
            assert torch.equal(a, b), (step, layer)
    assert cache.device_status() == 0 and restored.device_status() == 0
