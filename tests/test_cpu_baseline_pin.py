"""The reference arm's CPU port (oracle/cpu_baseline.py) is a checked port.

bench.py's ``--impl reference`` and ``cpu_baseline`` legs time
``RefLayer.decode_step`` (the reference's per-layer ``update()`` at
residual_window 0 followed by SDPA, kv_cache.py:445-490 and engine.py:389).
Here that same code path runs the CPU-runnable configuration (B1, Hq16/Hkv4,
D64, 512 tokens, K3/V3, layer 0) and must reproduce the outputs the reference
itself produced for it (tests/golden/config1.npz): codes and fp16 norms
exactly, the attention output within 1e-4.
"""
import numpy as np
import torch

import inputs as gi
from oracle import cpu_baseline as C

GOLD = "tests/golden/config1.npz"


def _unpack_nibbles(packed, shape):
    lo, hi = packed & 0xF, packed >> 4
    return np.stack([lo, hi], -1).reshape(-1)[:int(np.prod(shape))].reshape(shape)


def test_reflayer_decode_step_matches_reference_config1():
    import os
    z = np.load(os.path.join(os.path.dirname(os.path.dirname(__file__)), GOLD))
    k, v, q = gi.config1_inputs()
    kc, kb = C.codebook(64, 3)
    layer = C.RefLayer(1, 4, 64, 512, 3, 3, kc, kb, kc, kb, seed=42, dtype=torch.float32,
                       history=False)
    kt, vt, qt = torch.from_numpy(k), torch.from_numpy(v), torch.from_numpy(q)
    layer._compress(kt[:, :, :511], vt[:, :, :511])
    out = layer.decode_step(kt[:, :, 511:], vt[:, :, 511:], qt)
    shape = tuple(z["idx_shape"])
    assert np.array_equal(layer.k_idx[:512].numpy(), _unpack_nibbles(z["k_idx_packed"], shape))
    assert np.array_equal(layer.v_idx[:512].numpy(), _unpack_nibbles(z["v_idx_packed"], shape))
    assert np.array_equal(layer.k_norm[:512].numpy(), z["k_norm"])
    assert np.array_equal(layer.v_norm[:512].numpy(), z["v_norm"])
    np.testing.assert_allclose(out.numpy(), z["out_tq"], rtol=0, atol=1e-4)
