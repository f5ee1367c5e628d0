"""Generate the golden fixtures that pin the oracle to the reference.

Run in a container where the reference tree is readable:

    python tests/golden/make_golden.py <reference>/src
    (or set BHASKERA_REFERENCE_SRC to the reference checkout's src directory)

The reference is imported from source with bytecode caching redirected to a
scratch directory, so none of the compiled ``__pycache__`` files shipped with
it are ever loaded.  Every array written here is an *output of the reference*
(`bhaskera.inference.kv_cache` / `bhaskera.inference.lloyd_max`) on seeded
inputs that are regenerated bit-for-bit by ``tests/golden/inputs.py`` (numpy
PCG64 streams, platform independent), so the inputs themselves need not be
stored.

Files written (all ``.npz``):

* ``codebooks.npz``   solve_lloyd_max(d, b)         lloyd_max.py:44-100
* ``rotations.npz``   _generate_rotation_matrix      kv_cache.py:55-68
* ``quantize_edges.npz`` FastLloydMaxCodebook.quantize on boundary values
                                                    kv_cache.py:105-113
* ``config1.npz``     TurboQuantKVCache.update + SDPA on the CPU-runnable
                      configuration (B1 Hq16 Hkv4 D64 T512, K3/V3, fp32)
                                                    kv_cache.py:355-490
* ``incremental.npz`` residual-window / protected-layer update sequence
                                                    kv_cache.py:445-490, 556
* ``bf16_case.npz``   bf16 model dtype, D128, GQA 4, K4/V2
"""
from __future__ import annotations

import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import inputs as gi  # noqa: E402  (seeded input generators shared with tests)


def _import_reference(src: str):
    sys.dont_write_bytecode = True
    sys.pycache_prefix = tempfile.mkdtemp(prefix="pyc_")
    sys.path.insert(0, src)
    import torch  # noqa: F401
    from bhaskera.inference import kv_cache, lloyd_max
    return kv_cache, lloyd_max


def _pack_nibbles(idx: np.ndarray) -> np.ndarray:
    flat = idx.astype(np.uint8).reshape(-1)
    if flat.size % 2:
        flat = np.concatenate([flat, np.zeros(1, np.uint8)])
    return (flat[0::2] | (flat[1::2] << 4)).astype(np.uint8)


def main(src: str) -> None:
    import torch
    import torch.nn.functional as F

    kv_cache, lloyd_max = _import_reference(src)
    torch.set_num_threads(1)

    # ---------------------------------------------------------------- codebooks
    cb = {}
    for d in gi.CODEBOOK_DIMS:
        for b in range(1, 9):
            c, bd = lloyd_max.solve_lloyd_max(d, b)
            cb[f"c{d}_{b}"] = c.numpy().astype(np.float32)
            cb[f"b{d}_{b}"] = bd.numpy().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "codebooks.npz"), **cb)

    # ---------------------------------------------------------------- rotations
    rot = {}
    for d, seed in gi.ROTATION_CASES:
        R = kv_cache._generate_rotation_matrix(d, seed=seed)
        rot[f"R{d}_{seed}"] = R.numpy().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "rotations.npz"), **rot)

    # ----------------------------------------------------------- quantize edges
    qe = {}
    dev = torch.device("cpu")
    for d, b in gi.EDGE_CASES:
        fcb = kv_cache.FastLloydMaxCodebook.get(d, b, dev)
        y = gi.edge_values(cb[f"b{d}_{b}"], d, seed=d * 10 + b)
        idx = fcb.quantize(torch.from_numpy(y)).numpy().astype(np.int16)
        qe[f"y{d}_{b}"] = y
        qe[f"idx{d}_{b}"] = idx
    np.savez_compressed(os.path.join(HERE, "quantize_edges.npz"), **qe)

    # ------------------------------------------------------------------ config 1
    k, v, q = gi.config1_inputs()
    B, H, T, D = k.shape
    cache = kv_cache.TurboQuantKVCache(
        num_layers=1, batch_size=B, num_heads=H, head_dim=D,
        key_bits=3, value_bits=3, residual_window=0, protected_layers=0,
        dtype=torch.float32, device=dev, max_seq_len=T)
    kt, vt = torch.from_numpy(k), torch.from_numpy(v)
    fk, fv = cache.update(kt, vt, 0)
    st = cache._stores[0]
    # the rotated fp32 tensors the reference quantized, computed exactly as
    # _compress_chunk does (per token, (BH, D) rows)
    yk = np.empty((T, B * H, D), np.float32)
    yv = np.empty((T, B * H, D), np.float32)
    kf = kt.permute(2, 0, 1, 3).reshape(T, B * H, D)
    vf = vt.permute(2, 0, 1, 3).reshape(T, B * H, D)
    for t in range(T):
        for src_, dst in ((kf, yk), (vf, yv)):
            x = src_[t].float()
            n = x.norm(dim=-1)
            u = x / n.unsqueeze(-1).clamp(min=1e-8)
            dst[t] = st._rotate(u).numpy()
    k_idx = st._k_idx[:T].numpy()
    v_idx = st._v_idx[:T].numpy()
    assert (torch.bucketize(torch.from_numpy(yk).reshape(-1), st.k_cb.boundaries)
            .reshape(yk.shape).numpy() == k_idx).all()
    qt = torch.from_numpy(q)
    out_tq = F.scaled_dot_product_attention(qt, fk, fv, enable_gqa=True)
    out_fp = F.scaled_dot_product_attention(qt, kt, vt, enable_gqa=True)
    NSUB = 64
    np.savez_compressed(
        os.path.join(HERE, "config1.npz"),
        k_idx_packed=_pack_nibbles(k_idx), v_idx_packed=_pack_nibbles(v_idx),
        idx_shape=np.array(k_idx.shape, np.int64),
        k_norm=st._k_norms[:T].numpy(), v_norm=st._v_norms[:T].numpy(),
        yk_sub=yk[:NSUB], yv_sub=yv[:NSUB],
        fk_sub=fk[:, :, :NSUB].numpy(), fv_sub=fv[:, :, :NSUB].numpy(),
        fk_rowsum=fk.sum(-1).numpy(), fv_rowsum=fv.sum(-1).numpy(),
        fk_rowsq=(fk * fk).sum(-1).numpy(), fv_rowsq=(fv * fv).sum(-1).numpy(),
        out_tq=out_tq.numpy(), out_fp32=out_fp.numpy(),
        input_checksum=np.array([k.sum(dtype=np.float64), v.sum(dtype=np.float64),
                                 q.sum(dtype=np.float64)]),
    )

    # ------------------------------------------------------------- incremental
    inc = {}
    spec = gi.INCREMENTAL
    cache = kv_cache.TurboQuantKVCache(
        num_layers=spec["num_layers"], batch_size=spec["B"], num_heads=spec["H"],
        head_dim=spec["D"], key_bits=spec["key_bits"], value_bits=spec["value_bits"],
        residual_window=spec["residual_window"],
        protected_layers=spec["protected_layers"], dtype=torch.float32,
        device=dev, max_seq_len=spec["max_seq_len"])
    for layer in spec["layers"]:
        chunks = gi.incremental_inputs(layer)
        last = len(chunks) - 1
        for step, (kc, vc) in enumerate(chunks):
            ok, ov = cache.update(torch.from_numpy(kc), torch.from_numpy(vc), layer)
            if step in (0, last):   # full outputs; row sums for the steps between
                inc[f"L{layer}_s{step}_k"] = ok.numpy()
                inc[f"L{layer}_s{step}_v"] = ov.numpy()
            else:
                inc[f"L{layer}_s{step}_krow"] = ok.sum(-1).numpy()
                inc[f"L{layer}_s{step}_vrow"] = ov.sum(-1).numpy()
        s = cache._stores[layer]
        inc[f"L{layer}_bits"] = np.array([s.key_bits, s.value_bits], np.int64)
        inc[f"L{layer}_comp"] = np.array([s._comp_ptr], np.int64)
        inc[f"L{layer}_k_idx"] = s._k_idx[: s._comp_ptr].numpy()
        inc[f"L{layer}_v_idx"] = s._v_idx[: s._comp_ptr].numpy()
        inc[f"L{layer}_k_norm"] = s._k_norms[: s._comp_ptr].numpy()
        inc[f"L{layer}_v_norm"] = s._v_norms[: s._comp_ptr].numpy()
    st = cache.compression_stats()
    inc["stats"] = np.array([st["tq_mb"], st["bf16_mb"], st["compression_ratio"],
                             st["seq_len"]], np.float64)
    inc["memory_bytes"] = np.array([cache.memory_bytes()], np.int64)
    np.savez_compressed(os.path.join(HERE, "incremental.npz"), **inc)

    # ---------------------------------------------------------------- bf16 case
    spec = gi.BF16_CASE
    kb, vb, qb = gi.bf16_case_inputs()   # float32 arrays holding bf16 values
    kt = torch.from_numpy(kb).to(torch.bfloat16)
    vt = torch.from_numpy(vb).to(torch.bfloat16)
    qt = torch.from_numpy(qb).to(torch.bfloat16)
    assert (kt.float().numpy() == kb).all()
    cache = kv_cache.TurboQuantKVCache(
        num_layers=1, batch_size=spec["B"], num_heads=spec["Hkv"],
        head_dim=spec["D"], key_bits=spec["key_bits"], value_bits=spec["value_bits"],
        residual_window=0, protected_layers=0, dtype=torch.bfloat16, device=dev,
        max_seq_len=spec["T"])
    fk, fv = cache.update(kt, vt, 0)
    out = F.scaled_dot_product_attention(qt, fk, fv, enable_gqa=True)
    out_fp = F.scaled_dot_product_attention(qt.float(), kt.float(), vt.float(),
                                            enable_gqa=True)
    s = cache._stores[0]
    np.savez_compressed(
        os.path.join(HERE, "bf16_case.npz"),
        k_idx=s._k_idx[: spec["T"]].numpy().astype(np.uint8),
        v_idx=s._v_idx[: spec["T"]].numpy().astype(np.uint8),
        k_norm=s._k_norms[: spec["T"]].numpy(), v_norm=s._v_norms[: spec["T"]].numpy(),
        fk_bits=fk.contiguous().view(torch.int16).numpy().view(np.uint16),
        fv_bits=fv.contiguous().view(torch.int16).numpy().view(np.uint16),
        out_tq=out.float().numpy(), out_fp32=out_fp.numpy(),
    )
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("BHASKERA_REFERENCE_SRC")
    if not src:
        sys.exit("usage: make_golden.py <reference src directory> "
                 "(or set BHASKERA_REFERENCE_SRC)")
    main(src)
