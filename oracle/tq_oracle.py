"""CPU oracle for the TurboQuant KV-cache path — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The shipped package
(``bhaskera_col_b200``) never imports it and has no CPU fallback.

What it restates (reference = aditya25058/Bhaskera_col, paths relative to the
project root):

* ``solve_lloyd_max``   src/bhaskera/inference/lloyd_max.py:44-100
* ``rotation_matrix``   src/bhaskera/inference/kv_cache.py:55-68
* ``bucketize``         src/bhaskera/inference/kv_cache.py:105-113
* ``compress``          src/bhaskera/inference/kv_cache.py:378-398
* ``decode_range``      src/bhaskera/inference/kv_cache.py:422-439
* ``LayerStore``        src/bhaskera/inference/kv_cache.py:270-490
* ``TurboQuantCache``   src/bhaskera/inference/kv_cache.py:516-624
* ``sdpa``              the HF attention that consumes ``update()``'s output
                        (torch ``scaled_dot_product_attention``, GQA repeat)

Parity of these functions is pinned against golden vectors produced by the
reference itself (``tests/golden/*.npz``, script ``tests/golden/make_golden.py``).

Build-defined parts with no reference counterpart (parity unpinned against the
reference; pinned by properties instead — round trips, unbiasedness):

* the packed page layout (``k_order``, ``v_order``, ``qjl_*``, ``build_pages``)
* the 1-bit QJL residual sketch (TurboQuant arXiv:2504.19874 §3 / QJL
  arXiv:2406.03482), stored in the rotated basis
* ``decode_attention_pages``: attention straight off the packed pages
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

PAGE_TOKENS = 64              # tokens per page of one (batch, kv-head) stream
QJL_SEED_OFFSET = 1_000_003   # QJL matrix seed = rotation seed + this
NORM_CLAMP = 1e-8             # kv_cache.py:384


# =============================================================================
# Codebook  (lloyd_max.py:44-100)
# =============================================================================

def solve_lloyd_max(d: int, bits: int, max_iter: int = 300, tol: float = 1e-12):
    """Lloyd-Max quantiser for N(0, 1/d), same iteration as lloyd_max.py:44-100.

    Centroids start uniform on [-4s, 4s] (lloyd_max.py:62,77); each step sets
    the cell edges to the midpoints with outer edges at +-8s (:80-81) and moves
    each centroid to the conditional mean over its cell by adaptive quadrature
    (scipy.integrate.quad, limit=200, :69-72); stops when no centroid moves by
    more than tol (:90-94).  Boundaries are the final midpoints (:96).
    """
    from scipy import integrate

    n = 2 ** bits
    s2 = 1.0 / d
    s = math.sqrt(s2)
    lo, hi = -4.0 * s, 4.0 * s

    def pdf(x):
        return math.exp(-x * x / (2.0 * s2)) / math.sqrt(2.0 * math.pi * s2)

    def xpdf(x):
        return x * pdf(x)

    cent = [lo + (hi - lo) * (i + 0.5) / n for i in range(n)]
    for _ in range(max_iter):
        mids = [(cent[i] + cent[i + 1]) / 2.0 for i in range(n - 1)]
        edges = [lo * 2] + mids + [hi * 2]
        new = []
        for i in range(n):
            a, b = edges[i], edges[i + 1]
            num = integrate.quad(xpdf, a, b, limit=200)[0]
            den = integrate.quad(pdf, a, b, limit=200)[0]
            new.append(num / den if den > 1e-15 else cent[i])
        shift = max(abs(new[i] - cent[i]) for i in range(n))
        cent = new
        if shift < tol:
            break
    bnd = [(cent[i] + cent[i + 1]) / 2.0 for i in range(n - 1)]
    return np.array(cent, np.float32), np.array(bnd, np.float32)


# =============================================================================
# Rotation  (kv_cache.py:55-68)
# =============================================================================

def rotation_matrix(d: int, seed: int) -> np.ndarray:
    """Haar orthogonal matrix: QR of a seeded CPU Gaussian, columns sign-fixed
    by sign(diag(R)) with 0 -> +1 (kv_cache.py:61-67).  Uses torch's CPU
    generator because the reference's matrix is defined by that stream."""
    import torch
    nthreads = torch.get_num_threads()
    torch.set_num_threads(1)      # LAPACK QR rounding depends on thread count
    try:
        g = torch.Generator(device="cpu")
        g.manual_seed(seed)
        G = torch.randn(d, d, generator=g)
        Q, Rr = torch.linalg.qr(G)
        sg = torch.sign(torch.diag(Rr))
        sg[sg == 0] = 1.0
        return (Q * sg.unsqueeze(0)).numpy().astype(np.float32)
    finally:
        torch.set_num_threads(nthreads)


def qjl_matrix(d: int, rotation_seed: int) -> np.ndarray:
    """Gaussian sketch matrix S (d x d, i.i.d. N(0,1) rounded to bf16) for the
    QJL residual, acting in the rotated basis.  Build-defined (no reference
    counterpart)."""
    import torch
    g = torch.Generator(device="cpu")
    g.manual_seed(rotation_seed + QJL_SEED_OFFSET)
    return torch.randn(d, d, generator=g).bfloat16().float().numpy().astype(np.float32)


# =============================================================================
# Scalar quantiser  (kv_cache.py:105-117)
# =============================================================================

def bucketize(y: np.ndarray, boundaries: np.ndarray) -> np.ndarray:
    """torch.bucketize(right=False): number of boundaries strictly below y."""
    return np.searchsorted(boundaries, y, side="left").astype(np.int16)


def compress(x: np.ndarray, R: np.ndarray, boundaries: np.ndarray):
    """One append of vectors x (..., D) -> (codes, fp16 norm, rotated y).

    kv_cache.py:382-398: fp32 norm, u = x / max(n, 1e-8), y = u @ R^T,
    codes = bucketize(y), stored norm = fp16(n).
    """
    x = x.astype(np.float32)
    n = np.sqrt((x.astype(np.float64) ** 2).sum(-1)).astype(np.float32)
    u = x / np.maximum(n, np.float32(NORM_CLAMP))[..., None]
    y = (u @ R.T).astype(np.float32)
    return bucketize(y, boundaries), n.astype(np.float16), y


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 -> bfloat16 (nearest, ties to even) -> float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def cast_model_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "float32":
        return x.astype(np.float32)
    if dtype == "bfloat16":
        return bf16_round(x.astype(np.float32))
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    raise ValueError(dtype)


def decode_range(idx: np.ndarray, norms: np.ndarray, centroids: np.ndarray,
                 R: np.ndarray, dtype: str = "float32") -> np.ndarray:
    """x_hat = (c[idx] @ R) * fp32(norm), cast to the model dtype
    (kv_cache.py:433-439).  idx (..., D), norms (...)."""
    y = centroids[idx.astype(np.int64)]
    x = (y @ R).astype(np.float32) * norms.astype(np.float32)[..., None]
    return cast_model_dtype(x, dtype)


# =============================================================================
# Per-layer store and cache  (kv_cache.py:233-624)
# =============================================================================

class LayerStore:
    """Mirror of _LayerKVStore: fp-window + compressed history + decoded copy.

    store_and_get (kv_cache.py:445-490): append to the window, evict the
    oldest ``win - residual_window`` tokens into compressed storage, extend
    the decoded history, return concat(decoded, window).
    """

    def __init__(self, head_dim, key_bits, value_bits, rotation_seed, dtype,
                 full_precision=False, codebooks=None, R=None):
        self.D = head_dim
        self.key_bits = min(key_bits + 2, 8) if full_precision else key_bits
        self.value_bits = min(value_bits + 2, 8) if full_precision else value_bits
        self.dtype = dtype
        self.seed = rotation_seed
        cbk = (codebooks or {}).get((head_dim, self.key_bits))
        cbv = (codebooks or {}).get((head_dim, self.value_bits))
        self.kc, self.kb = cbk if cbk else solve_lloyd_max(head_dim, self.key_bits)
        self.vc, self.vb = cbv if cbv else solve_lloyd_max(head_dim, self.value_bits)
        self.R = R if R is not None else rotation_matrix(head_dim, rotation_seed)
        self.k_idx: List[np.ndarray] = []
        self.v_idx: List[np.ndarray] = []
        self.k_norm: List[np.ndarray] = []
        self.v_norm: List[np.ndarray] = []
        self.win_k = None
        self.win_v = None
        self.dec_k = None
        self.dec_v = None

    @property
    def comp_tokens(self) -> int:
        return len(self.k_idx)

    def _compress_chunk(self, k, v):
        B, H, T, D = k.shape
        kf = k.transpose(2, 0, 1, 3).reshape(T, B * H, D)
        vf = v.transpose(2, 0, 1, 3).reshape(T, B * H, D)
        ki, kn, _ = compress(kf, self.R, self.kb)
        vi, vn, _ = compress(vf, self.R, self.vb)
        for t in range(T):
            self.k_idx.append(ki[t]); self.k_norm.append(kn[t])
            self.v_idx.append(vi[t]); self.v_norm.append(vn[t])
        dk = decode_range(ki, kn, self.kc, self.R, self.dtype)
        dv = decode_range(vi, vn, self.vc, self.R, self.dtype)
        dk = dk.reshape(T, B, H, D).transpose(1, 2, 0, 3)
        dv = dv.reshape(T, B, H, D).transpose(1, 2, 0, 3)
        self.dec_k = dk if self.dec_k is None else np.concatenate([self.dec_k, dk], 2)
        self.dec_v = dv if self.dec_v is None else np.concatenate([self.dec_v, dv], 2)

    def store_and_get(self, k, v, residual_window):
        k = cast_model_dtype(k, self.dtype)
        v = cast_model_dtype(v, self.dtype)
        self.win_k = k if self.win_k is None else np.concatenate([self.win_k, k], 2)
        self.win_v = v if self.win_v is None else np.concatenate([self.win_v, v], 2)
        evict = self.win_k.shape[2] - residual_window
        if evict > 0:
            ek, ev = self.win_k[:, :, :evict], self.win_v[:, :, :evict]
            self.win_k, self.win_v = self.win_k[:, :, evict:], self.win_v[:, :, evict:]
            self._compress_chunk(ek, ev)
        if self.dec_k is None:
            return self.win_k, self.win_v
        return (np.concatenate([self.dec_k, self.win_k], 2),
                np.concatenate([self.dec_v, self.win_v], 2))


class TurboQuantCache:
    """Mirror of TurboQuantKVCache (kv_cache.py:516-624): per-layer stores,
    seeds 42 + 13*i (:566), protected layers i < P or i >= L - P get +2 bits
    capped at 8 (:290-291, :556)."""

    def __init__(self, num_layers, head_dim, key_bits=4, value_bits=2,
                 residual_window=128, protected_layers=2, dtype="float32",
                 codebooks=None):
        self.residual_window = residual_window
        self.stores = []
        for i in range(num_layers):
            prot = i < protected_layers or i >= num_layers - protected_layers
            self.stores.append(LayerStore(head_dim, key_bits, value_bits,
                                          42 + 13 * i, dtype, prot, codebooks))

    def update(self, k, v, layer_idx):
        return self.stores[layer_idx].store_and_get(k, v, self.residual_window)


# =============================================================================
# Attention the reference relies on (HF SDPA over update()'s output)
# =============================================================================

def sdpa(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool = False,
         out_dtype: str = "float32", kv_start=None) -> np.ndarray:
    """softmax(q k^T / sqrt(D)) v with GQA repeat (query head j uses kv head
    j // (Hq/Hkv)), computed in float64.  q (B,Hq,Tq,D), k/v (B,Hkv,T,D).
    ``kv_start`` (B,): keys of row b before that position are padding (the
    mask transformers builds from a left-padding mask); a query row with no
    key left gives zeros."""
    B, Hq, Tq, D = q.shape
    Hkv = k.shape[1]
    g = Hq // Hkv
    T = k.shape[2]
    kk = np.repeat(k.astype(np.float64), g, axis=1)
    vv = np.repeat(v.astype(np.float64), g, axis=1)
    s = np.einsum("bhqd,bhkd->bhqk", q.astype(np.float64), kk) / math.sqrt(D)
    keep = np.ones((B, 1, Tq, T), bool)
    if causal:
        qpos = np.arange(T - Tq, T)[:, None]
        keep &= (np.arange(T)[None, :] <= qpos)[None, None]
    if kv_start is not None:
        st = np.asarray(kv_start).reshape(B, 1, 1, 1)
        keep &= np.arange(T)[None, None, None, :] >= st
    s = np.where(keep, s, -np.inf)
    mx = s.max(-1, keepdims=True)
    none = ~np.isfinite(mx)
    p = np.exp(s - np.where(none, 0.0, mx))
    den = p.sum(-1, keepdims=True)
    p = np.where(none, 0.0, p / np.where(none, 1.0, den))
    o = np.einsum("bhqk,bhkd->bhqd", p, vv)
    return cast_model_dtype(o.astype(np.float32), out_dtype)


# =============================================================================
# QJL residual sketch (build-defined)
# =============================================================================

def qjl_sketch(y: np.ndarray, idx: np.ndarray, centroids: np.ndarray,
               norm: np.ndarray, S: np.ndarray):
    """Residual r = y - c[idx] (rotated, unit scale).  Returns sign bits
    (1 where (S r)_i >= 0) and gamma = fp16(norm * ||r||)."""
    r = y.astype(np.float32) - centroids[idx.astype(np.int64)]
    z = r @ S.T
    bits = (z >= 0).astype(np.uint8)
    gamma = (norm.astype(np.float32) *
             np.sqrt((r.astype(np.float64) ** 2).sum(-1)).astype(np.float32))
    return bits, gamma.astype(np.float16)


def qjl_alpha(d: int) -> float:
    """E[sign(<s,r>) <s,q>] = sqrt(2/pi) <q,r>/||r|| for s ~ N(0,I), so
    <q,r> ~= sqrt(pi/2)/m * ||r|| * sum_i sign(<s_i,r>)<s_i,q> with m = d rows."""
    return math.sqrt(math.pi / 2.0) / d


# =============================================================================
# Packed page layout (build-defined)
# =============================================================================

def k_order(D: int) -> np.ndarray:
    """Coordinate order of a packed K (and QJL) row: four quads; quad t holds,
    for each 16-coordinate chunk j, coords 16j+2t, 16j+2t+1, 16j+2t+8, 16j+2t+9."""
    out = []
    for t in range(4):
        for j in range(D // 16):
            out += [16 * j + 2 * t, 16 * j + 2 * t + 1, 16 * j + 2 * t + 8,
                    16 * j + 2 * t + 9]
    return np.array(out, np.int64)


def v_order(D: int) -> np.ndarray:
    """Coordinate order of a packed V row: eight octets; octet g holds coords
    g, g+8, g+16, ..."""
    return np.array([g + 8 * c for g in range(8) for c in range(D // 8)], np.int64)


def pack_bits_lsb(codes: np.ndarray, bits: int) -> np.ndarray:
    """Pack (..., n) codes into an LSB-first bit stream of n*bits bits."""
    n = codes.shape[-1]
    assert (n * bits) % 8 == 0
    c = codes.astype(np.uint64)
    bitpos = np.arange(n)[:, None] * bits + np.arange(bits)[None, :]     # (n, bits)
    bitval = (c[..., :, None] >> np.arange(bits, dtype=np.uint64)) & 1  # (..., n, bits)
    stream = np.zeros(codes.shape[:-1] + (n * bits,), np.uint8)
    stream[..., bitpos.reshape(-1)] = bitval.reshape(codes.shape[:-1] + (-1,))
    return np.packbits(stream, axis=-1, bitorder="little")


def unpack_bits_lsb(packed: np.ndarray, bits: int, n: int) -> np.ndarray:
    stream = np.unpackbits(packed, axis=-1, bitorder="little")[..., : n * bits]
    stream = stream.reshape(packed.shape[:-1] + (n, bits)).astype(np.int64)
    return (stream << np.arange(bits)).sum(-1).astype(np.int16)


def pack_k_row(codes: np.ndarray, bits: int) -> np.ndarray:
    D = codes.shape[-1]
    return pack_bits_lsb(codes[..., k_order(D)], bits)


def pack_v_row(codes: np.ndarray, bits: int) -> np.ndarray:
    D = codes.shape[-1]
    return pack_bits_lsb(codes[..., v_order(D)], bits)


def unpack_k_row(packed, bits, D):
    out = np.empty(packed.shape[:-1] + (D,), np.int16)
    out[..., k_order(D)] = unpack_bits_lsb(packed, bits, D)
    return out


def unpack_v_row(packed, bits, D):
    out = np.empty(packed.shape[:-1] + (D,), np.int16)
    out[..., v_order(D)] = unpack_bits_lsb(packed, bits, D)
    return out


def qjl_bit_positions(D: int) -> np.ndarray:
    """Bit position (within the row) of the sign of coordinate k_order(D)[i].

    The row is four quads of D/4 bits.  A quad is cut into chunks of 2*sp
    bits with sp = min(16, D/8); pair p of the chunk (quad entries 2p, 2p+1)
    puts the even entry at bit p and the odd entry at bit sp + p, so a 32-bit
    word holds 16 even signs in its low half and 16 odd signs in its high half.
    """
    q = D // 4
    sp = min(16, D // 8)
    pos = np.empty(D, np.int64)
    for t in range(4):
        for e in range(q):
            p = e // 2
            chunk, pin = divmod(p, sp)
            bit = chunk * 2 * sp + (sp if e % 2 else 0) + pin
            pos[t * q + e] = t * q + bit
    return pos


def pack_qjl_row(bits01: np.ndarray) -> np.ndarray:
    D = bits01.shape[-1]
    stream = np.zeros(bits01.shape, np.uint8)
    stream[..., qjl_bit_positions(D)] = bits01[..., k_order(D)]
    return np.packbits(stream, axis=-1, bitorder="little")


def unpack_qjl_row(packed: np.ndarray, D: int) -> np.ndarray:
    stream = np.unpackbits(packed, axis=-1, bitorder="little")[..., :D]
    out = np.empty(packed.shape[:-1] + (D,), np.uint8)
    out[..., k_order(D)] = stream[..., qjl_bit_positions(D)]
    return out


@dataclass
class PageGeom:
    D: int
    key_bits: int
    value_bits: int
    qjl: bool

    @property
    def krow(self):
        return self.D * self.key_bits // 8

    @property
    def vrow(self):
        return self.D * self.value_bits // 8

    @property
    def qrow(self):
        return self.D // 8 if self.qjl else 0

    def offsets(self) -> Dict[str, int]:
        T = PAGE_TOKENS
        o, off = {}, 0
        for name, size in (("kcodes", T * self.krow), ("vcodes", T * self.vrow),
                           ("kqjl", T * self.qrow), ("knorm", 2 * T),
                           ("vnorm", 2 * T), ("krnorm", 2 * T if self.qjl else 0)):
            o[name] = off
            off += size
        o["page_bytes"] = off
        return o

    @property
    def page_bytes(self):
        return self.offsets()["page_bytes"]

    def bytes_per_token(self):
        return self.page_bytes // PAGE_TOKENS


def build_pages(geom: PageGeom, k_idx, v_idx, k_norm, v_norm, qbits=None,
                gamma=None) -> np.ndarray:
    """Assemble pages for S streams x T tokens.

    k_idx/v_idx (S, T, D) codes, k_norm/v_norm/gamma (S, T) fp16, qbits
    (S, T, D) 0/1.  Returns uint8 (S, P, page_bytes), unused slots zero.
    """
    S, T, D = k_idx.shape
    P = (T + PAGE_TOKENS - 1) // PAGE_TOKENS
    off = geom.offsets()
    pages = np.zeros((S, P, off["page_bytes"]), np.uint8)
    kr = pack_k_row(k_idx, geom.key_bits)
    vr = pack_v_row(v_idx, geom.value_bits)
    qr = pack_qjl_row(qbits) if geom.qjl else None
    for t in range(T):
        p, slot = divmod(t, PAGE_TOKENS)
        pg = pages[:, p]
        pg[:, off["kcodes"] + slot * geom.krow: off["kcodes"] + (slot + 1) * geom.krow] = kr[:, t]
        pg[:, off["vcodes"] + slot * geom.vrow: off["vcodes"] + (slot + 1) * geom.vrow] = vr[:, t]
        if geom.qjl:
            pg[:, off["kqjl"] + slot * geom.qrow: off["kqjl"] + (slot + 1) * geom.qrow] = qr[:, t]
        for name, arr in (("knorm", k_norm), ("vnorm", v_norm),
                          ("krnorm", gamma if geom.qjl else None)):
            if arr is None:
                continue
            b = arr[:, t].astype(np.float16).view(np.uint8).reshape(S, 2)
            pg[:, off[name] + 2 * slot: off[name] + 2 * slot + 2] = b
    return pages


def parse_pages(geom: PageGeom, pages: np.ndarray, T: int):
    """Inverse of build_pages: returns dict of (S, T, ...) arrays."""
    S, P, _ = pages.shape
    off = geom.offsets()
    D = geom.D
    tok = np.arange(T)
    p, slot = tok // PAGE_TOKENS, tok % PAGE_TOKENS

    def rows(name, width):
        base = off[name] + slot[:, None] * width + np.arange(width)[None, :]
        return pages[:, p[:, None], base]

    def f16(name):
        base = off[name] + 2 * slot[:, None] + np.arange(2)[None, :]
        return np.ascontiguousarray(pages[:, p[:, None], base]).view(np.float16)[..., 0]

    out = dict(k_idx=unpack_k_row(rows("kcodes", geom.krow), geom.key_bits, D),
               v_idx=unpack_v_row(rows("vcodes", geom.vrow), geom.value_bits, D),
               k_norm=f16("knorm"), v_norm=f16("vnorm"))
    if geom.qjl:
        out["qbits"] = unpack_qjl_row(rows("kqjl", geom.qrow), D)
        out["gamma"] = f16("krnorm")
    return out


# =============================================================================
# Attention straight off the packed representation (what the kernels compute)
# =============================================================================

def decode_attention_codes(q, k_idx, v_idx, k_norm, v_norm, kc, vc, R,
                           qbits=None, gamma=None, S=None, T=None,
                           window_k=None, window_v=None, kv_start=None):
    """Single-query attention over a compressed history plus an optional
    full-precision window, in float64.

    q (B, Hq, D); codes (B*Hkv, T, D) stream-major (stream = b*Hkv + h);
    window (B, Hkv, W, D) unrotated.  The compressed part is evaluated in the
    rotated basis: q_rot = q R^T, score = n <q_rot, c[idx]> (+ QJL term
    gamma * alpha * <S q_rot, 2b-1>), output o = (sum p n_v c_v[idx]) R.
    ``kv_start`` (B,): positions of row b before it (compressed position t,
    window token w at T + w) are padding; a row with no key left gives zeros.
    Returns (B, Hq, D) float64.
    """
    B, Hq, D = q.shape
    SS = k_idx.shape[0]
    Hkv = SS // B
    g = Hq // Hkv
    if T is None:
        T = k_idx.shape[1]
    R64 = R.astype(np.float64)
    out = np.zeros((B, Hq, D))
    scale = 1.0 / math.sqrt(D)
    for b in range(B):
        for h in range(Hkv):
            s = b * Hkv + h
            qh = q[b, h * g:(h + 1) * g].astype(np.float64)          # (g, D)
            qr = qh @ R64.T
            kh = kc.astype(np.float64)[k_idx[s, :T].astype(np.int64)]  # (T, D)
            sc = (qr @ kh.T) * k_norm[s, :T].astype(np.float64)[None, :]
            if qbits is not None:
                sq = qr @ S.astype(np.float64).T
                sig = 2.0 * qbits[s, :T].astype(np.float64) - 1.0
                sc += qjl_alpha(D) * gamma[s, :T].astype(np.float64)[None, :] * (sq @ sig.T)
            sc *= scale
            parts = [sc]
            if window_k is not None and window_k.shape[2] > 0:
                parts.append((qh @ window_k[b, h].astype(np.float64).T) * scale)
            allsc = np.concatenate(parts, 1)
            if kv_start is not None:
                allsc = np.where(np.arange(allsc.shape[1])[None, :] >= kv_start[b], allsc,
                                 -np.inf)
            m = allsc.max(1, keepdims=True)
            if not np.isfinite(m).all():          # every key is padding
                continue
            p = np.exp(allsc - m)
            l = p.sum(1, keepdims=True)
            vh = vc.astype(np.float64)[v_idx[s, :T].astype(np.int64)] * \
                v_norm[s, :T].astype(np.float64)[:, None]
            o = (p[:, :T] @ vh) @ R64
            if window_k is not None and window_k.shape[2] > 0:
                o += p[:, T:] @ window_v[b, h].astype(np.float64)
            out[b, h * g:(h + 1) * g] = o / l
    return out


def causal_attention_codes(q, k_idx, v_idx, k_norm, v_norm, kc, vc, R, q_pos0=0):
    """Causal multi-query attention over a compressed cache, float64.

    q (B, Hq, Tq, D) with query i at absolute position q_pos0 + i attending
    to cached tokens 0..q_pos0+i.  Codes as in decode_attention_codes."""
    B, Hq, Tq, D = q.shape
    SS, T, _ = k_idx.shape
    Hkv = SS // B
    g = Hq // Hkv
    R64 = R.astype(np.float64)
    out = np.zeros((B, Hq, Tq, D))
    for b in range(B):
        for h in range(Hkv):
            s = b * Hkv + h
            kd = (kc.astype(np.float64)[k_idx[s].astype(np.int64)] @ R64) * \
                k_norm[s].astype(np.float64)[:, None]
            vd = (vc.astype(np.float64)[v_idx[s].astype(np.int64)] @ R64) * \
                v_norm[s].astype(np.float64)[:, None]
            qq = q[b, h * g:(h + 1) * g].astype(np.float64)            # (g, Tq, D)
            sc = np.einsum("gqd,kd->gqk", qq, kd) / math.sqrt(D)
            qpos = q_pos0 + np.arange(Tq)
            mask = np.arange(T)[None, :] <= qpos[:, None]
            sc = np.where(mask[None], sc, -np.inf)
            sc -= sc.max(-1, keepdims=True)
            p = np.exp(sc)
            p /= p.sum(-1, keepdims=True)
            out[b, h * g:(h + 1) * g] = np.einsum("gqk,kd->gqd", p, vd)
    return out
