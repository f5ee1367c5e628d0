"""Save and restore a TurboQuant cache: the packed-page format on disk.

The reference has no serialised form (its cache lives in per-token int16
tensors and a dense dequantised copy, kv_cache.py:270-339).  This file format
stores exactly the device bytes the kernels read, so a restored cache decodes
bit-identically (prefix caching: save after a prompt, restore later).

File layout (all integers little-endian):

    offset 0   b"TQKV"                      magic
           4   u32 version (= 1)
           8   u32 n = length of the header
          12   n bytes of UTF-8 JSON header
      12 + n   sections, each 64-byte aligned, at the offsets the header names

Header JSON:

    {"version": 1, "page_tokens": 64,
     "cache": {num_layers, batch_size, num_heads, head_dim, key_bits, value_bits,
               residual_window, protected_layers, qjl, dtype},
     "layers": [{"key_bits", "value_bits", "rotation_seed", "streams",
                 "page_bytes", "tokens", "pages",
                 "pages_offset", "pages_nbytes", "pages_crc32",
                 "window_tokens", "window_offset", "window_nbytes", "window_crc32"}, ...]}

A layer's page section is its first `pages` = ceil(tokens / 64) pages of
every stream, [streams][pages][page_bytes] uint8, in the page layout of
include/tq_b200.h (K codes, V codes, QJL signs, fp16 norms, fp16 residual
norms).  Unused slots of the last page are zero.  The window section (only
when residual_window > 0 and the window holds tokens) is the full-precision
window K then V, each (B, Hkv, window_tokens, D) in the cache dtype.  The
tables (codebooks, rotation, QJL matrix) are not stored: they are functions
of (head_dim, bits, rotation_seed) and are rebuilt on restore.
"""
from __future__ import annotations

import io
import json
import struct
import zlib
from typing import BinaryIO, Dict, List, Optional, Tuple, Union

import numpy as np
import torch

MAGIC = b"TQKV"
VERSION = 1
PAGE_TOKENS = 64
_ALIGN = 64

_DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


class FormatError(ValueError):
    """The file is not a valid TurboQuant cache file (or does not match)."""


def _dtype_name(dt: torch.dtype) -> str:
    for k, v in _DTYPES.items():
        if v == dt:
            return k
    raise FormatError(f"unsupported cache dtype {dt}")


def _raw(t: torch.Tensor) -> bytes:
    """Bytes of a CPU tensor (bf16 via its 16-bit pattern)."""
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return t.numpy().tobytes()


def _from_raw(b: bytes, dtype: torch.dtype, shape) -> torch.Tensor:
    if dtype == torch.bfloat16:
        return torch.from_numpy(np.frombuffer(b, np.int16).copy()).view(torch.bfloat16).reshape(shape)
    np_dt = {torch.uint8: np.uint8, torch.float16: np.float16, torch.float32: np.float32}[dtype]
    return torch.from_numpy(np.frombuffer(b, np_dt).copy()).reshape(shape)


def write(f: BinaryIO, cache_meta: dict, layers: List[dict]) -> None:
    """Write a file from plain data.  Each layer dict holds its metadata
    (key_bits, value_bits, rotation_seed, page_bytes, tokens) plus `pages`
    (uint8 tensor [streams][>= ceil(tokens/64)][page_bytes]) and optional
    `window_k` / `window_v` (B, Hkv, W, D) tensors."""
    entries, blobs = [], []
    for L in layers:
        tokens = int(L["tokens"])
        npg = -(-tokens // PAGE_TOKENS)
        pages = L["pages"]
        if pages.dtype != torch.uint8 or pages.dim() != 3 or pages.shape[2] != L["page_bytes"]:
            raise FormatError("pages must be uint8 [streams][pages][page_bytes]")
        if pages.shape[1] < npg:
            raise FormatError(f"{tokens} tokens need {npg} pages, only {pages.shape[1]} given")
        pb = _raw(pages[:, :npg])
        wk, wv = L.get("window_k"), L.get("window_v")
        wb = b"" if wk is None else _raw(wk) + _raw(wv)
        e = {k: L[k] for k in ("key_bits", "value_bits", "rotation_seed", "page_bytes")}
        e.update(streams=int(pages.shape[0]), tokens=tokens, pages=npg,
                 pages_nbytes=len(pb), pages_crc32=zlib.crc32(pb),
                 window_tokens=0 if wk is None else int(wk.shape[2]),
                 window_nbytes=len(wb), window_crc32=zlib.crc32(wb))
        entries.append(e)
        blobs.append((pb, wb))
    # offsets depend on the header length, which depends on the offsets' digits:
    # lay out with a fixed-width placeholder first
    header = {"version": VERSION, "page_tokens": PAGE_TOKENS, "cache": cache_meta,
              "layers": entries}
    for e in entries:
        e["pages_offset"] = e["window_offset"] = 10 ** 15
    n = len(json.dumps(header).encode())
    pos = -(-(12 + n) // _ALIGN) * _ALIGN
    for e, (pb, wb) in zip(entries, blobs):
        e["pages_offset"] = pos
        pos = -(-(pos + len(pb)) // _ALIGN) * _ALIGN
        e["window_offset"] = pos
        pos = -(-(pos + len(wb)) // _ALIGN) * _ALIGN
    hb = json.dumps(header).encode()
    hb += b" " * (n - len(hb))               # same length as the placeholder layout
    f.write(MAGIC + struct.pack("<II", VERSION, len(hb)) + hb)
    cur = 12 + len(hb)
    for e, (pb, wb) in zip(entries, blobs):
        for off, blob in ((e["pages_offset"], pb), (e["window_offset"], wb)):
            f.write(b"\0" * (off - cur))
            f.write(blob)
            cur = off + len(blob)


def read(f: BinaryIO) -> Tuple[dict, List[dict]]:
    """Read a file into (header, layers); each layer dict carries the header
    entry's fields, with `pages` replaced by the page data (uint8 CPU tensor
    [streams][pages][page_bytes]), and `window_k`/`window_v` (or None).
    Checks magic, version, bounds and CRCs."""
    head = f.read(12)
    if len(head) < 12 or head[:4] != MAGIC:
        raise FormatError("not a TurboQuant cache file (bad magic)")
    ver, n = struct.unpack("<II", head[4:])
    if ver != VERSION:
        raise FormatError(f"unsupported format version {ver}")
    header = json.loads(f.read(n).decode())
    data = f.read()
    base = 12 + n
    meta = header["cache"]
    dt = _DTYPES[meta["dtype"]]
    out = []
    for e in header["layers"]:
        def blob(off, nb, crc, what):
            lo = off - base
            if lo < 0 or lo + nb > len(data):
                raise FormatError(f"{what} section out of the file's bounds")
            b = data[lo:lo + nb]
            if zlib.crc32(b) != crc:
                raise FormatError(f"{what} section checksum mismatch")
            return b
        pb = blob(e["pages_offset"], e["pages_nbytes"], e["pages_crc32"], "pages")
        if len(pb) != e["streams"] * e["pages"] * e["page_bytes"]:
            raise FormatError("pages section size disagrees with its shape")
        L = dict(e)
        L["pages"] = _from_raw(pb, torch.uint8, (e["streams"], e["pages"], e["page_bytes"]))
        L["window_k"] = L["window_v"] = None
        if e["window_tokens"]:
            wb = blob(e["window_offset"], e["window_nbytes"], e["window_crc32"], "window")
            half = len(wb) // 2
            shape = (meta["batch_size"], meta["num_heads"], e["window_tokens"], meta["head_dim"])
            L["window_k"] = _from_raw(wb[:half], dt, shape)
            L["window_v"] = _from_raw(wb[half:], dt, shape)
        out.append(L)
    return header, out


def save(cache, path_or_file: Union[str, BinaryIO]) -> None:
    """Write a TurboQuantKVCache (every layer must have stored tokens or be
    empty) to a file or path."""
    meta = {"num_layers": cache.num_layers, "batch_size": cache.batch_size,
            "num_heads": cache.num_heads, "head_dim": cache.head_dim,
            "key_bits": cache.key_bits, "value_bits": cache.value_bits,
            "residual_window": cache.residual_window,
            "protected_layers": cache.protected_layers, "qjl": bool(cache.qjl),
            "dtype": _dtype_name(cache.dtype)}
    layers = []
    for st in cache._stores:
        if st._pages is None:
            pages = torch.zeros((st.batch_size * st.num_heads, 0, st.page_bytes), dtype=torch.uint8)
        else:
            pages = st._pages
        meta["batch_size"], meta["num_heads"] = st.batch_size, st.num_heads
        layers.append({"key_bits": st.key_bits, "value_bits": st.value_bits,
                       "rotation_seed": st.rotation_seed, "page_bytes": st.page_bytes,
                       "tokens": st._comp_ptr, "pages": pages,
                       "window_k": st._win_k, "window_v": st._win_v})
    torch.cuda.synchronize(cache.device)
    if isinstance(path_or_file, str):
        with open(path_or_file, "wb") as f:
            write(f, meta, layers)
    else:
        write(path_or_file, meta, layers)


def load(path_or_file: Union[str, BinaryIO], device, max_seq_len: Optional[int] = None,
         **cache_kwargs):
    """Rebuild a TurboQuantKVCache on `device` from a file written by save().
    Extra keyword arguments (fused_attention, ...) go to the constructor."""
    from .kv_cache import TurboQuantKVCache
    if isinstance(path_or_file, str):
        with open(path_or_file, "rb") as f:
            header, layers = read(f)
    else:
        header, layers = read(path_or_file)
    m = header["cache"]
    tokens = max([L["tokens"] for L in layers] + [1])
    cache = TurboQuantKVCache(num_layers=m["num_layers"], batch_size=m["batch_size"],
                              num_heads=m["num_heads"], head_dim=m["head_dim"],
                              key_bits=m["key_bits"], value_bits=m["value_bits"],
                              residual_window=m["residual_window"],
                              protected_layers=m["protected_layers"], dtype=_DTYPES[m["dtype"]],
                              device=device, max_seq_len=max(max_seq_len or 0, tokens),
                              qjl=m["qjl"], **cache_kwargs)
    for st, L in zip(cache._stores, layers):
        for k in ("key_bits", "value_bits", "rotation_seed", "page_bytes"):
            if getattr(st, k) != L[k]:
                raise FormatError(f"layer {k} {L[k]} does not match the rebuilt cache's {getattr(st, k)}")
        if L["tokens"] == 0 and L["window_k"] is None:
            continue
        st._lazy_alloc(m["batch_size"], m["num_heads"])
        if L["streams"] != st._pages.shape[0]:
            raise FormatError("stream count does not match batch_size * num_heads")
        st._ensure_capacity(L["tokens"])
        st._pages[:, :L["pages"].shape[1]] = L["pages"].to(st.device)
        st._comp_ptr = L["tokens"]
        if L["window_k"] is not None:
            st._win_k = L["window_k"].to(st.device)
            st._win_v = L["window_v"].to(st.device)
    return cache
