"""torch-facing wrappers of the libtq_b200 C ABI.

Tensors are owned by PyTorch; the kernels borrow raw device pointers and run
on the current CUDA stream.  Every wrapper raises (never falls back to a CPU
or PyTorch implementation) when the library or the device is unavailable.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Optional

import torch

from .. import _lib

_DT = {torch.float32: _lib.TQ_F32, torch.float16: _lib.TQ_F16, torch.bfloat16: _lib.TQ_BF16}


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("TurboQuant kernels need CUDA tensors (there is no CPU path)")


def tensor4(x: torch.Tensor) -> _lib.Tensor4:
    if x.dim() != 4:
        raise ValueError(f"expected a 4-d tensor, got shape {tuple(x.shape)}")
    if x.dtype not in _DT:
        raise ValueError(f"unsupported dtype {x.dtype}")
    t = _lib.Tensor4()
    t.data = x.data_ptr()
    t.dtype = _DT[x.dtype]
    t.shape[:] = x.shape
    t.stride[:] = x.stride()
    return t


@dataclass
class LayerTables:
    """Per-layer constant device tables (codebooks, rotation, QJL matrix)."""
    head_dim: int
    key_bits: int
    value_bits: int
    qjl: bool
    k_centroids: torch.Tensor
    k_boundaries: torch.Tensor
    v_centroids: torch.Tensor
    v_boundaries: torch.Tensor
    rot: torch.Tensor
    qjl_mat: Optional[torch.Tensor] = None
    rot_t: Optional[torch.Tensor] = None
    qjl_t: Optional[torch.Tensor] = None
    rot_bf16x3: Optional[torch.Tensor] = None
    rot_f16: Optional[torch.Tensor] = None
    qjl_bf16: Optional[torch.Tensor] = None

    def __post_init__(self):
        self.rot = self.rot.contiguous().float()
        self.rot_t = self.rot.t().contiguous()
        self.rot_f16 = self.rot.half().contiguous()      # prefill attention
        if self.head_dim == 128:
            # R = hi + mid + lo in bf16 (24 significant bits): the tensor-core
            # append computes x R^T as three exact bf16 products summed in fp32;
            # rows permuted into the packed K / V orders (tq_tables.rot_bf16x3)
            hi = self.rot.bfloat16()
            r1 = self.rot - hi.float()
            mid = r1.bfloat16()
            lo = (r1 - mid.float()).bfloat16()
            terms = torch.stack([hi, mid, lo])
            ko, vo = row_orders(self.head_dim)
            dev = self.rot.device
            self.rot_bf16x3 = torch.stack([terms[:, torch.as_tensor(ko, device=dev)],
                                           terms[:, torch.as_tensor(vo, device=dev)]]).contiguous()
        if self.qjl_mat is not None:
            self.qjl_mat = self.qjl_mat.contiguous().float()
            self.qjl_t = self.qjl_mat.t().contiguous()
            # the tensor-core append sketches with S in bf16: only when S is
            # exactly bf16 (the library's own S is), rows and columns in K
            # quad order (tq_tables.qjl_bf16)
            sb = self.qjl_mat.bfloat16()
            if self.head_dim == 128 and torch.equal(sb.float(), self.qjl_mat):
                ko = torch.as_tensor(row_orders(self.head_dim)[0], device=self.qjl_mat.device)
                self.qjl_bf16 = sb[ko][:, ko].contiguous()

    def __setattr__(self, name, value):
        # a changed table invalidates the cached C descriptors
        self.__dict__.pop("_geom", None)
        self.__dict__.pop("_ctab", None)
        super().__setattr__(name, value)

    def geom(self) -> _lib.Geom:
        g = self.__dict__.get("_geom")
        if g is None:
            g = _lib.Geom(self.head_dim, self.key_bits, self.value_bits, 1 if self.qjl else 0)
            self.__dict__["_geom"] = g
        return g

    def ctables(self) -> _lib.Tables:
        """The C table descriptor (built once: the tables never move)."""
        t = self.__dict__.get("_ctab")
        if t is None:
            t = self._build_ctables()
            self.__dict__["_ctab"] = t
        return t

    def _build_ctables(self) -> _lib.Tables:
        t = _lib.Tables()
        t.k_centroids = self.k_centroids.data_ptr()
        t.k_boundaries = self.k_boundaries.data_ptr()
        t.v_centroids = self.v_centroids.data_ptr()
        t.v_boundaries = self.v_boundaries.data_ptr()
        t.rot = self.rot.data_ptr()
        t.qjl = self.qjl_mat.data_ptr() if self.qjl_mat is not None else None
        t.rot_t = self.rot_t.data_ptr()
        t.qjl_t = self.qjl_t.data_ptr() if self.qjl_t is not None else None
        t.rot_bf16x3 = self.rot_bf16x3.data_ptr() if self.rot_bf16x3 is not None else None
        t.rot_f16 = self.rot_f16.data_ptr() if self.rot_f16 is not None else None
        t.qjl_bf16 = self.qjl_bf16.data_ptr() if self.qjl_bf16 is not None else None
        return t


def row_orders(head_dim: int):
    """Coordinate stored at each position of a packed K row (quad order: quad t
    lists 16j+2t, 16j+2t+1, 16j+2t+8, 16j+2t+9 for every 16-coordinate chunk j)
    and of a packed V row (octet order: octet g lists g, g+8, g+16, ...)."""
    k = [16 * j + 2 * t + e for t in range(4) for j in range(head_dim // 16)
         for e in (0, 1, 8, 9)]
    v = [g + 8 * c for g in range(8) for c in range(head_dim // 8)]
    return k, v


def page_bytes(head_dim: int, key_bits: int, value_bits: int, qjl: bool) -> int:
    """Bytes of one 64-token page (same formula as tq_page_bytes)."""
    krow, vrow = head_dim * key_bits // 8, head_dim * value_bits // 8
    qrow = head_dim // 8 if qjl else 0
    return _lib.PAGE_TOKENS * (krow + vrow + qrow + 4 + (2 if qjl else 0))


@dataclass
class PagedPages:
    """Paged storage (vLLM-style): a pool of pages and one block table row per
    stream; logical page p of stream s is pool[block_table[s, p]].  Accepted
    wherever a contiguous (streams, pages, page_bytes) tensor is.  Entries
    outside the pool are never dereferenced: the kernels read pool page 0 /
    drop the write and set _lib.DEV_BAD_BLOCK in the device status word."""
    pool: torch.Tensor          # uint8 (num_blocks, page_bytes)
    block_table: torch.Tensor   # int32 (streams, max_pages)

    def __post_init__(self):
        if self.pool.dtype != torch.uint8 or self.pool.dim() != 2:
            raise ValueError("pool must be uint8 (num_blocks, page_bytes)")
        if self.block_table.dtype != torch.int32 or self.block_table.dim() != 2 or \
                self.block_table.stride(1) != 1:
            raise ValueError("block_table must be int32 (streams, max_pages), rows contiguous")
        if self.block_table.device != self.pool.device:
            raise ValueError("pool and block_table must be on the same device")

    @property
    def is_cuda(self) -> bool:
        return self.pool.is_cuda

    @property
    def device(self) -> torch.device:
        return self.pool.device

    @property
    def shape(self):
        """(streams, pages per stream, page_bytes), as a contiguous page tensor."""
        return (self.block_table.shape[0], self.block_table.shape[1], self.pool.shape[1])


def _cache_desc(pages) -> _lib.Cache:
    if isinstance(pages, PagedPages):
        bt = pages.block_table
        return _lib.Cache(pages.pool.data_ptr(), bt.shape[0], bt.shape[1], bt.data_ptr(),
                          bt.stride(0), pages.pool.shape[0])
    return _lib.Cache(pages.data_ptr(), pages.shape[0], pages.shape[1])


# ---------------------------------------------------------------------------
def quantize_rotated(y: torch.Tensor, boundaries: torch.Tensor) -> torch.Tensor:
    """Bit-exact torch.bucketize(y, boundaries) -> int16, on the GPU."""
    _require_cuda(y, boundaries)
    y = y.contiguous().float()
    b = boundaries.contiguous().float()
    codes = torch.empty(y.shape, dtype=torch.int16, device=y.device)
    lib = _lib.load()
    _lib.check("tq_quantize_rotated",
               lib.tq_quantize_rotated(y.data_ptr(), y.numel(), b.data_ptr(), b.numel(),
                                       codes.data_ptr(), _stream(y.device)))
    return codes


def append(tables: LayerTables, pages: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
           pos: int) -> None:
    """Quantise and store tokens [pos, pos+T) of (B, H, T, D) k/v into pages."""
    _require_cuda(pages, k, v)
    lib = _lib.load()
    g, t, c = tables.geom(), tables.ctables(), _cache_desc(pages)
    kt, vt = tensor4(k), tensor4(v)
    _lib.check("tq_append", lib.tq_append(ctypes.byref(g), ctypes.byref(t), ctypes.byref(c),
                                          ctypes.byref(kt), ctypes.byref(vt), int(pos),
                                          _stream(k.device)))


def append_uses_tensor_cores(tables: LayerTables, k: torch.Tensor, v: torch.Tensor) -> bool:
    """True when append() with these inputs runs the tcgen05 kernel."""
    lib = _lib.load()
    g, t = tables.geom(), tables.ctables()
    kt, vt = tensor4(k), tensor4(v)
    return bool(lib.tq_append_tensor_core(ctypes.byref(g), ctypes.byref(t), ctypes.byref(kt),
                                          ctypes.byref(vt)))


def device_status(device: torch.device) -> int:
    """Read and clear the library's device status word (0: no kernel timed out)."""
    lib = _lib.load()
    st = ctypes.c_uint32(0)
    rc = lib.tq_device_status(ctypes.byref(st), _stream(device))
    if rc not in (_lib.TQ_OK, _lib.TQ_ERR_DEVICE):
        _lib.check("tq_device_status", rc)
    return int(st.value)


def dequantize(tables: LayerTables, pages: torch.Tensor, t0: int, t1: int,
               k_out: Optional[torch.Tensor], v_out: Optional[torch.Tensor]) -> None:
    """Write dequantised tokens [t0, t1) into (B, H, t1-t0, D) views."""
    _require_cuda(pages, k_out, v_out)
    lib = _lib.load()
    g, t, c = tables.geom(), tables.ctables(), _cache_desc(pages)
    ko = tensor4(k_out) if k_out is not None else None
    vo = tensor4(v_out) if v_out is not None else None
    _lib.check("tq_dequantize", lib.tq_dequantize(
        ctypes.byref(g), ctypes.byref(t), ctypes.byref(c), int(t0), int(t1),
        ctypes.byref(ko) if ko is not None else None,
        ctypes.byref(vo) if vo is not None else None, _stream(pages.device)))


class DecodeWorkspace:
    """Grow-only device scratch for tq_decode_attn (first 4 bytes: status word)."""

    def __init__(self):
        self.buf: Optional[torch.Tensor] = None

    def get(self, nbytes: int, device: torch.device) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        return self.buf

    def status(self) -> int:
        """Read and clear the device status word (synchronises the stream)."""
        if self.buf is None:
            return 0
        lib = _lib.load()
        st = ctypes.c_uint32(0)
        lib.tq_workspace_status(self.buf.data_ptr(), ctypes.byref(st), _stream(self.buf.device))
        return int(st.value)


def _seq_lens_ptr(seq_lens: Optional[torch.Tensor], q: torch.Tensor) -> Optional[int]:
    if seq_lens is None:
        return None
    if seq_lens.dtype != torch.int32 or seq_lens.dim() != 1 or \
            seq_lens.shape[0] != q.shape[0] or not seq_lens.is_contiguous():
        raise ValueError("seq_lens must be a contiguous int32 (B,) tensor")
    if seq_lens.device != q.device:
        raise ValueError("seq_lens must be on the query's device")
    return seq_lens.data_ptr()


def _row_ptr(x: Optional[torch.Tensor], q: torch.Tensor, name: str) -> Optional[int]:
    """Device pointer of an int32 (B,) per-row tensor (seq_lens, kv_start)."""
    if x is None:
        return None
    if x.dtype != torch.int32 or x.dim() != 1 or x.shape[0] != q.shape[0] or \
            not x.is_contiguous():
        raise ValueError(f"{name} must be a contiguous int32 (B,) tensor")
    if x.device != q.device:
        raise ValueError(f"{name} must be on the query's device")
    return x.data_ptr()


def _decode_args(q, out, n_tokens, window_k, window_v, scale, num_ctas, phases, keep,
                 seq_lens=None, kv_start=None):
    qt, ot = tensor4(q), tensor4(out)
    wk = tensor4(window_k) if window_k is not None and window_k.shape[2] > 0 else None
    wv = tensor4(window_v) if wk is not None else None
    keep += [qt, ot, wk, wv]
    a = _lib.DecodeArgs()
    a.q = ctypes.pointer(qt)
    a.out = ctypes.pointer(ot)
    a.window_k = ctypes.pointer(wk) if wk is not None else None
    a.window_v = ctypes.pointer(wv) if wv is not None else None
    a.n_tokens = int(n_tokens)
    a.num_q_heads = q.shape[1]
    a.scale = float(scale if scale is not None else 1.0 / math.sqrt(q.shape[-1]))
    a.num_ctas = int(num_ctas)
    a.phases = int(phases)
    a.seq_lens = _seq_lens_ptr(seq_lens, q)
    a.kv_start = _row_ptr(kv_start, q, "kv_start")
    return a


def decode_step(tables: LayerTables, pages: torch.Tensor, k_new: torch.Tensor,
                v_new: torch.Tensor, pos: int, q: torch.Tensor,
                window_k: Optional[torch.Tensor] = None,
                window_v: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                out: Optional[torch.Tensor] = None,
                workspace: Optional[DecodeWorkspace] = None,
                num_ctas: int = 0, gather: Optional[_lib.Gather] = None,
                seq_lens: Optional[torch.Tensor] = None,
                kv_start: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Store the new (B, Hkv, 1, D) token at ``pos`` and attend q over tokens
    [0, pos + 1) plus the window, in one call (tq_decode_step).  ``gather``
    (a filled _lib.Gather whose peer_out[rank] is ``out``) also delivers the
    output block to every rank's gathered buffer (fused all-gather).

    ``seq_lens`` (int32 (B,) on the device, each <= pos + 1) makes the batch
    ragged: row b stores its token at seq_lens[b] - 1 and attends tokens
    [0, seq_lens[b]); ``pos`` is then the bound (the longest row's position).
    ``kv_start`` (int32 (B,) on the device): row b's keys before that position
    take no weight (left padding)."""
    _require_cuda(pages, q, k_new, v_new)
    lib = _lib.load()
    if out is None:
        out = torch.empty_like(q)
    g, t, c = tables.geom(), tables.ctables(), _cache_desc(pages)
    keep = []
    a = _decode_args(q, out, pos + 1, window_k, window_v, scale, num_ctas, 0, keep, seq_lens,
                     kv_start)
    if gather is not None:
        a.gather = ctypes.pointer(gather)
    kt, vt = tensor4(k_new), tensor4(v_new)
    nbytes = lib.tq_decode_workspace_bytes(ctypes.byref(g), ctypes.byref(c), ctypes.byref(a))
    if nbytes == 0:
        raise _lib.TqError("tq_decode_workspace_bytes", _lib.TQ_ERR_INVALID, _lib.last_error())
    ws = (workspace or DecodeWorkspace()).get(nbytes, q.device)
    _lib.check("tq_decode_step", lib.tq_decode_step(
        ctypes.byref(g), ctypes.byref(t), ctypes.byref(c), ctypes.byref(kt), ctypes.byref(vt),
        int(pos), ctypes.byref(a), ws.data_ptr(), ws.numel(), _stream(q.device)))
    return out


def prefill_uses_tensor_cores(tables: LayerTables) -> bool:
    """Whether prefill_attention (engine 0) runs the tcgen05 kernel for this
    layer's geometry."""
    return bool(_lib.load().tq_prefill_tensor_core(ctypes.byref(tables.geom())))


def prefill_attention(tables: LayerTables, pages: torch.Tensor, q: torch.Tensor,
                      n_tokens: int, scale: Optional[float] = None, causal: bool = True,
                      out: Optional[torch.Tensor] = None, engine: int = 0,
                      kv_start: Optional[torch.Tensor] = None,
                      window_k: Optional[torch.Tensor] = None,
                      window_v: Optional[torch.Tensor] = None,
                      workspace: Optional[DecodeWorkspace] = None) -> torch.Tensor:
    """Attention of queries q (B, Hq, Tq, D) at positions n_tokens - Tq ..
    n_tokens - 1 over the packed tokens [0, n_tokens) of every stream (causal:
    a query sees keys at or before its position).  ``engine`` 0 picks the
    fastest kernel (tcgen05 where prefill_uses_tensor_cores), 1 the mma.sync
    kernel, 2 / 3 the tcgen05 kernel with 128 / 256 query rows per CTA.
    ``kv_start`` (int32 (B,) on the device): row b's keys before that position
    take no weight (left padding; a query with no key left returns zeros).
    ``window_k`` / ``window_v`` ((B, Hkv, W, D)): the residual window, dense
    keys at positions n_tokens - W .. n_tokens - 1 after the packed ones."""
    _require_cuda(pages, q)
    lib = _lib.load()
    if out is None:
        out = torch.empty_like(q)
    g, t, c = tables.geom(), tables.ctables(), _cache_desc(pages)
    qt, ot = tensor4(q), tensor4(out)
    a = _lib.PrefillArgs(ctypes.pointer(qt), ctypes.pointer(ot), int(n_tokens),
                         float(scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])),
                         1 if causal else 0, int(engine), _row_ptr(kv_start, q, "kv_start"))
    if window_k is not None and window_k.shape[2] > 0:
        wk, wv = tensor4(window_k), tensor4(window_v)
        a.window_k, a.window_v = ctypes.pointer(wk), ctypes.pointer(wv)
        nbytes = lib.tq_prefill_workspace_bytes(ctypes.byref(g), ctypes.byref(c), ctypes.byref(a))
        ws = (workspace or DecodeWorkspace()).get(nbytes, q.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check("tq_prefill_attn", lib.tq_prefill_attn(
        ctypes.byref(g), ctypes.byref(t), ctypes.byref(c), ctypes.byref(a), _stream(q.device)))
    return out


def decode_attention(tables: LayerTables, pages: torch.Tensor, q: torch.Tensor,
                     n_tokens: int, window_k: Optional[torch.Tensor] = None,
                     window_v: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                     out: Optional[torch.Tensor] = None,
                     workspace: Optional[DecodeWorkspace] = None,
                     num_ctas: int = 0, phases: int = 0,
                     seq_lens: Optional[torch.Tensor] = None,
                     kv_start: Optional[torch.Tensor] = None) -> torch.Tensor:
    """softmax(q K^T * scale) V over the packed tokens [0, n_tokens) of every
    stream plus an optional full-precision window.  q: (B, Hq, 1, D).

    ``phases`` (OR of _lib.PHASE_*) runs a subset of the three kernels; the
    later phases read what the earlier ones left in the same ``workspace``.
    ``seq_lens`` (int32 (B,) on the device) gives each batch row its own
    token count, clamped to [0, n_tokens] (continuous batching).  ``kv_start``
    (int32 (B,) on the device): row b's keys before that position, window
    tokens included, take no weight (left padding)."""
    _require_cuda(pages, q)
    lib = _lib.load()
    if out is None:
        out = torch.empty_like(q)
    g, t, c = tables.geom(), tables.ctables(), _cache_desc(pages)
    keep = []
    a = _decode_args(q, out, n_tokens, window_k, window_v, scale, num_ctas, phases, keep,
                     seq_lens, kv_start)
    nbytes = lib.tq_decode_workspace_bytes(ctypes.byref(g), ctypes.byref(c), ctypes.byref(a))
    if nbytes == 0:
        raise _lib.TqError("tq_decode_workspace_bytes", _lib.TQ_ERR_INVALID, _lib.last_error())
    ws = (workspace or DecodeWorkspace()).get(nbytes, q.device)
    _lib.check("tq_decode_attn", lib.tq_decode_attn(
        ctypes.byref(g), ctypes.byref(t), ctypes.byref(c), ctypes.byref(a),
        ws.data_ptr(), ws.numel(), _stream(q.device)))
    return out
