"""KV-head parallel decode over several GPUs (one process per GPU).

KV heads are independent: a KV head's packed pages, its append and its
decode attention touch only that head and its GQA group of query heads.  So
with `world` ranks each rank keeps the packed cache of num_kv_heads / world
consecutive KV heads (and serves the num_q_heads / world query heads that
attend them); the only exchange is one all-gather of the attention output per
layer, (B, Hq / world, T, D) from each rank, which rebuilds (B, Hq, T, D) in
global head order.

This is the multi-GPU form of the reference's single-process cache
(kv_cache.py:516-624, called from engine.py:361-389): the same per-layer
calls, with K/V/Q sliced to the rank's heads before the call and the output
gathered after it.

The gather runs one of two ways.  `HeadShard.gather` calls NCCL (or gloo on
CPU).  `SharedGather` fuses it into the decode itself: every rank maps every
other rank's gathered-output buffer (CUDA IPC, plain peer memory), the
merge kernel stores each finished output block into all ranks' buffers over
NVLink and counts its arrival on each rank, and each rank's last merge CTA
waits (bounded) for all blocks of the layer; no collective library call and
no extra kernel is left on the decode path.

Failure handling is on the host: the process group is created with a short
timeout, so when a rank dies or stalls the others' next all-gather raises
instead of waiting for ever; `HeadShard.gather` turns that into
`ShardFailure` naming the layer.  The fused gather's device wait gives up
after ~2 s and sets TQ_DEV_WAIT_TIMEOUT in the decode workspace's status word.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from .. import _lib


class ShardFailure(RuntimeError):
    """A collective of the head-parallel decode failed (a peer died or timed out)."""


@dataclass(frozen=True)
class HeadShard:
    """The heads one rank owns, and the per-layer output gather."""

    num_q_heads: int
    num_kv_heads: int
    rank: int = 0
    world: int = 1

    def __post_init__(self):
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside a world of {self.world}")
        if self.num_kv_heads % self.world:
            raise ValueError(f"{self.num_kv_heads} KV heads do not split over {self.world} ranks")
        if self.num_q_heads % self.num_kv_heads:
            raise ValueError(f"{self.num_q_heads} query heads are not a multiple of "
                             f"{self.num_kv_heads} KV heads")

    # -- head ranges ----------------------------------------------------------
    @property
    def kv_heads(self) -> int:
        return self.num_kv_heads // self.world

    @property
    def q_heads(self) -> int:
        return self.num_q_heads // self.world

    @property
    def kv_slice(self) -> slice:
        return slice(self.rank * self.kv_heads, (self.rank + 1) * self.kv_heads)

    @property
    def q_slice(self) -> slice:
        # query head h attends KV head h // (Hq / Hkv): the rank's KV heads
        # serve a contiguous block of query heads
        return slice(self.rank * self.q_heads, (self.rank + 1) * self.q_heads)

    def local_kv(self, x: torch.Tensor) -> torch.Tensor:
        """(B, Hkv, T, D) -> this rank's (B, Hkv / world, T, D)."""
        if x.shape[1] != self.num_kv_heads:
            raise ValueError(f"expected {self.num_kv_heads} KV heads, got {x.shape[1]}")
        return x[:, self.kv_slice]

    def local_q(self, q: torch.Tensor) -> torch.Tensor:
        """(B, Hq, T, D) -> this rank's (B, Hq / world, T, D)."""
        if q.shape[1] != self.num_q_heads:
            raise ValueError(f"expected {self.num_q_heads} query heads, got {q.shape[1]}")
        return q[:, self.q_slice]

    # -- the exchange ---------------------------------------------------------
    def gather(self, out_local: torch.Tensor, group=None, buf: Optional[torch.Tensor] = None,
               layer: Optional[int] = None) -> torch.Tensor:
        """All-gather the ranks' (B, Hq / world, T, D) outputs into (B, Hq, T, D)."""
        if self.world == 1:
            return out_local
        B, h, T, D = out_local.shape
        if h != self.q_heads:
            raise ValueError(f"local output has {h} heads, expected {self.q_heads}")
        if buf is None:
            buf = torch.empty((self.world * B, h, T, D), dtype=out_local.dtype,
                              device=out_local.device)
        try:
            # concatenated along dim 0 (the form every backend accepts)
            with torch.cuda.nvtx.range("tq.all_gather"):
                dist.all_gather_into_tensor(buf, out_local.contiguous(), group=group)
        except Exception as e:    # gloo / NCCL timeouts and peer failures
            where = f" at layer {layer}" if layer is not None else ""
            raise ShardFailure(f"rank {self.rank}: all-gather of attention outputs failed"
                               f"{where}: {e}") from e
        return buf.view(self.world, B, h, T, D).permute(1, 0, 2, 3, 4).reshape(
            B, self.num_q_heads, T, D)


class _CudaArray:
    """__cuda_array_interface__ over a raw device pointer (int16 elements)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i2",
                                         "data": (ptr, False), "version": 3}


class SharedGather:
    """Gathered-output buffers in peer-mapped memory for the fused all-gather.

    One buffer per rank holds, for every layer, the (world * B, Hq / world, 1,
    D) gathered output (rank r's block at rows r*B .. r*B + B - 1, the layout
    all_gather_into_tensor produces), followed by 16 bytes per layer: three
    uint32 words (arrivals from all ranks, which only grow; this rank's
    finished merge CTAs; this rank's completed calls).  Every rank maps every
    other rank's buffer.  Collective: all ranks construct it together (the IPC
    handles travel through the group)."""

    def __init__(self, shard: HeadShard, layers: int, batch: int, head_dim: int,
                 device: torch.device, group=None, dtype=torch.bfloat16):
        if shard.world > _lib.MAX_PEERS:
            raise ValueError(f"at most {_lib.MAX_PEERS} ranks")
        if dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("the gathered output is bf16 or fp16")
        self.shard, self.layers, self.batch, self.dtype = shard, layers, batch, dtype
        self.block = (batch, shard.q_heads, 1, head_dim)
        self.block_elems = batch * shard.q_heads * head_dim
        self.layer_elems = shard.world * self.block_elems
        out_bytes = layers * self.layer_elems * 2
        self.flag_off = (out_bytes + 255) // 256 * 256
        total = self.flag_off + 16 * layers
        lib = _lib.load()
        with torch.cuda.device(device):
            ptr = ctypes.c_void_p()
            handle = (ctypes.c_char * _lib.SHARED_HANDLE_BYTES)()
            _lib.check("tq_shared_alloc", lib.tq_shared_alloc(total, ctypes.byref(ptr), handle))
            self._own = ptr.value
            handles: List[bytes] = [b""] * shard.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            self.bases: List[int] = []
            self._opened: List[int] = []
            for r in range(shard.world):
                if r == shard.rank:
                    self.bases.append(self._own)
                    continue
                peer = ctypes.c_void_p()
                buf = (ctypes.c_char * _lib.SHARED_HANDLE_BYTES).from_buffer_copy(handles[r])
                _lib.check("tq_shared_open", lib.tq_shared_open(buf, ctypes.byref(peer)))
                self.bases.append(peer.value)
                self._opened.append(peer.value)
        own = torch.as_tensor(_CudaArray(self._own, layers * self.layer_elems), device=device)
        self.out = own.view(dtype).view(layers, shard.world * batch, *self.block[1:])
        self._args = []
        for layer in range(layers):
            g = _lib.Gather()
            g.world, g.rank = shard.world, shard.rank
            blk = (layer * self.layer_elems + shard.rank * self.block_elems) * 2
            for r in range(shard.world):
                g.peer_out[r] = self.bases[r] + blk
                g.peer_flag[r] = self.bases[r] + self.flag_off + 16 * layer
            self._args.append(g)
        dist.barrier(group=group)           # every rank has mapped every buffer

    def block_view(self, layer: int) -> torch.Tensor:
        """This rank's (B, Hq / world, 1, D) block of the layer, in its own buffer."""
        r, B = self.shard.rank, self.batch
        return self.out[layer, r * B:(r + 1) * B]

    def args(self, layer: int) -> "_lib.Gather":
        return self._args[layer]

    def gathered(self, layer: int) -> torch.Tensor:
        """The layer's gathered output, (world * B, Hq / world, 1, D)."""
        return self.out[layer]

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective)."""
        lib = _lib.load()
        torch.cuda.synchronize()
        dist.barrier()
        for p in self._opened:
            lib.tq_shared_close(p)
        self._opened = []
        dist.barrier()
        if self._own:
            lib.tq_shared_free(self._own)
            self._own = 0


class HeadParallelDecoder:
    """Per-layer decode over this rank's heads, output gathered over all ranks.

    `cache` holds only the rank's KV heads (a TurboQuantKVCache built with
    num_heads = shard.kv_heads); `decode` takes the full (B, Hq, 1, D) query
    and (B, Hkv, 1, D) new K/V of the step, as the single-GPU cache does.
    With `fused` (a SharedGather) the all-gather runs inside the decode.
    """

    def __init__(self, cache, shard: HeadShard, group=None,
                 fused: Optional[SharedGather] = None):
        self.cache = cache
        self.shard = shard
        self.group = group
        self.fused = fused

    def append(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int):
        self.cache.append(self.shard.local_kv(key_states), self.shard.local_kv(value_states),
                          layer_idx)

    def decode(self, query_states: torch.Tensor, key_states: torch.Tensor,
               value_states: torch.Tensor, layer_idx: int, scale: Optional[float] = None,
               buf: Optional[torch.Tensor] = None) -> torch.Tensor:
        s = self.shard
        if self.fused is not None and s.world > 1:
            f = self.fused
            self.cache.decode(s.local_q(query_states), s.local_kv(key_states),
                              s.local_kv(value_states), layer_idx, scale=scale,
                              out=f.block_view(layer_idx), gather=f.args(layer_idx))
            B = query_states.shape[0]
            return f.gathered(layer_idx).view(s.world, B, s.q_heads, 1, -1).permute(
                1, 0, 2, 3, 4).reshape(B, s.num_q_heads, 1, -1)
        # with one rank there is nothing to gather: the decode writes into buf
        kw = {"out": buf} if s.world == 1 and buf is not None else {}
        out = self.cache.decode(s.local_q(query_states), s.local_kv(key_states),
                                s.local_kv(value_states), layer_idx, scale=scale, **kw)
        return s.gather(out, group=self.group, buf=buf, layer=layer_idx)
