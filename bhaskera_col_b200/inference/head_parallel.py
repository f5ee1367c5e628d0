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

Failure handling is on the host: the process group is created with a short
timeout, so when a rank dies or stalls the others' next all-gather raises
instead of waiting for ever; `HeadShard.gather` turns that into
`ShardFailure` naming the layer.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


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
            dist.all_gather_into_tensor(buf, out_local.contiguous(), group=group)
        except Exception as e:    # gloo / NCCL timeouts and peer failures
            where = f" at layer {layer}" if layer is not None else ""
            raise ShardFailure(f"rank {self.rank}: all-gather of attention outputs failed"
                               f"{where}: {e}") from e
        return buf.view(self.world, B, h, T, D).permute(1, 0, 2, 3, 4).reshape(
            B, self.num_q_heads, T, D)


class HeadParallelDecoder:
    """Per-layer decode over this rank's heads, output gathered over all ranks.

    `cache` holds only the rank's KV heads (a TurboQuantKVCache built with
    num_heads = shard.kv_heads); `decode` takes the full (B, Hq, 1, D) query
    and (B, Hkv, 1, D) new K/V of the step, as the single-GPU cache does.
    """

    def __init__(self, cache, shard: HeadShard, group=None):
        self.cache = cache
        self.shard = shard
        self.group = group

    def append(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int):
        self.cache.append(self.shard.local_kv(key_states), self.shard.local_kv(value_states),
                          layer_idx)

    def decode(self, query_states: torch.Tensor, key_states: torch.Tensor,
               value_states: torch.Tensor, layer_idx: int, scale: Optional[float] = None,
               buf: Optional[torch.Tensor] = None) -> torch.Tensor:
        s = self.shard
        out = self.cache.decode(s.local_q(query_states), s.local_kv(key_states),
                                s.local_kv(value_states), layer_idx, scale=scale)
        return s.gather(out, group=self.group, buf=buf, layer=layer_idx)
