"""KV-head parallel decode, host logic, on CPU with gloo ranks (world size 2 and 4).

The per-rank attention is the oracle's (float64 SDPA over the rank's own
heads), standing in for the CUDA decode, so these tests check what the
multi-GPU path adds: which heads a rank owns, that the gathered output is the
single-process output in global head order, and that a rank that raises or
stalls makes its peers fail fast instead of hanging.
"""
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bhaskera_col_b200.inference.head_parallel import HeadParallelDecoder, HeadShard, ShardFailure
from oracle import tq_oracle as O

B, HQ, HKV, T, D, LAYERS = 2, 8, 4, 37, 16, 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data(seed=0):
    rng = np.random.Generator(np.random.PCG64(seed))
    hist_k = rng.standard_normal((LAYERS, B, HKV, T, D)).astype(np.float32)
    hist_v = rng.standard_normal((LAYERS, B, HKV, T, D)).astype(np.float32)
    q = rng.standard_normal((LAYERS, B, HQ, 1, D)).astype(np.float32)
    k1 = rng.standard_normal((LAYERS, B, HKV, 1, D)).astype(np.float32)
    v1 = rng.standard_normal((LAYERS, B, HKV, 1, D)).astype(np.float32)
    return hist_k, hist_v, q, k1, v1


class _OracleCache:
    """Holds (B, h, T, D) history per layer; decode = append + oracle SDPA."""

    def __init__(self, hist_k, hist_v):
        self.k = [torch.from_numpy(x) for x in hist_k]
        self.v = [torch.from_numpy(x) for x in hist_v]

    def append(self, k, v, layer):
        self.k[layer] = torch.cat([self.k[layer], k], 2)
        self.v[layer] = torch.cat([self.v[layer], v], 2)

    def decode(self, q, k, v, layer, scale=None):
        self.append(k, v, layer)
        return torch.from_numpy(O.sdpa(q.numpy(), self.k[layer].numpy(), self.v[layer].numpy()))


def _init(rank, world, port, timeout_s):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _worker_decode(rank, world, port, out_dir):
    _init(rank, world, port, 60)
    shard = HeadShard(HQ, HKV, rank, world)
    hk, hv, q, k1, v1 = _data()
    cache = _OracleCache(hk[:, :, shard.kv_slice], hv[:, :, shard.kv_slice])
    dec = HeadParallelDecoder(cache, shard)
    outs = [dec.decode(torch.from_numpy(q[l]), torch.from_numpy(k1[l]), torch.from_numpy(v1[l]), l)
            for l in range(LAYERS)]
    torch.save(torch.stack(outs), os.path.join(out_dir, f"out{rank}.pt"))
    dist.destroy_process_group()


def _worker_fault(rank, world, port, out_dir, mode):
    _init(rank, world, port, 4)
    shard = HeadShard(HQ, HKV, rank, world)
    out = torch.zeros((B, shard.q_heads, 1, D))
    if rank == 1:
        if mode == "raise":
            return                      # leaves between steps, never joins the gather
        time.sleep(12)                  # stalls past the group timeout
        return
    t0 = time.time()
    try:
        shard.gather(out, layer=5)
        result = "no error"
    except ShardFailure as e:
        result = f"ShardFailure {time.time() - t0:.1f}s {e}"
    with open(os.path.join(out_dir, "fault.txt"), "w") as f:
        f.write(result)


def test_head_ranges():
    s = [HeadShard(32, 8, r, 4) for r in range(4)]
    assert [x.kv_slice for x in s] == [slice(0, 2), slice(2, 4), slice(4, 6), slice(6, 8)]
    assert [x.q_slice for x in s] == [slice(0, 8), slice(8, 16), slice(16, 24), slice(24, 32)]
    # every query head of a rank attends one of the rank's KV heads (GQA group 4)
    for x in s:
        kv = range(x.kv_slice.start, x.kv_slice.stop)
        assert all(h // 4 in kv for h in range(x.q_slice.start, x.q_slice.stop))
    with pytest.raises(ValueError):
        HeadShard(32, 8, 0, 3)           # 8 KV heads over 3 ranks
    with pytest.raises(ValueError):
        HeadShard(30, 8, 0, 2)           # query heads not a multiple of KV heads
    with pytest.raises(ValueError):
        HeadShard(32, 8, 2, 2)           # rank out of range
    with pytest.raises(ValueError):
        HeadShard(32, 8, 0, 2).local_kv(torch.zeros(1, 4, 1, 8))


def test_single_rank_gather_is_identity():
    s = HeadShard(8, 4)
    x = torch.randn(2, 8, 1, 16)
    assert s.gather(x) is x


@pytest.mark.parametrize("world", [2, 4])
def test_multi_rank_decode_equals_single_process(tmp_path, world):
    """world 4 leaves one KV head per rank, the 8-GPU split of 8 KV heads."""
    port = _free_port()
    mp.start_processes(_worker_decode, args=(world, port, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    hk, hv, q, k1, v1 = _data()
    full = _OracleCache(hk, hv)
    want = torch.stack([full.decode(torch.from_numpy(q[l]), torch.from_numpy(k1[l]),
                                    torch.from_numpy(v1[l]), l) for l in range(LAYERS)])
    for r in range(world):
        got = torch.load(os.path.join(tmp_path, f"out{r}.pt"))
        assert got.shape == (LAYERS, B, HQ, 1, D)
        assert torch.equal(got, want), r


@pytest.mark.parametrize("mode", ["raise", "stall"])
def test_peer_failure_ends_the_gather(tmp_path, mode):
    port = _free_port()
    ctx = mp.start_processes(_worker_fault, args=(2, port, str(tmp_path), mode), nprocs=2,
                             join=False, start_method="spawn")
    deadline = time.time() + 60
    while not ctx.join(timeout=1):
        assert time.time() < deadline, "ranks did not finish"
    res = open(os.path.join(tmp_path, "fault.txt")).read()
    assert res.startswith("ShardFailure"), res
    assert "layer 5" in res
    assert float(res.split()[1][:-1]) < 30
