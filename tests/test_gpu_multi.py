"""Two-GPU parity of the fused output all-gather (SharedGather): the decode's
merge kernel stores each rank's output block into every rank's buffer over
peer memory; the gathered outputs must equal NCCL's all-gather of the same
per-rank outputs exactly (same kernels, same bytes), over several layers and
steps, and over a one-layer buffer called several times in a row (each call's
arrivals counted against its own target).  Skipped with fewer than two
GPUs."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result):
    import datetime
    import torch.distributed as dist
    from bhaskera_col_b200.inference import TurboQuantKVCache
    from bhaskera_col_b200.inference.head_parallel import (HeadParallelDecoder, HeadShard,
                                                           SharedGather)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        L, B, HQ, HKV, D, T = 3, 2, 16, 4, 128, 300
        shard = HeadShard(HQ, HKV, rank, world)
        g = torch.Generator(device=dev)
        g.manual_seed(11)                      # the same full inputs on every rank
        caches = []
        for _ in range(2):
            c = TurboQuantKVCache(num_layers=L, batch_size=B, num_heads=shard.kv_heads,
                                  head_dim=D, key_bits=4, value_bits=2, residual_window=0,
                                  protected_layers=0, device=dev, max_seq_len=T + 16, qjl=True)
            caches.append(c)
        kv = [(torch.randn(B, HKV, T, D, device=dev, generator=g).bfloat16(),
               torch.randn(B, HKV, T, D, device=dev, generator=g).bfloat16()) for _ in range(L)]
        for c in caches:
            for layer, (k, v) in enumerate(kv):
                c.append(shard.local_kv(k), shard.local_kv(v), layer)
        fused = SharedGather(shard, L, B, D, dev)
        dec_f = HeadParallelDecoder(caches[0], shard, fused=fused)
        dec_n = HeadParallelDecoder(caches[1], shard)
        worst = 0.0
        for step in range(3):
            for layer in range(L):
                q = torch.randn(B, HQ, 1, D, device=dev, generator=g).bfloat16()
                k = torch.randn(B, HKV, 1, D, device=dev, generator=g).bfloat16()
                v = torch.randn(B, HKV, 1, D, device=dev, generator=g).bfloat16()
                a = dec_f.decode(q, k, v, layer)
                b = dec_n.decode(q, k, v, layer)
                worst = max(worst, (a.float() - b.float()).abs().max().item())
        # one layer, back-to-back calls on the same counters
        one = SharedGather(shard, 1, B, D, dev)
        dec_1 = HeadParallelDecoder(caches[0], shard, fused=one)
        for step in range(4):
            q = torch.randn(B, HQ, 1, D, device=dev, generator=g).bfloat16()
            k = torch.randn(B, HKV, 1, D, device=dev, generator=g).bfloat16()
            v = torch.randn(B, HKV, 1, D, device=dev, generator=g).bfloat16()
            a = dec_1.decode(q, k, v, 0).clone()
            b = dec_n.decode(q, k, v, 0)
            worst = max(worst, (a.float() - b.float()).abs().max().item())
        torch.cuda.synchronize()
        status = caches[0].device_status() | caches[1].device_status()
        one.close()
        fused.close()
        result[rank] = (worst, status)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_gather_equals_nccl_all_gather():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        result = m.dict()
        mp.start_processes(_worker, args=(2, _free_port(), result), nprocs=2, join=True,
                           start_method="spawn")
        res = dict(result)
    for rank in range(2):
        worst, status = res[rank]
        assert status == 0
        assert worst == 0.0, (rank, worst)
