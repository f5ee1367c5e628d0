"""Benchmark: TurboQuant decode attention + append on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step"): one decode step of Mixtral-8x7B attention over a
packed TurboQuant KV cache — for each of 32 layers, append the new token's
K/V (B x Hkv vectors: norm, rotate, quantise, pack, QJL sketch) and run GQA
decode attention (Hq 32, Hkv 8, D 128) over 8192 cached tokens + the new one,
K 4-bit + 1-bit QJL residual, V 2-bit, bf16 in/out.  Synthetic seeded data:
K/V ~ N(0,1) with 1% of channels (2 of 128, fixed per head) scaled x8.

Multi-GPU (torchrun, one rank per GPU): KV heads are sharded over N ranks
(8/N heads per rank) and the global batch is 16*N sequences, so every rank
holds the same 128 (sequence, kv-head) streams as the 1-GPU run (weak
scaling).  Each layer's attention outputs are all-gathered inside the decode
itself (the merge kernel stores every output block into every rank's buffer
over NVLink); `--gather nccl` runs NCCL's all-gather after each layer
instead.  Before timing, one pass over all layers checks the fused gather
bitwise against NCCL's (`gather_exact`).

Extra keys of the same JSON line: `serving` (256 sequences x 4096 context,
K3+QJL/V3, KV heads split over the N ranks: strong scaling), `long_context`
(1 GPU: Qwen2.5-14B shapes, B1/B4 x 32K/128K, bit widths 2/3/4), `append`
(prefill append GB/s, 48 layers at 4 bits), `append_qjl` (the headline's
K4+QJL/V2 prefill append), `prefill_attention` (TFLOP/s) and `ragged_decode`
(continuous batching).

The JSON line's `value` is decode tokens/s over all ranks (global batch /
step time, max over ranks), timed on the device with CUDA events around K
CUDA-graph replays of the step.  Packed KV per step is 3.96 GB per rank,
far above L2 (126 MB), so no L2 flush is needed between steps.
"""
from __future__ import annotations

import argparse
import datetime
from dataclasses import dataclass, replace
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LAYERS, HQ, HKV, D, T_CTX, B_PER_GPU = 32, 32, 8, 128, 8192, 16
KEY_BITS, VALUE_BITS, QJL = 4, 2, True
APPEND_CFG = dict(layers=48, B=8, H=8, T=4096, D=128, bits=4)


@dataclass(frozen=True)
class Workload:
    """A decode-step workload: `batch` sequences per GPU (weak scaling) or in
    total (strong scaling, KV heads split over the GPUs)."""
    title: str
    layers: int
    hq: int
    hkv: int
    d: int
    t_ctx: int
    batch: int
    kb: int
    vb: int
    qjl: bool
    scaling: str
    data: str           # "outlier": N(0,1), 2 of 128 channels x8; "student-t": t(4)/sqrt(2)


WORKLOADS = {
    # the headline: Mixtral-8x7B attention shapes, B16 x 8192 context per GPU
    "mixtral": Workload("Mixtral-8x7B attention decode step", LAYERS, HQ, HKV, D, T_CTX,
                        B_PER_GPU, KEY_BITS, VALUE_BITS, QJL, "weak", "outlier"),
    # Qwen2.5-14B long context (GQA 5); --batch 1|4, --context 32768|131072, --bits 2|3|4
    "qwen-long": Workload("Qwen2.5-14B long-context decode step", 48, 40, 8, 128, 32768, 1,
                          3, 3, False, "weak", "student-t"),
    # 256 sequences x 4096 context of Mixtral, KV heads split over the GPUs
    "serving": Workload("Mixtral-8x7B head-sharded serving decode step", 32, 32, 8, 128, 4096,
                        256, 3, 3, True, "strong", "outlier"),
}


def _workload(args) -> Workload:
    w = WORKLOADS[args.workload]
    ch = {}
    if args.batch:
        ch["batch"] = args.batch
    if args.context:
        ch["t_ctx"] = args.context
    if args.bits:
        ch["kb"] = ch["vb"] = args.bits
    return replace(w, **ch) if ch else w


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _traffic_per_launch():
    """dram bytes per decode launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "decode_kernel_mixtral_b16_t8192.md")
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_launch:"):
                return int(float(line.split(":")[1]))
    except Exception:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        rows = [r.split(", ") for r in out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        loaded = [s for s in sm if s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------------------
def run_reference(args, rank, world):
    """--impl reference: the reference's CPU path on the host cores (rank 0)."""
    if rank != 0:
        return
    import torch
    from oracle import cpu_baseline as C
    C.use_all_host_threads()        # torchrun sets OMP_NUM_THREADS=1; the arm uses every core
    W = _workload(args)
    LAYERS, HQ, HKV, D, T_CTX, KEY_BITS, VALUE_BITS = (W.layers, W.hq, W.hkv, W.d, W.t_ctx,
                                                       W.kb, W.vb)
    B = W.batch * world if W.scaling == "weak" else W.batch
    kc, kb = C.codebook(D, KEY_BITS)
    vc, vb = C.codebook(D, VALUE_BITS)
    layer = C.RefLayer(B, HKV, D, T_CTX, KEY_BITS, VALUE_BITS, kc, kb, vc, vb)
    g = torch.Generator(device="cpu")
    g.manual_seed(0)
    q = torch.randn(B, HQ, 1, D, generator=g).to(torch.bfloat16)
    kv = [(torch.randn(B, HKV, 1, D, generator=g).to(torch.bfloat16),
           torch.randn(B, HKV, 1, D, generator=g).to(torch.bfloat16)) for _ in range(4)]
    for i in range(args.warmup):
        layer.decode_step(*kv[i % 4], q)
    t0 = time.perf_counter()
    for i in range(args.steps):
        layer.decode_step(*kv[i % 4], q)
    per_layer = (time.perf_counter() - t0) / args.steps
    step_s = per_layer * LAYERS
    value = B / step_s
    line = {
        "impl": "reference", "metric": "decode-attn tokens/s", "value": value,
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": W.scaling,
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": _config(W, world, args.gather),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": C.host_threads(),
                         "kind": "port",
                         "sample": f"1 of {LAYERS} layers per step timed, x{LAYERS}; "
                                   f"reference update()+SDPA, B{B} Hkv{HKV} T{T_CTX}, "
                                   "no QJL (the reference has none)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _config(W, world, gather="fused"):
    import math as _m
    B = W.batch * world if W.scaling == "weak" else W.batch
    bpt = W.d * (W.kb + W.vb) // 8 + 4 + ((W.d // 8 + 2) if W.qjl else 0)
    per_gpu = W.layers * B * (W.hkv // world) * W.t_ctx * bpt
    return {"workload": f"{W.title}: {W.layers} layers x (append 1 token + GQA decode), "
                        f"Hq{W.hq}/Hkv{W.hkv}, D{W.d}, context {W.t_ctx}, "
                        f"K{W.kb}{'+QJL' if W.qjl else ''}/V{W.vb}",
            "global_batch": B, "seq_len": W.t_ctx, "layers": W.layers,
            "q_heads": W.hq, "kv_heads": W.hkv, "head_dim": W.d, "key_bits": W.kb,
            "value_bits": W.vb, "qjl": W.qjl,
            "kv_data": ("N(0,1), 2 of 128 channels x8" if W.data == "outlier"
                        else "Student-t(4) / sqrt(2)"),
            "parallelism": f"kv-head shard x{world}" + (
                "" if world == 1 else " + NCCL all-gather" if gather == "nccl"
                else " + all-gather fused into the decode (peer NVLink stores)"),
            "l2": (f"no flush: {per_gpu / 1e9:.2f} GB packed KV per step per GPU > 126 MB L2"
                   if per_gpu > 4 * 126e6 else
                   f"{per_gpu / 1e6:.0f} MB packed KV per step per GPU over {W.layers} "
                   "layers read in order (each layer's pages evicted before reuse)")}


# ---------------------------------------------------------------------------
class DecodeRig:
    """One decode-step workload on this rank: the packed cache of the rank's
    KV heads for every layer, filled with `t_ctx` synthetic tokens, plus the
    step's inputs (q, the new K/V token) and outputs."""

    def __init__(self, W: Workload, rank: int, world: int, local_rank: int, extra_tokens: int,
                 gather: str = "fused"):
        import torch
        from bhaskera_col_b200.inference import TurboQuantKVCache, ops
        from bhaskera_col_b200.inference.head_parallel import HeadShard, SharedGather
        self.W, self.rank, self.world = W, rank, world
        dev = torch.device("cuda", local_rank)
        self.dev = dev
        self.shard = HeadShard(W.hq, W.hkv, rank, world)
        self.hkv, self.hq = self.shard.kv_heads, self.shard.q_heads
        self.B = W.batch * world if W.scaling == "weak" else W.batch
        self.S = self.B * self.hkv
        self.bpt = ops.page_bytes(W.d, W.kb, W.vb, W.qjl) // 64
        self.cache = TurboQuantKVCache(
            num_layers=W.layers, batch_size=self.B, num_heads=self.hkv, head_dim=W.d,
            key_bits=W.kb, value_bits=W.vb, residual_window=0, protected_layers=0,
            dtype=torch.bfloat16, device=dev, max_seq_len=W.t_ctx + 64 + extra_tokens, qjl=W.qjl)
        gen = torch.Generator(device=dev)
        gen.manual_seed(1234 + rank)
        out_ch = torch.randperm(W.d, generator=torch.Generator().manual_seed(7))[:2].to(dev)
        scale = torch.ones(W.d, device=dev)
        scale[out_ch] = 8.0
        student = torch.distributions.StudentT(torch.tensor(4.0, device=dev))
        torch.cuda.manual_seed(1234 + rank)

        def synth(shape):
            if W.data == "student-t":
                return (student.sample(shape) * (0.5 ** 0.5)).to(torch.bfloat16)
            return (torch.randn(shape, device=dev, generator=gen) * scale).to(torch.bfloat16)

        # four distinct chunks of synthetic K/V, appended round-robin: every
        # layer's pages are its own memory, so a step reads them all from HBM
        ch = min(2048, W.t_ctx)
        chunks = [(synth((self.B, self.hkv, ch, W.d)), synth((self.B, self.hkv, ch, W.d)))
                  for _ in range(4)]
        i = 0
        for layer in range(W.layers):
            for c0 in range(0, W.t_ctx, ch):
                n = min(ch, W.t_ctx - c0)
                k, v = chunks[i % 4]
                self.cache.append(k[:, :, :n], v[:, :, :n], layer)
                i += 1
        del chunks
        torch.cuda.synchronize()
        self.stores = self.cache._stores
        L = W.layers
        self.q = [synth((self.B, self.hq, 1, W.d)) for _ in range(min(L, 4))]
        self.k_new = [synth((self.B, self.hkv, 1, W.d)) for _ in range(min(L, 4))]
        self.v_new = [synth((self.B, self.hkv, 1, W.d)) for _ in range(min(L, 4))]
        self.o_loc = [torch.empty((self.B, self.hq, 1, W.d), dtype=torch.bfloat16, device=dev)
                      for _ in range(L)]
        self.fused = (SharedGather(self.shard, L, self.B, W.d, dev)
                      if world > 1 and gather == "fused" else None)
        self.o_all = (self.fused.out if self.fused is not None else
                      torch.empty((L, world * self.B, self.hq, 1, W.d), dtype=torch.bfloat16,
                                  device=dev))
        self.ws = ops.DecodeWorkspace()

    def inputs(self, layer):
        i = layer % len(self.q)
        return self.q[i], self.k_new[i], self.v_new[i]

    def step(self, phased_events=None):
        """One decode step over all layers (the new token stored at t_ctx)."""
        from bhaskera_col_b200 import _lib
        from bhaskera_col_b200.inference import ops
        T = self.W.t_ctx
        for layer in range(self.W.layers):
            st = self.stores[layer]
            q, k, v = self.inputs(layer)
            if phased_events is None and self.fused is not None:
                ops.decode_step(st.tables, st._pages, k, v, T, q,
                                out=self.fused.block_view(layer), workspace=self.ws,
                                gather=self.fused.args(layer))
                continue
            if phased_events is None:
                ops.decode_step(st.tables, st._pages, k, v, T, q, out=self.o_loc[layer],
                                workspace=self.ws)
            else:
                ops.append(st.tables, st._pages, k, v, T)
                ops.decode_attention(st.tables, st._pages, q, T + 1, out=self.o_loc[layer],
                                     workspace=self.ws, phases=_lib.PHASE_QPREP)
                e0, e1 = phased_events[layer]
                e0.record()
                ops.decode_attention(st.tables, st._pages, q, T + 1, out=self.o_loc[layer],
                                     workspace=self.ws, phases=_lib.PHASE_DECODE)
                e1.record()
                ops.decode_attention(st.tables, st._pages, q, T + 1, out=self.o_loc[layer],
                                     workspace=self.ws, phases=_lib.PHASE_MERGE)
            if self.world > 1:
                self.shard.gather(self.o_loc[layer], buf=self.o_all[layer], layer=layer)

    def check_gather(self):
        """Every layer once through the fused gather and once through NCCL's
        all_gather_into_tensor of the same per-rank outputs: the gathered
        buffers must be bitwise equal on every rank.  Returns (exact, status)."""
        import torch
        import torch.distributed as dist
        from bhaskera_col_b200.inference import ops
        T = self.W.t_ctx
        exact = True
        ref = torch.empty_like(self.o_all[0])
        for layer in range(self.W.layers):
            st = self.stores[layer]
            q, k, v = self.inputs(layer)
            ops.decode_step(st.tables, st._pages, k, v, T, q, out=self.fused.block_view(layer),
                            workspace=self.ws, gather=self.fused.args(layer))
            ops.decode_step(st.tables, st._pages, k, v, T, q, out=self.o_loc[layer],
                            workspace=self.ws)
            dist.all_gather_into_tensor(ref, self.o_loc[layer])
            exact &= bool(torch.equal(self.fused.gathered(layer), ref))
        flag = torch.tensor([1 if exact else 0], device=self.dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        status = self.ws.status()
        return bool(flag.item()), status

    def close(self):
        if self.fused is not None:
            self.fused.close()
            self.fused = None


def _max_over_ranks(ms, world, dev):
    if world == 1:
        return ms
    import torch
    import torch.distributed as dist
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world, local_rank):
    if world > 1:
        import torch.distributed as dist
        dist.barrier(device_ids=[local_rank])


def measure_decode(W: Workload, args, rank, world, local_rank, *, e2e=True, check_gather=False,
                   clocks=False):
    """Time one decode-step workload: K CUDA-graph replays of the whole step
    (CUDA events, max over ranks), the decode kernel alone (roofline pass),
    and optionally the end-to-end step through the public API with host
    buffers.  Every rank takes the same collective steps."""
    import torch
    rig = DecodeRig(W, rank, world, local_rank, args.steps + args.warmup + 8, args.gather)
    dev = rig.dev
    L, T = W.layers, W.t_ctx
    res = {}
    if check_gather and rig.fused is not None:
        res["gather_exact"], res["gather_check_status"] = rig.check_gather()

    for _ in range(max(1, args.warmup)):       # eager warm-up (attributes, workspace)
        rig.step()
    torch.cuda.synchronize()
    if rig.ws.status() != 0:
        raise RuntimeError("device status error after warm-up")

    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        rig.step()
    torch.cuda.current_stream(dev).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        rig.step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()

    sampler = None
    if clocks:
        phys = local_rank
        cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
        if cvd:
            try:
                phys = int(cvd.split(",")[local_rank])
            except ValueError:
                pass
        sampler = ClockSampler(phys)

    _barrier(world, local_rank)
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
        time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        graph.replay()
    ev1.record()
    torch.cuda.synchronize()
    res["clocks"] = sampler.stop() if sampler else None
    _barrier(world, local_rank)
    ms = _max_over_ranks(ev0.elapsed_time(ev1), world, dev)
    res["ms_step"] = ms / args.steps
    res["value"] = rig.B / (res["ms_step"] / 1e3)
    del graph

    # roofline pass: the decode kernel alone, timed with events on its stream
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(L)] for _ in range(args.steps)]
    torch.cuda.synchronize()
    torch.cuda._sleep(int(2e8))          # let the host queue the whole pass first
    for k in range(args.steps):
        # ~5 ms of device sleep per step keeps the host's launches ahead of the
        # GPU (with an all-gather per layer the host needs about as long per
        # layer as the GPU); otherwise an event can fire before the host has
        # queued the decode launch it brackets
        torch.cuda._sleep(int(1e7))
        rig.step(phased_events=evs[k])
    torch.cuda.synchronize()
    dec_ms = [e0.elapsed_time(e1) for row in evs for (e0, e1) in row]
    res["dec_avg_ms"] = sum(dec_ms) / len(dec_ms)
    res["alg_bytes"] = rig.S * (T + 1) * rig.bpt
    res["achieved_gbs"] = res["alg_bytes"] / (res["dec_avg_ms"] / 1e3) / 1e9
    res["packed_kv_gbs_per_gpu"] = L * res["alg_bytes"] / (res["ms_step"] / 1e3) / 1e9

    if e2e:
        res.update(_e2e(rig, args, rank, world, local_rank))
    res["status"] = rig.cache.device_status() | rig.ws.status()
    res["B"] = rig.B
    rig.close()
    del rig
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return res


def _e2e(rig, args, rank, world, local_rank):
    """The step through the public API (TurboQuantKVCache.decode, one call per
    layer, with the fused all-gather at N > 1) with host buffers: every step
    each rank copies its own heads' q / k / v in from pinned host memory (the
    per-rank slices a head-sharded model computes), and rank 0 reads the
    step's gathered outputs (all layers, all heads) back.  Copies run on their
    own stream, overlapped with the layers they do not feed."""
    import torch
    W, dev, L = rig.W, rig.dev, rig.W.layers
    qn, kn = rig.q[0].numel(), rig.k_new[0].numel()
    per = qn + 2 * kn
    in_h = torch.empty((L, per), dtype=torch.bfloat16).pin_memory()
    for layer in range(L):
        q, k, v = rig.inputs(layer)
        in_h[layer, :qn] = q.flatten().cpu()
        in_h[layer, qn:qn + kn] = k.flatten().cpu()
        in_h[layer, qn + kn:] = v.flatten().cpu()
    in_d = torch.empty((L, per), dtype=torch.bfloat16, device=dev)
    q_in = [in_d[l, :qn].view(rig.q[0].shape) for l in range(L)]
    k_in = [in_d[l, qn:qn + kn].view(rig.k_new[0].shape) for l in range(L)]
    v_in = [in_d[l, qn + kn:].view(rig.v_new[0].shape) for l in range(L)]
    reader = rank == 0
    o_h = torch.empty(rig.o_all.shape, dtype=torch.bfloat16).pin_memory() if reader else None
    main = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(dev)
    chunks = [(0, 1), (1, min(4, L)), (min(4, L), L)]
    ev_in = [torch.cuda.Event() for _ in chunks]
    # the gathered outputs come back in runs of layers as they finish, on the
    # copy stream, so the read-back overlaps the later layers' compute
    out_runs = [(a, min(a + 4, L)) for a in range(0, L, 4)]
    ev_out = [torch.cuda.Event() for _ in out_runs]
    cache, fused, shard = rig.cache, rig.fused, rig.shard

    def e2e_step():
        with torch.cuda.stream(copy_stream):
            for (a, b), ev in zip(chunks, ev_in):
                if b > a:
                    in_d[a:b].copy_(in_h[a:b], non_blocking=True)
                ev.record(copy_stream)
        for layer in range(L):
            for (a, _), ev in zip(chunks, ev_in):
                if layer == a:
                    main.wait_event(ev)
            if fused is not None:
                cache.decode(q_in[layer], k_in[layer], v_in[layer], layer,
                             out=fused.block_view(layer), gather=fused.args(layer))
            else:
                out = cache.decode(q_in[layer], k_in[layer], v_in[layer], layer,
                                   out=rig.o_loc[layer] if rig.world > 1 else rig.o_all[layer])
                if rig.world > 1:
                    shard.gather(out, buf=rig.o_all[layer], layer=layer)
            for (a, b), ev in zip(out_runs, ev_out):
                if layer == b - 1:
                    ev.record(main)
                    if reader:
                        with torch.cuda.stream(copy_stream):
                            copy_stream.wait_event(ev)
                            o_h[a:b].copy_(rig.o_all[a:b], non_blocking=True)
        copy_stream.synchronize()
        main.synchronize()

    T = W.t_ctx
    for st in rig.stores:      # the e2e leg appends for real: start from t_ctx tokens
        st._comp_ptr = T
    for _ in range(args.warmup):
        e2e_step()
    for st in rig.stores:
        st._comp_ptr = T
    _barrier(world, local_rank)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    _barrier(world, local_rank)
    ms = _max_over_ranks(e0.elapsed_time(e1), world, dev)
    return {"e2e_value": rig.B / (ms / args.steps / 1e3),
            "h2d_bytes_per_step": in_h.numel() * 2 * world,
            "d2h_bytes_per_step": rig.o_all.numel() * 2}


def run_ours(args, rank, world, local_rank):
    import torch
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    W = _workload(args)
    hbm_peak, peak_kind = _peaks()

    # ---- the headline workload ----------------------------------------------
    main = measure_decode(W, args, rank, world, local_rank, e2e=True,
                          check_gather=world > 1 and args.gather == "fused", clocks=True)

    # ---- config 5: head-sharded serving, strong scaling over the ranks ------
    serving = None
    if args.workload == "mixtral" and not args.skip_serving:
        SW = WORKLOADS["serving"]
        r = measure_decode(SW, args, rank, world, local_rank, e2e=True,
                           check_gather=world > 1 and args.gather == "fused")
        serving = _summary(SW, r, world, hbm_peak, args)

    # ---- config 3: long context (1 GPU) -------------------------------------
    long_ctx = None
    if args.workload == "mixtral" and world == 1 and not args.skip_long:
        long_ctx = []
        base = WORKLOADS["qwen-long"]
        for b, t, bits in LONG_CASES:
            LW = replace(base, batch=b, t_ctx=t, kb=bits, vb=bits)
            r = measure_decode(LW, args, rank, world, local_rank, e2e=False)
            long_ctx.append(_summary(LW, r, world, hbm_peak, args))

    append_line = append_qjl_line = prefill_line = ragged_line = None
    if rank == 0 and not args.skip_append and args.workload == "mixtral":
        append_line = bench_append(dev, args)
        append_qjl_line = bench_append_qjl(dev, args)
        prefill_line = bench_prefill(dev, args)
        ragged_line = bench_ragged(dev, args)

    cpu_line = None
    if rank == 0 and world == 1 and not args.skip_cpu and args.workload == "mixtral":
        from oracle import cpu_baseline as C
        C.use_all_host_threads()
        t_layer = C.time_decode(main["B"], W.hq, W.hkv, W.d, W.t_ctx, W.kb, W.vb, steps=2)
        cpu_line = {"value": main["B"] / (t_layer * W.layers), "unit": "tokens/s",
                    "cores": C.host_threads(), "kind": "port",
                    "sample": f"reference update()+SDPA, 1 of {W.layers} layers x 2 steps "
                              f"timed and scaled x{W.layers}; B{main['B']} Hkv{W.hkv} "
                              f"T{W.t_ctx}, no QJL"}

    if rank == 0:
        alg, dec_avg = main["alg_bytes"], main["dec_avg_ms"]
        line = {
            "metric": "decode-attn tokens/s", "value": main["value"], "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": main["ms_step"], "higher_is_better": True, "scaling": W.scaling,
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": _config(W, world, args.gather),
            "packed_kv_gbs_per_gpu": main["packed_kv_gbs_per_gpu"],
            "roofline": {"bound": "hbm", "achieved": main["achieved_gbs"], "peak": hbm_peak,
                         "unit": "GB/s", "frac": main["achieved_gbs"] / hbm_peak,
                         "traffic": _traffic_per_launch() if args.workload == "mixtral" else None,
                         "kernel": f"decode_kernel<{W.d},{W.kb},{W.vb},"
                                   f"{'qjl' if W.qjl else 'mse'}"
                                   f"{',self' if (W.d, W.kb) == (128, 4) and W.vb in (2, 4) else ''}>",
                         "algorithmic_bytes_per_launch": alg,
                         "avg_launch_ms": dec_avg, "peak_kind": peak_kind},
            "cpu_baseline": cpu_line,
            "e2e": {"value": main["e2e_value"], "unit": "tokens/s",
                    "h2d_bytes_per_step": main["h2d_bytes_per_step"],
                    "d2h_bytes_per_step": main["d2h_bytes_per_step"],
                    "path": "TurboQuantKVCache.decode per layer (fused store + attend"
                            + (", fused all-gather" if world > 1 else "") + "); each rank "
                            "copies its heads' q/k/v in from pinned host memory, rank 0 "
                            "reads the gathered outputs back (byte counts: all ranks)"},
            "gpu_launches": args.steps * W.layers * 3,
            "clocks": main["clocks"],
            "gather_exact": main.get("gather_exact"),
            "serving": serving,
            "long_context": long_ctx,
            "append": append_line,
            "append_qjl": append_qjl_line,
            "prefill_attention": prefill_line,
            "ragged_decode": ragged_line,
            "device_status": main["status"] | main.get("gather_check_status", 0),
        }
        print(json.dumps(line), flush=True)


LONG_CASES = [(1, 32768, 2), (1, 32768, 3), (1, 32768, 4), (4, 32768, 3), (1, 131072, 3),
              (4, 131072, 3)]


def _summary(W, r, world, hbm_peak, args):
    """An extra workload's key in the JSON line."""
    out = {"workload": _config(W, world, args.gather)["workload"],
           "scaling": W.scaling, "global_batch": r["B"], "n_gpus": world,
           "tokens_per_s": r["value"], "ms_per_step": r["ms_step"],
           "packed_kv_gbs_per_gpu": r["packed_kv_gbs_per_gpu"],
           "decode_kernel": {"avg_launch_ms": r["dec_avg_ms"], "achieved_gbs": r["achieved_gbs"],
                             "frac_of_hbm": r["achieved_gbs"] / hbm_peak,
                             "algorithmic_bytes_per_launch": r["alg_bytes"]},
           "device_status": r["status"] | r.get("gather_check_status", 0)}
    if "e2e_value" in r:
        out["e2e"] = {"tokens_per_s": r["e2e_value"],
                      "h2d_bytes_per_step": r["h2d_bytes_per_step"],
                      "d2h_bytes_per_step": r["d2h_bytes_per_step"]}
    if "gather_exact" in r:
        out["gather_exact"] = r["gather_exact"]
    return out


def bench_append(dev, args):
    """Prefill append GB/s: 48 layers x (B8 x Hkv8 x 4096 tokens x D128) bf16,
    K and V at 4 bits: 512 B read + 132 B written per token-head."""
    import torch
    from bhaskera_col_b200.inference import ops
    from bhaskera_col_b200.inference.kv_cache import (FastLloydMaxCodebook,
                                                      _generate_rotation_matrix)
    c = APPEND_CFG
    L, B, H, T, Dd, bits = c["layers"], c["B"], c["H"], c["T"], c["D"], c["bits"]
    cb = FastLloydMaxCodebook.get(Dd, bits, dev)
    tables = [ops.LayerTables(Dd, bits, bits, False, cb.centroids, cb.boundaries,
                              cb.centroids, cb.boundaries,
                              _generate_rotation_matrix(Dd, 42 + 13 * i, dev).contiguous())
              for i in range(L)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    sc = torch.exp(torch.empty(Dd, device=dev).uniform_(math.log(0.1), math.log(10.0),
                                                        generator=gen))
    xs = [((torch.randn((B, H, T, Dd), device=dev, generator=gen) * sc).to(torch.bfloat16),
           (torch.randn((B, H, T, Dd), device=dev, generator=gen) * sc).to(torch.bfloat16))
          for _ in range(4)]
    pb = ops.page_bytes(Dd, bits, bits, False)
    pages = [torch.zeros((B * H, T // 64, pb), dtype=torch.uint8, device=dev) for _ in range(L)]

    def run():
        for i in range(L):
            k, v = xs[i % 4]
            ops.append(tables[i], pages[i], k, v, 0)

    run()
    torch.cuda.synchronize()
    reps = max(1, min(args.steps, 3))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    th = L * B * H * T
    alg = th * (2 * Dd * 2 + 2 * (Dd * bits // 8 + 2))
    return {"workload": f"prefill append {L} layers x B{B} x Hkv{H} x {T} tokens, D{Dd}, "
                        f"K{bits}/V{bits}, bf16 in", "ms": ms, "gbs": alg / (ms / 1e3) / 1e9,
            "token_heads_per_s": th / (ms / 1e3), "algorithmic_bytes": alg}


def bench_append_qjl(dev, args):
    """Prefill append of the headline configuration (Mixtral attention shapes:
    B16 x Hkv8 x 8192 tokens x D128, K 4-bit + 1-bit QJL sketch, V 2-bit),
    bf16 K/V in: 512 B read + 118 B written per token-head.  Four layers' page
    sets written in turn (distinct memory; the 537 MB input exceeds L2)."""
    import torch
    from bhaskera_col_b200.inference import ops
    from bhaskera_col_b200.inference.kv_cache import (FastLloydMaxCodebook, _generate_qjl_matrix,
                                                      _generate_rotation_matrix)
    L, B, H, T, Dd, kb, vb = 4, 16, 8, 8192, 128, 4, 2
    kc, vc = FastLloydMaxCodebook.get(Dd, kb, dev), FastLloydMaxCodebook.get(Dd, vb, dev)
    tables = [ops.LayerTables(Dd, kb, vb, True, kc.centroids, kc.boundaries, vc.centroids,
                              vc.boundaries,
                              _generate_rotation_matrix(Dd, 42 + 13 * i, dev).contiguous(),
                              _generate_qjl_matrix(Dd, 42 + 13 * i, dev).contiguous())
              for i in range(L)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(17)
    sc = torch.ones(Dd, device=dev)
    sc[torch.randperm(Dd, generator=torch.Generator().manual_seed(7))[:2].to(dev)] = 8.0
    k = (torch.randn((B, H, T, Dd), device=dev, generator=gen) * sc).to(torch.bfloat16)
    v = (torch.randn((B, H, T, Dd), device=dev, generator=gen) * sc).to(torch.bfloat16)
    pb = ops.page_bytes(Dd, kb, vb, True)
    pages = [torch.zeros((B * H, T // 64, pb), dtype=torch.uint8, device=dev) for _ in range(L)]

    def run():
        for i in range(L):
            ops.append(tables[i], pages[i], k, v, 0)

    run()
    torch.cuda.synchronize()
    reps = max(1, min(args.steps, 3))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps / L
    th = B * H * T
    alg = th * (2 * Dd * 2 + pb // 64)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["hbm_gbs"])
    except Exception:
        peak = 6650.0
    gbs = alg / (ms / 1e3) / 1e9
    return {"workload": f"prefill append of one layer: B{B} x Hkv{H} x {T} tokens, D{Dd}, "
                        f"K{kb}+QJL/V{vb}, bf16 in (average over {L} layers' page sets)",
            "ms_per_layer": ms, "gbs": gbs, "frac_of_hbm": gbs / peak,
            "token_heads_per_s": th / (ms / 1e3), "algorithmic_bytes_per_layer": alg,
            "tensor_cores": ops.append_uses_tensor_cores(tables[0], k, v),
            "device_status": ops.device_status(dev)}


def bench_prefill(dev, args):
    """Prefill attention over the packed cache: one layer of B8 x Hq32/Hkv8 x
    4096 tokens, D128, K4/V4, causal (4 * B * Hq * T^2/2 * D flops)."""
    import torch
    from bhaskera_col_b200.inference import ops
    from bhaskera_col_b200.inference.kv_cache import (FastLloydMaxCodebook,
                                                      _generate_rotation_matrix)
    c = APPEND_CFG
    B, H, T, Dd, bits, g = c["B"], c["H"], c["T"], c["D"], c["bits"], 4
    cb = FastLloydMaxCodebook.get(Dd, bits, dev)
    t = ops.LayerTables(Dd, bits, bits, False, cb.centroids, cb.boundaries, cb.centroids,
                        cb.boundaries, _generate_rotation_matrix(Dd, 42, dev).contiguous())
    gen = torch.Generator(device=dev)
    gen.manual_seed(77)
    pages = torch.zeros((B * H, T // 64, ops.page_bytes(Dd, bits, bits, False)),
                        dtype=torch.uint8, device=dev)
    k = torch.randn((B, H, T, Dd), device=dev, generator=gen).to(torch.bfloat16)
    ops.append(t, pages, k, k, 0)
    q = torch.randn((B, H * g, T, Dd), device=dev, generator=gen).to(torch.bfloat16)
    out = torch.empty_like(q)
    flops = 4.0 * B * H * g * (T * T / 2) * Dd
    reps = max(2, min(args.steps, 5))

    def timed(engine):
        for _ in range(2):
            ops.prefill_attention(t, pages, q, T, out=out, engine=engine)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            ops.prefill_attention(t, pages, q, T, out=out, engine=engine)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    ms_cc = timed(1)                 # the mma.sync kernel, for comparison
    ms = timed(0)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        peak = 1590.0
    tc = ops.prefill_uses_tensor_cores(t)
    return {"workload": f"prefill attention over the packed cache, 1 layer: B{B} x Hq{H * g}/Hkv{H} "
                        f"x {T} tokens causal, D{Dd}, K{bits}/V{bits}", "ms": ms,
            "tflops": flops / (ms / 1e3) / 1e12, "frac_of_bf16_peak": flops / (ms / 1e3) / 1e12 / peak,
            "kernel": ("prefill_tc_kernel (tcgen05.mma, S/P and O in tensor memory)" if tc
                       else "prefill_kernel (mma.sync m16n8k16 fp16)"),
            "mma_sync_kernel_ms": ms_cc}


def bench_ragged(dev, args):
    """Continuous-batching decode step, vLLM-shaped: one layer (Hq32/Hkv8,
    D128, K4/V2 without QJL, as the reference's vLLM compressor), 64 requests
    whose context lengths are log-uniform in [256, 16384] (seeded), pages in a
    shuffled block-table pool, per-request lengths on the device: one
    tq_decode_step (store + attend).  Against it, the same batch padded to its
    longest request on contiguous pages (what a caller without per-request
    lengths runs).  Bytes = the requests' real packed tokens."""
    import numpy as np
    import torch
    from bhaskera_col_b200.inference import ops
    from bhaskera_col_b200.inference.kv_cache import (FastLloydMaxCodebook,
                                                      _generate_rotation_matrix)
    R, H, g, Dd, kb, vb, T = 64, 8, 4, 128, 4, 2, 16384
    rng = np.random.default_rng(11)
    lens = np.exp(rng.uniform(math.log(256), math.log(T), R)).astype(np.int64)
    lens[0] = T
    kc, vc = FastLloydMaxCodebook.get(Dd, kb, dev), FastLloydMaxCodebook.get(Dd, vb, dev)
    t = ops.LayerTables(Dd, kb, vb, False, kc.centroids, kc.boundaries, vc.centroids,
                        vc.boundaries, _generate_rotation_matrix(Dd, 42, dev).contiguous())
    pb = ops.page_bytes(Dd, kb, vb, False)
    P = T // 64
    cont = torch.zeros((R * H, P, pb), dtype=torch.uint8, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    for r0 in range(0, R, 8):
        k = torch.randn((8, H, T, Dd), device=dev, generator=gen).to(torch.bfloat16)
        ops.append(t, cont[r0 * H:(r0 + 8) * H], k, k, 0)
        del k
    perm = torch.randperm(R * H * P, device=dev, generator=gen)
    pool = torch.empty((R * H * P, pb), dtype=torch.uint8, device=dev)
    pool[perm] = cont.view(R * H * P, pb)
    paged = ops.PagedPages(pool, perm.view(R * H, P).to(torch.int32))
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    q = torch.randn((R, H * g, 1, Dd), device=dev, generator=gen).to(torch.bfloat16)
    kn = torch.randn((R, H, 1, Dd), device=dev, generator=gen).to(torch.bfloat16)
    out = torch.empty_like(q)
    ws = ops.DecodeWorkspace()
    reps = max(5, min(args.steps, 20))

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    ms = timed(lambda: ops.decode_step(t, paged, kn, kn, T - 1, q, out=out, workspace=ws,
                                       seq_lens=sl))
    ms_pad = timed(lambda: ops.decode_step(t, cont, kn, kn, T - 1, q, out=out, workspace=ws))
    status = ws.status()
    alg = int(lens.sum()) * H * (pb // 64)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["hbm_gbs"])
    except Exception:
        peak = 6650.0
    gbs = alg / (ms / 1e3) / 1e9
    return {"workload": f"continuous-batching decode step, 1 layer: {R} requests, context "
                        f"log-uniform 256..{T} (sum {int(lens.sum())}), Hq32/Hkv8, D128, "
                        f"K{kb}/V{vb}, block-table pool", "ms": ms, "gbs": gbs,
            "frac_of_hbm": gbs / peak, "tokens_per_s": R / (ms / 1e3),
            "padded_to_longest_ms": ms_pad, "speedup_vs_padded": ms_pad / ms,
            "algorithmic_bytes": alg, "device_status": status,
            "l2": "no flush: %.0f MB of packed KV per step > 126 MB L2" % (alg / 1e6)}


def run_profile(args):
    """Small single-GPU cases for ncu captures (no JSON line):
    --profile decode : one Mixtral layer (B16 Hkv8 T8192, K4+QJL/V2), 4 decode calls
    --profile append : one prefill-append layer (B8 Hkv8 T4096 D128 4-bit), 4 calls
    --profile step   : one layer's fused decode step (tq_decode_step), 4 calls
    --profile append_qjl : K4+QJL/V2 prefill append, B4 x Hkv8 x 8192 tokens, 4 calls
    --profile prefill    : prefill attention, B2 x Hq32/Hkv8 x 2048 tokens, 3 calls
    --profile step_long  : one Qwen2.5-14B long-context layer's decode step (B1, Hq40/Hkv8,
                           32768 tokens, K3/V3), 4 calls
    """
    import torch
    from bhaskera_col_b200.inference import TurboQuantKVCache, ops
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    if args.profile == "prefill":
        c = APPEND_CFG
        from bhaskera_col_b200.inference.kv_cache import FastLloydMaxCodebook
        cb = FastLloydMaxCodebook.get(c["D"], c["bits"], dev)
        from bhaskera_col_b200.inference.kv_cache import _generate_rotation_matrix
        t = ops.LayerTables(c["D"], c["bits"], c["bits"], False, cb.centroids, cb.boundaries,
                            cb.centroids, cb.boundaries,
                            _generate_rotation_matrix(c["D"], 42, dev).contiguous())
        Bp, Tp = 2, 2048          # a smaller case of the same kernel for ncu
        pages = torch.zeros((Bp * c["H"], Tp // 64, ops.page_bytes(c["D"], c["bits"], c["bits"], False)),
                            dtype=torch.uint8, device=dev)
        k = torch.randn((Bp, c["H"], Tp, c["D"]), device=dev, generator=gen).to(torch.bfloat16)
        ops.append(t, pages, k, k, 0)
        q = torch.randn((Bp, 4 * c["H"], Tp, c["D"]), device=dev, generator=gen).to(torch.bfloat16)
        for _ in range(3):
            ops.prefill_attention(t, pages, q, Tp)
        torch.cuda.synchronize()
        return
    if args.profile == "append_qjl":
        # one layer's K4+QJL/V2 prefill append, a quarter of the headline's
        # streams (B4 x Hkv8 x 8192 tokens; 134 MB of bf16 input > L2)
        from bhaskera_col_b200.inference.kv_cache import (FastLloydMaxCodebook,
                                                          _generate_qjl_matrix,
                                                          _generate_rotation_matrix)
        Bp, Hp, Tp, Dp = 4, 8, 8192, 128
        kc, vc = FastLloydMaxCodebook.get(Dp, 4, dev), FastLloydMaxCodebook.get(Dp, 2, dev)
        t = ops.LayerTables(Dp, 4, 2, True, kc.centroids, kc.boundaries, vc.centroids,
                            vc.boundaries, _generate_rotation_matrix(Dp, 42, dev).contiguous(),
                            _generate_qjl_matrix(Dp, 42, dev).contiguous())
        k = torch.randn((Bp, Hp, Tp, Dp), device=dev, generator=gen).to(torch.bfloat16)
        pages = torch.zeros((Bp * Hp, Tp // 64, ops.page_bytes(Dp, 4, 2, True)),
                            dtype=torch.uint8, device=dev)
        for _ in range(4):
            ops.append(t, pages, k, k, 0)
        torch.cuda.synchronize()
        if ops.device_status(dev) != 0:
            raise RuntimeError("device status error")
        return
    if args.profile == "append":
        c = APPEND_CFG
        cache = TurboQuantKVCache(num_layers=1, batch_size=c["B"], num_heads=c["H"],
                                  head_dim=c["D"], key_bits=c["bits"], value_bits=c["bits"],
                                  residual_window=0, protected_layers=0, device=dev,
                                  max_seq_len=c["T"])
        x = torch.randn((c["B"], c["H"], c["T"], c["D"]), device=dev,
                        generator=gen).to(torch.bfloat16)
        st = cache._stores[0]
        st._lazy_alloc(c["B"], c["H"])
        for _ in range(4):
            ops.append(st.tables, st._pages, x, x, 0)
        torch.cuda.synchronize()
        return
    if args.profile == "step_long":
        Tl, Bl, Hql = 32768, 1, 40
        cache = TurboQuantKVCache(num_layers=1, batch_size=Bl, num_heads=HKV, head_dim=D,
                                  key_bits=3, value_bits=3, residual_window=0,
                                  protected_layers=0, device=dev, max_seq_len=Tl + 64)
        for c0 in range(0, Tl, 8192):
            k = torch.randn((Bl, HKV, 8192, D), device=dev, generator=gen).to(torch.bfloat16)
            cache.append(k, k, 0)
        q = torch.randn((Bl, Hql, 1, D), device=dev, generator=gen).to(torch.bfloat16)
        k1 = torch.randn((Bl, HKV, 1, D), device=dev, generator=gen).to(torch.bfloat16)
        st = cache._stores[0]
        for _ in range(4):
            ops.decode_step(st.tables, st._pages, k1, k1, Tl, q, workspace=st.workspace)
        torch.cuda.synchronize()
        if st.workspace.status() != 0:
            raise RuntimeError("device status error")
        return
    cache = TurboQuantKVCache(num_layers=1, batch_size=B_PER_GPU, num_heads=HKV, head_dim=D,
                              key_bits=KEY_BITS, value_bits=VALUE_BITS, residual_window=0,
                              protected_layers=0, device=dev, max_seq_len=T_CTX + 64, qjl=QJL)
    for c0 in range(0, T_CTX, 2048):
        k = torch.randn((B_PER_GPU, HKV, 2048, D), device=dev, generator=gen).to(torch.bfloat16)
        cache.append(k, k, 0)
    q = torch.randn((B_PER_GPU, HQ, 1, D), device=dev, generator=gen).to(torch.bfloat16)
    k1 = torch.randn((B_PER_GPU, HKV, 1, D), device=dev, generator=gen).to(torch.bfloat16)
    st = cache._stores[0]
    for _ in range(4):
        if args.profile == "step":
            ops.decode_step(st.tables, st._pages, k1, k1, T_CTX, q, workspace=st.workspace)
        else:
            ops.decode_attention(st.tables, st._pages, q, T_CTX + 1, workspace=st.workspace)
    torch.cuda.synchronize()
    if st.workspace.status() != 0:
        raise RuntimeError("device status error")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-append", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-serving", action="store_true",
                    help="leave out the 256-sequence head-sharded serving workload")
    ap.add_argument("--skip-long", action="store_true",
                    help="leave out the long-context cases (1 GPU)")
    ap.add_argument("--profile", choices=["decode", "append", "append_qjl", "step", "prefill",
                                          "step_long"],
                    default=None,
                    help="run a small single-layer case for ncu and exit")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="mixtral",
                    help="decode-step workload (default: the Mixtral headline)")
    ap.add_argument("--batch", type=int, default=0, help="override the workload's batch")
    ap.add_argument("--context", type=int, default=0, help="override the context length")
    ap.add_argument("--bits", type=int, default=0, help="override K and V bit widths")
    ap.add_argument("--gather", choices=["fused", "nccl"], default="fused",
                    help="multi-GPU output all-gather: fused into the decode (peer stores) "
                         "or NCCL after it")
    args = ap.parse_args()
    if args.profile:
        run_profile(args)
        return
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", args.gpus))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if world != args.gpus and "WORLD_SIZE" in os.environ:
        args.gpus = world
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch.distributed as dist
    if world > 1:
        import torch
        torch.cuda.set_device(local_rank)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
