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
scaling); each layer ends with an NCCL all-gather of the attention outputs.

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
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from bhaskera_col_b200 import _lib
    from bhaskera_col_b200.inference import TurboQuantKVCache, ops
    from bhaskera_col_b200.inference.head_parallel import (HeadParallelDecoder, HeadShard,
                                                           SharedGather)

    W = _workload(args)
    LAYERS, HQ, HKV, D, T_CTX, KEY_BITS, VALUE_BITS, QJL = (W.layers, W.hq, W.hkv, W.d, W.t_ctx,
                                                            W.kb, W.vb, W.qjl)
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    shard = HeadShard(HQ, HKV, rank, world)
    hkv = shard.kv_heads
    hq = shard.q_heads
    B = W.batch * world if W.scaling == "weak" else W.batch
    S = B * hkv
    bpt = ops.page_bytes(D, KEY_BITS, VALUE_BITS, QJL) // 64

    # ---- cache: 32 layers, filled with T_CTX synthetic tokens -------------
    cache = TurboQuantKVCache(num_layers=LAYERS, batch_size=B, num_heads=hkv, head_dim=D,
                              key_bits=KEY_BITS, value_bits=VALUE_BITS, residual_window=0,
                              protected_layers=0, dtype=torch.bfloat16, device=dev,
                              max_seq_len=T_CTX + 64 + args.steps + args.warmup, qjl=QJL)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    out_ch = torch.randperm(D, generator=torch.Generator().manual_seed(7))[:2].to(dev)
    scale = torch.ones(D, device=dev)
    scale[out_ch] = 8.0

    student = torch.distributions.StudentT(torch.tensor(4.0, device=dev))
    torch.cuda.manual_seed(1234 + rank)

    def synth(shape):
        if W.data == "student-t":
            return (student.sample(shape) * (0.5 ** 0.5)).to(torch.bfloat16)
        return (torch.randn(shape, device=dev, generator=gen) * scale).to(torch.bfloat16)

    CH = 2048
    for layer in range(LAYERS):
        for c0 in range(0, T_CTX, CH):
            cache.append(synth((B, hkv, CH, D)), synth((B, hkv, CH, D)), layer)
    torch.cuda.synchronize()

    stores = cache._stores
    q_dev = [synth((B, hq, 1, D)) for _ in range(LAYERS)]
    k_new = [synth((B, hkv, 1, D)) for _ in range(LAYERS)]
    v_new = [synth((B, hkv, 1, D)) for _ in range(LAYERS)]
    o_loc = [torch.empty((B, hq, 1, D), dtype=torch.bfloat16, device=dev) for _ in range(LAYERS)]
    # the gathered outputs: for world > 1 by default in peer-mapped buffers
    # that the decode itself fills (fused all-gather), else NCCL into o_all
    fused = (SharedGather(shard, LAYERS, B, D, dev)
             if world > 1 and args.gather == "fused" else None)
    o_all = (fused.out if fused is not None else
             torch.empty((LAYERS, world * B, hq, 1, D), dtype=torch.bfloat16, device=dev))
    ws = ops.DecodeWorkspace()
    n_tok = T_CTX + 1

    def step(phased_events=None):
        for layer in range(LAYERS):
            st = stores[layer]
            if phased_events is None and fused is not None:
                ops.decode_step(st.tables, st._pages, k_new[layer], v_new[layer], T_CTX,
                                q_dev[layer], out=fused.block_view(layer), workspace=ws,
                                gather=fused.args(layer))
                continue
            if phased_events is None:
                ops.decode_step(st.tables, st._pages, k_new[layer], v_new[layer], T_CTX,
                                q_dev[layer], out=o_loc[layer], workspace=ws)
            else:
                ops.append(st.tables, st._pages, k_new[layer], v_new[layer], T_CTX)
                ops.decode_attention(st.tables, st._pages, q_dev[layer], n_tok,
                                     out=o_loc[layer], workspace=ws,
                                     phases=_lib.PHASE_QPREP)
                e0, e1 = phased_events[layer]
                e0.record()
                ops.decode_attention(st.tables, st._pages, q_dev[layer], n_tok,
                                     out=o_loc[layer], workspace=ws,
                                     phases=_lib.PHASE_DECODE)
                e1.record()
                ops.decode_attention(st.tables, st._pages, q_dev[layer], n_tok,
                                     out=o_loc[layer], workspace=ws,
                                     phases=_lib.PHASE_MERGE)
            if world > 1:
                shard.gather(o_loc[layer], buf=o_all[layer], layer=layer)

    # eager warm-up (sets kernel attributes, sizes the workspace)
    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize()
    if ws.status() != 0:
        raise RuntimeError("device status error after warm-up")

    # ---- CUDA graph of one step -------------------------------------------
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream(dev).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    phys = local_rank
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
    if cvd:
        try:
            phys = int(cvd.split(",")[local_rank])
        except ValueError:
            pass
    sampler = ClockSampler(phys)

    # ---- timed region: K graph replays --------------------------------------
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        graph.replay()
    ev1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    barrier()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = B / (ms_step / 1e3)

    # ---- roofline pass: decode kernel timed alone with events ---------------
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(LAYERS)] for _ in range(args.steps)]
    torch.cuda.synchronize()
    torch.cuda._sleep(int(2e8))          # let the host queue the whole pass first
    for k in range(args.steps):
        step(phased_events=evs[k])
    torch.cuda.synchronize()
    dec_ms = [e0.elapsed_time(e1) for row in evs for (e0, e1) in row]
    dec_avg = sum(dec_ms) / len(dec_ms)
    alg_bytes = S * n_tok * bpt
    hbm_peak, peak_kind = _peaks()
    achieved = alg_bytes / (dec_avg / 1e3) / 1e9

    # ---- e2e through the public API with host buffers -----------------------
    # each rank receives the full step inputs (all heads) from the host, keeps
    # its own heads, and reads back the gathered (B, Hq, 1, D) output
    full_q = [torch.cat([q] * world, 1) for q in q_dev[:4]]
    full_k = [torch.cat([k] * world, 1) for k in k_new[:4]]
    full_v = [torch.cat([v] * world, 1) for v in v_new[:4]]
    # every step copies all 32 layers' q/k/v from one pinned host buffer (in
    # three chunks: layer 0, layers 1-3, the rest, so layer 0 starts after a
    # 200 KB copy and later chunks land while earlier layers compute) and reads
    # all 32 gathered outputs back (layers 0-30 behind the last layer's
    # compute, then layer 31); copies run on their own stream
    qn, kn = full_q[0].numel(), full_k[0].numel()
    per = qn + 2 * kn
    in_h = torch.empty((LAYERS, per), dtype=torch.bfloat16).pin_memory()
    for layer in range(LAYERS):
        in_h[layer, :qn] = full_q[layer % 4].flatten().cpu()
        in_h[layer, qn:qn + kn] = full_k[layer % 4].flatten().cpu()
        in_h[layer, qn + kn:] = full_v[layer % 4].flatten().cpu()
    in_d = torch.empty((LAYERS, per), dtype=torch.bfloat16, device=dev)
    q_in = [in_d[l, :qn].view(full_q[0].shape) for l in range(LAYERS)]
    k_in = [in_d[l, qn:qn + kn].view(full_k[0].shape) for l in range(LAYERS)]
    v_in = [in_d[l, qn + kn:].view(full_v[0].shape) for l in range(LAYERS)]
    o_h = torch.empty(o_all.shape, dtype=torch.bfloat16).pin_memory()
    h2d = in_h.numel() * 2
    d2h = o_h.numel() * 2
    decoder = HeadParallelDecoder(cache, shard, fused=fused)
    main = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(dev)
    chunks = [(0, 1), (1, min(4, LAYERS)), (min(4, LAYERS), LAYERS)]
    ev_in = [torch.cuda.Event() for _ in chunks]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_step():
        with torch.cuda.stream(copy_stream):
            for (a, b), ev in zip(chunks, ev_in):
                if b > a:
                    in_d[a:b].copy_(in_h[a:b], non_blocking=True)
                ev.record(copy_stream)
        for layer in range(LAYERS):
            for (a, _), ev in zip(chunks, ev_in):
                if layer == a:
                    main.wait_event(ev)
            decoder.decode(q_in[layer], k_in[layer], v_in[layer], layer, buf=o_all[layer])
            if layer == LAYERS - 2:
                ev_out[0].record(main)
        ev_out[1].record(main)
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(ev_out[0])
            o_h[:LAYERS - 1].copy_(o_all[:LAYERS - 1], non_blocking=True)
            copy_stream.wait_event(ev_out[1])
            o_h[LAYERS - 1:].copy_(o_all[LAYERS - 1:], non_blocking=True)
        copy_stream.synchronize()
        main.synchronize()

    for st in stores:      # the e2e leg appends for real: start from T_CTX tokens
        st._comp_ptr = T_CTX
    for _ in range(args.warmup):
        e2e_step()
    for st in stores:
        st._comp_ptr = T_CTX
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_val = B / (e2e_ms / args.steps / 1e3)
    status = cache.device_status() | ws.status()
    del graph
    if fused is not None:
        fused.close()

    # ---- prefill append throughput (48 layers x B8 x Hkv8 x 4096, 4-bit) ----
    append_line = None
    prefill_line = None
    ragged_line = None
    if rank == 0 and not args.skip_append and args.workload == "mixtral":
        append_line = bench_append(dev, args)
        prefill_line = bench_prefill(dev, args)
        ragged_line = bench_ragged(dev, args)

    cpu_line = None
    if rank == 0 and world == 1 and not args.skip_cpu and args.workload == "mixtral":
        from oracle import cpu_baseline as C
        t_layer = C.time_decode(B, HQ, HKV, D, T_CTX, KEY_BITS, VALUE_BITS, steps=2)
        cpu_line = {"value": B / (t_layer * LAYERS), "unit": "tokens/s",
                    "cores": C.host_threads(), "kind": "port",
                    "sample": f"reference update()+SDPA, 1 of {LAYERS} layers x 2 steps "
                              f"timed and scaled x{LAYERS}; B{B} Hkv{HKV} T{T_CTX}, no QJL"}

    if rank == 0:
        line = {
            "metric": "decode-attn tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": W.scaling,
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": _config(W, world, args.gather),
            "packed_kv_gbs_per_gpu": LAYERS * alg_bytes / (ms_step / 1e3) / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak,
                         "unit": "GB/s", "frac": achieved / hbm_peak,
                         "traffic": _traffic_per_launch() if args.workload == "mixtral" else None,
                         "kernel": f"decode_kernel<{D},{KEY_BITS},{VALUE_BITS},"
                                   f"{'qjl' if QJL else 'mse'}>",
                         "algorithmic_bytes_per_launch": alg_bytes,
                         "avg_launch_ms": dec_avg, "peak_kind": peak_kind},
            "cpu_baseline": cpu_line,
            "e2e": {"value": e2e_val, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "path": "TurboQuantKVCache.decode per layer (fused store + attend), "
                            "pinned host q/k/v in, output out"},
            "gpu_launches": args.steps * LAYERS * 3,
            "clocks": clocks,
            "append": append_line,
            "prefill_attention": prefill_line,
            "ragged_decode": ragged_line,
            "device_status": status,
        }
        print(json.dumps(line), flush=True)


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
    ap.add_argument("--profile", choices=["decode", "append", "step", "prefill"], default=None,
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
