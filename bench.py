#!/usr/bin/env python
"""bench.py — decode attention KV GB/s on BASELINE config 2.

Workload (per rank, weak scaling): Llama-3-8B-shaped batched GQA decode,
B = 32 sequences, 32 query / 8 KV heads, head_dim 128, fp16 KV cache, one new
token per sequence, KV lengths ~ U[512, 8192] from a per-rank seed, Q/K/V
~ N(0, 1). The KV bytes (~570 MB per rank) exceed the 126 MB L2, so no flush
is needed between steps.

  value    device-resident: the decode attention call (split-KV kernel +
           combine) on inputs already in HBM, CUDA events on its stream.
  e2e      the same metric through the host-buffer C-ABI call
           aspida_attn_step_host: H2D of q/k/v/pos from pinned memory, RoPE
           + K/V append, decode, D2H of the output, every step.
  roofline algorithmic bytes per call / average call time vs the measured HBM
           copy bandwidth (MEASURED_PEAKS.json).
  cpu_baseline  the CPU oracle (C++ restatement of the reference's Ada loops)
           on the box's host cores, rank 0 at N=1.

--impl reference times that CPU implementation as the reference arm.
Launch: python bench.py [--gpus N --steps K --warmup W]; for N > 1 under
torch.distributed.run (one rank per GPU, NCCL).
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

NQ, NKV, HD, B = 32, 8, 128, 32
LEN_LO, LEN_HI = 512, 8192
METRIC = "decode attn KV GB/s (cfg2: Llama-3-8B GQA decode B32, 32/8 heads, hd128, fp16 KV)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="for ncu: only warm-up + timed steps of one leg, no clock soak, e2e or CPU")
    ap.add_argument("--profile-leg", choices=["decode", "prefill", "long", "q8", "fp8", "cfg4"],
                    default="decode")
    return ap.parse_args()


def seq_lens(seed):
    return np.random.RandomState(seed).randint(LEN_LO, LEN_HI + 1, size=B).tolist()


def algo_bytes(lens):
    kv = sum(lens) * NKV * HD * 2 * 2          # K and V, fp16
    qo = B * NQ * HD * (4 + 4)                 # f32 query in, f32 output out
    return kv + qo


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def peaks_tensor():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def traffic(leg):
    """DRAM bytes per launch of a leg's dominant kernel, from the ncu capture
    figures recorded in profiles/ncu_traffic.json (None if absent)."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(p) as f:
            return int(json.load(f)[leg]["traffic_bytes"])
    except (OSError, KeyError, ValueError, TypeError):
        return None


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def config(world, kv_bytes_per_gpu):
    """The workload description, identical in both arms."""
    return {"workload": "cfg2 batched GQA decode: B=32 per GPU, 32/8 heads, hd128, fp16 KV, "
                        "len~U[512,8192]",
            "global_batch": B * world, "kv_bytes_per_gpu": int(kv_bytes_per_gpu),
            "parallelism": f"dp{world} (sequence sharding, no collective)",
            "l2": "inputs (~570 MB KV per GPU) larger than the 126 MB L2; no flush"}


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons)}


def cpu_baseline(lens_list, seconds, K_host, V_host, q_host):
    """Time the oracle on the host cores over the full cfg-2 batch."""
    import oracle
    threads = os.cpu_count() or 1
    oracle.load()
    reps, t0 = 0, time.perf_counter()
    pos = [L - 1 for L in lens_list]
    while True:
        oracle.decode_batch(q_host, K_host, V_host, pos, NQ, NKV, HD, threads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds or reps >= 1000:
            break
    per = el / reps
    return {"value": algo_bytes(lens_list) / per / 1e9, "unit": "GB/s", "cores": threads,
            "cpu_model": cpu_model(), "kind": "port",
            "sample": f"full cfg-2 batch (B=32, {sum(lens_list)} keys), {reps} reps in {el:.1f} s, "
                      "C++ restatement of the Ada attention loops, one (seq x head) job per task"}


def prefill_leg(ab, torch, dev, seed, steps, warmup, stream):
    """causal prefill of 4 x 4096 tokens, 32/8 heads, hd 128,
    fp16 Q/K/V (seeded N(0,1)), fp16 output; one launch per step. Returns
    (ms per step, causal flops per step, host inputs for the CPU sample)."""
    nq, nkv, hd, S, NB = 32, 8, 128, 4096, 4
    g = torch.Generator(device=dev).manual_seed(seed)
    qs = [torch.randn(S, nq * hd, generator=g, device=dev).half() for _ in range(NB)]
    Ks = [torch.randn(S, nkv * hd, generator=g, device=dev).half() for _ in range(NB)]
    Vs = [torch.randn(S, nkv * hd, generator=g, device=dev).half() for _ in range(NB)]
    outs = [torch.empty(S, nq * hd, device=dev, dtype=torch.half) for _ in range(NB)]
    for _ in range(max(3, warmup)):
        ab.prefill_batch(qs, Ks, Vs, nq, nkv, hd, outs=outs, stream=stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        ab.prefill_batch(qs, Ks, Vs, nq, nkv, hd, outs=outs, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    flops = NB * nq * 2 * hd * S * (S + 1)
    return ms, flops, (qs[0], Ks[0], Vs[0])


def long_leg(ab, torch, dev, rank, world, steps, warmup, stream, dist):
    """BASELINE config 5a: one 131072-token sequence, 64/8 heads, hd 128, fp16
    KV split into contiguous chunks across the ranks; each step = partial
    (m, l, o) over the local chunk + the NVLink peer exchange fused with the
    merge (strong scaling: the total KV is fixed). Returns (ms per step, KV bytes of this rank)."""
    from aspida_b200 import shard
    nq, nkv, hd, L = 64, 8, 128, 131072
    lo, hi = shard.kv_chunks(L, world)[rank]
    n = hi - lo
    g = torch.Generator(device=dev).manual_seed(3000 + rank)
    K = torch.randn(max(n, 1), nkv * hd, generator=g, device=dev).half()
    V = torch.randn(max(n, 1), nkv * hd, generator=g, device=dev).half()
    q = torch.randn(1, nq * hd, generator=torch.Generator(device=dev).manual_seed(3000),
                    device=dev)
    # the NVLink peer exchange, unless setting it up or its first step fails on
    # some rank (then every rank falls back to NCCL)
    transport = "p2p"
    try:
        op = shard.SeqParallelDecode([K], [V], n, nq, nkv, hd, transport="p2p")
        op(q, stream=stream)
        bad = ab.device_status() != 0
    except (shard.ShardError, ab.GPUError):
        op, bad = None, True
    if dist:
        flag = torch.tensor([1 if bad else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        bad = int(flag.item()) != 0
    if bad:
        if op is not None:
            op.close()
        transport = "nccl"
        op = shard.SeqParallelDecode([K], [V], n, nq, nkv, hd, transport="nccl")

    def step():
        op(q, stream=stream)

    for _ in range(max(3, warmup)):
        step()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    op.close()
    return e0.elapsed_time(e1) / steps, n * nkv * hd * 2 * 2, transport


def q8_leg(ab, torch, dev, lens, steps, warmup, stream, seed, fp8=False):
    """Config-2 batch on Q8_0 caches (int8 + fp16 scale per 32 values, the
    reference's KVMODE 2 storage) or, with fp8, on fp8 e4m3 caches of the same
    geometry, quantised on the device from seeded N(0,1) f32. Returns (ms per
    step, algorithmic bytes per step)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    kvd = NKV * HD
    K8, V8, Ks, Vs = [], [], [], []
    for L in lens:
        for dst8, dsts in ((K8, Ks), (V8, Vs)):
            x = torch.randn(L, kvd, generator=g, device=dev)
            a, s = ab.quantize_fp8(x) if fp8 else ab.quantize_q8(x)
            dst8.append(a)
            dsts.append(s)
            del x
    tabs = [ab.ptr_table(t, dev) for t in (K8, V8, Ks, Vs)]
    q = torch.randn(len(lens), NQ * HD, generator=g, device=dev)
    pos = torch.tensor([L - 1 for L in lens], dtype=torch.int32, device=dev)
    out = torch.empty(len(lens), NQ * HD, device=dev)
    ws = ab.Workspace()
    maxkv = max(lens)

    dec = ab.decode_fp8 if fp8 else ab.decode_q8

    def step():
        dec(q, *tabs, pos, NQ, NKV, HD, max_kv_len=maxkv, out=out, workspace=ws, stream=stream)

    for _ in range(max(3, warmup)):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    nbytes = sum(lens) * kvd * 2 * (1 + 2 / 32) + len(lens) * NQ * HD * 8
    return e0.elapsed_time(e1) / steps, nbytes


def _time(torch, stream, fn, steps, warmup):
    for _ in range(max(3, warmup)):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def cfg4_legs(ab, torch, dev, steps, warmup, stream, seed):
    """BASELINE config 4 (Gemma-style: 16/8 heads, hd 256, softcap 50, scale
    1/16, layer pattern 5 sliding-window(1024) : 1 global). Prefill step: one
    8192-token prefill per layer of the pattern (6 launches). Decode step:
    B = 8 sequences at context 32768, one decode per layer of the pattern over
    the same caches (6 decode calls). Returns a dict of both legs."""
    nq, nkv, hd, S, W, cap, sc = 16, 8, 256, 8192, 1024, 50.0, 1.0 / 16
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(S, nq * hd, generator=g, device=dev).half()
    K = torch.randn(S, nkv * hd, generator=g, device=dev).half()
    V = torch.randn(S, nkv * hd, generator=g, device=dev).half()
    out = torch.empty(S, nq * hd, device=dev, dtype=torch.half)

    def prefill_step():
        ab.prefill(q, K, V, nq, nkv, hd, scale=sc, softcap=cap, out=out, stream=stream)
        for _ in range(5):
            ab.prefill(q, K, V, nq, nkv, hd, scale=sc, softcap=cap, window=W, out=out,
                       stream=stream)

    p_ms = _time(torch, stream, prefill_step, steps, warmup)
    f_glob = nq * 2 * hd * S * (S + 1)
    f_swa = 4 * hd * nq * sum(min(t + 1, W) for t in range(S))
    p_flops = f_glob + 5 * f_swa
    del q, K, V, out
    B, L = 8, 32768
    Ks = [torch.randn(L, nkv * hd, generator=g, device=dev).half() for _ in range(B)]
    Vs = [torch.randn(L, nkv * hd, generator=g, device=dev).half() for _ in range(B)]
    qd = torch.randn(B, nq * hd, generator=g, device=dev)
    Kt, Vt = ab.ptr_table(Ks, dev), ab.ptr_table(Vs, dev)
    pos = torch.full((B,), L - 1, dtype=torch.int32, device=dev)
    od = torch.empty(B, nq * hd, device=dev)
    ws = ab.Workspace()

    def decode_step():
        ab.decode(qd, Kt, Vt, pos, nq, nkv, hd, scale=sc, softcap=cap, max_kv_len=L, out=od,
                  workspace=ws, stream=stream)
        for _ in range(5):
            ab.decode(qd, Kt, Vt, pos, nq, nkv, hd, scale=sc, softcap=cap, window=W,
                      max_kv_len=L, out=od, workspace=ws, stream=stream)

    d_ms_eager = _time(torch, stream, decode_step, steps, warmup)
    # the same 6-layer step captured once in a CUDA graph and replayed: the
    # window layers read 67 MB each, so per-call host overhead would show
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        cs = torch.cuda.current_stream()
        for layer in range(6):
            ab.decode(qd, Kt, Vt, pos, nq, nkv, hd, scale=sc, softcap=cap,
                      window=0 if layer == 0 else W, max_kv_len=L, out=od, workspace=ws,
                      stream=cs)
    torch.cuda.synchronize()
    d_ms = _time(torch, stream, graph.replay, steps, warmup)
    d_bytes = B * nkv * hd * 2 * 2 * (L + 5 * W) + 6 * B * nq * hd * 8
    return {"prefill_ms": p_ms, "prefill_flops": p_flops, "decode_ms": d_ms,
            "decode_ms_eager": d_ms_eager, "decode_bytes": d_bytes}


def cfg5b_leg(ab, torch, dev, steps, warmup, stream, seed):
    """BASELINE config 5b: B = 256 sequences of 4096 tokens, 64/8 heads, hd 128,
    fp16 KV (4.3 GB), one decode per step. Returns (ms, algorithmic bytes)."""
    nq, nkv, hd, B, L = 64, 8, 128, 256, 4096
    g = torch.Generator(device=dev).manual_seed(seed)
    Ks = [torch.randn(L, nkv * hd, generator=g, device=dev).half() for _ in range(B)]
    Vs = [torch.randn(L, nkv * hd, generator=g, device=dev).half() for _ in range(B)]
    q = torch.randn(B, nq * hd, generator=g, device=dev)
    Kt, Vt = ab.ptr_table(Ks, dev), ab.ptr_table(Vs, dev)
    pos = torch.full((B,), L - 1, dtype=torch.int32, device=dev)
    out = torch.empty(B, nq * hd, device=dev)
    ws = ab.Workspace()
    ms = _time(torch, stream, lambda: ab.decode(q, Kt, Vt, pos, nq, nkv, hd, max_kv_len=L, out=out,
                                                workspace=ws, stream=stream), steps, warmup)
    return ms, B * L * nkv * hd * 2 * 2 + B * nq * hd * 8


def prefill_cpu_sample(q, K, V, seconds=8.0):
    """CPU oracle on the last rows of one config-3 sequence (causal flops of
    those rows / time), all host cores."""
    import oracle
    nq, nkv, hd = 32, 8, 128
    S = q.shape[0]
    qh, Kh, Vh = q.float().cpu().numpy(), K.float().cpu().numpy(), V.float().cpu().numpy()
    threads = os.cpu_count() or 1
    rows, t0, reps = list(range(S - 16, S)), time.perf_counter(), 0
    while True:
        oracle.prefill(qh, Kh, Vh, 0, nq, nkv, hd, rows=rows, threads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds or reps >= 100:
            break
    fl = sum(nq * 4 * hd * (r + 1) for r in rows)
    return {"value": round(fl * reps / el / 1e12, 5), "unit": "TFLOP/s", "cores": threads,
            "cpu_model": cpu_model(), "kind": "port", "sample": f"last 16 query rows of one 4096-token sequence, {reps} reps"}


def host_batch(seed, lens):
    """Same values as the device batch, as fp32 host arrays for the oracle."""
    import torch
    g = torch.Generator(device="cpu").manual_seed(seed)
    Ks, Vs = [], []
    for L in lens:
        Ks.append(torch.randn(L, NKV * HD, generator=g).half())
        Vs.append(torch.randn(L, NKV * HD, generator=g).half())
    q = torch.randn(B, NQ * HD, generator=g)
    return q, Ks, Vs


def run_reference(args, rank):
    if rank != 0:
        return
    lens = seq_lens(1000)
    q, Ks, Vs = host_batch(1000, lens)
    Kh = [k.float().numpy() for k in Ks]
    Vh = [v.float().numpy() for v in Vs]
    qh = q.numpy()
    import oracle
    oracle.load()
    threads = os.cpu_count() or 1
    pos = [L - 1 for L in lens]
    for _ in range(max(1, min(args.warmup, 2))):
        oracle.decode_batch(qh, Kh, Vh, pos, NQ, NKV, HD, threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.decode_batch(qh, Kh, Vh, pos, NQ, NKV, HD, threads=threads)
        times.append(time.perf_counter() - t0)
        if sum(times) > 120:
            break
    per = sum(times) / len(times)
    val = algo_bytes(lens) / per / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": len(times), "warmup": args.warmup,
        "ms_per_step": round(per * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config(max(1, int(os.environ.get("WORLD_SIZE", args.gpus))), algo_bytes(lens)),
        "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": threads,
                         "cpu_model": cpu_model(), "kind": "port",
                         "sample": f"full cfg-2 batch (rank 0's, host CPU), {len(times)} timed "
                                   "steps"},
        "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import aspida_b200 as ab

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)

    seed = 1000 + rank
    lens = seq_lens(seed)
    q_h, Ks_h, Vs_h = host_batch(seed, lens)
    caches = [ab.KVCache(L, NKV, HD, NQ) for L in lens]
    for c, k, v in zip(caches, Ks_h, Vs_h):
        c.K.copy_(k)
        c.V.copy_(v)
    q = q_h.to(dev)
    Kt = ab.ptr_table([c.K for c in caches], dev)
    Vt = ab.ptr_table([c.V for c in caches], dev)
    pos = torch.tensor([L - 1 for L in lens], dtype=torch.int32, device=dev)
    out = torch.empty(B, NQ * HD, device=dev)
    ws = ab.Workspace()
    stream = torch.cuda.current_stream()
    maxkv = max(lens)

    def step():
        ab.decode(q, Kt, Vt, pos, NQ, NKV, HD, max_kv_len=maxkv, out=out, workspace=ws,
                  stream=stream)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()

    if args.profile:
        if args.profile_leg == "decode":
            for _ in range(args.steps):
                step()
        elif args.profile_leg == "cfg4":
            for c in caches:
                c.free()
            cfg4_legs(ab, torch, dev, args.steps, args.warmup, stream, 5000 + rank)
        elif args.profile_leg in ("q8", "fp8"):
            for c in caches:
                c.free()
            q8_leg(ab, torch, dev, lens, args.steps, args.warmup, stream, 4000 + rank,
                   fp8=args.profile_leg == "fp8")
        elif args.profile_leg == "prefill":
            for c in caches:
                c.free()
            prefill_leg(ab, torch, dev, 2000 + rank, args.steps, args.warmup, stream)
        else:
            long_leg(ab, torch, dev, rank, world, args.steps, args.warmup, stream, dist)
        torch.cuda.synchronize()
        print(json.dumps({"profile_run": True, "leg": args.profile_leg, "steps": args.steps}))
        return
    sampler = ClockSampler(local)
    sampler.start()
    t_end = time.perf_counter() + 1.5        # keep the GPU under load for clock samples
    while time.perf_counter() < t_end:
        for _ in range(50):
            step()
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    if dist:
        dist.barrier()
    status = ab.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status}")

    # ---- e2e through the host-buffer C-ABI call ----
    qp = q_h.clone().pin_memory()
    kp = torch.randn(B, NKV * HD).pin_memory()
    vp = torch.randn(B, NKV * HD).pin_memory()
    op = torch.empty(B, NQ * HD).pin_memory()
    handles = [c.handle for c in caches]
    pos_l = [L - 1 for L in lens]
    for _ in range(max(3, args.warmup)):
        ab.step_host(handles, qp, kp, vp, pos_l, op, NQ, NKV, HD, rope_dim=HD,
                     rope_base=500000.0, stream=stream)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        ab.step_host(handles, qp, kp, vp, pos_l, op, NQ, NKV, HD, rope_dim=HD,
                     rope_base=500000.0, stream=stream)
    f1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = f0.elapsed_time(f1) / args.steps

    # ---- prefill leg (per rank) ----
    for c in caches:
        c.free()
    caches = []
    torch.cuda.empty_cache()
    p_steps = max(5, min(args.steps, 50))
    p_ms, p_flops, p_sample = prefill_leg(ab, torch, dev, 2000 + rank, p_steps, args.warmup,
                                          stream)
    if ab.device_status() != 0:
        raise RuntimeError("device status after prefill")
    l_ms, l_bytes, l_transport = long_leg(ab, torch, dev, rank, world,
                                          max(10, min(args.steps, 100)), args.warmup, stream,
                                          dist)
    torch.cuda.empty_cache()
    q_ms, q_bytes = q8_leg(ab, torch, dev, lens, args.steps, args.warmup, stream, 4000 + rank)
    torch.cuda.empty_cache()
    f_ms, f_bytes = q8_leg(ab, torch, dev, lens, args.steps, args.warmup, stream, 4500 + rank,
                           fp8=True)
    if ab.device_status() != 0:
        raise RuntimeError("device status after q8 / fp8 decode")
    torch.cuda.empty_cache()
    x_steps = max(5, min(args.steps, 20))
    c4 = cfg4_legs(ab, torch, dev, x_steps, args.warmup, stream, 5000 + rank)
    torch.cuda.empty_cache()
    b_ms, b_bytes = cfg5b_leg(ab, torch, dev, x_steps, args.warmup, stream, 6000 + rank)
    torch.cuda.empty_cache()
    if ab.device_status() != 0:
        raise RuntimeError("device status after cfg4 / cfg5b")

    nbytes = algo_bytes(lens)
    times = [ms, ms_e2e, p_ms, l_ms, q_ms, c4["prefill_ms"], c4["decode_ms"], b_ms, f_ms]
    work = [float(nbytes), float(p_flops), float(l_bytes), float(q_bytes),
            float(c4["prefill_flops"]), float(c4["decode_bytes"]), float(b_bytes), float(f_bytes)]
    stats = torch.tensor(times + work, dtype=torch.float64, device=dev)
    if dist:
        mx = stats[:len(times)].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tot = stats[len(times):].clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        times_max, work_all = [float(x) for x in mx], [float(x) for x in tot]
    else:
        times_max, work_all = times, work
    ms_max, ms_e2e_max, p_ms_max, l_ms_max, q_ms_max, c4p_max, c4d_max, b_ms_max, f_ms_max = \
        times_max
    bytes_all, flops_all, l_bytes_all, q_bytes_all, c4p_all, c4d_all, b_all, f_bytes_all = work_all

    if rank == 0:
        hbm, src = peaks()
        achieved = nbytes / (ms * 1e-3) / 1e9
        line = {
            "metric": METRIC,
            "value": round(bytes_all / (ms_max * 1e-3) / 1e9, 3),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_max, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16 KV / f32 accumulate",
            "data": "synthetic (seeded N(0,1) fp16 KV, lengths U[512,8192])",
            "config": config(world, nbytes),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(achieved / hbm, 4),
                         "traffic": traffic("decode_cfg2"), "peak_source": f"{src} hbm_gbs (copy, burst)"},
            "e2e": {"value": round(bytes_all / (ms_e2e_max * 1e-3) / 1e9, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": int(qp.numel() * 4 + kp.numel() * 4 + vp.numel() * 4
                                              + B * (2 * 4 + 2 * 8)),
                    "d2h_bytes_per_step": int(op.numel() * 4),
                    "ms_per_step": round(ms_e2e_max, 5)},
            "gpu_launches": args.steps * 2,   # decode_kernel + combine_kernel per step
            "clocks": clocks,
            "prefill": {
                "metric": "prefill attn TFLOP/s (cfg3: causal 4 x 4096, 32/8 heads, hd128, fp16)",
                "value": round(flops_all / (p_ms_max * 1e-3) / 1e12, 2),
                "unit": "TFLOP/s", "ms_per_step": round(p_ms_max, 4), "steps": p_steps,
                "flops_per_step_per_gpu": p_flops,
                "roofline": {"bound": "tensor",
                             "achieved": round(p_flops / (p_ms * 1e-3) / 1e12, 2),
                             "peak": peaks_tensor()[0], "unit": "TFLOP/s",
                             "frac": round(p_flops / (p_ms * 1e-3) / 1e12 / peaks_tensor()[0], 4),
                             "traffic": traffic("prefill_cfg3"),
                             "peak_source": f"{peaks_tensor()[1]} bf16_tflops (cuBLAS, burst)"},
                "gpu_launches": p_steps,
            },
            "decode_long": {
                "metric": "decode attn KV GB/s (cfg5a: one 131072-token sequence, 64/8 heads, "
                          "hd128, KV split across GPUs + (m,l,o) exchange and merge)",
                "transport": l_transport if world > 1 else "local",
                "value": round(l_bytes_all / (l_ms_max * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(l_ms_max, 5), "scaling": "strong",
                "kv_bytes_total": int(l_bytes_all),
                "frac_of_hbm_x_gpus": round(l_bytes_all / (l_ms_max * 1e-3) / 1e9
                                            / (peaks()[0] * world), 4),
            },
        }
        line["decode_q8"] = {
            "metric": "decode attn KV GB/s over Q8_0 caches (cfg2 lengths and heads, int8 + "
                      "fp16 scale per 32 values)",
            "value": round(q_bytes_all / (q_ms_max * 1e-3) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(q_ms_max, 5),
            "speedup_vs_fp16_kv": round(ms_max / q_ms_max, 3),
            "bytes_per_step_per_gpu": int(q_bytes),
            "roofline": {"bound": "hbm", "achieved": round(q_bytes / (q_ms * 1e-3) / 1e9, 1),
                         "peak": peaks()[0], "unit": "GB/s",
                         "frac": round(q_bytes / (q_ms * 1e-3) / 1e9 / peaks()[0], 4),
                         "traffic": traffic("decode_q8_cfg2")},
            "gpu_launches": args.steps * 2,
        }
        line["decode_fp8"] = {
            "metric": "decode attn KV GB/s over fp8 e4m3 caches (cfg2 lengths and heads, e4m3 + "
                      "fp16 scale per 32 values)",
            "value": round(f_bytes_all / (f_ms_max * 1e-3) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(f_ms_max, 5),
            "speedup_vs_fp16_kv": round(ms_max / f_ms_max, 3),
            "bytes_per_step_per_gpu": int(f_bytes),
            "roofline": {"bound": "hbm", "achieved": round(f_bytes / (f_ms * 1e-3) / 1e9, 1),
                         "peak": peaks()[0], "unit": "GB/s",
                         "frac": round(f_bytes / (f_ms * 1e-3) / 1e9 / peaks()[0], 4),
                         "traffic": traffic("decode_fp8_cfg2")},
            "gpu_launches": args.steps * 2,
        }
        hbm_peak, tc_peak = peaks()[0], peaks_tensor()[0]
        line["cfg4"] = {
            "metric": "cfg4 (16/8 heads, hd256, softcap 50, 5 SWA(1024) : 1 global): prefill "
                      "TFLOP/s over 8192 tokens x 6 layers; decode KV GB/s, B=8 at ctx 32768 x 6 "
                      "layers",
            "prefill": {"value": round(c4p_all / (c4p_max * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                        "ms_per_step": round(c4p_max, 4),
                        "frac_of_tensor_peak": round(c4["prefill_flops"] / (c4["prefill_ms"] * 1e-3)
                                                     / 1e12 / tc_peak, 4)},
            "decode": {"value": round(c4d_all / (c4d_max * 1e-3) / 1e9, 1), "unit": "GB/s",
                       "ms_per_step": round(c4d_max, 4), "cuda_graph": True,
                       "ms_per_step_eager": round(c4["decode_ms_eager"], 4),
                       "frac_of_hbm": round(c4["decode_bytes"] / (c4["decode_ms"] * 1e-3) / 1e9
                                            / hbm_peak, 4)},
            "gpu_launches": x_steps * 6 * 3,
        }
        line["cfg5b"] = {
            "metric": "cfg5b decode KV GB/s (B=256 x 4096 tokens, 64/8 heads, hd128, fp16 KV)",
            "value": round(b_all / (b_ms_max * 1e-3) / 1e9, 1), "unit": "GB/s",
            "ms_per_step": round(b_ms_max, 4),
            "frac_of_hbm": round(b_bytes / (b_ms * 1e-3) / 1e9 / hbm_peak, 4),
            "gpu_launches": x_steps * 2,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(lens, args.cpu_seconds,
                                                [k.float().numpy() for k in Ks_h],
                                                [v.float().numpy() for v in Vs_h], q_h.numpy())
            line["prefill"]["cpu_baseline"] = prefill_cpu_sample(*p_sample)
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
