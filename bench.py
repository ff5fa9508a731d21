"""Decode throughput of a Mistral-7B-shaped NF4 model on B200 (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl b200|reference]

Workload (N=1): random-init Mistral-7B-shaped model (32 layers, hidden 4096, 32 query / 8 KV heads,
head_dim 128, SwiGLU 14336, vocab 32768, RMSNorm eps 1e-5, RoPE theta 1e6), every decoder linear NF4
(blocksize 64, double-quantised scales, blocksize 256), fp16 activations; B seeded random prompts of
256 tokens are prefilled, then greedy decode. One step = one decode token for every sequence through
all 32 layers (7 fused NF4 dequant+matmul launches and one split-K attention + combine per layer),
replayed as a CUDA graph. The 3.9 GB of weights streamed per step exceed the 126 MB L2, so no flush
is needed between steps.

Reported: ``value`` = tokens/s with inputs resident on the device (events around K replays);
``e2e`` = the same through the public step API with the token ids copied host->device and the next
ids device->host every step; ``roofline`` = achieved HBM bandwidth of the dominant kernel (the
14336x4096 NF4 gate_proj matmul at batch B, each launch timed with CUDA events on its stream);
``cpu_baseline`` = the reference path (torch NF4 dequant + matmul, repeat_kv + SDPA) on the host cores.

``--impl reference`` times that CPU path alone (rank 0; other ranks exit) as the reference arm.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "llm-decode-triton-6gb_b200"))

METRIC = "decode tok/s @ batch 1/8 (Mistral-7B NF4 shape); kernel % of HBM peak"
PROMPT = 256
CONTEXT_FOR_CPU = PROMPT + 64


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = "clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []
        self.window = (0.0, float("inf"))

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "50"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.perf_counter(), line.strip()))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lo, hi = self.window
        for t, ln in self.lines:
            if not (lo <= t <= hi):
                continue
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 6:
                continue
            try:
                sm.append(float(parts[0]))
                mx = max(mx, float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[2:]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference(batch: int, layers: int, samples: int, seed: int = 0):
    """Reference CPU path (oracle/cpu_path) on the host: tok/s from per-layer samples, scaled."""
    import torch
    from oracle import cpu_path
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    layer = cpu_path.CpuDecodeLayer(seed=seed)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, 4096, generator=g).half()
    kc = torch.randn(batch, 8, CONTEXT_FOR_CPU, 128, generator=g).half()
    vc = torch.randn(batch, 8, CONTEXT_FOR_CPU, 128, generator=g).half()
    layer.forward(x, kc, vc)                        # warm-up
    t_head = cpu_path.time_lm_head(batch, threads=threads)
    ts = []
    for _ in range(samples):
        t = time.perf_counter()
        layer.forward(x, kc, vc)
        ts.append(time.perf_counter() - t)
    t_layer = statistics.median(ts)
    tok_s = batch / (layers * t_layer + t_head)
    sample = (f"{samples} timed decoder layer(s) of the 32 (7 NF4 linears dequantised + matmul in fp32, "
              f"repeat_kv + SDPA over {CONTEXT_FOR_CPU} cached keys) at batch {batch}, plus one lm_head; "
              f"per-token time = 32 x median layer + lm_head")
    return tok_s, threads, sample, ts


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    tok_s, threads, sample, _ = cpu_reference(args.batch, 32, max(1, args.steps))
    line = {"metric": METRIC, "value": round(tok_s, 4), "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "impl": "reference",
            "cpu_baseline": {"value": round(tok_s, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(tok_s, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "dtype": "f16", "data": "synthetic (seeded N(0, 0.02^2) weights, NF4-quantised on the host)",
            "config": {"workload": f"Mistral-7B-shaped NF4 decode, batch {args.batch}, context {CONTEXT_FOR_CPU}",
                       "batch": args.batch}}
    print(json.dumps(line), flush=True)


def traffic_from_profile():
    p = ROOT / "profiles" / "nf4_gemm_gate_proj_14336x4096_b8.txt"
    if not p.exists():
        return None
    for ln in p.read_text().splitlines():
        if ln.startswith("dram_bytes_per_launch:"):
            return int(float(ln.split(":")[1]))
    return None


def _init_ranks(args):
    """(rank, world, device, TPGroup|None). N > 1 runs one process per GPU under torchrun (NCCL)."""
    import datetime
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N > 1 with torch.distributed.run")
    rank = int(os.environ.get("RANK", "0"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    if world == 1:
        return rank, world, dev, None
    import torch.distributed as dist
    from b200kernels.tp import TPGroup
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    return rank, world, dev, TPGroup(rank, world)


def _max_over_ranks(v: float, world: int, dev) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world: int, dev):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier(device_ids=[dev.index])
    torch.cuda.synchronize(dev)


def run_b200(args):
    import torch
    from b200kernels import decode as dec

    rank, world, dev, tp = _init_ranks(args)
    B, K, W = args.batch, args.steps, args.warmup
    model = dec.build_random_mistral(seed=args.seed, num_hidden_layers=args.layers)
    context = args.context or PROMPT
    max_len = context + 2 * (K + W) + 16
    eng = dec.DecodeEngine(model, B, max_len, tp=tp, allreduce=args.allreduce)
    if args.context:   # long caches: seeded K/V written straight into the static cache (no prefill)
        eng.fill_random_cache(context, seed=args.seed + 1)
    else:
        g = torch.Generator().manual_seed(args.seed + 1)
        prompts = torch.randint(0, model.config.vocab_size, (B, PROMPT), generator=g)
        eng.prefill(prompts.to(dev))
    eng.capture()
    clk = ClockSampler(dev.index).start()
    # keep the GPU busy until nvidia-smi reports (its start-up takes ~1 s); every rank takes the same
    # number of steps (the ranks agree on "not ready" through a max over ranks)
    t_wait = time.perf_counter()
    while True:
        waiting = clk.proc is not None and not clk.lines and time.perf_counter() - t_wait < 15
        if _max_over_ranks(1.0 if waiting else 0.0, world, dev) == 0.0:
            break
        for _ in range(8):
            eng.step()
        torch.cuda.synchronize(dev)
    for _ in range(W):
        eng.step()
    _barrier(world, dev)

    # ---- device-resident throughput (clock samples kept only inside this window, padded 50 ms)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    profile_region = os.environ.get("B2D_PROFILE_STEPS") == "1"   # ncu --profile-from-start off
    if profile_region:
        torch.cuda.profiler.start()
    w0 = time.perf_counter()
    s.record()
    for _ in range(K):
        eng.step()
    e.record()
    torch.cuda.synchronize(dev)
    w1 = time.perf_counter()
    if profile_region:
        torch.cuda.profiler.stop()
    clk.window = (w0 - 0.05, w1 + 0.05)
    ms = _max_over_ranks(s.elapsed_time(e), world, dev)
    value = B * K / (ms / 1e3)

    # ---- end to end through the step API: ids host->device, next ids device->host, every step
    host_in = torch.empty(B, dtype=torch.long).pin_memory()
    host_out = torch.empty(B, dtype=torch.long).pin_memory()
    host_in.copy_(eng.next_ids.cpu())
    _barrier(world, dev)
    t0 = time.perf_counter()
    se, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    se.record()
    for _ in range(K):
        eng.ids.copy_(host_in, non_blocking=True)
        eng.step()
        host_out.copy_(eng.next_ids, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        host_in.copy_(host_out)
    ee.record()
    torch.cuda.synchronize(dev)
    e2e_ms = _max_over_ranks(se.elapsed_time(ee), world, dev)
    e2e_wall = time.perf_counter() - t0
    e2e = B * K / (e2e_ms / 1e3)
    clk.stop()
    _barrier(world, dev)

    # ---- roofline: the model's gate_proj matmuls (this rank's 14336/N x 4096 NF4 shards) at batch B,
    # launched back to back from a CUDA graph on the bench stream and timed with events on that stream
    # (no host gaps); consecutive launches read different weights, so every launch streams its
    # weights from HBM.
    x = torch.randn(B, 4096, generator=torch.Generator().manual_seed(3)).half().to(dev)
    gates = [wd["gate"] for wd in eng.w]
    st = torch.cuda.Stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(st):
        ys = [wgt.matmul(x) for wgt in gates]
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        for wgt, y in zip(gates, ys):
            wgt.matmul(x, out=y)
    durs = []
    for _ in range(3):
        with torch.cuda.stream(st):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            graph.replay()
            b.record(st)
        b.synchronize()
        durs.append(a.elapsed_time(b) * 1e3 / len(gates))
    us = min(durs)
    del graph
    alg = gates[0].nbytes + x.numel() * 2 + B * gates[0].N * 2
    peak, peak_kind = measured_peaks()
    achieved = alg / (us * 1e-6) / 1e9

    # ---- our kernel launches per step: per layer 2 add+RMSNorm, RoPE + KV append, attention partial +
    # combine and the NF4 launches (q/k/v, o, gate/up, down at B <= 8; else 7 NF4 launches and SiLU*mul),
    # plus the all-reduces under TP; plus the final add+RMSNorm
    per_layer = (5 + 4) if eng.pair else (5 + 7 + 1)
    if tp is not None and not eng.ar_fused:   # fused: the GEMMs push, the add+RMSNorm launches sum
        per_layer += 2
    launches_per_step = args.layers * per_layer + 1 + (1 if eng.lm_fused else 0)   # + final norm (+ lm_head)

    cpu = None
    if world == 1 and rank == 0:   # the reference CPU path on the host, at N=1 only
        cpu_tok_s, threads, sample, _ = cpu_reference(B, 32, samples=1)
        cpu = {"value": round(cpu_tok_s, 4), "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample}
    _barrier(world, dev)
    if rank == 0:
        shard = "" if world == 1 else f" (rank-0 shard {gates[0].N}x{gates[0].K})"
        line = {"metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": K,
                "warmup": W, "ms_per_step": round(ms / K, 4), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f16",
                "data": "synthetic (seeded random prompts, random-init N(0, 0.02^2) weights)",
                "config": {"workload": f"Mistral-7B-shaped NF4 greedy decode, batch {B}, "
                                       + (f"{context}-token seeded random KV cache" if args.context else
                                          f"prompt {PROMPT}") + f", {args.layers} layers, CUDA-graph step",
                           "batch": B, "prompt": None if args.context else PROMPT, "context": context,
                           "layers": args.layers,
                           "parallelism": "single GPU" if world == 1 else
                           f"tp{world} (" + {"fused": "o_proj/down_proj GEMM epilogues push partials to the peers "
                                                     "over NVLink, summed in the next add+RMSNorm",
                                             "peer": "one-shot NVLink peer-memory all-reduce after o_proj and "
                                                     "down_proj",
                                             "nccl": "NCCL all-reduce after o_proj and down_proj"}[
                               "fused" if eng.ar_fused else ("nccl" if args.allreduce == "nccl" else "peer")] + ")",
                           "l2": "no flush: 3.9 GB of weights per step exceed the 126 MB L2"},
                "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": B * 8,
                        "d2h_bytes_per_step": B * 8, "wall_s": round(e2e_wall, 4)},
                "roofline": {"bound": "hbm", "kernel": "nf4_gemm_pipe_kernel (gate_proj" + shard + ", nested)",
                             "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                             "frac": round(achieved / peak, 4),
                             "traffic": traffic_from_profile() if world == 1 else None,
                             "algorithmic_bytes_per_launch": alg, "avg_launch_us": round(us, 3)},
                "cpu_baseline": cpu,
                "gpu_launches": launches_per_step * K,
                "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    if tp is not None and tp.peer_errors():
        raise SystemExit(f"rank {rank}: {tp.peer_errors()} timed-out all-reduce waits; the run is invalid")
    eng.graph = None   # a graph holding NCCL calls must go before the process group
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist
        _barrier(world, dev)
        dist.destroy_process_group()


def _graph_time_us(fns, reps=3):
    """Per-launch device time (us) of a rotated list of launches captured in one CUDA graph."""
    import torch
    n = max(len(fns), 24)
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        for f in fns:
            f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(n):
            fns[i % len(fns)]()
    best = float("inf")
    for _ in range(reps):
        with torch.cuda.stream(st):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            g.replay()
            b.record(st)
        torch.cuda.synchronize()
        best = min(best, a.elapsed_time(b) * 1e3 / n)
    return best


def run_kernels(args):
    """Kernel micro-benchmarks (the reference's bench_nf4.py / bench_attention.py, on B200): per shape,
    device time per launch with weights/caches rotated through more than 2x L2, % of measured HBM
    peak. ``--profile-iters n`` instead launches each case n times (for ncu)."""
    import torch
    from b200kernels.decode_attention import decode_attention
    from b200kernels.linear4bit import quantize_nf4
    from b200kernels.nf4_gemm import NF4Weight
    peak, peak_kind = measured_peaks()
    dev = torch.device("cuda", 0)
    batches = [int(b) for b in args.batches.split(",")]
    if args.kernel == "nf4":
        shapes = [tuple(int(v) for v in s.split("x")) for s in args.shapes.split(",")]
        for (N, K) in shapes:
            copies = 1 if args.profile_iters else max(4, int(2 * 126e6 // (N * K // 2)) + 1)
            ws = []
            for c in range(copies):
                w = (torch.randn(N, K, generator=torch.Generator().manual_seed(c)) * 0.02).to(dev)
                packed, qs = quantize_nf4(w, nested=not args.plain)
                p = torch.nn.Parameter(packed, requires_grad=False)
                p.quant_state = qs
                ws.append(NF4Weight(p))
                del w
            for M in batches:
                x = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).half().to(dev)
                if args.profile_iters:
                    for _ in range(args.profile_iters):
                        ws[0].matmul(x)
                    torch.cuda.synchronize()
                    continue
                us = _graph_time_us([lambda w=w: w.matmul(x) for w in ws])
                nbytes = ws[0].nbytes + x.numel() * 2 + M * N * 2
                print(json.dumps({"kernel": "nf4_gemm", "N": N, "K": K, "M": M, "nested": not args.plain,
                                  "us": round(us, 2), "GBps": round(nbytes / us / 1e3, 1),
                                  "pct_peak": round(100 * nbytes / us / 1e3 / peak, 1), "peak_kind": peak_kind}),
                      flush=True)
            del ws
            torch.cuda.empty_cache()
    elif args.kernel == "prefill":   # many-row linears: bit-exact device dequant + cuBLAS vs the stock path
        import torch.nn.functional as F
        from b200kernels.linear4bit import dequantize_torch
        M = args.prefill_rows
        shapes = [tuple(int(v) for v in s.split("x")) for s in args.shapes.split(",")]
        for (N, K) in shapes:
            w = (torch.randn(N, K, generator=torch.Generator().manual_seed(N + K)) * 0.02).half().to(dev)
            packed, qs = quantize_nf4(w, nested=not args.plain)
            p = torch.nn.Parameter(packed, requires_grad=False)
            p.quant_state = qs
            nf = NF4Weight(p)
            del w
            x = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).half().to(dev)
            wbuf = torch.empty(N, K, dtype=torch.half, device=dev)
            y = torch.empty(M, N, dtype=torch.half, device=dev)
            t_deq = _graph_time_us([lambda: nf.dequantize(out=wbuf)])
            t_gemm = _graph_time_us([lambda: torch.matmul(x, wbuf.T, out=y)])
            t_ours = _graph_time_us([lambda: (nf.dequantize(out=wbuf), torch.matmul(x, wbuf.T, out=y))])
            t_stock = _graph_time_us([lambda: y.copy_(F.linear(x, dequantize_torch(p.data, qs, torch.half)))])
            deq_bytes = nf.nbytes + N * K * 2
            print(json.dumps({"kernel": "prefill_linear", "N": N, "K": K, "M": M, "nested": not args.plain,
                              "dequant_us": round(t_deq, 2), "dequant_GBps": round(deq_bytes / t_deq / 1e3, 1),
                              "dequant_pct_peak": round(100 * deq_bytes / t_deq / 1e3 / peak, 1),
                              "gemm_only_us": round(t_gemm, 2), "ours_us": round(t_ours, 2),
                              "stock_us": round(t_stock, 2), "dequant_tax_ours": round(t_ours / t_gemm - 1, 3),
                              "dequant_tax_stock": round(t_stock / t_gemm - 1, 3), "peak_kind": peak_kind}), flush=True)
            del nf, p, packed, qs, wbuf, y
            torch.cuda.empty_cache()
    elif args.kernel == "lm_head":   # Mistral-7B head 32000x4096 fp16 + argmax (two weight copies > 2x L2)
        from b200kernels.lm_head import lm_head_argmax
        V, K = 32000, 4096
        ws = [(torch.randn(V, K, generator=torch.Generator().manual_seed(c)) * 0.02).half().to(dev)
              for c in range(1 if args.profile_iters else 2)]
        for M in batches:
            x = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).half().to(dev)
            lg = torch.empty(M, V, dtype=torch.half, device=dev)
            ids = torch.empty(M, dtype=torch.int64, device=dev)
            if args.profile_iters:
                for _ in range(args.profile_iters):
                    lm_head_argmax(x, ws[0], logits=lg, ids=ids)
                torch.cuda.synchronize()
                continue
            us = _graph_time_us([lambda w=w: lm_head_argmax(x, w, logits=lg, ids=ids) for w in ws])
            nbytes = V * K * 2 + M * K * 2 + M * V * 2
            print(json.dumps({"kernel": "lm_head_argmax", "V": V, "K": K, "M": M, "us": round(us, 2),
                              "GBps": round(nbytes / us / 1e3, 1), "pct_peak": round(100 * nbytes / us / 1e3 / peak, 1),
                              "peak_kind": peak_kind}), flush=True)
    else:
        contexts = [int(s) for s in args.contexts.split(",")]
        for B in batches:
            for S in contexts:
                copies = 1 if args.profile_iters else max(2, int(2 * 126e6 // (2 * B * 8 * S * 256)) + 1)
                g = torch.Generator().manual_seed(B * 7919 + S)
                cases = [tuple(torch.randn(sh, generator=g).half().to(dev)
                               for sh in ((B, 32, 1, 128), (B, 8, S, 128), (B, 8, S, 128))) for _ in range(copies)]
                lens = None
                if args.ragged:
                    lens = torch.randint(min(512, S), S + 1, (B,), generator=g).to(torch.int32).to(dev)
                n_keys = int(lens.sum()) if lens is not None else B * S
                if args.profile_iters:
                    for _ in range(args.profile_iters):
                        decode_attention(*cases[0], 128 ** -0.5, seqlens=lens)
                    torch.cuda.synchronize()
                    continue
                us = _graph_time_us([lambda c=c: decode_attention(*c, 128 ** -0.5, seqlens=lens) for c in cases])
                nbytes = n_keys * 8 * 128 * 2 * 2 + B * 32 * 128 * 2 * 2
                print(json.dumps({"kernel": "gqa_decode", "B": B, "S": S, "ragged": bool(args.ragged),
                                  "us": round(us, 2), "GBps": round(nbytes / us / 1e3, 1),
                                  "pct_peak": round(100 * nbytes / us / 1e3 / peak, 1), "peak_kind": peak_kind}),
                      flush=True)
                del cases
                torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", choices=["nf4", "attention", "lm_head", "prefill"], default=None,
                    help="kernel micro-benchmark instead of the decode bench")
    ap.add_argument("--shapes", default="14336x4096,4096x4096,1024x4096,4096x14336")
    ap.add_argument("--batches", default="1,2,4,8")
    ap.add_argument("--prefill-rows", type=int, default=2048, help="rows (batch x prompt) for --kernel prefill")
    ap.add_argument("--contexts", default="128,512,2048,4096")
    ap.add_argument("--ragged", action="store_true")
    ap.add_argument("--plain", action="store_true", help="fp32 absmax instead of double quantisation")
    ap.add_argument("--profile-iters", type=int, default=0)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--context", type=int, default=0,
                    help="decode after a seeded random KV cache of this many tokens instead of a 256-token prefill "
                         "(long-context and tensor-parallel configurations)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--allreduce", choices=["fused", "peer", "nccl"], default="fused",
                    help="tensor-parallel all-reduce: fused into the o/down GEMM epilogue, peer-memory kernel, NCCL")
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    args = ap.parse_args()
    if args.kernel:
        run_kernels(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
