"""Decode throughput of a Mistral-7B-shaped NF4 model on B200 (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl b200|reference]

Workload (N=1): random-init Mistral-7B-shaped model (32 layers, hidden 4096, 32 query / 8 KV heads,
head_dim 128, SwiGLU 14336, vocab 32768, RMSNorm eps 1e-5, RoPE theta 1e6), every decoder linear NF4
(blocksize 64, double-quantised scales, blocksize 256), fp16 activations; B seeded random prompts of
256 tokens are prefilled, then greedy decode. One step = one decode token for every sequence through
all 32 layers (7 fused NF4 dequant+matmul launches and one split-K attention + combine per layer, the
step's RoPE + KV append inside the attention launch),
replayed as a CUDA graph. The 3.9 GB of weights streamed per step exceed the 126 MB L2, so no flush
is needed between steps.

Reported: ``value`` = tokens/s with inputs resident on the device (events around K replays);
``e2e`` = the same through the public step API with the token ids copied host->device and the next
ids device->host every step; ``roofline`` = achieved HBM bandwidth of the dominant kernel (the
14336x4096 NF4 gate_proj matmul at batch B, each launch timed with CUDA events on its stream);
``cpu_baseline`` = the reference path (torch NF4 dequant + matmul, repeat_kv + SDPA) on the host cores.

Also in the same line (one process per GPU, max over ranks for every device time):

* ``batch1``: the same decode at batch 1 (the metric names batch 1 and 8);
* ``long_context`` (N=1): batch 8 decoding after a 32768-token seeded random KV cache, with the attention
  kernel's time per launch at that length;
* ``tp_config5`` (every N): batch 64 after a 4096-token cache, tok/s and per-GPU HBM GB/s;
* ``tp_parity`` (N > 1): the tensor-parallel engine's greedy tokens and logits against the single-GPU
  engine fed the same tokens (teacher-forced, on rank 0);
* ``stock_hf`` / ``patched_hf`` (N=1): the Hugging Face forward with a ``DynamicCache`` on this GPU,
  stock (torch NF4 dequant + ``F.linear``, SDPA) and after ``patch_linear4bit`` + ``patch_attention``
  (the drop-in path), at batch 1 and 8;
* ``nf4_op`` / ``attention_op`` (N=1): the two single-op configurations (NF4 M=4 14336x4096 plain
  absmax; GQA decode B=8, S=2048, lengths U[512, 2048]) in us per launch and % of measured HBM peak.

Every device-timed decode number is the median of 5 timed regions of K steps, each started from the
same cache position (the steps before it -- clock start-up, warm-up -- never run past the cache).

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


def cpu_model_name() -> str:
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for ln in out.splitlines():
            if ln.strip().startswith("Model name:"):
                return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def _median_time(fn, reps: int, warmup: int):
    for _ in range(warmup):
        fn()
    ts = []
    for _ in range(reps):
        t = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t)
    return statistics.median(ts), ts


def cpu_reference(batch: int, layers: int, reps: int = 10, warmup: int = 3, context: int = PROMPT,
                  per_op: bool = True, seed: int = 0):
    """The reference's CPU path (oracle/cpu_path) on all host threads: tok/s of a decode step built from
    the median of ``reps`` timed decoder layers (after ``warmup``) x ``layers`` + the lm_head, and (with
    ``per_op``) the two single-op configurations, each the median of ``reps`` after ``warmup``."""
    import torch
    from oracle import attn_ref, cpu_path
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    layer = cpu_path.CpuDecodeLayer(seed=seed)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, 4096, generator=g).half()
    kc = torch.randn(batch, 8, context, 128, generator=g).half()
    vc = torch.randn(batch, 8, context, 128, generator=g).half()
    t_layer, _ = _median_time(lambda: layer.forward(x, kc, vc), reps, warmup)
    w = (torch.randn(32768, 4096, generator=g) * 0.02).half()
    t_head, _ = _median_time(lambda: (x.float() @ w.float().T).argmax(-1), max(3, reps // 3), 1)
    del w
    tok_s = batch / (layers * t_layer + t_head)
    out = {"value": round(tok_s, 4), "unit": "tok/s", "cores": threads, "kind": "port", "cpu": cpu_model_name(),
           "sample": (f"median of {reps} timed decoder layers (after {warmup} warm-up) of the 32: 7 NF4 linears "
                      f"dequantised + matmul in fp32, repeat_kv + SDPA over {context} cached keys, batch {batch}; "
                      f"per-token time = {layers} x median layer + lm_head (fp32 GEMV + argmax)"),
           "layer_s": round(t_layer, 4), "lm_head_s": round(t_head, 4)}
    if per_op:
        lin = cpu_path.CpuNF4Linear(14336, 4096, seed=seed + 7, nested=False)
        x1 = torch.randn(4, 4096, generator=g).half()
        t_nf4, _ = _median_time(lambda: lin.forward(x1), reps, warmup)
        q = torch.randn(8, 32, 1, 128, generator=g).half()
        k2 = torch.randn(8, 8, 2048, 128, generator=g).half()
        v2 = torch.randn(8, 8, 2048, 128, generator=g).half()
        sl = torch.randint(512, 2049, (8,), generator=g).to(torch.int32)
        t_att, _ = _median_time(lambda: attn_ref.stock_cpu(q, k2, v2, 128 ** -0.5, sl), reps, warmup)
        out["nf4_op_us"] = round(t_nf4 * 1e6, 1)
        out["nf4_op"] = "M=4 x [14336, 4096] NF4 plain absmax: torch dequant to fp16 + x.float() @ W.float().T"
        out["attention_op_us"] = round(t_att * 1e6, 1)
        out["attention_op"] = "B=8, 32 q / 8 KV heads, S=2048, lengths U[512, 2048]: repeat_kv + SDPA in fp32"
    return out


def headline_config(batch: int, world: int, layers: int = 32, allreduce: str = "fused") -> dict:
    """The workload both arms report (the reference arm times the same workload on the host)."""
    par = "single GPU" if world == 1 else (
        f"tp{world} (" + {"fused": "o_proj/down_proj GEMM epilogues push partials to the peers over NVLink, summed "
                                   "in the next add+RMSNorm",
                          "peer": "one-shot NVLink peer-memory all-reduce after o_proj and down_proj",
                          "nccl": "NCCL all-reduce after o_proj and down_proj"}[allreduce] + ")")
    return {"workload": f"Mistral-7B-shaped NF4 greedy decode, batch {batch}, prompt {PROMPT}, {layers} layers",
            "batch": batch, "prompt": PROMPT, "context": PROMPT, "layers": layers, "parallelism": par,
            "l2": "no flush: 3.9 GB of weights per step exceed the 126 MB L2"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cpu = cpu_reference(args.batch, 32, reps=max(10, args.steps), warmup=max(3, args.warmup), per_op=False)
    tok_s = cpu["value"]
    line = {"metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "impl": "reference",
            "cpu_baseline": cpu,
            "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "dtype": "f16", "data": "synthetic (seeded N(0, 0.02^2) weights, NF4-quantised on the host)",
            "config": headline_config(args.batch, args.gpus, allreduce=args.allreduce)}
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


REPEATS = 5   # timed regions of K steps; the median per-step time is reported


def _make_engine(model, B, context, steps, tp, allreduce, seed, prompt=True):
    """A captured DecodeEngine at batch B whose cache holds ``context`` tokens (a prefilled seeded random
    prompt, or a seeded random cache) plus ``steps`` more. Returns (engine, start position)."""
    import torch
    from b200kernels import decode as dec
    eng = dec.DecodeEngine(model, B, context + steps + 16, tp=tp, allreduce=allreduce)
    if prompt:
        g = torch.Generator().manual_seed(seed + 1)
        prompts = torch.randint(0, model.config.vocab_size, (B, context), generator=g)
        eng.prefill(prompts.to(eng.device))
    else:
        eng.fill_random_cache(context, seed=seed + 1)
    eng.capture()
    return eng, context


def _timed_decode(eng, start, K, world, dev, repeats=REPEATS):
    """Median over ``repeats`` timed regions of K graph replays (each from cache position ``start``) of the
    max-over-ranks device time per step, in ms; and the per-region values."""
    import torch
    per = []
    for _ in range(repeats):
        eng.pos.fill_(start)
        _barrier(world, dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(K):
            eng.step()
        e.record()
        torch.cuda.synchronize(dev)
        per.append(_max_over_ranks(s.elapsed_time(e), world, dev) / K)
    return statistics.median(per), per


def _engine_step_bytes(eng, mean_context: float) -> int:
    """HBM bytes one decode step of this engine (this rank) must read: its NF4 weights, the lm_head rows it
    streams, and the K/V of every cached token (mean context over the timed steps)."""
    w = sum(wt.nbytes for layer in eng.w for wt in layer.values())
    head = (eng.lm_w.numel() if eng.lm_fused else eng.model.lm_head.weight.numel()) * 2
    kv = int(eng.B * mean_context * eng.KVH * eng.D * 2 * 2 * eng.L)
    return w + head + kv


def _hf_decode(model, B, steps, patched, seed, dev):
    """tok/s of the Hugging Face forward with a DynamicCache (the reference's decode_step loop,
    profiling/common.py:80-85) on this GPU: stock, or after the drop-in patch."""
    import torch
    from transformers.cache_utils import DynamicCache
    from b200kernels import patch
    g = torch.Generator().manual_seed(seed + 11)
    ids = torch.randint(0, model.config.vocab_size, (B, PROMPT), generator=g).to(dev)
    if patched:
        patch.patch_attention()
        patch.patch_linear4bit(model, verbose=False)
    try:
        with torch.inference_mode():
            past = DynamicCache()
            out = model(input_ids=ids, past_key_values=past, use_cache=True, logits_to_keep=1)
            nxt = out.logits[:, -1:].argmax(-1)
            for _ in range(2):
                out = model(input_ids=nxt, past_key_values=past, use_cache=True)
                nxt = out.logits[:, -1:].argmax(-1)
            torch.cuda.synchronize(dev)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            s.record()
            for _ in range(steps):
                out = model(input_ids=nxt, past_key_values=past, use_cache=True)
                nxt = out.logits[:, -1:].argmax(-1)
            e.record()
            torch.cuda.synchronize(dev)
            wall = time.perf_counter() - t0
    finally:
        if patched:
            patch.unpatch_attention()
            patch.unpatch_linear4bit(model)
    ms = s.elapsed_time(e) / steps
    return {"batch": B, "tok_s": round(B / (ms / 1e3), 2), "ms_per_step": round(ms, 3),
            "wall_tok_s": round(B * steps / wall, 2), "steps": steps}


def _op_measurements(dev, peak):
    """The two single-op configurations on this GPU (us per launch, each launch reading different
    weights / caches, rotated through more than 2x L2; graph of launches, CUDA events)."""
    import torch
    from b200kernels.decode_attention import decode_attention
    from b200kernels.linear4bit import quantize_nf4
    from b200kernels.nf4_gemm import NF4Weight
    N, K, M = 14336, 4096, 4
    ws = []
    for c in range(8):
        w = (torch.randn(N, K, generator=torch.Generator().manual_seed(100 + c)) * 0.02).to(dev)
        packed, qs = quantize_nf4(w, nested=False)
        prm = torch.nn.Parameter(packed, requires_grad=False)
        prm.quant_state = qs
        ws.append(NF4Weight(prm))
        del w
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(4)).half().to(dev)
    us = _graph_time_us([lambda w=w: w.matmul(x) for w in ws])
    nbytes = ws[0].nbytes + x.numel() * 2 + M * N * 2
    nf4 = {"config": "M=4, 14336x4096, plain fp32 absmax (no double quant), fp16", "us": round(us, 3),
           "algorithmic_bytes": nbytes, "GBps": round(nbytes / us / 1e3, 1),
           "frac_of_peak": round(nbytes / us / 1e3 / peak, 4)}
    del ws
    g = torch.Generator().manual_seed(2048)
    B, S = 8, 2048
    lens = torch.randint(512, S + 1, (B,), generator=g).to(torch.int32)
    cases = [tuple(torch.randn(sh, generator=g).half().to(dev) for sh in ((B, 32, 1, 128), (B, 8, S, 128), (B, 8, S, 128)))
             for _ in range(5)]
    sl = lens.to(dev)
    us = _graph_time_us([lambda c=c: decode_attention(*c, 128 ** -0.5, seqlens=sl) for c in cases])
    nbytes = int(lens.sum()) * 8 * 128 * 2 * 2 + B * 32 * 128 * 2 * 2
    att = {"config": "B=8, 32 q / 8 KV heads, D=128, S=2048, lengths U[512, 2048] (seeded), fp16", "us": round(us, 3),
           "algorithmic_bytes": nbytes, "GBps": round(nbytes / us / 1e3, 1),
           "frac_of_peak": round(nbytes / us / 1e3 / peak, 4)}
    del cases
    torch.cuda.empty_cache()
    return nf4, att


def _tp_parity(eng, model, prompts, T, tp, world, rank, dev):
    """Greedy T steps of the tensor-parallel engine (all ranks), then on rank 0 the single-GPU engine
    consumes the same tokens (teacher-forced) and its argmax / logits are compared."""
    import torch
    from b200kernels import decode as dec
    first = eng.prefill(prompts)
    toks, logits = [first.clone()], []
    for _ in range(T):
        toks.append(eng.step().clone())
        logits.append(eng.full_logits().float().clone())
    eng.check_peers()
    res = None
    if rank == 0:
        single = dec.DecodeEngine(model, eng.B, PROMPT + T + 16)
        preds, lg = single.teacher_forced(prompts, torch.stack(toks, 1))
        ltp = torch.stack(logits, 1)
        res = {"steps": T, "batch": eng.B, "argmax_agreement": round((preds == torch.stack(toks[1:], 1)).float().mean().item(), 4),
               "max_abs_logit_diff_over_std": round(((ltp - lg).abs().max() / lg.std()).item(), 5),
               "rms_logit_diff_over_std": round(((ltp - lg).pow(2).mean().sqrt() / lg.std()).item(), 6),
               "reference": "single-GPU DecodeEngine, teacher-forced on the tensor-parallel tokens"}
        del single
        torch.cuda.empty_cache()
    _barrier(world, dev)
    return res


def run_b200(args):
    import torch
    from b200kernels import decode as dec

    rank, world, dev, tp = _init_ranks(args)
    B, K, W = args.batch, args.steps, args.warmup
    model = dec.build_random_mistral(seed=args.seed, num_hidden_layers=args.layers)
    context = args.context or PROMPT
    extra = K + W + 16
    eng, start = _make_engine(model, B, context, extra, tp, args.allreduce, args.seed, prompt=not args.context)
    clk = ClockSampler(dev.index).start()
    # keep the GPU busy until nvidia-smi reports (its start-up takes ~1 s); every rank takes the same
    # number of steps (the ranks agree on "not ready" through a max over ranks), always from the start
    # position so no step runs past the cache
    t_wait = time.perf_counter()
    while True:
        waiting = clk.proc is not None and not clk.lines and time.perf_counter() - t_wait < 15
        if _max_over_ranks(1.0 if waiting else 0.0, world, dev) == 0.0:
            break
        eng.pos.fill_(start)
        for _ in range(8):
            eng.step()
        torch.cuda.synchronize(dev)
    eng.pos.fill_(start)
    for _ in range(W):
        eng.step()
    _barrier(world, dev)

    # ---- device-resident throughput: median of REPEATS regions of K steps (clock samples kept only
    # inside this window, padded 50 ms)
    profile_region = os.environ.get("B2D_PROFILE_STEPS") == "1"   # ncu --profile-from-start off
    if profile_region:
        torch.cuda.profiler.start()
    w0 = time.perf_counter()
    ms, per = _timed_decode(eng, start, K, world, dev)
    w1 = time.perf_counter()
    if profile_region:
        torch.cuda.profiler.stop()
    clk.window = (w0 - 0.05, w1 + 0.05)
    value = B / (ms / 1e3)

    # ---- end to end through the step API: ids host->device, next ids device->host, every step
    host_in = torch.empty(B, dtype=torch.long).pin_memory()
    host_out = torch.empty(B, dtype=torch.long).pin_memory()
    e2e_ms = []
    e2e_wall = 0.0
    for _ in range(3):
        eng.pos.fill_(start)
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
        e2e_wall = time.perf_counter() - t0
        e2e_ms.append(_max_over_ranks(se.elapsed_time(ee), world, dev) / K)
    e2e = B / (statistics.median(e2e_ms) / 1e3)
    clk.stop()
    _barrier(world, dev)

    # ---- roofline: the model's gate_proj matmuls (this rank's 14336/N x 4096 NF4 shards) at batch B,
    # launched back to back from a CUDA graph on the bench stream and timed with events on that stream
    # (no host gaps), each launched as the decode step launches its GEMMs (programmatic dependent launch
    # with static weights: a launch's prologue overlaps the previous launch's tail); consecutive launches
    # read different weights, so every launch streams its weights from HBM.
    from b200kernels import _lib as L
    from b200kernels.nf4_gemm import NF4Group
    x = torch.randn(B, 4096, generator=torch.Generator().manual_seed(3)).half().to(dev)
    gates = [wd["gate"] for wd in eng.w]
    ggrps = [NF4Group([wgt]) for wgt in gates]
    st = torch.cuda.Stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(st):
        ys = [gr.matmul(x)[0] for gr in ggrps]
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        for gr, y in zip(ggrps, ys):
            gr.matmul(x, [y], flags=L.LAUNCH_PDL | L.STATIC_WEIGHTS)
    durs = []
    for _ in range(REPEATS):
        with torch.cuda.stream(st):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            graph.replay()
            b.record(st)
        b.synchronize()
        durs.append(a.elapsed_time(b) * 1e3 / len(gates))
    us = statistics.median(durs)
    del graph
    alg = gates[0].nbytes + x.numel() * 2 + B * gates[0].N * 2
    peak, peak_kind = measured_peaks()
    achieved = alg / (us * 1e-6) / 1e9

    # ---- our kernel launches per step: per layer 2 add+RMSNorm, RoPE + KV append (inside the attention
    # partial launch when the engine folds it in), attention partial + combine (one launch with
    # B2D_ATTN_COMBINE=fused) and the NF4 launches (q/k/v,
    # o, gate/up, down at B <= 8; else 7 NF4 launches and SiLU*mul), plus the all-reduces under TP; plus the
    # final add+RMSNorm
    glue = (3 if eng.attn_flags & L.ATTN_FUSED_COMBINE else 4) if eng.attn_append else 5
    per_layer = (glue + 4) if eng.pair else (glue + 7 + 1)
    if tp is not None and not eng.ar_fused:   # fused: the GEMMs push, the add+RMSNorm launches sum
        per_layer += 2
    launches_per_step = args.layers * per_layer + 1 + (1 if eng.lm_fused else 0)   # + final norm (+ lm_head)

    extras = {}
    g = torch.Generator().manual_seed(args.seed + 1)
    prompts = torch.randint(0, model.config.vocab_size, (B, PROMPT), generator=g).to(dev)
    if tp is not None and not args.context:
        extras["tp_parity"] = _tp_parity(eng, model, prompts, 16, tp, world, rank, dev)
    eng.graph = None   # a graph holding NCCL calls must go before the process group
    del eng
    torch.cuda.empty_cache()
    if not args.no_configs and not args.context:
        Kc = min(K, 32)
        if world == 1:
            e1, s1 = _make_engine(model, 1, PROMPT, Kc + 16, None, args.allreduce, args.seed)
            for _ in range(3):
                e1.step()
            m1, _ = _timed_decode(e1, s1, Kc, world, dev)
            extras["batch1"] = {"tok_s": round(1 / (m1 / 1e3), 2), "ms_per_step": round(m1, 4), "steps": Kc,
                                "config": "batch 1, prompt 256 (config 3)"}
            del e1
            torch.cuda.empty_cache()
            # config 4: batch 8 after a 32768-token seeded random cache
            LC = 32768
            el, sl_ = _make_engine(model, 8, LC, Kc + 16, None, args.allreduce, args.seed, prompt=False)
            for _ in range(3):
                el.step()
            ml, _ = _timed_decode(el, sl_, Kc, world, dev)
            from b200kernels.decode_attention import decode_attention
            qa = torch.randn(8, 32, 1, 128, generator=torch.Generator().manual_seed(5)).half().to(dev)
            lens = torch.full((8,), LC, dtype=torch.int32, device=dev)
            att_us = _graph_time_us([lambda i=i: decode_attention(qa, el.k_cache[i], el.v_cache[i], 128 ** -0.5,
                                                                  seqlens=lens) for i in range(8)])
            att_bytes = 8 * LC * 8 * 128 * 2 * 2 + 8 * 32 * 128 * 2 * 2
            step_bytes = _engine_step_bytes(el, LC + Kc / 2)
            extras["long_context"] = {
                "config": "batch 8, 32768-token seeded random KV cache per sequence (config 4)", "steps": Kc,
                "tok_s": round(8 / (ml / 1e3), 2), "ms_per_step": round(ml, 4),
                "step_bytes": step_bytes, "step_GBps": round(step_bytes / ml / 1e6, 1),
                "attention_us_per_launch": round(att_us, 3),
                "attention_frac_of_peak": round(att_bytes / att_us / 1e3 / peak, 4)}
            del el
            torch.cuda.empty_cache()
        # config 5: batch 64 after a 4096-token cache (every N)
        C5 = 4096
        e5, s5 = _make_engine(model, 64, C5, Kc + 16, tp, args.allreduce, args.seed, prompt=False)
        for _ in range(3):
            e5.step()
        m5, _ = _timed_decode(e5, s5, Kc, world, dev)
        e5.check_peers()
        b5 = _engine_step_bytes(e5, C5 + Kc / 2)
        extras["tp_config5"] = {"config": f"batch 64, 4096-token seeded random KV cache, tp{world} (config 5)",
                                "steps": Kc, "tok_s": round(64 / (m5 / 1e3), 2), "ms_per_step": round(m5, 4),
                                "per_gpu_step_bytes": b5, "per_gpu_GBps": round(b5 / m5 / 1e6, 1),
                                "per_gpu_frac_of_peak": round(b5 / m5 / 1e6 / peak, 4)}
        e5.graph = None
        del e5
        torch.cuda.empty_cache()
        if world == 1:
            extras["stock_hf"] = [_hf_decode(model, b, 8, False, args.seed, dev) for b in (1, 8)]
            extras["patched_hf"] = [_hf_decode(model, b, 16, True, args.seed, dev) for b in (1, 8)]
            nf4, att = _op_measurements(dev, peak)
            extras["nf4_op"], extras["attention_op"] = nf4, att

    cpu = None
    if world == 1 and rank == 0:   # the reference CPU path on the host, at N=1 only
        cpu = cpu_reference(B, 32)
    _barrier(world, dev)
    if rank == 0:
        shard = "" if world == 1 else f" (rank-0 shard {gates[0].N}x{gates[0].K})"
        cfg = headline_config(B, world, args.layers, "fused" if (tp is not None and args.allreduce == "fused")
                              else args.allreduce)
        if args.context:
            cfg.update(workload=f"Mistral-7B-shaped NF4 greedy decode, batch {B}, {context}-token seeded random KV "
                                f"cache, {args.layers} layers", prompt=None, context=context)
        line = {"metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": K,
                "warmup": W, "ms_per_step": round(ms, 4), "timed_regions_ms_per_step": [round(v, 4) for v in per],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
                "data": "synthetic (seeded random prompts, random-init N(0, 0.02^2) weights)",
                "config": cfg,
                "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": B * 8,
                        "d2h_bytes_per_step": B * 8, "wall_s": round(e2e_wall, 4)},
                "roofline": {"bound": "hbm", "kernel": "nf4_gemm_pipe_kernel (gate_proj" + shard + ", nested, "
                                                       "decode-step launch mode)",
                             "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                             "frac": round(achieved / peak, 4),
                             "traffic": traffic_from_profile() if world == 1 else None,
                             "algorithmic_bytes_per_launch": alg, "avg_launch_us": round(us, 3)},
                "cpu_baseline": cpu,
                "gpu_launches": launches_per_step * K, "gpu_launches_per_step": launches_per_step,
                "clocks": clk.summary(), **extras}
        print(json.dumps(line), flush=True)
    if tp is not None and tp.peer_errors():
        raise SystemExit(f"rank {rank}: {tp.peer_errors()} timed-out all-reduce waits; the run is invalid")
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
                if args.pdl:   # as the decode step launches it: programmatic dependent launch, static weights
                    from b200kernels import _lib as L
                    from b200kernels.nf4_gemm import NF4Group
                    grps = [NF4Group([w]) for w in ws]
                    yo = torch.empty(M, N, dtype=x.dtype, device=dev)
                    us = _graph_time_us([lambda gr=gr: gr.matmul(x, [yo], flags=L.LAUNCH_PDL | L.STATIC_WEIGHTS)
                                         for gr in grps])
                else:
                    us = _graph_time_us([lambda w=w: w.matmul(x) for w in ws])
                nbytes = ws[0].nbytes + x.numel() * 2 + M * N * 2
                print(json.dumps({"kernel": "nf4_gemm", "N": N, "K": K, "M": M, "nested": not args.plain, "pdl": args.pdl,
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
                nbytes = n_keys * 8 * 128 * 2 * 2 + B * 32 * 128 * 2 * 2
                for ch in [int(c) for c in args.chunks.split(",")]:   # 0: the default split choice
                    kw = {"chunk": ch} if ch > 0 else {}
                    us = _graph_time_us([lambda c=c: decode_attention(*c, 128 ** -0.5, seqlens=lens, **kw)
                                         for c in cases])
                    print(json.dumps({"kernel": "gqa_decode", "B": B, "S": S, "ragged": bool(args.ragged),
                                      "chunk": ch or "default", "us": round(us, 2), "GBps": round(nbytes / us / 1e3, 1),
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
    ap.add_argument("--chunks", default="0", help="attention: keys per split to sweep (0 = the default choice)")
    ap.add_argument("--plain", action="store_true", help="fp32 absmax instead of double quantisation")
    ap.add_argument("--profile-iters", type=int, default=0)
    ap.add_argument("--pdl", action="store_true",
                    help="nf4 micro-benchmark: launch as the decode step does (programmatic dependent launch, "
                         "static weights)")
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
    ap.add_argument("--no-configs", action="store_true",
                    help="headline decode only (skip batch1 / long_context / tp_config5 / HF / single-op measurements)")
    args = ap.parse_args()
    if args.kernel:
        run_kernels(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
