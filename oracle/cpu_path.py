"""The reference's decode path on host cores: torch NF4 dequant + matmul, repeat_kv + SDPA.

TEST / BASELINE INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): used by ``bench.py`` as the timed
CPU baseline (``cpu_baseline`` and ``--impl reference``), never by the product.

Per decoder layer (Mistral-shaped, ``profiling/common.py:73-85`` via HF ``MistralDecoderLayer``):
seven NF4 linears, each ``x.float() @ dequant(W).float().T`` with the dequant of
``oracle.nf4_ref`` (``bench_nf4.py:34,38``), and the stock attention ``repeat_kv`` + SDPA in fp32
over the cached keys (``bench_attention.py:40-41``). Glue (RMSNorm, RoPE, SiLU) is omitted: it is
<1% of the work.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from . import attn_ref, nf4_ref


class CpuNF4Linear:
    """One NF4 weight held on the host (bitsandbytes layout) with the reference forward."""

    def __init__(self, N: int, K: int, seed: int, nested: bool = True):
        rng = np.random.default_rng(seed)
        w = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
        self.q = nf4_ref.QuantizedWeight(w, nested)
        self.N, self.K = N, K
        self.code = torch.from_numpy(self.q.code)
        self.packed = torch.from_numpy(self.q.packed)
        self.scales = torch.from_numpy(self.q.scales())          # fp32 per 64-block

    def dequant(self, dtype=torch.float16) -> torch.Tensor:
        p = self.packed
        idx = torch.stack(((p >> 4).long(), (p & 0xF).long()), -1).view(-1, 64)
        return (self.code[idx] * self.scales[:, None]).view(self.N, self.K).to(dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x.float() @ self.dequant().float().T


class CpuDecodeLayer:
    """Mistral-shaped decoder layer on the host, for timing the reference path."""

    def __init__(self, hidden=4096, inter=14336, heads=32, kv_heads=8, head_dim=128, seed=0, nested=True):
        dims = {"q": (heads * head_dim, hidden), "k": (kv_heads * head_dim, hidden), "v": (kv_heads * head_dim, hidden),
                "o": (hidden, heads * head_dim), "gate": (inter, hidden), "up": (inter, hidden), "down": (hidden, inter)}
        self.lin = {n: CpuNF4Linear(N, K, seed * 31 + i, nested) for i, (n, (N, K)) in enumerate(dims.items())}
        self.H, self.KVH, self.D = heads, kv_heads, head_dim

    def forward(self, x: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor) -> torch.Tensor:
        B = x.shape[0]
        q = self.lin["q"].forward(x).view(B, self.H, 1, self.D)
        k = self.lin["k"].forward(x)
        v = self.lin["v"].forward(x)
        del k, v   # the new key/value would be appended to the cache; the cache below already holds them
        a = attn_ref.stock_cpu(q.half(), k_cache, v_cache, self.D ** -0.5).reshape(B, -1)
        h = x.float() + self.lin["o"].forward(a)
        g, u = self.lin["gate"].forward(h), self.lin["up"].forward(h)
        return h + self.lin["down"].forward(torch.nn.functional.silu(g) * u)


def time_decode_layer(batch: int, context: int, reps: int = 1, threads: int | None = None, seed: int = 0):
    """Seconds per decoder layer of the reference path on the host (median of ``reps`` after one
    warm-up), with the thread count used."""
    threads = threads or torch.get_num_threads()
    torch.set_num_threads(threads)
    layer = CpuDecodeLayer(seed=seed)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, 4096, generator=g).half()
    kc = torch.randn(batch, 8, context, 128, generator=g).half()
    vc = torch.randn(batch, 8, context, 128, generator=g).half()
    layer.forward(x, kc, vc)
    ts = []
    for _ in range(reps):
        t = time.perf_counter()
        layer.forward(x, kc, vc)
        ts.append(time.perf_counter() - t)
    return float(np.median(ts)), threads


def time_lm_head(batch: int, vocab: int = 32768, hidden: int = 4096, threads: int | None = None) -> float:
    if threads:
        torch.set_num_threads(threads)
    w = (torch.randn(vocab, hidden) * 0.02).half()
    x = torch.randn(batch, hidden).half()
    (x.float() @ w.float().T).argmax(-1)
    t = time.perf_counter()
    (x.float() @ w.float().T).argmax(-1)
    return time.perf_counter() - t
