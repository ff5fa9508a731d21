"""GPU (one device): the tensor-parallel all-reduce fused into the NF4 GEMM epilogue
(``b2d_nf4_gemm_multi`` mode B2D_SEG_ALLREDUCE) and its consumer ``b2d_allreduce_add_rmsnorm``.

The ranks of a world of 1, 2, 4 or 8 are emulated on one GPU: each rank's buffer is a plain device
allocation, every rank's GEMM pushes its partial product into all buffers, and only then (stream
order, nothing in flight) does each rank's consumer run, so no kernel ever waits for another launch.
Bar: bit-identical to the unfused sequence -- each rank's GEMM output rounded to fp16, summed over
ranks in rank order in fp32 and rounded once (what ``b2d_allreduce`` computes), then
``b2d_add_rmsnorm`` -- for every rank, over several steps and sites (both epoch parities).
The timeout path: a consumer whose peer never pushed gives up after its bounded polls, records the
error in its buffer and returns; the next call on that buffer returns without polling.
"""
import ctypes
import time

import pytest
import torch

from b200kernels import _lib
from b200kernels.glue import add_rmsnorm
from b200kernels.linear4bit import quantize_nf4
from b200kernels.nf4_gemm import NF4Group, NF4Weight

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def weight(N, K, nested, seed, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(N, K, generator=g) * 0.02).to(DEV)
    packed, qs = quantize_nf4(w.to(dtype), nested=nested)
    p = torch.nn.Parameter(packed, requires_grad=False)
    p.quant_state = qs
    return NF4Weight(p)


class World:
    """``world`` emulated ranks' all-reduce buffers on one GPU and their epilogue descriptors."""

    def __init__(self, world, rows, cols, sites, dtype=torch.float16):
        n_max = 2 * ((rows + 1) // 2) * cols
        n_max += -n_max % 8
        nbytes = _lib.load().b2d_allreduce_buffer_bytes(n_max, world, _lib.dtype_code(dtype))
        assert nbytes > 0
        self.bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=DEV) for _ in range(world)]
        self.ptrs = (ctypes.c_void_p * world)(*[b.data_ptr() for b in self.bufs])
        self.step = torch.zeros(1, dtype=torch.int64, device=DEV)
        self.eps = {}
        for r in range(world):
            for s in range(sites):
                e = _lib.AllreduceEpilogue()
                e.peer_bufs, e.rank, e.world, e.n_max = self.ptrs, r, world, n_max
                e.step, e.site, e.sites = self.step.data_ptr(), s, sites
                self.eps[r, s] = e

    def errors(self, rank):
        return int(self.bufs[rank][256:260].view(torch.int32).item())


def consume(ep, residual, weight_, eps, out, flags=0):
    M, D = residual.shape
    _lib.call("b2d_allreduce_add_rmsnorm", ctypes.byref(ep), residual.data_ptr(), residual.stride(0),
              weight_.data_ptr(), float(eps), out.data_ptr(), out.stride(0), M, D, _lib.dtype_code(residual.dtype),
              flags, _lib.stream_ptr(residual.device))


@pytest.mark.parametrize("kernel", ["register", "tma"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("M", [1, 3, 8])
@pytest.mark.parametrize("nested", [True, False])
def test_fused_allreduce_matches_unfused(world, M, nested, kernel, monkeypatch):
    if kernel == "tma":   # both the pushing GEMM and the unfused comparison run the TMA-staged kernel
        monkeypatch.setenv("B2D_NF4_KERNEL", "tma")
    N, Kr, sites, eps = 1024, 512, 2, 1e-5
    ws = {(r, s): weight(N, Kr, nested, 100 * s + r) for r in range(world) for s in range(sites)}
    groups = {k: NF4Group([w], mode="allreduce") for k, w in ws.items()}
    plain = {k: NF4Group([w]) for k, w in ws.items()}
    wn = (1 + 0.1 * torch.randn(N, generator=torch.Generator().manual_seed(9))).half().to(DEV)
    W = World(world, M, N, sites)
    res_ref = torch.randn(M, N, generator=torch.Generator().manual_seed(1)).half().to(DEV)
    res = [res_ref.clone() for _ in range(world)]
    gen = torch.Generator().manual_seed(M * 10 + world)
    for step in range(3):
        for s in range(sites):
            xs = [torch.randn(M, Kr, generator=gen).half().to(DEV) for _ in range(world)]
            flags = _lib.LAUNCH_PDL | _lib.STATIC_WEIGHTS if (step + s) % 2 else 0
            for r in range(world):
                groups[r, s].matmul(xs[r], flags=flags, epilogue=W.eps[r, s])
            outs = [torch.full((M, N), float("nan"), dtype=torch.float16, device=DEV) for _ in range(world)]
            for r in range(world):
                consume(W.eps[r, s], res[r], wn, eps, outs[r], flags=_lib.LAUNCH_PDL if r % 2 else 0)
            # the unfused sequence: per-rank GEMM output, rank-order fp32 sum, one rounding, add+RMSNorm
            parts = [plain[r, s].matmul(xs[r])[0] for r in range(world)]
            acc = torch.zeros(M, N, dtype=torch.float32, device=DEV)
            for p in parts:
                acc += p.float()
            out_ref = torch.empty(M, N, dtype=torch.float16, device=DEV)
            add_rmsnorm(res_ref, wn, eps, out_ref, x=acc.half())
            torch.cuda.synchronize()
            for r in range(world):
                assert torch.equal(res[r], res_ref), (step, s, r)
                assert torch.equal(outs[r], out_ref), (step, s, r)
        W.step.add_(1)
    assert all(W.errors(r) == 0 for r in range(world))


def test_fused_allreduce_bf16_and_odd_hidden():
    world, M, N, Kr = 2, 5, 1056, 256   # N = 33 row groups of 32
    dt = torch.bfloat16
    ws = [weight(N, Kr, True, 40 + r, dt) for r in range(world)]
    groups = [NF4Group([w], mode="allreduce") for w in ws]
    W = World(world, M, N, 1, dt)
    wn = torch.ones(N, dtype=dt, device=DEV)
    res0 = torch.randn(M, N, generator=torch.Generator().manual_seed(2)).to(dt).to(DEV)
    xs = [torch.randn(M, Kr, generator=torch.Generator().manual_seed(3 + r)).to(dt).to(DEV) for r in range(world)]
    for r in range(world):
        groups[r].matmul(xs[r], epilogue=W.eps[r, 0])
    res = [res0.clone() for _ in range(world)]
    outs = [torch.empty(M, N, dtype=dt, device=DEV) for _ in range(world)]
    for r in range(world):
        consume(W.eps[r, 0], res[r], wn, 1e-6, outs[r])
    acc = torch.zeros(M, N, dtype=torch.float32, device=DEV)
    for r in range(world):
        acc += NF4Group([ws[r]]).matmul(xs[r])[0].float()
    out_ref = torch.empty_like(outs[0])
    add_rmsnorm(res0, wn, 1e-6, out_ref, x=acc.to(dt))
    torch.cuda.synchronize()
    for r in range(world):
        assert torch.equal(res[r], res0) and torch.equal(outs[r], out_ref), r


def test_fused_allreduce_missing_peer_times_out():
    """Rank 1 never pushes: rank 0's consumer polls a bounded number of times, records the timeout in
    its buffer's error word and returns (its output is then invalid); a second call returns at once."""
    world, M, N, Kr = 2, 2, 256, 256
    w = weight(N, Kr, True, 7)
    W = World(world, M, N, 1)
    x = torch.randn(M, Kr, generator=torch.Generator().manual_seed(4)).half().to(DEV)
    NF4Group([w], mode="allreduce").matmul(x, epilogue=W.eps[0, 0])
    res = torch.zeros(M, N, dtype=torch.float16, device=DEV)
    out = torch.empty_like(res)
    wn = torch.ones(N, dtype=torch.float16, device=DEV)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    consume(W.eps[0, 0], res, wn, 1e-5, out)
    torch.cuda.synchronize()
    first = time.perf_counter() - t0
    assert W.errors(0) > 0
    assert first < 30, first
    t0 = time.perf_counter()
    consume(W.eps[0, 0], res, wn, 1e-5, out)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 0.5
    # the context is still usable
    assert torch.equal(torch.ones(4, device=DEV).sum(), torch.tensor(4.0, device=DEV))


def test_fused_allreduce_rejects_bad_descriptors():
    w = weight(256, 256, True, 1)
    g = NF4Group([w], mode="allreduce")
    x = torch.randn(2, 256).half().to(DEV)
    W = World(2, 2, 256, 1)
    bad = _lib.AllreduceEpilogue()
    ctypes.pointer(bad)[0] = W.eps[0, 0]
    bad.world = 9
    with pytest.raises(_lib.B2DError):
        g.matmul(x, epilogue=bad)
    bad.world, bad.site = 2, 1            # site outside [0, sites)
    with pytest.raises(_lib.B2DError):
        g.matmul(x, epilogue=bad)
    bad.site, bad.n_max = 0, 256          # room for 128 words per rank, the GEMM needs 256
    with pytest.raises(_lib.B2DError):
        g.matmul(x, epilogue=bad)
    res = torch.zeros(2, 256, dtype=torch.float16, device=DEV)
    with pytest.raises(_lib.B2DError):
        consume(bad, res, torch.ones(256, dtype=torch.float16, device=DEV), 1e-5, torch.empty_like(res))
    assert W.errors(0) == 0
