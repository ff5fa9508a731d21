"""Fused NF4 dequant + skinny matmul on B200, behind the reference's ``NF4Weight`` surface.

Mirrors ``profiling/kernels/nf4_gemm.py`` of the reference:

* ``NF4Weight(param)`` (reference ``nf4_gemm.py:77-92``) -- a zero-copy view of one
  bitsandbytes ``Linear4bit`` weight: ``param.data`` (packed nibbles) and
  ``param.quant_state.{quant_type, blocksize, shape, nested, absmax, code, offset,
  state2.{blocksize, code, absmax}}``. Same format assertions, relaxed shape limits
  (``N % 16 == 0``, ``K % 64 == 0`` instead of ``N % 64``, ``K % 256``).
* ``NF4Weight.matmul(x)`` (reference ``nf4_gemm.py:94-106``) -- ``x[..., K] -> [..., N]``.
  The reference always returns bf16; this returns ``x.dtype`` (fp16 or bf16) and accepts up to
  ``MAX_M = 64`` rows (the reference: 8).
* ``calibrate(module, w, min_m, max_m)`` (reference ``nf4_gemm.py:109-119``) -- times the
  module's stock forward against the B200 kernel per M and returns ``(wins, table)``. It is
  informational: the patch routes every M <= MAX_M to the B200 kernel (no per-shape dispatch).
* ``dequantize(...)`` -- bit-exact bitsandbytes dequant on the device (added).

All compute runs in ``libb200decode.so`` (``b2d_nf4_gemm`` / ``b2d_nf4_dequant``); there is no
Python or CPU fallback.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib

_WS: dict = {}


ERR_WORD_OFFSET = 65536 - 64   # workspace byte offset of the TMA-staged kernel's timeout counter


def gemm_errors(device: torch.device) -> int:
    """Timed-out pipeline waits recorded by the TMA-staged NF4 kernel in this stream's workspace (0 when
    healthy; a nonzero count means some launch computed from incomplete weight tiles)."""
    stream = torch.cuda.current_stream(device)
    ws = _WS.get((device.index, stream.cuda_stream))
    return 0 if ws is None else int(ws[ERR_WORD_OFFSET:ERR_WORD_OFFSET + 4].view(torch.int32).item())


def gemm_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-initialised scratch for ``b2d_nf4_gemm``, one per (device, stream). The kernel leaves
    its counters at zero, so the buffer is reused across calls on the same stream."""
    stream = torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _WS[key] = ws
    return ws


class NF4Weight:
    """View of one bitsandbytes NF4 weight for the B200 kernels (reads the tensors in place)."""

    MIN_M, MAX_M = 1, 64

    def __init__(self, param):
        qs = param.quant_state
        assert qs.quant_type == "nf4" and qs.blocksize == 64, (qs.quant_type, qs.blocksize)
        self.N, self.K = (int(s) for s in qs.shape)
        assert self.K % 64 == 0 and self.N % 16 == 0, (self.N, self.K)
        self.packed = param.data.view(-1)
        assert self.packed.dtype == torch.uint8, self.packed.dtype
        self.nested = bool(qs.nested)
        if self.nested:
            assert qs.state2.blocksize == 256, qs.state2.blocksize
            self.absmax, self.code2, self.absmax2 = qs.absmax, qs.state2.code.float().contiguous(), qs.state2.absmax
            self.offset = float(qs.offset)
        else:
            self.absmax = qs.absmax.float()
            self.code2 = self.absmax2 = None
            self.offset = 0.0
        self.code = qs.code.float().contiguous()
        # layout of this view inside the full tensor (a shard changes these; see shard())
        self.ld_packed = self.K // 2
        self.ld_absmax = self.K // 64
        self.gblk_base = 0
        self.gblk_row_stride = self.K // 64

    # --------------------------------------------------------------- shards (tensor parallel)
    @classmethod
    def from_parts(cls, packed, absmax, code, N, K, nested=False, code2=None, absmax2=None, offset=0.0,
                   ld_packed=None, ld_absmax=None, gblk_base=0, gblk_row_stride=None):
        self = cls.__new__(cls)
        self.N, self.K = int(N), int(K)
        self.packed, self.absmax, self.code = packed, absmax, code.float().contiguous()
        self.nested = bool(nested)
        self.code2 = None if code2 is None else code2.float().contiguous()
        self.absmax2, self.offset = absmax2, float(offset)
        self.ld_packed = self.K // 2 if ld_packed is None else int(ld_packed)
        self.ld_absmax = self.K // 64 if ld_absmax is None else int(ld_absmax)
        self.gblk_base = int(gblk_base)
        self.gblk_row_stride = self.K // 64 if gblk_row_stride is None else int(gblk_row_stride)
        return self

    def shard(self, rows: tuple[int, int] | None = None, cols: tuple[int, int] | None = None,
              copy: bool = True) -> "NF4Weight":
        """Rows [r0, r1) (column-parallel split of the output features) and/or columns [k0, k1)
        (row-parallel split of the input features) of this weight. With ``copy`` the shard's packed
        bytes and per-block scales are materialised contiguously (what a tensor-parallel rank keeps);
        ``absmax2`` stays whole and is indexed by the block's position in the full tensor."""
        r0, r1 = rows if rows is not None else (0, self.N)
        k0, k1 = cols if cols is not None else (0, self.K)
        assert (r1 - r0) % 16 == 0 and k0 % 64 == 0 and (k1 - k0) % 64 == 0, (rows, cols)
        p2d = self.packed.view(-1)[: self.N * self.ld_packed].view(self.N, self.ld_packed)
        a2d = self.absmax.view(-1)[: self.N * self.ld_absmax].view(self.N, self.ld_absmax)
        packed = p2d[r0:r1, k0 // 2: k1 // 2]
        absmax = a2d[r0:r1, k0 // 64: k1 // 64]
        if copy:
            packed, absmax = packed.contiguous(), absmax.contiguous()
            ldp, lda = (k1 - k0) // 2, (k1 - k0) // 64
        else:
            ldp, lda = self.ld_packed, self.ld_absmax
        return NF4Weight.from_parts(
            packed, absmax, self.code, r1 - r0, k1 - k0, self.nested, self.code2, self.absmax2, self.offset,
            ldp, lda, self.gblk_base + r0 * self.gblk_row_stride + k0 // 64, self.gblk_row_stride)

    # --------------------------------------------------------------- kernels
    def _weight_args(self):
        return (_lib.ptr(self.packed), self.ld_packed, _lib.ptr(self.absmax), self.ld_absmax, int(self.nested),
                _lib.ptr(self.code2), _lib.ptr(self.absmax2), self.offset, self.gblk_base, self.gblk_row_stride,
                _lib.ptr(self.code))

    def matmul(self, x: torch.Tensor, out: torch.Tensor | None = None, out_dtype=None) -> torch.Tensor:
        """x: [..., K] fp16/bf16 with at most MAX_M rows -> [..., N] in ``out_dtype`` (x.dtype or
        torch.float32; default x.dtype)."""
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.K)
        if x2.stride(-1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
            x2 = x2.contiguous()
        M = x2.shape[0]
        odt = out.dtype if out is not None else (out_dtype or x.dtype)
        y = out if out is not None else torch.empty((M, self.N), device=x.device, dtype=odt)
        if M == 0:
            return y.reshape(*lead, self.N)
        nbytes = _lib.load().b2d_nf4_gemm_workspace_bytes(M, self.N, self.K)
        ws = gemm_workspace(x.device, nbytes)
        _lib.call("b2d_nf4_gemm", x2.data_ptr(), x2.stride(0), *self._weight_args(), y.data_ptr(), y.stride(0),
                  M, self.N, self.K, _lib.dtype_code(x.dtype), _lib.dtype_code(odt), ws.data_ptr(), ws.numel(),
                  _lib.stream_ptr(x.device))
        return y.reshape(*lead, self.N)

    def matmul_simt(self, x: torch.Tensor, out_dtype=None) -> torch.Tensor:
        """CUDA-core variant (M <= 8), kept for the tensor-core vs CUDA-core comparison."""
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.K).contiguous()
        M = x2.shape[0]
        odt = out_dtype or x.dtype
        y = torch.empty((M, self.N), device=x.device, dtype=odt)
        _lib.call("b2d_nf4_gemv_simt", x2.data_ptr(), x2.stride(0), *self._weight_args(), y.data_ptr(),
                  y.stride(0), M, self.N, self.K, _lib.dtype_code(x.dtype), _lib.dtype_code(odt),
                  _lib.stream_ptr(x.device))
        return y.reshape(*lead, self.N)

    def dequantize(self, dtype=torch.float16, out: torch.Tensor | None = None) -> torch.Tensor:
        """[N, K] weights in ``dtype``, bit-identical to bitsandbytes' dequantize_4bit."""
        dev = self.packed.device
        w = out if out is not None else torch.empty((self.N, self.K), device=dev, dtype=dtype)
        _lib.call("b2d_nf4_dequant", *self._weight_args(), w.data_ptr(), w.stride(0), self.N, self.K,
                  _lib.dtype_code(dtype), _lib.stream_ptr(dev))
        return w

    @property
    def nbytes(self) -> int:
        """Bytes one matmul must read for the weight: packed nibbles + per-block scales (+ absmax2)."""
        n = self.N * self.K // 2 + self.N * self.K // 64 * (1 if self.nested else 4)
        if self.nested:
            n += -(-self.N * self.K // 64 // 256) * 4
        return n


class NF4Group:
    """Several NF4 weights applied to one activation in a single launch (``b2d_nf4_gemm_multi``;
    no counterpart in the reference, which runs one kernel per projection).

    ``mode="independent"``: ``outs[i] = x @ W_i^T`` (q/k/v of a decoder layer).
    ``mode="silu_mul"``: two weights of equal shape, ``out = silu(x @ W_0^T) * (x @ W_1^T)`` with the
    model-dtype rounding of a Mistral MLP (gate/up fused with the SwiGLU).
    ``mode="allreduce"``: one weight (a row-parallel shard); the product goes to the tensor-parallel
    peers instead of an output (``matmul(x, epilogue=...)``, summed by ``TPGroup.allreduce_add_rmsnorm``).
    Up to ``MAX_M = 8`` rows. ``flags``: ``_lib.LAUNCH_PDL | _lib.STATIC_WEIGHTS``."""

    MAX_M = 8

    def __init__(self, weights: list, mode: str = "independent"):
        assert 1 <= len(weights) <= 4 and mode in ("independent", "silu_mul", "allreduce"), (len(weights), mode)
        w0 = weights[0]
        for w in weights:
            assert w.K == w0.K and w.nested == w0.nested, "segments must share K and the nested flag"
            assert torch.equal(w.code, w0.code), "segments must share the NF4 codebook"
        self.mode = {"independent": _lib.SEG_INDEPENDENT, "silu_mul": _lib.SEG_SILU_MUL,
                     "allreduce": _lib.SEG_ALLREDUCE}[mode]
        if self.mode == _lib.SEG_SILU_MUL:
            assert len(weights) == 2 and weights[0].N == weights[1].N
        if self.mode == _lib.SEG_ALLREDUCE:
            assert len(weights) == 1
        self.weights = list(weights)
        self.K, self.nested = w0.K, w0.nested
        self.Ns = [w.N for w in weights]
        self.n_out = [weights[0].N] if self.mode == _lib.SEG_SILU_MUL else self.Ns
        import ctypes
        self._code_host = (ctypes.c_float * 16)(*w0.code.float().cpu().tolist())   # codebook passed by value
        self._segs = (_lib.Nf4Segment * len(weights))()
        # segments whose double-quant tables hold the same values share one table (the TMA-staged kernel
        # keeps a single table per launch)
        same_code2 = w0.nested and all(torch.equal(w.code2, w0.code2) for w in weights)
        for i, w in enumerate(weights):
            sg = self._segs[i]
            sg.packed, sg.ld_packed = _lib.ptr(w.packed), w.ld_packed
            sg.absmax, sg.ld_absmax = _lib.ptr(w.absmax), w.ld_absmax
            sg.code2 = _lib.ptr(w0.code2 if same_code2 else w.code2)
            sg.absmax2, sg.offset = _lib.ptr(w.absmax2), w.offset
            sg.gblk_base, sg.gblk_row_stride = w.gblk_base, w.gblk_row_stride
            sg.code, sg.N = _lib.ptr(w.code), w.N

    @property
    def nbytes(self) -> int:
        return sum(w.nbytes for w in self.weights)

    def matmul(self, x: torch.Tensor, outs: list | None = None, flags: int = 0, epilogue=None) -> list:
        """x [M, K] (row stride multiple of 8) -> list of outputs [M, N_i] (or one for silu_mul);
        mode "allreduce": no outputs, ``epilogue`` (a ``_lib.AllreduceEpilogue``) says where to send."""
        assert x.dim() == 2 and x.shape[1] == self.K and x.stride(1) == 1, tuple(x.shape)
        M = x.shape[0]
        if self.mode == _lib.SEG_ALLREDUCE:
            assert epilogue is not None
            self._segs[0].y, self._segs[0].ldy = None, self.Ns[0]
            nbytes = _lib.load().b2d_nf4_gemm_workspace_bytes(max(M, 1), sum(self.Ns), self.K)
            ws = gemm_workspace(x.device, nbytes)
            dt = _lib.dtype_code(x.dtype)
            _lib.call("b2d_nf4_gemm_multi", x.data_ptr(), x.stride(0), self._segs, 1, int(self.nested), M, self.K,
                      dt, dt, self.mode, flags, self._code_host, C.byref(epilogue), ws.data_ptr(), ws.numel(),
                      _lib.stream_ptr(x.device))
            return []
        if outs is None:
            outs = [torch.empty((M, n), device=x.device, dtype=x.dtype) for n in self.n_out]
        for i, o in enumerate(outs):
            self._segs[i].y, self._segs[i].ldy = o.data_ptr(), o.stride(0)
        if self.mode == _lib.SEG_SILU_MUL:
            self._segs[1].y, self._segs[1].ldy = outs[0].data_ptr(), outs[0].stride(0)
        nbytes = _lib.load().b2d_nf4_gemm_workspace_bytes(max(M, 1), sum(self.Ns), self.K)
        ws = gemm_workspace(x.device, nbytes)
        dt = _lib.dtype_code(x.dtype)
        _lib.call("b2d_nf4_gemm_multi", x.data_ptr(), x.stride(0), self._segs, len(self.weights), int(self.nested),
                  M, self.K, dt, _lib.dtype_code(outs[0].dtype), self.mode, flags, self._code_host, None,
                  ws.data_ptr(), ws.numel(), _lib.stream_ptr(x.device))
        return outs


def dequantize(param, dtype=torch.float16) -> torch.Tensor:
    """Bit-exact dequant of a bitsandbytes-format NF4 parameter on the device."""
    return NF4Weight(param).dequantize(dtype)


def calibrate(module, w: NF4Weight, min_m: int = 1, max_m: int = 8, iters: int = 20):
    """Time the module's stock forward vs the B200 kernel for each M (L2 flushed between
    launches). Returns ``(wins, table)``: the M values where the kernel is faster and
    ``{M: (stock_us, kernel_us)}``. Informational -- the patch does not dispatch on it."""
    wins, table = set(), {}
    dev = w.packed.device
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    dt = getattr(module, "compute_dtype", torch.float16)
    for M in range(min_m, max_m + 1):
        x = torch.randn(M, 1, w.K, device=dev, dtype=dt)
        res = []
        for fn in (lambda: module.forward_bnb(x), lambda: w.matmul(x)):
            fn()
            ts = []
            for _ in range(iters):
                flush.zero_()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                fn()
                e.record()
                torch.cuda.synchronize(dev)
                ts.append(s.elapsed_time(e) * 1e3)
            res.append(sorted(ts)[len(ts) // 2])
        table[M] = (round(res[0], 1), round(res[1], 1))
        if res[1] < res[0]:
            wins.add(M)
    return wins, table
