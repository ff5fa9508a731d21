"""numpy restatement of the bitsandbytes NF4 storage format and of the reference matmul.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the product never imports this.

Storage format (what the reference kernel reads, ``profiling/kernels/nf4_gemm.py:3-6,48-56``):

* ``W[N, K]`` is flattened row-major and cut into blocks of 64 consecutive weights.
* Each weight is a 4-bit index into a 16-entry codebook ``code``; two indices share one
  byte, the EVEN element in the HIGH nibble and the odd element in the low nibble
  (``nf4_gemm.py:4,55-56``).
* One fp32 scale ("absmax") per block (``nf4_gemm.py:53``), or, with double quantisation,
  an 8-bit index per block into a 256-entry table ``code2`` scaled per group of 256
  blocks by ``absmax2`` and shifted by a scalar ``offset``:
  ``scale = code2[q] * absmax2[blk // 256] + offset`` (``nf4_gemm.py:50-51``).

Dequantisation follows the reference's stock path, ``bitsandbytes.functional
.dequantize_4bit`` (called at ``profiling/kernels/bench_nf4.py:34``): the nested scale is
produced by an 8-bit blockwise dequant (an fp32 multiply) followed by a separate fp32 add
of ``offset``; each weight is then the fp32 product ``code[nib] * scale`` rounded once to
the compute dtype. Every multiply/add below is a separately rounded fp32 operation, which
is what the CUDA kernels reproduce with ``__fmul_rn`` / ``__fadd_rn``.

Quantisation restates the published methods, not bitsandbytes source:
NF4 (Dettmers et al. 2023, "QLoRA", sec. 3 and appendix E) and the signed dynamic 8-bit
map used for double quantisation (Dettmers et al. 2022, "8-bit Optimizers via
Block-wise Quantization", dynamic tree quantisation). Rounding is to the nearest code,
ties to the lower code. The mean used as the double-quant ``offset`` is a float64 sum in
a fixed order (1024 strided partial sums, then those partials in order), so the CUDA
quantiser can reproduce it bit for bit.
"""
from __future__ import annotations

import numpy as np

BLOCK = 64          # weights per absmax block (bitsandbytes blocksize for NF4)
BLOCK2 = 256        # absmax blocks per double-quant group (state2.blocksize)

# The 16 NF4 values as published in the QLoRA paper (appendix E). ``nf4_code_from_quantiles``
# re-derives them from the construction in the paper; tests check the two agree to 1e-6.
NF4_CODE = np.array([
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0], dtype=np.float32)


def nf4_code_from_quantiles(delta: float = 0.9677083) -> np.ndarray:
    """QLoRA's NF4 construction: 8 positive and 7 negative N(0,1) quantiles taken on an
    evenly spaced probability grid from ``delta`` down to 0.5 (the 0.5 end excluded),
    plus an exact zero, normalised into [-1, 1]."""
    from scipy.stats import norm
    pos = norm.ppf(np.linspace(delta, 0.5, 9)[:-1])
    neg = -norm.ppf(np.linspace(delta, 0.5, 8)[:-1])
    vals = np.sort(np.concatenate([pos, [0.0], neg]))
    return (vals / vals.max()).astype(np.float32)


def dynamic_map_signed(exponent_levels: int = 7) -> np.ndarray:
    """Signed dynamic-tree 8-bit map (Dettmers et al. 2022): level ``i`` holds ``2**i``
    linearly spaced fractions (mid-points of ``2**i`` equal bins over [0.1, 1]) scaled by
    ``10**(i - levels + 1)``, mirrored for the sign; 0 and 1 complete the 256 entries."""
    vals = []
    for i in range(exponent_levels):
        n = 2 ** i
        edges = np.linspace(0.1, 1.0, n + 1)
        mids = (edges[:-1] + edges[1:]) / 2.0
        mag = 10.0 ** (i - exponent_levels + 1)
        vals.extend((mag * mids).tolist())
        vals.extend((-mag * mids).tolist())
    vals.extend([0.0, 1.0])
    out = np.sort(np.asarray(vals, dtype=np.float64)).astype(np.float32)
    assert out.size == 256
    return out


# ----------------------------------------------------------------------------- rounding

def nearest_code(v: np.ndarray, code: np.ndarray) -> np.ndarray:
    """Index of the nearest entry of the ascending table ``code``; ties go to the lower
    entry. Distances are fp32 subtractions, exactly as the CUDA quantiser computes them."""
    v = np.asarray(v, dtype=np.float32)
    code = np.asarray(code, dtype=np.float32)
    hi = np.searchsorted(code, v, side="left")          # codes strictly below v
    hi_c = np.clip(hi, 1, code.size - 1)
    lo_c = hi_c - 1
    d_lo = (v - code[lo_c]).astype(np.float32)
    d_hi = (code[hi_c] - v).astype(np.float32)
    idx = np.where(d_hi < d_lo, hi_c, lo_c)
    idx = np.where(hi == 0, 0, idx)
    idx = np.where(hi >= code.size, code.size - 1, idx)
    return idx.astype(np.uint8)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (nearest, ties to even); returns the raw uint16 bit patterns."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(a)
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint32) << 16).view(np.float32)


def round_to(a32: np.ndarray, dtype: str) -> np.ndarray:
    """fp32 -> compute dtype. fp16 returns float16; bf16 returns uint16 bit patterns."""
    if dtype == "fp16":
        return a32.astype(np.float16)
    if dtype == "bf16":
        return f32_to_bf16_bits(a32)
    raise ValueError(dtype)


def as_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    return a.astype(np.float32) if dtype == "fp16" else bf16_bits_to_f32(a)


# ----------------------------------------------------------------------------- quantise

def fixed_order_mean(a: np.ndarray) -> np.float32:
    """Mean as the CUDA quantiser computes it: 1024 float64 partial sums over a stride-1024
    split (each summed in index order), those partials summed in order, divided in float64,
    rounded to fp32."""
    a = np.asarray(a, dtype=np.float32).astype(np.float64).reshape(-1)
    n = a.size
    pad = (-n) % 1024
    parts = np.concatenate([a, np.zeros(pad)]).reshape(-1, 1024)
    partial = np.zeros(1024, dtype=np.float64)
    for row in parts:                      # row-by-row keeps the per-lane order
        partial = partial + row
    total = 0.0
    for p in partial:
        total = total + p
    return np.float32(total / n)


def quantize_nf4(w: np.ndarray, code: np.ndarray = NF4_CODE):
    """Blockwise NF4 quantisation of a tensor whose element count is a multiple of 64.
    Returns (packed uint8 [numel/2], absmax fp32 [numel/64])."""
    flat = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    assert flat.size % BLOCK == 0, "element count must be a multiple of 64"
    blocks = flat.reshape(-1, BLOCK)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    with np.errstate(divide="ignore"):
        recip = np.where(absmax > 0, np.float32(1.0) / absmax, np.float32(0.0)).astype(np.float32)
    v = (blocks * recip[:, None]).astype(np.float32)
    idx = nearest_code(v, code).reshape(-1)
    packed = ((idx[0::2] << 4) | idx[1::2]).astype(np.uint8)
    return packed, absmax


def double_quant(absmax: np.ndarray, code2: np.ndarray | None = None):
    """Double quantisation of the per-block scales: subtract their mean, then blockwise
    8-bit quantisation (groups of 256) against the signed dynamic map.
    Returns (qabsmax uint8, absmax2 fp32 [ceil(nb/256)], code2 fp32 [256], offset fp32)."""
    code2 = dynamic_map_signed() if code2 is None else np.asarray(code2, np.float32)
    absmax = np.asarray(absmax, dtype=np.float32)
    offset = fixed_order_mean(absmax)
    a = (absmax - offset).astype(np.float32)
    nb = a.size
    ng = (nb + BLOCK2 - 1) // BLOCK2
    pad = np.zeros(ng * BLOCK2, dtype=np.float32)
    pad[:nb] = a
    g = pad.reshape(ng, BLOCK2)
    absmax2 = np.abs(g).max(axis=1).astype(np.float32)
    with np.errstate(divide="ignore"):
        recip = np.where(absmax2 > 0, np.float32(1.0) / absmax2, np.float32(0.0)).astype(np.float32)
    v = (g * recip[:, None]).astype(np.float32).reshape(-1)[:nb]
    q = nearest_code(v, code2)
    return q, absmax2, code2, offset


# ----------------------------------------------------------------------------- dequantise

def block_scales(absmax, nested=False, code2=None, absmax2=None, offset=0.0) -> np.ndarray:
    """fp32 scale per 64-weight block: ``absmax`` directly, or for double quantisation
    ``fp32(fp32(code2[q] * absmax2[b // 256]) + offset)`` with each op rounded."""
    if not nested:
        return np.asarray(absmax, dtype=np.float32)
    q = np.asarray(absmax, dtype=np.uint8).astype(np.int64)
    gi = np.arange(q.size) // BLOCK2
    prod = (np.asarray(code2, np.float32)[q] * np.asarray(absmax2, np.float32)[gi]).astype(np.float32)
    return (prod + np.float32(offset)).astype(np.float32)


def dequantize_f32(packed, scales, code=NF4_CODE, shape=None) -> np.ndarray:
    """The fp32 products ``code[nib] * scale`` (before rounding to the compute dtype)."""
    packed = np.asarray(packed, dtype=np.uint8).reshape(-1)
    idx = np.empty(packed.size * 2, dtype=np.int64)
    idx[0::2] = packed >> 4
    idx[1::2] = packed & 0xF
    vals = np.asarray(code, np.float32)[idx]
    sc = np.repeat(np.asarray(scales, np.float32), BLOCK)
    out = (vals * sc).astype(np.float32)
    return out.reshape(shape) if shape is not None else out


def dequantize(packed, absmax, shape, dtype="fp16", nested=False, code2=None, absmax2=None,
               offset=0.0, code=NF4_CODE) -> np.ndarray:
    """Reference dequant: one rounding of the fp32 product to ``dtype`` (fp16 -> float16,
    bf16 -> uint16 bit patterns)."""
    sc = block_scales(absmax, nested, code2, absmax2, offset)
    return round_to(dequantize_f32(packed, sc, code, shape), dtype)


def dequantize_view(packed2d, absmax2d, k_cols, dtype="fp16", nested=False, code2=None, absmax2=None,
                    offset=0.0, gblk_base=0, gblk_row_stride=None, code=NF4_CODE) -> np.ndarray:
    """Dequant of a strided view of a larger weight (a tensor-parallel shard), as the C ABI defines
    it: row r of the view holds ``k_cols`` weights in ``packed2d[r, :k_cols // 2]`` with per-block
    scales ``absmax2d[r, :k_cols // 64]``; a double-quantised block's group scale is
    ``absmax2[(gblk_base + r * gblk_row_stride + j) // 256]`` -- the block's index in the FULL tensor,
    as the reference kernel indexes it (``profiling/kernels/nf4_gemm.py:50-51``)."""
    packed2d = np.asarray(packed2d, np.uint8)
    n = packed2d.shape[0]
    nb = k_cols // BLOCK
    a = np.asarray(absmax2d)[:, :nb]
    if nested:
        gidx = (gblk_base + np.arange(n)[:, None] * gblk_row_stride + np.arange(nb)[None, :]) // BLOCK2
        prod = (np.asarray(code2, np.float32)[a.astype(np.int64)] * np.asarray(absmax2, np.float32)[gidx])
        sc = (prod.astype(np.float32) + np.float32(offset)).astype(np.float32)
    else:
        sc = a.astype(np.float32)
    out = dequantize_f32(packed2d[:, : k_cols // 2], sc.reshape(-1), code, (n, k_cols))
    return round_to(out, dtype)


def nf4_matmul_ref(x, w_deq, dtype="fp16") -> np.ndarray:
    """The reference path ``x.float() @ dequant(W).float().T`` (``bench_nf4.py:34,38``),
    evaluated in float64 so the oracle itself adds no accumulation error."""
    xf = as_f32(np.asarray(x), dtype).astype(np.float64)
    wf = as_f32(np.asarray(w_deq), dtype).astype(np.float64)
    return xf @ wf.T


class QuantizedWeight:
    """A bitsandbytes-format weight held as numpy arrays (oracle side)."""

    def __init__(self, w: np.ndarray, nested: bool, code=NF4_CODE):
        self.N, self.K = w.shape
        self.packed, absmax = quantize_nf4(w, code)
        self.code = np.asarray(code, np.float32)
        self.nested = nested
        if nested:
            self.absmax, self.absmax2, self.code2, self.offset = double_quant(absmax)
        else:
            self.absmax, self.absmax2, self.code2, self.offset = absmax, None, None, np.float32(0.0)

    def scales(self):
        return block_scales(self.absmax, self.nested, self.code2, self.absmax2, self.offset)

    def dequantize(self, dtype="fp16"):
        return dequantize(self.packed, self.absmax, (self.N, self.K), dtype, self.nested,
                          self.code2, self.absmax2, self.offset, self.code)
