"""CPU: the oracle is pinned against the reference implementation's own outputs (golden fixtures)."""
import glob
from pathlib import Path

import numpy as np
import pytest

from oracle import attn_ref, nf4_ref

GOLDEN = Path(__file__).resolve().parent / "golden"
DEQ = sorted(glob.glob(str(GOLDEN / "nf4_gemm_ref_deq_*.npz")))
GEMM = sorted(set(glob.glob(str(GOLDEN / "nf4_gemm_ref_*.npz"))) - set(DEQ))
ATTN = sorted(glob.glob(str(GOLDEN / "attn_ref_*.npz")))


def _load(path):
    return dict(np.load(path))


def _qw_from(d):
    return dict(packed=d["packed"], absmax=d["absmax"], nested=bool(d["nested"]), code=d["code"],
                code2=d.get("code2"), absmax2=d.get("absmax2"), offset=d.get("offset", np.float32(0)))


def test_nf4_codebook_matches_quantile_construction():
    derived = nf4_ref.nf4_code_from_quantiles()
    np.testing.assert_allclose(derived, nf4_ref.NF4_CODE, atol=1e-6, rtol=0)
    assert nf4_ref.NF4_CODE[7] == 0.0 and np.all(np.diff(nf4_ref.NF4_CODE) > 0)


def test_dynamic_map_is_sorted_signed_and_complete():
    m = nf4_ref.dynamic_map_signed()
    assert m.shape == (256,) and m.dtype == np.float32
    assert np.all(np.diff(m) > 0)
    assert m[-1] == 1.0 and 0.0 in m and m.min() > -1.0


def test_product_codebooks_equal_oracle():
    from b200kernels import linear4bit
    np.testing.assert_array_equal(np.asarray(linear4bit.NF4_CODE, np.float32), nf4_ref.NF4_CODE)
    np.testing.assert_array_equal(linear4bit.dynamic_map_signed().numpy(), nf4_ref.dynamic_map_signed())


@pytest.mark.parametrize("path", DEQ)
def test_dequant_pinned_to_reference_kernel(path):
    """Each weight the reference kernel computes (one-hot x, bf16 store) equals the oracle's fp32
    product code[nib] * scale converted to bf16, bit for bit.

    The Triton CPU interpreter that ran the reference kernel converts fp32 -> bf16 by truncating
    the low 16 bits (compiled for a GPU, the same store rounds to nearest), so the golden values are
    the truncated oracle products. This pins the nibble order, the block/group indexing and the
    ``code2[q]*absmax2[b//256] + offset`` formula: a wrong index or formula differs by far more than
    one bf16 unit."""
    d = _load(path)
    q = _qw_from(d)
    N, K = int(d["N"]), int(d["K"])
    sc = nf4_ref.block_scales(q["absmax"], q["nested"], q["code2"], q["absmax2"], q["offset"])
    w32 = nf4_ref.dequantize_f32(q["packed"], sc, q["code"], (N, K))
    got = (np.ascontiguousarray(w32).view(np.uint32) >> 16).astype(np.uint16)
    np.testing.assert_array_equal(got, d["w_bf16"])


@pytest.mark.parametrize("path", GEMM)
def test_gemm_pinned_to_reference_kernel(path):
    """y = x @ W^T from the oracle (fp64 of the same fp32 weights) matches the reference kernel's
    bf16 output to within its bf16 store (truncating under the interpreter: < 1 unit, 2^-7 relative)."""
    d = _load(path)
    q = _qw_from(d)
    N, K = int(d["N"]), int(d["K"])
    sc = nf4_ref.block_scales(q["absmax"], q["nested"], q["code2"], q["absmax2"], q["offset"])
    w32 = nf4_ref.dequantize_f32(q["packed"], sc, q["code"], (N, K)).astype(np.float64)
    x = nf4_ref.bf16_bits_to_f32(d["x_bf16"]).astype(np.float64)
    y = x @ w32.T
    y_ref = nf4_ref.bf16_bits_to_f32(d["y_bf16"]).astype(np.float64)
    # one truncating bf16 store of the reference output (relative 2^-7) plus fp32 accumulation noise
    assert np.all(np.abs(y_ref - y) <= np.abs(y) * 2.0 ** -7 + 1e-6 * np.abs(y).max())


@pytest.mark.parametrize("path", ATTN)
def test_attention_oracle_matches_reference_stock_formula(path):
    d = _load(path)
    out = attn_ref.gqa_decode_ref(d["q"], d["k"], d["v"], float(d["scale"]), d["seqlens"])
    np.testing.assert_allclose(out, d["out"], atol=2e-6, rtol=0)


def test_attention_stock_cpu_matches_oracle():
    torch = pytest.importorskip("torch")
    g = torch.Generator().manual_seed(5)
    q = torch.randn(2, 8, 1, 64, generator=g).half()
    k = torch.randn(2, 2, 50, 64, generator=g).half()
    v = torch.randn(2, 2, 50, 64, generator=g).half()
    sl = torch.tensor([50, 9], dtype=torch.int32)
    a = attn_ref.stock_cpu(q, k, v, 0.125, sl).numpy()
    b = attn_ref.gqa_decode_ref(q.numpy(), k.numpy(), v.numpy(), 0.125, sl.numpy())
    np.testing.assert_allclose(a, b, atol=2e-6, rtol=0)


def test_nearest_code_is_argmin_with_ties_low():
    rng = np.random.default_rng(0)
    code = nf4_ref.NF4_CODE
    mids = ((code[:-1] + code[1:]) / 2).astype(np.float32)
    v = np.concatenate([rng.uniform(-1.2, 1.2, 5000).astype(np.float32), code, mids, [-5, 5, 0]]).astype(np.float32)
    idx = nf4_ref.nearest_code(v, code)
    d = np.abs(v[:, None].astype(np.float64) - code[None, :].astype(np.float64))
    best = d.min(1)
    # chosen code is a nearest one (fp32 distances can tie where fp64 does not)
    assert np.all(d[np.arange(v.size), idx] <= best + 1e-7)
    exact = v[:, None] == code[None, :]
    hit = exact.any(1)
    assert np.all(idx[hit] == exact[hit].argmax(1))


def test_quantize_roundtrip_error_bound():
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((32, 256)) * 0.02).astype(np.float32)
    packed, absmax = nf4_ref.quantize_nf4(w)
    deq = nf4_ref.dequantize_f32(packed, absmax, nf4_ref.NF4_CODE, w.shape)
    gap = np.diff(nf4_ref.NF4_CODE).max() / 2
    err = np.abs(deq - w).reshape(-1, 64).max(1)
    assert np.all(err <= gap * absmax * (1 + 1e-6))
    # packing: even element in the high nibble
    idx0 = nf4_ref.nearest_code(w.reshape(-1)[:2] / absmax[0], nf4_ref.NF4_CODE)
    assert packed[0] == (idx0[0] << 4) | idx0[1]


def test_double_quant_reconstruction():
    rng = np.random.default_rng(2)
    absmax = rng.uniform(0.03, 0.09, 1000).astype(np.float32)
    q, a2, code2, off = nf4_ref.double_quant(absmax)
    assert a2.shape == (4,) and q.dtype == np.uint8
    rec = nf4_ref.block_scales(q, True, code2, a2, off)
    assert np.abs(rec - absmax).max() < 0.02 * absmax.max()
    assert np.isclose(off, absmax.astype(np.float64).mean(), rtol=1e-6)


def test_fixed_order_mean_exact_for_fp32_inputs():
    rng = np.random.default_rng(3)
    a = rng.uniform(0.01, 0.1, 3001).astype(np.float32)
    m = nf4_ref.fixed_order_mean(a)
    assert m == np.float32(np.sum(a.astype(np.float64)) / a.size)
