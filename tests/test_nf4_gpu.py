"""GPU parity of the NF4 kernels (through the C ABI) against the CPU oracle.

Bars (stated per test): dequant and quantise are bit-exact; the matmul is within
max|y - ref| <= 2e-3 * rms(ref) of the reference path ``x.float() @ dequant(W).float().T`` for an
fp32 output, plus one output unit for an fp16 output; bf16 activations carry bf16's 8-bit
significand, so their bar is 2e-2 * rms(ref).
"""
import glob
from pathlib import Path

import numpy as np
import pytest
import torch

from b200kernels import _lib
from b200kernels.linear4bit import QuantState, dequantize_torch, quantize_nf4
from b200kernels.nf4_gemm import NF4Weight
from oracle import nf4_ref

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
GOLDEN = Path(__file__).resolve().parent / "golden"
TOL_F32 = 2e-3
TOL_BF16 = 2e-2


def _param(packed, qs):
    p = torch.nn.Parameter(packed, requires_grad=False)
    p.quant_state = qs
    return p


def make_weight(N, K, nested, seed=0, scale=0.02):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(N, K, generator=g) * scale).to(DEV)
    packed, qs = quantize_nf4(w, nested=nested)
    return w, _param(packed, qs)


def oracle_state(param):
    qs = param.quant_state
    st = dict(packed=param.data.view(-1).cpu().numpy(), code=qs.code.cpu().numpy(), nested=qs.nested,
              absmax=qs.absmax.cpu().numpy())
    if qs.nested:
        st.update(code2=qs.state2.code.cpu().numpy(), absmax2=qs.state2.absmax.cpu().numpy(),
                  offset=np.float32(qs.offset.cpu().numpy()))
    else:
        st.update(code2=None, absmax2=None, offset=np.float32(0))
    return st


def oracle_dequant(st, shape, dtype):
    return nf4_ref.dequantize(st["packed"], st["absmax"], shape, dtype, st["nested"], st["code2"], st["absmax2"],
                              st["offset"], st["code"])


def bits(t):
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).cpu().numpy().view(np.uint16)
    return t.cpu().numpy()


# ------------------------------------------------------------------------------ format kernels
@pytest.mark.parametrize("N,K", [(64, 256), (128, 4096), (4096, 4096)])
@pytest.mark.parametrize("src", [torch.float32, torch.float16, torch.bfloat16])
def test_quantize_bitexact(N, K, src):
    g = torch.Generator().manual_seed(N + K)
    w = (torch.randn(N, K, generator=g) * 0.02).to(src)
    w[0, :64] = 0          # an all-zero block
    w[1, 3] = 1.5          # an outlier block
    packed, qs = quantize_nf4(w.to(DEV), nested=False)
    p_ref, a_ref = nf4_ref.quantize_nf4(w.float().numpy())
    np.testing.assert_array_equal(packed.view(-1).cpu().numpy(), p_ref)
    np.testing.assert_array_equal(qs.absmax.cpu().numpy(), a_ref)


@pytest.mark.parametrize("nblocks", [1, 255, 1000, 917504])
def test_double_quant_bitexact(nblocks):
    rng = np.random.default_rng(nblocks)
    absmax = rng.uniform(0.02, 0.12, nblocks).astype(np.float32)
    a = torch.from_numpy(absmax).to(DEV)
    code2 = torch.from_numpy(nf4_ref.dynamic_map_signed()).to(DEV)
    q = torch.empty(nblocks, dtype=torch.uint8, device=DEV)
    a2 = torch.empty(-(-nblocks // 256), dtype=torch.float32, device=DEV)
    off = torch.empty((), dtype=torch.float32, device=DEV)
    _lib.call("b2d_nf4_double_quant", a.data_ptr(), nblocks, code2.data_ptr(), q.data_ptr(), a2.data_ptr(),
              off.data_ptr(), _lib.stream_ptr(DEV))
    q_ref, a2_ref, _, off_ref = nf4_ref.double_quant(absmax)
    assert off.item() == off_ref
    np.testing.assert_array_equal(a2.cpu().numpy(), a2_ref)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)


@pytest.mark.parametrize("N,K,nested", [(64, 256, False), (64, 1024, True), (1024, 4096, True),
                                        (14336, 4096, False), (4096, 14336, True)])
@pytest.mark.parametrize("dtype,odt", [(torch.float16, "fp16"), (torch.bfloat16, "bf16")])
def test_dequant_bitexact(N, K, nested, dtype, odt):
    _, p = make_weight(N, K, nested, seed=N ^ K)
    nf = NF4Weight(p)
    got = nf.dequantize(dtype)
    ref = oracle_dequant(oracle_state(p), (N, K), odt)
    np.testing.assert_array_equal(bits(got), ref)
    # the stock torch dequant (the reference path on this machine) is the same bits
    stock = dequantize_torch(p.data, p.quant_state, dtype)
    assert torch.equal(stock.view(torch.int16), got.view(torch.int16))


@pytest.mark.parametrize("path", sorted(glob.glob(str(GOLDEN / "nf4_gemm_ref_deq_*.npz"))))
def test_dequant_against_reference_kernel_golden(path):
    """The reference kernel's per-weight values (bf16, truncating store) vs ours (bf16, nearest):
    identical up to the rounding mode, i.e. at most one bf16 unit apart and never further."""
    d = dict(np.load(path))
    N, K = int(d["N"]), int(d["K"])
    nested = bool(d["nested"])
    absmax = torch.from_numpy(d["absmax"]).to(DEV)
    nf = NF4Weight.from_parts(torch.from_numpy(d["packed"]).to(DEV), absmax, torch.from_numpy(d["code"]).to(DEV),
                              N, K, nested,
                              torch.from_numpy(d["code2"]).to(DEV) if nested else None,
                              torch.from_numpy(d["absmax2"]).to(DEV) if nested else None,
                              float(d["offset"]) if nested else 0.0)
    ours = bits(nf.dequantize(torch.bfloat16)).astype(np.int32)
    gold = d["w_bf16"].astype(np.int32)
    same_sign = (ours >> 15) == (gold >> 15)
    assert np.all(same_sign | (gold & 0x7FFF == 0))
    assert np.abs((ours & 0x7FFF) - (gold & 0x7FFF)).max() <= 1


# ------------------------------------------------------------------------------ matmul
def reference_matmul(x, p, odt):
    """x.float() @ dequant(W).float().T in float64 (oracle)."""
    N, K = p.quant_state.shape
    w = oracle_dequant(oracle_state(p), (N, K), odt)
    return nf4_ref.nf4_matmul_ref(bits(x), w, odt)


def check(y, ref, tol, unit_slack=False):
    y = y.double().cpu().numpy().reshape(ref.shape)
    rms = np.sqrt((ref ** 2).mean())
    err = np.abs(y - ref)
    bound = tol * rms
    if unit_slack:   # one unit of the fp16 output
        bound = bound + np.abs(ref) * 2.0 ** -10
    assert np.all(err <= bound), f"max err {err.max():.3e}, rms {rms:.3e}, ratio {err.max() / rms:.2e}"


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 9, 16, 33, 64])
@pytest.mark.parametrize("N,K,nested", [(64, 256, False), (48, 192, True), (1024, 4096, True)])
def test_gemm_fp16_vs_oracle(M, N, K, nested):
    _, p = make_weight(N, K, nested, seed=M + N)
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, K, generator=g).half().to(DEV)
    nf = NF4Weight(p)
    ref = reference_matmul(x, p, "fp16")
    check(nf.matmul(x, out_dtype=torch.float32), ref, TOL_F32)
    check(nf.matmul(x), ref, TOL_F32, unit_slack=True)


@pytest.mark.parametrize("M", [1, 4, 8])
@pytest.mark.parametrize("nested", [False, True])
def test_gemm_config_shape(M, nested):
    """The headline op shape: x [M, 4096] fp16, W [14336, 4096] NF4 (blocksize 64)."""
    _, p = make_weight(14336, 4096, nested, seed=7)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(M, 4096, generator=g).half().to(DEV)
    ref = reference_matmul(x, p, "fp16")
    check(NF4Weight(p).matmul(x, out_dtype=torch.float32), ref, TOL_F32)


@pytest.mark.parametrize("M", [1, 4, 8])
def test_gemm_down_proj_shape(M):
    _, p = make_weight(4096, 14336, True, seed=8)
    x = torch.randn(M, 14336, generator=torch.Generator().manual_seed(3)).half().to(DEV)
    check(NF4Weight(p).matmul(x, out_dtype=torch.float32), reference_matmul(x, p, "fp16"), TOL_F32)


@pytest.mark.parametrize("M", [1, 4, 8, 64])
def test_gemm_bf16_vs_oracle(M):
    _, p = make_weight(1024, 4096, True, seed=5)
    x = torch.randn(M, 4096, generator=torch.Generator().manual_seed(9)).bfloat16().to(DEV)
    ref = reference_matmul(x, p, "bf16")
    check(NF4Weight(p).matmul(x, out_dtype=torch.float32), ref, TOL_BF16)


@pytest.mark.parametrize("M", [1, 3, 8])
def test_gemv_simt_vs_oracle(M):
    _, p = make_weight(1024, 4096, True, seed=6)
    x = torch.randn(M, 4096, generator=torch.Generator().manual_seed(4)).half().to(DEV)
    check(NF4Weight(p).matmul_simt(x, out_dtype=torch.float32), reference_matmul(x, p, "fp16"), TOL_F32)


@pytest.mark.parametrize("path", sorted(set(glob.glob(str(GOLDEN / "nf4_gemm_ref_*.npz")))
                                        - set(glob.glob(str(GOLDEN / "nf4_gemm_ref_deq_*.npz")))))
def test_gemm_against_reference_kernel_golden(path):
    """Reference kernel outputs (bf16 x, truncated bf16 y) vs this kernel on the same state."""
    d = dict(np.load(path))
    N, K, M = int(d["N"]), int(d["K"]), int(d["M"])
    nested = bool(d["nested"])
    nf = NF4Weight.from_parts(torch.from_numpy(d["packed"]).to(DEV), torch.from_numpy(d["absmax"]).to(DEV),
                              torch.from_numpy(d["code"]).to(DEV), N, K, nested,
                              torch.from_numpy(d["code2"]).to(DEV) if nested else None,
                              torch.from_numpy(d["absmax2"]).to(DEV) if nested else None,
                              float(d["offset"]) if nested else 0.0)
    x = torch.from_numpy(d["x_bf16"].view(np.int16)).view(torch.bfloat16).to(DEV)
    y = nf.matmul(x, out_dtype=torch.float32).double().cpu().numpy()
    gold = nf4_ref.bf16_bits_to_f32(d["y_bf16"]).astype(np.float64)
    rms = np.sqrt((gold ** 2).mean())
    assert np.all(np.abs(y - gold) <= np.abs(gold) * 2.0 ** -7 + TOL_BF16 * rms)


def test_gemm_deterministic_and_workspace_reuse():
    """Bit-identical across runs; one workspace serves interleaved shapes (counters self-reset)."""
    shapes = [(14336, 4096, 4), (1024, 4096, 1), (4096, 14336, 8), (48, 192, 3), (4096, 4096, 64)]
    ws, outs = [], {}
    for rep in range(3):
        for (N, K, M) in shapes:
            torch.manual_seed(N + K)
            if rep == 0:
                ws.append(make_weight(N, K, True, seed=N + K)[1])
            p = ws[shapes.index((N, K, M))]
            x = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).half().to(DEV)
            y = NF4Weight(p).matmul(x, out_dtype=torch.float32)
            if rep == 0:
                outs[(N, K, M)] = y
                check(y, reference_matmul(x, p, "fp16"), TOL_F32)
            else:
                assert torch.equal(y, outs[(N, K, M)])


def test_gemm_strided_io():
    _, p = make_weight(256, 1024, True, seed=2)
    base = torch.randn(5, 1024 + 64, generator=torch.Generator().manual_seed(1)).half().to(DEV)
    x = base[:, :1024]                       # row stride 1088 (multiple of 8)
    yb = torch.full((5, 256 + 16), float("nan"), dtype=torch.float32, device=DEV)
    NF4Weight(p).matmul(x, out=yb[:, :256])
    check(yb[:, :256], reference_matmul(x.contiguous(), p, "fp16"), TOL_F32)
    assert torch.isnan(yb[:, 256:]).all()    # nothing written outside the output view


@pytest.mark.parametrize("nested", [False, True])
def test_gemm_tensor_parallel_shards(nested):
    """Column (output-row) and row (input-column) shards read in place reproduce slices of the
    full product; double-quant groups straddle the shard boundaries."""
    N, K, M = 1024, 4096, 4
    _, p = make_weight(N, K, nested, seed=12)
    full = NF4Weight(p)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(2)).half().to(DEV)
    y = full.matmul(x, out_dtype=torch.float32)
    for r0, r1 in [(0, 256), (384, 512), (1008, 1024)]:
        ys = full.shard(rows=(r0, r1)).matmul(x, out_dtype=torch.float32)
        torch.testing.assert_close(ys, y[:, r0:r1], atol=1e-5, rtol=1e-5)
    parts = []
    for k0, k1 in [(0, 1024), (1024, 2048), (2048, 3072), (3072, 4096)]:
        for copy in (True, False):
            ys = full.shard(cols=(k0, k1), copy=copy).matmul(x[:, k0:k1].contiguous(), out_dtype=torch.float32)
            if copy:
                parts.append(ys)
    torch.testing.assert_close(sum(parts), y, atol=2e-3 * y.pow(2).mean().sqrt().item(), rtol=0)
    # a shard's dequant is bit-identical to the same slice of the full dequant
    dq = full.dequantize(torch.float16)
    sh = full.shard(rows=(256, 512), cols=(1024, 3072)).dequantize(torch.float16)
    assert torch.equal(sh, dq[256:512, 1024:3072])


@pytest.mark.parametrize("N,K,M,nested", [(14336, 4096, 8, True), (4096, 14336, 4, True), (6144, 4096, 1, True),
                                          (1024, 4096, 8, False), (1040, 512, 5, True), (144, 1024, 3, False)])
def test_tma_and_register_kernels_agree_with_oracle(N, K, M, nested, monkeypatch):
    """The M <= 8 launches run the register-staged kernel by default and the TMA-staged kernel with
    B2D_NF4_KERNEL=tma: both meet the oracle bar, they are different kernels (different summation
    orders, so the outputs are not bit-identical on the large shapes), and the TMA-staged kernel
    records no timed-out pipeline wait."""
    from b200kernels.nf4_gemm import gemm_errors
    _, p = make_weight(N, K, nested, seed=N + M)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(M + 1)).half().to(DEV)
    ref = reference_matmul(x, p, "fp16")
    nf = NF4Weight(p)
    y_reg = nf.matmul(x, out_dtype=torch.float32)
    monkeypatch.setenv("B2D_NF4_KERNEL", "tma")
    y_tma = nf.matmul(x, out_dtype=torch.float32)
    y_tma2 = nf.matmul(x, out_dtype=torch.float32)
    monkeypatch.delenv("B2D_NF4_KERNEL")
    torch.cuda.synchronize()
    check(y_tma, ref, TOL_F32)
    check(y_reg, ref, TOL_F32)
    assert torch.equal(y_tma, y_tma2)                        # deterministic
    if N * K >= 4096 * 4096:
        assert not torch.equal(y_tma, y_reg)
    assert gemm_errors(DEV) == 0


def test_gemm_rejects_bad_arguments():
    _, p = make_weight(64, 256, False)
    nf = NF4Weight(p)
    with pytest.raises(_lib.B2DError):
        nf.matmul(torch.randn(65, 256, device=DEV).half())       # M > 64
    with pytest.raises(_lib.B2DError):
        nf.matmul(torch.randn(2, 256, device=DEV))               # fp32 activations


@pytest.mark.parametrize("N,K,M,nested,dtype", [(14336, 4096, 64, True, torch.float16),
                                                (4096, 14336, 64, True, torch.float16),
                                                (6144, 4096, 33, True, torch.float16),
                                                (1040, 4096, 16, False, torch.float16),
                                                (4096, 4096, 48, True, torch.bfloat16),
                                                (1024, 1024, 9, True, torch.float16),
                                                (64, 256, 24, False, torch.float16)])
def test_tcgen05_and_mma_sync_kernels_agree_with_oracle(N, K, M, nested, dtype, monkeypatch):
    """9..64 tokens run the tcgen05 kernel (TMEM accumulator, weights rounded to the activation dtype
    with their block scale before the MMA) by default and the register-staged mma.sync kernel with
    B2D_NF4_TC5=0: both meet the oracle bar for fp32 and model-dtype outputs, the tcgen05 kernel is
    deterministic (split-K partials summed in cluster rank order) and records no timed-out wait."""
    from b200kernels.nf4_gemm import gemm_errors
    _, p = make_weight(N, K, nested, seed=N + M)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(M + 2)).to(dtype).to(DEV)
    odt = "fp16" if dtype == torch.float16 else "bf16"
    tol = TOL_F32 if dtype == torch.float16 else TOL_BF16
    ref = reference_matmul(x, p, odt)
    nf = NF4Weight(p)
    y5 = nf.matmul(x, out_dtype=torch.float32)
    y5b = nf.matmul(x, out_dtype=torch.float32)
    y5h = nf.matmul(x)
    monkeypatch.setenv("B2D_NF4_TC5", "0")
    y_old = nf.matmul(x, out_dtype=torch.float32)
    monkeypatch.delenv("B2D_NF4_TC5")
    torch.cuda.synchronize()
    check(y5, ref, tol)
    check(y_old, ref, tol)
    check(y5h, ref, tol, unit_slack=dtype == torch.float16)
    assert torch.equal(y5, y5b)
    assert gemm_errors(DEV) == 0
