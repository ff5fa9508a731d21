"""GPU parity of the split-K GQA decode attention (through the C ABI) against the CPU oracle.

Bar: max|out - ref| <= 2e-3 * rms(ref) for an fp32 output (the reference formula is fp32 SDPA on
repeated KV heads, ``bench_attention.py:40-41``), plus one output unit for fp16/bf16 outputs.
"""
import glob
from pathlib import Path

import numpy as np
import pytest
import torch

from b200kernels import _lib
from b200kernels.decode_attention import decode_attention, plan_splits
from oracle import attn_ref

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
GOLDEN = Path(__file__).resolve().parent / "golden"
TOL = 2e-3


def rand_case(B, H, KVH, S, D, dtype=torch.float16, seed=0, lens=None):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, 1, D, generator=g).to(dtype)
    k = torch.randn(B, KVH, S, D, generator=g).to(dtype)
    v = torch.randn(B, KVH, S, D, generator=g).to(dtype)
    sl = None if lens is None else torch.tensor(lens, dtype=torch.int32)
    return q, k, v, sl


def check(out, ref, tol=TOL, unit=None):
    out = out.double().cpu().numpy().reshape(ref.shape)
    rms = np.sqrt((ref ** 2).mean())
    bound = tol * rms + (0 if unit is None else np.abs(ref) * unit)
    err = np.abs(out - ref)
    assert np.all(err <= bound), f"max err {err.max():.3e} rms {rms:.3e}"


def run(q, k, v, sl, out_dtype=torch.float32, **kw):
    return decode_attention(q.to(DEV), k.to(DEV), v.to(DEV), q.shape[-1] ** -0.5,
                            seqlens=None if sl is None else sl.to(DEV), out_dtype=out_dtype, **kw)


def oracle(q, k, v, sl):
    return attn_ref.gqa_decode_ref(q.float().numpy(), k.float().numpy(), v.float().numpy(), q.shape[-1] ** -0.5,
                                   None if sl is None else sl.numpy())


def test_config_shape_ragged_lengths():
    """B=8, H=32, KVH=8, S=2048, D=128, fp16, lengths uniform in [512, 2048]."""
    g = torch.Generator().manual_seed(1)
    lens = torch.randint(512, 2049, (8,), generator=g).tolist()
    q, k, v, sl = rand_case(8, 32, 8, 2048, 128, seed=2, lens=lens)
    ref = oracle(q, k, v, sl)
    check(run(q, k, v, sl), ref)
    check(run(q, k, v, sl, out_dtype=torch.float16), ref, unit=2.0 ** -10)


@pytest.mark.parametrize("B,H,KVH,S,D", [(1, 32, 8, 1, 128), (2, 32, 8, 15, 128), (3, 32, 8, 17, 128),
                                         (1, 8, 8, 300, 64), (2, 16, 2, 129, 64), (1, 16, 1, 777, 128),
                                         (2, 4, 1, 33, 128), (1, 12, 4, 95, 128)])
def test_odd_shapes_full_length(B, H, KVH, S, D):
    q, k, v, sl = rand_case(B, H, KVH, S, D, seed=S)
    check(run(q, k, v, sl), oracle(q, k, v, sl))


def test_ragged_with_empty_and_single_key():
    q, k, v, sl = rand_case(4, 32, 8, 200, 128, seed=9, lens=[0, 1, 200, 63])
    out = run(q, k, v, sl)
    ref = oracle(q, k, v, sl)
    assert torch.all(out[0] == 0)
    check(out[1:], ref[1:])


@pytest.mark.parametrize("chunk", [16, 64, 100, 2048])
def test_explicit_chunks(chunk):
    q, k, v, sl = rand_case(2, 32, 8, 1000, 128, seed=4, lens=[1000, 517])
    check(run(q, k, v, sl, chunk=chunk), oracle(q, k, v, sl))


def test_bf16():
    q, k, v, sl = rand_case(4, 32, 8, 512, 128, dtype=torch.bfloat16, seed=5, lens=[512, 100, 333, 1])
    ref = oracle(q, k, v, sl)
    check(run(q, k, v, sl), ref)
    check(run(q, k, v, sl, out_dtype=torch.bfloat16), ref, unit=2.0 ** -7)


def test_strided_cache_views():
    """K/V as views into a larger preallocated cache (HF static-cache style), q from a [B,1,H,D] buffer."""
    B, H, KVH, S, D, SMAX = 2, 32, 8, 300, 128, 512
    g = torch.Generator().manual_seed(6)
    kc = torch.randn(B, KVH, SMAX, D, generator=g).half()
    vc = torch.randn(B, KVH, SMAX, D, generator=g).half()
    qb = torch.randn(B, 1, H, D, generator=g).half()
    q = qb.transpose(1, 2)                        # [B, H, 1, D], strides (H*D, D, .., 1)
    k, v = kc[:, :, :S], vc[:, :, :S]
    out = decode_attention(q.to(DEV), kc.to(DEV)[:, :, :S], vc.to(DEV)[:, :, :S], D ** -0.5,
                           out_dtype=torch.float32)
    check(out, oracle(q.contiguous(), k.contiguous(), v.contiguous(), None))


@pytest.mark.parametrize("path", sorted(glob.glob(str(GOLDEN / "attn_ref_*.npz"))))
def test_against_reference_stock_golden(path):
    d = dict(np.load(path))
    q, k, v = (torch.from_numpy(d[n]).to(DEV) for n in ("q", "k", "v"))
    sl = torch.from_numpy(d["seqlens"]).to(DEV)
    out = decode_attention(q, k, v, float(d["scale"]), seqlens=sl, out_dtype=torch.float32)
    check(out, d["out"].astype(np.float64))


def test_matches_torch_sdpa_on_device():
    """The reference's stock path on the same GPU: repeat_kv + SDPA (fp32), no mask."""
    import torch.nn.functional as F
    from transformers.integrations.sdpa_attention import repeat_kv
    q, k, v, _ = rand_case(4, 32, 8, 1024, 128, seed=7)
    q, k, v = q.to(DEV), k.to(DEV), v.to(DEV)
    ref = F.scaled_dot_product_attention(q.float(), repeat_kv(k, 4).float(), repeat_kv(v, 4).float(),
                                         scale=128 ** -0.5).transpose(1, 2)
    out = decode_attention(q, k, v, 128 ** -0.5, out_dtype=torch.float32)
    check(out, ref.double().cpu().numpy())


def test_split_plan_and_workspace():
    ns, chunk = plan_splits(8, 8, 2048)
    assert ns * chunk >= 2048 and chunk % 32 == 0
    assert ns == -(-2048 // chunk)
    lib = _lib.load()
    assert lib.b2d_gqa_workspace_bytes(8, 32, ns, 128) == 65536 + 8 * 32 * ns * 130 * 4


def test_rejects_bad_inputs():
    q, k, v, _ = rand_case(1, 32, 8, 16, 128)
    with pytest.raises(TypeError):
        decode_attention(q.to(DEV), k.to(DEV).float(), v.to(DEV), 0.1)
    with pytest.raises(ValueError):
        decode_attention(torch.randn(1, 32, 2, 128, device=DEV).half(), k.to(DEV), v.to(DEV), 0.1)
    with pytest.raises(_lib.B2DError):
        decode_attention(torch.randn(1, 32, 1, 96, device=DEV).half(), torch.randn(1, 8, 16, 96, device=DEV).half(),
                         torch.randn(1, 8, 16, 96, device=DEV).half(), 0.1)


@pytest.mark.parametrize("B,H,KVH,S,D", [(8, 32, 8, 320, 128), (3, 64, 4, 1000, 64), (2, 32, 8, 4096, 128)])
@pytest.mark.parametrize("odt", [torch.float16, torch.float32])
@pytest.mark.parametrize("kernel", ["reg", "stream"])
def test_single_launch_combine_matches_two_kernels(B, H, KVH, S, D, odt, kernel, monkeypatch):
    """B2D_ATTN_FUSED_COMBINE (the last split CTA of the partial kernel combines) gives the two-kernel
    result of the same partial kernel bit for bit, for both partial kernels, including empty and ragged
    sequences, and leaves the workspace counters at zero."""
    monkeypatch.setenv("B2D_ATTN_KERNEL", kernel)
    g = torch.Generator().manual_seed(S + B)
    q = torch.randn(B, H, 1, D, generator=g).half().to(DEV)
    k = torch.randn(B, KVH, S, D, generator=g).half().to(DEV)
    v = torch.randn(B, KVH, S, D, generator=g).half().to(DEV)
    lens = torch.randint(1, S + 1, (B,), generator=g).to(torch.int32)
    lens[0] = 0
    sl = lens.to(DEV)
    ws = torch.zeros(_lib.load().b2d_gqa_workspace_bytes(B, H, 64, D), dtype=torch.uint8, device=DEV)
    for chunk in (64, 128, None):
        two = decode_attention(q, k, v, D ** -0.5, chunk=chunk, seqlens=sl, out_dtype=odt, workspace=ws)
        one = decode_attention(q, k, v, D ** -0.5, chunk=chunk, seqlens=sl, out_dtype=odt, workspace=ws,
                               flags=_lib.ATTN_FUSED_COMBINE | _lib.LAUNCH_PDL)
        again = decode_attention(q, k, v, D ** -0.5, chunk=chunk, seqlens=sl, out_dtype=odt, workspace=ws,
                                 flags=_lib.ATTN_FUSED_COMBINE)
        torch.cuda.synchronize()
        assert torch.equal(one, two) and torch.equal(again, two), chunk
        assert one[0].abs().max().item() == 0
    assert ws[:65536].view(torch.int32).abs().sum().item() == 0


@pytest.mark.parametrize("B,H,KVH,S,D,dtype,lens", [
    (8, 32, 8, 2048, 128, torch.float16, "ragged"),
    (2, 32, 8, 100, 128, torch.bfloat16, None),
    (3, 64, 4, 333, 64, torch.float16, [333, 0, 65]),
    (1, 32, 8, 4097, 128, torch.float16, None),
    (2, 16, 1, 200, 128, torch.float16, [1, 200]),
    (8, 32, 8, 2048, 128, torch.float16, [2048, 1, 0, 5, 100, 2048, 17, 512])])
def test_streaming_and_register_kernels_agree_with_oracle(B, H, KVH, S, D, dtype, lens, monkeypatch):
    """Two-kernel launches run the streaming partial kernel (K/V staged through a shared-memory ring) by
    default (B2D_ATTN_KERNEL=stream) and the register-prefetch kernel with B2D_ATTN_KERNEL=reg: both meet the oracle bar for
    ragged, empty and single-key lengths, G = 4, 16 and D = 64, 128, and the streaming kernel is
    deterministic (the skewed case has sequences of 0 to 2048 keys in one batch). bf16 inputs: both kernels round P to bf16 (8-bit significand) for the P V product, so
    over ~100 keys the error reaches ~5e-3 * rms(ref); their bar is 1e-2 * rms(ref)."""
    if lens == "ragged":
        lens = torch.randint(512, S + 1, (B,), generator=torch.Generator().manual_seed(7)).tolist()
    q, k, v, sl = rand_case(B, H, KVH, S, D, dtype=dtype, seed=S, lens=lens)
    ref = oracle(q, k, v, sl)
    tol = TOL if dtype == torch.float16 else 1e-2
    monkeypatch.setenv("B2D_ATTN_KERNEL", "stream")
    y1, y2 = run(q, k, v, sl), run(q, k, v, sl)
    monkeypatch.setenv("B2D_ATTN_KERNEL", "reg")
    yr = run(q, k, v, sl)
    monkeypatch.delenv("B2D_ATTN_KERNEL")
    check(y1, ref, tol)
    check(yr, ref, tol)
    assert torch.equal(y1, y2)


def test_static_prefix_flag_matches_oracle():
    """B2D_KV_STATIC_PREFIX (with B2D_LAUNCH_PDL) lets the streaming kernel fetch whole stages below each
    sequence's newest key before the dependency wait; right after a kernel that wrote the cache the result
    is the same: the oracle bar on ragged lengths, and equal to the plain launch."""
    q, k, v, sl = rand_case(8, 32, 8, 2048, 128, seed=11,
                            lens=[2048, 1, 64, 65, 700, 1500, 129, 1024])
    ref = oracle(q, k, v, sl)
    qd, kd, vd, sld = q.to(DEV), k.to(DEV), v.to(DEV), sl.to(DEV)
    plain = decode_attention(qd, kd, vd, 128 ** -0.5, seqlens=sld, out_dtype=torch.float32)
    kd2, vd2 = torch.empty_like(kd), torch.empty_like(vd)
    kd2.copy_(kd)   # the preceding kernels of the stream write the caches
    vd2.copy_(vd)
    pre = decode_attention(qd, kd2, vd2, 128 ** -0.5, seqlens=sld, out_dtype=torch.float32,
                           flags=_lib.LAUNCH_PDL | _lib.KV_STATIC_PREFIX)
    torch.cuda.synchronize()
    check(pre, ref)
    assert torch.equal(pre, plain)


@pytest.mark.parametrize("B,H,KVH,S,D,dtype", [(8, 32, 8, 357, 128, torch.float16), (3, 16, 2, 130, 64, torch.bfloat16)])
def test_append_launch_matches_rotary_kernel_then_attention(B, H, KVH, S, D, dtype):
    """b2d_gqa_decode_append (RoPE and the KV append inside the attention launch) gives the numbers of
    b2d_rope_kv_append followed by the attention launch bit for bit: the output, both caches and the
    lengths, for positions from 0 to S - 1 (and one outside the cache, which yields length 0); so does
    the append launch with the single-launch combine, on two calls in a row."""
    from b200kernels.decode_attention import decode_attention_append
    from b200kernels.glue import rope_kv_append
    g = torch.Generator().manual_seed(S + B)
    q = torch.randn(B, H * D, generator=g).to(dtype).to(DEV)
    k = torch.randn(B, KVH * D, generator=g).to(dtype).to(DEV)
    v = torch.randn(B, KVH * D, generator=g).to(dtype).to(DEV)
    kc = torch.randn(B, KVH, S, D, generator=g).to(dtype).to(DEV)
    vc = torch.randn(B, KVH, S, D, generator=g).to(dtype).to(DEV)
    pos = torch.randint(0, S, (B,), generator=g)
    pos[0], pos[-1] = 0, S - 1
    if B > 2:
        pos[1] = S   # outside the cache: length 0, nothing appended
    pos = pos.to(DEV)
    ang = torch.arange(S, dtype=torch.float32).view(-1, 1) * (1e-2 * torch.arange(D // 2, dtype=torch.float32) + 0.01)
    cos = torch.cat([ang.cos(), ang.cos()], 1).to(dtype).to(DEV)
    sin = torch.cat([ang.sin(), ang.sin()], 1).to(dtype).to(DEV)
    # path 1: the rotary kernel, then the attention launch
    kc1, vc1, q1 = kc.clone(), vc.clone(), q.clone()
    sl1 = torch.zeros(B, dtype=torch.int32, device=DEV)
    rope_kv_append(q1, k, v, pos, cos, sin, q1.view(B, H, D), kc1, vc1, sl1)
    out1 = decode_attention(q1.view(B, H, 1, D), kc1, vc1, D ** -0.5, seqlens=sl1)
    # path 2: one launch
    kc2, vc2 = kc.clone(), vc.clone()
    sl2 = torch.full((B,), -7, dtype=torch.int32, device=DEV)
    out2 = torch.full((B, 1, H, D), float("nan"), dtype=dtype, device=DEV)
    decode_attention_append(q, k, v, pos, cos, sin, kc2, vc2, D ** -0.5, sl2, out2)
    # path 3: one launch with the single-launch combine, twice (the arrival counters return to zero)
    kc3, vc3 = kc.clone(), vc.clone()
    sl3 = torch.full((B,), -7, dtype=torch.int32, device=DEV)
    outs3 = []
    for _ in range(2):
        outs3.append(torch.full((B, 1, H, D), float("nan"), dtype=dtype, device=DEV))
        decode_attention_append(q, k, v, pos, cos, sin, kc3, vc3, D ** -0.5, sl3, outs3[-1],
                                flags=_lib.ATTN_FUSED_COMBINE | _lib.LAUNCH_PDL)
    # path 4: one launch that also prefetches unrelated static data into L2 (a hint: same numbers)
    from b200kernels.decode_attention import l2_prefetch_hint
    kc4, vc4 = kc.clone(), vc.clone()
    sl4 = torch.full((B,), -7, dtype=torch.int32, device=DEV)
    out4 = torch.full((B, 1, H, D), float("nan"), dtype=dtype, device=DEV)
    junk = torch.randn(3 << 20, generator=g).to(DEV)
    l2_prefetch_hint([junk, kc, vc[1:]])
    decode_attention_append(q, k, v, pos, cos, sin, kc4, vc4, D ** -0.5, sl4, out4, flags=_lib.LAUNCH_PDL)
    torch.cuda.synchronize()
    assert torch.equal(sl1, sl2) and torch.equal(sl1, sl3) and torch.equal(sl1, sl4)
    assert torch.equal(kc1, kc4) and torch.equal(vc1, vc4) and torch.equal(out4, out2)
    assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2)
    assert torch.equal(kc1, kc3) and torch.equal(vc1, vc3)
    assert torch.equal(out1, out2)
    assert torch.equal(outs3[0], out2) and torch.equal(outs3[1], out2)
