"""GPU: the allocation-free attention entry point agrees with the workspace one.

``b2d_gqa_decode_noalloc`` exists for callers that cannot allocate device memory themselves (a
serving process whose allocator owns the device budget, a plugin inside another framework's memory
pool): it keeps the split partials in a static device array inside the library instead of a caller
workspace. This file is collected last on purpose, so a failure here comes after every other test.
"""
import numpy as np
import pytest
import torch

from b200kernels import _lib
from b200kernels.decode_attention import decode_attention
from oracle.attn_ref import gqa_decode_ref

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _noalloc(q, k, v, sl, chunk, out, nsplit=0, scale=None):
    B, H, _, D = q.shape
    KVH, S = k.shape[1], k.shape[2]
    return _lib.load().b2d_gqa_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
        v.data_ptr(), v.stride(0), v.stride(1), v.stride(2), sl.data_ptr(), B, H, KVH, S, D,
        D ** -0.5 if scale is None else float(scale), nsplit, chunk, _lib.dtype_code(q.dtype), out.data_ptr(),
        out.stride(0), out.stride(2), _lib.dtype_code(out.dtype), torch.cuda.current_stream(DEV).cuda_stream)


def _check(out, ref, unit=None):
    o = out.double().cpu().numpy()
    bound = 2e-3 * np.sqrt((ref ** 2).mean()) + (0 if unit is None else np.abs(ref) * unit)
    assert (np.abs(o - ref) <= bound).all(), np.abs(o - ref).max()


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    for call, (B, S, seed) in enumerate([(4, 1000, 1), (8, 2048, 2)]):
        g = torch.Generator().manual_seed(seed)
        q = torch.randn(B, 32, 1, 128, generator=g).half().to(DEV)
        k = torch.randn(B, 8, S, 128, generator=g).half().to(DEV)
        v = torch.randn(B, 8, S, 128, generator=g).half().to(DEV)
        sl = torch.randint(1, S + 1, (B,), generator=g).to(torch.int32).to(DEV)
        chunk = 128
        ref = decode_attention(q, k, v, 128 ** -0.5, chunk=chunk, seqlens=sl, out_dtype=torch.float32)
        out = torch.full((B, 1, 32, 128), float("nan"), dtype=torch.float32, device=DEV)
        st = _noalloc(q, k, v, sl, chunk, out)
        assert st == 0, (call, _lib.load().b2d_last_cuda_error())
        torch.cuda.synchronize()
        r = ref.double().cpu().numpy()
        err = np.abs(out.double().cpu().numpy() - r).max()
        assert err <= 2e-3 * np.sqrt((r ** 2).mean()), (call, err)


def test_noalloc_matches_oracle_with_its_own_split_choice(golden_dir):
    """Against the oracle (float64 restatement of the reference's repeat_kv + SDPA) rather than the
    workspace entry point, so a fault shared by both entry points cannot hide: the committed D=64
    fixture with 3 splits and the chunk left to the entry point, then a bf16 case with both the split
    count and the chunk left to it (several splits at S=300), each called twice in a row."""
    z = np.load(golden_dir / "attn_ref_b2_h8_kv2_s40_d64.npz")
    q, k, v = (torch.from_numpy(z[n]).to(DEV) for n in ("q", "k", "v"))
    sl = torch.from_numpy(z["seqlens"]).to(DEV)
    ref = gqa_decode_ref(z["q"], z["k"], z["v"], float(z["scale"]), z["seqlens"])
    assert np.abs(ref - z["out"]).max() <= 1e-5 * np.abs(ref).max()      # the oracle is the fixture
    for _ in range(2):
        out = torch.full((2, 1, 8, 64), float("nan"), dtype=torch.float32, device=DEV)
        assert _noalloc(q, k, v, sl, 0, out, nsplit=3, scale=z["scale"]) == 0, _lib.load().b2d_last_cuda_error()
        torch.cuda.synchronize()
        _check(out, ref)
    assert _lib.load().b2d_gqa_default_splits(3, 4, 300) > 1                # the next case really splits
    g = torch.Generator().manual_seed(7)
    q = torch.randn(3, 16, 1, 128, generator=g).bfloat16()
    k = torch.randn(3, 4, 300, 128, generator=g).bfloat16()
    v = torch.randn(3, 4, 300, 128, generator=g).bfloat16()
    lens = torch.tensor([300, 1, 177], dtype=torch.int32)
    ref = gqa_decode_ref(q.float().numpy(), k.float().numpy(), v.float().numpy(), 128 ** -0.5, lens.numpy())
    for _ in range(2):
        out = torch.full((3, 1, 16, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
        assert _noalloc(q.to(DEV), k.to(DEV), v.to(DEV), lens.to(DEV), 0, out) == 0
        torch.cuda.synchronize()
        _check(out, ref, unit=2.0 ** -7)


def test_noalloc_rejects_oversized_partials():
    B, S = 64, 8192
    q = torch.zeros(B, 32, 1, 128, dtype=torch.half, device=DEV)
    k = torch.zeros(B, 8, S, 128, dtype=torch.half, device=DEV)
    sl = torch.full((B,), S, dtype=torch.int32, device=DEV)
    out = torch.empty(B, 1, 32, 128, dtype=torch.float32, device=DEV)
    st = _noalloc(q, k, k, sl, 128, out)      # 64*32*64 splits*(128+2)*4 B = 68 MB > 8 MiB
    assert st == 5
    assert b"static scratch" in _lib.load().b2d_last_cuda_error()
