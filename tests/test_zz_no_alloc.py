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

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _noalloc(q, k, v, sl, chunk, out):
    B, H, _, D = q.shape
    KVH, S = k.shape[1], k.shape[2]
    return _lib.load().b2d_gqa_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
        v.data_ptr(), v.stride(0), v.stride(1), v.stride(2), sl.data_ptr(), B, H, KVH, S, D, D ** -0.5,
        0, chunk, _lib.F16, out.data_ptr(), out.stride(0), out.stride(2), _lib.F32,
        torch.cuda.current_stream(DEV).cuda_stream)


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


def test_noalloc_rejects_oversized_partials():
    B, S = 64, 8192
    q = torch.zeros(B, 32, 1, 128, dtype=torch.half, device=DEV)
    k = torch.zeros(B, 8, S, 128, dtype=torch.half, device=DEV)
    sl = torch.full((B,), S, dtype=torch.int32, device=DEV)
    out = torch.empty(B, 1, 32, 128, dtype=torch.float32, device=DEV)
    st = _noalloc(q, k, k, sl, 128, out)      # 64*32*64 splits*(128+2)*4 B = 68 MB > 8 MiB
    assert st == 5
    assert b"static scratch" in _lib.load().b2d_last_cuda_error()
