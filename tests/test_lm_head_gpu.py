"""GPU: lm_head + greedy argmax in one launch (``b2d_lm_head_argmax``) against the stock ops it
replaces, ``F.linear`` (the head GEMV) followed by ``argmax(-1)``.

Bars: logits within 2e-3 * rms of the fp32 product ``x.float() @ W.float().T`` plus half a unit in
the last place of the model dtype (they are that product rounded once); ids equal ``torch.argmax`` of
the kernel's own logits exactly, ties included (the first index of the maximum wins); vocabulary
shards merged through their keys give the unsharded ids.
"""
import pytest
import torch

from b200kernels import _lib
from b200kernels.lm_head import lm_head_argmax, merge_keys

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def make(M, V, K, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(dtype).to(DEV)
    w = (torch.randn(V, K, generator=g) * 0.02).to(dtype).to(DEV)
    return x, w


def check_logits(logits, x, w, dtype):
    ref = x.float() @ w.float().T
    rms = ref.pow(2).mean().sqrt().item()
    half_ulp = (2 ** -11 if dtype == torch.float16 else 2 ** -8) * ref.abs()
    assert ((logits.float() - ref).abs() <= 2e-3 * rms + half_ulp).all(), (logits.float() - ref).abs().max().item()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,V,K", [(1, 1000, 256), (3, 4099, 512), (8, 32000, 4096), (5, 17, 1024), (9, 3001, 512),
                                   (16, 32000, 4096), (27, 777, 1024), (64, 32000, 4096)])
def test_logits_and_argmax(dtype, M, V, K):
    x, w = make(M, V, K, dtype, M * 7 + V)
    for flags in (0, _lib.LAUNCH_PDL | _lib.STATIC_WEIGHTS):
        for _ in range(2):   # the workspace counter returns to zero between calls
            logits, ids, _ = lm_head_argmax(x, w, flags=flags)
            torch.cuda.synchronize()
            check_logits(logits, x, w, dtype)
            assert torch.equal(ids, torch.argmax(logits, -1)), (ids, torch.argmax(logits, -1))


def test_ties_take_the_first_index():
    M, V, K = 4, 5000, 512
    x, w = make(M, V, K, torch.float16, 3)
    for r in (4999, 7, 2500):           # identical rows pointing along token 0 -> identical top logits
        w[r] = (x[0].float() / x[0].float().norm() * 2).half()
    logits, ids, _ = lm_head_argmax(x, w)
    torch.cuda.synchronize()
    assert logits[0, 7] == logits[0, 2500] == logits[0, 4999] and ids[0].item() == 7
    assert torch.equal(ids, torch.argmax(logits, -1))


def test_signed_zero_and_nan_follow_torch_argmax():
    """Logits of -0 and +0 are equal maxima (the lower index wins) and a NaN logit is the maximum (the
    first NaN wins), as torch.argmax decides. Every other row is strongly negative."""
    M, V, K = 2, 64, 256
    x = torch.zeros(M, K, dtype=torch.float16, device=DEV)
    x[:, 0] = 0.25
    x[:, 1] = 1.0
    w = torch.zeros(V, K, dtype=torch.float16, device=DEV)
    w[:, 1] = -4.0                                  # every row: logit -4 ...
    w[5, 1] = 0.0
    w[5, 0] = -(2.0 ** -24)                         # ... row 5: -2^-26, which rounds to -0 in fp16
    w[9, 1] = 0.0                                   # ... row 9: exactly +0
    logits, ids, _ = lm_head_argmax(x, w)
    torch.cuda.synchronize()
    assert logits[0, 5].item() == 0.0 and str(logits[0, 5].item()) == "-0.0" and str(logits[0, 9].item()) == "0.0"
    assert ids.tolist() == [5, 5] and torch.equal(ids, torch.argmax(logits, -1))
    w[12, 2] = float("nan")                         # rows 12 and 20 give NaN logits (NaN * 0 is NaN)
    w[20, 3] = float("nan")
    logits, ids, _ = lm_head_argmax(x, w)
    torch.cuda.synchronize()
    assert logits[:, 12].isnan().all() and logits[:, 20].isnan().all()
    assert ids.tolist() == [12, 12] and torch.equal(ids, torch.argmax(logits, -1))


@pytest.mark.parametrize("M", [8, 64])
def test_vocab_shards_merge_to_full_argmax(M):
    V, K, R = 32000, 4096, 4
    x, w = make(M, V, K, torch.float16, 11)
    full_logits, full_ids, _ = lm_head_argmax(x, w)
    keys = torch.empty(R, M, dtype=torch.int64, device=DEV)
    Vl = V // R
    for r in range(R):
        part = torch.empty(M, Vl, dtype=torch.float16, device=DEV)
        lm_head_argmax(x, w[r * Vl:(r + 1) * Vl].contiguous(), logits=part, keys=keys[r], vocab_offset=r * Vl)
        torch.cuda.synchronize()
        assert torch.equal(part, full_logits[:, r * Vl:(r + 1) * Vl]), r
    assert torch.equal(merge_keys(keys), full_ids)


def test_matches_stock_linear_argmax_up_to_near_ties():
    M, V, K = 8, 32000, 4096
    x, w = make(M, V, K, torch.float16, 5)
    logits, ids, _ = lm_head_argmax(x, w)
    stock = torch.nn.functional.linear(x, w)
    stock_ids = stock.argmax(-1)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().T
    for m in range(M):
        if ids[m] != stock_ids[m]:   # allowed only when the two candidates are within rounding of each other
            gap = (ref[m, ids[m]] - ref[m, stock_ids[m]]).abs().item()
            assert gap <= 2e-3 * ref.pow(2).mean().sqrt().item(), (m, gap)


def test_rejects_unsupported_arguments():
    x, w = make(65, 64, 256, torch.float16, 1)
    with pytest.raises(_lib.B2DError):
        lm_head_argmax(x, w)                       # more than 64 rows
    x, w = make(2, 64, 320, torch.float16, 1)
    with pytest.raises(_lib.B2DError):
        lm_head_argmax(x, w)                       # K not a multiple of 256
    x, w = make(2, 64, 256, torch.float16, 1)
    ws = torch.zeros(64, dtype=torch.uint8, device=DEV)
    st = _lib.load().b2d_lm_head_argmax(x.data_ptr(), 256, w.data_ptr(), 256, 2, 64, 256, 0, None, 0,
                                       torch.empty(2, dtype=torch.int64, device=DEV).data_ptr(), None,
                                       _lib.F16, 0, ws.data_ptr(), ws.numel(), _lib.stream_ptr(DEV))
    assert st == 5                                 # workspace smaller than b2d_lm_head_workspace_bytes
