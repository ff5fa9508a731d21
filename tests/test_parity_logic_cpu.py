"""CPU: the host-side logic that the GPU parity tests and the patch surface rely on.

* ``near_tie_report`` (used by the 7B greedy test) must flag a flip that is not a near-tie: one with a
  stock margin larger than our error at that step, and one where our choice is not the stock runner-up.
  The mistakes are planted in synthetic logits here, on the CPU.
* ``patch.STATS`` answers the reference's keys (``attn_triton`` / ``attn_fallback``).
"""
import torch

from b200kernels import patch
from test_decode_gpu import near_tie_report


def _case():
    g = torch.Generator().manual_seed(0)
    B, T, V = 2, 6, 50
    sl = torch.randn(B, T, V, generator=g)
    stock = sl.argmax(-1)
    ol = sl[:, 1:] + 1e-3 * torch.randn(B, T - 1, V, generator=g)   # our logits: small errors
    preds = ol.argmax(-1)
    return stock, sl, ol, preds


def test_no_flips_when_argmaxes_agree():
    stock, sl, ol, preds = _case()
    assert torch.equal(preds, stock[:, 1:])
    assert near_tie_report(preds, stock, ol, sl) == []


def test_genuine_near_tie_passes():
    stock, sl, ol, preds = _case()
    b, j = 1, 2
    top2 = sl[b, j + 1].topk(2)
    sl[b, j + 1, top2.indices[1]] = top2.values[0] - 1e-4             # stock runner-up 1e-4 below
    ol[b, j] = sl[b, j + 1]
    ol[b, j, top2.indices[1]] += 5e-4                                  # ours prefers it (error 5e-4)
    preds = ol.argmax(-1)
    (f,) = near_tie_report(preds, stock, ol, sl)
    assert f["ours_is_stock_runner_up"] and f["ours_stock_rank"] == 2
    assert f["stock_margin"] <= 2 * f["step_err_max"]


def test_planted_non_tie_flips_are_flagged():
    stock, sl, ol, preds = _case()
    b, j = 0, 3
    s = sl[b, j + 1]
    third = s.topk(3).indices[2]
    preds[b, j] = third                        # ours picks the stock third choice ...
    (f,) = near_tie_report(preds, stock, ol, sl)
    assert not f["ours_is_stock_runner_up"] and f["ours_stock_rank"] == 3
    assert f["stock_margin"] > 2 * f["step_err_max"]   # ... with a margin far above our 1e-3 errors


def test_stats_answers_the_reference_keys():
    patch.STATS.update(attn_triton=0, attn_fallback=0)
    assert set(patch.STATS.keys()) == {"attn_triton", "attn_fallback"}
    patch.STATS["attn_triton"] += 2
    assert patch.STATS["attn_kernel"] == 2 and patch.STATS.get("attn_kernel") == 2
    patch.STATS.update(attn_kernel=0)
    assert patch.STATS["attn_triton"] == 0
