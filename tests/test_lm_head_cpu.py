"""CPU: merging vocabulary-parallel argmax keys (``b200kernels.lm_head.merge_keys``).

A key packs a logit and its vocabulary index as ``(ordered float bits) << 32 | (0xFFFFFFFF - index)``,
compared as signed 64-bit integers (the encoding ``b2d_lm_head_argmax`` writes); the maximum key over
shards is the largest logit with the lowest index, i.e. ``torch.argmax`` over the concatenated logits.
"""
import struct

import torch

from b200kernels.lm_head import merge_keys


def key(value: float, index: int) -> int:
    """The key ``b2d_lm_head_argmax`` forms (``argmax_key`` in csrc/lm_head.cu): -0 is folded onto +0 and
    every NaN onto the largest key, as torch.argmax orders them."""
    b = struct.unpack("<i", struct.pack("<f", value))[0]
    if value != value:
        b = 0x7FFFFFFF
    elif b == -0x80000000:
        b = 0
    elif b < 0:
        b ^= 0x7FFFFFFF
    return (b << 32) | (0xFFFFFFFF - index)


def test_merge_keys_is_argmax_with_first_index_ties():
    g = torch.Generator().manual_seed(0)
    R, M, Vl = 4, 5, 64
    logits = torch.randn(M, R * Vl, generator=g).half().float()
    logits[1, 70] = logits[1, 200] = logits[1].max() + 1      # tie across shards: the lower index wins
    logits[2] = -torch.rand(R * Vl, generator=g) - 1          # all negative
    logits[3, 5] = logits[3, 6] = 1e4                         # tie inside one shard
    keys = torch.empty(R, M, dtype=torch.int64)
    for r in range(R):
        for m in range(M):
            sl = logits[m, r * Vl:(r + 1) * Vl]
            keys[r, m] = max(key(float(v), r * Vl + i) for i, v in enumerate(sl))
    assert torch.equal(merge_keys(keys), torch.argmax(logits, -1))
    out = torch.empty(M, dtype=torch.int64)
    assert merge_keys(keys, out=out) is out and out[1].item() == 70 and out[3].item() == 5


def test_key_order_matches_float_order():
    vals = [-3.5, -1.0, -0.0, 0.0, 1e-8, 0.5, 2.0, 65504.0]
    ks = [key(v, 10) for v in vals]
    assert ks == sorted(ks)
    assert key(1.0, 3) > key(1.0, 4)


def test_signed_zero_and_nan_follow_torch_argmax():
    """torch.argmax treats -0 and +0 as equal (first index wins) and NaN as the maximum (first NaN wins)."""
    cases = [[0.0, -0.0, 0.0], [-0.0, 0.0], [-1.0, -0.0, 0.0, -0.0], [1.0, float("nan"), 2.0, float("nan")],
             [float("inf"), float("nan")], [float("-inf"), -0.0], [-2.0, float("-nan"), 5.0]]
    for vals in cases:
        t = torch.tensor(vals)
        best = max(range(len(vals)), key=lambda i: key(vals[i], i))
        assert best == torch.argmax(t).item(), vals
        keys = torch.tensor([[key(v, i) for i, v in enumerate(vals)]]).T   # one shard per element
        assert merge_keys(keys).item() == torch.argmax(t).item(), vals
