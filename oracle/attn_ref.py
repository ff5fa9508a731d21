"""Restatement of the reference's stock decode attention.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the product never imports this.

The reference checks its flash-decoding kernel against
``SDPA(q.float(), repeat_kv(k, G).float(), repeat_kv(v, G).float(), scale)``
(``profiling/kernels/bench_attention.py:40-41``); its stock path is ``repeat_kv`` + SDPA
(``bench_attention.py:27-29``). Query head ``h`` reads KV head ``h // G`` with
``G = H // KVH`` (``repeat_kv`` repeats each KV head G times in place). The reference kernel
attends over every cached key (``decode_attention.py:35-36``); the per-sequence lengths
``seqlens`` add the key mask ``key_index < seqlens[b]``.
"""
from __future__ import annotations

import numpy as np


def gqa_decode_ref(q, k, v, scale, seqlens=None) -> np.ndarray:
    """float64 oracle. q [B,H,1,D], k/v [B,KVH,S,D] (any float dtype) -> out [B,1,H,D]."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    B, H, _, D = q.shape
    KVH, S = k.shape[1], k.shape[2]
    G = H // KVH
    out = np.zeros((B, 1, H, D), dtype=np.float64)
    for b in range(B):
        n = S if seqlens is None else int(seqlens[b])
        if n <= 0:
            continue
        for h in range(H):
            kv = h // G
            s = (k[b, kv, :n] @ q[b, h, 0]) * scale
            s = s - s.max()
            p = np.exp(s)
            out[b, 0, h] = (p / p.sum()) @ v[b, kv, :n]
    return out


def stock_cpu(q, k, v, scale, seqlens=None):
    """The reference's stock formula on torch CPU in fp32: ``repeat_kv`` + SDPA with a
    boolean key mask for ragged lengths. Used as the timed CPU baseline."""
    import torch
    import torch.nn.functional as F

    B, H, _, D = q.shape
    KVH, S = k.shape[1], k.shape[2]
    G = H // KVH
    qf, kf, vf = q.float(), k.float(), v.float()
    kr = kf[:, :, None].expand(B, KVH, G, S, D).reshape(B, H, S, D)
    vr = vf[:, :, None].expand(B, KVH, G, S, D).reshape(B, H, S, D)
    mask = None
    if seqlens is not None:
        idx = torch.arange(S)
        mask = (idx[None, :] < seqlens.reshape(B, 1).to(torch.int64))[:, None, None, :]
    out = F.scaled_dot_product_attention(qf, kr, vr, attn_mask=mask, scale=scale)
    return out.transpose(1, 2)
