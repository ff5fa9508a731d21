"""Flash-decoding grouped-query attention on B200, behind the reference's ``decode_attention``.

Mirrors ``profiling/kernels/decode_attention.py:75-91``:
``decode_attention(q, k, v, scale, chunk, block_s) -> [B, 1, H, D]`` with q ``[B, H, 1, D]`` and
the HF KV-cache layout k/v ``[B, KVH, S, D]`` (arbitrary b/h/s strides, contiguous last dim).
Query head ``h`` reads KV head ``h // (H // KVH)``.

Differences from the reference:
* ``chunk`` (keys per split) defaults to a split count chosen from the SM count and ``B*KVH``
  (the reference fixes 64); an explicit ``chunk`` is honoured, rounded up to a multiple of 16.
* ``block_s`` is accepted for signature compatibility; the kernel's key tile is 16.
* ``seqlens`` (int32 ``[B]``, optional) limits sequence b to its first ``seqlens[b]`` keys.
* fp16 and bf16 (the reference: bf16 only); the output dtype is q's dtype.

Work runs in ``libb200decode.so`` (``b2d_gqa_decode``: split-K partial kernel + log-sum-exp
combine kernel); there is no fallback.
"""
from __future__ import annotations

import torch

from . import _lib

_WS: dict = {}


def attention_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    stream = torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)   # counters start at zero
        _WS[key] = ws
    return ws


def plan_splits(B: int, KVH: int, S: int, chunk: int | None = None) -> tuple[int, int]:
    """(nsplit, chunk) for a cache of S keys."""
    if chunk is None:
        ns = _lib.load().b2d_gqa_default_splits(B, KVH, S)
        chunk = -(-S // ns)
        chunk = -(-chunk // 32) * 32
    else:
        chunk = max(16, -(-int(chunk) // 16) * 16)
    return max(1, -(-S // chunk)), chunk


def decode_attention(q, k, v, scale=None, chunk=None, block_s=None, seqlens=None, out=None, workspace=None,
                     out_dtype=None, flags=0):
    """q [B, H, 1, D], k/v [B, KVH, S, D] (fp16/bf16, last dim contiguous) -> [B, 1, H, D] in
    ``out_dtype`` (q's dtype or torch.float32; default q's dtype). ``flags``: ``_lib.LAUNCH_PDL``
    launches the partial kernel as a programmatic dependent of the previous kernel."""
    B, H, one, D = q.shape
    KVH, S = k.shape[1], k.shape[2]
    if one != 1:
        raise ValueError(f"decode_attention takes one query token per sequence, got q_len={one}")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError(f"q/k/v dtypes differ: {q.dtype}, {k.dtype}, {v.dtype}")
    if v.shape != k.shape or k.shape[0] != B or H % KVH != 0:
        raise ValueError(f"incompatible shapes q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if scale is None:
        scale = D ** -0.5
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k.stride(-1) != 1:
        k = k.contiguous()
    if v.stride(-1) != 1:
        v = v.contiguous()
    if out is None:
        out = torch.empty((B, 1, H, D), device=q.device, dtype=out_dtype or q.dtype)
    if B == 0 or H == 0:
        return out
    nsplit, chunk = plan_splits(B, KVH, S, chunk)
    nbytes = _lib.load().b2d_gqa_workspace_bytes(B, H, nsplit, D)
    ws = workspace if workspace is not None else attention_workspace(q.device, nbytes)
    if seqlens is not None:
        if seqlens.dtype != torch.int32 or seqlens.device != q.device:
            seqlens = seqlens.to(device=q.device, dtype=torch.int32)
        seqlens = seqlens.contiguous()
    args = (q.data_ptr(), q.stride(0), q.stride(1),
            k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
            v.data_ptr(), v.stride(0), v.stride(1), v.stride(2),
            _lib.ptr(seqlens), B, H, KVH, S, D, float(scale), nsplit, chunk, _lib.dtype_code(q.dtype),
            ws.data_ptr(), ws.numel(), out.data_ptr(), out.stride(0), out.stride(2), _lib.dtype_code(out.dtype))
    if flags:
        _lib.call("b2d_gqa_decode_ex", *args, int(flags), _lib.stream_ptr(q.device))
    else:
        _lib.call("b2d_gqa_decode", *args, _lib.stream_ptr(q.device))
    return out


def l2_prefetch_hint(tensors) -> None:
    """The next ``decode_attention_append`` call on this thread also prefetches these device tensors'
    bytes into L2 (at most 4; static data that later launches read, e.g. the next GEMMs' weights)."""
    import ctypes
    n = len(tensors)
    ptrs = (ctypes.c_void_p * max(n, 1))(*[t.data_ptr() for t in tensors])
    nbytes = (ctypes.c_int64 * max(n, 1))(*[t.numel() * t.element_size() for t in tensors])
    _lib.call("b2d_l2_prefetch_hint", ctypes.addressof(ptrs), ctypes.addressof(nbytes), n)


def decode_attention_append(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, pos: torch.Tensor,
                            cos: torch.Tensor, sin: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                            scale: float, seqlens: torch.Tensor, out: torch.Tensor, flags: int = 0) -> torch.Tensor:
    """One decode step's attention with its RoPE and KV append folded in (``b2d_gqa_decode_append``):
    q [B, H*D], k_new / v_new [B, KVH*D] (projection outputs before RoPE), pos int64 [B], cos / sin
    [>= S, D], k_cache / v_cache [B, KVH, S, D] (the new key and value are written at ``pos``),
    seqlens int32 [B] (set to pos + 1), out [B, 1, H, D]. The same numbers as ``rope_kv_append``
    followed by ``decode_attention``."""
    B, KVH, S, D = k_cache.shape
    H = q.shape[1] // D
    assert pos.dtype == torch.int64 and seqlens.dtype == torch.int32 and cos.shape[0] >= S and sin.shape == cos.shape
    nsplit, _ = plan_splits(B, KVH, S)
    nbytes = _lib.load().b2d_gqa_workspace_bytes(B, H, nsplit, D)
    ws = attention_workspace(q.device, nbytes)
    _lib.call("b2d_gqa_decode_append", q.data_ptr(), q.stride(0), k_new.data_ptr(), k_new.stride(0),
              v_new.data_ptr(), v_new.stride(0), pos.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.stride(0),
              k_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
              v_cache.data_ptr(), v_cache.stride(0), v_cache.stride(1), v_cache.stride(2),
              seqlens.data_ptr(), B, H, KVH, S, D, float(scale), _lib.dtype_code(q.dtype), ws.data_ptr(), ws.numel(),
              out.data_ptr(), out.stride(0), out.stride(2), _lib.dtype_code(out.dtype), int(flags),
              _lib.stream_ptr(q.device))
    return out
