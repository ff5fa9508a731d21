"""Decode-step glue of a Mistral decoder layer as B200 kernels (no counterpart in the reference,
whose decode step runs these as torch ops inside transformers' ``MistralDecoderLayer``).

* ``add_rmsnorm`` -- ``residual += x`` then ``MistralRMSNorm`` (one kernel);
* ``rope_kv_append`` -- ``apply_rotary_pos_emb`` on q and k of one new token per sequence plus the
  KV-cache write (``DynamicCache.update`` / a static-cache index_copy) and the attention lengths;
* ``silu_mul`` -- ``act_fn(gate) * up``.

All take ``flags=_lib.LAUNCH_PDL`` to overlap their launch with the previous kernel's tail. Work
runs in ``libb200decode.so``; there is no fallback.
"""
from __future__ import annotations

import torch

from . import _lib


def add_rmsnorm(residual: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor,
                x: torch.Tensor | None = None, flags: int = 0) -> torch.Tensor:
    """residual [M, D] (updated in place to residual + x when x is given); out = RMSNorm(residual)."""
    M, D = residual.shape
    _lib.call("b2d_add_rmsnorm", _lib.ptr(x), 0 if x is None else x.stride(0), residual.data_ptr(),
              residual.stride(0), weight.data_ptr(), float(eps), out.data_ptr(), out.stride(0), M, D,
              _lib.dtype_code(residual.dtype), int(flags), _lib.stream_ptr(residual.device))
    return out


def rope_kv_append(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pos: torch.Tensor, cos: torch.Tensor,
                   sin: torch.Tensor, q_out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                   seqlens: torch.Tensor | None = None, flags: int = 0):
    """q [B, H*D], k/v [B, KVH*D] (projection outputs), pos int64 [B], cos/sin [S_max, D] ->
    q_out [B, H, D] (may alias q), k_cache/v_cache [B, KVH, S_max, D] at pos, seqlens = pos + 1."""
    B, KVH, S_max, D = k_cache.shape
    H = q_out.shape[1]
    assert pos.dtype == torch.int64 and cos.shape[0] >= S_max and sin.shape == cos.shape
    _lib.call("b2d_rope_kv_append", q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
              pos.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.stride(0),
              q_out.data_ptr(), q_out.stride(0), q_out.stride(1),
              k_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
              v_cache.data_ptr(), v_cache.stride(0), v_cache.stride(1), v_cache.stride(2),
              _lib.ptr(seqlens), B, H, KVH, D, S_max, _lib.dtype_code(q.dtype), int(flags), _lib.stream_ptr(q.device))


def silu_mul(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor | None = None, flags: int = 0) -> torch.Tensor:
    """out = act_fn(gate) * up for [M, N] tensors, rounded like the torch ops."""
    M, N = gate.shape
    if out is None:
        out = torch.empty_like(gate)
    _lib.call("b2d_silu_mul", gate.data_ptr(), gate.stride(0), up.data_ptr(), up.stride(0), out.data_ptr(),
              out.stride(0), M, N, _lib.dtype_code(gate.dtype), int(flags), _lib.stream_ptr(gate.device))
    return out
