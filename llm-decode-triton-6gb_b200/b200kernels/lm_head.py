"""lm_head + greedy argmax in one launch (``b2d_lm_head_argmax``).

Replaces the reference decode step's ``lm_head`` GEMV followed by ``logits.argmax(-1)``
(``profiling/common.py`` ``decode_step``): the fp16/bf16 head weight is streamed once, the logits are
rounded to the model dtype exactly as the torch GEMV's output would be, and each row's argmax (first
index of the maximum, torch's rule) is formed on the device. For a vocabulary-parallel shard,
``vocab_offset`` shifts the indices and ``keys`` returns packed (value, index) maxima that merge across
ranks by a plain maximum (``merge_keys``). Work runs in ``libb200decode.so``; there is no fallback.
"""
from __future__ import annotations

import torch

from . import _lib

MAX_M = 64
_WS: dict = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-initialised scratch per (device, stream); the kernel returns its counter to zero."""
    stream = torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _WS[key] = ws
    return ws


def lm_head_argmax(x: torch.Tensor, weight: torch.Tensor, logits: torch.Tensor | None = None,
                   ids: torch.Tensor | None = None, keys: torch.Tensor | None = None, vocab_offset: int = 0,
                   flags: int = 0):
    """x [M, K] (M <= 64), weight [V, K] -> (logits [M, V] or None, ids int64 [M] or None, keys or None).

    Pass preallocated outputs to reuse them (CUDA-graph capture); with none given, logits and ids are
    allocated."""
    assert x.dim() == 2 and weight.dim() == 2 and x.shape[1] == weight.shape[1], (x.shape, weight.shape)
    assert x.stride(1) == 1 and weight.stride(1) == 1 and x.dtype == weight.dtype
    M, K = x.shape
    V = weight.shape[0]
    if logits is None and ids is None and keys is None:
        logits = torch.empty(M, V, dtype=x.dtype, device=x.device)
        ids = torch.empty(M, dtype=torch.int64, device=x.device)
    if ids is not None:
        assert ids.dtype == torch.int64 and ids.is_contiguous() and ids.numel() >= M
    if keys is not None:
        assert keys.dtype == torch.int64 and keys.is_contiguous() and keys.numel() >= M
    if logits is not None:
        assert logits.dtype == x.dtype and logits.stride(1) == 1 and tuple(logits.shape) == (M, V)
    nbytes = _lib.load().b2d_lm_head_workspace_bytes(V)
    ws = _workspace(x.device, nbytes)
    _lib.call("b2d_lm_head_argmax", x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0), M, V, K,
              int(vocab_offset), _lib.ptr(logits), 0 if logits is None else logits.stride(0), _lib.ptr(ids),
              _lib.ptr(keys), _lib.dtype_code(x.dtype), int(flags), ws.data_ptr(), ws.numel(),
              _lib.stream_ptr(x.device))
    return logits, ids, keys


def merge_keys(keys: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """[R, M] packed keys of R vocabulary shards -> int64 ids [M] of the overall maxima."""
    best = keys.max(0).values
    ids = 0xFFFFFFFF - (best & 0xFFFFFFFF)
    if out is None:
        return ids
    out.copy_(ids)
    return out
