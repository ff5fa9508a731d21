"""Swap the B200 kernels into a loaded Hugging Face Mistral-shaped model.

Same surface as the reference's ``profiling/kernels/patch.py``:

  patch_attention()        decode steps (q_len == 1, no mask, q/k same dtype) -> B200 flash-decoding
                           (``patch.py:19-24,27-29``); everything else -> HF's SDPA path
  unpatch_attention()      restore HF's SDPA attention function (``patch.py:32-33``)
  patch_linear4bit(model)  every NF4 ``Linear4bit`` -> B200 fused dequant+matmul for M <= 64 rows
                           (``patch.py:43-59``); larger M (prefill) -> bit-exact B200 dequant + cuBLAS
  STATS                    attention fast-path / fallback counters (``patch.py:16``)

``patch_linear4bit`` matches bitsandbytes' ``bnb.nn.Linear4bit`` when bitsandbytes is importable,
and this package's ``Linear4bit`` otherwise. It returns ``{(N, K): (set of M on the B200 kernel,
{M: (stock_us, kernel_us)})}`` like the reference; the timing table is filled only with
``calibrate=True`` and never changes which path runs (no per-shape dispatch).
"""
from __future__ import annotations

import types

import torch
import torch.nn.functional as F
from transformers import AttentionInterface
from transformers.integrations.sdpa_attention import sdpa_attention_forward

from .decode_attention import decode_attention
from .linear4bit import Linear4bit
from .nf4_gemm import NF4Weight, calibrate as _calibrate

class _Stats(dict):
    """Attention path counters with the reference's keys (``attn_triton``: decode steps served by the
    fast kernel, ``attn_fallback``: calls handed to HF's SDPA). ``attn_kernel`` is accepted as another
    name for ``attn_triton`` (reads, writes and ``update``)."""

    _ALIAS = {"attn_kernel": "attn_triton"}

    def __getitem__(self, k):
        return super().__getitem__(self._ALIAS.get(k, k))

    def __setitem__(self, k, v):
        super().__setitem__(self._ALIAS.get(k, k), v)

    def get(self, k, default=None):
        return super().get(self._ALIAS.get(k, k), default)

    def update(self, *args, **kw):
        for k, v in dict(*args, **kw).items():
            self[k] = v


STATS = _Stats(attn_triton=0, attn_fallback=0)


def _attention(module, query, key, value, attention_mask, scaling=None, **kwargs):
    if query.shape[2] == 1 and attention_mask is None and query.dtype == key.dtype:
        STATS["attn_triton"] += 1
        return decode_attention(query, key, value, scaling), None
    STATS["attn_fallback"] += 1
    return sdpa_attention_forward(module, query, key, value, attention_mask, scaling=scaling, **kwargs)


def patch_attention():
    # The hook takes over the "sdpa" name rather than registering a new one: models configured for
    # SDPA keep building their masks the SDPA way, and that builder passes no mask at all when a decode
    # step needs none, which is the condition the fast path above tests for.
    AttentionInterface.register("sdpa", _attention)


def unpatch_attention():
    AttentionInterface.register("sdpa", sdpa_attention_forward)


def _linear4bit_types():
    types_ = [Linear4bit]
    try:  # pragma: no cover - bitsandbytes is not installed on the build machines
        import bitsandbytes as bnb
        types_.append(bnb.nn.Linear4bit)
    except Exception:
        pass
    return tuple(types_)


def _forward(self, x):
    M = x.numel() // x.shape[-1]
    xc = x.to(self.compute_dtype)
    if M <= NF4Weight.MAX_M:
        return self.nf4.matmul(xc).to(x.dtype)
    # prefill-sized M: bit-exact dequant on the device, then a library GEMM
    w = self.nf4.dequantize(self.compute_dtype)
    return F.linear(xc, w, getattr(self, "bias", None)).to(x.dtype)


def patch_linear4bit(model, verbose=True, calibrate=False):
    """Returns {(N, K): (set of M using the B200 kernel, {M: (stock_us, kernel_us)})}."""
    by_shape = {}
    lin_types = _linear4bit_types()
    for name, mod in model.named_modules():
        if not isinstance(mod, lin_types):
            continue
        mod.nf4 = NF4Weight(mod.weight)
        mod.forward_bnb = types.MethodType(type(mod).forward, mod)
        shape = (mod.nf4.N, mod.nf4.K)
        if shape not in by_shape:
            table = _calibrate(mod, mod.nf4)[1] if calibrate else {}
            by_shape[shape] = (set(range(NF4Weight.MIN_M, NF4Weight.MAX_M + 1)), table)
            if verbose:
                print(f"  {name:28s} {shape}: B200 kernel for M in [{NF4Weight.MIN_M}, {NF4Weight.MAX_M}]"
                      + (f"   (stock_us, kernel_us) {table}" if table else ""))
        mod.kernel_m = by_shape[shape][0]
        mod.forward = types.MethodType(_forward, mod)
    return by_shape


def unpatch_linear4bit(model):
    for _, mod in model.named_modules():
        if hasattr(mod, "forward_bnb"):
            mod.forward = mod.forward_bnb
            del mod.forward_bnb


def is_patched(model) -> bool:
    return any(hasattr(m, "nf4") and hasattr(m, "forward_bnb") for m in model.modules())


__all__ = ["STATS", "patch_attention", "unpatch_attention", "patch_linear4bit", "unpatch_linear4bit",
           "is_patched", "torch"]
