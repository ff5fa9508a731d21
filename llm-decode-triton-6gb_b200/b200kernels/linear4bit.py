"""bitsandbytes-format NF4 linear layer (storage + stock forward) for machines without bitsandbytes.

The reference loads a bitsandbytes checkpoint whose linears are ``bnb.nn.Linear4bit`` with
``Params4bit`` weights (``profiling/common.py:37-42``) and reads exactly these attributes
(``profiling/kernels/nf4_gemm.py:78-92``): ``weight.data`` (uint8 packed nibbles, shape
``[N*K/2, 1]``) and ``weight.quant_state.{quant_type, blocksize, shape, nested, absmax, code,
offset, dtype, state2.{blocksize, code, absmax}}``. This module provides a layer with the same
attributes so the patch applies unchanged, plus:

* ``Linear4bit.from_linear`` -- quantise a dense ``nn.Linear`` on the device with the library's
  NF4 quantiser (blocksize 64, optional double quantisation of the scales, blocksize 256);
* ``Linear4bit.forward`` -- the STOCK path the reference compares against: dequantise the weight
  with plain torch ops (each fp32 multiply/add rounded separately, then one rounding to the compute
  dtype, as ``bitsandbytes.functional.dequantize_4bit``) and ``F.linear``. The patch rebinds
  ``forward`` to the B200 kernel, exactly as the reference rebinds ``bnb.nn.Linear4bit.forward``.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

from . import _lib

# QLoRA NF4 codebook (appendix E of the paper) and the signed dynamic 8-bit map used for double
# quantisation of the scales (dynamic tree quantisation: level i holds 2**i linear fractions of
# [0.1, 1] scaled by 10**(i-6), mirrored for the sign, plus 0 and 1).
NF4_CODE = [
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0]


def dynamic_map_signed() -> torch.Tensor:
    vals = []
    for i in range(7):
        n = 2 ** i
        edges = np.linspace(0.1, 1.0, n + 1)
        mids = (edges[:-1] + edges[1:]) / 2.0
        mag = 10.0 ** (i - 6)
        vals.extend((mag * mids).tolist())
        vals.extend((-mag * mids).tolist())
    vals.extend([0.0, 1.0])
    return torch.tensor(np.sort(np.asarray(vals, dtype=np.float64)).astype(np.float32))


class QuantState:
    """The subset of ``bitsandbytes.functional.QuantState`` the NF4 path reads."""

    def __init__(self, absmax, shape=None, code=None, blocksize=64, quant_type="nf4", dtype=torch.float16,
                 offset=None, state2=None):
        self.absmax = absmax
        self.shape = torch.Size(shape) if shape is not None else None
        self.code = code
        self.blocksize = blocksize
        self.quant_type = quant_type
        self.dtype = dtype
        self.offset = offset
        self.state2 = state2
        self.nested = state2 is not None

    def to(self, device):
        mv = lambda t: t.to(device) if isinstance(t, torch.Tensor) else t  # noqa: E731
        s2 = self.state2.to(device) if self.state2 is not None else None
        return QuantState(mv(self.absmax), self.shape, mv(self.code), self.blocksize, self.quant_type, self.dtype,
                          mv(self.offset), s2)


def quantize_nf4(w: torch.Tensor, nested: bool = True, code=None):
    """Quantise a CUDA tensor [N, K] (fp32/fp16/bf16) to (packed uint8 [N*K/2, 1], QuantState)."""
    if not w.is_cuda:
        raise ValueError("quantize_nf4 runs on the device; move the weight to CUDA first")
    N, K = w.shape
    w = w.contiguous()
    dev = w.device
    code = torch.tensor(NF4_CODE, dtype=torch.float32, device=dev) if code is None else code.to(dev).float()
    n = w.numel()
    packed = torch.empty(n // 2, dtype=torch.uint8, device=dev)
    absmax = torch.empty(n // 64, dtype=torch.float32, device=dev)
    s = _lib.stream_ptr(dev)
    _lib.call("b2d_nf4_quantize", w.data_ptr(), n, _lib.dtype_code(w.dtype), code.data_ptr(), packed.data_ptr(),
              absmax.data_ptr(), s)
    if not nested:
        return packed.view(-1, 1), QuantState(absmax, (N, K), code, 64, "nf4", w.dtype)
    code2 = dynamic_map_signed().to(dev)
    nb = absmax.numel()
    q = torch.empty(nb, dtype=torch.uint8, device=dev)
    absmax2 = torch.empty(-(-nb // 256), dtype=torch.float32, device=dev)
    offset = torch.empty((), dtype=torch.float32, device=dev)
    _lib.call("b2d_nf4_double_quant", absmax.data_ptr(), nb, code2.data_ptr(), q.data_ptr(), absmax2.data_ptr(),
              offset.data_ptr(), s)
    state2 = QuantState(absmax2, None, code2, 256, None, torch.float32)
    return packed.view(-1, 1), QuantState(q, (N, K), code, 64, "nf4", w.dtype, offset, state2)


def dequantize_torch(packed: torch.Tensor, qs: QuantState, dtype=None) -> torch.Tensor:
    """Stock dequant in plain torch ops (the reference's bitsandbytes path, restated)."""
    dtype = dtype or qs.dtype
    N, K = qs.shape
    p = packed.view(-1)
    idx = torch.stack(((p >> 4).long(), (p & 0xF).long()), dim=-1).view(-1)
    vals = qs.code.float()[idx].view(-1, 64)
    if qs.nested:
        q = qs.absmax.long()
        grp = torch.arange(q.numel(), device=q.device) // qs.state2.blocksize
        scale = qs.state2.code.float()[q] * qs.state2.absmax[grp]
        scale = scale + qs.offset
    else:
        scale = qs.absmax.float()
    return (vals * scale[:, None]).view(N, K).to(dtype)


class Linear4bit(nn.Module):
    """NF4 linear with bitsandbytes' attribute layout; ``forward`` is the stock dequant+matmul."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, compute_dtype=torch.float16,
                 device=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.compute_dtype = compute_dtype
        self.weight = nn.Parameter(torch.empty(out_features * in_features // 2, 1, dtype=torch.uint8, device=device),
                                   requires_grad=False)
        self.weight.quant_state = None
        self.bias = None if not bias else nn.Parameter(torch.zeros(out_features, dtype=compute_dtype, device=device))

    @classmethod
    def from_linear(cls, lin: nn.Linear, nested: bool = True, compute_dtype=None) -> "Linear4bit":
        w = lin.weight.data
        compute_dtype = compute_dtype or w.dtype
        mod = cls(lin.in_features, lin.out_features, lin.bias is not None, compute_dtype, device=w.device)
        packed, qs = quantize_nf4(w, nested=nested)
        qs.dtype = compute_dtype
        mod.weight = nn.Parameter(packed, requires_grad=False)
        mod.weight.quant_state = qs
        if lin.bias is not None:
            mod.bias = nn.Parameter(lin.bias.data.to(compute_dtype), requires_grad=False)
        return mod

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = dequantize_torch(self.weight.data, self.weight.quant_state, self.compute_dtype)
        out = F.linear(x.to(self.compute_dtype), w, self.bias)
        return out.to(x.dtype)

    def extra_repr(self) -> str:
        nested = self.weight.quant_state.nested if self.weight.quant_state is not None else None
        return f"in_features={self.in_features}, out_features={self.out_features}, nf4, nested={nested}"


def quantize_model_linears(model: nn.Module, nested: bool = True, skip=("lm_head",)) -> int:
    """Replace every ``nn.Linear`` (except names in ``skip``) by a ``Linear4bit`` in place, freeing
    each dense weight as it goes. Returns the number of layers replaced."""
    names = [n for n, m in model.named_modules() if isinstance(m, nn.Linear) and n.split(".")[-1] not in skip]
    for name in names:
        parent_name, _, attr = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        lin = getattr(parent, attr)
        setattr(parent, attr, Linear4bit.from_linear(lin, nested=nested))
        del lin
    return len(names)
