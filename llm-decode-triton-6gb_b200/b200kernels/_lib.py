"""ctypes binding of libb200decode.so (the C ABI declared in include/b200decode.h).

There is no fallback: if the shared library is missing or no sm_100 device is present the
calls raise. Tensors cross the boundary as raw device pointers plus sizes/strides; the CUDA
stream is torch's current stream for the tensors' device.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libb200decode.so"

B2D_OK = 0
F16, BF16, F32 = 0, 1, 2

_p, _i64, _i32, _f32, _sz = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_size_t

LAUNCH_PDL, STATIC_WEIGHTS, ATTN_FUSED_COMBINE, KV_STATIC_PREFIX = 1, 2, 4, 8   # launch flags
SEG_INDEPENDENT, SEG_SILU_MUL, SEG_ALLREDUCE = 0, 1, 2   # b2d_nf4_gemm_multi modes


class Nf4Segment(C.Structure):
    """b2d_nf4_segment (include/b200decode.h)."""
    _fields_ = [("packed", _p), ("ld_packed", _i64), ("absmax", _p), ("ld_absmax", _i64),
                ("code2", _p), ("absmax2", _p), ("offset", _f32), ("gblk_base", _i64),
                ("gblk_row_stride", _i64), ("code", _p), ("N", _i32), ("y", _p), ("ldy", _i64)]


class AllreduceEpilogue(C.Structure):
    """b2d_allreduce_epilogue (include/b200decode.h)."""
    _fields_ = [("peer_bufs", C.POINTER(C.c_void_p)), ("rank", _i32), ("world", _i32), ("n_max", _i64),
                ("step", _p), ("site", _i32), ("sites", _i32)]


# name -> (restype, argtypes); mirrors include/b200decode.h
SIGNATURES = {
    "b2d_strerror": (C.c_char_p, [_i32]),
    "b2d_last_cuda_error": (C.c_char_p, []),
    "b2d_version": (_i32, []),
    "b2d_nf4_dequant": (_i32, [_p, _i64, _p, _i64, _i32, _p, _p, _f32, _i64, _i64, _p,
                               _p, _i64, _i64, _i64, _i32, _p]),
    "b2d_nf4_gemm_workspace_bytes": (_sz, [_i32, _i32, _i32]),
    "b2d_nf4_gemm": (_i32, [_p, _i64, _p, _i64, _p, _i64, _i32, _p, _p, _f32, _i64, _i64, _p,
                            _p, _i64, _i32, _i32, _i32, _i32, _i32, _p, _sz, _p]),
    "b2d_nf4_gemv_simt": (_i32, [_p, _i64, _p, _i64, _p, _i64, _i32, _p, _p, _f32, _i64, _i64, _p,
                                 _p, _i64, _i32, _i32, _i32, _i32, _i32, _p]),
    "b2d_nf4_quantize": (_i32, [_p, _i64, _i32, _p, _p, _p, _p]),
    "b2d_nf4_double_quant": (_i32, [_p, _i64, _p, _p, _p, _p, _p]),
    "b2d_gqa_default_splits": (_i32, [_i32, _i32, _i32]),
    "b2d_gqa_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "b2d_gqa_decode_partial": (_i32, [_p, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64, _i64,
                                      _p, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _i32, _i32, _p, _sz, _p]),
    "b2d_gqa_decode_combine": (_i32, [_p, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _p, _sz,
                                      _p, _i64, _i64, _p]),
    "b2d_gqa_decode": (_i32, [_p, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64, _i64,
                              _p, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _i32, _i32, _p, _sz,
                              _p, _i64, _i64, _i32, _p]),
    "b2d_nf4_gemm_multi": (_i32, [_p, _i64, C.POINTER(Nf4Segment), _i32, _i32, _i32, _i32, _i32, _i32,
                                  _i32, _i32, C.POINTER(C.c_float), C.POINTER(AllreduceEpilogue), _p, _sz, _p]),
    "b2d_gqa_decode_ex": (_i32, [_p, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64, _i64,
                                 _p, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _i32, _i32, _p, _sz,
                                 _p, _i64, _i64, _i32, _i32, _p]),
    "b2d_gqa_decode_append": (_i32, [_p, _i64, _p, _i64, _p, _i64, _p, _p, _p, _i64,
                                     _p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p,
                                     _i32, _i32, _i32, _i32, _i32, _f32, _i32, _p, _sz,
                                     _p, _i64, _i64, _i32, _i32, _p]),
    "b2d_l2_prefetch_hint": (_i32, [_p, _p, _i32]),
    "b2d_add_rmsnorm": (_i32, [_p, _i64, _p, _i64, _p, _f32, _p, _i64, _i32, _i32, _i32, _i32, _p]),
    "b2d_rope_kv_append": (_i32, [_p, _i64, _p, _i64, _p, _i64, _p, _p, _p, _i64, _p, _i64, _i64,
                                  _p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p,
                                  _i32, _i32, _i32, _i32, _i32, _i32, _i32, _p]),
    "b2d_silu_mul": (_i32, [_p, _i64, _p, _i64, _p, _i64, _i32, _i32, _i32, _i32, _p]),
    "b2d_allreduce_buffer_bytes": (_sz, [_i64, _i32, _i32]),
    "b2d_allreduce": (_i32, [_p, _p, _i64, _i32, C.POINTER(C.c_void_p), _i32, _i32, _i64, _i32, _p]),
    "b2d_lm_head_workspace_bytes": (_sz, [_i32]),
    "b2d_lm_head_argmax": (_i32, [_p, _i64, _p, _i64, _i32, _i32, _i32, _i64, _p, _i64, _p, _p, _i32, _i32, _p, _sz,
                                  _p]),
    "b2d_allreduce_add_rmsnorm": (_i32, [C.POINTER(AllreduceEpilogue), _p, _i64, _p, _f32, _p, _i64, _i32, _i32,
                                         _i32, _i32, _p]),
    "b2d_gqa_decode_noalloc": (_i32, [_p, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64, _i64,
                                      _p, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _i32, _i32,
                                      _p, _i64, _i64, _i32, _p]),
}

_lib = None


class B2DError(RuntimeError):
    def __init__(self, fn: str, status: int):
        lib = load()
        msg = lib.b2d_strerror(status).decode()
        detail = lib.b2d_last_cuda_error().decode()
        super().__init__(f"{fn} failed with status {status} ({msg}){': ' + detail if detail else ''}")
        self.status = status


def load():
    """Load (once) and return the ctypes handle; raises if the library has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python llm-decode-triton-6gb_b200/build.py` "
                               "(or __graft_entry__.build()); there is no fallback implementation")
        import torch  # noqa: F401  (loads torch's CUDA runtime first; the library shares it)
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Call an int-status entry point and raise B2DError on a nonzero status."""
    st = getattr(load(), name)(*args)
    if st != B2D_OK:
        raise B2DError(name, st)


def dtype_code(dt) -> int:
    import torch
    if dt == torch.float16:
        return F16
    if dt == torch.bfloat16:
        return BF16
    if dt == torch.float32:
        return F32
    raise TypeError(f"unsupported dtype {dt}")


def stream_ptr(device) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()
