"""B200 (sm_100a) decode kernels behind the reference's ``kernels`` package surface.

    from b200kernels.nf4_gemm import NF4Weight            # fused NF4 dequant + skinny matmul
    from b200kernels.decode_attention import decode_attention   # split-K GQA flash-decoding
    from b200kernels.patch import patch_attention, patch_linear4bit, STATS

Every op runs in ``libb200decode.so`` (C ABI in ``include/b200decode.h``) through ctypes.
"""
from ._lib import LIB_PATH, load  # noqa: F401

__version__ = "1.0"
