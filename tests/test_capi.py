"""CPU: the C-ABI library loads, exports every symbol the header declares, and validates its
arguments before touching a device (no compute calls here)."""
import ctypes as C
import re
from pathlib import Path

import pytest

from b200kernels import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "b200decode.h"


def declared_symbols():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(b2d_[a-z0-9_]+)\s*\(", text)))


def test_library_built_in_tree():
    assert _lib.LIB_PATH.exists(), "run __graft_entry__.build() first"
    assert _lib.LIB_PATH.parent.name == "b200kernels"


def test_exports_every_declared_symbol():
    lib = _lib.load()
    syms = declared_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(lib, s), s


def test_ctypes_signatures_cover_header():
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_header_argument_counts_match_ctypes():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    for name, (_, args) in _lib.SIGNATURES.items():
        m = re.search(rf"\b{name}\s*\(([^;]*?)\)\s*;", text, flags=re.S)
        assert m, name
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), (name, len(params), len(args))


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.b2d_strerror(0) == b"ok"
    assert b"shape" in lib.b2d_strerror(2)
    assert lib.b2d_version() >> 16 == 1


def test_workspace_size_arithmetic():
    lib = _lib.load()
    assert lib.b2d_gqa_workspace_bytes(8, 32, 16, 128) == 65536 + 8 * 32 * 16 * 130 * 4
    assert lib.b2d_gqa_workspace_bytes(0, 32, 16, 128) == 0


@pytest.mark.parametrize("M,N,K,dtype,ydt,expect", [
    (4, 17, 4096, 0, 0, 2),      # N % 16
    (4, 64, 100, 0, 0, 2),       # K % 64
    (65, 64, 256, 0, 0, 2),      # M > 64
    (4, 64, 256, 7, 7, 3),       # dtype
    (4, 64, 256, 0, 1, 3),       # output dtype neither input dtype nor fp32
    (0, 64, 256, 0, 0, 0),       # empty batch: nothing to do
    (4, 0, 256, 0, 0, 0),        # no output features
    (-1, 64, 256, 0, 0, 1),      # negative size
])
def test_gemm_argument_validation(M, N, K, dtype, ydt, expect):
    lib = _lib.load()
    st = lib.b2d_nf4_gemm(None, K, None, K // 2, None, K // 64, 0, None, None, 0.0, 0, K // 64, None,
                          None, N, M, N, K, dtype, ydt, None, 0, None)
    assert st == expect


def test_gemm_null_pointers_rejected():
    lib = _lib.load()
    assert lib.b2d_nf4_gemm(None, 256, None, 128, None, 4, 0, None, None, 0.0, 0, 4, None, None, 64,
                            4, 64, 256, 0, 0, None, 0, None) == 1


def test_attention_argument_validation():
    lib = _lib.load()
    # head_dim 96 unsupported, group 32/5 not integral, group > 16
    assert lib.b2d_gqa_decode(None, 0, 0, None, 0, 0, 0, None, 0, 0, 0, None, 1, 32, 8, 16, 96, 1.0, 0, 0, 0,
                              None, 0, None, 0, 0, 0, None) == 2
    assert lib.b2d_gqa_decode(None, 0, 0, None, 0, 0, 0, None, 0, 0, 0, None, 1, 32, 5, 16, 128, 1.0, 0, 0, 0,
                              None, 0, None, 0, 0, 0, None) == 2
    assert lib.b2d_gqa_decode(None, 0, 0, None, 0, 0, 0, None, 0, 0, 0, None, 1, 64, 2, 16, 128, 1.0, 0, 0, 0,
                              None, 0, None, 0, 0, 0, None) == 2
    assert lib.b2d_gqa_decode(None, 0, 0, None, 0, 0, 0, None, 0, 0, 0, None, 1, 32, 8, 16, 128, 1.0, 0, 0, 5,
                              None, 0, None, 0, 0, 5, None) == 3
    # empty batch is a no-op
    assert lib.b2d_gqa_decode(None, 0, 0, None, 0, 0, 0, None, 0, 0, 0, None, 0, 32, 8, 16, 128, 1.0, 0, 0, 0,
                              None, 0, None, 0, 0, 0, None) == 0


def test_dequant_and_quantize_validation():
    lib = _lib.load()
    assert lib.b2d_nf4_dequant(None, 0, None, 0, 0, None, None, 0.0, 0, 0, None, None, 0, 4, 100, 0, None) == 2
    assert lib.b2d_nf4_quantize(None, 100, 0, None, None, None, None) == 2
    assert lib.b2d_nf4_quantize(None, 0, 0, None, None, None, None) == 0
    assert lib.b2d_nf4_double_quant(None, -1, None, None, None, None, None) == 1


def test_device_calls_fail_loudly_without_gpu():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = _lib.load()
    # well-formed arguments reach the device query and report it missing
    buf = (C.c_uint8 * 64)()
    p = C.addressof(buf)
    st = lib.b2d_nf4_quantize(p, 64, 2, p, p, p, None)
    assert st == 7


def test_l2_prefetch_hint_validation():
    """The one-shot L2 hint is host-side only: its checks run without a GPU."""
    lib = _lib.load()
    buf = C.create_string_buffer(64 + 32)
    base = (C.addressof(buf) + 15) & ~15
    ptrs = (C.c_void_p * 5)(*([base] * 5))
    nb = (C.c_int64 * 5)(*([64] * 5))
    assert lib.b2d_l2_prefetch_hint(C.addressof(ptrs), C.addressof(nb), 0) == 0
    assert lib.b2d_l2_prefetch_hint(C.addressof(ptrs), C.addressof(nb), 4) == 0
    assert lib.b2d_l2_prefetch_hint(C.addressof(ptrs), C.addressof(nb), 5) == 1   # B2D_ERR_ARG
    assert lib.b2d_l2_prefetch_hint(None, None, 1) == 1   # B2D_ERR_ARG
    odd = (C.c_void_p * 1)(base + 8)
    assert lib.b2d_l2_prefetch_hint(C.addressof(odd), C.addressof(nb), 1) == 4   # B2D_ERR_ALIGN
    assert lib.b2d_l2_prefetch_hint(C.addressof(ptrs), C.addressof(nb), 0) == 0   # leaves no hint pending
