"""Generate the golden fixtures that pin the CPU oracle to the reference implementation.

Run in a container that has the reference checkout (read-only) and Triton:

    python tests/golden/make_golden.py /path/to/reference-checkout

* ``nf4_gemm_ref_*.npz`` -- outputs of the reference's own NF4 Triton kernel
  (``profiling/kernels/nf4_gemm.py:37-64``) executed by the Triton CPU interpreter
  (``TRITON_INTERPRET=1``; the autotuner is bypassed through ``.fn`` with an explicit
  tile). Quantised states come from ``oracle.nf4_ref`` (any valid bitsandbytes-format state
  works: the kernel only reads the stored tables). ``deq_*`` cases feed one-hot rows of x,
  so each output element is one dequantised weight as the reference computes it (fp32
  ``code[nib] * scale``, stored as bf16; the interpreter's bf16 store truncates).
* ``attn_ref_*.npz`` -- the reference's stock attention formula
  (``profiling/kernels/bench_attention.py:40-41``: ``repeat_kv`` from transformers + torch
  SDPA in fp32) with a boolean key mask for ragged lengths.

The fixtures are small and committed; the tests never need the reference checkout.
"""
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"
HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from oracle import nf4_ref  # noqa: E402


def _ref_kernel(ref_root):
    sys.path.insert(0, str(Path(ref_root) / "profiling"))
    from kernels import nf4_gemm  # the reference module (imports triton only)
    return nf4_gemm._nf4_gemm_kernel.fn


def _run_ref(kern, qw, x_bf16):
    M, K = x_bf16.shape
    N = qw.N
    packed = torch.from_numpy(qw.packed.copy())
    code = torch.from_numpy(qw.code.copy())
    if qw.nested:
        absmax = torch.from_numpy(qw.absmax.copy())
        code2 = torch.from_numpy(qw.code2.copy())
        absmax2 = torch.from_numpy(qw.absmax2.copy())
        offset = float(qw.offset)
    else:
        absmax = torch.from_numpy(qw.absmax.copy())
        code2 = absmax2 = absmax
        offset = 0.0
    y = torch.empty(M, N, dtype=torch.bfloat16)
    m_pad = 1 << max(0, (M - 1).bit_length())
    kern[(N // 16,)](x_bf16, packed, absmax, code2, absmax2, offset, code, y, M, N, K,
                     x_bf16.stride(0), y.stride(0), NESTED=qw.nested, M_PAD=m_pad,
                     BLOCK_N=16, BLOCK_K=128)
    return y


def _bits(t_bf16):
    return t_bf16.view(torch.int16).numpy().view(np.uint16)


def _state(qw):
    d = dict(N=qw.N, K=qw.K, nested=int(qw.nested), packed=qw.packed, absmax=qw.absmax, code=qw.code)
    if qw.nested:
        d.update(code2=qw.code2, absmax2=qw.absmax2, offset=np.float32(qw.offset))
    return d


def gemm_cases(kern):
    cases = [("plain_n64_k256_m3", 64, 256, 3, False, 11),
             ("plain_n128_k512_m8", 128, 512, 8, False, 12),
             ("nested_n128_k512_m4", 128, 512, 4, True, 13),
             ("nested_n64_k1024_m1", 64, 1024, 1, True, 14)]
    for name, N, K, M, nested, seed in cases:
        g = torch.Generator().manual_seed(seed)
        w = (torch.randn(N, K, generator=g) * 0.02).numpy()
        qw = nf4_ref.QuantizedWeight(w, nested)
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        y = _run_ref(kern, qw, x)
        np.savez_compressed(HERE / f"nf4_gemm_ref_{name}.npz", x_bf16=_bits(x), y_bf16=_bits(y), M=M, **_state(qw))
        print("wrote", name)


def dequant_cases(kern):
    for name, N, K, nested, seed in [("deq_plain_n64_k256", 64, 256, False, 21),
                                     ("deq_nested_n64_k1024", 64, 1024, True, 22)]:
        g = torch.Generator().manual_seed(seed)
        w = (torch.randn(N, K, generator=g) * 0.02).numpy()
        qw = nf4_ref.QuantizedWeight(w, nested)
        cols = []
        for k0 in range(0, K, 8):
            x = torch.zeros(8, K, dtype=torch.bfloat16)
            x[torch.arange(8), k0 + torch.arange(8)] = 1.0
            cols.append(_run_ref(kern, qw, x))       # [8, N] = W[:, k0:k0+8]^T
        wt = torch.cat(cols, 0).T.contiguous()      # [N, K] bf16
        np.savez_compressed(HERE / f"nf4_gemm_ref_{name}.npz", w_bf16=_bits(wt), **_state(qw))
        print("wrote", name)


def attention_cases():
    from transformers.integrations.sdpa_attention import repeat_kv
    import torch.nn.functional as F
    for name, B, H, KVH, S, D, lens, seed in [("b2_h8_kv2_s40_d64", 2, 8, 2, 40, 64, [40, 17], 31),
                                              ("b1_h4_kv1_s33_d128", 1, 4, 1, 33, 128, [33], 32),
                                              ("b3_h16_kv4_s48_d128", 3, 16, 4, 48, 128, [48, 1, 40], 33)]:
        g = torch.Generator().manual_seed(seed)
        q = torch.randn(B, H, 1, D, generator=g).half()
        k = torch.randn(B, KVH, S, D, generator=g).half()
        v = torch.randn(B, KVH, S, D, generator=g).half()
        sl = torch.tensor(lens, dtype=torch.int32)
        mask = (torch.arange(S)[None, :] < sl[:, None].long())[:, None, None, :]
        G = H // KVH
        out = F.scaled_dot_product_attention(q.float(), repeat_kv(k, G).float(), repeat_kv(v, G).float(),
                                             attn_mask=mask, scale=D ** -0.5).transpose(1, 2)
        np.savez_compressed(HERE / f"attn_ref_{name}.npz", q=q.numpy(), k=k.numpy(), v=v.numpy(),
                            seqlens=sl.numpy(), out=out.numpy(), scale=np.float32(D ** -0.5))
        print("wrote", name)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <path to the reference checkout>")
    ref_root = sys.argv[1]
    kern = _ref_kernel(ref_root)
    gemm_cases(kern)
    dequant_cases(kern)
    attention_cases()
