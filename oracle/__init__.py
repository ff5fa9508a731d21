"""CPU oracle for the NF4 decode matmul and the GQA decode attention.

TEST INFRASTRUCTURE ONLY. Nothing in the product path imports this package: only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` use it, and only as the checker or as the timed CPU baseline.

Modules
-------
nf4_ref   numpy restatement of the bitsandbytes NF4 storage format (quantise, double
          quantise, dequantise) and of the reference path's matmul
          ``x.float() @ dequant(W).float().T``.
attn_ref  numpy/torch-CPU restatement of the reference's stock decode attention
          ``SDPA(q, repeat_kv(k), repeat_kv(v))`` with a per-sequence length mask.

Parity status: the storage layout and the dequant formula are pinned against the
reference's own Triton kernel, run through the Triton CPU interpreter to produce
``tests/golden/nf4_gemm_ref_*.npz`` (script: ``tests/golden/make_golden.py``).
The bitsandbytes 0.50.2 arithmetic that produced real checkpoints (its quantiser's
rounding thresholds and its codebook literals) is not installed here, so that part
is "parity unpinned": the quantiser below follows the published method.
"""
