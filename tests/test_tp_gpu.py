"""GPU (2 GPUs): tensor-parallel decode (all-reduce after o_proj and down_proj: fused into the GEMM
epilogue, the peer-memory kernel, or NCCL) against the single-GPU engine and the stock HF greedy path.
Skipped on a machine with fewer than 2 GPUs."""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_decode_matches_single_gpu():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(_port()), str(ROOT / "tests" / "tp_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
    line = [ln for ln in res.stdout.splitlines() if ln.startswith("TP_RESULT")]
    assert res.returncode == 0 and line, res.stdout[-2000:] + res.stderr[-4000:]
    ranks = json.loads(line[0].split(" ", 1)[1])
    for r in ranks:
        for mode in ("fused", "peer", "nccl"):
            m = r[mode]
            assert m["max_rel_logit_diff_vs_1gpu"] < 2e-2, (mode, r)
            assert m["argmax_agree_vs_1gpu"] >= 0.9, (mode, r)
            assert m["greedy_equal_stock"], (mode, r)
            assert m["peer_errors"] == 0, (mode, r)
        # the fused all-reduce sums the same rounded partials in the same order as the peer kernel
        assert r["fused"]["logits_sha"] == r["peer"]["logits_sha"], r
    # the peer all-reduce gives every rank identical sums, so identical logits
    assert len({r["peer"]["logits_sha"] for r in ranks}) == 1, ranks
