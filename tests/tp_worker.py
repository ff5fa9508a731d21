"""One rank of the tensor-parallel decode check (launched by tests/test_tp_gpu.py under
torch.distributed.run, one process per GPU, NCCL). Every rank builds the same seeded model, decodes
with its shards (all-reduce after o_proj and down_proj, captured in the CUDA graph) and compares the
teacher-forced logits with the unsharded engine on its own GPU, for each all-reduce mode (fused into
the GEMM epilogue, peer kernel, NCCL). Rank 0 prints one JSON line."""
import datetime
import hashlib
import json
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "llm-decode-triton-6gb_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from b200kernels import decode as dec  # noqa: E402
from b200kernels.tp import TPGroup  # noqa: E402

SMALL = dict(hidden_size=1024, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2, head_dim=128,
             intermediate_size=2048, vocab_size=2048)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        model = dec.build_random_mistral(seed=0, **SMALL)
        B = 4
        ids = torch.randint(0, SMALL["vocab_size"], (B, 32), generator=torch.Generator().manual_seed(5)).to(dev)
        stock = dec.hf_greedy(model, ids, 12)
        one = dec.DecodeEngine(model, B, 64)
        p_one, l_one = one.teacher_forced(ids, stock)
        res = {"rank": rank, "world": world}
        for mode in ("fused", "peer", "nccl"):
            grp = TPGroup(rank, world)
            tp_eng = dec.DecodeEngine(model, B, 64, tp=grp, allreduce=mode)
            p_tp, l_tp = tp_eng.teacher_forced(ids, stock)
            ours = tp_eng.generate(ids, 12)
            tp_eng.graph = None
            torch.cuda.synchronize(dev)
            res[mode] = {"max_rel_logit_diff_vs_1gpu": (l_tp - l_one).abs().max().item() / l_one.abs().max().item(),
                         "argmax_agree_vs_1gpu": (p_tp == p_one).float().mean().item(),
                         "greedy_equal_stock": bool(torch.equal(ours, stock)), "peer_errors": grp.peer_errors(),
                         "logits_sum": float(l_tp.double().sum()),
                         "logits_sha": hashlib.sha256(l_tp.float().cpu().numpy().tobytes()).hexdigest()}
            dist.barrier(device_ids=[dev.index])
        out = [None] * world
        dist.all_gather_object(out, res)
        if rank == 0:
            print("TP_RESULT", json.dumps(out), flush=True)
        torch.cuda.synchronize(dev)
        dist.barrier(device_ids=[dev.index])
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
