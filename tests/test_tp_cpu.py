"""CPU (gloo, world size 2): the tensor-parallel split of the decode step.

Each rank cuts its NF4 shards of one decoder layer with the same code the GPU engine uses
(``b200kernels.tp.shard_layer``); the oracle dequantises every shard through its strided view and
must reproduce the matching slice of the full weight bit for bit (including double-quantised group
scales indexed by the block's position in the full tensor). A row-parallel product all-reduced over
gloo and the column-parallel products all-gathered then equal the unsharded products.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from transformers import MistralConfig

from b200kernels.nf4_gemm import NF4Weight
from b200kernels.tp import local_heads, shard_layer, shard_ranges
from oracle import nf4_ref

CFG = dict(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=64, intermediate_size=1024,
           num_hidden_layers=1, vocab_size=64)
SHAPES = {"q": (256, 256), "k": (128, 256), "v": (128, 256), "o": (256, 256), "gate": (1024, 256),
          "up": (1024, 256), "down": (256, 1024)}


def make_layer(seed, nested):
    rng = np.random.default_rng(seed)
    qw, nf = {}, {}
    for i, (name, (N, K)) in enumerate(SHAPES.items()):
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        q = nf4_ref.QuantizedWeight(w, nested)
        qw[name] = q
        t = lambda a, dt=None: None if a is None else torch.from_numpy(np.ascontiguousarray(a))
        nf[name] = NF4Weight.from_parts(t(q.packed), t(q.absmax), t(q.code), N, K, nested, t(q.code2), t(q.absmax2),
                                        float(q.offset))
    return qw, nf


def _worker(rank, world, port, nested, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = MistralConfig(**CFG)
        qw, nf = make_layer(7, nested)
        shards = shard_layer(nf, cfg, world, rank)
        for name, (kind, (a, b)) in shard_ranges(cfg, world, rank).items():
            s, q = shards[name], qw[name]
            full = q.dequantize("fp16")
            ref = full[a:b] if kind == "rows" else full[:, a:b]
            got = nf4_ref.dequantize_view(s.packed.view(s.N, s.ld_packed).numpy(),
                                          s.absmax.view(s.N, s.ld_absmax).numpy(), s.K, "fp16", s.nested,
                                          None if s.code2 is None else s.code2.numpy(),
                                          None if s.absmax2 is None else s.absmax2.numpy(), s.offset,
                                          s.gblk_base, s.gblk_row_stride, s.code.numpy())
            assert got.shape == ref.shape and np.array_equal(got, ref), (rank, name)
        # row parallel o_proj: partial products summed across ranks == full product
        x = torch.from_numpy(np.random.default_rng(3).standard_normal((3, 256))).double()
        wo = torch.from_numpy(qw["o"].dequantize("fp16").astype(np.float64))
        a, b = shard_ranges(cfg, world, rank)["o"][1]
        part = x[:, a:b] @ wo[:, a:b].T
        dist.all_reduce(part)
        assert torch.allclose(part, x @ wo.T, rtol=1e-12, atol=1e-12)
        # column parallel q: this rank's heads; gathered in rank order == full product
        wq = torch.from_numpy(qw["q"].dequantize("fp16").astype(np.float64))
        a, b = shard_ranges(cfg, world, rank)["q"][1]
        mine = x @ wq[a:b].T
        got = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(got, mine)
        assert torch.allclose(torch.cat(got, 1), x @ wq.T, rtol=1e-12, atol=1e-12)
        h0, hl, kv0, kvl = local_heads(cfg, world, rank)
        assert (h0, hl, kv0, kvl) == (rank * 2, 2, rank, 1)
        results[rank] = "ok"
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("nested", [True, False])
def test_tp_shards_and_collectives_gloo(nested):
    world = 2
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), nested, results), nprocs=world, join=True)
    assert dict(results) == {0: "ok", 1: "ok"}


def test_shard_ranges_reject_uneven_split():
    cfg = MistralConfig(**CFG)
    with pytest.raises(ValueError):
        shard_ranges(cfg, 4, 0)          # 2 KV heads cannot be split 4 ways
