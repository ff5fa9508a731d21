"""Tensor-parallel decode across the GPUs of one node (Megatron-style, one process per GPU).

The same split as transformers' Mistral ``base_model_tp_plan``: q/k/v/gate/up are split by output
rows (column parallel), o/down by input columns (row parallel), KV heads ``KVH / world`` per rank with
their ``H / KVH`` query heads kept together; after o_proj and after down_proj the partial hidden
states are summed with an NCCL all-reduce. Embedding, norms and lm_head stay replicated. No
counterpart in the reference (single GPU); this is the tensor-parallel mode it plans.

NF4 shards are cut from the bitsandbytes tensors without re-quantising: a column-parallel shard is a
row range of packed bytes and per-block scales; a row-parallel shard is a column range of every row.
Double-quantised group scales (``absmax2``) stay whole and are indexed by each block's position in
the full tensor (``gblk_base``/``gblk_row_stride``), so the shard dequantises to exactly the same
values as the corresponding slice of the full weight.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .nf4_gemm import NF4Weight

COLWISE = ("q", "k", "v", "gate", "up")
ROWWISE = ("o", "down")


@dataclass
class TPGroup:
    """This process's place in the tensor-parallel group (``group`` is a torch.distributed group or
    None for the default one)."""
    rank: int
    world: int
    group: object = None

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t


def shard_ranges(cfg, world: int, rank: int) -> dict:
    """name -> ("rows" | "cols", (start, end)) for one decoder layer's seven linears."""
    H, KVH = cfg.num_attention_heads, cfg.num_key_value_heads
    D = getattr(cfg, "head_dim", None) or cfg.hidden_size // H
    inter = cfg.intermediate_size
    if KVH % world or H % world or inter % world:
        raise ValueError(f"tensor parallel size {world} must divide KV heads {KVH}, heads {H} and {inter}")
    hq, hk, fi = H // world * D, KVH // world * D, inter // world
    return {"q": ("rows", (rank * hq, (rank + 1) * hq)),
            "k": ("rows", (rank * hk, (rank + 1) * hk)),
            "v": ("rows", (rank * hk, (rank + 1) * hk)),
            "gate": ("rows", (rank * fi, (rank + 1) * fi)),
            "up": ("rows", (rank * fi, (rank + 1) * fi)),
            "o": ("cols", (rank * hq, (rank + 1) * hq)),
            "down": ("cols", (rank * fi, (rank + 1) * fi))}


def shard_layer(weights: dict, cfg, world: int, rank: int) -> dict:
    """This rank's NF4 shards (contiguous copies) of one layer's ``{name: NF4Weight}``."""
    out = {}
    for name, (kind, rng) in shard_ranges(cfg, world, rank).items():
        w = weights[name]
        out[name] = w.shard(rows=rng, copy=True) if kind == "rows" else w.shard(cols=rng, copy=True)
    return out


def local_heads(cfg, world: int, rank: int) -> tuple[int, int, int, int]:
    """(first query head, query heads, first KV head, KV heads) of this rank."""
    H, KVH = cfg.num_attention_heads, cfg.num_key_value_heads
    return rank * H // world, H // world, rank * KVH // world, KVH // world
