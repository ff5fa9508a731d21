"""Tensor-parallel decode across the GPUs of one node (Megatron-style, one process per GPU).

The same split as transformers' Mistral ``base_model_tp_plan``: q/k/v/gate/up are split by output
rows (column parallel), o/down by input columns (row parallel), KV heads ``KVH / world`` per rank with
their ``H / KVH`` query heads kept together; after o_proj and after down_proj the partial hidden
states are summed across the ranks (fused into the GEMM epilogue, the one-shot peer kernel, or NCCL).
The decode engine splits lm_head by vocabulary rows (``lm_head.merge_keys`` merges the ranks' argmax);
embedding and norms stay replicated. No counterpart in the reference (single GPU); this is the
tensor-parallel mode it plans.

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
    None for the default one).

    ``all_reduce`` sums a tensor over the group in place: with ``enable_peer_allreduce`` (called once,
    collectively) through ``b2d_allreduce`` -- every rank pushes its slice into its peers' memory over
    NVLink and sums locally, one launch -- otherwise through NCCL.

    ``enable_fused_allreduce`` (collective) sets up the all-reduce fused into the row-parallel GEMM's
    epilogue: an ``NF4Group(mode="allreduce")`` launch with ``epilogue(site)`` pushes its partial
    product to every peer, and ``allreduce_add_rmsnorm(site, ...)`` sums the partials and applies the
    residual add + RMSNorm that follows. Each of a step's all-reduces has its own site; ``advance()``
    (once per step, after the last site) moves the device step counter the epochs are derived from."""
    rank: int
    world: int
    group: object = None
    _peer: object = None
    _fused: object = None

    def _symmetric_buffer(self, n_max: int, dtype, device):
        """One zero-filled buffer per rank, mapped by every peer (torch symmetric memory)."""
        import ctypes
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        from . import _lib
        nbytes = _lib.load().b2d_allreduce_buffer_bytes(n_max, self.world, _lib.dtype_code(dtype))
        if nbytes == 0:
            raise ValueError(f"unsupported all-reduce size {n_max} / world {self.world} / {dtype}")
        buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        buf.zero_()
        torch.cuda.synchronize(device)
        group = self.group if self.group is not None else dist.group.WORLD
        hdl = symm_mem.rendezvous(buf, group.group_name)
        ptrs = [int(p) for p in hdl.buffer_ptrs]
        dist.barrier(group=group, device_ids=[torch.device(device).index])
        return dict(buf=buf, hdl=hdl, n_max=int(n_max), ptrs=(ctypes.c_void_p * self.world)(*ptrs))

    def enable_peer_allreduce(self, n_max: int, dtype, device) -> None:
        """Map the buffers of the one-shot all-reduce of up to ``n_max`` elements."""
        self._peer = self._symmetric_buffer(n_max, dtype, device)

    def enable_fused_allreduce(self, rows: int, cols: int, sites: int, dtype, device) -> None:
        """Map the buffers of the GEMM-fused all-reduce of ``rows`` x ``cols`` outputs (tokens x
        hidden) at ``sites`` points per step, with a device step counter starting at 0."""
        from . import _lib
        n_max = 2 * ((rows + 1) // 2) * cols
        n_max += -n_max % 8
        f = self._symmetric_buffer(n_max, dtype, device)
        f["step"] = torch.zeros(1, dtype=torch.int64, device=device)
        f["sites"] = int(sites)
        f["eps"] = []
        for site in range(sites):
            e = _lib.AllreduceEpilogue()
            e.peer_bufs, e.rank, e.world, e.n_max = f["ptrs"], self.rank, self.world, n_max
            e.step, e.site, e.sites = f["step"].data_ptr(), site, sites
            f["eps"].append(e)
        self._fused = f

    def epilogue(self, site: int):
        """The ``b2d_allreduce_epilogue`` of one site (kept alive by this group)."""
        return self._fused["eps"][site]

    def allreduce_add_rmsnorm(self, site: int, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                              out: torch.Tensor, flags: int = 0) -> torch.Tensor:
        """residual += (sum over ranks of the site's partials); out = RMSNorm(residual) * weight."""
        import ctypes
        from . import _lib
        M, D = residual.shape
        _lib.call("b2d_allreduce_add_rmsnorm", ctypes.byref(self._fused["eps"][site]), residual.data_ptr(),
                  residual.stride(0), weight.data_ptr(), float(eps), out.data_ptr(), out.stride(0), M, D,
                  _lib.dtype_code(residual.dtype), int(flags), _lib.stream_ptr(residual.device))
        return out

    def advance(self) -> None:
        """Move the fused all-reduce to the next step (stream-ordered; capturable in a CUDA graph)."""
        self._fused["step"].add_(1)

    def peer_errors(self) -> int:
        """Timed-out waits recorded by the peer all-reduces on this rank (0 when healthy)."""
        n = 0
        for b in (self._peer, self._fused):
            if b is not None:
                n += int(b["buf"][256:260].view(torch.int32).item())
        return n

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return t
        if self._peer is not None and t.is_contiguous() and t.numel() <= self._peer["n_max"]:
            from . import _lib
            _lib.call("b2d_allreduce", t.data_ptr(), t.data_ptr(), t.numel(), _lib.dtype_code(t.dtype),
                      self._peer["ptrs"], self.rank, self.world, self._peer["n_max"], _lib.LAUNCH_PDL,
                      _lib.stream_ptr(t.device))
            return t
        import torch.distributed as dist
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
