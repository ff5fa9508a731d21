"""CPU: the Mistral-7B tensor-parallel splits used by ``bench.py --gpus N`` (N = 1, 2, 4, 8) meet every
shape and alignment rule the B200 entry points check (include/b200decode.h), so each rank's launches
are valid before any GPU runs them:

* NF4 shards (``NF4Weight.shard`` arithmetic): K a multiple of 256 (whole 4-block units), 4-block
  aligned double-quantisation group indexing (``gblk_base``, ``gblk_row_stride`` % 4), q/k/v segment
  rows % 32, paired gate/up rows % 16 and equal;
* the GEMM-fused all-reduce: ``(B + 1) / 2 * hidden <= n_max / 2`` with ``n_max % 8 == 0``;
* the vocabulary-parallel lm_head: vocab % N == 0, K % 256 == 0, at most 8 rows;
* attention: whole KV heads per rank with their query heads.
"""
import pytest
from transformers import MistralConfig

from b200kernels.tp import local_heads, shard_ranges

MISTRAL_7B = dict(hidden_size=4096, num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                  intermediate_size=14336, num_hidden_layers=32, vocab_size=32000)
FULL = {"q": (4096, 4096), "k": (1024, 4096), "v": (1024, 4096), "o": (4096, 4096), "gate": (14336, 4096),
        "up": (14336, 4096), "down": (4096, 14336)}


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_mistral7b_tp_shards_meet_kernel_rules(world):
    cfg = MistralConfig(**MISTRAL_7B)
    for rank in range(world):
        shapes = {}
        for name, (kind, (a, b)) in shard_ranges(cfg, world, rank).items():
            N, K = FULL[name]
            r0, r1, k0, k1 = (a, b, 0, K) if kind == "rows" else (0, N, a, b)
            n, k = r1 - r0, k1 - k0
            stride = K // 64                                  # blocks per full row
            base = r0 * stride + k0 // 64                     # NF4Weight.shard's gblk_base
            assert k % 256 == 0 and (k // 64) % 4 == 0, (world, rank, name, k)
            assert base % 4 == 0 and stride % 4 == 0, (world, rank, name, base, stride)
            assert n % 16 == 0, (world, rank, name, n)
            shapes[name] = (n, k)
        for name in ("q", "k", "v", "o", "down"):
            assert shapes[name][0] % 32 == 0, (world, rank, name)
        assert shapes["gate"] == shapes["up"]
        # the o/down outputs are the full hidden size on every rank (row-parallel partial sums)
        assert shapes["o"][0] == shapes["down"][0] == cfg.hidden_size
        h0, hl, kv0, kvl = local_heads(cfg, world, rank)
        assert kvl >= 1 and hl == kvl * (cfg.num_attention_heads // cfg.num_key_value_heads)
        assert shapes["q"][0] == hl * 128 and shapes["k"][0] == kvl * 128


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("batch", [1, 3, 8])
def test_fused_allreduce_and_vocab_split_sizes(world, batch):
    hidden, vocab = MISTRAL_7B["hidden_size"], MISTRAL_7B["vocab_size"]
    n_max = 2 * ((batch + 1) // 2) * hidden          # TPGroup.enable_fused_allreduce
    n_max += -n_max % 8
    assert n_max % 8 == 0 and (batch + 1) // 2 * hidden <= n_max // 2
    assert vocab % world == 0 and hidden % 256 == 0 and batch <= 8
