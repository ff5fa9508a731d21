"""GPU: greedy decode through the B200 kernels vs the stock HF path on seeded random-init models.

Stock path = HF ``MistralForCausalLM`` forward with a ``DynamicCache``, NF4 linears dequantised by
plain torch ops + ``F.linear``, SDPA attention (the reference's ``04_compare.py`` "stock" variant).
Compared: (a) the drop-in path -- the same HF forward after ``patch_linear4bit`` +
``patch_attention``; (b) the static-cache CUDA-graph engine. Greedy tokens must be identical; on a
random-init model logits are nearly flat, so the first-step logits are also compared directly.
"""
import pytest
import torch

from b200kernels import decode as dec
from b200kernels import patch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
SMALL = dict(hidden_size=1024, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2, head_dim=128,
             intermediate_size=2048, vocab_size=2048)


def prompts(B, P, vocab, seed=1):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (B, P), generator=g).to(DEV)


@pytest.fixture(scope="module")
def small_model():
    return dec.build_random_mistral(seed=0, **SMALL)


def test_engine_matches_stock_small(small_model):
    ids = prompts(4, 64, SMALL["vocab_size"])
    stock, stock_logits = dec.hf_greedy(small_model, ids, 32, return_logits=True)
    eng = dec.DecodeEngine(small_model, 4, 128)
    ours = eng.generate(ids, 32)
    assert torch.equal(ours, stock), (ours != stock).float().mean().item()


def test_patched_hf_matches_stock_small(small_model):
    ids = prompts(3, 40, SMALL["vocab_size"], seed=2)
    stock, ls = dec.hf_greedy(small_model, ids, 24, return_logits=True)
    patch.patch_attention()
    patch.patch_linear4bit(small_model, verbose=False)
    try:
        patch.STATS.update(attn_triton=0, attn_fallback=0)
        ours, lo = dec.hf_greedy(small_model, ids, 24, return_logits=True)
        assert patch.STATS["attn_triton"] > 0 and patch.STATS["attn_kernel"] == patch.STATS["attn_triton"]
    finally:
        patch.unpatch_attention()
        patch.unpatch_linear4bit(small_model)
    assert torch.equal(ours, stock)
    # first decode step logits: B200 kernels vs stock, within the fp16 rounding of the logits
    d = (lo[:, 1] - ls[:, 1]).abs().max().item()
    assert d < 2e-2 * ls[:, 1].abs().max().item(), d


def test_engine_step_is_graph_replay(small_model):
    eng = dec.DecodeEngine(small_model, 2, 96)
    ids = prompts(2, 16, SMALL["vocab_size"], seed=3)
    eng.prefill(ids)
    eng.capture()
    a = [eng.step().clone() for _ in range(4)]
    eng.prefill(ids)                        # same prompts again: replays give the same tokens
    b = [eng.step().clone() for _ in range(4)]
    assert all(torch.equal(x, y) for x, y in zip(a, b))
    assert int(eng.pos[0]) == 16 + 4


def _first_div(a, b):
    return [(r != s).nonzero()[0].item() if (r != s).any() else None for r, s in zip(a, b)]


def near_tie_report(preds, stock, ol, sl):
    """Every teacher-forced step where our argmax differs from the stock one, with the evidence that it is
    a rounding near-tie: the stock logits' margin between the stock choice and ours, the largest logit
    error of ours at that step (the measured error bound there), and whether ours is the stock runner-up.

    preds [B, T-1] / ol [B, T-1, V]: our predictions and logits after consuming stock[:, :t]; stock [B, T]
    and sl [B, T, V]: the stock tokens and logits (sl[:, t] predicts stock[:, t])."""
    flips = []
    for b, j in (preds != stock[:, 1:]).nonzero().tolist():
        s, o = sl[b, j + 1], ol[b, j]
        ours, theirs = int(preds[b, j]), int(stock[b, j + 1])
        second = s.topk(2).values[1].item()
        flips.append({"seq": b, "step": j + 1, "stock": theirs, "ours": ours,
                      "stock_margin": (s[theirs] - s[ours]).item(),
                      "step_err_max": (o - s).abs().max().item(),
                      "ours_stock_rank": int((s > s[ours]).sum().item()) + 1,
                      "ours_is_stock_runner_up": s[ours].item() >= second})
    return flips


def test_mistral7b_greedy_128_vs_stock():
    """Full Mistral-7B shape (NF4, double quant), 4 x 256-token prompts, 128 greedy tokens.

    A random-init model has nearly flat logits, so greedy decoding amplifies any rounding difference
    at a near-tie. What is asserted:
      * teacher-forced (both paths consume the stock tokens): our logit error stays below 1% of the
        stock logits' standard deviation in RMS and 10% at its maximum over every step and vocabulary
        entry, and our argmax agrees with stock on >= 98% of the steps;
      * every teacher-forced step where the argmaxes differ is a near-tie: the stock margin between
        its choice and ours is within twice the largest logit error we make at that step (the
        measured bound there), so the stock logits cannot tell the two apart at our precision. Our
        choice's rank in the stock logits is reported (the runner-up in most flips; a third choice
        happens when three candidates lie within the bound);
      * every free-running divergence starts at such a step: up to its first differing token a
        sequence has consumed exactly the stock tokens, so its first divergence is one of the
        teacher-forced flips above.
    Reported: the flips with their margins, the free-running match, and a control (the stock path
    itself with an fp32-accumulated matmul, ``x.float() @ W.float().T`` -- equally valid rounding)."""
    import json
    from b200kernels import linear4bit

    B = 4
    model = dec.build_random_mistral(seed=0)
    ids = prompts(B, 256, model.config.vocab_size, seed=5)
    stock, sl = dec.hf_greedy(model, ids, 128, return_logits=True)
    eng = dec.DecodeEngine(model, B, 256 + 136)
    ours = eng.generate(ids, 128)
    preds, ol = eng.teacher_forced(ids, stock)
    scale = sl.std().item()
    err = ol - sl[:, 1:]
    rel = (err.abs().max() / scale).item()
    rms = (err.pow(2).mean().sqrt() / scale).item()
    agree = (preds == stock[:, 1:]).float().mean().item()
    flips = near_tie_report(preds, stock, ol, sl)

    orig = linear4bit.Linear4bit.forward

    def fp32_forward(self, x):
        w = linear4bit.dequantize_torch(self.weight.data, self.weight.quant_state, self.compute_dtype)
        return (x.float() @ w.float().T).to(x.dtype)

    linear4bit.Linear4bit.forward = fp32_forward
    try:
        ctl = dec.hf_greedy(model, ids, 128)
    finally:
        linear4bit.Linear4bit.forward = orig
    first_div = _first_div(ours, stock)
    report = {"teacher_forced_max_logit_err_over_std": rel, "teacher_forced_rms_logit_err_over_std": rms,
              "teacher_forced_argmax_agreement": agree, "teacher_forced_flips": flips,
              "ours_vs_stock_match": (ours == stock).float().mean().item(), "ours_first_div": first_div,
              "control_vs_stock_match": (ctl == stock).float().mean().item(),
              "control_first_div": _first_div(ctl, stock)}
    print("GREEDY_PARITY", json.dumps(report))
    assert rel < 0.1 and rms < 1e-2, report
    assert agree >= 0.98, report
    for f in flips:
        assert f["stock_margin"] <= 2 * f["step_err_max"], f
    flip_steps = {(f["seq"], f["step"]) for f in flips}
    for b, d in enumerate(first_div):
        if d is not None:
            assert d >= 1 and (b, d) in flip_steps, (b, d, sorted(flip_steps))
