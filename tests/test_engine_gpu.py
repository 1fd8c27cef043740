"""GPU tests of the Qwen2-shaped engine on the W8A16 kernels.

The greedy tokens are judged against the same engine with the reference
semantics in every projection (fp32 matmul of the dequantised weight, fp16
result) and fp16 logits with the reference sampler's lowest-index argmax.
The oracle is run teacher-forced on this engine's tokens, so every step is
compared on the same context; a step may differ only where the oracle's fp16
logit of its own pick and of the token this engine picked are within 2 fp16
ulps (a near-tie that the rounding of an intermediate fp16 activation can
flip) - on the full config-5 run, within one ulp of the largest margin at
which two valid summations of the reference semantics (fp32 and fp64
accumulation) disagree with each other on the same contexts.  No minimum
share of exact steps is assumed."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def small_cfg():
    from ddq_b200.engine import Config
    return Config(hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, vocab_size=1000)


def judge(fp8, oracle, prompts, tokens, max_ulps=2):
    """Teacher-forced oracle picks at each generated position; every step must
    equal the oracle's pick or be an fp16-level tie (the oracle's logit of its
    own pick and of this engine's pick within `max_ulps` fp16 ulps).  Returns
    the report (``ddq_b200.parity``)."""
    from ddq_b200 import parity
    rep = parity.teacher_forced_report(oracle, prompts, tokens)
    assert rep["max_margin_ulps"] <= max_ulps, rep
    return rep


def make_pair(cfg, seed=0):
    from ddq_b200.engine import Engine
    fp8 = Engine.random(cfg, "cuda", seed=seed)
    w = {"embed": fp8.embed, "final_norm": fp8.final_norm, "layers": fp8.layers,
         "lm_head": fp8.lm_head}
    oracle = Engine(cfg, w, "cuda", linear="oracle")
    return fp8, oracle


def test_small_engine_greedy_matches_oracle():
    cfg = small_cfg()
    fp8, oracle = make_pair(cfg)
    g = torch.Generator(device="cuda").manual_seed(1)
    prompts = torch.randint(0, cfg.vocab_size, (6, 40), generator=g, device="cuda")
    tokens = fp8.generate(prompts, 24, prefill_chunk=4)
    assert tokens.shape == (6, 24) and tokens.min() >= 0 and tokens.max() < cfg.vocab_size
    judge(fp8, oracle, prompts, tokens)


def test_graph_replay_equals_eager_decode():
    cfg = small_cfg()
    fp8, _ = make_pair(cfg, seed=2)
    g = torch.Generator(device="cuda").manual_seed(3)
    prompts = torch.randint(0, cfg.vocab_size, (4, 17), generator=g, device="cuda")
    a = fp8.generate(prompts, 12, use_graph=True)
    b = fp8.generate(prompts, 12, use_graph=False)
    assert torch.equal(a, b)


def test_forward_logits_match_oracle():
    from oracle import w8a16 as o
    cfg = small_cfg()
    fp8, oracle = make_pair(cfg, seed=4)
    g = torch.Generator(device="cuda").manual_seed(5)
    ids = torch.randint(0, cfg.vocab_size, (2, 33), generator=g, device="cuda")
    lf, _ = fp8.forward(ids)
    lo, _ = oracle.forward(ids)
    assert lf.shape == (2, 33, cfg.vocab_size) and lf.dtype == torch.float16
    err = o.normwise_rel_err(lf.reshape(-1, cfg.vocab_size).cpu().numpy(),
                             lo.reshape(-1, cfg.vocab_size).cpu().numpy())
    assert err < 2e-2, err


def test_full_size_engine_short_generation():
    """BASELINE config 5 architecture (24 layers, 151936 vocab) on a short run."""
    from ddq_b200.engine import Config
    cfg = Config()
    fp8, oracle = make_pair(cfg, seed=7)
    g = torch.Generator(device="cuda").manual_seed(8)
    prompts = torch.randint(0, cfg.vocab_size, (4, 64), generator=g, device="cuda")
    tokens = fp8.generate(prompts, 8, prefill_chunk=2)
    judge(fp8, oracle, prompts, tokens)


def test_decode_in_two_chains_matches_oracle_and_replays():
    """A decode batch of 64 runs as two 32-sequence slices on their own streams:
    the graph replay equals the eager run, and every pick agrees with the
    oracle up to near-ties."""
    cfg = small_cfg()
    fp8, oracle = make_pair(cfg, seed=9)
    assert fp8.decode_chains == 2
    g = torch.Generator(device="cuda").manual_seed(10)
    prompts = torch.randint(0, cfg.vocab_size, (64, 24), generator=g, device="cuda")
    a = fp8.generate(prompts, 10, prefill_chunk=8, use_graph=True)
    b = fp8.generate(prompts, 10, prefill_chunk=8, use_graph=False)
    assert torch.equal(a, b)
    judge(fp8, oracle, prompts, a)


def test_config5_greedy_parity():
    """BASELINE config 5 in full - 64 prompts of 512 uniform ids, 256 greedy
    tokens on the 24-layer Qwen2.5-0.5B shape (the bench's seeds) - judged
    step by step against the teacher-forced oracle.  Every step equals the
    oracle's greedy pick or is an fp16-level tie.  What counts as a tie is
    measured, not chosen: the same oracle with fp64 accumulation (another
    valid summation of the reference semantics) runs on the same contexts,
    and the largest margin at which the two oracles' picks disagree is the
    reference's own floor; a differing step of this engine may lie at most
    one ulp above it (and is always allowed up to 2 ulps).  Measured on B200:
    the two oracles disagree on 102 of 16,384 steps (max 3 ulps), this
    engine and the fp32 oracle on 87 (max 2 ulps).  The oracles, the
    kernels and the seeds are deterministic, so the test is too.  The
    free-running oracle's agreement is reported, not asserted: after a tie
    flips one token the two continuations are different texts."""
    import json
    from ddq_b200 import parity
    from ddq_b200.engine import Config, Engine
    cfg = Config()
    fp8, oracle = make_pair(cfg, seed=99)
    w = {"embed": fp8.embed, "final_norm": fp8.final_norm, "layers": fp8.layers,
         "lm_head": fp8.lm_head}
    oracle64 = Engine(cfg, w, "cuda", linear="oracle64")
    g = torch.Generator(device="cuda").manual_seed(1000)
    prompts = torch.randint(0, cfg.vocab_size, (64, 512), generator=g, device="cuda")
    tokens = fp8.generate(prompts, 256)
    rep = parity.teacher_forced_report(oracle, prompts, tokens)
    floor = parity.oracle_noise_report(oracle, oracle64, prompts, tokens)
    free = parity.free_run_report(oracle, prompts, tokens)
    print(json.dumps({"teacher_forced": {k: v for k, v in rep.items() if k != "differing_steps"},
                      "reference_floor": floor, "differing_steps": rep["differing_steps"][:16],
                      "free_run": free}))
    assert rep["steps"] == 64 * 256 and floor["steps"] == 64 * 256
    assert rep["max_margin_ulps"] <= max(2.0, floor["max_margin_ulps"] + 1.0), (rep, floor)
    assert free["sequences"] == 64
