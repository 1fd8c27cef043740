"""GPU tests of the Qwen2-shaped engine on the W8A16 kernels.

The greedy tokens are judged against the same engine with the reference
semantics in every projection (fp32 matmul of the dequantised weight, fp16
result) and fp32 logits for the greedy pick.  The oracle is run teacher-forced
on this engine's tokens, so every step is compared on the same context; a
step may differ only where the oracle's own top logit and the logit of the
token this engine picked are within 2 fp16 ulps (a near-tie that fp32
summation order alone can flip)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def small_cfg():
    from ddq_b200.engine import Config
    return Config(hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, vocab_size=1000)


def judge(fp8, oracle, prompts, tokens):
    """Teacher-forced oracle logits at each generated position; returns (#equal, #near-tie)."""
    seq = torch.cat([prompts, tokens[:, :-1]], dim=1)
    logits, _ = oracle.forward(seq)
    S = prompts.shape[1]
    lg = logits[:, S - 1:, :].float()                   # predicts tokens[:, t]
    best = lg.max(dim=-1).values
    chosen = lg.gather(-1, tokens[..., None]).squeeze(-1)
    ulp = torch.from_numpy(np.spacing(np.abs(best.cpu().numpy()).astype(np.float16)).astype(
        np.float32)).to(lg.device)
    ref_ids = lg.argmax(dim=-1)
    equal = (ref_ids == tokens)
    near = (~equal) & ((best - chosen) <= 2 * ulp)
    assert bool((equal | near).all()), "a greedy pick differs from the oracle beyond a near-tie"
    return int(equal.sum()), int(near.sum())


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
    eq, near = judge(fp8, oracle, prompts, tokens)
    assert eq >= 0.95 * tokens.numel(), (eq, near)


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
    eq, near = judge(fp8, oracle, prompts, tokens)
    assert eq >= 0.9 * tokens.numel(), (eq, near)


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
    eq, near = judge(fp8, oracle, prompts, a)
    assert eq >= 0.95 * a.numel(), (eq, near)
