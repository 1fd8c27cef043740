"""The drop-in at the reference engine's projection dispatch point
(``engine.py:85-86``), replayed on a B200.

``tests/golden/make_dropin.py`` ran the reference's own ``engine.py`` (2
Qwen2.5-0.5B-shaped layers, seeded fp16 weights) with ``_linear`` rebound to
``f8_forward(x, m.wq, m.scales, m.bias)`` and recorded every call's input as
the engine passed it, plus the greedy tokens and each step's logits.  Here
every recorded call goes through ``ddq_b200.gemm_fp8.f8_forward`` with the
module's own arguments (fp16 bias, ``[B, S, K]`` leading dims) and must give
the reference semantics; and this library's engine, built on the same
weights, must reproduce the reference engine's greedy tokens (a step may
differ only at an fp16-level tie of the reference engine's logits)."""
import os
import sys

import numpy as np
import pytest
import torch

from oracle import w8a16 as o

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_dropin as md  # noqa: E402

FIX = os.path.join(HERE, "golden", "dropin_engine.npz")
TIGHT = 3e-3


@pytest.fixture(scope="module")
def fix():
    return np.load(FIX)


def module_weight(w, name):
    key = "model.embed_tokens.weight" if name == "lm_head" else name + ".weight"
    b = None if name == "lm_head" else w.get(name + ".bias")
    return w[key], b


def test_fixture_follows_the_reference_graph(fix):
    """CPU check of the recorded call sequence: per forward, layer by layer
    q, k, v (fp16 bias, the same input), o, gate, up (the same input), down,
    then the tied lm_head; prefill inputs [1, 6, K], decode inputs [1, 1, K];
    every call satisfies the operator's argument contract."""
    mods = list(fix["call_module"])
    per_fwd = []
    for i in range(2):
        p = f"model.layers.{i}."
        per_fwd += [p + "self_attn.q_proj", p + "self_attn.k_proj", p + "self_attn.v_proj",
                    p + "self_attn.o_proj", p + "mlp.gate_proj", p + "mlp.up_proj",
                    p + "mlp.down_proj"]
    per_fwd.append("lm_head")
    steps = md.NEW_TOKENS
    assert mods == per_fwd * steps
    xs = fix["call_x"]
    for f in range(steps):
        base = f * len(per_fwd)
        S = md.PROMPT_LEN if f == 0 else 1
        for li in range(2):
            q, k, v, _, g, u, _ = range(base + 7 * li, base + 7 * li + 7)
            assert xs[q] == xs[k] == xs[v] and xs[g] == xs[u]
        for j in range(base, base + len(per_fwd)):
            x = fix[f"x{xs[j]}"]
            assert x.dtype == np.float16 and x.shape[:2] == (1, S)
    bias = list(fix["call_bias"])
    assert all((b == "float16") == ("_proj" in m and m.split(".")[-1] in ("q_proj", "k_proj",
                                                                           "v_proj"))
               for m, b in zip(mods, bias))


@pytest.mark.gpu
def test_every_recorded_call_through_f8_forward(fix, cuda_device):
    from ddq_b200 import gemm_fp8
    w = md.weights(int(fix["seed"]))
    cache = {}
    for name, xi, bk in zip(fix["call_module"], fix["call_x"], fix["call_bias"]):
        wt, b = module_weight(w, str(name))
        if name not in cache:
            wq, s = gemm_fp8.quantize(torch.from_numpy(wt).cuda())
            wq_ref, s_ref = o.quantize(wt.astype(np.float32))
            assert np.array_equal(wq.cpu().numpy(), wq_ref) and np.array_equal(s.cpu().numpy(),
                                                                               s_ref)
            cache[name] = (wq, s)
        wq, s = cache[name]
        x = fix[f"x{xi}"]
        bias = None if bk == "none" else torch.from_numpy(b).cuda()
        assert bias is None or bias.dtype == torch.float16
        y = gemm_fp8.f8_forward(torch.from_numpy(x).cuda(), wq, s, bias)
        assert y.shape == x.shape[:-1] + (wt.shape[0],) and y.dtype == torch.float16
        want = o.f8_forward(x.reshape(-1, x.shape[-1]), wq.cpu().numpy(), s.cpu().numpy(), b)
        err = o.normwise_rel_err(y.reshape(-1, wt.shape[0]).cpu().numpy(), want)
        assert err <= TIGHT, (name, err)


@pytest.mark.gpu
def test_engine_tokens_match_the_reference_engine(fix, cuda_device):
    from ddq_b200.engine import Config, Engine, FP8Linear
    w = md.weights(int(fix["seed"]))
    c = md.CFG
    cfg = Config(hidden_size=c["hidden_size"], intermediate_size=c["intermediate_size"],
                 num_hidden_layers=c["num_hidden_layers"],
                 num_attention_heads=c["num_attention_heads"],
                 num_key_value_heads=c["num_key_value_heads"], rms_norm_eps=c["rms_norm_eps"],
                 rope_theta=c["rope_theta"], vocab_size=c["vocab_size"])

    def t(k):
        return torch.from_numpy(w[k]).cuda()
    layers = []
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        a, m = p + "self_attn.", p + "mlp."
        layers.append({
            "in_norm": t(p + "input_layernorm.weight").float(),
            "post_norm": t(p + "post_attention_layernorm.weight").float(),
            "qkv": FP8Linear.quantize(torch.cat([t(a + "q_proj.weight"), t(a + "k_proj.weight"),
                                                 t(a + "v_proj.weight")]),
                                      torch.cat([t(a + "q_proj.bias"), t(a + "k_proj.bias"),
                                                 t(a + "v_proj.bias")])),
            "o": FP8Linear.quantize(t(a + "o_proj.weight")),
            "gate_up": FP8Linear.quantize(torch.cat([t(m + "gate_proj.weight"),
                                                     t(m + "up_proj.weight")])),
            "down": FP8Linear.quantize(t(m + "down_proj.weight"))})
    embed = t("model.embed_tokens.weight")
    eng = Engine(cfg, {"embed": embed, "final_norm": t("model.norm.weight").float(),
                       "layers": layers, "lm_head": FP8Linear.quantize(embed)}, "cuda")
    prompt = torch.from_numpy(fix["prompt"]).cuda()
    ref_tokens = fix["tokens"]
    # teacher-forced on the reference engine's tokens: each step sees its context
    teacher = torch.from_numpy(ref_tokens[None, :]).cuda()
    ours = eng.generate(prompt, len(ref_tokens), teacher=teacher).cpu().numpy()[0]
    for step, (a_tok, r_tok) in enumerate(zip(ours, ref_tokens)):
        if a_tok == r_tok:
            continue
        lg = fix["step_logits"][step, 0].astype(np.float32)
        best = lg[r_tok]
        ulp = float(np.spacing(np.float16(abs(best))))
        assert (best - lg[a_tok]) <= 2 * ulp, (step, a_tok, r_tok, best, lg[a_tok])
