"""Golden fixture of the drop-in at the reference engine's projection dispatch point.

This script imports the reference engine itself (``engine.py`` of
hdahroug/ddq) from a reference checkout, builds a 2-layer Qwen2.5-0.5B-shaped
``Engine`` with seeded random fp16 weights, quantizes every ``nn.Linear``
once, and rebinds the engine's projection dispatch point
(``engine.py:85-86``) the way a maintainer adopting this library would:

    engine._linear = lambda m, x: gemm_fp8.f8_forward(x, m.wq, m.scales, m.bias)

Here, with no GPU, ``f8_forward`` is the CPU oracle (the reference
semantics) behind the argument contract of ``ddq_b200.gemm_fp8.f8_forward``,
checked on every call: fp16 x of any leading dims with K last, uint8 wq
[N, K], fp32 scales [N], the module's own bias (fp16 after ``.to(dtype)``,
``engine.py:325``) or None.  The engine then runs unmodified: prefill of one
6-token prompt and 3 decode steps of ``Engine.generate`` (``engine.py:
341-353``).  The reference's CUDA operator modules, loaded by
``torch.utils.cpp_extension.load`` when ``engine.py`` is imported
(``engine.py:25-79``), are replaced for this run by CPU restatements of those
kernels (test infrastructure, defined below): RMSNorm (``RMSnorm_d.cu:23-
110``), the RoPE table and rotation (``RoPe_d.cu:12-128``), SwiGLU
(``SwiGLU_d.cu:12-42``) and the greedy sampler (``sampler_d.cu:10-70``).  The
fp16 GEMM and both FlashAttention modules are replaced by stubs that raise:
after the swap nothing may call the fp16 GEMM, and the flash paths run on
Hopper only (``engine.py:56-57, 225-251``); elsewhere the engine uses torch
SDPA.

Recorded in ``dropin_engine.npz`` (the weights are not stored: they are
regenerated from the seed by ``weights()``):
* every ``_linear`` call: module name, x exactly as the engine passed it
  (leading dims included; identical inputs stored once), bias dtype;
* the prompt, the greedy tokens and the fp16 logits of each step's last
  position (what ``sampler_d`` saw).

tests/test_dropin_gpu.py replays every recorded call through
``gemm_fp8.f8_forward`` on a B200 and judges this library's engine, built on
the same weights, against the recorded tokens and logits.

    python tests/golden/make_dropin.py [--reference DIR]
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "dropin_engine.npz")

SEED = 20260
CFG = {"hidden_size": 896, "intermediate_size": 4864, "num_hidden_layers": 2,
       "num_attention_heads": 14, "num_key_value_heads": 2, "rms_norm_eps": 1e-6,
       "rope_theta": 1000000.0, "max_position_embeddings": 64, "vocab_size": 1024}
PROMPT_LEN, NEW_TOKENS = 6, 4


def weights(seed=SEED, cfg=CFG):
    """Seeded fp16 weights keyed by the reference module names (numpy, so any
    machine regenerates the same bytes): projections and the embedding
    N(0, 0.02), q/k/v biases N(0, 0.02), norm weights 1."""
    rng = np.random.default_rng(seed)
    H, I, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    hd = H // cfg["num_attention_heads"]
    nkv = cfg["num_key_value_heads"] * hd

    def n(*shape):
        return rng.normal(0, 0.02, shape).astype(np.float32).astype(np.float16)

    w = {"model.embed_tokens.weight": n(cfg["vocab_size"], H),
         "model.norm.weight": np.ones(H, np.float16)}
    for i in range(L):
        p = f"model.layers.{i}."
        w.update({p + "self_attn.q_proj.weight": n(H, H), p + "self_attn.q_proj.bias": n(H),
                  p + "self_attn.k_proj.weight": n(nkv, H), p + "self_attn.k_proj.bias": n(nkv),
                  p + "self_attn.v_proj.weight": n(nkv, H), p + "self_attn.v_proj.bias": n(nkv),
                  p + "self_attn.o_proj.weight": n(H, H),
                  p + "mlp.gate_proj.weight": n(I, H), p + "mlp.up_proj.weight": n(I, H),
                  p + "mlp.down_proj.weight": n(H, I),
                  p + "input_layernorm.weight": np.ones(H, np.float16),
                  p + "post_attention_layernorm.weight": np.ones(H, np.float16)})
    return w


def prompt(seed=SEED, cfg=CFG):
    return np.random.default_rng(seed + 1).integers(0, cfg["vocab_size"], (1, PROMPT_LEN))


# ----------------------------------------------------------------------------- CPU stand-ins
def _cpu_operator_modules(torch, record):
    """CPU restatements of the reference's operator modules, by the names
    engine.py loads them under."""
    F = torch.nn.functional

    def rmsnorm_forward(x, weight, eps=1e-6):          # RMSnorm_d.cu:23-87
        xf = x.float()
        rms = torch.rsqrt(xf.pow(2).sum(-1, keepdim=True) / x.shape[-1] + eps)
        return (xf * rms * weight.float()).half()

    def rope_init_table(inv_freq, max_seq_len):         # RoPe_d.cu:70-87, 113-128
        t = torch.arange(max_seq_len, dtype=torch.float32)[:, None]
        a = t * inv_freq.float()[None, :]
        return [a.cos().half(), a.sin().half()]

    def rope_forward(x, cos, sin):                       # RoPe_d.cu:12-68
        half = x.shape[-1] // 2
        v0, v1 = x[..., :half].float(), x[..., half:].float()
        c, s = cos.float()[None, None], sin.float()[None, None]
        return torch.cat([v0 * c - v1 * s, v0 * s + v1 * c], dim=-1).half()

    def swiglu_forward(gate, up):                        # SwiGLU_d.cu:12-26
        g, u = gate.float(), up.float()
        return ((g / (1.0 + torch.exp(-g))) * u).half()

    def sampler_forward(logits):                         # sampler_d.cu:10-70
        record["logits"].append(logits.reshape(logits.shape[0], -1).clone())
        return logits.reshape(logits.shape[0], -1).float().argmax(-1, keepdim=True)

    def refuse(name):
        def f(*a, **k):
            raise RuntimeError(f"{name} must not be called in the drop-in run")
        return f

    return {
        "engine_rmsnorm": types.SimpleNamespace(forward=rmsnorm_forward),
        "engine_rope": types.SimpleNamespace(init_table=rope_init_table, forward=rope_forward),
        "engine_swiglu": types.SimpleNamespace(forward=swiglu_forward),
        "engine_sampler": types.SimpleNamespace(forward=sampler_forward),
        "engine_gemm": types.SimpleNamespace(forward=refuse("the fp16 GEMM (gemm_d)")),
        "engine_fa": types.SimpleNamespace(forward=refuse("FA_d")),
        "engine_fad": types.SimpleNamespace(forward=refuse("FAD_d")),
    }, F


def f8_forward_contract(torch, x, wq, scales, bias):
    """The argument contract of ddq_b200.gemm_fp8.f8_forward (and of the
    reference's f8_forward, gemm_FP8_d.cu:171-210, widened to fp32 bias),
    checked on CPU tensors; raises like the library would."""
    if x.dtype != torch.float16:
        raise RuntimeError("gemm_fp8: fp16 x required")
    if wq.dtype != torch.uint8:
        raise RuntimeError("gemm_fp8: wq must be uint8 e4m3")
    if wq.dim() != 2 or wq.size(0) != scales.numel():
        raise RuntimeError("gemm_fp8: shape mismatch")
    if scales.dtype != torch.float32:
        raise RuntimeError("gemm_fp8: scales must be fp32 CUDA")
    if x.dim() < 1 or x.size(-1) != wq.size(1):
        raise RuntimeError("gemm_fp8: inner dim mismatch")
    if bias is not None and bias.numel() > 0:
        if bias.numel() != wq.size(0):
            raise RuntimeError("gemm_fp8: bias length mismatch")
        if bias.dtype not in (torch.float16, torch.float32):
            raise RuntimeError("gemm_fp8: bias must be fp16 or fp32 CUDA")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get(
        "DDQ_REFERENCE_DIR", os.path.join(os.path.dirname(REPO), "reference")))
    a = ap.parse_args()
    import torch
    import torch.utils.cpp_extension as ce
    sys.path.insert(0, REPO)
    from oracle import w8a16 as o

    record = {"logits": [], "calls": [], "xs": [], "x_keys": {}}
    mods, _ = _cpu_operator_modules(torch, record)
    real_load = ce.load
    ce.load = lambda name, **kw: mods[name]
    try:
        spec = importlib.util.spec_from_file_location("ref_engine",
                                                      os.path.join(a.reference, "engine.py"))
        eng_mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(eng_mod)
    finally:
        ce.load = real_load

    torch.manual_seed(0)
    engine = eng_mod.Engine(eng_mod._Config(dict(CFG)))
    w = weights()
    sd = {k: torch.from_numpy(v) for k, v in w.items()}
    missing, unexpected = engine.load_state_dict(sd, strict=False)
    assert not unexpected and set(missing) <= {"lm_head.weight"}, (missing, unexpected)
    engine.lm_head.weight = engine.model.embed_tokens.weight      # engine.py:323
    engine = engine.to(torch.float16).eval()                      # engine.py:325 (CPU)

    names = {}
    for name, m in engine.named_modules():
        if isinstance(m, torch.nn.Linear):
            wq, s = o.quantize(m.weight.detach().float().numpy())
            m.wq, m.scales = torch.from_numpy(wq), torch.from_numpy(s)
            names[id(m)] = name

    def linear(m, x):  # the swapped dispatch point
        f8_forward_contract(torch, x, m.wq, m.scales, m.bias)
        key = (x.data_ptr(), tuple(x.shape))
        if key not in record["x_keys"]:
            record["x_keys"][key] = len(record["xs"])
            record["xs"].append(x.detach().clone().numpy())
        b = None if m.bias is None else m.bias.detach().numpy()
        record["calls"].append((names[id(m)], record["x_keys"][key],
                                "none" if b is None else str(b.dtype)))
        x2 = x.detach().reshape(-1, x.shape[-1]).numpy()
        y = o.f8_forward(x2, m.wq.numpy(), m.scales.numpy(), b)
        return torch.from_numpy(y).reshape(*x.shape[:-1], -1)

    eng_mod._linear = linear
    ids = torch.from_numpy(prompt())
    with torch.no_grad():
        tokens = engine.generate(ids, max_new_tokens=NEW_TOKENS)
    calls = record["calls"]
    out = {"prompt": ids.numpy(), "tokens": np.array(tokens, np.int64),
           "step_logits": np.stack([lg.numpy() for lg in record["logits"]]),
           "call_module": np.array([c[0] for c in calls]),
           "call_x": np.array([c[1] for c in calls], np.int64),
           "call_bias": np.array([c[2] for c in calls]),
           "seed": np.array(SEED), "prompt_len": np.array(PROMPT_LEN)}
    for i, x in enumerate(record["xs"]):
        out[f"x{i}"] = x
    np.savez_compressed(OUT, **out)
    print(f"{len(calls)} calls, {len(record['xs'])} distinct inputs, tokens {tokens} -> {OUT}")


if __name__ == "__main__":
    main()
