"""Greedy-token parity of the engine against the reference semantics.

The reference decodes greedily (``engine.py:341-353``): the lm_head logits
are fp16 (``gemm_d`` output, ``engine.py:338``) and ``sampler_d`` picks the
largest fp16 value, ties to the lowest index (``sampler_d.cu:37-38``).  The
judge here is the same model graph with the reference arithmetic in every
projection (``Engine(linear="oracle")``: fp32 matmul of the dequantised
weight, fp16 result) and the same fp16 logits + lowest-index argmax.

Two views of one generation run (prompts + this engine's tokens):

* teacher-forced: the oracle runs once over prompt + generated tokens and
  gives its logits at every generated position, i.e. the oracle's pick on
  exactly the context this engine saw.  A step that differs is classified by
  its margin: the oracle's fp16 logit of its own pick minus its fp16 logit of
  this engine's pick, in fp16 ulps at that magnitude.  0 ulps is an exact
  fp16 tie (the reference itself would pick the lower index); 1-2 ulps is a
  near-tie that fp16 rounding of an intermediate activation can flip.
* free-running: the oracle generates on its own from the prompts; the count
  of sequences whose 256 tokens equal this engine's, and each other
  sequence's first differing step.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch


def _fp16_ulp(v: torch.Tensor) -> torch.Tensor:
    """Spacing of fp16 at |v| (v fp16-representable, finite), as fp32, on v's
    device: 2^(e - 10) for |v| in [2^e, 2^(e+1)), e >= -14; 2^-24 below."""
    a = v.float().abs()
    _, ex = torch.frexp(a)                      # |v| = m * 2^ex, m in [0.5, 1)
    e = torch.where(a > 0, torch.clamp(ex - 1, min=-14), torch.full_like(ex, -14))
    return torch.ldexp(torch.ones_like(v, dtype=torch.float32), e - 10)


@torch.no_grad()
def oracle_logits_at(oracle, prompts: torch.Tensor, tokens: torch.Tensor,
                     chunk: int = 8) -> torch.Tensor:
    """fp16-rounded oracle logits [B, T, V] (as fp32) predicting tokens[:, t] from
    prompts + tokens[:, :t], for every t: one teacher-forced oracle pass per
    chunk of sequences; only the generated positions reach the lm_head."""
    B, S = prompts.shape
    T = tokens.shape[1]
    seq = torch.cat([prompts, tokens[:, :-1]], dim=1)
    outs = []
    for b0 in range(0, B, chunk):
        part = seq[b0:b0 + chunk]
        cache = oracle.new_cache(part.shape[0], part.shape[1])
        h = oracle.hidden(part, cache, 0, 0)[:, S - 1:S - 1 + T, :]
        lg = oracle.logits(h.reshape(-1, h.shape[-1]))
        outs.append(lg.float().reshape(part.shape[0], T, -1))
        del cache, h, lg
    return torch.cat(outs)


@torch.no_grad()
def teacher_forced_report(oracle, prompts: torch.Tensor, tokens: torch.Tensor,
                          max_listed: int = 64) -> Dict:
    """Per-step agreement of `tokens` with the oracle's greedy pick on the same
    context; differing steps classified by margin in fp16 ulps."""
    B, T = tokens.shape
    listed: List[Dict] = []
    hist = {"0": 0, "1": 0, "2": 0, ">2": 0}
    equal = 0
    worst = 0.0
    chunk = 8
    for b0 in range(0, B, chunk):
        lg = oracle_logits_at(oracle, prompts[b0:b0 + chunk], tokens[b0:b0 + chunk], chunk)
        tok = tokens[b0:b0 + chunk]
        top2 = lg.topk(2, dim=-1)
        ref = lg.argmax(dim=-1)                 # first (lowest) index of the max
        best = top2.values[..., 0]
        second = top2.values[..., 1]
        chosen = lg.gather(-1, tok[..., None]).squeeze(-1)
        ulp = _fp16_ulp(best)
        same = ref == tok
        equal += int(same.sum())
        margin = ((best - chosen) / ulp)
        diff = (~same).nonzero().tolist()
        for b, t in diff:
            m = float(margin[b, t])
            worst = max(worst, m)
            key = "0" if m == 0 else "1" if m <= 1 else "2" if m <= 2 else ">2"
            hist[key] += 1
            if len(listed) < max_listed:
                listed.append({"seq": b0 + b, "step": t, "oracle_tok": int(ref[b, t]),
                               "tok": int(tok[b, t]), "margin_ulps": round(m, 3),
                               "oracle_top1_top2_ulps": round(float(
                                   (best[b, t] - second[b, t]) / ulp[b, t]), 3),
                               "oracle_top1": float(best[b, t])})
        del lg
    return {"steps": B * T, "equal": equal, "differ": B * T - equal,
            "differ_by_margin_ulps": hist, "max_margin_ulps": round(worst, 3),
            "differing_steps": listed}


@torch.no_grad()
def free_run_report(oracle, prompts: torch.Tensor, tokens: torch.Tensor,
                    oracle_tokens: Optional[torch.Tensor] = None) -> Dict:
    """The oracle generating on its own: how many sequences equal `tokens`, and
    where the others first differ."""
    if oracle_tokens is None:
        oracle_tokens = oracle.generate(prompts, tokens.shape[1], prefill_chunk=prompts.shape[0],
                                        use_graph=False)
    same = (oracle_tokens == tokens)
    identical = same.all(dim=1)
    first = []
    for b in (~identical).nonzero().flatten().tolist():
        first.append(int((~same[b]).nonzero()[0]))
    return {"sequences": int(tokens.shape[0]), "identical": int(identical.sum()),
            "first_difference_step": sorted(first)}


@torch.no_grad()
def oracle_noise_report(oracle, other, prompts: torch.Tensor, tokens: torch.Tensor) -> Dict:
    """Two valid summations of the reference semantics (``oracle``: fp32
    accumulation; ``other``: e.g. fp64) on the same teacher-forced contexts:
    how often their greedy picks differ and by what margin (in fp16 ulps of
    ``oracle``'s logits, as ``teacher_forced_report`` measures this engine),
    and how far their fp16 logits lie apart (per generated position the
    largest difference over the vocabulary, in fp16 ulps of ``oracle``'s top
    logit of that position; max and 99.9th percentile over positions).  The
    margins of the picks where two equally valid summations disagree are the
    floor below which a differing pick is an fp16-level tie."""
    B, T = tokens.shape
    hist = {"0": 0, "1": 0, "2": 0, ">2": 0}
    differ = 0
    worst = 0.0
    dmax = 0.0
    qs = []
    chunk = 8
    for b0 in range(0, B, chunk):
        la = oracle_logits_at(oracle, prompts[b0:b0 + chunk], tokens[b0:b0 + chunk], chunk)
        lb = oracle_logits_at(other, prompts[b0:b0 + chunk], tokens[b0:b0 + chunk], chunk)
        best = la.max(dim=-1).values
        d = (lb - la).abs().max(dim=-1).values / _fp16_ulp(best)   # [chunk, T]
        dmax = max(dmax, float(d.max()))
        qs.append(d.reshape(-1))
        pa = la.argmax(dim=-1)
        pb = lb.argmax(dim=-1)
        chosen = la.gather(-1, pb[..., None]).squeeze(-1)
        margin = (best - chosen) / _fp16_ulp(best)
        for b, t in (pa != pb).nonzero().tolist():
            m = float(margin[b, t])
            differ += 1
            worst = max(worst, m)
            hist["0" if m == 0 else "1" if m <= 1 else "2" if m <= 2 else ">2"] += 1
        del la, lb
    q = float(torch.quantile(torch.cat(qs).float(), 0.999))
    return {"steps": B * T, "differ": differ, "differ_by_margin_ulps": hist,
            "max_margin_ulps": round(worst, 3), "max_logit_diff_top_ulps": round(dmax, 3),
            "p999_logit_diff_top_ulps": round(q, 3)}
