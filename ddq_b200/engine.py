"""Qwen2-shaped greedy engine whose projections run on the W8A16 kernels.

Mirrors the reference engine (``engine.py`` of hdahroug/ddq) layer for
layer - embedding, 24 x [RMSNorm -> QKV (+bias) -> RoPE -> KV cache ->
attention -> O -> +residual -> RMSNorm -> gate/up -> SwiGLU -> down ->
+residual], final RMSNorm, lm_head tied to the embedding
(``engine.py:136-353``) - with three changes on the hot path:

* every projection is an e4m3 W8A16 GEMM from this library (the reference's
  ``_linear`` dispatch point, ``engine.py:85-86``, now calls
  ``gemm_fp8.f8_forward``); q/k/v are stacked into one GEMM, and gate/up
  into one GEMM whose epilogue applies SwiGLU (``gemm_fp8.f8_forward_swiglu``:
  the [M, 2I] gate/up output is never written), where the reference runs
  gate, up and ``swiglu_naive`` separately (``engine.py:189-193, 215-217``);
* a decode step's RoPE, KV-cache write and attention run as one kernel
  (``attention.decode_attention``) instead of the reference's RoPE kernel,
  cache copy and attention call (``engine.py:126-130, 225-251``);
* the lm_head runs only on the last position of each sequence and never
  writes logits: the fused kernel returns the greedy token directly
  (replacing ``engine.py:338`` + ``sampler_d`` at ``engine.py:345/351``);
* generation is batched (the reference's ``generate`` is batch-1,
  ``engine.py:346,352``) and each decode step is captured once in a CUDA
  graph and replayed.

The other operators run on this library's kernels too: residual add +
RMSNorm (``norm.add_rmsnorm``; on the decode path ``norm.add_rmsnorm_split``,
which also emits the next GEMM's operand), the prefill RoPE + cache write
(``attention.qkv_rope_kv``: in the q/k/v GEMM's epilogue at prefill sizes)
and the decode attention above.  Prefill
attention itself is ``scaled_dot_product_attention``.  Their arithmetic
follows the reference kernels (fp32 math, fp16 storage); the plain-PyTorch
versions of RMSNorm, RoPE and SwiGLU below serve the oracle engine.

``Engine(linear="oracle")`` swaps every projection for the reference
semantics in fp32 (dequantised weight, fp32 matmul, fp16 output) and the
lm_head for fp32 logits rounded to fp16 + lowest-index argmax: the same graph
with the reference arithmetic, used by the tests to judge the greedy tokens.
``linear="oracle64"`` is the same with fp64 accumulation (one rounding to
fp16): another valid summation of the reference semantics, which measures how
far fp32 summation order alone moves the fp16 logits.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.nn.functional as F

from . import attention, gemm_fp8, lm_head as lmh, norm

E4M3_DECODE_LUT = None


def _e4m3_lut(device):
    global E4M3_DECODE_LUT
    if E4M3_DECODE_LUT is None or E4M3_DECODE_LUT.device != device:
        b = torch.arange(256, dtype=torch.uint8)
        E4M3_DECODE_LUT = b.view(torch.float8_e4m3fn).float().to(device)
    return E4M3_DECODE_LUT


@dataclass
class Config:
    """Model shape (field names of the reference ``_Config``, ``engine.py:136-149``)."""
    hidden_size: int = 896
    intermediate_size: int = 4864
    num_hidden_layers: int = 24
    num_attention_heads: int = 14
    num_key_value_heads: int = 2
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    max_position_embeddings: int = 32768
    vocab_size: int = 151936

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @classmethod
    def from_dict(cls, raw: dict) -> "Config":
        keys = {f for f in cls.__dataclass_fields__}
        return cls(**{k: raw[k] for k in keys if k in raw})


class FP8Linear:
    """One projection: e4m3 weight [N,K] (uint8), fp32 per-row scale, optional fp32 bias."""

    def __init__(self, wq: torch.Tensor, scales: torch.Tensor, bias: Optional[torch.Tensor]):
        self.wq, self.scales, self.bias = wq, scales, bias
        self._wdeq = None
        self._il = None

    @classmethod
    def quantize(cls, w: torch.Tensor, bias: Optional[torch.Tensor] = None) -> "FP8Linear":
        wq, s = gemm_fp8.quantize(w.contiguous())
        return cls(wq, s, None if bias is None else bias.float().contiguous())

    def gate_up_interleaved(self):
        """(wq, scales, bias) of a stacked [gate; up] projection in the fused SwiGLU
        kernel's row order (``gemm_fp8.interleave_gate_up``), built once."""
        if self._il is None:
            self._il = gemm_fp8.interleave_gate_up(self.wq, self.scales, self.bias)
        return self._il

    def dequantized(self) -> torch.Tensor:
        """fp32 [N,K] = e4m3 value * scale (the reference semantics' weight)."""
        if self._wdeq is None:
            self._wdeq = _e4m3_lut(self.wq.device)[self.wq.long()] * self.scales[:, None]
        return self._wdeq


class KVCache:
    """Preallocated [L, B, Hkv, capacity, D] fp16 K/V (``engine.py:103-133``).

    The capacity is fixed up front (prompt + new tokens) so a decode step has
    static shapes and can be captured in a CUDA graph.
    """

    def __init__(self, cfg: Config, batch: int, capacity: int, device):
        shape = (cfg.num_hidden_layers, batch, cfg.num_key_value_heads, capacity, cfg.head_dim)
        self.k = torch.zeros(shape, dtype=torch.float16, device=device)
        self.v = torch.zeros(shape, dtype=torch.float16, device=device)
        self.capacity = capacity


class Engine:
    def __init__(self, cfg: Config, weights: dict, device, linear: str = "fp8"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.linear_kind = linear
        self.embed = weights["embed"]                 # fp16 [V, H]
        self.final_norm = weights["final_norm"]       # fp32 [H]
        self.layers = weights["layers"]
        self.lm_head: FP8Linear = weights["lm_head"]  # e4m3 copy of the embedding
        hd = cfg.head_dim
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, hd, 2, dtype=torch.float32) / hd))
        self._inv_freq2 = torch.cat([inv, inv]).to(self.device)  # both halves of a head
        self._split_bufs: dict = {}   # (tokens, hidden, stream) -> reusable split buffers
        # decode steps run as this many independent slices of >= 32 sequences
        # on their own streams (the step is latency-bound; the slices overlap;
        # measured: 64 = 2 x 32 beats 1 x 64 and 4 x 16, 1 x 32 beats 2 x 16)
        self.decode_chains = 2
        # decode steps of <= 64 sequences: the norms and the attention emit the
        # e4m3 planes of the split-plane decode GEMM (True), or fp16 operands
        # for the resident-slice GEMMs (False)
        self.decode_planes = True
        # prefill chunks: RoPE and the cache write in the q/k/v GEMM's epilogue
        # (True), or the GEMM and then the separate RoPE + cache kernel (False;
        # the same bits, one more launch and a round trip of the projection)
        self.fused_qkv_rope = True
        self._chain_streams: List[torch.cuda.Stream] = []
        self._graphs = {}

    # ------------------------------------------------------------------ construction
    @classmethod
    def random(cls, cfg: Config, device="cuda", seed: int = 0, linear: str = "fp8") -> "Engine":
        """Random-init weights as BASELINE config 5 states: N(0, 0.02) projections and
        embedding, N(0, 0.02) fp32 q/k/v biases, unit RMSNorm weights."""
        dev = torch.device(device)
        g = torch.Generator(device=dev).manual_seed(seed)
        H, I, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
        nq, nkv = cfg.num_attention_heads * hd, cfg.num_key_value_heads * hd

        def randn(*shape):
            return torch.randn(*shape, generator=g, device=dev) * 0.02

        layers = []
        for _ in range(cfg.num_hidden_layers):
            qkv_w = torch.cat([randn(nq, H), randn(nkv, H), randn(nkv, H)])
            qkv_b = torch.cat([randn(nq), randn(nkv), randn(nkv)])
            layers.append({
                "in_norm": torch.ones(H, device=dev),
                "post_norm": torch.ones(H, device=dev),
                "qkv": FP8Linear.quantize(qkv_w, qkv_b),
                "o": FP8Linear.quantize(randn(H, nq)),
                "gate_up": FP8Linear.quantize(torch.cat([randn(I, H), randn(I, H)])),
                "down": FP8Linear.quantize(randn(H, I)),
            })
            del qkv_w
        embed = randn(cfg.vocab_size, H)
        weights = {"embed": embed.half(), "final_norm": torch.ones(H, device=dev),
                   "layers": layers, "lm_head": FP8Linear.quantize(embed)}
        return cls(cfg, weights, dev, linear)

    @classmethod
    def load(cls, model_dir: str, device="cuda", linear: str = "fp8") -> "Engine":
        """Load a Qwen2 checkpoint (config.json + model.safetensors), as the reference's
        ``Engine.load`` (``engine.py:314-325``), quantizing every projection to e4m3 and
        tying the lm_head to the embedding (``engine.py:323``)."""
        from safetensors.torch import load_file
        cfg = Config.from_dict(json.load(open(os.path.join(model_dir, "config.json"))))
        sd = load_file(os.path.join(model_dir, "model.safetensors"), device="cpu")
        dev = torch.device(device)

        def t(name):
            return sd[name].to(dev)

        layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"model.layers.{i}."
            a = p + "self_attn."
            m = p + "mlp."
            layers.append({
                "in_norm": t(p + "input_layernorm.weight").float(),
                "post_norm": t(p + "post_attention_layernorm.weight").float(),
                "qkv": FP8Linear.quantize(
                    torch.cat([t(a + "q_proj.weight"), t(a + "k_proj.weight"), t(a + "v_proj.weight")]),
                    torch.cat([t(a + "q_proj.bias"), t(a + "k_proj.bias"), t(a + "v_proj.bias")])),
                "o": FP8Linear.quantize(t(a + "o_proj.weight")),
                "gate_up": FP8Linear.quantize(torch.cat([t(m + "gate_proj.weight"), t(m + "up_proj.weight")])),
                "down": FP8Linear.quantize(t(m + "down_proj.weight")),
            })
        embed = t("model.embed_tokens.weight")
        weights = {"embed": embed.half(), "final_norm": t("model.norm.weight").float(),
                   "layers": layers, "lm_head": FP8Linear.quantize(embed)}
        return cls(cfg, weights, dev, linear)

    def new_cache(self, batch: int, capacity: int) -> KVCache:
        return KVCache(self.cfg, batch, capacity, self.device)

    # ------------------------------------------------------------------ operators
    def linear(self, x: torch.Tensor, p: FP8Linear) -> torch.Tensor:
        """The projection dispatch point (reference ``_linear``, ``engine.py:85-86``)."""
        if self.linear_kind == "fp8":
            return gemm_fp8.f8_forward(x, p.wq, p.scales, p.bias)
        acc = torch.float64 if self.linear_kind == "oracle64" else torch.float32
        y = x.reshape(-1, x.shape[-1]).to(acc) @ p.dequantized().to(acc).T
        if p.bias is not None:
            y = y + p.bias.to(acc)
        return y.half().reshape(*x.shape[:-1], -1)

    def rmsnorm(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """fp32 math, fp16 result (``RMSnorm_d.cu:22-87``)."""
        xf = x.float()
        r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.cfg.rms_norm_eps)
        return (xf * r * w).half()

    def add_rmsnorm(self, x: torch.Tensor, w: torch.Tensor, delta: Optional[torch.Tensor] = None):
        """(x + delta, rmsnorm(x + delta)): one kernel on the fp8 path, the fp32
        torch operations of ``rmsnorm`` otherwise."""
        if self.linear_kind == "fp8":
            return norm.add_rmsnorm(x.contiguous(), w, self.cfg.rms_norm_eps,
                                    None if delta is None else delta.contiguous())
        if delta is not None:
            x = x + delta
        return x, self.rmsnorm(x, w)

    def rope_tables(self, positions: torch.Tensor):
        """cos/sin [S, D] of rotate-half RoPE: fp32(position) * inv_freq for both
        halves of the head (one multiply, the same values as concatenating the
        half-width product with itself)."""
        emb = positions[:, None] * self._inv_freq2[None, :]
        return emb.cos(), emb.sin()

    @staticmethod
    def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        """Rotate-half RoPE on [B, H, S, D] in fp32 (``RoPe_d.cu:12-68``)."""
        xf = x.float()
        half = xf.shape[-1] // 2
        rot = torch.cat([-xf[..., half:], xf[..., :half]], dim=-1)
        return (xf * cos + rot * sin).half()

    @staticmethod
    def swiglu(gu: torch.Tensor, inter: int) -> torch.Tensor:
        """silu(gate) * up with fp32 math (``SwiGLU_d.cu:12-26``)."""
        g = gu[..., :inter].float()
        u = gu[..., inter:].float()
        return (g * torch.sigmoid(g) * u).half()

    # ------------------------------------------------------------------ layers
    def _layer(self, li: int, x: torch.Tensor, delta: Optional[torch.Tensor], cache: KVCache,
               b0: int, cos, sin, pos: Optional[torch.Tensor], start: int):
        """One decoder layer.  The previous layer's MLP output `delta` is added to
        the residual stream `x` inside this layer's first RMSNorm; returns the
        new stream and this layer's MLP output, still to be added."""
        cfg = self.cfg
        L = self.layers[li]
        B, S, H = x.shape
        hd, nh, nkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
        scale = hd ** -0.5
        if (pos is not None and S == 1 and self.linear_kind == "fp8" and B <= 64
                and self.decode_planes):
            return self._decode_layer(li, x, delta, cache, b0, cos, sin, pos)
        x, h = self.add_rmsnorm(x, L["in_norm"], delta)
        if pos is None and self.linear_kind == "fp8" and hd in (64, 128):
            # prefill chunk: the q/k/v projection, RoPE of q and k and the cache
            # write (one GEMM with them in its epilogue where the prefill kernel
            # takes the shape, else the GEMM and one RoPE + cache kernel); q, k,
            # v come back token-major (attention strides independent of the
            # cache capacity)
            p = L["qkv"]
            kc, vc = cache.k[li, b0:b0 + B], cache.v[li, b0:b0 + B]
            if self.fused_qkv_rope:
                q, k, v = attention.qkv_rope_kv(h, p.wq, p.scales, p.bias, kc, vc, cos, sin,
                                                start, nh, nkv, hd, kv_out=True)
            else:
                q, k, v = attention.prefill_rope_kv(self.linear(h, p), kc, vc, cos, sin, start,
                                                    nh, nkv, hd, kv_out=True)
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                               v.transpose(1, 2), is_causal=True, scale=scale,
                                               enable_gqa=True)
            o = o.transpose(1, 2).reshape(B, S, nh * hd)
            return self._mlp_block(x, self.linear(o, L["o"]), L)
        qkv = self.linear(h, L["qkv"])
        if pos is not None and S == 1 and self.linear_kind == "fp8":
            # one decode step: RoPE, the cache write and the attention in one kernel
            o = attention.decode_attention(qkv.reshape(B, -1), cache.k[li, b0:b0 + B],
                                           cache.v[li, b0:b0 + B], cos, sin, pos, nh, nkv, hd,
                                           scale)
            return self._mlp_block(x, self.linear(o.reshape(B, S, nh * hd), L["o"]), L)
        q = qkv[..., : nh * hd].reshape(B, S, nh, hd).transpose(1, 2)
        k = qkv[..., nh * hd: (nh + nkv) * hd].reshape(B, S, nkv, hd).transpose(1, 2)
        v = qkv[..., (nh + nkv) * hd:].reshape(B, S, nkv, hd).transpose(1, 2)
        q = self.apply_rope(q, cos, sin)
        k = self.apply_rope(k, cos, sin)
        kc = cache.k[li, b0:b0 + B]
        vc = cache.v[li, b0:b0 + B]
        if pos is None:  # prefill from position `start` (0): causal attention over the chunk
            kc[:, :, start:start + S] = k
            vc[:, :, start:start + S] = v
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=scale,
                                               enable_gqa=True)
        else:            # one decode step at device position `pos`, static cache length
            kc.index_copy_(2, pos, k)
            vc.index_copy_(2, pos, v)
            mask = (torch.arange(cache.capacity, device=x.device) <= pos)[None, None, None, :]
            o = F.scaled_dot_product_attention(q, kc, vc, attn_mask=mask, scale=scale,
                                               enable_gqa=True)
        o = o.transpose(1, 2).reshape(B, S, nh * hd)
        return self._mlp_block(x, self.linear(o, L["o"]), L)

    def _decode_layer(self, li: int, x: torch.Tensor, delta: Optional[torch.Tensor],
                      cache: KVCache, b0: int, cos, sin, pos: torch.Tensor):
        """A decode-step layer (B <= 64 tokens) with the fewest kernels: each RMSNorm
        also splits its output into the operand form of the GEMM that follows
        (no split pre-pass there), then RoPE + cache write + attention in one
        kernel, and gate/up with the SwiGLU epilogue."""
        cfg = self.cfg
        L = self.layers[li]
        B, S, H = x.shape
        hd, nh, nkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
        eps = cfg.rms_norm_eps
        # per stream: decode chains on different streams may run at the same time
        key = (B, H, torch.cuda.current_stream(x.device).cuda_stream)
        bufs = self._split_bufs.setdefault(key, [None, None, None])
        x, bufs[0] = norm.add_rmsnorm_split(x.contiguous(), L["in_norm"], eps, delta, bufs[0])
        p = L["qkv"]
        qkv = gemm_fp8.f8_forward_planes(bufs[0], p.wq, p.scales, p.bias)
        if hd == 64 and nkv <= 8:  # attention emits the o projection's operand directly
            # the position and the cache rows before it come from earlier steps
            bufs[2], _ = attention.decode_attention_split(
                qkv, cache.k[li, b0:b0 + B], cache.v[li, b0:b0 + B], cos, sin, pos, nh, nkv, hd,
                hd ** -0.5, bufs[2], kv_ready=True)
            p = L["o"]
            attn = gemm_fp8.f8_forward_planes(bufs[2], p.wq, p.scales, p.bias).reshape(x.shape)
        else:
            o = attention.decode_attention(qkv, cache.k[li, b0:b0 + B], cache.v[li, b0:b0 + B],
                                           cos, sin, pos, nh, nkv, hd, hd ** -0.5)
            attn = self.linear(o.reshape(B, S, nh * hd), L["o"])
        x, bufs[1] = norm.add_rmsnorm_split(x, L["post_norm"], eps, attn.contiguous(), bufs[1])
        wq, sc, b = L["gate_up"].gate_up_interleaved()
        z = gemm_fp8.f8_forward_planes(bufs[1], wq, sc, b, swiglu=True)
        return x, self.linear(z.reshape(B, S, -1), L["down"])

    def _mlp_block(self, x: torch.Tensor, attn: torch.Tensor, L: dict):
        """+attention residual -> RMSNorm -> gate/up -> SwiGLU -> down; returns the
        stream and the down projection (the residual add happens in the next norm)."""
        x, h = self.add_rmsnorm(x, L["post_norm"], attn)
        if self.linear_kind == "fp8":   # gate/up GEMM with the SwiGLU epilogue
            z = gemm_fp8.f8_forward_swiglu(h, *L["gate_up"].gate_up_interleaved())
        else:
            z = self.swiglu(self.linear(h, L["gate_up"]), self.cfg.intermediate_size)
        return x, self.linear(z, L["down"])

    def hidden(self, ids: torch.Tensor, cache: KVCache, b0: int = 0, start: int = 0,
               pos: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Final-normed hidden states for ids [B, S] (prefill) or [B, 1] at `pos`."""
        x = F.embedding(ids, self.embed)
        if pos is None:
            cos, sin = self.rope_tables(torch.arange(start, start + ids.shape[1], device=ids.device))
        else:
            cos, sin = self.rope_tables(pos)
        delta = None
        for li in range(self.cfg.num_hidden_layers):
            x, delta = self._layer(li, x, delta, cache, b0, cos, sin, pos, start)
        return self.add_rmsnorm(x, self.final_norm, delta)[1]

    def decode_hidden(self, tok: torch.Tensor, cache: KVCache, pos: torch.Tensor) -> torch.Tensor:
        """Final-normed hidden state [B, H] of one decode step of tok [B, 1] at
        `pos`.  With `decode_chains` > 1 and at least 32 sequences per slice, the
        batch is cut into that many slices, each run on its own stream; the
        sequences are independent, so only the streams' joins order them."""
        B = tok.shape[0]
        n = self.decode_chains
        if n <= 1 or B < 32 * n or B % n:
            return self.hidden(tok, cache, 0, 0, pos)[:, -1, :]
        per = B // n
        main = torch.cuda.current_stream(self.device)
        while len(self._chain_streams) < n:
            self._chain_streams.append(torch.cuda.Stream(self.device))
        streams = self._chain_streams[:n]
        outs = []
        for i, s in enumerate(streams):
            s.wait_stream(main)
            with torch.cuda.stream(s):
                outs.append(self.hidden(tok[i * per:(i + 1) * per], cache, i * per, 0,
                                        pos)[:, -1, :])
        for s in streams:
            main.wait_stream(s)
        return torch.cat(outs)

    def greedy(self, h: torch.Tensor) -> torch.Tensor:
        """Greedy token of each row of h [M, H] (fused lm_head argmax, or the oracle)."""
        if self.linear_kind == "fp8":
            ids, _ = lmh.lm_head_argmax(h, self.lm_head.wq, self.lm_head.scales)
            return ids
        return self.logits(h).float().argmax(dim=-1)

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        if self.linear_kind == "fp8":
            return gemm_fp8.f8_forward(h, self.lm_head.wq, self.lm_head.scales)
        acc = torch.float64 if self.linear_kind == "oracle64" else torch.float32
        return (h.to(acc) @ self.lm_head.dequantized().to(acc).T).half()

    # ------------------------------------------------------------------ reference-style API
    def forward(self, input_ids: torch.Tensor, cache: Optional[KVCache] = None, start: int = 0):
        """Logits for every position, as the reference ``Engine.forward`` (``engine.py:334-339``)."""
        if cache is None:
            cache = self.new_cache(input_ids.shape[0], start + input_ids.shape[1])
        h = self.hidden(input_ids, cache, 0, start)
        return self.logits(h), cache

    # ------------------------------------------------------------------ generation
    @torch.no_grad()
    def generate(self, prompts: torch.Tensor, max_new_tokens: int, prefill_chunk: int = 64,
                 use_graph: bool = True, teacher: Optional[torch.Tensor] = None,
                 stats: Optional[dict] = None) -> torch.Tensor:
        """Greedy generation for a batch of equal-length prompts [B, S] -> tokens [B, max_new].

        Prefill runs in chunks of `prefill_chunk` sequences (M = chunk * S tokens per
        GEMM; the eager prefill launches ~300 kernels per chunk, so few large
        chunks keep the host ahead of the GPU); decode runs all B sequences at
        once (M = B), one captured step per token with its bookkeeping on the
        device.  With `teacher` [B, max_new]
        the next input at each step is the teacher's token instead of the generated
        one (used to compare against the oracle step by step); the returned tokens
        are still this engine's greedy picks.  A `stats` dict receives
        "decode_events": CUDA events recorded around the decode steps (after
        the step's capture) and "decode_steps", their number.
        """
        B, S = prompts.shape
        cap = S + max_new_tokens
        cache = self.new_cache(B, cap)
        out = torch.empty(B, max_new_tokens, dtype=torch.int64, device=self.device)
        for b0 in range(0, B, prefill_chunk):
            chunk = prompts[b0:b0 + prefill_chunk]
            h = self.hidden(chunk, cache, b0, 0)
            out[b0:b0 + chunk.shape[0], 0] = self.greedy(h[:, -1, :])
        if max_new_tokens == 1:
            return out
        # One decode step, entirely on the device: t counts the tokens already
        # emitted (t = 0 .. max_new - 2); the step reads token t (the previous
        # pick, or the teacher's), runs at position S + t and writes its pick
        # to out[:, t + 1].  The host only replays the captured step.
        src = out if teacher is None else teacher
        t = torch.zeros(1, dtype=torch.int64, device=self.device)
        tok = torch.empty(B, 1, dtype=torch.int64, device=self.device)
        pos = torch.empty(1, dtype=torch.int64, device=self.device)

        def step():
            tok.copy_(src.index_select(1, t))
            torch.add(t, S, out=pos)
            nxt = self.greedy(self.decode_hidden(tok, cache, pos))
            out.index_copy_(1, t + 1, nxt[:, None])
            t.add_(1)

        graph = None
        if use_graph and self.linear_kind == "fp8":
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                step()  # warm-up outside capture (kernel attributes, workspaces)
            torch.cuda.current_stream(self.device).wait_stream(s)
            t.zero_()   # the warm-up step is redone by the first replay (same cache row)
            # captured on a side stream without the device-wide synchronisation
            # of the torch.cuda.graph context: the host records the step while
            # the GPU still runs the prefill and the warm-up
            graph = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream(self.device)
            with torch.cuda.stream(cap):
                graph.capture_begin()
                try:
                    step()
                finally:
                    graph.capture_end()
        if stats is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        for _ in range(1, max_new_tokens):
            if graph is not None:
                graph.replay()
            else:
                step()
        if stats is not None:
            ev[1].record()
            stats["decode_events"] = ev
            stats["decode_steps"] = max_new_tokens - 1
        if graph is not None:
            del graph
        return out
