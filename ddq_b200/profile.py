"""Micro-benchmark of one W8A16 GEMM shape (also the target of ncu captures).

Runs ``--iters`` launches of ``ddq_w8a16_gemm`` (or the fused lm_head with
``--lm-head``) for one (M, N, K), rotating through enough distinct weight
copies that each launch reads its weight from HBM (the copies total more than
twice the 126 MB L2, unless ``--copies`` says otherwise).  Each launch is
bracketed by CUDA events on the launch stream; the host first parks the GPU
on a sleep kernel so that every launch is queued before the first one runs
and the events time the GPU alone.  Prints one JSON line.

    python -m ddq_b200.profile --m 64 --n 9728 --k 896 --iters 50

With ``--attention`` it times the decode-step attention kernel instead
(``ddq_decode_attention`` at the engine's shapes, rotating KV-cache copies):

    python -m ddq_b200.profile --attention --batch 64 --pos 640 --iters 20
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from . import _lib, attention, gemm_fp8, lm_head


def algorithmic_bytes(M, N, K, bias=False, lm=False):
    out = 8 * M if lm else 2 * M * N
    return N * K + 4 * N + (4 * N if bias else 0) + 2 * M * K + out


def attention_bytes(B, Hq, Hkv, D, pos):
    """K and V rows 0..pos read, q/k/v in, o out, the new K/V row written."""
    return (2 * B * Hkv * (pos + 1) * D * 2 + B * (Hq + 2 * Hkv) * D * 2 + B * Hq * D * 2
            + 2 * B * Hkv * D * 2)


def run_attention(a, dev):
    B, Hq, Hkv, D, cap, pos = a.batch, a.heads, a.kv_heads, a.head_dim, a.cap, a.pos
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    per = 2 * B * Hkv * cap * D * 2
    copies = a.copies or max(2, math.ceil(2.2 * l2 / per))
    g = torch.Generator(device=dev).manual_seed(0)
    caches = [(torch.randn(B, Hkv, cap, D, generator=g, device=dev).half(),
               torch.randn(B, Hkv, cap, D, generator=g, device=dev).half()) for _ in range(copies)]
    qkv = torch.randn(B, (Hq + 2 * Hkv) * D, generator=g, device=dev).half()
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.float32, device=dev) / D))
    f = float(pos) * inv
    cos, sin = torch.cat([f, f]).cos(), torch.cat([f, f]).sin()
    p = torch.tensor([pos], dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)

    def launch(i):
        kc, vc = caches[i % copies]
        attention.decode_attention(qkv, kc, vc, cos, sin, p, Hq, Hkv, D, D ** -0.5)

    for i in range(a.warmup):
        launch(i)
    torch.cuda.synchronize(dev)
    torch.cuda._sleep(int(2e8))  # every launch below is queued before the first runs
    if a.chain:
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for i in range(a.iters):
            launch(a.warmup + i)
        c1.record(stream)
        torch.cuda.synchronize(dev)
        t = [c0.elapsed_time(c1) * 1e3 / a.iters]
    else:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(a.iters)]
        for i, (e0, e1) in enumerate(evs):
            e0.record(stream)
            launch(a.warmup + i)
            e1.record(stream)
        torch.cuda.synchronize(dev)
        t = sorted(e0.elapsed_time(e1) * 1e3 for e0, e1 in evs)
    med = t[len(t) // 2]
    nb = attention_bytes(B, Hq, Hkv, D, pos)
    print(json.dumps({"kernel": "decode_attention", "B": B, "Hq": Hq, "Hkv": Hkv, "D": D,
                      "pos": pos, "cap": cap, "copies": copies,
                      "mode": "chain" if a.chain else "events", "us_median": round(med, 3),
                      "bytes": nb, "gbs_median": round(nb / (med * 1e-6) / 1e9, 1)}))


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=64)
    ap.add_argument("--n", type=int, default=9728)
    ap.add_argument("--k", type=int, default=896)
    ap.add_argument("--bias", action="store_true")
    ap.add_argument("--lm-head", action="store_true")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--copies", type=int, default=0, help="distinct weight copies (0: > 2x L2)")
    ap.add_argument("--chain", action="store_true",
                    help="time --iters launches back to back (no events between) and report per launch")
    ap.add_argument("--torch-fp16", action="store_true",
                    help="time torch.matmul on an fp16 weight (cuBLAS, the reference engine's path)")
    ap.add_argument("--empty", action="store_true",
                    help="time a trivial one-thread kernel instead (launch + event floor)")
    ap.add_argument("--trace", action="store_true",
                    help="also run one launch with the per-CTA phase trace and summarise it "
                         "(with --chain: the chain's last launch, traced in place)")
    ap.add_argument("--qkv-rope", action="store_true",
                    help="time the q/k/v GEMM with RoPE and the KV-cache write in its epilogue "
                         "(ddq_w8a16_gemm_qkv_rope_kv): --batch sequences of --m / --batch tokens, "
                         "--heads / --kv-heads / --head-dim, N from them, fp32 bias")
    ap.add_argument("--attention", action="store_true",
                    help="time the decode-step attention kernel instead of a GEMM")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--pos", type=int, default=640)
    ap.add_argument("--cap", type=int, default=768)
    ap.add_argument("--heads", type=int, default=14)
    ap.add_argument("--kv-heads", type=int, default=2)
    ap.add_argument("--head-dim", type=int, default=64)
    a = ap.parse_args(argv)
    dev = torch.device("cuda", torch.cuda.current_device())
    if a.attention:
        run_attention(a, dev)
        return
    L = _lib.load()
    M, N, K = a.m, a.n, a.k
    if a.qkv_rope:
        if M % a.batch:
            raise SystemExit("--qkv-rope: --m must be a multiple of --batch")
        N = (a.heads + 2 * a.kv_heads) * a.head_dim
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    copies = a.copies or max(2, math.ceil(2.2 * l2 / (N * K)))
    copies = min(copies, max(2, int(4e9 // (N * K))))
    g = torch.Generator(device=dev).manual_seed(0)
    ws_list = []
    for _ in range(copies):
        wq, s = gemm_fp8.quantize(torch.randn(N, K, generator=g, device=dev) * 0.02)
        ws_list.append((wq, s))
    x = torch.randn(M, K, generator=g, device=dev).half()
    b = torch.randn(N, generator=g, device=dev) * 0.02 if a.bias else None
    y = torch.empty(M, N, dtype=torch.float16, device=dev)
    packed = torch.empty(M, dtype=torch.int64, device=dev)
    nws = (L.ddq_lm_head_argmax_workspace_size(M, N, K) if a.lm_head
           else L.ddq_w8a16_gemm_workspace_size(M, N, K))
    if a.lm_head:
        ws = lm_head.lm_workspace(dev, nws) if nws else None
    else:
        ws = gemm_fp8.workspace(dev, nws) if nws else None
    stream = torch.cuda.current_stream(dev)

    ids = torch.empty(M, dtype=torch.int64, device=dev)

    if a.qkv_rope:  # one sequence batch: caches of exactly S positions, written at 0
        S = M // a.batch
        kc = torch.zeros(a.batch, a.kv_heads, S, a.head_dim, dtype=torch.float16, device=dev)
        vc = torch.zeros_like(kc)
        cs = torch.rand(S, a.head_dim, generator=g, device=dev)
        sn = torch.rand(S, a.head_dim, generator=g, device=dev)
        q_out = torch.empty(M, a.heads * a.head_dim, dtype=torch.float16, device=dev)
        kv_out = torch.empty(2, M, a.kv_heads * a.head_dim, dtype=torch.float16, device=dev)
        b = torch.randn(N, generator=g, device=dev) * 0.02

    w16 = None
    if a.torch_fp16:
        w16 = [torch.randn(N, K, generator=g, device=dev).half() * 0.02 for _ in range(copies)]

    def launch(i):
        wq, s = ws_list[i % copies]
        if a.torch_fp16:
            torch.matmul(x, w16[i % copies].t(), out=y)
            return
        if a.qkv_rope:
            st = L.ddq_w8a16_gemm_qkv_rope_kv(
                x.data_ptr(), wq.data_ptr(), s.data_ptr(), b.data_ptr(), _lib.DTYPE_F32,
                a.batch, M // a.batch, K, a.heads, a.kv_heads, a.head_dim, kc.data_ptr(),
                vc.data_ptr(), kc.stride(0), kc.shape[2], cs.data_ptr(), sn.data_ptr(), 0,
                q_out.data_ptr(), kv_out[0].data_ptr(), kv_out[1].data_ptr(),
                ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
                stream.cuda_stream)
        elif a.empty:  # a trivial kernel of this library: the launch + event floor
            st = L.ddq_unpack_argmax(packed.data_ptr(), 1, ids.data_ptr(), stream.cuda_stream)
        elif a.lm_head:
            st = L.ddq_lm_head_argmax(x.data_ptr(), wq.data_ptr(), s.data_ptr(), M, N, K, 0,
                                      packed.data_ptr(), None,
                                      ws.data_ptr() if ws is not None else None,
                                      ws.numel() if ws is not None else 0, stream.cuda_stream)
        else:
            st = L.ddq_w8a16_gemm(x.data_ptr(), wq.data_ptr(), s.data_ptr(),
                                  b.data_ptr() if b is not None else None,
                                  _lib.DTYPE_F32 if b is not None else _lib.DTYPE_NONE,
                                  y.data_ptr(), M, N, K,
                                  ws.data_ptr() if ws is not None else None,
                                  ws.numel() if ws is not None else 0, stream.cuda_stream)
        _lib.check(st, "profile launch")

    for i in range(a.warmup):
        launch(i)
    torch.cuda.synchronize(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(a.iters)]
    torch.cuda._sleep(int(2e8))  # ~0.1 s of GPU spin so every launch below is queued first
    if a.chain:
        c0, c1 = evs[0]
        c0.record(stream)
        for i in range(a.iters):
            if a.trace and i == a.iters - 1:
                L.ddq_set_debug(2, 0)   # trace the last launch of the chain, in place
            launch(a.warmup + i)
        L.ddq_set_debug(0, 0)
        c1.record(stream)
        torch.cuda.synchronize(dev)
        per = c0.elapsed_time(c1) * 1e3 / a.iters
        evs = [(c0, c1)]
    else:
        for i, (e0, e1) in enumerate(evs):
            e0.record(stream)
            launch(a.warmup + i)
            e1.record(stream)
    torch.cuda.synchronize(dev)
    trace = None
    if a.trace:
        import ctypes
        import numpy as np
        if not a.chain:
            L.ddq_set_debug(2, 0)
            launch(a.warmup + a.iters)       # cold weights (next copy in the rotation)
            torch.cuda.synchronize(dev)
            L.ddq_set_debug(0, 0)
        buf = np.zeros((2048, 16), dtype=np.uint64)  # 16 stamp slots per CTA
        _lib.check(L.ddq_read_trace(buf.ctypes.data_as(ctypes.c_void_p), 2048,
                                    stream.cuda_stream), "read trace")
        used = buf[(buf[:, 0] > 0) & (buf[:, 7] > 0)].astype(np.int64)
        if len(used):
            t0 = used[:, 0].min()
            rel = (used - t0) / 1e3
            names = ["entry", "setup", "w_issued", "w_landed", "mma_done", "acc_ready",
                     "epi_done", "exit",
                     # kernels with more phases (rt.cu): half-way and last
                     # activation atom ready, converters done, last activation
                     # load issued, accumulator complete
                     "x_half", "x_last", "conv_done", "x_issued_last", "acc_full",
                     "epi_chunk0", "epi_stored", "producer_drained"]
            trace = {"ctas": int(len(used)), "span_us": round(float(rel[:, 7].max()), 3)}
            for j, nm in enumerate(names):
                col = rel[:, j][used[:, j] > 0]
                if len(col):
                    trace[nm] = [round(float(np.min(col)), 3), round(float(np.median(col)), 3),
                                 round(float(col.max()), 3)]
            w = rel[:, 3][used[:, 3] > 0]
            if len(w):   # from the earliest grid-dependency resolution to the last exit
                trace["after_dependency_us"] = round(float(rel[:, 7].max() - w.min()), 3)
    t = sorted(e0.elapsed_time(e1) * 1e3 for e0, e1 in evs)
    if a.chain:
        t = [per]
    med = t[len(t) // 2]
    avg = sum(t) / len(t)
    nb = algorithmic_bytes(M, N, K, a.bias, a.lm_head)
    if a.torch_fp16:
        nb = 2 * N * K + 2 * M * K + 2 * M * N
    print(json.dumps({"M": M, "N": N, "K": K, "lm_head": a.lm_head, "copies": copies,
                      "mode": ("torch_fp16" if a.torch_fp16 else "ddq") + ("_chain" if a.chain else ""),
                      "us_median": round(med, 3), "us_avg": round(avg, 3),
                      "us_min": round(t[0], 3), "bytes": nb,
                      "gbs_median": round(nb / (med * 1e-6) / 1e9, 1),
                      "tflops_median": round(2 * M * N * K / (med * 1e-6) / 1e12, 2),
                      "workspace": nws, "trace_us_median_max": trace}))


if __name__ == "__main__":
    main()
