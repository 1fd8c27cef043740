"""Benchmark of the W8A16 projection-GEMM path (BASELINE.json metric).

Workload of the headline (`value`): BASELINE config 2 - the decode projection
set of a Qwen2.5-0.5B-shaped decoder, 24 layers x {q 896->896 +bias,
k 896->128 +bias, v 896->128 +bias, o 896->896, gate/up 896->9728,
down 4864->896}, e4m3 weights with fp32 per-channel scales drawn from
N(0, 0.02), fp16 activations from N(0, 1), fp32 biases, run at
M in {1, 8, 32, 64}.  q, k and v run as one 896->1152 projection (their
weights stacked at load time, as the engine does; the weight bytes are the
same), so a layer is 4 GEMMs ordered on one stream (each starts its
activation reads only after the previous one has completed, as dependent
GEMMs do).  One pass = the 24-layer set at each of the four M (384 GEMMs);
one step = SETS_PER_STEP passes, so that the timed region lasts long enough
for the clock sampler.  `value` is algorithmic bytes (weights + scales +
bias + activations in + outputs) per second over all ranks, in TB/s, with
every input resident in HBM; the 357.8 MB of weights per pass exceed the
126 MB L2, so every pass reads them from HBM.  The pass is captured once in a
CUDA graph and replayed.

`e2e` is the same metric through the public API (ddq_b200.gemm_fp8.f8_forward,
one call per GEMM) with each step's activations copied in from pinned host
memory and every output copied back inside the timed region, the calls and
copies replayed as a CUDA graph; `e2e.eager` makes the same calls and copies
eagerly from Python.

`--impl reference` times the reference semantics on the host cores (the CPU
oracle in PyTorch: per-call dequantisation + fp32 matmul), which is the
reference's CPU path for this metric; where a GPU and the reference's own
CUDA operators (built from its sources into oracle/_ref) are present, that
line also carries those kernels' times on the same shapes.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "W8A16 GEMM HBM TB/s (M<=64) & TFLOP/s (M=4096); decode tok/s at 1/8 GPU"
LAYERS = 24
HIDDEN, INTER = 896, 4864
# (name, K, N, has_bias) - engine.py:185-187, 206-209 with q/k/v and gate/up fused
PROJS = [("qkv", 896, 1152, True), ("o", 896, 896, False), ("gate_up", 896, 9728, False),
         ("down", 4864, 896, False)]
GATE_UP = 2  # index of gate/up in PROJS
DECODE_M = (1, 8, 32, 64)
SETS_PER_STEP = 32  # passes of the 384-GEMM set per timed step
# ncu summaries whose traffic line belongs to the roofline kernel (the one the
# library dispatches for gate/up at 64 tokens: one launch = the tensor-core
# resident-slice kernel, two = the split pre-pass + e4m3 decode kernel)
ROOFLINE_PROFILES = {1: os.path.join(REPO, "profiles", "w8a16_rt_gateup_m64.md"),
                     2: os.path.join(REPO, "profiles", "w8a16_dec_gateup_m64.md")}
ROOFLINE_KERNELS = {1: "w8a16_rt_kernel (gate/up 896->9728, M=64)",
                    2: "w8a16_dec_kernel + xsplit_kernel (gate/up 896->9728, M=64)"}


def proj_bytes(M, K, N, bias):
    """Algorithmic bytes of one GEMM: wq + scales + fp32 bias + x in + y out."""
    return N * K + 4 * N + (4 * N if bias else 0) + 2 * M * K + 2 * M * N


def step_bytes():
    return sum(LAYERS * proj_bytes(M, K, N, b) for M in DECODE_M for _, K, N, b in PROJS)


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            t0 = time.time()  # the timed region starts only once sampling has begun
            while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.01)
            self._n0 = len(self.lines)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[getattr(self, "_n0", 0):]:
            p = [t.strip() for t in ln.split(",")]
            if len(p) < 8:
                continue
            try:
                sm.append(float(p[0]))
                mx = float(p[1])
            except ValueError:
                continue
            for nm, v in zip(names, p[4:8]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- workload
class DecodeWorkload:
    def __init__(self, device, seed=0):
        from ddq_b200 import gemm_fp8
        self.device = device
        g = torch.Generator(device=device).manual_seed(seed)
        self.layers = []
        for _ in range(LAYERS):
            layer = {}
            for name, K, N, has_bias in PROJS:
                w = torch.randn(N, K, generator=g, device=device) * 0.02
                wq, s = gemm_fp8.quantize(w)
                b = (torch.randn(N, generator=g, device=device) * 0.02) if has_bias else None
                layer[name] = (wq, s, b)
                del w
            self.layers.append(layer)
        self.x = {M: {name: torch.randn(M, K, generator=g, device=device).half()
                      for name, K, _, _ in PROJS} for M in DECODE_M}
        self.y = {M: [{name: torch.empty(M, N, dtype=torch.float16, device=device)
                       for name, _, N, _ in PROJS} for _ in range(LAYERS)] for M in DECODE_M}
        torch.cuda.synchronize(device)

    def launch_list(self):
        """Raw C-ABI argument tuples for every GEMM of one step (no allocation)."""
        from ddq_b200 import _lib
        L = _lib.load()
        # one workspace sized for the largest shape, allocated before any pointer is
        # taken; the step's own (it is recorded into a CUDA graph, and the library
        # never expands prefill weights early into a workspace a graph has used)
        need = max(L.ddq_w8a16_gemm_workspace_size(M, N, K) for M in DECODE_M
                   for _, K, N, _ in PROJS)
        ws_all = torch.empty(need, dtype=torch.uint8, device=self.device) if need else None
        self.ws = ws_all
        out = []
        for M in DECODE_M:
            for li, layer in enumerate(self.layers):
                for name, K, N, has_bias in PROJS:
                    wq, s, b = layer[name]
                    nws = L.ddq_w8a16_gemm_workspace_size(M, N, K)
                    ws = ws_all if nws else None
                    out.append((self.x[M][name].data_ptr(), wq.data_ptr(), s.data_ptr(),
                                b.data_ptr() if b is not None else None,
                                _lib.DTYPE_F32 if b is not None else _lib.DTYPE_NONE,
                                self.y[M][li][name].data_ptr(), M, N, K,
                                ws.data_ptr() if ws is not None else None,
                                ws.numel() if ws is not None else 0))
        return out


def run_ours(args, rank, world, device):
    from ddq_b200 import _lib, gemm_fp8
    L = _lib.load()
    wl = DecodeWorkload(device, seed=1234 + rank)
    calls = wl.launch_list()
    gemm = L.ddq_w8a16_gemm

    def step(stream_ptr):
        for c in calls:
            st = gemm(*c, stream_ptr)
            if st:
                raise RuntimeError(f"ddq_w8a16_gemm failed: {_lib.status_string(st)}")

    # capture one step in a CUDA graph on a side stream
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        step(side.cuda_stream)          # eager warm-up (module load, attributes)
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        step(side.cuda_stream)
    torch.cuda.synchronize(device)

    for _ in range(args.warmup * SETS_PER_STEP):
        graph.replay()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clk:
        ev0.record()
        for _ in range(args.steps * SETS_PER_STEP):
            graph.replay()
        ev1.record()
        torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    ms = ev0.elapsed_time(ev1)
    ms_max = reduce_max(ms, world, device)
    sbytes = step_bytes() * SETS_PER_STEP
    value = sbytes * args.steps * world / (ms_max * 1e-3) / 1e12

    # ---- roofline of the dominant kernel: gate/up (58% of the bytes).  Its
    # average launch duration is taken over a back-to-back chain of the 24
    # layers' gate/up calls (cold weights: 24 distinct 8.7 MB matrices in turn),
    # as the calls run inside the step, between two CUDA events on the launch
    # stream; also, per launch with events around each call (launch gaps
    # included), for reference.
    peaks = load_peaks()
    per_m = {}
    dom = None
    stream = torch.cuda.current_stream(device)
    for M in DECODE_M:
        sel = [c for c in calls if c[6] == M]
        gu = [sel[li * len(PROJS) + GATE_UP] for li in range(LAYERS)]
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(LAYERS)]
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(int(2e8))  # park the GPU so all launches below queue before any runs
        for c in gu:                  # warm-up pass
            gemm(*c, stream.cuda_stream)
        c0.record(stream)
        for rep in range(4):
            for c in gu:
                gemm(*c, stream.cuda_stream)
        c1.record(stream)
        for li, c in enumerate(gu):
            e0, e1 = evs[li]
            e0.record(stream)
            gemm(*c, stream.cuda_stream)
            e1.record(stream)
        torch.cuda.synchronize(device)
        chain = c0.elapsed_time(c1) / (4 * LAYERS)
        single = sum(a.elapsed_time(b) for a, b in evs) / LAYERS
        nb = proj_bytes(M, 896, 9728, False)
        per_m[M] = {"gate_up_us": round(chain * 1e3, 3), "gate_up_gbs": round(nb / (chain * 1e-3) / 1e9, 1),
                    "gate_up_us_single_launch": round(single * 1e3, 3)}
        if M == 64:
            dom = (nb, chain)

    nb, avg = dom
    achieved = nb / (avg * 1e-3) / 1e9
    nk = L.ddq_w8a16_gemm_kernel_count(64, PROJS[GATE_UP][2], PROJS[GATE_UP][1])
    traffic, traffic_src = profile_traffic(ROOFLINE_PROFILES.get(nk, ROOFLINE_PROFILES[2]))
    roofline = {"kernel": ROOFLINE_KERNELS.get(nk, ROOFLINE_KERNELS[2]),
                "bound": "hbm",
                "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                "traffic": traffic, "traffic_source": traffic_src, "bytes_per_launch": nb,
                "timing": "average over a back-to-back chain of 96 calls, CUDA events on the launch stream"}

    # ---- e2e through the public API, host buffers, copies inside the timed region
    e2e = run_e2e(args, wl, device, world)

    # ---- the other parts of the BASELINE metric: prefill TFLOP/s (config 3),
    # the fused lm_head (config 4) and greedy generation tok/s (config 5)
    n_gemms, n_launches = len(calls), launches_per_step(calls)
    del wl, calls, graph
    torch.cuda.empty_cache()
    prefill = None if args.skip_extra else run_prefill(args, device, world, peaks)
    lmhead = None if args.skip_extra else run_lm_head(args, device, rank, world, peaks)
    config1 = None if args.skip_extra else run_config1(args, device, world, peaks)
    generation = None if args.skip_extra else run_generation(args, device, rank, world, peaks)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_seconds)

    line = {
        "metric": METRIC, "value": round(value, 4), "unit": "TB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
        "ms_per_pass": round(ms_max / (args.steps * SETS_PER_STEP), 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e4m3xf16->f32",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations; no dataset)",
        "config": {"workload": "config2: 24-layer decode projection set at M=1,8,32,64",
                   "layers": LAYERS, "M": list(DECODE_M),
                   "shapes": [f"{n} {k}->{nn}" + ("+bias" if b else "") for n, k, nn, b in PROJS],
                   "qkv": "q 896->896, k 896->128, v 896->128 (+bias) stacked into one GEMM",
                   "passes_per_step": SETS_PER_STEP, "bytes_per_step": sbytes,
                   "gemms_per_pass": n_gemms,
                   "l2": "inputs larger than L2 (357.8 MB of weights per M pass > 126 MB)",
                   "timing": "CUDA graph of one pass, replayed SETS_PER_STEP times per step; "
                             "CUDA events; max over ranks",
                   "parallelism": f"replicas x{world}"},
        "per_m_gate_up": per_m,
        "prefill": prefill,
        "config1": config1,
        "lm_head": lmhead,
        "generation": generation,
        "roofline": roofline,
        "e2e": e2e,
        "gpu_launches": n_launches * args.steps * SETS_PER_STEP,
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
    }
    return line


def run_prefill(args, device, world, peaks):
    """Config 3: the 24-layer projection set at M = 4096 tokens (8 x 512), TFLOP/s."""
    from ddq_b200 import _lib, gemm_fp8
    L = _lib.load()
    M = 4096
    g = torch.Generator(device=device).manual_seed(77)
    mats = []
    for _ in range(LAYERS):
        for name, K, N, has_bias in PROJS:
            wq, sc = gemm_fp8.quantize(torch.randn(N, K, generator=g, device=device) * 0.02)
            b = torch.randn(N, generator=g, device=device) * 0.02 if has_bias else None
            mats.append((wq, sc, b, K, N))
    xs = {K: torch.randn(M, K, generator=g, device=device).half() for K in (HIDDEN, INTER)}
    ys = {N: torch.empty(M, N, dtype=torch.float16, device=device) for _, _, N, _ in PROJS}
    flops = 2 * M * sum(K * N for _, K, N, _ in PROJS) * LAYERS
    stream = torch.cuda.current_stream(device)
    nws = max(L.ddq_w8a16_gemm_workspace_size(M, N, K) for _, K, N, _ in PROJS)
    ws = gemm_fp8.workspace(device, nws) if nws else None
    ws_ptr, ws_bytes = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)

    def one():
        for wq, sc, b, K, N in mats:
            st = L.ddq_w8a16_gemm(xs[K].data_ptr(), wq.data_ptr(), sc.data_ptr(),
                                  b.data_ptr() if b is not None else None,
                                  _lib.DTYPE_F32 if b is not None else _lib.DTYPE_NONE,
                                  ys[N].data_ptr(), M, N, K, ws_ptr, ws_bytes, stream.cuda_stream)
            _lib.check(st, "prefill gemm")
    for _ in range(2):
        one()
    torch.cuda.synchronize(device)
    reps = 5
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        one()
    e1.record()
    torch.cuda.synchronize(device)
    ms = reduce_max(e0.elapsed_time(e1), world, device) / reps
    tf = flops * world / (ms * 1e-3) / 1e12
    per_gpu = flops / (ms * 1e-3) / 1e12
    return {"workload": "config3: 24-layer projection set at M=4096 (q/k/v stacked)",
            "tflops": round(tf, 1), "ms_per_pass": round(ms, 3), "flops_per_pass": flops,
            "frac_of_bf16_peak_per_gpu": round(per_gpu / peaks["bf16_tflops"], 4),
            "peak_tflops": peaks["bf16_tflops"], "peak_source": peaks["source"],
            "kernel": "e4m3_to_f16_kernel + w8a16_pf_kernel (exact weight expansion, tcgen05 kind::f16; CTA pairs with cta_group::2 for the 9728-row gate/up)"}


def run_config1(args, device, world, peaks):
    """Config 1: one W8A16 GEMM, x fp16 [16, 896] ~ N(0, 1), W [4864, 896] ~ N(0, 0.02)
    quantized to e4m3 with per-row scales, no bias; per call in a replayed CUDA
    graph of 64 calls over 64 weight copies (more than twice L2, so every call
    reads its weight from HBM)."""
    from ddq_b200 import gemm_fp8
    M, N, K = 16, 4864, 896
    g = torch.Generator(device=device).manual_seed(11)
    ncopy = 64  # 64 x 4.36 MB > 2 x L2
    copies = [gemm_fp8.quantize(torch.randn(N, K, generator=g, device=device) * 0.02)
              for _ in range(ncopy)]
    x = torch.randn(M, K, generator=g, device=device).half()
    reps = 64
    side = torch.cuda.Stream(device)

    def calls():
        for i in range(reps):
            gemm_fp8.f8_forward(x, *copies[i % ncopy])
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        calls()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        calls()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(3):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(device)
    del graph, copies
    us = reduce_max(e0.elapsed_time(e1), world, device) * 1e3 / (3 * reps)
    nb = N * K + 4 * N + 2 * M * K + 2 * M * N
    return {"workload": "config1: M=16, 896->4864, no bias", "us": round(us, 2),
            "gbs": round(nb / (us * 1e-6) / 1e9, 1),
            "frac_of_hbm_peak": round(nb / (us * 1e-6) / 1e9 / peaks["hbm_gbs"], 4)}


def run_lm_head(args, device, rank, world, peaks):
    """Config 4: fused lm_head 896 -> 151936 with greedy argmax at M = 1, 16, 64.

    At N = 1 the whole vocabulary is on one GPU.  Under torchrun with N > 1
    the vocabulary is sharded: rank r owns the contiguous rows
    shard_range(V, r, N), runs the fused kernel on them, and the per-rank
    packed (max, index) words are combined with one NCCL all-gather of M int64
    per rank and an element-wise max (``lm_head.sharded_greedy``).  Reported
    per M: the shard kernel per call (a replayed CUDA graph cycling through
    copies of the shard that together exceed twice the L2, so every call reads
    HBM), its HBM fraction, the all-gather per call and the whole sharded pick
    per call (eager, CUDA events, max over ranks), the same pick captured as
    one CUDA graph and replayed, and on rank 0 the number of token ids that
    differ from the unsharded pick over the full vocabulary."""
    import torch.distributed as dist
    from ddq_b200 import gemm_fp8, lm_head
    V = 151936
    lo, hi = lm_head.shard_range(V, rank, world)
    g = torch.Generator(device=device).manual_seed(88)
    w = torch.randn(V, HIDDEN, generator=g, device=device) * 0.02  # same draw on every rank
    wq, sc = gemm_fp8.quantize(w[lo:hi].contiguous())
    full = gemm_fp8.quantize(w) if (world > 1 and rank == 0) else None
    del w
    shard_bytes = (hi - lo) * HIDDEN
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    ncopy = max(2, -(-2 * l2 // shard_bytes) + 1)
    copies = [(wq, sc)] + [(wq.clone(), sc.clone()) for _ in range(ncopy - 1)]
    out = {"shards": world, "rows_per_shard": hi - lo, "weight_copies": ncopy}
    side = torch.cuda.Stream(device)
    xs = {M: torch.randn(M, HIDDEN, generator=g, device=device).half() for M in (1, 16, 64)}
    for M, x in xs.items():
        reps = max(10, ncopy)

        def calls():
            for i in range(reps):
                lm_head.lm_head_argmax(x, *copies[i % ncopy], vocab_offset=lo)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            calls()
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            calls()
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(3):
            graph.replay()
        e1.record()
        torch.cuda.synchronize(device)
        del graph
        us = reduce_max(e0.elapsed_time(e1), world, device) * 1e3 / (3 * reps)
        nb = shard_bytes + 4 * (hi - lo) + 2 * M * HIDDEN + 8 * M
        rec = {"us": round(us, 2), "gbs": round(nb / (us * 1e-6) / 1e9, 1),
               "frac_of_hbm_peak": round(nb / (us * 1e-6) / 1e9 / peaks["hbm_gbs"], 4),
               "bytes_per_call": nb}
        if world > 1:
            # the exchange alone, then the whole sharded pick (kernel + all-gather + max)
            _, packed = lm_head.lm_head_argmax(x, wq, sc, vocab_offset=lo)
            gathered = torch.empty(world * M, dtype=torch.int64, device=device)
            for _ in range(5):
                dist.all_gather_into_tensor(gathered, packed)
            torch.cuda.synchronize(device)
            dist.barrier()
            n = 50
            e0.record()
            for _ in range(n):
                dist.all_gather_into_tensor(gathered, packed)
            e1.record()
            torch.cuda.synchronize(device)
            rec["all_gather_us"] = round(reduce_max(e0.elapsed_time(e1), world, device)
                                         * 1e3 / n, 2)
            for _ in range(3):
                ids = lm_head.sharded_greedy(x, wq, sc, lo)
            torch.cuda.synchronize(device)
            dist.barrier()
            e0.record()
            for _ in range(n):
                ids = lm_head.sharded_greedy(x, wq, sc, lo)
            e1.record()
            torch.cuda.synchronize(device)
            rec["sharded_pick_us"] = round(reduce_max(e0.elapsed_time(e1), world, device)
                                           * 1e3 / n, 2)
            # the same pick captured once as a CUDA graph (kernel, all-gather,
            # combine) and replayed: the per-step latency of a serving loop
            pick = lm_head.ShardedGreedyGraph(x.clone(), wq, sc, lo)
            for _ in range(3):
                pick.replay()
            torch.cuda.synchronize(device)
            dist.barrier()
            e0.record()
            for _ in range(n):
                gids = pick.replay()
            e1.record()
            torch.cuda.synchronize(device)
            rec["sharded_pick_graph_us"] = round(reduce_max(e0.elapsed_time(e1), world, device)
                                                 * 1e3 / n, 2)
            gids = gids.clone()
            pick.release()
            del pick
            torch.cuda.synchronize(device)
            if rank == 0:
                ref_ids, _ = lm_head.lm_head_argmax(x, *full)
                rec["mismatch_vs_unsharded"] = int((ids != ref_ids).sum())
                rec["graph_mismatch_vs_unsharded"] = int((gids != ref_ids).sum())
        out[str(M)] = rec
    if world > 1:
        m = [out[k] for k in ("1", "16", "64")]
        limit = ("all-gather" if all(r["all_gather_us"] > r["us"] for r in m)
                 else "shard kernel" if all(r["all_gather_us"] < r["us"] for r in m) else "mixed")
        out["limited_by"] = limit
        out["timing"] = ("shard kernel: replayed CUDA graph; all-gather and sharded pick: eager "
                         "calls between CUDA events (host launch gaps included); sharded pick "
                         "graph: the whole pick captured once (lm_head.ShardedGreedyGraph) and "
                         "replayed; max over ranks")
    del copies, full
    torch.cuda.empty_cache()
    return out


def run_generation(args, device, rank, world, peaks):
    """Config 5: greedy generation, 64 prompts x 512 random ids, 256 new tokens,
    data-parallel replicas (64 / world prompts per GPU), random-init weights."""
    from ddq_b200.engine import Config, Engine
    cfg = Config()
    eng = Engine.random(cfg, device, seed=99)
    per = max(1, args.gen_prompts // world)
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    prompts = torch.randint(0, cfg.vocab_size, (per, args.gen_prompt_len), generator=g, device=device)
    eng.generate(prompts, 4)   # warm-up on the same shapes (kernel attributes, attention plans)
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st = {}
    e0.record()
    toks = eng.generate(prompts, args.gen_new_tokens, stats=st)
    e1.record()
    torch.cuda.synchronize(device)
    ms = reduce_max(e0.elapsed_time(e1), world, device)
    # the replayed decode steps alone (device time between events recorded
    # after the step's capture), max over ranks
    d0, d1 = st["decode_events"]
    decode_ms = reduce_max(d0.elapsed_time(d1), world, device)
    # the prefill share of that time: the same prompts, first token only
    e0.record()
    eng.generate(prompts, 1)
    e1.record()
    torch.cuda.synchronize(device)
    prefill_ms = reduce_max(e0.elapsed_time(e1), world, device)
    total = per * world * args.gen_new_tokens
    # one decode step's algorithmic HBM bytes on a GPU: every projection weight
    # with its scales and biases, the lm_head, and the K/V rows attended to (the
    # step's mean context, S + new/2 positions)
    L, Hkv, D = cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim
    layer_w = sum(N * K + 4 * N + (4 * N if b else 0) for _, K, N, b in PROJS)
    lm_w = cfg.vocab_size * cfg.hidden_size + 4 * cfg.vocab_size
    ctx = args.gen_prompt_len + args.gen_new_tokens / 2
    kv = L * 2 * per * Hkv * ctx * D * 2
    step_bytes_gpu = L * layer_w + lm_w + kv
    step_ms = decode_ms / max(1, st["decode_steps"])
    parity = None
    if world == 1 and not args.no_parity:
        parity = generation_parity(eng, prompts, toks)
    del eng
    torch.cuda.empty_cache()
    return {"workload": f"config5: {per * world} prompts x {args.gen_prompt_len} random ids, "
                        f"{args.gen_new_tokens} greedy tokens, replicas x{world}",
            "tok_s": round(total / (ms * 1e-3), 1), "ms": round(ms, 1),
            "prefill_ms": round(prefill_ms, 1),
            "decode_ms_per_step": round(step_ms, 3),
            "capture_and_host_ms": round(ms - prefill_ms - decode_ms, 1),
            "decode_timing": "CUDA events around the replayed decode steps (the step is "
                             "captured once per generate call, after the prefill is queued; "
                             "tok_s and ms include prefill, capture and any host wait)",
            "decode_step_hbm_bytes_per_gpu": int(step_bytes_gpu),
            "decode_roofline_frac": round(step_bytes_gpu / (step_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                                          4),
            "tokens": int(total), "checksum": int(toks.sum().item()) % 1000003,
            "parity": parity}


def generation_parity(eng, prompts, toks):
    """Greedy parity of the timed run's tokens against the reference semantics
    (``ddq_b200.parity``): the oracle engine (fp32 projections of the same
    dequantised weights, fp16 logits, lowest-index argmax) teacher-forced on
    the same context at every step, and running free from the same prompts."""
    from ddq_b200 import parity
    from ddq_b200.engine import Engine
    w = {"embed": eng.embed, "final_norm": eng.final_norm, "layers": eng.layers,
         "lm_head": eng.lm_head}
    oracle = Engine(eng.cfg, w, eng.device, linear="oracle")
    tf = parity.teacher_forced_report(oracle, prompts, toks, max_listed=32)
    # the reference semantics' own floor: fp64 accumulation on the same contexts
    floor = parity.oracle_noise_report(oracle, Engine(eng.cfg, w, eng.device, linear="oracle64"),
                                       prompts, toks)
    free = parity.free_run_report(oracle, prompts, toks)
    for layer in eng.layers:    # drop the oracle's fp32 weight copies
        for p in layer.values():
            if hasattr(p, "_wdeq"):
                p._wdeq = None
    eng.lm_head._wdeq = None
    return {"teacher_forced": tf, "reference_floor": floor, "free_run": free,
            "judge": "same graph with fp32 projections of the dequantised weights, fp16 logits, "
                     "lowest-index argmax; margin = oracle fp16 logit of its pick minus of ours; "
                     "reference_floor = the same oracle with fp64 accumulation against it"}


def launches_per_step(calls):
    """Kernels of this library per step, as the library reports them per shape:
    one for a GEMM of <= 16 tokens that the thin kernel takes, two (activation
    split + GEMM) for the other decode shapes."""
    from ddq_b200 import _lib
    L = _lib.load()
    return sum(L.ddq_w8a16_gemm_kernel_count(c[6], c[7], c[8]) for c in calls)


def run_e2e(args, wl, device, world):
    """Config 2 end to end through the public API (``gemm_fp8.f8_forward``): every
    step copies the activations in from pinned host memory and every GEMM's output
    back to pinned host memory.  Timed as a replayed CUDA graph of those calls (how
    a serving loop, and this repo's engine, runs them): the outputs of each M pass
    go back on a side stream while the next pass computes.  The same calls made
    eagerly, one Python call per GEMM and per copy, are reported as ``eager``."""
    from ddq_b200 import gemm_fp8
    host_x = {M: {n: t.cpu().pin_memory() for n, t in wl.x[M].items()} for M in DECODE_M}
    host_y = {M: [{n: torch.empty(t.shape, dtype=t.dtype).pin_memory() for n, t in d.items()}
                  for d in wl.y[M]] for M in DECODE_M}
    h2d = sum(t.numel() * 2 for M in DECODE_M for t in host_x[M].values())
    d2h = sum(t.numel() * 2 for M in DECODE_M for d in host_y[M] for t in d.values())
    side = torch.cuda.Stream(device)

    def eager_step():
        for M in DECODE_M:
            xs = {n: t.to(device, non_blocking=True) for n, t in host_x[M].items()}
            for li, layer in enumerate(wl.layers):
                for name, _, _, _ in PROJS:
                    wq, s, b = layer[name]
                    y = gemm_fp8.f8_forward(xs[name], wq, s, b)
                    host_y[M][li][name].copy_(y, non_blocking=True)

    def graph_step():
        main = torch.cuda.current_stream(device)
        for M in DECODE_M:
            xs = {n: t.to(device, non_blocking=True) for n, t in host_x[M].items()}
            outs = []
            for li, layer in enumerate(wl.layers):
                for name, _, _, _ in PROJS:
                    wq, s, b = layer[name]
                    outs.append((host_y[M][li][name], gemm_fp8.f8_forward(xs[name], wq, s, b)))
            side.wait_stream(main)
            with torch.cuda.stream(side):
                for h, y in outs:
                    h.copy_(y, non_blocking=True)
        main.wait_stream(side)

    def timed(step, steps):
        torch.cuda.synchronize(device)
        if world > 1:
            torch.distributed.barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(steps):
            step()
        ev1.record()
        torch.cuda.synchronize(device)
        return reduce_max(ev0.elapsed_time(ev1), world, device)

    # graph of the public-API step (warmed up eagerly first: kernel attributes, workspaces)
    cap = torch.cuda.Stream(device)
    cap.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(cap):
        for _ in range(2):
            graph_step()
    torch.cuda.current_stream(device).wait_stream(cap)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        graph_step()
    for _ in range(2):
        graph.replay()
    steps = max(1, args.steps)
    ms = timed(graph.replay, steps)
    del graph
    # the same calls, eagerly
    esteps = max(1, min(args.steps, args.e2e_steps))
    for _ in range(2):
        eager_step()
    ems = timed(eager_step, esteps)
    value = step_bytes() * steps * world / (ms * 1e-3) / 1e12
    evalue = step_bytes() * esteps * world / (ems * 1e-3) / 1e12
    return {"value": round(value, 4), "unit": "TB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps, "ms_per_step": round(ms / steps, 3),
            "api": "ddq_b200.gemm_fp8.f8_forward, one call per GEMM, replayed as a CUDA graph "
                   "with the host copies inside",
            "eager": {"value": round(evalue, 4), "ms_per_step": round(ems / esteps, 3),
                      "steps": esteps,
                      "api": "the same calls and copies made eagerly from Python"}}


# ----------------------------------------------------------------------------- CPU side
def cpu_sample_once(layers=1, seed=0):
    """One bounded sample of the reference path on the host: `layers` layers of the
    projection set at every M, per-call dequant + fp32 matmul (oracle, PyTorch CPU)."""
    from oracle.w8a16 import f8_forward_torch_cpu, quantize
    rng = np.random.default_rng(seed)
    mats = []
    for _ in range(layers):
        for name, K, N, has_bias in PROJS:
            wq, s = quantize(rng.normal(0, 0.02, (N, K)).astype(np.float32))
            b = torch.from_numpy(rng.normal(0, 0.02, N).astype(np.float32)) if has_bias else None
            mats.append((torch.from_numpy(wq), torch.from_numpy(s), b, K, N, has_bias))
    xs = {(M, K): torch.from_numpy(rng.normal(0, 1, (M, K)).astype(np.float16))
          for M in DECODE_M for K in (HIDDEN, INTER)}
    nbytes = sum(proj_bytes(M, K, N, hb) for M in DECODE_M for (_, _, _, K, N, hb) in mats)

    def run():
        for M in DECODE_M:
            for wq, s, b, K, N, _ in mats:
                f8_forward_torch_cpu(xs[(M, K)], wq, s, b)
    return run, nbytes


def cpu_baseline(budget_s=15.0):
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    run, nbytes = cpu_sample_once(layers=1)
    run()  # warm-up
    t0 = time.perf_counter()
    reps = 0
    while True:
        run()
        reps += 1
        if time.perf_counter() - t0 > budget_s or reps >= 50:
            break
    dt = time.perf_counter() - t0
    return {"value": round(nbytes * reps / dt / 1e12, 6), "unit": "TB/s", "cores": threads,
            "kind": "port",
            "sample": f"1 of 24 layers of the projection set at M=1,8,32,64, {reps} reps "
                      f"({dt:.1f} s); oracle in PyTorch CPU with per-call e4m3 dequant",
            "cpu": cpu_model()}


def cpu_model():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def run_reference(args, rank, world):
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    run, nbytes = cpu_sample_once(layers=1)
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    dt = time.perf_counter() - t0
    value = nbytes * args.steps / dt / 1e12
    sample = ("each step = 1 of the 24 layers of the config-2 projection set at M=1,8,32,64 "
              "(14.9 MB of weights per M), PyTorch CPU oracle with per-call dequant")
    gpu = reference_gpu_kernels()
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": "TB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e4m3xf16->f32",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations; no dataset)",
        "config": {"workload": "config2: 24-layer decode projection set at M=1,8,32,64 "
                               "(bounded sample: 1 layer per step)",
                   "parallelism": "host cores of rank 0"},
        "cpu_baseline": {"value": round(value, 6), "unit": "TB/s", "cores": threads,
                         "kind": "port", "sample": sample, "cpu": cpu_model()},
        "e2e": {"value": round(value, 6), "unit": "TB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "reference_gpu_kernels": gpu,
    }


def reference_gpu_kernels():
    """The reference's own CUDA operators on this box's GPU, on the shapes this
    repo's line reports: gemm_FP8_d.cu f8_forward (its W8A16 kernel,
    gemm_FP8_d.cu:94-146, 171-210), gemm_d.cu forward (the engine's cuBLAS fp16
    projection, gemm_d.cu:36-87) and sampler_d.cu forward (greedy argmax,
    sampler_d.cu:51-70), compiled unmodified from the reference's sources for
    sm_100 into oracle/_ref.  Each shape cycles through weight copies that
    together exceed twice the L2; eager calls on the default stream (the
    operators allocate their outputs and gemm_d's cuBLAS handle is not bound
    to a stream) between CUDA events, after warm-up.  None when no GPU or no
    prebuilt operators are present."""
    if not torch.cuda.is_available():
        return None
    try:
        from oracle.build_ref import available, load_ref
        if not all(available(n) for n in ("ref_gemm_fp8", "ref_gemm_d", "ref_sampler")):
            return {"unavailable": "reference operators not built into oracle/_ref"}
        fp8, gd, smp = load_ref("ref_gemm_fp8"), load_ref("ref_gemm_d"), load_ref("ref_sampler")
    except Exception as exc:  # an import failure is reported, not fatal to the CPU arm
        return {"unavailable": f"loading the reference operators failed: {exc!r}"[:300]}
    dev = torch.device("cuda", 0)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    g = torch.Generator(device=dev).manual_seed(5)
    out = {}

    def timed(fn, reps):
        for _ in range(3):
            fn(0)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            fn(i)
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) * 1e3 / reps

    for name, M, N, K in (("config1 M=16 896->4864", 16, 4864, 896),
                          ("gate_up M=64 896->9728", 64, 9728, 896),
                          ("gate_up M=4096 896->9728", 4096, 9728, 896)):
        w16 = (torch.randn(N, K, generator=g, device=dev) * 0.02).half()
        wq, scales = fp8.quantize(w16)
        x = torch.randn(M, K, generator=g, device=dev).half()
        nc = max(2, -(-2 * l2 // (N * K)) + 1)
        q_copies = [(wq.clone(), scales.clone()) for _ in range(nc)]
        h_copies = [w16.clone() for _ in range(max(2, -(-2 * l2 // (2 * N * K)) + 1))]
        reps = 5 if M >= 4096 else 50
        us_f8 = timed(lambda i: fp8.f8_forward(x, *q_copies[i % nc]), reps)
        us_gd = timed(lambda i: gd.forward(x, h_copies[i % len(h_copies)], None), reps)
        nb8 = N * K + 4 * N + 2 * M * K + 2 * M * N
        nb16 = 2 * N * K + 2 * M * K + 2 * M * N
        fl = 2 * M * N * K
        out[name] = {
            "f8_forward_us": round(us_f8, 2), "f8_forward_gbs": round(nb8 / us_f8 / 1e3, 1),
            "f8_forward_tflops": round(fl / us_f8 / 1e6, 2),
            "gemm_d_cublas_fp16_us": round(us_gd, 2), "gemm_d_gbs": round(nb16 / us_gd / 1e3, 1),
            "gemm_d_tflops": round(fl / us_gd / 1e6, 2)}
        del q_copies, h_copies, w16, wq, scales
    lg = torch.randn(64, 1, 151936, generator=g, device=dev).half()
    out["sampler argmax [64,1,151936]"] = {"us": round(timed(lambda i: smp.forward(lg), 50), 2)}
    out["timing"] = ("eager calls, CUDA events on the default stream, weight copies > 2x L2; "
                     "reference operators compiled unmodified for sm_100 (oracle/_ref)")
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- utils
def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured (MEASURED_PEAKS.json)"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                "source": "fallback (profiling recipe)"}


def profile_traffic(path):
    """DRAM bytes per launch of the roofline kernel (dram__bytes_read.sum +
    dram__bytes_write.sum from one ncu capture), read from the summary's
    `traffic_bytes_per_launch:` line; (None, reason) if the summary lacks it."""
    try:
        for ln in open(path):
            if ln.strip().startswith("traffic_bytes_per_launch:"):
                return int(ln.split(":", 1)[1].strip().split()[0]), os.path.relpath(path, REPO)
    except (OSError, ValueError):
        pass
    return None, f"no traffic_bytes_per_launch line in {os.path.relpath(path, REPO)}"


def reduce_max(v, world, device):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--skip-extra", action="store_true",
                    help="only the config-2 headline (no prefill / lm_head / generation)")
    ap.add_argument("--gen-prompts", type=int, default=64)
    ap.add_argument("--gen-prompt-len", type=int, default=512)
    ap.add_argument("--gen-new-tokens", type=int, default=256)
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the greedy-parity check of the generation run (not timed)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)
    try:
        line = run_ours(args, rank, world, device)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
