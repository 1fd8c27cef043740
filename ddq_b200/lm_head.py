"""Fused lm_head GEMM + greedy argmax, optionally vocab-sharded across ranks.

Replaces ``engine.py:338`` (lm_head through the fp16 GEMM, materialising
``[B,S,151936]`` logits) followed by ``sampler_d.forward`` on the last
position (``engine.py:345,351``; ``sampler_d.cu:10-49``).  The logits are
never written: the CUDA kernel reduces each token row to one packed word

    (ordered fp16 logit << 32) | (0xFFFFFFFF - global vocab index)

whose maximum is the largest fp16-rounded logit with ties to the lowest index
- exactly the reference sampler's pick.  With the vocabulary split into
contiguous shards over ranks, one all-gather of M packed words per rank (NCCL
over NVLink on GPUs, gloo on CPU) and an element-wise max give the global
token on every rank.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib

_lm_workspaces: dict = {}


def lm_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """The lm_head's own zero-filled workspace per (device, current stream),
    grown on demand.  It is not shared with the other GEMM entry points: its
    first bytes hold the streaming kernel's arrival counter, which every call
    leaves at zero for the next one."""
    key = (device.type, device.index, torch.cuda.current_stream(device).cuda_stream)
    buf = _lm_workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _lm_workspaces[key] = buf
    return buf


def shard_range(vocab: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous vocab rows [lo, hi) owned by `rank` (sizes differ by at most 1)."""
    base, rem = divmod(vocab, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)


def unpack(packed: torch.Tensor) -> torch.Tensor:
    """Packed words -> int64 token ids (0 for a row with no finite logit)."""
    low = packed & 0xFFFFFFFF
    ids = 0xFFFFFFFF - low
    return torch.where(packed == 0, torch.zeros_like(ids), ids)


def combine_shards(packed: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather every rank's packed words and reduce them with max.

    Works for any backend (NCCL on GPU tensors, gloo on CPU tensors); every
    rank returns the same int64 token ids.  Signed int64 comparison is safe:
    the key occupies bits 32..47 only, so every packed word is non-negative.
    """
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if world == 1:
        return unpack(packed)
    flat = packed.contiguous().reshape(-1)
    gathered = torch.empty((world * flat.numel(),), dtype=packed.dtype, device=packed.device)
    dist.all_gather_into_tensor(gathered, flat, group=group)
    best = gathered.view(world, -1).max(dim=0).values
    return unpack(best.view(packed.shape))


def lm_head_argmax(x: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor,
                   vocab_offset: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Greedy token per row of x over this shard's vocab rows.

    x fp16 [..., K]; wq uint8 [N_shard, K]; scales fp32 [N_shard].
    Returns (ids int64 [M], packed int64 [M]); ids are global vocab indices.
    """
    if not (x.is_cuda and wq.is_cuda and scales.is_cuda):
        raise RuntimeError("lm_head_argmax: CUDA tensors required")
    if x.dtype != torch.float16 or wq.dtype != torch.uint8 or scales.dtype != torch.float32:
        raise RuntimeError("lm_head_argmax: expected fp16 x, uint8 wq, fp32 scales")
    N, K = wq.shape
    if x.size(-1) != K or scales.numel() != N:
        raise RuntimeError("lm_head_argmax: shape mismatch")
    x2 = x.contiguous().reshape(-1, K)
    M = x2.size(0)
    packed = torch.empty((M,), dtype=torch.int64, device=x.device)
    ids = torch.empty((M,), dtype=torch.int64, device=x.device)
    L = _lib.load()
    with torch.cuda.device(x.device):
        nws = L.ddq_lm_head_argmax_workspace_size(M, N, K)
        ws = lm_workspace(x.device, nws) if nws else None
        st = L.ddq_lm_head_argmax(x2.data_ptr(), wq.contiguous().data_ptr(),
                                  scales.contiguous().data_ptr(), M, N, K, int(vocab_offset),
                                  packed.data_ptr(), ids.data_ptr(),
                                  ws.data_ptr() if ws is not None else None,
                                  ws.numel() if ws is not None else 0,
                                  torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(st, "lm_head_argmax")
    return ids, packed


def sharded_greedy(x: torch.Tensor, wq_shard: torch.Tensor, scales_shard: torch.Tensor,
                   vocab_offset: int, group: Optional[object] = None) -> torch.Tensor:
    """Global greedy ids from a vocab-sharded lm_head (one all-gather of M int64/rank)."""
    _, packed = lm_head_argmax(x, wq_shard, scales_shard, vocab_offset)
    return combine_shards(packed, group)


class ShardedGreedyGraph:
    """The vocab-sharded greedy pick (shard kernel, NCCL all-gather, combine)
    captured once as a CUDA graph and replayed, for serving loops that pick
    a token every step: no host work between the three parts.

    ``x`` is the static input: copy each step's activations into it, then call
    ``replay()``, which returns the static int64 ids tensor.  Every rank of
    ``group`` builds and replays its graph in the same order.  Call
    ``release()`` on every rank before the process group is destroyed (a
    graph that still holds an NCCL operation keeps the communicator alive)."""

    def __init__(self, x: torch.Tensor, wq_shard: torch.Tensor, scales_shard: torch.Tensor,
                 vocab_offset: int, group=None):
        if not x.is_cuda:
            raise RuntimeError("ShardedGreedyGraph: CUDA tensors required")
        self.x = x
        dev = x.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        # warm-up on the capture stream: its lm_head workspace and the
        # communicator exist before capture
        with torch.cuda.stream(side):
            sharded_greedy(x, wq_shard, scales_shard, vocab_offset, group)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=side):
            self.ids = sharded_greedy(x, wq_shard, scales_shard, vocab_offset, group)
        torch.cuda.synchronize(dev)

    def replay(self) -> torch.Tensor:
        if self.graph is None:
            raise RuntimeError("ShardedGreedyGraph: released")
        self.graph.replay()
        return self.ids

    def release(self) -> None:
        self.graph = None
