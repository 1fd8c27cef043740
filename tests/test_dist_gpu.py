"""Multi-GPU: the vocab-sharded lm_head over NCCL (one process per GPU).

Each rank quantizes its contiguous shard of the same seeded 151936 x 896
weight, runs the fused lm_head argmax on it, and the (max, index) words are
combined with one NCCL all-gather; every rank must get exactly the token ids
the unsharded kernel picks on one GPU, eagerly and through the pick captured
as one CUDA graph (kernel, all-gather, combine) and replayed on new input.  Needs >= 2 GPUs (skipped otherwise)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

VOCAB, HIDDEN = 151936, 896


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(device):
    g = torch.Generator(device=device).manual_seed(1234)
    w = torch.randn(VOCAB, HIDDEN, generator=g, device=device) * 0.02
    x = torch.randn(64, HIDDEN, generator=g, device=device).half()
    return w, x


def _rank(rank, world, port, out):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from ddq_b200 import gemm_fp8, lm_head
        w, x = _weights(dev)
        lo, hi = lm_head.shard_range(VOCAB, rank, world)
        wq, s = gemm_fp8.quantize(w[lo:hi])
        res = {}
        for M in (1, 16, 64):
            res[M] = lm_head.sharded_greedy(x[:M], wq, s, lo).cpu()
            # the same pick captured as one CUDA graph, replayed on a new input
            pick = lm_head.ShardedGreedyGraph(torch.zeros_like(x[:M]), wq, s, lo)
            pick.x.copy_(x[:M])
            res[("graph", M)] = pick.replay().clone().cpu()
            pick.release()
            torch.cuda.synchronize()
        if rank == 0:
            wq_full, s_full = gemm_fp8.quantize(w)
            for M in (1, 16, 64):
                ids, _ = lm_head.lm_head_argmax(x[:M], wq_full, s_full)
                res[("full", M)] = ids.cpu()
        torch.cuda.synchronize()
        out[rank] = res
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_vocab_sharded_lm_head_over_nccl(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_rank, args=(world, free_port(), out), nprocs=world, join=True)
    for M in (1, 16, 64):
        full = out[0][("full", M)]
        for r in range(world):
            assert torch.equal(out[r][M], full), (r, M)
            assert torch.equal(out[r][("graph", M)], full), (r, M)
