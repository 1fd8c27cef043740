"""Multi-rank host logic on CPU (gloo, world_size 2 and 4): vocab shard
ranges and the (max, index) all-gather combine used by the sharded lm_head."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import w8a16 as o


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_ranges_cover_vocab_exactly():
    from ddq_b200.lm_head import shard_range
    for vocab in (151936, 1001, 7):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(vocab, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == vocab
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1
    assert shard_range(151936, 3, 8) == (3 * 18992, 4 * 18992)


def packed_words(logits: np.ndarray, offset: int) -> np.ndarray:
    """CPU restatement of the kernel's packed key, for each row's best logit."""
    h = logits.astype(np.float16)
    b = h.view(np.uint16).astype(np.int64)
    key = np.where(b & 0x8000, (~b) & 0xFFFF, b | 0x8000)
    idx = np.arange(h.shape[1], dtype=np.int64) + offset
    word = (key << 32) | (0xFFFFFFFF - idx)
    with np.errstate(invalid="ignore"):
        ok = h.astype(np.float32) > -np.finfo(np.float32).max  # NaN and -inf never win
    word = np.where(ok, word, 0)
    return word.max(axis=1)


def _worker(rank, world, port, logits, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        from ddq_b200.lm_head import combine_shards, shard_range
        lo, hi = shard_range(logits.shape[1], rank, world)
        packed = torch.from_numpy(packed_words(logits[:, lo:hi], lo))
        ids = combine_shards(packed)
        out[rank] = ids.numpy()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_all_gather_combine_gives_global_greedy_pick(world):
    rng = np.random.default_rng(world)
    logits = rng.normal(0, 2, (8, 4099)).astype(np.float16)
    logits[0, 10] = logits[0, 4000] = 50.0      # tie across shards -> 10
    logits[1, :] = 1.0                          # all equal -> 0
    logits[2, 3000:] = np.nan
    logits[3, :] = -np.inf                      # nothing above -FLT_MAX -> 0
    logits[4, :5] = np.nan
    logits[4, 5:] = -np.inf
    logits[4, 4090] = -60000.0
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, free_port(), logits, out), nprocs=world, join=True)
    want = o.argmax_f16(logits)
    assert want[0] == 10 and want[1] == 0 and want[3] == 0 and want[4] == 4090
    for r in range(world):
        np.testing.assert_array_equal(out[r], want)


def test_rank_failure_surfaces_as_error_not_hang():
    """A rank that never joins makes the others' init fail within the timeout."""
    import datetime
    port = free_port()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    with pytest.raises(Exception):
        dist.init_process_group("gloo", rank=0, world_size=2,
                                timeout=datetime.timedelta(seconds=3))
    if dist.is_initialized():
        dist.destroy_process_group()
