"""Host-side pieces of the greedy-parity judge (``ddq_b200.parity``) that need
no GPU: the fp16 spacing used to express logit margins in ulps, checked
against numpy on every finite fp16 magnitude, and the margin classification
of a crafted teacher-forced report."""
import numpy as np
import torch

from ddq_b200 import parity


def test_fp16_ulp_matches_numpy_spacing_on_every_value():
    h = np.arange(0, 0x7BFF, dtype=np.uint16).view(np.float16)  # 0 .. 65472
    vals = np.concatenate([h, -h]).astype(np.float32)
    got = parity._fp16_ulp(torch.from_numpy(vals)).numpy()
    ref = np.spacing(np.abs(vals).astype(np.float16)).astype(np.float32)
    np.testing.assert_array_equal(got, ref)
    # the largest finite value: the spacing below it (numpy reports inf)
    assert parity._fp16_ulp(torch.tensor([65504.0])).item() == 32.0


class _FakeOracle:
    """Stands in for Engine(linear="oracle") in oracle_logits_at: fixed fp16
    logits per (sequence, step) regardless of the context."""

    def __init__(self, logits):
        self._lg = logits  # [B, T, V] fp32 holding fp16 values

    def new_cache(self, b, s):
        return None

    def hidden(self, part, cache, b0, start):
        B, S = part.shape
        T = self._lg.shape[1]
        # position S - T .. S - 1 carry the index of the step
        h = torch.zeros(B, S, 1)
        h[:, S - T:, 0] = torch.arange(T, dtype=torch.float32)
        self._rows = part[:, 0].long()
        return h

    def logits(self, h):
        T = self._lg.shape[1]
        steps = h[:, 0].long()
        rows = self._rows.repeat_interleave(T)
        return self._lg[rows, steps].half()


def test_teacher_forced_margins_in_ulps():
    B, T, V = 2, 3, 5
    lg = torch.zeros(B, T, V)
    lg[0, 0] = torch.tensor([1.0, 2.0, 2.0, 0.0, 0.0])       # exact tie: lowest index 1
    lg[0, 1] = torch.tensor([4.0, 4.0 - 2 * 2 ** -8, 0, 0, 0])  # 2 ulps at 4.0 (ulp 2^-8)
    lg[0, 2] = torch.tensor([0.0, 0.0, 1.0, 0.0, 0.0])
    lg[1, :] = torch.tensor([0.0, 0.0, 0.0, 8.0, 8.0 - 5 * 2 ** -7])  # 5 ulps at 8.0
    prompts = torch.tensor([[0, 9, 9], [1, 9, 9]])         # column 0 selects the row
    tokens = torch.tensor([[2, 1, 2], [3, 4, 3]])
    rep = parity.teacher_forced_report(_FakeOracle(lg), prompts, tokens)
    assert rep["steps"] == 6 and rep["equal"] == 3
    assert rep["differ_by_margin_ulps"] == {"0": 1, "1": 0, "2": 1, ">2": 1}
    assert rep["max_margin_ulps"] == 5.0
