"""Record golden vectors from the reference's own CUDA operators.

Runs on a CUDA machine with the reference modules prebuilt by
``python -m oracle.build_ref`` (``oracle/_ref/``).  It draws seeded inputs,
calls the UNMODIFIED reference operators through their own pybind11 API
(``gemm_FP8_d.cu:221-228``, ``gemm_d.cu:91-93``, ``sampler_d.cu:74-76``) and
writes ``ref_golden.npz`` with inputs and outputs.  ``tests/test_golden.py``
then checks the CPU oracle against these recorded outputs, which pins the
oracle to the reference itself (the reference ships no tests or golden data).

    python tests/golden/make_golden.py --out tests/golden/ref_golden.npz
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, REPO)

from oracle.build_ref import load_ref  # noqa: E402


def crafted_weight_rows(K: int) -> np.ndarray:
    """Rows that hit the encoder's corner cases once scaled by 448/absmax."""
    rows = []
    # exact e4m3 ties after scaling (absmax 448 keeps scale == 1)
    r = np.zeros(K, np.float32)
    r[0] = 448.0
    r[1:9] = [1.0625, 1.1875, 3.25, 0.0146, 0.0155, 2.0 ** -10, 1.5 * 2.0 ** -10, 17.0]
    r[9:17] = -r[1:9]
    rows.append(r)
    rows.append(np.zeros(K, np.float32))                 # all-zero row -> scale 1
    r = np.full(K, 2.0 ** -12, np.float32)               # tiny row (fp16 subnormal scale)
    r[3] = 2.0 ** -11
    rows.append(r)
    return np.stack(rows).astype(np.float16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(REPO, "tests", "golden", "ref_golden.npz"))
    a = ap.parse_args()
    dev = torch.device("cuda:0")
    fp8 = load_ref("ref_gemm_fp8")
    gd = load_ref("ref_gemm_d")
    smp = load_ref("ref_sampler")

    gen = torch.Generator().manual_seed(2024)
    K, N, M = 896, 125, 16
    w = (torch.randn(N, K, generator=gen) * 0.02).half().numpy()
    w = np.concatenate([w, crafted_weight_rows(K)])     # N + 3 = 128 rows
    x = torch.randn(M, K, generator=gen).half().numpy()
    b16 = (torch.randn(w.shape[0], generator=gen) * 0.02).half().numpy()

    wq, sc = fp8.quantize(torch.from_numpy(w).to(dev))
    y_f8 = fp8.f8_forward(torch.from_numpy(x).to(dev), wq, sc, torch.from_numpy(b16).to(dev))
    y_fw = fp8.forward(torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev), None)
    y_gd = gd.forward(torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev),
                      torch.from_numpy(b16).to(dev))

    V = 4099
    lg = (torch.randn(8, V, generator=gen) * 3).half().numpy()
    lg[0, 10] = lg[0, 4000] = 50.0
    lg[1, :] = 1.0
    lg[2, 3000:] = np.nan
    lg[3, :] = -np.inf
    lg[4, :5] = np.nan
    lg[4, 5:] = -np.inf
    lg[4, 4090] = -60000.0
    lg[5, 7] = np.inf
    am = smp.forward(torch.from_numpy(lg).to(dev).reshape(8, 1, V))
    torch.cuda.synchronize()

    np.savez_compressed(
        a.out, w=w, x=x, bias16=b16,
        ref_wq=wq.cpu().numpy(), ref_scales=sc.cpu().numpy(),
        ref_y_f8=y_f8.cpu().numpy(), ref_y_forward=y_fw.cpu().numpy(),
        ref_y_gemm_d=y_gd.cpu().numpy(),
        logits=lg, ref_argmax=am.cpu().numpy().reshape(-1),
        torch_version=np.array(torch.__version__),
        device=np.array(torch.cuda.get_device_name(0)))
    print("wrote", a.out)


if __name__ == "__main__":
    main()
