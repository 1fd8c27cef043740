"""Compile the reference's own CUDA operators into ``oracle/_ref/`` (test infrastructure).

The reference (hdahroug/ddq) builds each ``*_d.cu`` file as a standalone
PyTorch extension with ``torch.utils.cpp_extension.load`` and
``-O3 --use_fast_math`` (``engine.py:25-79``).  This recipe compiles three of
them, unmodified and where they lie in the reference checkout, for sm_100:

* ``gemm_FP8_d.cu`` -> ``ref_gemm_fp8``  (quantize / f8_forward / forward)
* ``gemm_d.cu``     -> ``ref_gemm_d``    (the engine's cuBLAS fp16 projection)
* ``sampler_d.cu``  -> ``ref_sampler``   (greedy argmax)

Output goes only to ``oracle/_ref/<name>/<name>.so`` (git-ignored, carried to
the GPU box with the working tree).  On the GPU box, where the reference
checkout does not exist, ``load_ref`` imports the prebuilt modules.  They are
used only by ``tests/`` and ``tests/golden/make_golden.py`` to pin the oracle
against the reference itself; nothing in the ``ddq_b200`` product touches
them.

    python -m oracle.build_ref [--reference DIR] [--force]
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_OUT = os.path.join(HERE, "_ref")
# The reference checkout: --reference, else DDQ_REFERENCE_DIR, else a
# directory named "reference" beside this repository (absent on the GPU box,
# which only imports the prebuilt modules).
DEFAULT_REFERENCE = os.environ.get(
    "DDQ_REFERENCE_DIR", os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))

MODULES = {
    "ref_gemm_fp8": "gemm_FP8_d.cu",
    "ref_gemm_d": "gemm_d.cu",
    "ref_sampler": "sampler_d.cu",
}


def so_path(name: str) -> str:
    return os.path.join(REF_OUT, name, f"{name}.so")


def _build_one(name: str, src: str) -> str:
    """Runs in a child process: one cpp_extension build (ninja, minutes)."""
    import torch.utils.cpp_extension as ce
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    bdir = os.path.join(REF_OUT, name)
    os.makedirs(bdir, exist_ok=True)
    ce.load(name=name, sources=[src], extra_cuda_cflags=["-O3", "--use_fast_math"],
            build_directory=bdir, verbose=False)
    return so_path(name)


def build(reference: str = DEFAULT_REFERENCE, force: bool = False) -> list[str]:
    """Build every module whose .so is missing or older than its source.

    Returns the list of built paths; returns [] without error when the
    reference checkout is absent (e.g. on the GPU box).
    """
    if not os.path.isdir(reference):
        return []
    procs = []
    for name, fname in MODULES.items():
        src = os.path.join(reference, fname)
        out = so_path(name)
        if not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(src):
            continue
        code = (f"import sys; sys.path.insert(0, {os.path.dirname(HERE)!r}); "
                f"from oracle.build_ref import _build_one; _build_one({name!r}, {src!r})")
        procs.append((name, subprocess.Popen([sys.executable, "-c", code],
                                             stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    built = []
    for name, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            raise RuntimeError(f"building reference module {name} failed:\n{out.decode()[-4000:]}")
        built.append(so_path(name))
    return built


def available(name: str) -> bool:
    return os.path.exists(so_path(name))


def load_ref(name: str):
    """Import a prebuilt reference module (pybind11 extension) from oracle/_ref."""
    import torch  # noqa: F401  (loads libc10/libtorch the extension links against)
    path = so_path(name)
    if not os.path.exists(path):
        raise FileNotFoundError(f"reference module {name} not built at {path}")
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=DEFAULT_REFERENCE)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    for p in build(a.reference, a.force):
        print(p)
