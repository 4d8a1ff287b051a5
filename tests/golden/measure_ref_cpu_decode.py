"""REFERENCE CPU DECODE AGAINST THE ORACLE PORT -- baseline bookkeeping, never
part of the product path and never run on a GPU box (the reference checkout
is not there).

The benchmark's CPU baseline and its reference arm time the oracle port
(oracle.c, OpenMP over chunks) because the reference cannot run on the GPU
box. This script times both on the same tensor and host threads here: the
reference's decompress_layer_gpu(layer, device="cpu") (numba prange decode
plus _recombine) and oracle.decompress. It checks that the outputs are
bit-identical. The ratio says how far the port's figure overstates the
reference's own CPU speed.

Usage (in a container that has an Afterimage checkout):

    python tests/golden/measure_ref_cpu_decode.py <path to the checkout> [--rows 5120 --cols 5120]

Prints one line per thread count: best of 3 for each, the ratio, and
whether the outputs are equal.
"""
from __future__ import annotations

import argparse
import os
import pathlib
import sys
import tempfile
import time

os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")
os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="numba_compare_"))
sys.dont_write_bytecode = True

import numpy as np  # noqa: E402
import torch  # noqa: E402

REPO = pathlib.Path(__file__).resolve().parents[2]


def best_of(fn, n: int = 3) -> float:
    best = float("inf")
    for _ in range(n):
        t0 = time.perf_counter()
        fn()
        best = min(best, time.perf_counter() - t0)
    return best


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("checkout")
    ap.add_argument("--rows", type=int, default=5120)
    ap.add_argument("--cols", type=int, default=5120)
    args = ap.parse_args()
    sys.path.insert(0, str(REPO))
    from oracle import oracle as O
    from afterimage_b200.runtime.compressed_store import compress_layer
    sys.path.insert(0, str(pathlib.Path(args.checkout).resolve()))
    import numba
    from afterimage.runtime import compressed_store as ref
    W = (torch.randn(args.rows, args.cols, generator=torch.Generator().manual_seed(1)) * 0.02).to(torch.bfloat16)
    ours, theirs = compress_layer(W), ref.compress_layer(W)
    sm = ours.sign_mantissa.numpy()
    for threads in sorted({O.max_threads(), 1}, reverse=True):
        numba.set_num_threads(min(threads, numba.config.NUMBA_NUM_THREADS))
        ref.decompress_layer_gpu(theirs, device="cpu")  # numba JIT
        t_ref = best_of(lambda: ref.decompress_layer_gpu(theirs, device="cpu"))
        O.decompress(ours.encoded, sm, threads)
        t_port = best_of(lambda: O.decompress(ours.encoded, sm, threads))
        a = ref.decompress_layer_gpu(theirs, device="cpu").view(torch.int16).numpy().reshape(-1)
        b = np.asarray(O.decompress(ours.encoded, sm, threads)).view(np.int16).reshape(-1)
        print("%d thread(s), %dx%d: reference numba %.3f s, oracle port %.3f s, port %.1fx faster, equal=%s"
              % (threads, args.rows, args.cols, t_ref, t_port, t_ref / t_port, bool(np.array_equal(a, b))),
              flush=True)


if __name__ == "__main__":
    main()
