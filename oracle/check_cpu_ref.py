"""Check `oracle/cpu_ref.py` against the reference's own Numba CPU kernels (BUILD-CONTAINER ONLY).

Runs where the reference source tree is mounted (it imports `ramvi_engine.cpu.cpu_layer` and
`ramvi_engine.generation.head` from it): the restated kernels must give the reference's bits and run at its speed,
so that bench.py's CPU baseline stands for the reference's CPU path on the GPU box, where the reference package does
not travel. Prints one line per kernel: best-of-5 microseconds for both and the largest output difference.

Usage:  python oracle/check_cpu_ref.py [/path/to/reference/ramvi/engine]
"""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
REF = sys.argv[1] if len(sys.argv) > 1 else "/root/reference/ramvi/engine"
sys.path.insert(0, REF)

from ramvi_engine.cpu import cpu_layer as R  # noqa: E402
from ramvi_engine.generation import head as RH  # noqa: E402
from oracle import cpu_ref as O, codec  # noqa: E402


def best(fn, *a):
    fn(*a)
    t = 1e9
    for _ in range(5):
        t0 = time.perf_counter()
        fn(*a)
        t = min(t, time.perf_counter() - t0)
    return t * 1e6


def main():
    g = np.random.default_rng(0)
    for n, k in [(6144, 1024), (1024, 3072), (6144, 4096), (24576, 4096), (4096, 12288)]:
        W = codec.f32_to_bf16_bits((g.standard_normal((n, k)) * 0.02).astype(np.float32))
        X = g.standard_normal((1, k)).astype(np.float32)
        Y1, Y2 = np.zeros((1, n), np.float32), np.zeros((1, n), np.float32)
        t1, t2 = best(R.matmat16, W, X, Y1, False), best(O.matmat16, W, X, Y2, False)
        print(f"matmat16 [{n},{k}]: reference {t1:.1f} us, restated {t2:.1f} us, max|diff| {np.abs(Y1 - Y2).max()}")
    V, D = 151936 // 8, 4096
    W = codec.f32_to_bf16_bits((g.standard_normal((V, D)) * 0.02).astype(np.float32))
    H = g.standard_normal((1, D)).astype(np.float32)
    toks, rows = np.arange(V), np.zeros(V, np.int64)
    o1, o2 = np.empty(V, np.float32), np.empty(V, np.float32)
    t1, t2 = best(RH.exact_rows, W, toks, rows, H, o1), best(O.exact_rows, W, toks, rows, H, o2)
    print(f"exact_rows [{V},{D}]: reference {t1:.1f} us, restated {t2:.1f} us, bit-identical {np.array_equal(o1, o2)}")


if __name__ == "__main__":
    main()
