"""Generates tests/golden/known_answers.npz: known answers for Oct's own test inputs.

Every answer is computed here by exact or correctly-rounded arithmetic that is
independent of both the CUDA library and the C oracle, so the fixtures can pin
the oracle (tests/test_oracle_pins.py) and check the CUDA path (GPU tests):

  * SGEMM on the reference's test matrices
      - Marionette Matrix(count, seed) = ((i*7+seed)%23-11)/8
        (internal/prometheus/native/Marionette/reactor_concept_sgemm_tests.cpp:14-19):
        integers / 8, so the product is (integer matmul) / 64, exact;
      - StarterCorpus shapes with deterministicMatrix ((i%23)-11)/7
        (internal/prometheus/runtime.go:83-89, 242-249): exact rationals of the
        fp32 inputs (fractions.Fraction), rounded once to fp32;
      - the M20 exact-tail shapes (DevelopmentReport/SDSL_V_M20_EXACTTAIL_SGEMM.md)
        on Marionette inputs, exact;
      - the Gemma small-M corpus (internal/prometheus/gemma4e2b_sgemm_corpus_test.go:44-122):
        exact fp64 products summed with math.fsum (correctly rounded), then fp32.
  * Row reductions on deterministic_input and its constant / extreme /
    heterogeneous variants (internal/prometheus/native/Marionette/reactor_reduction_tests.cpp:77-114)
    at the planner boundary widths (:191-197): SUM exact (sixteenths), MAX exact,
    SOFTMAX with math.fsum denominators in binary64.
  * RMSNorm rows (canonical_contract.go:91-105 formula) in binary64 with fsum.

Run:  python tests/golden/make_golden.py   (takes well under a minute)
"""
from __future__ import annotations

import math
import sys
from fractions import Fraction
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
from oracle.oracle import (  # noqa: E402  (input generators only)
    deterministic_matrix, gemma_corpus_a, gemma_corpus_b, marionette_matrix, reduction_input)

STARTER = [(1, 1, 1), (4, 4, 4), (16, 16, 16), (32, 32, 32), (3, 5, 7)]
M20 = [(8, 8, 8), (16, 16, 16), (32, 32, 32), (17, 17, 17), (31, 29, 23), (64, 16, 64), (16, 64, 64), (64, 64, 8),
       (128, 128, 128)]
GEMMA = [(33, 256, 1536), (15, 2048, 1536), (17, 19, 17)]
WIDTHS = [1, 2, 3, 31, 32, 33, 63, 64, 65, 127, 128, 129, 255, 256, 257, 511, 512, 513, 1024, 4096]
DISTS = ["deterministic", "constant", "positive-extreme", "negative-extreme", "heterogeneous"]
RED_ROWS = 4


def exact_int_product(ai: np.ndarray, bi: np.ndarray, scale: int) -> np.ndarray:
    prod = ai.astype(np.int64) @ bi.astype(np.int64)
    return (prod.astype(np.float64) / scale).astype(np.float32)  # exact: |prod| < 2^53, scale a power of 2


def fraction_product(a: np.ndarray, b: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
    fa = [Fraction(float(v)) for v in a]
    fb = [Fraction(float(v)) for v in b]
    out = np.empty(m * n, dtype=np.float32)
    for r in range(m):
        for c in range(n):
            s = sum((fa[r * k + i] * fb[i * n + c] for i in range(k)), Fraction(0))
            out[r * n + c] = np.float32(float(s))  # float(Fraction) rounds correctly; then to fp32
    return out


def fsum_product(a: np.ndarray, b: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
    A = a.astype(np.float64).reshape(m, k)
    B = b.astype(np.float64).reshape(k, n)
    out = np.empty((m, n), dtype=np.float32)
    for r in range(m):
        prods = A[r][:, None] * B  # exact: fp32 x fp32 fits binary64
        for c in range(n):
            out[r, c] = np.float32(math.fsum(prods[:, c]))
    return out.ravel()


def main() -> None:
    g: dict[str, np.ndarray] = {}
    for m, n, k in STARTER:
        a, b = deterministic_matrix(m, k), deterministic_matrix(k, n)
        g[f"sgemm_starter_{m}x{n}x{k}"] = fraction_product(a, b, m, n, k)
    for sa, sb in [(3, 5), (19, 5)]:
        m, n, k = 37, 29, 13
        ai = ((np.arange(m * k) * 7 + sa) % 23 - 11).reshape(m, k)
        bi = ((np.arange(k * n) * 7 + sb) % 23 - 11).reshape(k, n)
        assert np.array_equal(ai / 8, marionette_matrix(m * k, sa).reshape(m, k))
        g[f"sgemm_marionette_{m}x{n}x{k}_s{sa}_s{sb}"] = exact_int_product(ai, bi, 64).ravel()
    for m, n, k in M20:
        ai = ((np.arange(m * k) * 7 + 3) % 23 - 11).reshape(m, k)
        bi = ((np.arange(k * n) * 7 + 5) % 23 - 11).reshape(k, n)
        g[f"sgemm_m20_{m}x{n}x{k}"] = exact_int_product(ai, bi, 64).ravel()
    for m, n, k in GEMMA:
        g[f"sgemm_gemma_{m}x{n}x{k}"] = fsum_product(gemma_corpus_a(m * k), gemma_corpus_b(k * n), m, n, k)

    for dist in DISTS:
        for w in WIDTHS:
            x = reduction_input(RED_ROWS, w, dist).astype(np.float64)
            g[f"red_sum_{dist}_{w}"] = np.array([np.float32(math.fsum(row)) for row in x], dtype=np.float32)
            g[f"red_max_{dist}_{w}"] = x.max(axis=1).astype(np.float32)
            mx = x.max(axis=1, keepdims=True)
            e = np.exp(x - mx)
            den = np.array([math.fsum(row) for row in e])[:, None]
            g[f"red_softmax_{dist}_{w}"] = (e / den).astype(np.float32).ravel()
    x = reduction_input(1024, 513).astype(np.float64)
    g["red_max_deterministic_rows1024_513"] = x.max(axis=1).astype(np.float32)

    for w in (256, 2048):
        x = reduction_input(8, w).astype(np.float32)
        wt = (np.float32(0.5) + ((np.arange(w) * 13) % 100).astype(np.float32) / np.float32(100.0)).astype(np.float32)
        xd = x.astype(np.float64)
        ss = np.array([math.fsum(r * r) for r in xd])
        inv = 1.0 / np.sqrt(ss / w + float(np.float32(1e-6)))
        g[f"rms_deterministic_{w}_out"] = (xd * inv[:, None] * wt.astype(np.float64)).astype(np.float32).ravel()
        g[f"rms_deterministic_{w}_inv"] = inv.astype(np.float32)
        g[f"rms_deterministic_{w}_weight"] = wt

    np.savez_compressed(HERE / "known_answers.npz", **g)
    total = sum(v.size for v in g.values())
    print(f"wrote {len(g)} arrays, {total} values -> {HERE / 'known_answers.npz'}")


if __name__ == "__main__":
    main()
