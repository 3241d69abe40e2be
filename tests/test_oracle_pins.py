"""Pins the CPU oracle to known answers before any GPU result is trusted.

The known answers (tests/golden/known_answers.npz, made by make_golden.py with
exact or correctly-rounded arithmetic) come from the reference's own test
inputs.  If the oracle's restatement of Oct's CPU code drifted, these fail.
"""
from __future__ import annotations

import numpy as np
import pytest

from tests.golden.make_golden import DISTS, GEMMA, M20, STARTER, WIDTHS, RED_ROWS


def test_marionette_product_is_exact(oracle_mod, golden):
    o = oracle_mod
    for sa, sb in [(3, 5), (19, 5)]:
        m, n, k = 37, 29, 13
        a, b = o.marionette_matrix(m * k, sa), o.marionette_matrix(k * n, sb)
        want = golden[f"sgemm_marionette_{m}x{n}x{k}_s{sa}_s{sb}"]
        # Every partial sum is a small multiple of 1/64: fp32 and fp64 are exact.
        assert np.array_equal(o.cpu_sgemm_f32(a, b, m, n, k), want)
        assert np.array_equal(o.sgemm_f64(a, b, m, n, k).astype(np.float32), want)


@pytest.mark.parametrize("shape", M20)
def test_m20_exact_tail_shapes_exact(oracle_mod, golden, shape):
    o = oracle_mod
    m, n, k = shape
    a, b = o.marionette_matrix(m * k, 3), o.marionette_matrix(k * n, 5)
    assert np.array_equal(o.cpu_sgemm_f32(a, b, m, n, k), golden[f"sgemm_m20_{m}x{n}x{k}"])


@pytest.mark.parametrize("shape", STARTER)
def test_starter_corpus_within_reference_gate(oracle_mod, golden, shape):
    o = oracle_mod
    m, n, k = shape
    a, b = o.deterministic_matrix(m, k), o.deterministic_matrix(k, n)
    want = golden[f"sgemm_starter_{m}x{n}x{k}"]
    res = o.compare_against_oracle(want, o.cpu_sgemm_f32(a, b, m, n, k))
    assert res.pass_ == 1, (res.max_abs_error, res.max_rel_error)
    # the fp64 oracle rounds to the exact answer
    got64 = o.sgemm_f64(a, b, m, n, k)
    assert np.max(np.abs(got64.astype(np.float32) - want)) <= np.max(np.abs(want)) * 2 ** -23


@pytest.mark.parametrize("shape", GEMMA)
def test_gemma_small_m_corpus(oracle_mod, golden, shape):
    o = oracle_mod
    m, n, k = shape
    a, b = o.gemma_corpus_a(m * k), o.gemma_corpus_b(k * n)
    want = golden[f"sgemm_gemma_{m}x{n}x{k}"]
    got = o.cpu_sgemm_f32(a, b, m, n, k)
    assert o.compare_against_oracle(want, got).pass_ == 1
    got64 = o.sgemm_f64(a, b, m, n, k).astype(np.float32)
    assert np.max(np.abs(got64 - want) / np.maximum(np.abs(want), 1e-6)) <= 2 ** -23


def test_oct_compiled_matmul_f64_matches_exact(oracle_mod, golden):
    o = oracle_mod
    m, n, k = 31, 29, 23
    a, b = o.marionette_matrix(m * k, 3), o.marionette_matrix(k * n, 5)
    got = o.oct_matmul_f64(a.astype(np.float64), b.astype(np.float64), m, n, k)
    assert np.array_equal(got.astype(np.float32), golden["sgemm_m20_31x29x23"])


@pytest.mark.parametrize("dist", DISTS)
def test_reduction_oracle_pins(oracle_mod, golden, dist):
    o = oracle_mod
    for w in WIDTHS:
        x = o.reduction_input(RED_ROWS, w, dist)
        for op, name in ((1, "sum"), (2, "max")):
            rc, got = o.reduction_cpu_reference(x, op)
            assert rc == 0
            assert np.array_equal(got, golden[f"red_{name}_{dist}_{w}"]), (name, w)
        rc, got = o.reduction_cpu_reference(x, 3)
        want = golden[f"red_softmax_{dist}_{w}"]
        assert rc == 0
        assert np.max(np.abs(got - want) / np.maximum(want, 1e-30)) <= 4 * 2 ** -24, w
        assert o.reduction_compare(RED_ROWS, w, 3, want, got)[0] == 0


def test_reduction_oracle_rejects_nonfinite(oracle_mod):
    o = oracle_mod
    x = o.reduction_input(3, 65)
    x[2, 7] = np.nan
    assert o.find_nonfinite(x) == 2 * 65 + 7
    assert o.reduction_cpu_reference(x, 1)[0] == -6814


def test_reduction_compare_catches_planted_mistakes(oracle_mod):
    """Plants an error in an oracle output (on the CPU) and checks the gate trips."""
    o = oracle_mod
    x = o.reduction_input(4, 257)
    _, mx = o.reduction_cpu_reference(x, 2)
    bad = mx.copy()
    bad[3] = np.nextafter(bad[3], np.float32(np.inf))  # MAX must be exact
    rc, mm = o.reduction_compare(4, 257, 2, mx, bad)
    assert rc == 1 and mm.row == 3
    _, sm = o.reduction_cpu_reference(x, 3)
    bad = sm.copy().reshape(4, 257)
    bad[1] *= np.float32(1.001)  # within per-element tolerance but breaks the row sum
    rc, mm = o.reduction_compare(4, 257, 3, sm, bad.ravel())
    assert rc == 1 and mm.row == 1


def test_compare_against_oracle_semantics(oracle_mod):
    o = oracle_mod
    e = np.array([1.0, 0.0, 100.0, 2.0], dtype=np.float32)
    a = e.copy()
    a[2] = 100.005  # abs 5e-3 > 1e-4 but rel 5e-5 <= 1e-4: passes
    assert o.compare_against_oracle(e, a).pass_ == 1
    a[3] = 2.001  # abs 1e-3 and rel 5e-4 both over: fails
    res = o.compare_against_oracle(e, a)
    assert res.pass_ == 0 and res.first_failing_index == 3 and res.failing_count == 1
    a[1] = np.inf
    assert o.compare_against_oracle(e, a).failing_count == 2


@pytest.mark.parametrize("w", [256, 2048])
def test_rmsnorm_oracle_pins(oracle_mod, golden, w):
    o = oracle_mod
    x = o.reduction_input(8, w)
    wt = golden[f"rms_deterministic_{w}_weight"]
    out64, inv64 = o.rmsnorm_f64(x, wt, 1e-6)
    want = golden[f"rms_deterministic_{w}_out"]
    got64 = out64.astype(np.float32).ravel()
    assert np.max(np.abs(got64 - want) / np.maximum(np.abs(want), 1e-6)) <= 2 ** -22
    assert np.max(np.abs(inv64.astype(np.float32) - golden[f"rms_deterministic_{w}_inv"])) <= 2 ** -22
    out32, inv32 = o.rmsnorm_f32(x, wt, 1e-6)
    assert np.max(np.abs(out32.ravel() - want) / np.maximum(np.abs(want), 1e-3)) <= 1e-5


def test_multithreaded_oracle_matches_serial(oracle_mod):
    o = oracle_mod
    m, n, k = 67, 45, 33
    a, b = o.uniform_matrix(m, k, 1).ravel(), o.uniform_matrix(k, n, 2).ravel()
    assert np.array_equal(o.cpu_sgemm_f32(a, b, m, n, k), o.cpu_sgemm_f32(a, b, m, n, k, threads=4))
    x = o.normal_matrix(40, 300, 3)
    for op in (1, 2, 3):
        assert np.array_equal(o.reduction_cpu_reference(x, op, 1)[1], o.reduction_cpu_reference(x, op, 4)[1])


def _go_rmsnorm_f32(x, w, eps, canonical):
    """Direct numpy float32 transcription of the two Go loops, for pinning the C oracle."""
    out = np.empty_like(x)
    for r in range(x.shape[0]):
        acc = np.float32(0.0)
        for v in x[r]:
            acc = np.float32(acc + np.float32(v * v))
        m = np.float32(acc / np.float32(x.shape[1])) + np.float32(eps)
        m = np.float32(m)
        if canonical:
            scale = np.float32(np.float32(1.0) / np.float32(np.sqrt(np.float64(m))))
        else:
            scale = np.float32(1.0 / np.sqrt(np.float64(m)))
        out[r] = (x[r] * scale).astype(np.float32) * w
    return out


@pytest.mark.parametrize("form", ["head", "canonical"])
def test_rmsnorm_fp32_forms_follow_the_go_loops_bit_for_bit(oracle_mod, form):
    """cpuHeadRMSNorm rounds 1/sqrt once from binary64; CanonicalRMSNorm rounds the square
    root to fp32 and divides in fp32.  The C oracle reproduces each exactly."""
    o = oracle_mod
    x = o.normal_matrix(24, 300, 41)
    w = (o.uniform_matrix(1, 300, 42).ravel() + np.float32(1.0)).astype(np.float32)
    got, _ = o.rmsnorm_f32(x, w, 1e-5, form=form)
    assert np.array_equal(got, _go_rmsnorm_f32(x, w, 1e-5, form == "canonical"))
