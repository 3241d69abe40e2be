"""FFT on a B200 through the C ABI.  fp64: bit-exact against the reference's
binary64 radix-2 network (oracle.c oracle_fft64) at every size up to 2^20, and
within the reference's 2e-12 * n of an independent DFT.  fp32: within 1e-5
normwise of the fp32 oracle and of a binary64 DFT (the reference's fp32 route
uses native shader cos / sin, so its exact bits are not defined)."""
from __future__ import annotations

import numpy as np
import pytest

from oct_b200 import reactor as R

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("log2n", [0, 1, 3, 5, 7, 10, 11, 12, 14, 17, 20])
def test_fft64_is_bit_exact_with_the_reference_network(runtime, oracle_mod, log2n):
    n = 1 << log2n
    rng = np.random.Generator(np.random.PCG64(log2n))
    x = rng.standard_normal(n) + 1j * rng.standard_normal(n)
    y, st = runtime.fft64(x)
    assert st.ok and (st.stage, st.detail) == (R.STAGE_TRANSFER_OUT, 0), st
    want, _ = oracle_mod.fft64(x)
    assert np.array_equal(y.view(np.uint64), want.view(np.uint64))
    assert np.max(np.abs(y - np.fft.fft(x))) <= 2e-12 * n * max(1.0, np.sqrt(n) / 32)


def test_fft64_reference_cases(runtime, oracle_mod):
    """reactor_fft64_tests.cpp:15-94: low-bit inputs, impulse, binary64 dynamic range."""
    for n in (1, 2, 8, 32, 128):
        i = np.arange(n)
        x = (1.0 + np.ldexp(i + 1.0, -35)) + 1j * (np.sin(i.astype(np.float64)) + np.ldexp(1.0, -40))
        keep = x.copy()
        y, st = runtime.fft64(x)
        assert st.ok and np.array_equal(x, keep)  # the input stays unchanged
        assert np.max(np.abs(y - np.fft.fft(x))) <= 2e-12 * n
    impulse = np.zeros(64, np.complex128)
    impulse[0] = 1
    y, st = runtime.fft64(impulse)
    assert st.ok and np.all(y == 1.0)
    for scale in (1e-200, 1e200):
        x = np.array([1 - 1j, 2 + 1j, -1 + 0j, 0 + 2j]) * scale
        y, st = runtime.fft64(x)
        assert st.ok and np.max(np.abs(y / scale - np.fft.fft(x / scale))) <= 1e-12


def test_fft64_injected_failures_leave_the_output_untouched(lib):
    """reactor_fft64_tests.cpp:59-76: no CPU fallback and no partial output."""
    for flag in (R.TESTCFG_FAIL_BUFFER_ALLOC, R.TESTCFG_FAIL_UPLOAD, R.TESTCFG_FAIL_DISPATCH,
                 R.TESTCFG_FAIL_DOWNLOAD):
        rt = R.Runtime(lib, test_flags=flag)
        try:
            out = np.array([91 + 92j, 93 + 94j])
            y, st = rt.fft64(np.array([1 + 0j, 2 + 0j]), out=out)
            assert not st.ok and st.detail != 0
            assert out[0] == 91 + 92j and out[1] == 93 + 94j
        finally:
            rt.close()


def test_fft32_known_answers_and_diagnostics(runtime):
    """reactor_fft_api_tests.cpp:198-233."""
    y, st = runtime.fft(np.array([1, 2], np.complex64), 2)
    assert st.ok and (st.stage, st.detail) == (R.STAGE_TRANSFER_OUT, 0)
    assert abs(y[0] - 3) <= 1e-5 and abs(y[1] + 1) <= 1e-5
    d = runtime.fft_diagnostics()
    assert (d.last_element_count, d.last_batch_count, d.plan_valid, d.plan_pass_count) == (2, 1, 1, 1)
    assert (d.plan_first_span, d.plan_last_span, d.executed_path_id) == (2, 2, R.FFT_PATH_RADIX2)
    assert (d.capability_reported, d.production_enabled) == (1, 1)
    y, st = runtime.fft(np.array([1, 2, 3, 4], np.complex64), 4)
    assert st.ok and np.max(np.abs(y - np.array([10, -2 + 2j, -2, -2 - 2j]))) <= 2e-5


@pytest.mark.parametrize("n,batch,stride", [(8, 3, 0), (4096, 4, 4100), (8192, 2, 0), (1 << 20, 2, 0),
                                            (1 << 16, 5, (1 << 16) + 3)])
def test_fft32_batched_forward_and_inverse(runtime, oracle_mod, n, batch, stride):
    s = stride or n
    rng = np.random.Generator(np.random.PCG64(n + batch))
    x = (rng.standard_normal(s * batch) + 1j * rng.standard_normal(s * batch)).astype(np.complex64)
    fill = np.complex64(7 - 7j)
    out = np.full_like(x, fill)
    y, st = runtime.fft(x, n, batch, stride, R.FFT_FLAG_FORWARD, out=out)
    assert st.ok, st
    want = oracle_mod.fft32(x, n, batch, s)
    for b in range(batch):
        seg = slice(b * s, b * s + n)
        ref64 = np.fft.fft(x[seg].astype(np.complex128))
        scale = np.max(np.abs(ref64))
        assert np.max(np.abs(y[seg] - want[seg])) <= 1e-5 * scale
        assert np.max(np.abs(y[seg] - ref64)) <= 1e-5 * scale
        assert np.all(y[b * s + n:(b + 1) * s] == fill)  # nothing written between batches
    back, st = runtime.fft(y, n, batch, stride, R.FFT_FLAG_INVERSE | R.FFT_FLAG_INVERSE_NORMALIZE)
    assert st.ok
    for b in range(batch):
        seg = slice(b * s, b * s + n)
        assert np.max(np.abs(back[seg] - x[seg])) <= 1e-5 * np.max(np.abs(x[seg]))
