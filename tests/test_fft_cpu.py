"""FFT on CPU: the oracle pinned to the reference's known answers and an
independent DFT, and the entry points' validation without a device
(internal/prometheus/native/Marionette/reactor_fft_api_tests.cpp:127-236,
reactor_fft64_tests.cpp:15-94; reactor_vulkan_fft.c:59-86)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from oct_b200 import reactor as R


def test_fft32_oracle_known_answers(oracle_mod):
    """reactor_fft_api_tests.cpp:198-233: [1, 2] -> [3, -1]; [1, 2, 3, 4] -> [10, -2+2i, -2, -2-2i]."""
    o = oracle_mod
    y = o.fft32(np.array([1, 2], np.complex64), 2)
    assert abs(y[0] - 3) <= 1e-5 and abs(y[1] + 1) <= 1e-5
    y = o.fft32(np.array([1, 2, 3, 4], np.complex64), 4)
    want = np.array([10, -2 + 2j, -2, -2 - 2j])
    assert np.max(np.abs(y - want)) <= 2e-5


@pytest.mark.parametrize("n", [1, 2, 8, 32, 128, 4096])
def test_fft64_oracle_against_an_independent_dft(oracle_mod, n):
    """reactor_fft64_tests.cpp:15-42: inputs with low bits an fp32 conversion would lose;
    the binary64 network stays within 2e-12 * n of a long-double DFT (numpy's for large n)."""
    i = np.arange(n)
    x = (1.0 + np.ldexp(i + 1.0, -35)) + 1j * (np.sin(i.astype(np.float64)) + np.ldexp(1.0, -40))
    y, tw = oracle_mod.fft64(x)
    if n <= 128:
        k = np.arange(n, dtype=np.longdouble)
        ang = -2.0 * np.pi * np.outer(k, k).astype(np.longdouble) / n
        want = (np.cos(ang) * x.real - np.sin(ang) * x.imag).sum(axis=1) + 1j * (
            np.cos(ang) * x.imag + np.sin(ang) * x.real).sum(axis=1)
        want = want.astype(np.complex128)
    else:
        want = np.fft.fft(x)
    assert np.max(np.abs(y - want)) <= 2e-12 * n
    if n >= 2:
        assert tw[0] == 1.0 and tw[1] == 0.0  # i = 0: cos 0, sin -0


def test_fft64_oracle_keeps_binary64_dynamic_range(oracle_mod):
    """reactor_fft64_tests.cpp:77-94."""
    for scale in (1e-200, 1e200):
        x = np.array([1 - 1j, 2 + 1j, -1 + 0j, 0 + 2j]) * scale
        y, _ = oracle_mod.fft64(x)
        assert np.max(np.abs(y / scale - np.fft.fft(x / scale))) <= 1e-12


def test_fft32_oracle_inverse_round_trip(oracle_mod):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(3 * 300) + 1j * rng.standard_normal(3 * 300)).astype(np.complex64)
    y = oracle_mod.fft32(x, 256, batch=3, stride=300)
    back = oracle_mod.fft32(y, 256, batch=3, stride=300, inverse=True, normalize=True)
    for b in range(3):
        seg = slice(300 * b, 300 * b + 256)
        assert np.max(np.abs(back[seg] - x[seg])) <= 1e-5 * np.max(np.abs(x))


@pytest.fixture()
def nodev(lib):
    cfg = R.PrometheusReactorConfig()
    cfg.struct_size = C.sizeof(cfg)
    cfg.test_flags = R.TESTCFG_FAIL_DEVICE_CREATE
    h = C.c_void_p()
    assert lib.prometheus_reactor_runtime_create(C.byref(cfg), C.byref(h)) == R.PROM_OK
    yield h
    lib.prometheus_reactor_runtime_destroy(h)


def test_fft_validation_order_and_diagnostics(lib, nodev):
    x = np.zeros(8, np.complex64)
    y = np.zeros(8, np.complex64)
    st, d = C.c_uint32(), C.c_int()

    def run(**over):
        req = R.PrometheusFftRequest()
        req.struct_size = C.sizeof(req)
        req.input, req.output, req.element_count, req.batch_count = x.ctypes.data, y.ctypes.data, 8, 1
        for k, v in over.items():
            setattr(req, k, v)
        rc = lib.prometheus_reactor_runtime_fft(nodev, C.byref(req), C.byref(st), C.byref(d))
        return rc, d.value

    diag = R.PrometheusFftDiagnostics()
    assert lib.prometheus_reactor_runtime_fft_diagnostics(nodev, C.byref(diag)) == R.PROM_OK
    assert (diag.api_declared, diag.capability_reported, diag.production_enabled, diag.executed_path_id) == (
        1, 0, 0, R.FFT_PATH_UNAVAILABLE)  # reactor_fft_api_tests.cpp:127-141
    assert run(struct_size=4) == (R.PROM_ERROR, -6702)
    assert run(input=None) == (R.PROM_ERROR, -6703)
    assert run(output=None) == (R.PROM_ERROR, -6704)
    assert run(element_count=0) == (R.PROM_ERROR, -6705)
    assert run(element_count=6) == (R.PROM_ERROR, -6706)
    assert run(element_count=1 << 21) == (R.PROM_ERROR, -6713)
    assert run(batch_count=0) == (R.PROM_ERROR, -6710)
    assert run(flags=3) == (R.PROM_ERROR, -6707)
    assert run(flags=4) == (R.PROM_ERROR, -6711)
    assert run(stride_elements=4) == (R.PROM_ERROR, -6708)
    assert run(element_count=512, batch_count=32768) == (R.PROM_ERROR, -6713)  # past the dispatch envelope
    assert run() == (R.PROM_ERROR, -6712)  # a valid request on a handle without a device
    assert lib.prometheus_reactor_runtime_fft_diagnostics(nodev, C.byref(diag)) == R.PROM_OK
    assert (diag.plan_valid, diag.plan_pass_count, diag.plan_first_span, diag.plan_last_span) == (1, 3, 2, 8)
    assert diag.last_failure_detail == -6712 and diag.last_element_count == 8
    req = R.PrometheusFftRequest()
    req.struct_size = C.sizeof(req)
    assert lib.prometheus_reactor_runtime_fft_benchmark_variant(nodev, C.byref(req), 1, C.byref(st),
                                                               C.byref(d)) == R.PROM_ERROR
    assert d.value == -6719
    a = np.zeros(8)
    assert lib.prometheus_reactor_runtime_fft64(None, a.ctypes.data, a.ctypes.data, 4, C.byref(st),
                                                C.byref(d)) == R.PROM_INVALID_HANDLE
    assert lib.prometheus_reactor_runtime_fft64(nodev, a.ctypes.data, a.ctypes.data, 3, C.byref(st),
                                                C.byref(d)) == R.PROM_ERROR and d.value == -6702
    assert lib.prometheus_reactor_runtime_fft64(nodev, a.ctypes.data, a.ctypes.data, 4, C.byref(st),
                                                C.byref(d)) == R.PROM_ERROR and d.value == -6712
    assert lib.prometheus_reactor_runtime_fft_diagnostics_sized(nodev, C.byref(diag), 0) == R.PROM_ERROR
