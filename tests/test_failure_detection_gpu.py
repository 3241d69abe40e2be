"""Failure detection on the B200, without a GPU fault.

Every spin-wait in the library's kernels is bounded by a wall-clock budget; when
it runs out the kernel sets an error bit in a device status word, stops waiting
and returns, so the context stays usable and the host reports
OCT_B200_DETAIL_DEVICE_TIMEOUT.  Here the tensor-parallel peer-wait kernel is
pointed at a flag that nothing sets (the situation of a rank that never
arrives), with a short budget.
"""
from __future__ import annotations

import time

import numpy as np
import pytest

from oct_b200 import reactor as R

pytestmark = pytest.mark.gpu


def test_peer_wait_gives_up_and_reports_timeout(runtime):
    t0 = time.perf_counter()
    st = runtime.selftest_wait_timeout(50_000_000)  # 50 ms
    dt = time.perf_counter() - t0
    assert (st.rc, st.detail) == (R.PROM_ERROR, R.DETAIL_DEVICE_TIMEOUT), st
    assert 0.04 <= dt < 5.0, dt
    # the status word was read and cleared, and the context still computes
    assert runtime.sync_status().ok
    a = np.arange(64, dtype=np.float32) / 8
    c = runtime.sgemm(8, 8, 8, a, a)
    ref = a.reshape(8, 8).astype(np.float64) @ a.reshape(8, 8).astype(np.float64)
    assert np.array_equal(c.reshape(8, 8), ref.astype(np.float32))


def test_wait_budget_is_validated(runtime):
    st = runtime.selftest_wait_timeout(10)
    assert st.rc == R.PROM_ERROR and st.detail == R.DETAIL_INVALID_ARGUMENT
