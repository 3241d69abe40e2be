"""Reduction diagnostics / benchmark and async SGEMM diagnostics on a B200.

reactor_vulkan_fused_reduction.c:1122-1206 (benchmark: warm-up, measured runs,
correctness of the last output), reactor_concept_reduction.cpp:96-110 and
reactor_sgemm.cpp:6371-6412 (diagnostics)."""
from __future__ import annotations

import ctypes as C
import time

import numpy as np
import pytest

from oct_b200 import reactor as R

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("op", [R.OP_SUM, R.OP_MAX, R.OP_SOFTMAX])
@pytest.mark.parametrize("rows,width", [(1024, 4096), (32768, 256)])
def test_reduction_benchmark_and_diagnostics(lib, oracle_mod, op, rows, width):
    rt = R.Runtime(lib)
    try:
        x = oracle_mod.normal_matrix(rows, width, seed=rows + width + op)
        y = np.empty(rows * width if op == R.OP_SOFTMAX else rows, np.float32)
        before = R.PrometheusReductionDiagnostics()
        assert lib.prometheus_reactor_runtime_reduction_diagnostics(rt.handle, C.byref(before)) == R.PROM_OK
        req = R.PrometheusReductionBenchmarkRequest()
        req.struct_size = C.sizeof(req)
        req.reduction = R.make_reduction_request(x, y, rows, width, op)
        req.warmup_iterations, req.measured_iterations = 2, 5
        res = R.PrometheusReductionBenchmarkResult()
        rc = lib.prometheus_reactor_runtime_reduction_benchmark(rt.handle, C.byref(req), C.byref(res))
        assert rc == R.PROM_OK, res.detail_code
        assert (res.completed_iterations, res.correctness_passed, res.validation_passed) == (5, 1, 1)
        assert 0 < res.gpu_min_ns <= res.gpu_median_ns <= res.gpu_max_ns
        assert res.gpu_median_ns <= res.end_to_end_median_ns
        rc_plan, plan = R.reduction_plan(lib, rows, width, op)
        assert rc_plan == R.PROM_OK and res.replay_id == plan.replay_id and res.stage_count == plan.stage_count
        # the caller's output is the last measured execution's, and it matches the oracle
        _, ref = oracle_mod.reduction_cpu_reference(x, op)
        assert oracle_mod.reduction_compare(rows, width, op, ref, y)[0] == 0
        after = R.PrometheusReductionDiagnostics()
        assert lib.prometheus_reactor_runtime_reduction_diagnostics(rt.handle, C.byref(after)) == R.PROM_OK
        assert after.initialized == 1
        assert after.total_requests - before.total_requests == 7
        assert after.successful_requests - before.successful_requests == 7
        assert after.last_replay_id == plan.replay_id and after.last_detail_code == 0
        assert after.queue_submit_count - before.queue_submit_count == 7
    finally:
        rt.close()


def test_async_diagnostics_follow_the_task_lifecycle(lib, oracle_mod):
    rt = R.Runtime(lib)
    try:
        m = n = k = 512
        a, b = oracle_mod.uniform_matrix(m, k, 1).ravel(), oracle_mod.uniform_matrix(k, n, 2).ravel()
        ids = []
        for _ in range(4):
            tid, st = rt.submit_async(m, n, k, a, b)
            assert st.ok
            ids.append(tid)
        _, st = rt.submit_async(m, n, k, a, b)
        assert not st.ok and st.detail == R.DETAIL_ASYNC_QUEUE_FULL
        for tid in ids:
            deadline = time.time() + 30
            while rt.query_async(tid)[1].ready != 1:
                assert time.time() < deadline
                time.sleep(0.001)
        c = np.empty(m * n, np.float32)
        assert rt.consume_async(ids[0], c).ok
        assert rt.abandon_async(ids[1]) == R.PROM_OK  # released before it was consumed
        assert rt.consume_async(9999, c).detail == R.DETAIL_ASYNC_INVALID_TASK
        d = R.PrometheusSgemmAsyncDiagnostics()
        assert lib.prometheus_reactor_runtime_sgemm_async_diagnostics(rt.handle, C.byref(d)) == R.PROM_OK
        assert (d.task_capacity, d.active_task_count, d.ready_count, d.consumed_count) == (4, 3, 2, 1)
        assert d.queue_full_count == 1 and d.stale_id_rejection_count >= 1 and d.max_in_flight >= 1
        live = [t for t in d.tasks if t.task_id in ids]
        assert len(live) == 3 and all(t.timing_valid == 1 and t.gpu_duration_ns > 0 for t in live)
        assert sorted(t.submission_sequence for t in live) == sorted(set(t.submission_sequence for t in live))
        ref64 = oracle_mod.sgemm_f64(a, b, m, n, k)
        assert np.max(np.abs(c - ref64)) <= 1e-5 * np.max(np.abs(ref64))
    finally:
        rt.close()
