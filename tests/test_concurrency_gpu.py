"""Several host threads calling one handle at once (the reference requires thread
safety per handle: prom_reactor_runtime_validate_handle, reactor_sgemm.cpp:1370-1388,
and the per-executor mutexes of reactor_concept_reduction.cpp:15-20).  Go calls the
library from any goroutine, so calls on one handle may overlap.  Every result is
checked against the CPU oracle."""
from __future__ import annotations

import threading
import time

import numpy as np
import pytest

from oct_b200 import reactor as R

pytestmark = pytest.mark.gpu


def test_threads_share_one_handle(lib, oracle_mod):
    o = oracle_mod
    rt = R.Runtime(lib)
    errors: list[str] = []
    lock = threading.Lock()

    def fail(msg):
        with lock:
            errors.append(msg)

    def sgemm_worker(tid):
        for it in range(6):
            m, n, k = 96 + 37 * tid + it, 130 + 11 * it, 77 + 5 * tid
            a, b = o.uniform_matrix(m, k, 100 * tid + it).ravel(), o.uniform_matrix(k, n, 100 * tid + it + 50).ravel()
            c, st = rt.sgemm_with_status(m, n, k, a, b)
            if not st.ok:
                fail(f"sgemm {tid}/{it}: {st}")
                continue
            ref = o.sgemm_f64(a, b, m, n, k)
            if np.max(np.abs(c - ref)) > 1e-5 * np.max(np.abs(ref)):
                fail(f"sgemm {tid}/{it} mismatch")

    def reduction_worker(tid):
        for it in range(6):
            op = (R.OP_SUM, R.OP_MAX, R.OP_SOFTMAX)[(tid + it) % 3]
            rows, width = 200 + 13 * it, 300 + 64 * tid
            x = o.normal_matrix(rows, width, 1000 * tid + it)
            y, res = rt.reduction(x, op)
            if y is None:
                fail(f"reduction {tid}/{it}: detail {res.detail_code}")
                continue
            _, ref = o.reduction_cpu_reference(x, op)
            if o.reduction_compare(rows, width, op, ref, y)[0] != 0:
                fail(f"reduction {tid}/{it} mismatch")

    def async_worker(tid):
        for it in range(4):
            m, n, k = 128 + 16 * tid, 192, 160 + it
            a, b = o.uniform_matrix(m, k, 7 * tid + it).ravel(), o.uniform_matrix(k, n, 7 * tid + it + 9).ravel()
            deadline = time.time() + 60
            while True:
                task, st = rt.submit_async(m, n, k, a, b)
                if st.ok:
                    break
                if st.detail != R.DETAIL_ASYNC_QUEUE_FULL or time.time() > deadline:
                    fail(f"async submit {tid}/{it}: {st}")
                    return
                time.sleep(0.002)  # the four task slots are shared by every thread
            while rt.query_async(task)[1].ready != 1:
                if time.time() > deadline:
                    fail(f"async {tid}/{it} never ready")
                    return
                time.sleep(0.001)
            c = np.empty(m * n, np.float32)
            st = rt.consume_async(task, c)
            rt.abandon_async(task)
            if not st.ok:
                fail(f"async consume {tid}/{it}: {st}")
                continue
            ref = o.sgemm_f64(a, b, m, n, k)
            if np.max(np.abs(c - ref)) > 1e-5 * np.max(np.abs(ref)):
                fail(f"async {tid}/{it} mismatch")

    threads = [threading.Thread(target=w, args=(t,)) for t in range(3)
               for w in (sgemm_worker, reduction_worker, async_worker)]
    try:
        for th in threads:
            th.start()
        for th in threads:
            th.join(timeout=300)
        assert not any(th.is_alive() for th in threads)
        assert not errors, errors
    finally:
        rt.close()
