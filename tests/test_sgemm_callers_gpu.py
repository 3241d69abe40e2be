"""The SGEMM callers beside the path, on the B200.

Covers the reference entries `prometheus_reactor_runtime_sgemm_benchmark_variant`,
`..._sgemm_resident_benchmark` and `..._sgemm_batch` (reactor_api.h:2596-2615;
reactor_sgemm.cpp:5629-6009; reactor_batch.c:89-520).  Every product is checked
against the one-shot `prometheus_reactor_runtime_sgemm` bit for bit (same
kernel, same inputs), and that one against the binary64 oracle with the
SGEMM tolerance of the other parity tests (max relative error <= 1e-5).
"""
from __future__ import annotations

import numpy as np
import pytest

from oct_b200 import reactor as R

pytestmark = pytest.mark.gpu
REL_TOL = 1e-5


def _problem(m, n, k, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    a = rng.uniform(-1, 1, m * k).astype(np.float32)
    b = rng.uniform(-1, 1, k * n).astype(np.float32)
    return a, b


def _check_fp64(c, a, b, m, n, k):
    ref = a.astype(np.float64).reshape(m, k) @ b.astype(np.float64).reshape(k, n)
    err = np.max(np.abs(c.reshape(m, n) - ref)) / max(np.max(np.abs(ref)), 1e-20)
    assert err <= REL_TOL, err


VARIANTS = [R.SGEMM_AUTO, R.SGEMM_TC3XTF32, R.SGEMM_FMA, R.SGEMM_TC_BK16, R.SGEMM_TC_BK32, R.SGEMM_TC_PAIR16,
            R.SGEMM_TC_PAIR32]


@pytest.mark.parametrize("shape", [(300, 260, 170), (512, 512, 512)])
@pytest.mark.parametrize("variant", VARIANTS)
def test_benchmark_variant_runs_the_named_kernel(runtime, shape, variant):
    m, n, k = shape
    a, b = _problem(m, n, k, seed=m + variant)
    c, st = runtime.sgemm_variant(m, n, k, a, b, variant)
    assert st.ok and (st.stage, st.detail) == (R.STAGE_TRANSFER_OUT, 6101), st
    _check_fp64(c, a, b, m, n, k)
    if variant == R.SGEMM_AUTO:
        assert np.array_equal(c, runtime.sgemm(m, n, k, a, b))


def test_benchmark_variant_rejects_unknown_ids(runtime):
    a, b = _problem(8, 8, 8, seed=1)
    c, st = runtime.sgemm_variant(8, 8, 8, a, b, 7)
    assert c is None and (st.rc, st.stage, st.detail) == (R.PROM_ERROR, R.STAGE_INIT, R.DETAIL_BAD_VARIANT)


def test_resident_benchmark_serial(runtime):
    m = n = k = 1024
    a, b = _problem(m, n, k, seed=5)
    rc, res, c = runtime.resident_benchmark(m, n, k, a, b, iterations=4, warmup=2)
    assert rc == R.PROM_OK
    assert (res.setup_stage, res.setup_detail_code) == (R.STAGE_TRANSFER_OUT, 6101)
    assert (res.final_stage, res.final_detail_code) == (R.STAGE_SUBMIT, R.DETAIL_PATH_STAGED_UPLOAD_TILED)
    assert res.resident_mode_available == 1 and res.resident_mode_used == 1
    assert res.executed_variant == res.production_selected_variant == R.SGEMM_TC3XTF32
    assert res.requested_variant == 0 and res.iterations == 4 and res.queue_submissions == 4
    assert res.gpu_timestamp_valid == 1
    assert 0 < res.kernel_min_ns <= res.kernel_median_ns <= res.kernel_p95_ns
    assert res.upload_once_wall_ns > 0 and res.setup_wall_ns >= res.upload_once_wall_ns
    assert res.readback_once_wall_ns > 0 and res.total_loop_wall_ns > 0
    assert np.array_equal(c, runtime.sgemm(m, n, k, a, b))
    _check_fp64(c, a, b, m, n, k)


def test_resident_benchmark_explicit_variant_and_depth(runtime):
    m, n, k = 640, 384, 200
    a, b = _problem(m, n, k, seed=6)
    rc, res, c = runtime.resident_benchmark(m, n, k, a, b, iterations=3, warmup=0, variant=R.SGEMM_FMA, depth=2)
    assert rc == R.PROM_OK
    assert res.requested_variant == R.SGEMM_FMA and res.executed_variant == R.SGEMM_FMA
    assert res.executed_compute_mode == 2 and res.production_selected_variant == R.SGEMM_TC3XTF32
    assert res.iterations == 6 and res.diagnostic_batch_depth == 2
    ref, st = runtime.sgemm_variant(m, n, k, a, b, R.SGEMM_FMA)
    assert st.ok and np.array_equal(c, ref)


def test_resident_benchmark_submission_ring(runtime):
    m = n = k = 512
    a, b = _problem(m, n, k, seed=7)
    rc, res, c = runtime.resident_benchmark(m, n, k, a, b, iterations=7, warmup=2, depth=3, ring=True)
    assert rc == R.PROM_OK
    assert res.configured_ring_depth == 3 and res.physical_slot_count == 4 and res.max_in_flight_depth == 3
    assert res.iterations == 7 and res.ring_full_count == 4 and res.ring_slot_recycle_count == 4
    # the ring counters include the 2 warm-up products, as the reference's (reactor_sgemm.cpp:5788-5800)
    assert res.ring_query_harvest_count == 9 and list(res.ring_final_slot_state) == [0, 0, 0, 0]
    assert res.gpu_timestamp_valid == 1 and 0 < res.kernel_min_ns <= res.kernel_p95_ns
    assert np.array_equal(c, runtime.sgemm(m, n, k, a, b))
    rc, res, _ = runtime.resident_benchmark(m, n, k, a, b, iterations=2, depth=5, ring=True)
    assert (rc, res.final_stage, res.final_detail_code) == (R.PROM_ERROR, R.STAGE_SUBMIT, R.PROM_ERROR)


BATCH_SHAPES = [(17, 19, 23), (256, 300, 128), (1000, 1000, 1000), (64, 64, 8), (513, 257, 129), (2048, 512, 384),
                (1, 4096, 64)]


@pytest.mark.parametrize("flags", [0, 3, 8, 3 | R.BATCH_FLAG_PARTITION_CONTIGUOUS, 200])
def test_batch_matches_single_products(runtime, flags):
    problems = [(m, n, k, *_problem(m, n, k, seed=100 + i)) for i, (m, n, k) in enumerate(BATCH_SHAPES)]
    outs, st = runtime.sgemm_batch(problems, flags)
    assert st.ok and (st.stage, st.detail) == (R.STAGE_TRANSFER_OUT, 0), st
    for (m, n, k, a, b), c in zip(problems, outs):
        assert np.array_equal(c, runtime.sgemm(m, n, k, a, b)), (m, n, k)
        _check_fp64(c, a, b, m, n, k)


def test_batch_rejects_an_invalid_entry_without_touching_outputs(runtime):
    problems = [(m, n, k, *_problem(m, n, k, seed=i)) for i, (m, n, k) in enumerate(BATCH_SHAPES[:3])]
    entries = (R.PrometheusSgemmBatchEntry * 3)()
    outs = []
    for e, (m, n, k, a, b) in zip(entries, problems):
        c = np.full(m * n, np.nan, dtype=np.float32)
        outs.append(c)
        e.a, e.b, e.c, e.m, e.n, e.k = a.ctypes.data, b.ctypes.data, c.ctypes.data, m, n, k
    entries[1].k = 0
    import ctypes as C
    stage, detail = C.c_uint32(), C.c_int()
    rc = runtime.lib.prometheus_reactor_runtime_sgemm_batch(runtime.handle, entries, 3, 2, C.byref(stage),
                                                            C.byref(detail))
    assert (rc, stage.value, detail.value) == (R.PROM_ERROR, R.STAGE_INIT, R.DETAIL_BATCH_PLAN_INVALID)
    assert all(np.isnan(c).all() for c in outs)
