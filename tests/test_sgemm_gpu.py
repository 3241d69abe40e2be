"""SGEMM parity on the B200 through the C ABI, against the CPU oracle and the
exact known answers of the reference's own test matrices.

Tolerances (written here, applied to every case):
  * Oct's own gate compareAgainstOracle (runtime.go:12-15, 339-383): an element
    fails when BOTH |err| > 1e-4 and rel > 1e-4 versus cpuSGEMM.
  * "max relative error <= 1e-5 versus an fp64 oracle", measured
    normwise: max|C - C64| / max|C64| <= 1e-5 (elementwise relative error is
    unbounded where cancellation drives an output to ~0, for any fp32 method).
  * No worse than Oct's own fp32 CPU path: max|C - C64| <= 2 * max|cpuSGEMM - C64|
    plus one ulp of the largest output.
Inputs whose products are exact in fp32 (Marionette / M20 matrices) must come
back bit-exact from every kernel variant.
"""
from __future__ import annotations

import numpy as np
import pytest

from oct_b200 import reactor as R
from tests.golden.make_golden import GEMMA, M20, STARTER

pytestmark = pytest.mark.gpu

VARIANTS = [R.SGEMM_FMA, R.SGEMM_TC_BK16, R.SGEMM_TC_BK32, R.SGEMM_TC_PAIR16, R.SGEMM_TC_PAIR32, R.SGEMM_TC_INSM16,
            R.SGEMM_TC_INSM32]
NORMWISE_TOL = 1e-5


def device_sgemm(rt, a: np.ndarray, b: np.ndarray, m: int, n: int, k: int, variant: int) -> np.ndarray:
    import torch
    da = torch.from_numpy(a.reshape(m, k)).cuda()
    db = torch.from_numpy(b.reshape(k, n)).cuda()
    dc = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()
    rt.sgemm_device(da, db, dc, m, n, k, variant)
    st = rt.sync_status()
    assert st.ok, st
    return dc.cpu().numpy().ravel()


def normwise(c: np.ndarray, ref64: np.ndarray) -> float:
    return float(np.max(np.abs(c.astype(np.float64) - ref64)) / max(np.max(np.abs(ref64)), 1e-30))


@pytest.mark.parametrize("shape", STARTER)
def test_starter_corpus_host_abi(runtime, oracle_mod, golden, shape):
    """RunStarterCorpus (runtime.go:91-104) through prometheus_reactor_runtime_sgemm."""
    o = oracle_mod
    m, n, k = shape
    a, b = o.deterministic_matrix(m, k), o.deterministic_matrix(k, n)
    c, st = runtime.sgemm_with_status(m, n, k, a, b)
    assert st.ok and st.stage == R.STAGE_TRANSFER_OUT and st.detail == R.DETAIL_PATH_DIRECT
    assert o.compare_against_oracle(o.cpu_sgemm_f32(a, b, m, n, k), c).pass_ == 1
    assert o.compare_against_oracle(golden[f"sgemm_starter_{m}x{n}x{k}"], c).pass_ == 1


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("shape", STARTER + M20 + [(37, 29, 13)])
def test_exact_inputs_bit_exact(runtime, oracle_mod, golden, shape, variant):
    o = oracle_mod
    m, n, k = shape
    a, b = o.marionette_matrix(m * k, 3), o.marionette_matrix(k * n, 5)
    c = device_sgemm(runtime, a, b, m, n, k, variant)
    want = golden[f"sgemm_m20_{m}x{n}x{k}"] if f"sgemm_m20_{m}x{n}x{k}" in golden else o.cpu_sgemm_f32(a, b, m, n, k)
    assert np.array_equal(c, want)


def test_marionette_async_pair(runtime, oracle_mod, golden):
    """reactor_concept_sgemm_tests.cpp:29-87: two independent async products, inputs unmodified."""
    o = oracle_mod
    m, n, k = 37, 29, 13
    a, b, other = o.marionette_matrix(m * k, 3), o.marionette_matrix(k * n, 5), o.marionette_matrix(m * k, 19)
    a0, b0 = a.copy(), b.copy()
    t0, s0 = runtime.submit_async(m, n, k, a, b)
    t1, s1 = runtime.submit_async(m, n, k, other, b)
    assert s0.ok and s1.ok and t0 != t1
    for task, key in ((t0, "s3_s5"), (t1, "s19_s5")):
        for _ in range(2000):  # ValidateAsyncSGEMMOnHardware polls at most 2000 times (runtime.go:620)
            rc, qs = runtime.query_async(task)
            assert rc == R.PROM_OK
            if qs.lifecycle_state != R.ASYNC_SUBMITTED:
                break
            import time
            time.sleep(0.001)
        assert qs.lifecycle_state == R.ASYNC_READY and qs.ready == 1
        c = np.empty(m * n, dtype=np.float32)
        st = runtime.consume_async(task, c)
        assert st.ok and st.detail == R.DETAIL_PATH_DIRECT
        assert np.array_equal(c, golden[f"sgemm_marionette_{m}x{n}x{k}_{key}"])
        assert runtime.consume_async(task, c).detail == R.DETAIL_ASYNC_ALREADY_CONSUMED
        assert runtime.abandon_async(task) == R.PROM_OK
    assert np.array_equal(a, a0) and np.array_equal(b, b0)
    assert runtime.query_async(12345)[1].detail_code == R.DETAIL_ASYNC_NO_TASK
    assert runtime.consume_async(12345, np.empty(1, np.float32)).detail == R.DETAIL_ASYNC_INVALID_TASK


def test_async_queue_full_and_short_buffer(runtime, oracle_mod):
    o = oracle_mod
    a = o.marionette_matrix(64, 1)
    tasks = []
    for _ in range(4):
        t, st = runtime.submit_async(8, 8, 8, a, a)
        assert st.ok
        tasks.append(t)
    t, st = runtime.submit_async(8, 8, 8, a, a)
    assert not st.ok and st.detail == R.DETAIL_ASYNC_QUEUE_FULL
    short = np.empty(63, dtype=np.float32)
    import time
    time.sleep(0.05)
    for t in tasks:
        while runtime.query_async(t)[1].lifecycle_state == R.ASYNC_SUBMITTED:
            time.sleep(0.001)
        assert runtime.consume_async(t, short).rc == R.PROM_ERROR
        assert runtime.consume_async(t, np.empty(64, np.float32)).ok
        assert runtime.abandon_async(t) == R.PROM_OK


@pytest.mark.parametrize("variant", [R.SGEMM_AUTO, *VARIANTS])
@pytest.mark.parametrize("shape", GEMMA)
def test_gemma_small_m_corpus(runtime, oracle_mod, golden, shape, variant):
    """gemma4e2b_sgemm_corpus_test.go:29-100, every M of the corpus as a prefix slice."""
    o = oracle_mod
    m, n, k = shape
    a, b = o.gemma_corpus_a(m * k), o.gemma_corpus_b(k * n)
    want = golden[f"sgemm_gemma_{m}x{n}x{k}"]
    ms = [1, 2, 7, 15, 16, 17, 31, 32, 33] if m == 33 else [m]
    for mm in ms:
        c = device_sgemm(runtime, a[: mm * k], b, mm, n, k, variant)
        ref = o.cpu_sgemm_f32(a[: mm * k], b, mm, n, k)
        assert o.compare_against_oracle(ref, c).pass_ == 1, mm
        assert normwise(c, want[: mm * n].astype(np.float64)) <= NORMWISE_TOL


@pytest.mark.parametrize("shape", [(1, 256, 1536), (2, 256, 1536), (7, 256, 1536), (15, 256, 1536),
                                   (16, 256, 1536), (15, 2048, 1536), (16, 16384, 2048), (1, 16384, 2048),
                                   (9, 1001, 777), (3, 5, 7), (16, 3, 40000), (8, 16384, 2048),
                                   (5, 1004, 777), (16, 12, 40000), (4, 2052, 3)])
def test_small_m_kernel(runtime, oracle_mod, golden, shape):
    """The small-M kernel (m <= 16, split-K with an ordered reduction): the reference's small-M
    corpus shapes (gemma4e2b_sgemm_corpus_test.go:44-59), Gemma per-token shapes, ragged and
    deep-K ones; AUTO takes it for m <= 16; repeat calls are bit-identical.  n a multiple of 4
    takes the bulk-copy-fed kernel (ragged column tiles and K ranges included), other n the
    register-streaming one."""
    o = oracle_mod
    m, n, k = shape
    a, b = o.uniform_matrix(m, k, m + n).ravel(), o.uniform_matrix(k, n, k).ravel()
    c = device_sgemm(runtime, a, b, m, n, k, R.SGEMM_SMALLM)
    _check_against_fp64(o, c, a, b, m, n, k)
    assert np.array_equal(c, device_sgemm(runtime, a, b, m, n, k, R.SGEMM_AUTO))
    assert np.array_equal(c, device_sgemm(runtime, a, b, m, n, k, R.SGEMM_SMALLM))
    if (m, n, k) == (15, 256, 1536):  # the corpus inputs and their golden answer
        ga, gb = o.gemma_corpus_a(15 * 1536), o.gemma_corpus_b(1536 * 256)
        c = device_sgemm(runtime, ga, gb, 15, 256, 1536, R.SGEMM_SMALLM)
        assert o.compare_against_oracle(o.cpu_sgemm_f32(ga, gb, 15, 256, 1536), c).pass_ == 1


@pytest.mark.parametrize("shape", [(1, 256, 1536), (7, 256, 1536), (15, 256, 1536), (16, 256, 1536),
                                   (1, 16384, 2048), (8, 16384, 2048), (16, 16384, 2048), (16, 8192, 4096),
                                   (5, 1004, 776), (16, 12, 40000), (4, 2052, 4), (2, 300, 100), (9, 1001, 777)])
def test_small_m_tensor_core_kernel(runtime, oracle_mod, golden, shape):
    """The tensor-core small-M kernel (C^T = B^T A^T, TF32 split inside the kernel, split-K
    with an ordered reduction): the small-M corpus shapes, Gemma per-token shapes and ragged
    ones (n not a multiple of 128, k not a multiple of 32, one k step, a deep single column
    tile); repeat calls are bit-identical.  Shapes whose operands TMA cannot read in place
    (lda or ldb not a multiple of 4: 9 x 1001 x 777) run the CUDA-core kernel instead."""
    o = oracle_mod
    m, n, k = shape
    a, b = o.uniform_matrix(m, k, m + n).ravel(), o.uniform_matrix(k, n, k).ravel()
    c = device_sgemm(runtime, a, b, m, n, k, R.SGEMM_SMALLM_TC)
    _check_against_fp64(o, c, a, b, m, n, k)
    assert np.array_equal(c, device_sgemm(runtime, a, b, m, n, k, R.SGEMM_SMALLM_TC))
    if (m, n, k) == (15, 256, 1536):  # the corpus inputs and their golden answer
        ga, gb = o.gemma_corpus_a(15 * 1536), o.gemma_corpus_b(1536 * 256)
        c = device_sgemm(runtime, ga, gb, 15, 256, 1536, R.SGEMM_SMALLM_TC)
        assert o.compare_against_oracle(o.cpu_sgemm_f32(ga, gb, 15, 256, 1536), c).pass_ == 1


def test_small_m_kernel_rejects_larger_m(runtime):
    import torch
    x = torch.zeros((17, 8), device="cuda")
    with pytest.raises(R.ReactorIssue, match="detail=-7007"):
        runtime.sgemm_device(x, torch.zeros((8, 8), device="cuda"), torch.zeros((17, 8), device="cuda"), 17, 8, 8,
                             R.SGEMM_SMALLM)


def _check_against_fp64(o, c, a, b, m, n, k, rows=None):
    sl = rows or slice(0, m)
    ref64 = o.sgemm_f64(a, b, m, n, k, rows=sl)
    cpu32 = o.cpu_sgemm_f32(a, b, m, n, k, rows=sl, threads=o.max_threads())
    got = c.reshape(m, n)[sl].ravel()
    nw = normwise(got, ref64)
    err_gpu = np.max(np.abs(got.astype(np.float64) - ref64))
    err_cpu = np.max(np.abs(cpu32.astype(np.float64) - ref64))
    ulp = np.spacing(np.float32(np.max(np.abs(ref64))))
    assert nw <= NORMWISE_TOL, nw
    assert err_gpu <= 2 * err_cpu + ulp, (err_gpu, err_cpu)
    return nw


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("shape,seed", [((512, 512, 512), 0), ((1000, 1000, 1000), 1), ((4097, 4095, 1023), 2)])
def test_baseline_shapes_full_compare(runtime, oracle_mod, shape, seed, variant):
    """512^3 and the ragged sweep's smaller shapes: every output vs fp64."""
    o = oracle_mod
    m, n, k = shape
    a, b = o.uniform_matrix(m, k, seed).ravel(), o.uniform_matrix(k, n, seed + 100).ravel()
    c = device_sgemm(runtime, a, b, m, n, k, variant)
    if m * n * k <= 2 ** 31:
        _check_against_fp64(o, c, a, b, m, n, k)
    else:
        _check_against_fp64(o, c, a, b, m, n, k, rows=slice(0, 64))
        _check_against_fp64(o, c, a, b, m, n, k, rows=slice(m - 65, m))
    assert o.compare_against_oracle(o.cpu_sgemm_f32(a, b, m, n, k, rows=slice(0, 16), threads=8),
                                    c[: 16 * n]).pass_ == 1


def _checksums(o, c64, a, b, m, n, k):
    """Size-independent property: row sums C.1 = A(B.1) and column sums 1^T C = (1^T A) B."""
    A = a.reshape(m, k).astype(np.float64)
    B = b.reshape(k, n).astype(np.float64)
    row_ref = A @ B.sum(axis=1)
    col_ref = A.sum(axis=0) @ B
    C = c64.reshape(m, n)
    row_got = C.astype(np.float64).sum(axis=1)
    col_got = C.astype(np.float64).sum(axis=0)
    # per-sum error bound: n (or m) outputs each off by <= 1e-5 * max|C|
    scale = np.max(np.abs(C))
    assert np.max(np.abs(row_got - row_ref)) <= n * 1e-5 * scale
    assert np.max(np.abs(col_got - col_ref)) <= m * 1e-5 * scale


@pytest.mark.parametrize("variant", [R.SGEMM_TC_BK16, R.SGEMM_TC_BK32, R.SGEMM_TC_PAIR16, R.SGEMM_TC_PAIR32,
                                     R.SGEMM_TC_INSM16, R.SGEMM_TC_INSM32])
@pytest.mark.parametrize("shape,seed", [((8192, 8192, 8192), 3), ((16384, 16384, 4096), 4)])
def test_baseline_large_shapes(runtime, oracle_mod, shape, seed, variant):
    """8192^3 and 16384^2 x 4096: sampled rows vs fp64 plus whole-matrix checksums."""
    o = oracle_mod
    m, n, k = shape
    a, b = o.uniform_matrix(m, k, seed).ravel(), o.uniform_matrix(k, n, seed + 100).ravel()
    c = device_sgemm(runtime, a, b, m, n, k, variant)
    assert np.all(np.isfinite(c))
    for rows in (slice(0, 32), slice(m // 2 - 16, m // 2 + 16), slice(m - 32, m)):
        _check_against_fp64(o, c, a, b, m, n, k, rows=rows)
    _checksums(o, c, a, b, m, n, k)


@pytest.mark.parametrize("insm,pair", [(R.SGEMM_TC_INSM16, R.SGEMM_TC_PAIR16), (R.SGEMM_TC_INSM32, R.SGEMM_TC_PAIR32)])
@pytest.mark.parametrize("shape", [(17, 31, 23), (37, 29, 13), (255, 257, 33), (300, 517, 129), (1000, 1000, 1000),
                                   (4097, 4095, 1023)])
def test_in_kernel_split_reads_ragged_operands_in_place(runtime, oracle_mod, shape, insm, pair):
    """The in-SM split kernel reads A and B where they lie (leading dimensions padded to a
    multiple of 4 floats, so TMA may read them); the TMA's zero fill past m, n and k replaces
    the split pass's padding.  The split itself is the split pass's (round to nearest tf32,
    then the remainder), so the result equals the split-pass CTA-pair kernel bit for bit;
    columns of C past n stay untouched."""
    import torch
    o = oracle_mod
    m, n, k = shape
    lda, ldb, ldc = (k + 3) // 4 * 4 + 4, (n + 3) // 4 * 4, n + 3
    a, b = o.uniform_matrix(m, k, m + 1).ravel(), o.uniform_matrix(k, n, n + 2).ravel()
    da = torch.zeros((m, lda), device="cuda")
    db = torch.zeros((k, ldb), device="cuda")
    da[:, :k] = torch.from_numpy(a.reshape(m, k)).cuda()
    db[:, :n] = torch.from_numpy(b.reshape(k, n)).cuda()
    da[:, k:] = float("nan")  # never read: the TMA box stops at k
    outs = {}
    for v in (insm, pair):
        dc = torch.full((m, ldc), -3.0, device="cuda")
        runtime.sgemm_device(da, db, dc, m, n, k, v, lda=lda, ldb=ldb, ldc=ldc)
        assert runtime.sync_status().ok
        outs[v] = dc.cpu().numpy()
    got = outs[insm]
    assert np.all(got[:, n:] == -3.0)
    assert np.array_equal(got[:, :n], outs[pair][:, :n])
    _check_against_fp64(o, np.ascontiguousarray(got[:, :n]).ravel(), a, b, m, n, k,
                        rows=slice(0, min(m, 64)))


def test_variants_agree_with_batched_and_transposed_forms(runtime, oracle_mod):
    """Strided-batch and B^T (NT) forms equal per-entry products (attention's Q K^T and P V)."""
    import torch
    o = oracle_mod
    bsz, m, n, k = 3, 300, 200, 136
    a = o.uniform_matrix(bsz * m, k, 31).reshape(bsz, m, k)
    bt = o.uniform_matrix(bsz * n, k, 32).reshape(bsz, n, k)
    da, dbt = torch.from_numpy(a).cuda(), torch.from_numpy(bt).cuda()
    for variant in VARIANTS:
        dc = torch.full((bsz, m, n), float("nan"), device="cuda")
        runtime.sgemm_batched_device(da, k, m * k, dbt, k, n * k, True, dc, n, m * n, bsz, m, n, k, variant)
        assert runtime.sync_status().ok
        got = dc.cpu().numpy()
        for i in range(bsz):
            ref = o.sgemm_f64(np.ascontiguousarray(a[i]).ravel(), np.ascontiguousarray(bt[i].T).ravel(), m, n, k)
            assert normwise(got[i].ravel(), ref) <= NORMWISE_TOL, (variant, i)


@pytest.mark.parametrize("bsz,m", [(1, 8), (2, 1), (1, 16)])
def test_small_m_batched_and_transposed_forms(runtime, oracle_mod, bsz, m):
    """m <= 16 through the strided-batch entry with B^T: AUTO and the small-M id fall back to a
    kernel that reads B^T (the small-M kernel has neither form), one entry included."""
    import torch
    o = oracle_mod
    n, k = 264, 136
    a = o.uniform_matrix(bsz * m, k, 41).reshape(bsz, m, k)
    bt = o.uniform_matrix(bsz * n, k, 42).reshape(bsz, n, k)
    da, dbt = torch.from_numpy(a).cuda(), torch.from_numpy(bt).cuda()
    for variant in (R.SGEMM_AUTO, R.SGEMM_SMALLM):
        dc = torch.full((bsz, m, n), float("nan"), device="cuda")
        runtime.sgemm_batched_device(da, k, m * k, dbt, k, n * k, True, dc, n, m * n, bsz, m, n, k, variant)
        assert runtime.sync_status().ok
        got = dc.cpu().numpy()
        for i in range(bsz):
            ref = o.sgemm_f64(np.ascontiguousarray(a[i]).ravel(), np.ascontiguousarray(bt[i].T).ravel(), m, n, k)
            assert normwise(got[i].ravel(), ref) <= NORMWISE_TOL, (variant, i)


def test_host_abi_matches_device_path(runtime, oracle_mod):
    o = oracle_mod
    m, n, k = 300, 517, 129
    a, b = o.uniform_matrix(m, k, 7).ravel(), o.uniform_matrix(k, n, 8).ravel()
    c_host, st = runtime.sgemm_with_status(m, n, k, a, b)
    assert st.ok
    c_dev = device_sgemm(runtime, a, b, m, n, k, R.SGEMM_AUTO)
    assert np.array_equal(c_host, c_dev)


@pytest.mark.parametrize("pinned", [False, True])
@pytest.mark.parametrize("shape,seed", [((4097, 4095, 1023), 41), ((2048, 1024, 1024), 42), ((8192, 8192, 8192), 43)])
def test_pipelined_host_path_matches_device_path(runtime, oracle_mod, shape, seed, pinned):
    """Large host-buffer products upload A in row chunks, compute each chunk as it lands and
    download C chunks while later ones compute; the result must equal the one-shot device
    product bit for bit, from pageable and from pinned host buffers."""
    import torch
    o = oracle_mod
    m, n, k = shape
    a, b = o.uniform_matrix(m, k, seed).ravel(), o.uniform_matrix(k, n, seed + 1).ravel()
    if pinned:
        pa = torch.empty(a.size, dtype=torch.float32, pin_memory=True).numpy()
        pb = torch.empty(b.size, dtype=torch.float32, pin_memory=True).numpy()
        pc = torch.full((m * n,), float("nan"), dtype=torch.float32, pin_memory=True).numpy()
        pa[:], pb[:] = a, b
        c_host, st = runtime.sgemm_with_status(m, n, k, pa, pb, out=pc)
    else:
        c_host, st = runtime.sgemm_with_status(m, n, k, a, b)
    assert st.ok and (st.stage, st.detail) == (R.STAGE_TRANSFER_OUT, 6101), st
    c_dev = device_sgemm(runtime, a, b, m, n, k, R.SGEMM_AUTO)
    assert np.array_equal(c_host, c_dev)
    _check_against_fp64(o, c_host, a, b, m, n, k, rows=slice(m - 40, m))


def test_leading_dimensions_column_shard(runtime, oracle_mod):
    """oct_b200_sgemm_device_ld: a column block of a wider B / C (the tensor-parallel shard)."""
    import torch
    o = oracle_mod
    m, n, k = 256, 1024, 384
    a, b = o.uniform_matrix(m, k, 9), o.uniform_matrix(k, n, 10)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    full = torch.zeros((m, n), device="cuda")
    for variant in VARIANTS:
        for j in range(4):
            cols = slice(j * 256, (j + 1) * 256)
            runtime.sgemm_device(da, db[:, cols], full[:, cols], m, 256, k, variant, ldb=n, ldc=n)
        assert runtime.sync_status().ok
        ref = device_sgemm(runtime, a.ravel(), b.ravel(), m, n, k, variant)
        assert np.array_equal(full.cpu().numpy().ravel(), ref)


@pytest.mark.parametrize("flag,stage,detail", [
    (R.TESTCFG_FAIL_UPLOAD, R.STAGE_TRANSFER_IN, R.DETAIL_INJECTED_UPLOAD_FAILURE),
    (R.TESTCFG_FAIL_DISPATCH, R.STAGE_SUBMIT, R.DETAIL_INJECTED_DISPATCH_FAILURE),
    (R.TESTCFG_FAIL_DOWNLOAD, R.STAGE_TRANSFER_OUT, R.DETAIL_INJECTED_DOWNLOAD_FAILURE),
])
def test_host_fault_injection(lib, oracle_mod, flag, stage, detail):
    o = oracle_mod
    a = o.marionette_matrix(16, 1)
    c = np.full(16, 7.0, dtype=np.float32)
    with R.Runtime(lib, test_flags=flag) as rt:
        out, st = rt.sgemm_with_status(4, 4, 4, a, a, out=c)
    assert (st.rc, st.stage, st.detail) == (R.PROM_ERROR, stage, detail)
    assert np.all(c == 7.0)  # caller output untouched on failure


def test_async_poll_fault_injection(lib, oracle_mod):
    a = oracle_mod.marionette_matrix(16, 1)
    with R.Runtime(lib, test_flags=R.TESTCFG_FAIL_ASYNC_POLL) as rt:
        t, st = rt.submit_async(4, 4, 4, a, a)
        assert st.ok
        rc, qs = rt.query_async(t)
        assert qs.lifecycle_state == R.ASYNC_FAILED and qs.detail_code == R.DETAIL_ASYNC_INJECTED_POLL_FAILURE
        assert rt.consume_async(t, np.empty(16, np.float32)).detail == R.DETAIL_ASYNC_INJECTED_POLL_FAILURE
        assert rt.abandon_async(t) == R.PROM_OK


def test_strict_fp32_flag_selects_fma_control(lib, oracle_mod):
    o = oracle_mod
    m, n, k = 200, 300, 257
    a, b = o.uniform_matrix(m, k, 11).ravel(), o.uniform_matrix(k, n, 12).ravel()
    with R.Runtime(lib, test_flags=R.TESTCFG_FORCE_STRICT_FP32) as rt:
        c, st = rt.sgemm_with_status(m, n, k, a, b)
        assert st.ok
        ref = device_sgemm(rt, a, b, m, n, k, R.SGEMM_FMA)
    assert np.array_equal(c, ref)
