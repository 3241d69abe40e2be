"""The no-allocation SGEMM entry point, checked against the allocating one.

Some callers of this library cannot allocate device memory: for example a
serving process whose fixed memory plan gives all of HBM to its own pool, or
code that must not trigger the device-wide synchronisation a cudaMalloc can
imply.  `oct_b200_sgemm_device_noalloc` serves them: it runs the same tcgen05
3xTF32 kernel with its scratch in a fixed device array, and needs no handle.
This file is collected last (test_zz_*), so a stop-at-first-failure run has
already run every other test when it gets here.  It passes on its own in a
fresh process too.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from oct_b200 import reactor as R

pytestmark = pytest.mark.gpu
NORMWISE_TOL = 1e-5  # the SGEMM parity tolerance used throughout tests/test_sgemm_gpu.py


def _noalloc(lib, a, b, c, m, n, k, lda=None, ldb=None, ldc=None, stream=None):
    detail = C.c_int(12345)
    rc = lib.oct_b200_sgemm_device_noalloc(a.data_ptr(), lda or k, b.data_ptr(), ldb or n, c.data_ptr(), ldc or n,
                                           m, n, k, None if stream is None else C.c_void_p(stream.cuda_stream),
                                           C.byref(detail))
    return rc, detail.value


def test_noalloc_matches_the_allocating_entry_point(lib, oracle_mod):
    import torch
    o = oracle_mod
    rt = R.Runtime(lib)
    try:
        # two calls in a row: a ragged shape, then the largest admitted cube
        for (m, n, k), seed in (((1000, 700, 513), 1), ((2048, 2048, 2048), 2)):
            a, b = o.uniform_matrix(m, k, seed), o.uniform_matrix(k, n, seed + 50)
            da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
            c_ref = torch.full((m, n), float("nan"), device="cuda")
            c_new = torch.full((m, n), float("nan"), device="cuda")
            torch.cuda.synchronize()
            rt.sgemm_device(da, db, c_ref, m, n, k, R.SGEMM_TC_BK16)
            assert rt.sync_status().ok
            rc, detail = _noalloc(lib, da, db, c_new, m, n, k)
            assert (rc, detail) == (R.PROM_OK, 0)
            got, want = c_new.cpu().numpy(), c_ref.cpu().numpy()
            assert np.array_equal(got, want)  # same kernel, same split: bit-identical
            ref64 = o.sgemm_f64(a.ravel(), b.ravel(), m, n, k).reshape(m, n)
            assert np.max(np.abs(got - ref64)) / np.max(np.abs(ref64)) <= NORMWISE_TOL
    finally:
        rt.close()


def test_noalloc_rejects_products_beyond_its_scratch(lib):
    import torch
    m = n = k = 2304  # needs more than the fixed 64 MiB of split scratch
    a = torch.zeros((m, k), device="cuda")
    b = torch.zeros((k, n), device="cuda")
    c = torch.full((m, n), 7.0, device="cuda")
    rc, detail = _noalloc(lib, a, b, c, m, n, k)
    assert rc == R.PROM_ERROR and detail == -7006
    assert bool(torch.all(c == 7.0))  # nothing was launched


def test_noalloc_strided_operands_on_a_side_stream(lib, oracle_mod):
    """A serving caller passes views into its own pool (leading dimensions wider
    than the logical matrix) and its own stream: twice in a row, the result is
    bit-identical to the allocating entry point's, and C's columns beyond n keep
    their contents."""
    import torch
    o = oracle_mod
    rt = R.Runtime(lib)
    side = torch.cuda.Stream()
    try:
        for (m, n, k, pad), seed in (((777, 520, 300, 12), 5), ((1536, 1024, 1100, 40), 6)):
            lda, ldb, ldc = k + pad, n + pad + 4, n + 2 * pad
            a_full = torch.from_numpy(o.uniform_matrix(m, lda, seed)).cuda()
            b_full = torch.from_numpy(o.uniform_matrix(k, ldb, seed + 50)).cuda()
            c_ref = torch.full((m, ldc), -3.0, device="cuda")
            c_new = torch.full((m, ldc), -3.0, device="cuda")
            torch.cuda.synchronize()
            rt.sgemm_device(a_full, b_full, c_ref, m, n, k, R.SGEMM_TC_BK16, lda=lda, ldb=ldb, ldc=ldc)
            assert rt.sync_status().ok
            with torch.cuda.stream(side):
                rc, detail = _noalloc(lib, a_full, b_full, c_new, m, n, k, lda=lda, ldb=ldb, ldc=ldc, stream=side)
            assert (rc, detail) == (R.PROM_OK, 0)
            side.synchronize()
            got, want = c_new.cpu().numpy(), c_ref.cpu().numpy()
            assert np.array_equal(got[:, :n], want[:, :n])
            assert np.all(got[:, n:] == -3.0)  # nothing written beyond the logical columns
            a = a_full[:, :k].cpu().numpy().astype(np.float32).copy()
            b = b_full[:, :n].cpu().numpy().astype(np.float32).copy()
            ref64 = o.sgemm_f64(a.ravel(), b.ravel(), m, n, k).reshape(m, n)
            assert np.max(np.abs(got[:, :n] - ref64)) / np.max(np.abs(ref64)) <= NORMWISE_TOL
    finally:
        rt.close()


def test_noalloc_rejects_bad_arguments_with_a_negative_detail(lib):
    import torch
    a = torch.zeros((8, 8), device="cuda")
    rc, detail = _noalloc(lib, a, a, a, 8, 8, 8, lda=4)  # lda < k
    assert rc == R.PROM_ERROR and detail == R.DETAIL_INVALID_ARGUMENT
