"""Row reductions, softmax and RMSNorm on the B200 through the C ABI.

Gates (written here): the reference comparator prom_reduction_compare
(reactor_vulkan_fused_reduction.c:1038-1114, restated in the oracle), plus
max relative error <= 1e-5 versus the fp64 oracle, elementwise with
the comparator's floor (|ref| < 1e-20 -> denominator 1).  SUM accumulates in
binary64 on the device and MAX is exact, so both also match the known answers
bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest

from oct_b200 import reactor as R
from tests.golden.make_golden import DISTS, RED_ROWS, WIDTHS

pytestmark = pytest.mark.gpu
REL_TOL = 1e-5


def rel_err(got, ref):
    ref = np.asarray(ref, dtype=np.float64)
    den = np.where(np.abs(ref) < 1e-20, 1.0, np.abs(ref))
    return float(np.max(np.abs(np.asarray(got, dtype=np.float64) - ref) / den))


@pytest.mark.parametrize("dist", DISTS)
def test_planner_widths_all_distributions(runtime, oracle_mod, golden, dist):
    o = oracle_mod
    for w in WIDTHS:
        x = o.reduction_input(RED_ROWS, w, dist)
        for op, name in ((R.OP_SUM, "sum"), (R.OP_MAX, "max"), (R.OP_SOFTMAX, "softmax")):
            y, res = runtime.reduction(x, op)
            assert y is not None, (name, w, res.detail_code)
            assert res.stage == R.STAGE_NONE and res.detail_code == 0 and res.gpu_timestamp_valid == 1
            want = golden[f"red_{name}_{dist}_{w}"]
            _, ref = o.reduction_cpu_reference(x, op)
            assert o.reduction_compare(RED_ROWS, w, op, ref, y)[0] == 0, (name, w)
            if op == R.OP_SOFTMAX:
                assert rel_err(y, want) <= REL_TOL, (name, w)
            else:
                assert np.array_equal(y, want), (name, w)


@pytest.mark.parametrize("rows", [1, 2, 16, 128, 1024])
def test_row_counts(runtime, oracle_mod, golden, rows):
    o = oracle_mod
    x = o.reduction_input(rows, 513)
    y, res = runtime.reduction(x, R.OP_MAX)
    assert np.array_equal(y, golden["red_max_deterministic_rows1024_513"][:rows])
    assert res.plan.stages[0].groups_x == rows


@pytest.mark.parametrize("width", [256, 2048, 4096])
@pytest.mark.parametrize("op", [R.OP_SUM, R.OP_MAX, R.OP_SOFTMAX])
def test_baseline_shapes(runtime, oracle_mod, width, op):
    """Benchmark shapes: 32768 rows x {256, 2048, 4096}, N(0,1) seeded."""
    o = oracle_mod
    rows = 32768
    x = o.normal_matrix(rows, width, seed=width)
    y, res = runtime.reduction(x, op)
    assert y is not None, res.detail_code
    _, ref = o.reduction_cpu_reference(x, op, threads=o.max_threads())
    assert o.reduction_compare(rows, width, op, ref, y)[0] == 0
    if op == R.OP_SOFTMAX:
        assert rel_err(y, ref) <= REL_TOL
        sums = y.reshape(rows, width).astype(np.float64).sum(axis=1)
        assert np.max(np.abs(sums - 1.0)) <= 1e-5
    else:
        assert np.array_equal(y, ref)


@pytest.mark.parametrize("rows,width", [(30001, 256), (40000, 128), (32768, 512), (1001, 128), (999, 512), (5, 1024)])
@pytest.mark.parametrize("op", [R.OP_SUM, R.OP_MAX, R.OP_SOFTMAX])
def test_tall_short_rows(runtime, oracle_mod, rows, width, op):
    """Tall matrices of short rows whose row count leaves the last ring slot ragged, and
    rows too many for every warp to hold all of its rows in the ring at once; row counts
    that leave the last warp of the register-resident kernels (8 / 4 / 2 / 1 rows per warp
    at widths 128 / 256 / 512 / 1024) part-filled."""
    o = oracle_mod
    x = o.normal_matrix(rows, width, seed=rows + width)
    y, res = runtime.reduction(x, op)
    assert y is not None, res.detail_code
    _, ref = o.reduction_cpu_reference(x, op, threads=o.max_threads())
    assert o.reduction_compare(rows, width, op, ref, y)[0] == 0
    if op == R.OP_SOFTMAX:
        assert rel_err(y, ref) <= REL_TOL
    else:
        assert np.array_equal(y, ref)


@pytest.mark.parametrize("width", [7, 33, 1057, 9000])
def test_unaligned_and_wide_rows_use_same_arithmetic(runtime, oracle_mod, width):
    o = oracle_mod
    x = o.normal_matrix(37, width, seed=width)
    for op in (R.OP_SUM, R.OP_MAX, R.OP_SOFTMAX):
        y, res = runtime.reduction(x, op)
        _, ref = o.reduction_cpu_reference(x, op)
        assert o.reduction_compare(37, width, op, ref, y)[0] == 0
        if op == R.OP_SOFTMAX:
            assert rel_err(y, ref) <= REL_TOL
        else:
            assert np.array_equal(y, ref)


def test_nonfinite_rejected_and_output_untouched(runtime, oracle_mod):
    o = oracle_mod
    x = o.reduction_input(64, 256)
    x[17, 3] = np.inf
    x[40, 9] = np.nan
    out = np.full(64, 5.0, dtype=np.float32)
    y, res = runtime.reduction(x, R.OP_SUM, out=out)
    assert y is None and res.detail_code == -6814
    assert res.first_nonfinite_index == 17 * 256 + 3
    assert np.all(out == 5.0)
    rc, y, sres = runtime.row_wise_softmax(x)
    assert rc == R.PROM_ERROR and sres.detail_code == -6860 and sres.output_written == 0


def test_row_wise_softmax_abi(runtime, oracle_mod):
    o = oracle_mod
    x = o.reduction_input(1024, 1056, "heterogeneous")
    rc, y, res = runtime.row_wise_softmax(x)
    assert rc == R.PROM_OK and res.output_written == 1 and res.physical_dispatch_count == 1
    _, ref = o.reduction_cpu_reference(x, R.OP_SOFTMAX)
    assert rel_err(y.ravel(), ref) <= REL_TOL
    inplace = x.copy()
    rc, y2, _ = runtime.row_wise_softmax(inplace, out=inplace)  # exact in-place is admitted
    assert rc == R.PROM_OK and np.array_equal(inplace.ravel(), y.ravel())


@pytest.mark.parametrize("flag,detail", [
    (R.REDUCTION_TESTCFG_FAIL_COMMAND_RECORD, -6820),
    (R.REDUCTION_TESTCFG_FAIL_QUEUE_SUBMIT, -6821),
    (R.REDUCTION_TESTCFG_FAIL_COMPLETION_OBSERVATION, -6822),
])
def test_reduction_fault_injection(lib, oracle_mod, flag, detail):
    x = oracle_mod.reduction_input(4, 64)
    out = np.full(4, 9.0, dtype=np.float32)
    with R.Runtime(lib, reduction_test_flags=flag) as rt:
        y, res = rt.reduction(x, R.OP_SUM, out=out)
    assert y is None and res.detail_code == detail and res.stage == R.STAGE_SUBMIT
    assert np.all(out == 9.0)


@pytest.mark.parametrize("w", [256, 2048])
def test_rmsnorm_known_answers(runtime, oracle_mod, golden, w):
    o = oracle_mod
    x = o.reduction_input(8, w)
    wt = golden[f"rms_deterministic_{w}_weight"]
    rc, y, inv, res = runtime.rmsnorm(x, wt, 1e-6)
    assert rc == R.PROM_OK and res.output_written == 1, res.detail_code
    assert rel_err(y.ravel(), golden[f"rms_deterministic_{w}_out"]) <= REL_TOL
    assert rel_err(inv, golden[f"rms_deterministic_{w}_inv"]) <= REL_TOL


@pytest.mark.parametrize("width", [256, 2048, 4096, 33])
def test_rmsnorm_baseline(runtime, oracle_mod, width):
    """Benchmark RMSNorm: 32768 rows, eps 1e-6, gamma ~ U[0.5, 1.5)."""
    o = oracle_mod
    rows = 32768 if width != 33 else 100
    x = o.normal_matrix(rows, width, seed=width + 1)
    wt = (o.uniform_matrix(1, width, seed=width + 2).ravel() * np.float32(0.5) + np.float32(1.0)).astype(np.float32)
    rc, y, inv, res = runtime.rmsnorm(x, wt, 1e-6)
    assert rc == R.PROM_OK, res.detail_code
    ref64, inv64 = o.rmsnorm_f64(x, wt, 1e-6)
    assert rel_err(y, ref64) <= REL_TOL
    assert rel_err(inv, inv64) <= REL_TOL
    for form in ("head", "canonical"):  # Gemma's and Z-Image's fp32 CPU forms
        ref32, _ = o.rmsnorm_f32(x, wt, 1e-6, threads=o.max_threads(), form=form)
        assert rel_err(y, ref32) <= 1e-4  # each fp32 CPU formula differs by its own rounding only
    if width == 256:
        # the head entry rounds its input and output through BF16 (reactor_api.c:370-395)
        rc, yh, invh, res = runtime.rmsnorm(x, wt, 1e-6, mode="head")
        assert rc == R.PROM_OK, res.detail_code
        want, want_inv = o.m1_rmsnorm(x, wt, 1e-6, True, True)
        assert np.array_equal(yh.ravel(), want) and np.array_equal(invh, want_inv)


def test_device_output_read_right_after_the_call(runtime, oracle_mod):
    """A long device-path launch whose output is copied back right after the status read: the
    copy must see every row (outputs start as NaN)."""
    import torch
    o = oracle_mod
    x = o.normal_matrix(32768, 4096, seed=9)
    dx = torch.from_numpy(x).cuda()
    w = torch.ones(4096, device="cuda")
    for _ in range(2):
        yr = torch.full_like(dx, float("nan"))
        inv = torch.full((32768,), float("nan"), device="cuda")
        ys = torch.full((32768,), float("nan"), device="cuda")
        torch.cuda.synchronize()
        runtime.reduction_device(dx, ys, 32768, 4096, R.OP_SUM)
        runtime.rmsnorm_device(dx, w, yr, inv, 32768, 4096, 1e-6)
        assert runtime.sync_status().ok
        y = yr.cpu().numpy()
        assert not np.isnan(y).any() and not np.isnan(inv.cpu().numpy()).any()
        assert np.array_equal(ys.cpu().numpy(), o.reduction_cpu_reference(x, R.OP_SUM, o.max_threads())[1])


def test_device_entry_points(runtime, oracle_mod):
    import torch
    o = oracle_mod
    x = o.normal_matrix(4096, 2048, seed=5)
    dx = torch.from_numpy(x).cuda()
    ys = torch.empty(4096, device="cuda")
    ym = torch.empty_like(dx)
    runtime.reduction_device(dx, ys, 4096, 2048, R.OP_SUM)
    runtime.reduction_device(dx, ym, 4096, 2048, R.OP_SOFTMAX)
    w = torch.ones(2048, device="cuda")
    yr = torch.empty_like(dx)
    inv = torch.empty(4096, device="cuda")
    runtime.rmsnorm_device(dx, w, yr, inv, 4096, 2048, 1e-6)
    assert runtime.sync_status().ok
    assert np.array_equal(ys.cpu().numpy(), o.reduction_cpu_reference(x, R.OP_SUM, 8)[1])
    assert rel_err(ym.cpu().numpy().ravel(), o.reduction_cpu_reference(x, R.OP_SOFTMAX, 8)[1]) <= REL_TOL
    assert rel_err(yr.cpu().numpy(), o.rmsnorm_f64(x, np.ones(2048, np.float32), 1e-6)[0]) <= REL_TOL
