"""The C-ABI boundary, checked without a GPU: library load, exported symbols,
struct layouts, handle/validation semantics, and the host-only reduction planner.

Mirrors internal/prometheus/bridge_test.go (ABI version, missing symbols,
unavailable runtime) and the planner FACT of
internal/prometheus/native/Marionette/reactor_reduction_tests.cpp:191-290.
"""
from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oct_b200 import reactor as R

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "prometheus_reactor.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"PROM_REACTOR_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported(lib):
    names = declared_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_version_is_one(lib):
    assert lib.prometheus_reactor_abi_version() == 1


def test_missing_library_is_reported(tmp_path):
    with pytest.raises(R.ReactorIssue) as exc:
        R.load_library(tmp_path / "libprometheus_reactor.so")
    assert exc.value.code == R.ReactorIssue.NOT_FOUND


def test_symbol_missing_is_reported(tmp_path):
    # A library exporting only the ABI version must fail with symbol_missing (bridge.go:276-300).
    src = tmp_path / "stub.c"
    src.write_text("unsigned prometheus_reactor_abi_version(void){return 1u;}\n")
    so = tmp_path / "libprometheus_reactor.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-o", str(so), str(src)], check=True)
    with pytest.raises(R.ReactorIssue) as exc:
        R.load_library(so)
    assert exc.value.code == R.ReactorIssue.SYMBOL_MISSING


def test_abi_mismatch_is_reported(tmp_path):
    src = tmp_path / "stub.c"
    body = "unsigned prometheus_reactor_abi_version(void){return 2u;}\n"
    for name in ("prometheus_reactor_runtime_create", "prometheus_reactor_runtime_destroy",
                 "prometheus_reactor_runtime_probe", "prometheus_reactor_runtime_sgemm"):
        body += f"int {name}(void){{return 1;}}\n"
    src.write_text(body)
    so = tmp_path / "libprometheus_reactor.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-o", str(so), str(src)], check=True)
    with pytest.raises(R.ReactorIssue) as exc:
        R.load_library(so)
    assert exc.value.code == R.ReactorIssue.ABI_MISMATCH


STRUCTS = {
    "PrometheusCaps": R.PrometheusCaps,
    "PrometheusReactorConfig": R.PrometheusReactorConfig,
    "PrometheusAsyncStatus": R.PrometheusAsyncStatus,
    "PrometheusReductionRequest": R.PrometheusReductionRequest,
    "PrometheusReductionStageDispatch": R.PrometheusReductionStageDispatch,
    "PrometheusReductionPlan": R.PrometheusReductionPlan,
    "PrometheusReductionExecutionResult": R.PrometheusReductionExecutionResult,
    "PrometheusRowWiseSoftmaxRequest": R.PrometheusRowWiseSoftmaxRequest,
    "PrometheusRowWiseSoftmaxResult": R.PrometheusRowWiseSoftmaxResult,
    "PrometheusGemma4E2BM1InputRmsNormRequest": R.PrometheusGemma4E2BM1InputRmsNormRequest,
    "PrometheusGemma4E2BM1InputRmsNormResult": R.PrometheusGemma4E2BM1InputRmsNormResult,
    "PrometheusSgemmBatchEntry": R.PrometheusSgemmBatchEntry,
    "PrometheusSgemmResidentBenchmarkRequest": R.PrometheusSgemmResidentBenchmarkRequest,
    "PrometheusSgemmResidentBenchmarkResult": R.PrometheusSgemmResidentBenchmarkResult,
    "PrometheusGemma4E2BM1RopeRequest": R.PrometheusGemma4E2BM1RopeRequest,
    "PrometheusGemma4E2BM1RopeResult": R.PrometheusGemma4E2BM1RopeResult,
    "PrometheusGemma4E2BM1HeadRmsNormRopeRequest": R.PrometheusGemma4E2BM1HeadRmsNormRopeRequest,
    "PrometheusGemma4E2BM1HeadRmsNormRopeResult": R.PrometheusGemma4E2BM1HeadRmsNormRopeResult,
    "PrometheusGemma4E2BM1AttentionScoresRequest": R.PrometheusGemma4E2BM1AttentionScoresRequest,
    "PrometheusGemma4E2BM1AttentionScoresResult": R.PrometheusGemma4E2BM1AttentionScoresResult,
    "PrometheusReductionDiagnostics": R.PrometheusReductionDiagnostics,
    "PrometheusReductionBenchmarkRequest": R.PrometheusReductionBenchmarkRequest,
    "PrometheusReductionBenchmarkResult": R.PrometheusReductionBenchmarkResult,
    "PrometheusSgemmAsyncTaskDiagnostics": R.PrometheusSgemmAsyncTaskDiagnostics,
    "PrometheusSgemmAsyncDiagnostics": R.PrometheusSgemmAsyncDiagnostics,
    "PrometheusModelBlockWeightDeclaration": R.PrometheusModelBlockWeightDeclaration,
    "PrometheusModelBlockCreateRequest": R.PrometheusModelBlockCreateRequest,
    "PrometheusModelBlockWeightUpload": R.PrometheusModelBlockWeightUpload,
    "PrometheusNoiseRefinerRebindRequest": R.PrometheusNoiseRefinerRebindRequest,
    "PrometheusContextRefinerCreateRequest": R.PrometheusContextRefinerCreateRequest,
    "PrometheusModelBlockExecuteRequest": R.PrometheusModelBlockExecuteRequest,
    "PrometheusNoiseRefiner0ExecuteRequest": R.PrometheusNoiseRefiner0ExecuteRequest,
    "PrometheusNoiseRefinerResidentExecuteRequest": R.PrometheusNoiseRefinerResidentExecuteRequest,
    "PrometheusContextRefiner0ExecuteRequest": R.PrometheusContextRefiner0ExecuteRequest,
    "PrometheusContextRefinerResidentExecuteRequest": R.PrometheusContextRefinerResidentExecuteRequest,
    "PrometheusNoiseRefinerFinalAuditRequest": R.PrometheusNoiseRefinerFinalAuditRequest,
    "PrometheusModelBlockEvidence": R.PrometheusModelBlockEvidence,
    "OctB200BlockConfig": R.OctB200BlockConfig,
    "OctB200TpSgemmConfig": R.OctB200TpSgemmConfig,
}


def test_struct_layouts_match_the_c_header(tmp_path):
    """sizeof and every field offset agree between the header (compiled by gcc) and ctypes."""
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void){"]
    for cname, py in STRUCTS.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for fname, *_ in py._fields_:
            lines.append(f'printf("{cname}.{fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0;}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-o", str(exe), str(src)], check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    for cname, py in STRUCTS.items():
        assert int(got[cname]) == C.sizeof(py), cname
        for fname, *_ in py._fields_:
            assert int(got[f"{cname}.{fname}"]) == getattr(py, fname).offset, f"{cname}.{fname}"


def test_struct_layouts_match_the_reference_header():
    """Every struct this header shares with the reference's reactor_api.h has the
    reference's field names, offsets and size (fixture: tests/golden/make_layouts.py,
    measured by gcc on the reference header itself)."""
    import json
    import sys
    sys.path.insert(0, str(REPO / "tests" / "golden"))
    import make_layouts as ML
    fixture = json.loads((REPO / "tests" / "golden" / "reference_layouts.json").read_text())["structs"]
    ours = ML.parse_structs(HEADER.read_text())
    assert len(fixture) >= 37
    for name, ref in fixture.items():
        assert name in ours, name
        assert ours[name] == [f for f, _ in ref["fields"]], name
    got = ML.measure(HEADER, {name: ours[name] for name in fixture})
    assert got == fixture


# ---- handle semantics without a device ------------------------------------------
def _handle(lib, flags=0):
    cfg = R.PrometheusReactorConfig()
    cfg.struct_size = C.sizeof(cfg)
    cfg.test_flags = flags
    h = C.c_void_p()
    assert lib.prometheus_reactor_runtime_create(C.byref(cfg), C.byref(h)) == R.PROM_OK
    return h


def test_create_probe_destroy_and_stale_handle(lib):
    h = _handle(lib, R.TESTCFG_FAIL_DEVICE_CREATE)  # host-injected: handle without a device
    caps = R.PrometheusCaps()
    assert lib.prometheus_reactor_runtime_probe(h, C.byref(caps)) == R.PROM_OK
    assert caps.available == 0 and caps.reason_code != 0
    assert lib.prometheus_reactor_runtime_destroy(h) == R.PROM_OK
    assert lib.prometheus_reactor_runtime_destroy(h) == R.PROM_INVALID_HANDLE
    assert lib.prometheus_reactor_runtime_probe(h, C.byref(caps)) == R.PROM_INVALID_HANDLE
    # NULL config is admitted (reactor_concept_sgemm_tests.cpp:31)
    h2 = C.c_void_p()
    assert lib.prometheus_reactor_runtime_create(None, C.byref(h2)) == R.PROM_OK
    assert lib.prometheus_reactor_runtime_destroy(h2) == R.PROM_OK


def test_runtime_without_device_fails_loudly(lib):
    with pytest.raises(R.ReactorIssue) as exc:
        R.Runtime(lib, test_flags=R.TESTCFG_FAIL_DEVICE_CREATE)
    assert exc.value.code == R.ReactorIssue.PROBE_FAILED


def test_sgemm_validation_order(lib):
    """reactor_sgemm.cpp:4149-4176: handle, then pointers, then dims, then device."""
    a = np.ones(4, dtype=np.float32)
    st, d = C.c_uint32(), C.c_int()
    rc = lib.prometheus_reactor_runtime_sgemm(None, a.ctypes.data, a.ctypes.data, a.ctypes.data, 2, 2, 2,
                                              C.byref(st), C.byref(d))
    assert (rc, st.value, d.value) == (R.PROM_INVALID_HANDLE, R.STAGE_INIT, R.PROM_INVALID_HANDLE)
    h = _handle(lib, R.TESTCFG_FAIL_DEVICE_CREATE)
    try:
        rc = lib.prometheus_reactor_runtime_sgemm(h, a.ctypes.data, None, a.ctypes.data, 2, 2, 2, C.byref(st),
                                                  C.byref(d))
        assert (rc, st.value, d.value) == (R.PROM_ERROR, R.STAGE_TRANSFER_IN, R.PROM_ERROR)
        rc = lib.prometheus_reactor_runtime_sgemm(h, a.ctypes.data, a.ctypes.data, a.ctypes.data, 0, 2, 2,
                                                  C.byref(st), C.byref(d))
        assert (rc, st.value, d.value) == (R.PROM_ERROR, R.STAGE_INIT, R.PROM_ERROR)
        rc = lib.prometheus_reactor_runtime_sgemm(h, a.ctypes.data, a.ctypes.data, a.ctypes.data, 2, 2, 2,
                                                  C.byref(st), C.byref(d))
        assert rc == R.PROM_ERROR and st.value == R.STAGE_INIT  # no device: no CPU fallback
    finally:
        lib.prometheus_reactor_runtime_destroy(h)


def test_sgemm_caller_entries_validation(lib):
    """benchmark_variant, resident benchmark and batch: the checks that precede any device work
    (reactor_sgemm.cpp:5629-5700, 5984-6009; reactor_batch.c:244-282)."""
    a = np.ones(4, dtype=np.float32)
    st, d = C.c_uint32(), C.c_int()
    h = _handle(lib, R.TESTCFG_FAIL_DEVICE_CREATE)
    try:
        # unknown variant id is rejected before the device check
        rc = lib.prometheus_reactor_runtime_sgemm_benchmark_variant(h, a.ctypes.data, a.ctypes.data, a.ctypes.data,
                                                                    2, 2, 2, 99, C.byref(st), C.byref(d))
        assert (rc, st.value, d.value) == (R.PROM_ERROR, R.STAGE_INIT, R.DETAIL_BAD_VARIANT)
        rc = lib.prometheus_reactor_runtime_sgemm_benchmark_variant(h, a.ctypes.data, a.ctypes.data, a.ctypes.data,
                                                                    2, 2, 2, 2, C.byref(st), C.byref(d))
        assert rc == R.PROM_ERROR and st.value == R.STAGE_INIT  # no device
        # resident benchmark
        assert lib.prometheus_reactor_runtime_sgemm_resident_benchmark(h, None, None) == R.PROM_ERROR
        res = R.PrometheusSgemmResidentBenchmarkResult()
        rc = lib.prometheus_reactor_runtime_sgemm_resident_benchmark(None, None, C.byref(res))
        assert (rc, res.setup_stage, res.setup_detail_code) == (R.PROM_INVALID_HANDLE, R.STAGE_INIT,
                                                                R.PROM_INVALID_HANDLE)
        assert res.struct_size == C.sizeof(res)
        rc = lib.prometheus_reactor_runtime_sgemm_resident_benchmark(h, None, C.byref(res))
        assert (rc, res.setup_stage, res.setup_detail_code) == (R.PROM_ERROR, R.STAGE_TRANSFER_IN, R.PROM_ERROR)
        assert res.resident_mode_available == 0
        req = R.PrometheusSgemmResidentBenchmarkRequest()
        req.struct_size = C.sizeof(req)
        req.a = req.b = a.ctypes.data
        req.m = req.n = req.k = 2
        req.flags = R.RESIDENT_FLAG_VALIDATE_READBACK  # and c is NULL
        rc = lib.prometheus_reactor_runtime_sgemm_resident_benchmark(h, C.byref(req), C.byref(res))
        assert (rc, res.setup_stage, res.setup_detail_code) == (R.PROM_ERROR, R.STAGE_TRANSFER_IN, R.PROM_ERROR)
        req.flags = 0
        rc = lib.prometheus_reactor_runtime_sgemm_resident_benchmark(h, C.byref(req), C.byref(res))
        assert (rc, res.setup_stage) == (R.PROM_ERROR, R.STAGE_INIT)  # no device
        # batch: flag mask first, then the device, then the entry list
        entries = (R.PrometheusSgemmBatchEntry * 1)()
        entries[0].a = entries[0].b = entries[0].c = a.ctypes.data
        entries[0].m = entries[0].n = entries[0].k = 2
        rc = lib.prometheus_reactor_runtime_sgemm_batch(None, entries, 1, 0, C.byref(st), C.byref(d))
        assert (rc, st.value, d.value) == (R.PROM_INVALID_HANDLE, R.STAGE_INIT, R.PROM_INVALID_HANDLE)
        rc = lib.prometheus_reactor_runtime_sgemm_batch(h, entries, 1, 1 << 9, C.byref(st), C.byref(d))
        assert (rc, st.value, d.value) == (R.PROM_ERROR, R.STAGE_INIT, R.DETAIL_BATCH_UNSUPPORTED_OPTION)
        rc = lib.prometheus_reactor_runtime_sgemm_batch(h, entries, 1, 0, C.byref(st), C.byref(d))
        assert (rc, st.value, d.value) == (R.PROM_ERROR, R.STAGE_INIT, R.DETAIL_BATCH_EXECUTION_FAILED)
    finally:
        lib.prometheus_reactor_runtime_destroy(h)


def test_reduction_validation_codes(lib):
    h = _handle(lib, R.TESTCFG_FAIL_DEVICE_CREATE)
    x = np.ones(64, dtype=np.float32)
    y = np.ones(64, dtype=np.float32)
    res = R.PrometheusReductionExecutionResult()

    def run(rows, width, op, fin=None, flags=0, in_count=None, out_count=None, inp=x, out=y):
        req = R.make_reduction_request(inp, out, rows, width, op, flags)
        if fin is not None:
            req.finalization = fin
        if in_count is not None:
            req.input_element_count = in_count
        if out_count is not None:
            req.output_element_count = out_count
        if inp is None:
            req.input = None
        if out is None:
            req.output = None
        return lib.prometheus_reactor_runtime_reduction(h, C.byref(req), C.byref(res)), res.detail_code

    try:
        assert run(0, 4, R.OP_SUM) == (R.PROM_ERROR, -6804)
        assert run(4, 0, R.OP_SUM) == (R.PROM_ERROR, -6805)
        assert run(4, 4, 9) == (R.PROM_ERROR, -6806)
        assert run(4, 4, R.OP_SOFTMAX, fin=0) == (R.PROM_ERROR, -6807)
        assert run(4, 4, R.OP_SUM, fin=1) == (R.PROM_ERROR, -6807)
        assert run(4, 4, R.OP_SUM, flags=1) == (R.PROM_ERROR, -6815)
        assert run(4, 2048, R.OP_SOFTMAX, flags=1) == (R.PROM_ERROR, -6815)
        assert run(4, 4, R.OP_SUM, in_count=15) == (R.PROM_ERROR, -6809)
        assert run(4, 4, R.OP_SUM, out_count=5) == (R.PROM_ERROR, -6810)
        assert run(4, 4, R.OP_SUM, inp=None) == (R.PROM_ERROR, -6802)
        assert run(4, 4, R.OP_SUM, out=None) == (R.PROM_ERROR, -6803)
        assert run(4, 1048577, R.OP_SUM) == (R.PROM_ERROR, -6812)
        # in-envelope and widened shapes both validate; this handle has no device
        assert run(4, 4, R.OP_SUM) == (R.PROM_ERROR, -6825)
        assert run(32768, 4, R.OP_SUM) == (R.PROM_ERROR, -6825)
        assert lib.prometheus_reactor_runtime_reduction(None, None, C.byref(res)) == R.PROM_INVALID_HANDLE
        assert res.detail_code == -6825
    finally:
        lib.prometheus_reactor_runtime_destroy(h)


def test_softmax_validation_codes(lib):
    h = _handle(lib, R.TESTCFG_FAIL_DEVICE_CREATE)
    buf = np.zeros(64, dtype=np.float32)
    res = R.PrometheusRowWiseSoftmaxResult()

    def run(inp, out, rows, width, count=None):
        req = R.PrometheusRowWiseSoftmaxRequest()
        req.struct_size = C.sizeof(req)
        req.input, req.output = inp, out
        req.row_count, req.elements_per_row = rows, width
        req.input_element_count = req.output_element_count = rows * width if count is None else count
        return lib.prometheus_reactor_runtime_row_wise_softmax(h, C.byref(req), C.byref(res)), res.detail_code

    base = buf.ctypes.data
    try:
        assert run(base, base + 128, 2, 8, count=15) == (R.PROM_ERROR, -6854)
        assert run(0, base, 0, 0) == (R.PROM_OK, 0)  # empty request is a no-op
        assert run(None, base, 2, 8) == (R.PROM_ERROR, -6852)
        assert run(base, None, 2, 8) == (R.PROM_ERROR, -6853)
        assert run(base, base + 4, 2, 8) == (R.PROM_ERROR, -6859)  # partial alias
        assert run(base, base, 1, 1057) == (R.PROM_ERROR, -6857)
        assert run(base, base, 2, 8) == (R.PROM_ERROR, -6861)  # exact in-place admitted; no device here
    finally:
        lib.prometheus_reactor_runtime_destroy(h)


# ---- the reference's planner FACT, verbatim expectations -------------------------
PLANNER_WIDTHS = [1, 2, 3, 31, 32, 33, 63, 64, 65, 127, 128, 129, 255, 256, 257, 511, 512, 513, 1024, 4096]


def test_planner_boundaries(lib):
    for w in PLANNER_WIDTHS:
        rc, first = R.reduction_plan(lib, 1, w, R.OP_SUM)
        rc2, replay = R.reduction_plan(lib, 1, w, R.OP_SUM)
        assert rc == rc2 == R.PROM_OK
        assert first.replay_id == replay.replay_id
        assert first.stage_count == (2 if w > 1024 else 1)
        assert first.partial_count == (w + 1023) // 1024
        assert first.temporary_alignment_bytes == 4
        rc, sm = R.reduction_plan(lib, 1, w, R.OP_SOFTMAX)
        assert rc == R.PROM_OK
        assert sm.stage_count == (5 if w > 1024 else 1)
        want = 2 if w > 1024 else (3 if w <= 128 else 1)
        assert sm.strategy == want, w
    for rows in (1, 2, 16, 128, 1024):
        rc, plan = R.reduction_plan(lib, rows, 513, R.OP_MAX)
        assert rc == R.PROM_OK and plan.stages[0].groups_x == rows
    for op in (R.OP_SUM, R.OP_SOFTMAX):
        rc, plan = R.reduction_plan(lib, 512, 64, op)
        assert rc == R.PROM_OK and plan.strategy == 3 and plan.stages[0].groups_x == 64
        rc, plan = R.reduction_plan(lib, 1, 64, op)
        if op == R.OP_SUM:
            assert plan.strategy != 3
        else:
            assert plan.strategy == 3


def test_planner_replay_id_is_fnv1a_over_stage_words(lib):
    rc, plan = R.reduction_plan(lib, 3, 2048, R.OP_SOFTMAX)
    assert rc == R.PROM_OK
    h = 1469598103934665603

    def mix(h, v):
        for i in range(4):
            h ^= (v >> (8 * i)) & 0xFF
            h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
        return h

    for v in (plan.operation, plan.row_count, plan.elements_per_row, plan.strategy, plan.partial_count,
              plan.stage_count):
        h = mix(h, v)
    for i in range(plan.stage_count):
        s = plan.stages[i]
        for v in (s.stage_role, s.shader_id, s.implementation_id, s.groups_x, s.input_elements_per_row,
                  s.output_partials_per_row, s.temporary_role, s.temporary_bytes_written & 0xFFFFFFFF,
                  s.temporary_bytes_written >> 32):
            h = mix(h, v)
    assert plan.replay_id == h
    # composed softmax: max partial/final, exp-sum partial/final, normalise
    assert [plan.stages[i].stage_role for i in range(plan.stage_count)] == [2, 2, 3, 1, 4]


def test_block_create_without_device_is_rejected(lib):
    h = _handle(lib, R.TESTCFG_FAIL_DEVICE_CREATE)
    try:
        cfg = R.OctB200BlockConfig()
        cfg.struct_size = C.sizeof(cfg)
        cfg.family, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim = 1, 512, 4, 1, 128
        cfg.ffn, cfg.seq_len, cfg.max_batch, cfg.tp_world = 1024, 128, 1, 1
        bid, detail = C.c_uint64(), C.c_int()
        rc = lib.oct_b200_block_create(h, C.byref(cfg), C.byref(bid), C.byref(detail))
        assert rc == R.PROM_ERROR and detail.value == -6006
        cfg.struct_size = 8  # too small: rejected before anything else
        rc = lib.oct_b200_block_create(h, C.byref(cfg), C.byref(bid), C.byref(detail))
        assert rc == R.PROM_ERROR and detail.value == -7010
    finally:
        lib.prometheus_reactor_runtime_destroy(h)


def test_tp_sgemm_create_is_validated_on_the_host(lib):
    """Configuration checks run before any device or NCCL work."""
    h = _handle(lib, R.TESTCFG_FAIL_DEVICE_CREATE)
    try:
        cfg = R.OctB200TpSgemmConfig()
        cfg.struct_size = 8  # too small
        tid, detail = C.c_uint64(), C.c_int()
        rc = lib.oct_b200_tp_sgemm_create(h, C.byref(cfg), C.byref(tid), C.byref(detail))
        assert rc == R.PROM_ERROR and detail.value == R.DETAIL_TP_INVALID
        cfg.struct_size = C.sizeof(cfg)
        cfg.rank, cfg.world, cfg.max_m, cfg.max_n = 0, 2, 64, 64
        rc = lib.oct_b200_tp_sgemm_create(h, C.byref(cfg), C.byref(tid), C.byref(detail))
        assert rc == R.PROM_ERROR and detail.value == -6006  # handle without a device
        rc = lib.oct_b200_sgemm_tp_device(h, 1, None, 0, None, 0, None, 0, 1, 8, 1, None, None, C.byref(detail))
        assert rc == R.PROM_ERROR and detail.value == R.DETAIL_TP_NOT_FOUND
        assert lib.oct_b200_tp_sgemm_destroy(h, 1) == R.PROM_ERROR
    finally:
        lib.prometheus_reactor_runtime_destroy(h)


def test_block_oracle_flops_match_baseline_accounting():
    from oracle import blocks as OB
    g = OB.gemma_config()
    per_token_linear = 2 * 2048 * 2560 + 2 * 2048 * 2048 + 3 * 2 * 2048 * 16384
    attn = 1024 * 1025 / 2 * 8 * 4 * 256 * 4
    assert OB.flops_per_forward(g, 4) == pytest.approx(4096 * per_token_linear + attn)
    d = OB.dit_config()
    assert OB.flops_per_forward(d, 2) == pytest.approx(8192 * (2 * 3072 * 9216 + 2 * 3072 * 3072 + 6 * 3072 * 8192)
                                                       + 4096 ** 2 * 24 * 512 * 2)


def test_diagnostics_entries_without_a_device(lib):
    """reactor_concept_reduction.cpp:96-110, reactor_sgemm.cpp:6371-6412,
    reactor_vulkan_fused_reduction.c:1122-1145: null outputs, handles, request checks."""
    assert lib.prometheus_reactor_runtime_reduction_diagnostics(None, None) == R.PROM_ERROR
    d = R.PrometheusReductionDiagnostics()
    assert lib.prometheus_reactor_runtime_reduction_diagnostics(None, C.byref(d)) == R.PROM_INVALID_HANDLE
    a = R.PrometheusSgemmAsyncDiagnostics()
    assert lib.prometheus_reactor_runtime_sgemm_async_diagnostics(None, C.byref(a)) == R.PROM_INVALID_HANDLE
    cfg = R.PrometheusReactorConfig()
    cfg.struct_size = C.sizeof(cfg)
    cfg.test_flags = R.TESTCFG_FAIL_DEVICE_CREATE
    cfg.reduction_ring_depth = 3
    h = C.c_void_p()
    assert lib.prometheus_reactor_runtime_create(C.byref(cfg), C.byref(h)) == R.PROM_OK
    try:
        assert lib.prometheus_reactor_runtime_reduction_diagnostics(h, C.byref(d)) == R.PROM_OK
        assert (d.struct_size, d.initialized, d.configured_ring_depth, d.total_requests) == (C.sizeof(d), 0, 3, 0)
        assert lib.prometheus_reactor_runtime_sgemm_async_diagnostics(h, C.byref(a)) == R.PROM_OK
        assert (a.task_capacity, a.active_task_count, a.queue_full_count) == (4, 0, 0)
        x = np.ones(8, np.float32)
        y = np.empty(2, np.float32)
        req = R.PrometheusReductionBenchmarkRequest()
        req.struct_size = C.sizeof(req)
        req.reduction = R.make_reduction_request(x, y, 2, 4, R.OP_SUM)
        res = R.PrometheusReductionBenchmarkResult()
        assert lib.prometheus_reactor_runtime_reduction_benchmark(h, C.byref(req), C.byref(res)) == R.PROM_ERROR
        assert res.detail_code == -6801 and res.first_mismatch_row == 0xFFFFFFFF  # no measured iterations
        req.measured_iterations = 3
        assert lib.prometheus_reactor_runtime_reduction_benchmark(h, C.byref(req), C.byref(res)) == R.PROM_ERROR
        assert res.detail_code == -6825 and res.completed_iterations == 0  # the device is unavailable
    finally:
        lib.prometheus_reactor_runtime_destroy(h)
