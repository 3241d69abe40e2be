"""Gemma M1 boundary on CPU: the oracle pinned to the reference's own known-answer
tests, and the entry points' validation order and detail codes (no GPU needed:
every check here precedes device work).

Known answers: internal/prometheus/native/Marionette/reactor_concept_rmsnorm_tests.cpp
  * :75-125  RMSNorm at widths 31 / 1536 / 4096, row stride width + 7, every
             BF16 input / output rounding mode, against its double-sum oracle;
  * :146-179 head RMSNorm -> RoPE (cos 0.75, sin 0.5) and the score chain
             (binary64 dot * 0.0625);
  * :181-200 all-ones Q, K and weight with cos 1, sin 0: every score is 16;
  * :336-362 standalone RoPE: BF16 products and sums, exact.
Each expected value below is transcribed from those tests' own formulas in
plain Python (sequential binary64 / fp32 loops), independently of oracle.c.
"""
from __future__ import annotations

import ctypes as C
import math
import struct

import numpy as np
import pytest

from oct_b200 import reactor as R


def bf16(v: float) -> float:
    bits = struct.unpack("<I", struct.pack("<f", v))[0]
    bits = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
    return struct.unpack("<f", struct.pack("<I", bits))[0]


def f32(v: float) -> float:
    return float(np.float32(v))


def normalized(inp, weight, rows, stride, round_in, round_out, eps):
    """reactor_concept_rmsnorm_tests.cpp:17-35 in Python: binary64 sum, fp32 product."""
    width = len(weight)
    out, inv_all = [], []
    for r in range(rows):
        s = 0.0
        for c in range(width):
            x = bf16(inp[r * stride + c]) if round_in else inp[r * stride + c]
            s += x * x
        inv = f32(1.0 / math.sqrt(s / width + float(np.float32(eps))))
        inv_all.append(inv)
        for c in range(width):
            x = bf16(inp[r * stride + c]) if round_in else inp[r * stride + c]
            v = f32(f32(x * inv) * weight[c])
            out.append(bf16(v) if round_out else v)
    return np.array(out, np.float32), np.array(inv_all, np.float32)


def positional(inp, weight, heads):
    """reactor_concept_rmsnorm_tests.cpp:59-70: head norm, then RoPE with cos 0.75, sin 0.5."""
    norm, _ = normalized(inp, weight, 15 * heads, 256, True, True, 1e-6)
    out = np.empty_like(norm)
    for i in range(norm.size):
        comp = i % 256
        pair = i + 128 if comp < 128 else i - 128
        a, b = bf16(f32(float(norm[i]) * 0.75)), bf16(f32(float(norm[pair]) * 0.5))
        out[i] = bf16(f32(a - b) if comp < 128 else f32(a + b))
    return out


@pytest.mark.parametrize("width", [31, 1536, 4096])
@pytest.mark.parametrize("precision", [0, 1, 2, 3])
def test_m1_rmsnorm_oracle_matches_the_reference_test_oracle(oracle_mod, width, precision):
    rows, stride = 3, width + 7
    inp = [float(np.float32((int((i * 7) % 31) - 15) / 63.0)) for i in range(rows * stride)]
    weight = [float(np.float32(0.75 + float(i % 7) / 64)) for i in range(width)]
    round_in, round_out = bool(precision & 1), bool(precision >> 1)
    want, want_inv = normalized(inp, weight, rows, stride, round_in, round_out, 1e-6)
    got, inv = oracle_mod.m1_rmsnorm(np.array(inp, np.float32), np.array(weight, np.float32), 1e-6, round_in,
                                     round_out, stride=stride, rows=rows, width=width)
    assert np.array_equal(got, want)
    assert np.array_equal(inv, want_inv)


def _rope_fixture(heads):
    """reactor_concept_rmsnorm_tests.cpp:341-362: BF16-exact input and tables."""
    cos = np.array([bf16(f32(0.5 + float(i % 17) / 53)) for i in range(3840)], np.float32)
    sin = np.array([bf16(f32(float(int(i % 13) - 6) / 31)) for i in range(3840)], np.float32)
    src = np.array([bf16(f32(float(int((i * 17) % 83) - 41) / 79)) for i in range(15 * heads * 256)], np.float32)
    want = np.empty_like(src)
    for i in range(src.size):
        comp = i % 256
        pair = i + 128 if comp < 128 else i - 128
        table = (i // (heads * 256)) * 256 + comp % 128
        a = bf16(f32(float(src[i]) * float(cos[table])))
        b = bf16(f32(float(src[pair]) * float(sin[table])))
        want[i] = bf16(f32(a - b) if comp < 128 else f32(a + b))
    return src, cos, sin, want


@pytest.mark.parametrize("heads", [1, 8])
def test_m1_rope_oracle_is_exact_on_the_reference_fixture(oracle_mod, heads):
    src, cos, sin, want = _rope_fixture(heads)
    got = oracle_mod.m1_rope(src, cos, sin, 15, heads, 256)
    assert np.array_equal(got, want)  # the reference asserts max error 0.0


def _score_fixture():
    q = np.array([float(np.float32((int(i * 13 % 61) - 30) / 71.0)) for i in range(15 * 8 * 256)], np.float32)
    k = np.array([float(np.float32((int(i * 7 % 41) - 20) / 53.0)) for i in range(15 * 256)], np.float32)
    w = np.array([float(np.float32(0.75 + float(i % 5) / 32)) for i in range(256)], np.float32)
    cos = np.full(15 * 256, 0.75, np.float32)
    sin = np.full(15 * 256, 0.5, np.float32)
    return q, k, w, cos, sin


def test_m1_positional_and_score_oracles_match_the_reference_chain(oracle_mod):
    q, k, w, cos, sin = _score_fixture()
    want_q, want_k = positional(q.tolist(), w.tolist(), 8), positional(k.tolist(), w.tolist(), 1)
    got_q = oracle_mod.m1_head_rmsnorm_rope(q, w, cos, sin, 15, 8, 256)
    got_k = oracle_mod.m1_head_rmsnorm_rope(k, w, cos, sin, 15, 1, 256)
    assert np.array_equal(got_q, want_q) and np.array_equal(got_k, want_k)
    want = np.empty(8 * 15 * 15, np.float32)
    for h in range(8):
        for r in range(15):
            for c in range(15):
                dot = 0.0
                for d in range(256):
                    dot += float(want_q[(r * 8 + h) * 256 + d]) * float(want_k[c * 256 + d])
                want[(h * 15 + r) * 15 + c] = np.float32(dot * 0.0625)
    got = oracle_mod.m1_scores(got_q, got_k, 15, 8, 256, 0.0625)
    assert np.array_equal(got, want)
    # Go's own cpuGemma4e2bRawScores (fp32 loop) sits within the reference's 1e-3 gate
    go = oracle_mod.m1_scores(got_q, got_k, 15, 8, 256, 0.0625, form="go")
    assert np.max(np.abs(go - want)) < 1e-3


def test_m1_constant_vector_scores_are_sixteen(oracle_mod):
    ones = np.ones(15 * 8 * 256, np.float32)
    w = np.ones(256, np.float32)
    cos, sin = np.ones(15 * 256, np.float32), np.zeros(15 * 256, np.float32)
    q = oracle_mod.m1_head_rmsnorm_rope(ones, w, cos, sin, 15, 8, 256)
    k = oracle_mod.m1_head_rmsnorm_rope(ones[:15 * 256], w, cos, sin, 15, 1, 256)
    assert np.all(oracle_mod.m1_scores(q, k, 15, 8, 256, 0.0625) == 16.0)


# ---------------------------------------------------------------- validation without a device
@pytest.fixture()
def nodev(lib):
    cfg = R.PrometheusReactorConfig()
    cfg.struct_size = C.sizeof(cfg)
    cfg.test_flags = R.TESTCFG_FAIL_DEVICE_CREATE  # a handle whose device is unavailable
    h = C.c_void_p()
    assert lib.prometheus_reactor_runtime_create(C.byref(cfg), C.byref(h)) == R.PROM_OK
    yield h
    lib.prometheus_reactor_runtime_destroy(h)


def _rope_req(src, cos, sin, out, heads=8):
    r = R.PrometheusGemma4E2BM1RopeRequest()
    r.struct_size = C.sizeof(r)
    r.source, r.cosine, r.sine, r.output = src.ctypes.data, cos.ctypes.data, sin.ctypes.data, out.ctypes.data
    r.source_element_count, r.output_element_count = src.size, out.size
    r.cosine_element_count, r.sine_element_count = cos.size, sin.size
    r.tokens, r.heads, r.head_width = 15, heads, 256
    r.source_generation = r.table_generation = 1
    return r


def test_m1_rope_validation_order(lib, nodev):
    """reactor_concept_rmsnorm.cpp:157-176: handle, request, finiteness, then the device."""
    src, cos, sin, _ = _rope_fixture(8)
    out = np.full(src.size, -99.0, np.float32)
    res = R.PrometheusGemma4E2BM1RopeResult()
    fn = lib.prometheus_reactor_runtime_gemma4e2b_m1_rope
    assert fn(nodev, C.byref(_rope_req(src, cos, sin, out)), None) == R.PROM_ERROR
    assert fn(None, C.byref(_rope_req(src, cos, sin, out)), C.byref(res)) == R.PROM_INVALID_HANDLE
    assert res.detail_code == R.M46_INVALID_REQUEST and res.stage == R.STAGE_INIT
    alias = _rope_req(src, cos, sin, src)
    alias.output_element_count = src.size
    assert fn(nodev, C.byref(alias), C.byref(res)) == R.PROM_ERROR and res.detail_code == R.M46_INVALID_REQUEST
    short = _rope_req(src, cos, sin, out)
    short.sine_element_count -= 1
    assert fn(nodev, C.byref(short), C.byref(res)) == R.PROM_ERROR and res.detail_code == R.M46_INVALID_REQUEST
    wrong_heads = _rope_req(src, cos, sin, out, heads=2)  # element counts no longer match
    assert fn(nodev, C.byref(wrong_heads), C.byref(res)) == R.PROM_ERROR
    bad = sin.copy()
    bad[0] = np.inf
    assert fn(nodev, C.byref(_rope_req(src, cos, bad, out)), C.byref(res)) == R.PROM_ERROR
    assert res.detail_code == R.M46_NONFINITE_INPUT
    assert fn(nodev, C.byref(_rope_req(src, cos, sin, out)), C.byref(res)) == R.PROM_ERROR
    assert res.detail_code == R.M46_RESOURCE  # a valid request reaches the device check: no CPU fallback
    assert np.all(out == -99.0)


def test_m1_head_rope_and_score_validation(lib, nodev):
    q, k, w, cos, sin = _score_fixture()
    out = np.empty_like(q)
    req = R.PrometheusGemma4E2BM1HeadRmsNormRopeRequest()
    req.struct_size = C.sizeof(req)
    req.input, req.weight, req.cosine, req.sine, req.output = (q.ctypes.data, w.ctypes.data, cos.ctypes.data,
                                                               sin.ctypes.data, out.ctypes.data)
    req.input_element_count, req.weight_element_count, req.output_element_count = q.size, 256, q.size
    req.cosine_element_count = req.sine_element_count = 3840
    req.tokens, req.heads, req.head_width, req.epsilon = 15, 8, 256, 1e-6
    req.input_generation = req.weight_generation = req.table_generation = req.exact_source_hash = 1
    res = R.PrometheusGemma4E2BM1HeadRmsNormRopeResult()
    fn = lib.prometheus_reactor_runtime_gemma4e2b_m1_head_rmsnorm_rope
    assert fn(nodev, C.byref(req), C.byref(res)) == R.PROM_ERROR and res.detail_code == R.M46_RESOURCE
    req.epsilon = 1e-5  # the entry admits only the model's 1e-6
    assert fn(nodev, C.byref(req), C.byref(res)) == R.PROM_ERROR and res.detail_code == R.M46_INVALID_REQUEST
    req.epsilon = 1e-6
    req.output = None  # no readback requires a zero output count
    assert fn(nodev, C.byref(req), C.byref(res)) == R.PROM_ERROR and res.detail_code == R.M46_INVALID_REQUEST
    req.output_element_count = 0
    assert fn(None, C.byref(req), C.byref(res)) == R.PROM_INVALID_HANDLE
    req.exact_source_hash = 0
    assert fn(nodev, C.byref(req), C.byref(res)) == R.PROM_ERROR and res.detail_code == R.M46_INVALID_REQUEST

    scores = np.full(1800, -99.0, np.float32)
    sr = R.PrometheusGemma4E2BM1AttentionScoresRequest()
    sr.struct_size = C.sizeof(sr)
    sr.query_input, sr.key_input, sr.query_weight, sr.key_weight = (q.ctypes.data, k.ctypes.data, w.ctypes.data,
                                                                    w.ctypes.data)
    sr.cosine, sr.sine, sr.scores = cos.ctypes.data, sin.ctypes.data, scores.ctypes.data
    sr.query_input_element_count, sr.key_input_element_count = q.size, k.size
    sr.query_weight_element_count = sr.key_weight_element_count = 256
    sr.cosine_element_count = sr.sine_element_count = 3840
    sr.score_element_count = 1801  # malformed extent (reactor_concept_rmsnorm_tests.cpp:218-221)
    sr.tokens, sr.query_heads, sr.key_heads, sr.head_width = 15, 8, 1, 256
    sr.epsilon, sr.scale = 1e-6, 0.0625
    sr.query_input_generation, sr.key_input_generation, sr.table_generation = 1, 2, 1
    sr.query_weight_generation, sr.key_weight_generation = 2, 3
    sr.query_exact_source_hash, sr.key_exact_source_hash = 11, 12
    sres = R.PrometheusGemma4E2BM1AttentionScoresResult()
    fn = lib.prometheus_reactor_runtime_gemma4e2b_m1_attention_scores
    assert fn(nodev, C.byref(sr), C.byref(sres)) == R.PROM_ERROR and sres.detail_code == R.M46_INVALID_REQUEST
    sr.score_element_count = 1800
    sr.key_heads = 2
    assert fn(nodev, C.byref(sr), C.byref(sres)) == R.PROM_ERROR and sres.detail_code == R.M46_INVALID_REQUEST
    sr.key_heads = 1
    sr.preparation_order = 2
    assert fn(nodev, C.byref(sr), C.byref(sres)) == R.PROM_ERROR and sres.detail_code == R.M46_INVALID_REQUEST
    sr.preparation_order = 1
    # an invalid handle surfaces through the first preparation as PROM_ERROR (reactor_api.c:573-581)
    assert fn(None, C.byref(sr), C.byref(sres)) == R.PROM_ERROR and sres.positional_dispatch_count == 0
    assert fn(nodev, C.byref(sr), C.byref(sres)) == R.PROM_ERROR and sres.detail_code == R.M46_RESOURCE
    assert np.all(scores == -99.0)


def test_m1_rmsnorm_family_validation(lib, nodev):
    x = np.ones((4, 256), np.float32)
    w = np.ones(256, np.float32)
    y, inv = np.empty_like(x), np.empty(4, np.float32)
    req = R.PrometheusGemma4E2BM1InputRmsNormRequest()
    req.struct_size = C.sizeof(req)
    req.input, req.weight, req.output, req.inv_rms_output = (x.ctypes.data, w.ctypes.data, y.ctypes.data,
                                                             inv.ctypes.data)
    req.input_element_count = req.output_element_count = x.size
    req.weight_element_count, req.inv_rms_output_element_count = 256, 4
    req.tokens, req.model_width, req.input_row_stride, req.epsilon = 4, 256, 256, 1e-6
    req.input_generation = req.weight_generation = req.exact_source_hash = 1
    res = R.PrometheusGemma4E2BM1InputRmsNormResult()
    for name in ("input_rmsnorm", "projection_activation_rmsnorm", "head_rmsnorm"):
        fn = getattr(lib, f"prometheus_reactor_runtime_gemma4e2b_m1_{name}")
        assert fn(nodev, C.byref(req), C.byref(res)) == R.PROM_ERROR and res.detail_code == R.M46_RESOURCE
        assert fn(None, C.byref(req), C.byref(res)) == R.PROM_INVALID_HANDLE
        req.inv_rms_output = None
        assert fn(nodev, C.byref(req), C.byref(res)) == R.PROM_ERROR and res.detail_code == R.M46_INVALID_REQUEST
        req.inv_rms_output = inv.ctypes.data
        req.weight_generation = 0
        assert fn(nodev, C.byref(req), C.byref(res)) == R.PROM_ERROR and res.detail_code == R.M46_INVALID_REQUEST
        req.weight_generation = 1
        w[3] = np.nan
        assert fn(nodev, C.byref(req), C.byref(res)) == R.PROM_ERROR and res.detail_code == R.M46_NONFINITE_INPUT
        w[3] = 1.0
    head = lib.prometheus_reactor_runtime_gemma4e2b_m1_head_rmsnorm
    req.epsilon = 1e-5  # the head entry admits only 1e-6 (reactor_api.c:388)
    assert head(nodev, C.byref(req), C.byref(res)) == R.PROM_ERROR and res.detail_code == R.M46_INVALID_REQUEST
