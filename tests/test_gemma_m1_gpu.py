"""Gemma M1 boundary on a B200: every entry point through the C ABI against the
CPU oracle (oracle.c, itself pinned to the reference's known-answer tests in
tests/test_gemma_m1_cpu.py).  Tolerances: the BF16-rounded outputs and the
binary64 score chain are bit-exact; the fp32 input RMSNorm is within 1e-5
relative of binary64 (and the reference's own 1e-4 absolute gate)."""
from __future__ import annotations

import numpy as np
import pytest

from oct_b200 import reactor as R

pytestmark = pytest.mark.gpu


@pytest.fixture()
def rt(lib):
    r = R.Runtime(lib)
    yield r
    r.close()


def _rope_fixture(o, heads):
    i = np.arange(3840)
    cos = o.bf16_round((0.5 + (i % 17).astype(np.float32) / np.float32(53)).astype(np.float32))
    sin = o.bf16_round((((i % 13) - 6).astype(np.float32) / np.float32(31)).astype(np.float32))
    j = np.arange(15 * heads * 256)
    src = o.bf16_round((((j * 17) % 83 - 41).astype(np.float32) / np.float32(79)).astype(np.float32))
    return src, cos, sin


def test_rope_reference_fixture_is_exact_and_warm_calls_reuse(rt, oracle_mod):
    """reactor_concept_rmsnorm_tests.cpp:336-372: heads 1, 8, 1; exact; warm repeats allocate nothing."""
    o = oracle_mod
    last = None
    for heads in (1, 8, 1):
        src, cos, sin = _rope_fixture(o, heads)
        rc, out, res = rt.gemma_rope(src, cos, sin, 15, heads, 256)
        assert rc == R.PROM_OK, res.detail_code
        assert np.array_equal(out, o.m1_rope(src, cos, sin, 15, heads, 256))
        assert res.dispatch_count == 1 and res.output_written == 1
        rc, out2, res2 = rt.gemma_rope(src, cos, sin, 15, heads, 256)
        assert rc == R.PROM_OK and res2.output_hash == res.output_hash and res2.buffer_allocation_count == 0
        if heads == 1 and last is not None:
            assert last == res.output_hash  # shrinking the capacity publishes no stale tail
        if heads == 1:
            last = res.output_hash


def test_rope_failures_leave_the_output_untouched(rt, oracle_mod):
    src, cos, sin = _rope_fixture(oracle_mod, 8)
    out = np.full(src.size, -99.0, np.float32)
    bad = sin.copy()
    bad[0] = np.inf
    rc, _, res = rt.gemma_rope(src, cos, bad, 15, 8, 256, out=out)
    assert rc == R.PROM_ERROR and res.detail_code == R.M46_NONFINITE_INPUT and res.output_written == 0
    assert np.all(out == -99.0)
    rc, _, res = rt.gemma_rope(src, cos, sin, 15, 8, 256, out=out)  # the handle stays usable
    assert rc == R.PROM_OK and np.array_equal(out, oracle_mod.m1_rope(src, cos, sin, 15, 8, 256))


def _score_fixture():
    i = np.arange(15 * 8 * 256)
    q = (((i * 13) % 61 - 30).astype(np.float32) / np.float32(71.0)).astype(np.float32)
    j = np.arange(15 * 256)
    k = (((j * 7) % 41 - 20).astype(np.float32) / np.float32(53.0)).astype(np.float32)
    w = (np.float32(0.75) + (np.arange(256) % 5).astype(np.float32) / np.float32(32)).astype(np.float32)
    return q, k, w, np.full(3840, 0.75, np.float32), np.full(3840, 0.5, np.float32)


def test_head_rmsnorm_rope_and_scores_match_the_oracle_bit_for_bit(rt, oracle_mod):
    """reactor_concept_rmsnorm_tests.cpp:146-179 at the M1 shapes, both preparation orders."""
    o = oracle_mod
    q, k, w, cos, sin = _score_fixture()
    rc, got_q, res = rt.gemma_head_rmsnorm_rope(q, w, cos, sin, 15, 8, 256)
    assert rc == R.PROM_OK, res.detail_code
    want_q = o.m1_head_rmsnorm_rope(q, w, cos, sin, 15, 8, 256)
    assert np.array_equal(got_q, want_q)
    assert res.normalized_readback_count == 0 and res.dispatch_count == 1
    want_k = o.m1_head_rmsnorm_rope(k, w, cos, sin, 15, 1, 256)
    want = o.m1_scores(want_q, want_k, 15, 8, 256, 0.0625)
    for order in (0, 1):
        rc, scores, sres = rt.gemma_attention_scores(q, k, w, w, cos, sin, 15, 8, 256, 0.0625, order=order)
        assert rc == R.PROM_OK, sres.detail_code
        assert np.array_equal(scores, want)
        assert (sres.positional_dispatch_count, sres.score_dispatch_count, sres.score_readback_count,
                sres.host_detour_count, sres.score_written) == (2, 1, 1, 0, 1)
        assert len({sres.query_slot_id, sres.key_slot_id, sres.score_slot_id}) == 3


def test_constant_vectors_give_scores_of_sixteen(rt):
    ones = np.ones(15 * 8 * 256, np.float32)
    w = np.ones(256, np.float32)
    rc, scores, res = rt.gemma_attention_scores(ones, ones[:3840].copy(), w, w, np.ones(3840, np.float32),
                                                np.zeros(3840, np.float32), 15, 8, 256, 0.0625)
    assert rc == R.PROM_OK, res.detail_code
    assert np.all(scores == 16.0)


def test_stale_weight_generation_is_rejected_before_any_dispatch(rt):
    q, k, w, cos, sin = _score_fixture()
    gen = rt.next_weight_generation() + 5
    rc, _, res = rt.gemma_head_rmsnorm_rope(q, w, cos, sin, 15, 8, 256, weight_generation=gen)
    assert rc == R.PROM_OK
    rc, _, res = rt.gemma_head_rmsnorm_rope(q, w, cos, sin, 15, 8, 256, weight_generation=gen)
    assert rc == R.PROM_ERROR and res.detail_code == R.M46_STALE_WEIGHT_GENERATION and res.dispatch_count == 0
    assert (res.observed_weight_generation, res.requested_weight_generation) == (gen, gen)
    rt._generation = gen  # the mirror's counter continues above the committed generation
    rc, _, res = rt.gemma_head_rmsnorm_rope(q, w, cos, sin, 15, 8, 256)
    assert rc == R.PROM_OK


@pytest.mark.parametrize("mode", ["input", "projection", "head"])
@pytest.mark.parametrize("width", [31, 1536, 4096])
def test_rmsnorm_family_reference_fixture(rt, oracle_mod, mode, width):
    """reactor_concept_rmsnorm_tests.cpp:75-125: strided rows, each BF16 boundary mode."""
    rows = 3
    stride = width if mode == "head" else width + 7
    i = np.arange(rows * stride)
    x = (((i * 7) % 31 - 15).astype(np.float32) / np.float32(63.0)).astype(np.float32)
    w = (np.float32(0.75) + (np.arange(width) % 7).astype(np.float32) / np.float32(64)).astype(np.float32)
    rc, y, inv, res = rt.rmsnorm(x, w, 1e-6, mode=mode, stride=stride, width=width, rows=rows)
    assert rc == R.PROM_OK, res.detail_code
    round_in, round_out = mode == "head", mode in ("projection", "head")
    want, want_inv = oracle_mod.m1_rmsnorm(x, w, 1e-6, round_in, round_out, stride=stride, rows=rows, width=width)
    if mode == "input":
        assert np.max(np.abs(y.ravel() - want)) < 1e-4  # the reference test's gate
        assert np.max(np.abs(y.ravel() - want) / np.maximum(np.abs(want), 1e-6)) <= 1e-5
        assert np.max(np.abs(inv - want_inv)) < 1e-5
    else:
        assert np.array_equal(y.ravel(), want)
        assert np.array_equal(inv, want_inv)
    assert res.output_written == 1 and res.submit_count == 1


def test_uncertain_completion_leaves_outputs_untouched(lib):
    """reactor_concept_rmsnorm_tests.cpp:281-312: an uncertain completion publishes nothing."""
    r = R.Runtime(lib, reduction_test_flags=R.REDUCTION_TESTCFG_FAIL_COMPLETION_OBSERVATION)
    try:
        x = np.ones((1, 4096), np.float32)
        w = np.ones(4096, np.float32)
        y = np.full((1, 4096), -99.0, np.float32)
        inv = np.full(1, -99.0, np.float32)
        import ctypes as C
        req = R.PrometheusGemma4E2BM1InputRmsNormRequest()
        req.struct_size = C.sizeof(req)
        req.input, req.weight, req.output, req.inv_rms_output = (x.ctypes.data, w.ctypes.data, y.ctypes.data,
                                                                 inv.ctypes.data)
        req.input_element_count = req.output_element_count = 4096
        req.weight_element_count, req.inv_rms_output_element_count = 4096, 1
        req.tokens, req.model_width, req.input_row_stride, req.epsilon = 1, 4096, 4096, 1e-6
        req.input_generation = req.weight_generation = req.exact_source_hash = 1
        res = R.PrometheusGemma4E2BM1InputRmsNormResult()
        rc = lib.prometheus_reactor_runtime_gemma4e2b_m1_input_rmsnorm(r.handle, C.byref(req), C.byref(res))
        assert rc == R.PROM_ERROR and res.detail_code == R.M46_COMPLETION_UNCERTAIN
        assert np.all(y == -99.0) and inv[0] == -99.0
    finally:
        r.close()


def test_widened_gemma_shapes_scores(rt, oracle_mod):
    """Beyond the reference's 15-token envelope: 256 tokens, 8 query heads of 256, bit-exact."""
    o = oracle_mod
    T, H, D = 256, 8, 256
    g = np.random.Generator(np.random.PCG64(3))
    q = g.standard_normal(T * H * D).astype(np.float32)
    k = g.standard_normal(T * D).astype(np.float32)
    wq = (1.0 + 0.02 * g.standard_normal(D)).astype(np.float32)
    wk = (1.0 + 0.02 * g.standard_normal(D)).astype(np.float32)
    pos = np.arange(T, dtype=np.float64)[:, None] * (10000.0 ** (-np.arange(D) % (D // 2) * 2.0 / D))[None, :]
    cos = o.bf16_round(np.cos(pos).astype(np.float32).ravel())
    sin = o.bf16_round(np.sin(pos).astype(np.float32).ravel())
    rc, scores, res = rt.gemma_attention_scores(q, k, wq, wk, cos, sin, T, H, D, 0.0625)
    assert rc == R.PROM_OK, res.detail_code
    want = o.m1_scores(o.m1_head_rmsnorm_rope(q, wq, cos, sin, T, H, D), o.m1_head_rmsnorm_rope(k, wk, cos, sin,
                                                                                                   T, 1, D),
                       T, H, D, 0.0625)
    assert np.array_equal(scores, want)
