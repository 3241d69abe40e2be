"""Z-Image model-block executors on CPU: request validation and detail codes of
create / upload / execute (reactor_vulkan_model_block.c:393-477, 1603-1829,
2204-2303, 2305-2367), all of which precede device work."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from oct_b200 import reactor as R
from oracle import blocks as OB


@pytest.fixture()
def nodev(lib):
    cfg = R.PrometheusReactorConfig()
    cfg.struct_size = C.sizeof(cfg)
    cfg.test_flags = R.TESTCFG_FAIL_DEVICE_CREATE
    h = C.c_void_p()
    assert lib.prometheus_reactor_runtime_create(C.byref(cfg), C.byref(h)) == R.PROM_OK
    yield h
    lib.prometheus_reactor_runtime_destroy(h)


def _zero_payloads(context=False):
    return [np.zeros(s, np.float16) for s in OB.zimage_weight_shapes(context).values()]


def _noise_request(payloads, **over):
    req = R.PrometheusModelBlockCreateRequest()
    req.struct_size = C.sizeof(req)
    req.assembly_family, req.parameter_set = R.NOISE_REFINER_FAMILY, 1
    req.parameter_set_aggregate_identity = R.ZIMAGE_NOISE_AGGREGATES[0]
    req.model_contract_identity = req.weight_identity = req.shader_portfolio_identity = R.ZIMAGE_LOCK_ID
    req.precision_policy_identity = req.capability_route_identity = R.ZIMAGE_LOCK_ID
    req.memory_ceiling_bytes = 1 << 31
    req.external_input_bytes = 2 * 1024 * 3840
    req.audit_bytes = R.ZIMAGE_AUDIT_ARENA_BYTES
    req.shader_id, req.weight_count, req.step_count = 24, len(payloads), R.MODEL_BLOCK_MAX_STEPS
    for i, p in enumerate(payloads):
        req.weights[i].content_identity, req.weights[i].layout_identity = i + 1, i + 100
        req.weights[i].byte_count = p.nbytes
    for i in range(R.MODEL_BLOCK_MAX_STEPS):
        req.steps[i] = i + 1
    for k, v in over.items():
        setattr(req, k, v)
    return req


def _create(lib, h, req):
    bid, ev = C.c_uint64(99), R.PrometheusModelBlockEvidence()
    rc = lib.prometheus_reactor_runtime_model_block_create(h, C.byref(req), C.byref(bid), C.byref(ev))
    return rc, bid.value, ev


def test_manifest_matches_the_reference_byte_table():
    want = [30720, 7864320, 256, 29491200, 256, 88473600, 7680, 7680, 78643200, 78643200, 78643200, 7680, 7680]
    assert [int(np.prod(s)) * 2 for s in OB.zimage_weight_shapes().values()] == want
    assert [int(np.prod(s)) * 2 for s in OB.zimage_weight_shapes(True).values()] == want[2:]


def test_model_block_create_validation(lib, nodev):
    p = _zero_payloads()
    rc, bid, ev = _create(lib, nodev, _noise_request(p))
    assert (rc, bid, ev.detail_code) == (R.PROM_ERROR, 0, R.MB_RESOURCE_CREATE_FAILED)  # valid, but no device
    for over in ({"struct_size": 8}, {"parameter_set_aggregate_identity": 5}, {"parameter_set": 3},
                 {"shader_id": 25}, {"memory_ceiling_bytes": 100 << 20}, {"audit_bytes": 0},
                 {"external_input_bytes": 4}, {"step_count": 6}, {"assembly_family": 3}, {"weight_count": 12},
                 {"model_contract_identity": 0}):
        rc, bid, ev = _create(lib, nodev, _noise_request(p, **over))
        assert (rc, bid, ev.detail_code) == (R.PROM_ERROR, 0, R.MB_INVALID_REQUEST), over
        assert ev.struct_size == C.sizeof(ev) and ev.created == 0
    req = _noise_request(p)
    req.weights[3].byte_count += 2  # not the manifest's byte count
    assert _create(lib, nodev, req)[2].detail_code == R.MB_INVALID_REQUEST
    rc, _, ev = _create(lib, None, _noise_request(p))
    assert (rc, ev.detail_code) == (R.PROM_ERROR, R.MB_INVALID_REQUEST)


def test_refiner_entries_without_a_block(lib, nodev):
    ev = R.PrometheusModelBlockEvidence()
    ups = R.weight_uploads(_zero_payloads(True))
    cr = R.PrometheusContextRefinerCreateRequest()
    cr.struct_size = C.sizeof(cr)
    cr.lock_identity, cr.model_local_block_id, cr.upload_count, cr.uploads = R.ZIMAGE_LOCK_ID, 1, 11, ups
    bid = C.c_uint64()
    fn = lib.prometheus_reactor_runtime_context_refiner_create
    assert fn(nodev, C.byref(cr), C.byref(bid), C.byref(ev)) == R.PROM_ERROR
    assert ev.detail_code == R.MB_INVALID_REQUEST  # block 1 is a rebind target, not a create
    cr.model_local_block_id, cr.lock_identity = 0, 5
    assert fn(nodev, C.byref(cr), C.byref(bid), C.byref(ev)) == R.PROM_ERROR and ev.detail_code == R.MB_INVALID_REQUEST
    cr.lock_identity = R.ZIMAGE_LOCK_ID
    assert fn(nodev, C.byref(cr), C.byref(bid), C.byref(ev)) == R.PROM_ERROR
    assert ev.detail_code == R.MB_RESOURCE_CREATE_FAILED
    x = np.zeros(1024 * 3840, np.uint16)
    t = np.zeros(256, np.uint16)
    req = R.PrometheusNoiseRefiner0ExecuteRequest()
    req.struct_size = C.sizeof(req)
    req.model_input_bf16, req.timestep_bf16 = x.ctypes.data, t.ctypes.data
    req.model_input_bytes, req.timestep_bytes = x.nbytes, t.nbytes
    req.input_identity = req.timestep_identity = req.output_identity = 1
    ex = lib.prometheus_reactor_runtime_noise_refiner0_execute
    assert ex(nodev, 1, C.byref(req), C.byref(ev)) == R.PROM_ERROR
    assert ev.detail_code == R.MB_PARAMETER_SET_MISMATCH  # no block on this handle
    req.timestep_bytes = 510
    assert ex(nodev, 1, C.byref(req), C.byref(ev)) == R.PROM_ERROR and ev.detail_code == R.MB_INVALID_REQUEST
    req.timestep_bytes, req.audit_enabled = 512, 1
    assert ex(nodev, 1, C.byref(req), C.byref(ev)) == R.PROM_ERROR and ev.detail_code == R.MB_INVALID_REQUEST
    au = R.PrometheusNoiseRefinerFinalAuditRequest()
    au.struct_size = C.sizeof(au)
    out = np.empty(1024 * 3840, np.float32)
    au.output, au.output_element_capacity, au.output_identity, au.required_output_generation = (
        out.ctypes.data, out.size, 1, 1)
    assert lib.prometheus_reactor_runtime_noise_refiner_audit_final(nodev, 1, C.byref(au), C.byref(ev)) == R.PROM_ERROR
    assert ev.detail_code == R.MB_NOT_FOUND
    assert lib.prometheus_reactor_runtime_model_block_upload_weights(nodev, 1, ups, 11, C.byref(ev)) == R.PROM_ERROR
    assert ev.detail_code == R.MB_NOT_FOUND
    assert lib.prometheus_reactor_runtime_model_block_get_evidence(nodev, 1, None) == R.PROM_ERROR
    assert lib.prometheus_reactor_runtime_model_block_destroy(nodev, 1) == R.PROM_ERROR


def test_zimage_oracle_context_mode_is_the_unmodulated_block():
    """With zero adaLN weights and bias (scale 1, gate tanh(0) = 0 ...) the modulated path
    is not the context block; with the context flag the gates are exactly one."""
    w = OB.zimage_random_weights_f16(3, context=True)
    x = np.random.default_rng(1).standard_normal((32, 3840)).astype(np.float32)
    y = OB.zimage_refiner_forward(w, x, None, 32, context=True)
    assert y.shape == (32, 3840) and np.all(np.isfinite(y))
    assert np.linalg.norm(y - x) > 0.1 * np.linalg.norm(x)  # both residual branches contribute
