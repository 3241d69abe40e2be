"""Z-Image model-block executors on a B200 against the binary64 oracle
(oracle/blocks.py zimage_refiner_forward, restating runCanonicalNoiseRefiner0 and
runCanonicalContextRefiner) at the reference dimensions: 1024 image tokens / 32
caption tokens of 3840, 30 heads of 128, SwiGLU 10240, binary16 weights.
Gates, as for the other block outputs: normwise <= 1e-4 and relative L2 <= 1e-5."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from oct_b200 import reactor as R
from oracle import blocks as OB

pytestmark = pytest.mark.gpu


def _close(got, want, what):
    got = np.asarray(got, np.float64).reshape(want.shape)
    normwise = np.max(np.abs(got - want)) / np.max(np.abs(want))
    l2 = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert normwise <= 1e-4 and l2 <= 1e-5, (what, normwise, l2)


def _timestep_bf16(t: float):
    emb = OB.timestep_embedding(t).astype(np.float32)
    return OB.bf16_values(emb)


def test_noise_refiner_chain_matches_the_oracle(lib):
    rt = R.Runtime(lib)
    mb = R.ModelBlock(rt)
    try:
        w0 = OB.zimage_random_weights_f16(11)
        w1 = OB.zimage_random_weights_f16(12)
        rng = np.random.Generator(np.random.PCG64(5))
        x, x16 = OB.bf16_values(rng.standard_normal((1024, 3840)).astype(np.float32))
        temb, t16 = _timestep_bf16(700.0)
        rc, ev = mb.create_noise_refiner(list(w0.values()))
        assert rc == R.PROM_OK, ev.detail_code
        assert (ev.weights_uploaded, ev.binding_state, ev.binding_generation, ev.weight_count) == (1, 1, 1, 13)
        rc, ev = mb.noise_execute(x16, t16, block=1)  # the block holds parameter set 0
        assert rc == R.PROM_ERROR and ev.detail_code == R.MB_PARAMETER_SET_MISMATCH
        rc, ev = mb.noise_execute(x16, t16)
        assert rc == R.PROM_OK, ev.detail_code
        assert (ev.output_valid, ev.output_generation) == (1, 1)
        rc, y0, ev = mb.audit_final(1024, 1)
        assert rc == R.PROM_OK, ev.detail_code
        _close(y0, OB.zimage_refiner_forward(w0, x, temb, 1024, context=False), "noise_refiner.0")
        assert mb.audit_final(1024, 2)[2].detail_code == R.MB_STALE_OUTPUT
        rc, ev = mb.execute_resident(1)  # block 1 needs its weights first
        assert rc == R.PROM_ERROR and ev.detail_code == R.MB_STALE_OUTPUT
        rc, ev = mb.noise_execute(x16, t16)  # a fresh external chain
        assert rc == R.PROM_OK and ev.output_generation == 2
        rc, ev = mb.rebind(list(w1.values()))
        assert rc == R.PROM_OK, ev.detail_code
        assert (ev.parameter_set, ev.parameter_set_aggregate_identity, ev.binding_generation) == (
            2, R.ZIMAGE_NOISE_AGGREGATES[1], 2)
        rc, ev = mb.execute_resident(1)  # not the resident output's generation
        assert rc == R.PROM_ERROR and ev.detail_code == R.MB_STALE_OUTPUT
        rc, ev = mb.execute_resident(2)
        assert rc == R.PROM_OK, ev.detail_code
        rc, y1, _ = mb.audit_final(1024, 3)
        assert rc == R.PROM_OK
        # block 1 on block 0's resident output (the device's own y0 isolates block 1)
        _close(y1, OB.zimage_refiner_forward(w1, y0, temb, 1024, context=False), "noise_refiner.1 resident")
        rc, ev = mb.execute_resident(2)  # the pinned predecessor again: the same output
        assert rc == R.PROM_OK and ev.output_generation == 4
        rc, y1b, _ = mb.audit_final(1024, 4)
        assert rc == R.PROM_OK and np.array_equal(y1, y1b)
        # one model block per handle
        rc, ev = R.ModelBlock(rt).create_noise_refiner(list(w0.values()))
        assert rc == R.PROM_ERROR and ev.detail_code == R.MB_ALREADY_CREATED
        assert mb.destroy() == R.PROM_OK
        ev = R.PrometheusModelBlockEvidence()
        assert lib.prometheus_reactor_runtime_model_block_get_evidence(rt.handle, 1, C.byref(ev)) == R.PROM_ERROR
    finally:
        rt.close()


def test_context_refiner_chain_matches_the_oracle(lib):
    rt = R.Runtime(lib)
    mb = R.ModelBlock(rt)
    try:
        w0 = OB.zimage_random_weights_f16(21, context=True)
        w1 = OB.zimage_random_weights_f16(22, context=True)
        x = np.random.Generator(np.random.PCG64(6)).standard_normal((32, 3840)).astype(np.float32)
        rc, ev = mb.create_context_refiner(list(w0.values()))
        assert rc == R.PROM_OK, ev.detail_code
        assert (ev.assembly_family, ev.parameter_set, ev.weight_count) == (R.CONTEXT_REFINER_FAMILY, 1, 11)
        rc, ev = mb.context_execute(x)
        assert rc == R.PROM_OK, ev.detail_code
        rc, y0, _ = mb.audit_final(32, 1, context=True)
        assert rc == R.PROM_OK
        _close(y0, OB.zimage_refiner_forward(w0, x, None, 32, context=True), "context_refiner.0")
        rc, ev = mb.rebind(list(w1.values()), context=True)
        assert rc == R.PROM_OK, ev.detail_code
        rc, ev = mb.execute_resident(1, context=True)
        assert rc == R.PROM_OK, ev.detail_code
        rc, y1, _ = mb.audit_final(32, 2, context=True)
        assert rc == R.PROM_OK
        _close(y1, OB.zimage_refiner_forward(w1, y0, None, 32, context=True), "context_refiner.1 resident")
    finally:
        rt.close()


def test_resident_identity_block(lib):
    """Family 0, shader 23: the resident proof copies input to output and the first
    audit elements to the audit buffer (resident_identity.sdslv)."""
    rt = R.Runtime(lib)
    try:
        payloads = [np.arange(100, dtype=np.float16), np.ones(40, np.float16)]
        ups = R.weight_uploads(payloads)
        req = R.PrometheusModelBlockCreateRequest()
        req.struct_size = C.sizeof(req)
        req.model_contract_identity = req.weight_identity = req.shader_portfolio_identity = 3
        req.precision_policy_identity = req.capability_route_identity = 3
        req.memory_ceiling_bytes = 1 << 20
        req.external_input_bytes = req.external_output_bytes = 4000
        req.audit_bytes = 256
        req.shader_id, req.weight_count, req.step_count = 23, 2, 7
        for i in range(2):
            req.weights[i].content_identity = ups[i].content_identity
            req.weights[i].layout_identity = ups[i].layout_identity
            req.weights[i].byte_count = ups[i].byte_count
        for i in range(7):
            req.steps[i] = i + 1
        bid, ev = C.c_uint64(), R.PrometheusModelBlockEvidence()
        assert lib.prometheus_reactor_runtime_model_block_create(rt.handle, C.byref(req), C.byref(bid),
                                                                 C.byref(ev)) == R.PROM_OK, ev.detail_code
        x = np.random.default_rng(2).standard_normal(1000).astype(np.float32)
        y = np.zeros_like(x)
        audit = np.full(64, -1.0, np.float32)
        ex = R.PrometheusModelBlockExecuteRequest()
        ex.struct_size = C.sizeof(ex)
        ex.input, ex.output, ex.element_count, ex.input_identity = x.ctypes.data, y.ctypes.data, 1000, 4
        ex.audit_enabled, ex.audit_output, ex.audit_element_capacity = 1, audit.ctypes.data, 64
        fn = lib.prometheus_reactor_runtime_model_block_execute
        assert fn(rt.handle, bid.value, C.byref(ex), C.byref(ev)) == R.PROM_ERROR
        assert ev.detail_code == R.MB_STALE_OUTPUT  # no weights yet
        assert lib.prometheus_reactor_runtime_model_block_upload_weights(rt.handle, bid.value, ups, 2,
                                                                         C.byref(ev)) == R.PROM_OK
        assert lib.prometheus_reactor_runtime_model_block_upload_weights(rt.handle, bid.value, ups, 2,
                                                                         C.byref(ev)) == R.PROM_ERROR
        assert ev.detail_code == R.MB_WEIGHT_MISMATCH  # uploaded once
        assert fn(rt.handle, bid.value, C.byref(ex), C.byref(ev)) == R.PROM_OK, ev.detail_code
        assert np.array_equal(y, x) and np.array_equal(audit, x[:64])
        assert (ev.output_valid, ev.audit_valid, ev.execution_count) == (1, 1, 1)
    finally:
        rt.close()
