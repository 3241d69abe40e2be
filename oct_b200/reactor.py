"""Host-side binding of ``libprometheus_reactor.so``, mirroring Oct's Go bridge.

Oct's Go host (internal/prometheus/bridge.go, bridge_dlopen_linux.go) finds the
reactor library, checks ``prometheus_reactor_abi_version() == 1``, resolves the
mandatory symbols, creates a runtime handle, probes it, and then calls
``SGEMM`` / the async family / the Gemma entry points.  This module does the
same through ctypes, with the same discovery order, issue codes and status
conventions, so the parity tests read like the reference's own bridge tests.

There is no CPU fallback: if the library or a usable B200 is missing, every
constructor raises :class:`ReactorIssue`.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Optional

import numpy as np

EXPECTED_ABI = 1
ENV_VAR = "OCT_PROMETHEUS_REACTOR"  # bridge.go:13
LIB_NAME = "libprometheus_reactor.so"

# ---- constants (include/prometheus_reactor.h) --------------------------------
PROM_OK, PROM_ERROR, PROM_INVALID_HANDLE, PROM_INTERNAL_ERROR = 0, 1, 2, 3
PROM_BACKEND_VULKAN = 2
STAGE_NONE, STAGE_INIT, STAGE_TRANSFER_IN, STAGE_SUBMIT, STAGE_TRANSFER_OUT, STAGE_CLEANUP = range(6)
ASYNC_IDLE, ASYNC_SUBMITTED, ASYNC_READY, ASYNC_FAILED, ASYNC_CONSUMED = range(5)

TESTCFG_FAIL_DEVICE_CREATE = 1 << 0
TESTCFG_FAIL_BUFFER_ALLOC = 1 << 2
TESTCFG_FAIL_UPLOAD = 1 << 3
TESTCFG_FAIL_DISPATCH = 1 << 4
TESTCFG_FAIL_DOWNLOAD = 1 << 5
TESTCFG_FAIL_ASYNC_POLL = 1 << 15
TESTCFG_FORCE_STRICT_FP32 = 1 << 17
RESIDENT_MODE_PRODUCTION_SELECTOR, RESIDENT_MODE_EXPLICIT_VARIANT = 0, 1
RESIDENT_FLAG_VALIDATE_READBACK, RESIDENT_FLAG_M29_SUBMISSION_RING = 1 << 0, 1 << 1
BATCH_FLAG_PARTITION_CONTIGUOUS = 1 << 8
DETAIL_BATCH_PLAN_INVALID, DETAIL_BATCH_EXECUTION_FAILED, DETAIL_BATCH_UNSUPPORTED_OPTION = -6602, -6604, -6613
DETAIL_PATH_STAGED_UPLOAD_TILED = 6106
DETAIL_BAD_VARIANT = -7004
DETAIL_DEVICE_TIMEOUT = -7002  # a bounded in-kernel wait gave up
DETAIL_NOALLOC_TOO_LARGE = -7006  # product needs more than the no-alloc entry's fixed scratch
DETAIL_INVALID_ARGUMENT = -7008  # null pointer, short leading dimension or out-of-range argument
M46_INVALID_REQUEST, M46_STALE_WEIGHT_GENERATION, M46_RESOURCE = -7401, -7406, -7411
M46_COMPLETION_UNCERTAIN, M46_READBACK, M46_NONFINITE_INPUT = -7414, -7416, -7418
REDUCTION_TESTCFG_FAIL_COMMAND_RECORD = 1 << 0
REDUCTION_TESTCFG_FAIL_QUEUE_SUBMIT = 1 << 1
REDUCTION_TESTCFG_FAIL_COMPLETION_OBSERVATION = 1 << 2

DETAIL_PATH_DIRECT = 6101
DETAIL_INJECTED_UPLOAD_FAILURE = -6001
DETAIL_INJECTED_DISPATCH_FAILURE = -6002
DETAIL_INJECTED_DOWNLOAD_FAILURE = -6003
DETAIL_SIZE_OVERFLOW = -6004
DETAIL_ASYNC_NOT_READY = -6108
DETAIL_ASYNC_NO_TASK = -6109
DETAIL_ASYNC_ALREADY_CONSUMED = -6110
DETAIL_ASYNC_INVALID_TASK = -6111
DETAIL_ASYNC_INJECTED_POLL_FAILURE = -6116
DETAIL_ASYNC_QUEUE_FULL = -6117

OP_SUM, OP_MAX, OP_SOFTMAX = 1, 2, 3
FINALIZATION_NONE, FINALIZATION_STABLE_SOFTMAX = 0, 1
SGEMM_AUTO, SGEMM_TC3XTF32, SGEMM_FMA, SGEMM_SMALLM = 0, 1, 2, 3
SGEMM_TC_BK16, SGEMM_TC_BK32 = 16, 32  # explicit tensor-core stage depths, one CTA per tile
SGEMM_TC_PAIR16, SGEMM_TC_PAIR32 = 216, 232  # CTA-pair (cta_group::2) 256x256 tiles
SGEMM_TC_INSM16, SGEMM_TC_INSM32 = 316, 332  # CTA pair, TF32 split inside the kernel (no split pass)
SGEMM_SMALLM_TC = 4  # m <= 16 on the tensor cores, TF32 split inside the kernel

MAX_STAGES = 8


# ---- ABI structs (byte-compatible with the C header) -------------------------
class PrometheusCaps(C.Structure):
    _fields_ = [("available", C.c_uint32), ("backend_type", C.c_uint32), ("reason_code", C.c_uint32)]


class PrometheusReactorConfig(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("test_flags", C.c_uint32),
        ("p15_shadow_disabled", C.c_uint32),
        ("async_test_flags", C.c_uint32),
        ("batch_ring_depth", C.c_uint32),
        ("reduction_test_flags", C.c_uint32),
        ("reduction_ring_depth", C.c_uint32),
        ("shader_package_root", C.c_char_p),
    ]


class PrometheusSgemmBatchEntry(C.Structure):
    """reactor_api.h:1307-1314."""
    _fields_ = [("a", C.c_void_p), ("b", C.c_void_p), ("c", C.c_void_p), ("m", C.c_uint32), ("n", C.c_uint32),
                ("k", C.c_uint32)]


class PrometheusSgemmResidentBenchmarkRequest(C.Structure):
    """reactor_api.h:2034-2050."""
    _fields_ = [("struct_size", C.c_uint32), ("a", C.c_void_p), ("b", C.c_void_p), ("c", C.c_void_p),
                ("m", C.c_uint32), ("n", C.c_uint32), ("k", C.c_uint32), ("mode", C.c_uint32),
                ("requested_variant", C.c_uint32), ("warmup_iterations", C.c_uint32), ("iterations", C.c_uint32),
                ("diagnostic_batch_depth", C.c_uint32), ("flags", C.c_uint32)]


class PrometheusSgemmResidentBenchmarkResult(C.Structure):
    """reactor_api.h:2052-2095."""
    _fields_ = [(name, C.c_uint32) for name in (
        "struct_size", "resident_mode_available", "resident_mode_used", "requested_variant",
        "production_selected_variant", "executed_variant", "executed_compute_mode", "setup_stage")] + [
        ("setup_detail_code", C.c_int32), ("final_stage", C.c_uint32), ("final_detail_code", C.c_int32),
        ("iterations", C.c_uint32), ("gpu_timestamp_valid", C.c_uint32), ("gpu_timing_failure_reason", C.c_uint32)] + [
        (name, C.c_uint64) for name in (
            "setup_wall_ns", "upload_once_wall_ns", "total_loop_wall_ns", "kernel_min_ns", "kernel_median_ns",
            "kernel_p95_ns", "readback_once_wall_ns", "validation_wall_ns", "dispatch_submit_wall_ns_median",
            "sync_wait_wall_ns_median")] + [
        (name, C.c_uint32) for name in (
            "diagnostic_batch_depth", "queue_submissions", "fence_waits", "command_buffer_recordings",
            "command_buffer_resets", "descriptor_updates")] + [
        ("query_result_wall_ns_median", C.c_uint64), ("configured_ring_depth", C.c_uint32),
        ("physical_slot_count", C.c_uint32), ("max_in_flight_depth", C.c_uint32)] + [
        (name, C.c_uint64) for name in (
            "ring_poll_count", "ring_forced_wait_count", "ring_query_harvest_count", "ring_full_count",
            "ring_slot_recycle_count", "ring_failure_count")] + [
        ("ring_final_slot_state", C.c_uint32 * 4)]


class PrometheusAsyncStatus(C.Structure):
    _fields_ = [
        ("lifecycle_state", C.c_uint32),
        ("stage", C.c_uint32),
        ("detail_code", C.c_int),
        ("ready", C.c_uint32),
        ("failed", C.c_uint32),
        ("consumed", C.c_uint32),
        ("outstanding_tasks", C.c_uint32),
    ]


class PrometheusReductionRequest(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("input", C.c_void_p),
        ("output", C.c_void_p),
        ("row_count", C.c_uint32),
        ("elements_per_row", C.c_uint32),
        ("input_element_count", C.c_uint64),
        ("output_element_count", C.c_uint64),
        ("operation", C.c_uint32),
        ("finalization", C.c_uint32),
        ("flags", C.c_uint32),
    ]


class PrometheusReductionStageDispatch(C.Structure):
    _fields_ = [
        ("stage_role", C.c_uint32),
        ("shader_id", C.c_uint32),
        ("implementation_id", C.c_uint32),
        ("groups_x", C.c_uint32),
        ("groups_y", C.c_uint32),
        ("groups_z", C.c_uint32),
        ("input_elements_per_row", C.c_uint32),
        ("output_partials_per_row", C.c_uint32),
        ("temporary_role", C.c_uint32),
        ("temporary_bytes_written", C.c_uint64),
    ]


class PrometheusReductionPlan(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("operation", C.c_uint32),
        ("row_count", C.c_uint32),
        ("elements_per_row", C.c_uint32),
        ("strategy", C.c_uint32),
        ("local_size", C.c_uint32),
        ("elements_per_partial", C.c_uint32),
        ("partial_count", C.c_uint32),
        ("stage_count", C.c_uint32),
        ("temporary_alignment_bytes", C.c_uint32),
        ("temporary_bytes", C.c_uint64),
        ("replay_id", C.c_uint64),
        ("stages", PrometheusReductionStageDispatch * MAX_STAGES),
    ]


class PrometheusReductionExecutionResult(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("stage", C.c_uint32),
        ("detail_code", C.c_int32),
        ("logical_request_id", C.c_uint64),
        ("physical_slot_id", C.c_uint32),
        ("physical_slot_generation", C.c_uint32),
        ("physical_slot_recyclable", C.c_uint32),
        ("gpu_timestamp_valid", C.c_uint32),
        ("gpu_duration_ns", C.c_uint64),
        ("end_to_end_ns", C.c_uint64),
        ("first_nonfinite_index", C.c_uint64),
        ("validation_error_count_before", C.c_uint32),
        ("validation_error_count_after", C.c_uint32),
        ("plan", PrometheusReductionPlan),
    ]


class PrometheusRowWiseSoftmaxRequest(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("input", C.c_void_p),
        ("output", C.c_void_p),
        ("row_count", C.c_uint32),
        ("elements_per_row", C.c_uint32),
        ("input_element_count", C.c_uint64),
        ("output_element_count", C.c_uint64),
    ]


class PrometheusRowWiseSoftmaxResult(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("stage", C.c_uint32),
        ("detail_code", C.c_int32),
        ("output_written", C.c_uint32),
        ("physical_dispatch_count", C.c_uint32),
        ("physical_submission_count", C.c_uint32),
        ("gpu_timestamp_valid", C.c_uint32),
        ("gpu_duration_ns", C.c_uint64),
        ("end_to_end_ns", C.c_uint64),
        ("first_nonfinite_index", C.c_uint64),
    ]


class PrometheusGemma4E2BM1InputRmsNormRequest(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("input", C.c_void_p),
        ("weight", C.c_void_p),
        ("output", C.c_void_p),
        ("inv_rms_output", C.c_void_p),
        ("input_element_count", C.c_uint64),
        ("weight_element_count", C.c_uint64),
        ("output_element_count", C.c_uint64),
        ("inv_rms_output_element_count", C.c_uint64),
        ("tokens", C.c_uint32),
        ("model_width", C.c_uint32),
        ("input_row_stride", C.c_uint32),
        ("epsilon", C.c_float),
        ("input_generation", C.c_uint64),
        ("weight_generation", C.c_uint64),
        ("exact_source_hash", C.c_uint64),
    ]


class PrometheusGemma4E2BM1InputRmsNormResult(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("stage", C.c_uint32),
        ("detail_code", C.c_int32),
        ("output_written", C.c_uint32),
        ("matched_input", C.c_uint32),
        ("input_hash", C.c_uint64),
        ("weight_hash", C.c_uint64),
        ("output_hash", C.c_uint64),
        ("inv_rms_hash", C.c_uint64),
        ("submit_count", C.c_uint32),
        ("final_readback_count", C.c_uint32),
        ("no_product_intermediate_readback_change", C.c_uint32),
        ("reserved0", C.c_uint32),
        ("retained_bytes", C.c_uint64),
        ("buffer_allocation_count", C.c_uint64),
        ("buffer_reuse_count", C.c_uint64),
        ("descriptor_update_count", C.c_uint64),
        ("pipeline_create_count", C.c_uint64),
        ("command_buffer_reuse_count", C.c_uint64),
        ("reduction_gpu_ns", C.c_uint64),
        ("final_reduction_gpu_ns", C.c_uint64),
        ("inv_rms_gpu_ns", C.c_uint64),
        ("apply_gpu_ns", C.c_uint64),
        ("end_to_end_ns", C.c_uint64),
    ]


class PrometheusReductionDiagnostics(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "struct_size", "initialized", "production_enabled", "experimental_enabled", "configured_ring_depth",
        "physical_slot_count", "acquire_cursor", "outstanding_slots", "quarantined_slots")] + [
        (n, C.c_uint64) for n in (
            "next_logical_request_id", "total_requests", "successful_requests", "logical_failure_count",
            "physical_recycle_count", "quarantine_count", "reap_count", "pipeline_create_count",
            "descriptor_update_count", "command_record_count", "queue_submit_count", "buffer_allocation_count",
            "buffer_reuse_count", "temporary_capacity_bytes", "last_replay_id", "last_gpu_duration_ns",
            "last_end_to_end_ns")] + [
        ("last_stage_count", C.c_uint32), ("last_physical_slot_id", C.c_uint32),
        ("last_physical_slot_generation", C.c_uint32), ("last_detail_code", C.c_int32),
        ("validation_enabled", C.c_uint32), ("validation_error_count", C.c_uint32)]


class PrometheusReductionBenchmarkRequest(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("reduction", PrometheusReductionRequest),
                ("warmup_iterations", C.c_uint32), ("measured_iterations", C.c_uint32)]


class PrometheusReductionBenchmarkResult(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "struct_size", "completed_iterations", "correctness_passed", "validation_passed", "device_lost",
        "stage_count")] + [(n, C.c_uint64) for n in (
            "temporary_bytes", "replay_id", "gpu_min_ns", "gpu_median_ns", "gpu_max_ns", "end_to_end_min_ns",
            "end_to_end_median_ns", "end_to_end_max_ns")] + [
        ("first_mismatch_row", C.c_uint32), ("first_mismatch_column", C.c_uint32), ("first_expected", C.c_float),
        ("first_actual", C.c_float), ("first_absolute_error", C.c_float), ("first_relative_error", C.c_float),
        ("detail_code", C.c_int32)]


class PrometheusSgemmAsyncTaskDiagnostics(C.Structure):
    _fields_ = [("task_id", C.c_int32), ("generation", C.c_uint32), ("lifecycle_state", C.c_uint32),
                ("physical_slot_id", C.c_uint32), ("physical_slot_generation", C.c_uint32),
                ("submission_sequence", C.c_uint64), ("timing_valid", C.c_uint32), ("gpu_duration_ns", C.c_uint64),
                ("feedback_pending", C.c_uint32), ("feedback_committed", C.c_uint32), ("failure_detail", C.c_int32),
                ("failure_class", C.c_uint32), ("abandoned", C.c_uint32), ("physical_slot_state", C.c_uint32),
                ("quarantined", C.c_uint32), ("physical_completion_confirmed", C.c_uint32),
                ("reap_pending", C.c_uint32), ("reap_completed", C.c_uint32)]


class PrometheusSgemmAsyncDiagnostics(C.Structure):
    _fields_ = [("task_capacity", C.c_uint32), ("active_task_count", C.c_uint32), ("submitted_count", C.c_uint32),
                ("ready_count", C.c_uint32), ("failed_count", C.c_uint32), ("consumed_count", C.c_uint32),
                ("abandoned_count", C.c_uint32), ("queue_full_count", C.c_uint64),
                ("stale_id_rejection_count", C.c_uint64), ("max_in_flight", C.c_uint32),
                ("feedback_pending_count", C.c_uint32), ("feedback_committed_count", C.c_uint64),
                ("feedback_skipped_count", C.c_uint64), ("next_feedback_sequence", C.c_uint64),
                ("quarantined_slot_count", C.c_uint32), ("quarantine_event_count", C.c_uint64),
                ("reap_poll_count", C.c_uint64), ("reap_success_count", C.c_uint64), ("reap_wait_count", C.c_uint64),
                ("reap_failure_count", C.c_uint64), ("max_quarantine_depth", C.c_uint32),
                ("runtime_unsafe_to_reuse", C.c_uint32), ("tasks", PrometheusSgemmAsyncTaskDiagnostics * 4)]


class PrometheusGemma4E2BM1RopeRequest(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("source", C.c_void_p), ("cosine", C.c_void_p), ("sine", C.c_void_p), ("output", C.c_void_p),
        ("source_element_count", C.c_uint64), ("cosine_element_count", C.c_uint64),
        ("sine_element_count", C.c_uint64), ("output_element_count", C.c_uint64),
        ("tokens", C.c_uint32), ("heads", C.c_uint32), ("head_width", C.c_uint32), ("reserved0", C.c_uint32),
        ("source_generation", C.c_uint64), ("table_generation", C.c_uint64),
    ]


class PrometheusGemma4E2BM1RopeResult(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32), ("stage", C.c_uint32), ("detail_code", C.c_int32),
        ("output_written", C.c_uint32), ("dispatch_count", C.c_uint32),
        ("source_hash", C.c_uint64), ("cosine_hash", C.c_uint64), ("sine_hash", C.c_uint64),
        ("output_hash", C.c_uint64), ("buffer_allocation_count", C.c_uint64), ("buffer_reuse_count", C.c_uint64),
        ("descriptor_update_count", C.c_uint64), ("pipeline_create_count", C.c_uint64),
        ("command_buffer_reuse_count", C.c_uint64),
    ]


class PrometheusGemma4E2BM1HeadRmsNormRopeRequest(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("input", C.c_void_p), ("weight", C.c_void_p), ("cosine", C.c_void_p), ("sine", C.c_void_p),
        ("output", C.c_void_p),
        ("input_element_count", C.c_uint64), ("weight_element_count", C.c_uint64),
        ("cosine_element_count", C.c_uint64), ("sine_element_count", C.c_uint64),
        ("output_element_count", C.c_uint64),
        ("tokens", C.c_uint32), ("heads", C.c_uint32), ("head_width", C.c_uint32), ("reserved0", C.c_uint32),
        ("epsilon", C.c_float),
        ("input_generation", C.c_uint64), ("weight_generation", C.c_uint64), ("table_generation", C.c_uint64),
        ("exact_source_hash", C.c_uint64),
    ]


class PrometheusGemma4E2BM1HeadRmsNormRopeResult(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32), ("stage", C.c_uint32), ("detail_code", C.c_int32),
        ("output_written", C.c_uint32), ("dispatch_count", C.c_uint32), ("resident_source_bound", C.c_uint32),
        ("normalized_readback_count", C.c_uint32),
        ("source_byte_offset", C.c_uint64), ("source_byte_range", C.c_uint64),
        ("destination_byte_offset", C.c_uint64), ("destination_byte_range", C.c_uint64),
        ("input_hash", C.c_uint64), ("weight_hash", C.c_uint64), ("output_hash", C.c_uint64),
        ("buffer_allocation_count", C.c_uint64), ("buffer_reuse_count", C.c_uint64),
        ("descriptor_update_count", C.c_uint64), ("pipeline_create_count", C.c_uint64),
        ("command_buffer_reuse_count", C.c_uint64),
        ("observed_weight_generation", C.c_uint64), ("requested_weight_generation", C.c_uint64),
    ]


class PrometheusGemma4E2BM1AttentionScoresRequest(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("query_input", C.c_void_p), ("key_input", C.c_void_p), ("query_weight", C.c_void_p),
        ("key_weight", C.c_void_p), ("cosine", C.c_void_p), ("sine", C.c_void_p), ("scores", C.c_void_p),
        ("query_input_element_count", C.c_uint64), ("key_input_element_count", C.c_uint64),
        ("query_weight_element_count", C.c_uint64), ("key_weight_element_count", C.c_uint64),
        ("cosine_element_count", C.c_uint64), ("sine_element_count", C.c_uint64),
        ("score_element_count", C.c_uint64),
        ("tokens", C.c_uint32), ("query_heads", C.c_uint32), ("key_heads", C.c_uint32), ("head_width", C.c_uint32),
        ("epsilon", C.c_float), ("scale", C.c_float), ("preparation_order", C.c_uint32),
        ("query_input_generation", C.c_uint64), ("key_input_generation", C.c_uint64),
        ("query_weight_generation", C.c_uint64), ("key_weight_generation", C.c_uint64),
        ("table_generation", C.c_uint64), ("query_exact_source_hash", C.c_uint64),
        ("key_exact_source_hash", C.c_uint64),
    ]


class PrometheusGemma4E2BM1AttentionScoresResult(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32), ("stage", C.c_uint32), ("detail_code", C.c_int32),
        ("score_written", C.c_uint32), ("positional_dispatch_count", C.c_uint32),
        ("score_dispatch_count", C.c_uint32), ("score_readback_count", C.c_uint32),
        ("host_detour_count", C.c_uint32), ("query_slot_id", C.c_uint32), ("query_slot_generation", C.c_uint32),
        ("key_slot_id", C.c_uint32), ("key_slot_generation", C.c_uint32), ("score_slot_id", C.c_uint32),
        ("score_slot_generation", C.c_uint32),
        ("query_byte_range", C.c_uint64), ("key_byte_range", C.c_uint64), ("score_byte_range", C.c_uint64),
        ("score_hash", C.c_uint64), ("buffer_allocation_count", C.c_uint64), ("buffer_reuse_count", C.c_uint64),
        ("descriptor_update_count", C.c_uint64), ("pipeline_create_count", C.c_uint64),
        ("observed_weight_generation", C.c_uint64), ("requested_weight_generation", C.c_uint64),
    ]


MODEL_BLOCK_MAX_WEIGHTS, MODEL_BLOCK_MAX_STEPS = 13, 7
NOISE_REFINER_FAMILY, CONTEXT_REFINER_FAMILY = 1, 2
ZIMAGE_LOCK_ID = 0x71ef202b4e34b562
ZIMAGE_NOISE_AGGREGATES = (0xa1ba526898a2a752, 0x80c0cd75f44cc434)
ZIMAGE_AUDIT_ARENA_BYTES = 47186176
MB_INVALID_REQUEST, MB_NOT_FOUND, MB_ALREADY_CREATED, MB_WEIGHT_MISMATCH = -6901, -6902, -6903, -6904
MB_RESOURCE_CREATE_FAILED, MB_AUDIT_FAILED, MB_STALE_OUTPUT = -6905, -6911, -6912
MB_PARAMETER_SET_MISMATCH, MB_REBIND_FAILED = -6920, -6921


FFT_FLAG_FORWARD, FFT_FLAG_INVERSE, FFT_FLAG_INVERSE_NORMALIZE = 1, 2, 4
FFT_PATH_UNAVAILABLE, FFT_PATH_RADIX2 = 1, 3


class PrometheusFftRequest(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("input", C.c_void_p), ("output", C.c_void_p),
                ("element_count", C.c_uint32), ("batch_count", C.c_uint32), ("stride_elements", C.c_uint32),
                ("flags", C.c_uint32)]


class PrometheusFftDiagnostics(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "struct_size", "api_declared", "capability_reported", "production_enabled", "benchmark_enabled",
        "last_element_count", "last_batch_count", "last_stride_elements", "last_effective_stride_elements",
        "last_flags", "last_direction", "last_validation_status")] + [("last_failure_detail", C.c_int32)] + [
        (n, C.c_uint32) for n in ("requested_path_id", "executed_path_id", "requested_radix", "executed_radix",
                                  "fallback_reason", "plan_pass_count", "ping_pong_swap_count",
                                  "final_output_role")] + [
        (n, C.c_uint64) for n in ("ping_arena_reuse_count", "ping_arena_grow_count", "pong_arena_reuse_count",
                                  "pong_arena_grow_count", "twiddle_arena_reuse_count",
                                  "twiddle_arena_grow_count")] + [
        (n, C.c_uint32) for n in ("selector_cache_valid", "plan_valid", "plan_element_count",
                                  "plan_log2_element_count", "plan_first_span", "plan_last_span", "plan_radix_mask",
                                  "plan_bit_reversal_required", "plan_first_source_role",
                                  "plan_first_destination_role", "plan_direction", "plan_twiddle_mode")] + [
        (n, C.c_uint64) for n in ("selector_cache_reuse_count", "selector_cache_recompute_count",
                                  "selector_cache_invalidation_count", "selector_cache_last_dependency_mask")]


class PrometheusModelBlockWeightDeclaration(C.Structure):
    _fields_ = [("content_identity", C.c_uint64), ("layout_identity", C.c_uint64), ("byte_count", C.c_uint64)]


class PrometheusModelBlockCreateRequest(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("assembly_family", C.c_uint32), ("parameter_set", C.c_uint32)] + [
        (n, C.c_uint64) for n in ("parameter_set_aggregate_identity", "model_contract_identity", "weight_identity",
                                  "shader_portfolio_identity", "precision_policy_identity",
                                  "capability_route_identity", "memory_ceiling_bytes", "external_input_bytes",
                                  "external_output_bytes", "audit_bytes")] + [
        ("shader_id", C.c_uint32), ("weight_count", C.c_uint32),
        ("weights", PrometheusModelBlockWeightDeclaration * MODEL_BLOCK_MAX_WEIGHTS),
        ("step_count", C.c_uint32), ("steps", C.c_uint32 * MODEL_BLOCK_MAX_STEPS)]


class PrometheusModelBlockWeightUpload(C.Structure):
    _fields_ = [("binding_index", C.c_uint32), ("bytes", C.c_void_p), ("byte_count", C.c_uint64),
                ("content_identity", C.c_uint64), ("layout_identity", C.c_uint64)]


class PrometheusNoiseRefinerRebindRequest(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("model_local_block_id", C.c_uint32), ("lock_identity", C.c_uint64),
                ("upload_count", C.c_uint32), ("uploads", C.POINTER(PrometheusModelBlockWeightUpload))]


PrometheusContextRefinerCreateRequest = PrometheusNoiseRefinerRebindRequest  # same layout (reactor_api.h:842-848)


class PrometheusModelBlockExecuteRequest(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("input", C.c_void_p), ("output", C.c_void_p),
                ("element_count", C.c_uint64), ("input_identity", C.c_uint64), ("audit_enabled", C.c_uint32),
                ("audit_output", C.c_void_p), ("audit_element_capacity", C.c_uint64)]


class PrometheusNoiseRefiner0ExecuteRequest(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("model_input_bf16", C.c_void_p), ("timestep_bf16", C.c_void_p),
                ("model_input_bytes", C.c_uint64), ("timestep_bytes", C.c_uint64), ("input_identity", C.c_uint64),
                ("timestep_identity", C.c_uint64), ("output_identity", C.c_uint64), ("audit_enabled", C.c_uint32)]


class PrometheusNoiseRefinerResidentExecuteRequest(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("input_generation", C.c_uint64), ("output_identity", C.c_uint64),
                ("audit_enabled", C.c_uint32), ("audit_family", C.c_uint32), ("audit_stage", C.c_uint32),
                ("audit_output", C.c_void_p), ("audit_element_capacity", C.c_uint64)]


class PrometheusContextRefiner0ExecuteRequest(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("context_input", C.c_void_p), ("context_input_bytes", C.c_uint64),
                ("input_identity", C.c_uint64), ("output_identity", C.c_uint64), ("audit_enabled", C.c_uint32)]


class PrometheusContextRefinerResidentExecuteRequest(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("input_generation", C.c_uint64), ("output_identity", C.c_uint64),
                ("audit_enabled", C.c_uint32)]


class PrometheusNoiseRefinerFinalAuditRequest(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("required_output_generation", C.c_uint64),
                ("output_identity", C.c_uint64), ("output", C.c_void_p), ("output_element_capacity", C.c_uint64)]


class PrometheusModelBlockEvidence(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("struct_size",)] + [("detail_code", C.c_int32)] + [
        (n, C.c_uint32) for n in ("created", "weights_uploaded", "quarantined", "output_valid", "audit_valid",
                                  "fixed_step_count", "weight_count")] + [
        (n, C.c_uint64) for n in ("persistent_bytes", "reusable_bytes", "audit_bytes", "external_bytes",
                                  "total_committed_bytes", "peak_plan_bytes", "cold_buffer_allocation_count",
                                  "warm_buffer_allocation_count", "pipeline_create_count", "descriptor_set_count",
                                  "weight_upload_count", "execution_count", "last_execution_ns",
                                  "execution_plan_identity", "replay_identity")] + [
        (n, C.c_uint32) for n in ("assembly_family", "parameter_set", "binding_state", "active_weight_window")] + [
        (n, C.c_uint64) for n in ("parameter_set_aggregate_identity", "binding_generation", "output_generation",
                                  "descriptor_generation")] + [
        ("m1b_boundary_gpu_ns", C.c_uint64 * 6)] + [
        (n, C.c_uint64) for n in ("gpu_total_begin_tick", "gpu_total_end_tick", "gpu_total_ns",
                                  "gpu_compute_begin_tick", "gpu_compute_end_tick", "gpu_compute_ns",
                                  "gpu_ingress_transfer_ns", "gpu_joint_copy_ns", "gpu_readback_ns")] + [
        ("main_stage_gpu_begin_tick", C.c_uint64 * 13), ("main_stage_gpu_end_tick", C.c_uint64 * 13),
        ("main_stage_gpu_ns", C.c_uint64 * 13)] + [
        (n, C.c_uint64) for n in (
            "last_active_target_validation_ns", "last_command_reset_ns", "last_command_begin_ns",
            "last_command_record_ns", "last_command_end_ns", "last_queue_submit_ns", "last_fence_wait_ns",
            "last_descriptor_update_ns", "last_staging_memcpy_ns", "last_output_readback_ns",
            "vk_create_buffer_count", "vk_destroy_buffer_count", "vk_allocate_memory_count", "vk_free_memory_count",
            "vk_create_shader_module_count", "vk_destroy_shader_module_count", "vk_create_compute_pipelines_count",
            "vk_allocate_descriptor_sets_count", "vk_update_descriptor_sets_count", "vk_create_command_pool_count",
            "vk_allocate_command_buffers_count", "vk_reset_command_buffer_count", "vk_queue_submit_count",
            "vk_fence_wait_count", "vk_timeline_wait_count", "vk_map_memory_count", "vk_unmap_memory_count",
            "vk_flush_count", "vk_invalidate_count", "m6a_activation_pack_gpu_ns", "m6a_cooperative_execute_gpu_ns",
            "m6a_w3_segment_repack_gpu_ns")]


class OctB200BlockConfig(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("family", C.c_uint32),
        ("hidden", C.c_uint32),
        ("heads", C.c_uint32),
        ("kv_heads", C.c_uint32),
        ("head_dim", C.c_uint32),
        ("ffn", C.c_uint32),
        ("seq_len", C.c_uint32),
        ("max_batch", C.c_uint32),
        ("eps", C.c_float),
        ("rope_base", C.c_float),
        ("grid_w", C.c_uint32),
        ("rope_frame", C.c_uint32),
        ("tp_rank", C.c_uint32),
        ("tp_world", C.c_uint32),
        ("nccl_id", C.c_uint8 * 128),
    ]


BLOCK_GEMMA, BLOCK_DIT = 1, 2


class OctB200TpSgemmConfig(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("rank", C.c_uint32),
        ("world", C.c_uint32),
        ("max_m", C.c_uint32),
        ("max_n", C.c_uint32),
        ("collective", C.c_uint32),
        ("nccl_id", C.c_uint8 * 128),
    ]


TP_COLLECTIVE_AUTO, TP_COLLECTIVE_PEER, TP_COLLECTIVE_NCCL = 0, 1, 2
DETAIL_TP_INVALID, DETAIL_TP_ALLOC, DETAIL_TP_NCCL, DETAIL_TP_NOT_FOUND, DETAIL_TP_EXEC = (
    -7020, -7021, -7022, -7023, -7024)
GEMMA_SLOTS = {"norm1": 0, "wqkv": 1, "wo": 2, "norm2": 3, "wgu": 4, "wd": 5}
DIT_SLOTS = {"ada_w": 0, "ada_b": 1, "attn_norm1": 2, "wqkv": 3, "q_norm": 4, "k_norm": 5, "wo": 6,
             "attn_norm2": 7, "ffn_norm1": 8, "w13": 9, "w2": 10, "ffn_norm2": 11}


# ---- signatures ---------------------------------------------------------------
_vp, _u32, _u64, _i32p, _u32p = C.c_void_p, C.c_uint32, C.c_uint64, C.POINTER(C.c_int), C.POINTER(C.c_uint32)

SIGNATURES = {
    "prometheus_reactor_abi_version": (C.c_uint32, []),
    "prometheus_reactor_runtime_create": (C.c_int, [_vp, C.POINTER(C.c_void_p)]),
    "prometheus_reactor_runtime_destroy": (C.c_int, [_vp]),
    "prometheus_reactor_runtime_probe": (C.c_int, [_vp, C.POINTER(PrometheusCaps)]),
    "prometheus_reactor_runtime_sgemm": (C.c_int, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32p, _i32p]),
    "prometheus_reactor_runtime_sgemm_benchmark_variant": (
        C.c_int, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32p, _i32p]),
    "prometheus_reactor_runtime_sgemm_resident_benchmark": (
        C.c_int, [_vp, C.POINTER(PrometheusSgemmResidentBenchmarkRequest),
                  C.POINTER(PrometheusSgemmResidentBenchmarkResult)]),
    "prometheus_reactor_runtime_sgemm_batch": (
        C.c_int, [_vp, C.POINTER(PrometheusSgemmBatchEntry), _u32, _u32, _u32p, _i32p]),
    "prometheus_reactor_runtime_sgemm_submit_async": (
        C.c_int, [_vp, _vp, _vp, _u32, _u32, _u32, _i32p, _u32p, _i32p]),
    "prometheus_reactor_runtime_sgemm_query_async": (C.c_int, [_vp, C.c_int, C.POINTER(PrometheusAsyncStatus)]),
    "prometheus_reactor_runtime_sgemm_consume_async": (C.c_int, [_vp, C.c_int, _vp, _u32, _u32p, _i32p]),
    "prometheus_reactor_runtime_sgemm_abandon_async": (C.c_int, [_vp, C.c_int]),
    "prometheus_reactor_reduction_plan": (
        C.c_int, [C.POINTER(PrometheusReductionRequest), C.POINTER(PrometheusReductionPlan)]),
    "prometheus_reactor_runtime_reduction": (
        C.c_int, [_vp, C.POINTER(PrometheusReductionRequest), C.POINTER(PrometheusReductionExecutionResult)]),
    "prometheus_reactor_runtime_reduction_diagnostics": (
        C.c_int, [_vp, C.POINTER(PrometheusReductionDiagnostics)]),
    "prometheus_reactor_runtime_reduction_benchmark": (
        C.c_int, [_vp, C.POINTER(PrometheusReductionBenchmarkRequest), C.POINTER(PrometheusReductionBenchmarkResult)]),
    "prometheus_reactor_runtime_sgemm_async_diagnostics": (
        C.c_int, [_vp, C.POINTER(PrometheusSgemmAsyncDiagnostics)]),
    "prometheus_reactor_runtime_row_wise_softmax": (
        C.c_int, [_vp, C.POINTER(PrometheusRowWiseSoftmaxRequest), C.POINTER(PrometheusRowWiseSoftmaxResult)]),
    "prometheus_reactor_runtime_gemma4e2b_m1_input_rmsnorm": (
        C.c_int,
        [_vp, C.POINTER(PrometheusGemma4E2BM1InputRmsNormRequest), C.POINTER(PrometheusGemma4E2BM1InputRmsNormResult)]),
    "prometheus_reactor_runtime_gemma4e2b_m1_head_rmsnorm": (
        C.c_int,
        [_vp, C.POINTER(PrometheusGemma4E2BM1InputRmsNormRequest), C.POINTER(PrometheusGemma4E2BM1InputRmsNormResult)]),
    "prometheus_reactor_runtime_gemma4e2b_m1_projection_activation_rmsnorm": (
        C.c_int,
        [_vp, C.POINTER(PrometheusGemma4E2BM1InputRmsNormRequest), C.POINTER(PrometheusGemma4E2BM1InputRmsNormResult)]),
    "prometheus_reactor_runtime_gemma4e2b_m1_rope": (
        C.c_int, [_vp, C.POINTER(PrometheusGemma4E2BM1RopeRequest), C.POINTER(PrometheusGemma4E2BM1RopeResult)]),
    "prometheus_reactor_runtime_gemma4e2b_m1_head_rmsnorm_rope": (
        C.c_int, [_vp, C.POINTER(PrometheusGemma4E2BM1HeadRmsNormRopeRequest),
                  C.POINTER(PrometheusGemma4E2BM1HeadRmsNormRopeResult)]),
    "prometheus_reactor_runtime_gemma4e2b_m1_attention_scores": (
        C.c_int, [_vp, C.POINTER(PrometheusGemma4E2BM1AttentionScoresRequest),
                  C.POINTER(PrometheusGemma4E2BM1AttentionScoresResult)]),
    "prometheus_reactor_runtime_model_block_create": (
        C.c_int, [_vp, C.POINTER(PrometheusModelBlockCreateRequest), C.POINTER(C.c_uint64), C.POINTER(PrometheusModelBlockEvidence)]),
    "prometheus_reactor_runtime_model_block_upload_weights": (
        C.c_int, [_vp, C.c_uint64, C.POINTER(PrometheusModelBlockWeightUpload), _u32, C.POINTER(PrometheusModelBlockEvidence)]),
    "prometheus_reactor_runtime_model_block_execute": (
        C.c_int, [_vp, C.c_uint64, C.POINTER(PrometheusModelBlockExecuteRequest), C.POINTER(PrometheusModelBlockEvidence)]),
    "prometheus_reactor_runtime_noise_refiner0_execute": (
        C.c_int, [_vp, C.c_uint64, C.POINTER(PrometheusNoiseRefiner0ExecuteRequest), C.POINTER(PrometheusModelBlockEvidence)]),
    "prometheus_reactor_runtime_noise_refiner1_execute": (
        C.c_int, [_vp, C.c_uint64, C.POINTER(PrometheusNoiseRefiner0ExecuteRequest), C.POINTER(PrometheusModelBlockEvidence)]),
    "prometheus_reactor_runtime_noise_refiner_rebind": (
        C.c_int, [_vp, C.c_uint64, C.POINTER(PrometheusNoiseRefinerRebindRequest), C.POINTER(PrometheusModelBlockEvidence)]),
    "prometheus_reactor_runtime_noise_refiner_execute_resident": (
        C.c_int, [_vp, C.c_uint64, C.POINTER(PrometheusNoiseRefinerResidentExecuteRequest), C.POINTER(PrometheusModelBlockEvidence)]),
    "prometheus_reactor_runtime_noise_refiner_audit_final": (
        C.c_int, [_vp, C.c_uint64, C.POINTER(PrometheusNoiseRefinerFinalAuditRequest), C.POINTER(PrometheusModelBlockEvidence)]),
    "prometheus_reactor_runtime_context_refiner_create": (
        C.c_int, [_vp, C.POINTER(PrometheusContextRefinerCreateRequest), C.POINTER(C.c_uint64), C.POINTER(PrometheusModelBlockEvidence)]),
    "prometheus_reactor_runtime_context_refiner_rebind": (
        C.c_int, [_vp, C.c_uint64, C.POINTER(PrometheusContextRefinerCreateRequest), C.POINTER(PrometheusModelBlockEvidence)]),
    "prometheus_reactor_runtime_context_refiner0_execute": (
        C.c_int, [_vp, C.c_uint64, C.POINTER(PrometheusContextRefiner0ExecuteRequest), C.POINTER(PrometheusModelBlockEvidence)]),
    "prometheus_reactor_runtime_context_refiner_execute_resident": (
        C.c_int, [_vp, C.c_uint64, C.POINTER(PrometheusContextRefinerResidentExecuteRequest), C.POINTER(PrometheusModelBlockEvidence)]),
    "prometheus_reactor_runtime_context_refiner_audit_final": (
        C.c_int, [_vp, C.c_uint64, C.POINTER(PrometheusNoiseRefinerFinalAuditRequest), C.POINTER(PrometheusModelBlockEvidence)]),
    "prometheus_reactor_runtime_model_block_get_evidence": (C.c_int, [_vp, C.c_uint64, C.POINTER(PrometheusModelBlockEvidence)]),
    "prometheus_reactor_runtime_model_block_destroy": (C.c_int, [_vp, C.c_uint64]),
    "prometheus_reactor_runtime_fft64": (C.c_int, [_vp, _vp, _vp, _u32, _u32p, _i32p]),
    "prometheus_reactor_runtime_fft": (C.c_int, [_vp, C.POINTER(PrometheusFftRequest), _u32p, _i32p]),
    "prometheus_reactor_runtime_fft_benchmark_variant": (
        C.c_int, [_vp, C.POINTER(PrometheusFftRequest), _u32, _u32p, _i32p]),
    "prometheus_reactor_runtime_fft_diagnostics": (C.c_int, [_vp, C.POINTER(PrometheusFftDiagnostics)]),
    "prometheus_reactor_runtime_fft_diagnostics_sized": (
        C.c_int, [_vp, C.POINTER(PrometheusFftDiagnostics), _u32]),
    "prometheus_runtime_create": (C.c_int, [_vp, C.POINTER(C.c_void_p)]),
    "prometheus_runtime_destroy": (C.c_int, [_vp]),
    "prometheus_runtime_probe": (C.c_int, [_vp, C.POINTER(PrometheusCaps)]),
    "oct_b200_sgemm_device": (C.c_int, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _vp, _i32p]),
    "oct_b200_sgemm_device_ld": (
        C.c_int, [_vp, _vp, _u64, _vp, _u64, _vp, _u64, _u32, _u32, _u32, _u32, _vp, _i32p]),
    "oct_b200_sgemm_batched_device": (
        C.c_int, [_vp, _vp, _u64, _u64, _vp, _u64, _u64, _u32, _vp, _u64, _u64, _u32, _u32, _u32, _u32, _u32, _vp,
                  _i32p]),
    "oct_b200_reduction_device": (C.c_int, [_vp, _vp, _vp, _u32, _u32, _u32, _vp, _i32p]),
    "oct_b200_rmsnorm_device": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, C.c_float, _vp, _i32p]),
    "oct_b200_attention_device": (
        C.c_int, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, C.c_float, _vp, _i32p]),
    "oct_b200_selftest_wait_timeout": (C.c_int, [_vp, _u64, _i32p]),
    "oct_b200_sync_status": (C.c_int, [_vp, _vp, _i32p]),
    "oct_b200_sgemm_device_noalloc": (
        C.c_int, [_vp, _u64, _vp, _u64, _vp, _u64, _u32, _u32, _u32, _vp, _i32p]),
    "oct_b200_set_kernel_timing": (C.c_int, [_vp, C.c_int]),
    "oct_b200_read_kernel_timing": (
        C.c_int, [_vp, C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(C.c_uint32)]),
    "oct_b200_nccl_unique_id": (C.c_int, [_vp]),
    "oct_b200_block_create": (C.c_int, [_vp, C.POINTER(OctB200BlockConfig), C.POINTER(C.c_uint64), _i32p]),
    "oct_b200_tp_sgemm_create": (C.c_int, [_vp, C.POINTER(OctB200TpSgemmConfig), C.POINTER(C.c_uint64), _i32p]),
    "oct_b200_sgemm_tp_device": (C.c_int, [_vp, C.c_uint64, _vp, _u64, _vp, _u64, _vp, _u64, _u32, _u32, _u32, _vp,
                                           C.POINTER(C.c_void_p), _i32p]),
    "oct_b200_tp_sgemm_sync": (C.c_int, [_vp, C.c_uint64, _vp, _i32p]),
    "oct_b200_tp_sgemm_collective": (C.c_int, [_vp, C.c_uint64, C.POINTER(C.c_uint32)]),
    "oct_b200_tp_sgemm_destroy": (C.c_int, [_vp, C.c_uint64]),
    "oct_b200_block_set_weight": (C.c_int, [_vp, C.c_uint64, _u32, _vp, _u64, _u32]),
    "oct_b200_block_forward_device": (C.c_int, [_vp, C.c_uint64, _vp, _vp, _u32, _vp, _vp, _i32p]),
    "oct_b200_block_forward": (C.c_int, [_vp, C.c_uint64, _vp, _vp, _u32, _vp, _i32p]),
    "oct_b200_block_destroy": (C.c_int, [_vp, C.c_uint64]),
    "oct_b200_build_info": (C.c_char_p, []),
}

# Symbols Go refuses to run without (bridge.go:276-340).
MANDATORY = (
    "prometheus_reactor_abi_version",
    "prometheus_reactor_runtime_create",
    "prometheus_reactor_runtime_destroy",
    "prometheus_reactor_runtime_probe",
    "prometheus_reactor_runtime_sgemm",
)


class ReactorIssue(RuntimeError):
    """Mirror of bridge.go's ReactorIssue: a typed failure to reach the reactor."""

    NOT_FOUND = "reactor_not_found"
    LOAD_FAILED = "reactor_load_failed"
    SYMBOL_MISSING = "symbol_missing"
    ABI_MISMATCH = "abi_mismatch"
    CREATE_FAILED = "runtime_create_failed"
    PROBE_FAILED = "runtime_probe_unavailable"
    SGEMM_FAILED = "runtime_sgemm_failed"

    def __init__(self, code: str, message: str = "", *, path: str = "", symbol: str = "", stage: int = 0,
                 detail: int = 0):
        super().__init__(f"{code}: {message}" if message else code)
        self.code, self.path, self.symbol, self.stage, self.detail = code, path, symbol, stage, detail


@dataclass
class CallStatus:
    """reactorCallStatus in bridge.go: the native stage and detail of one call."""

    rc: int
    stage: int
    detail: int

    @property
    def ok(self) -> bool:
        return self.rc == PROM_OK


def default_library_path() -> Path:
    return Path(__file__).resolve().parent / LIB_NAME


def candidate_paths() -> list[Path]:
    """Discovery order of bridge.go:552-601: the env var, then the in-tree build."""
    out = []
    env = os.environ.get(ENV_VAR)
    if env:
        out.append(Path(env))
    out.append(default_library_path())
    return out


def load_library(path: Optional[os.PathLike] = None) -> C.CDLL:
    """dlopen the reactor, check the ABI, bind every known symbol's signature."""
    paths = [Path(path)] if path is not None else candidate_paths()
    found = next((p for p in paths if p.exists()), None)
    if found is None:
        raise ReactorIssue(ReactorIssue.NOT_FOUND, "no libprometheus_reactor.so (build it: python -m oct_b200.build)")
    try:
        lib = C.CDLL(str(found), mode=os.RTLD_NOW | os.RTLD_LOCAL)
    except OSError as exc:
        raise ReactorIssue(ReactorIssue.LOAD_FAILED, str(exc), path=str(found)) from exc
    for name in MANDATORY:
        if not hasattr(lib, name):
            raise ReactorIssue(ReactorIssue.SYMBOL_MISSING, name, path=str(found), symbol=name)
    for name, (res, args) in SIGNATURES.items():
        if hasattr(lib, name):
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = res, args
    abi = lib.prometheus_reactor_abi_version()
    if abi != EXPECTED_ABI:
        raise ReactorIssue(ReactorIssue.ABI_MISMATCH, f"expected {EXPECTED_ABI}, library reports {abi}",
                           path=str(found))
    lib._oct_path = str(found)  # type: ignore[attr-defined]
    return lib


def _f32(x: np.ndarray, name: str) -> np.ndarray:
    if not isinstance(x, np.ndarray) or x.dtype != np.float32 or not x.flags.c_contiguous:
        raise TypeError(f"{name} must be a C-contiguous float32 numpy array")
    return x


def _ptr(x) -> int:
    """Address of a numpy array or of a torch tensor's storage."""
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    if hasattr(x, "data_ptr"):
        return int(x.data_ptr())
    if x is None:
        return 0
    return int(x)


class Runtime:
    """One reactor handle: Go's nativeRuntime (bridge.go:276-520)."""

    def __init__(self, lib: Optional[C.CDLL] = None, *, test_flags: int = 0, async_test_flags: int = 0,
                 reduction_test_flags: int = 0, require_device: bool = True):
        self.lib = lib if lib is not None else load_library()
        cfg = PrometheusReactorConfig()
        cfg.struct_size = C.sizeof(PrometheusReactorConfig)
        cfg.test_flags = test_flags
        cfg.async_test_flags = async_test_flags
        cfg.reduction_test_flags = reduction_test_flags
        cfg.reduction_ring_depth = 3  # what Go always passes (bridge.go:318)
        handle = C.c_void_p()
        rc = self.lib.prometheus_reactor_runtime_create(C.byref(cfg), C.byref(handle))
        if rc != PROM_OK or not handle.value:
            raise ReactorIssue(ReactorIssue.CREATE_FAILED, f"rc={rc}")
        self.handle = handle
        caps = PrometheusCaps()
        rc = self.lib.prometheus_reactor_runtime_probe(self.handle, C.byref(caps))
        self.caps = caps
        if require_device and (rc != PROM_OK or not caps.available):
            self.close()
            raise ReactorIssue(ReactorIssue.PROBE_FAILED, f"rc={rc} available={caps.available} reason={caps.reason_code}")

    # -- lifetime
    def close(self) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            self.lib.prometheus_reactor_runtime_destroy(self.handle)
            self.handle = C.c_void_p()

    def __enter__(self) -> "Runtime":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    # -- SGEMM (bridge.go:410-436)
    def sgemm_with_status(self, m: int, n: int, k: int, a: np.ndarray, b: np.ndarray,
                          out: Optional[np.ndarray] = None) -> tuple[Optional[np.ndarray], CallStatus]:
        _f32(a, "a")
        _f32(b, "b")
        if a.size != m * k or b.size != k * n:
            return None, CallStatus(PROM_ERROR, STAGE_INIT, -2)  # "invalid matrix lengths"
        c = out if out is not None else np.empty(m * n, dtype=np.float32)
        _f32(c, "c")
        stage, detail = C.c_uint32(), C.c_int()
        rc = self.lib.prometheus_reactor_runtime_sgemm(self.handle, _ptr(a), _ptr(b), _ptr(c), m, n, k,
                                                       C.byref(stage), C.byref(detail))
        st = CallStatus(rc, stage.value, detail.value)
        return (c if rc == PROM_OK else None), st

    def sgemm(self, m: int, n: int, k: int, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        c, st = self.sgemm_with_status(m, n, k, a, b)
        if not st.ok:
            raise ReactorIssue(ReactorIssue.SGEMM_FAILED, f"stage={st.stage} detail={st.detail}", stage=st.stage,
                               detail=st.detail)
        return c

    # -- explicit variant, resident benchmark, batch (reactor_api.h:2596-2615)
    def sgemm_variant(self, m: int, n: int, k: int, a: np.ndarray, b: np.ndarray,
                      variant: int) -> tuple[Optional[np.ndarray], CallStatus]:
        _f32(a, "a")
        _f32(b, "b")
        c = np.empty(m * n, dtype=np.float32)
        stage, detail = C.c_uint32(), C.c_int()
        rc = self.lib.prometheus_reactor_runtime_sgemm_benchmark_variant(
            self.handle, _ptr(a), _ptr(b), _ptr(c), m, n, k, variant, C.byref(stage), C.byref(detail))
        st = CallStatus(rc, stage.value, detail.value)
        return (c if rc == PROM_OK else None), st

    def resident_benchmark(self, m: int, n: int, k: int, a: np.ndarray, b: np.ndarray, *, iterations: int = 5,
                           warmup: int = 1, variant: Optional[int] = None, depth: int = 0, ring: bool = False,
                           readback: bool = True) -> tuple[int, PrometheusSgemmResidentBenchmarkResult,
                                                          Optional[np.ndarray]]:
        _f32(a, "a")
        _f32(b, "b")
        c = np.empty(m * n, dtype=np.float32) if readback else None
        req = PrometheusSgemmResidentBenchmarkRequest()
        req.struct_size = C.sizeof(req)
        req.a, req.b, req.c = _ptr(a), _ptr(b), (_ptr(c) if c is not None else None)
        req.m, req.n, req.k = m, n, k
        req.mode = RESIDENT_MODE_EXPLICIT_VARIANT if variant is not None else RESIDENT_MODE_PRODUCTION_SELECTOR
        req.requested_variant = variant or 0
        req.warmup_iterations, req.iterations, req.diagnostic_batch_depth = warmup, iterations, depth
        req.flags = (RESIDENT_FLAG_VALIDATE_READBACK if readback else 0) | (RESIDENT_FLAG_M29_SUBMISSION_RING if ring
                                                                            else 0)
        res = PrometheusSgemmResidentBenchmarkResult()
        rc = self.lib.prometheus_reactor_runtime_sgemm_resident_benchmark(self.handle, C.byref(req), C.byref(res))
        return rc, res, c

    def sgemm_batch(self, problems: list, flags: int = 0) -> tuple[Optional[list], CallStatus]:
        """problems: [(m, n, k, a, b), ...]; returns the C of every entry, or None on failure."""
        entries = (PrometheusSgemmBatchEntry * len(problems))()
        outs = []
        for e, (m, n, k, a, b) in zip(entries, problems):
            _f32(a, "a")
            _f32(b, "b")
            c = np.full(m * n, np.nan, dtype=np.float32)
            outs.append(c)
            e.a, e.b, e.c, e.m, e.n, e.k = _ptr(a), _ptr(b), _ptr(c), m, n, k
        stage, detail = C.c_uint32(), C.c_int()
        rc = self.lib.prometheus_reactor_runtime_sgemm_batch(self.handle, entries, len(problems), flags,
                                                             C.byref(stage), C.byref(detail))
        st = CallStatus(rc, stage.value, detail.value)
        return (outs if rc == PROM_OK else None), st

    # -- async SGEMM (bridge.go:342-361, runtime.go:573-650)
    def submit_async(self, m: int, n: int, k: int, a: np.ndarray, b: np.ndarray) -> tuple[int, CallStatus]:
        _f32(a, "a")
        _f32(b, "b")
        task, stage, detail = C.c_int(), C.c_uint32(), C.c_int()
        rc = self.lib.prometheus_reactor_runtime_sgemm_submit_async(self.handle, _ptr(a), _ptr(b), m, n, k,
                                                                    C.byref(task), C.byref(stage), C.byref(detail))
        return task.value, CallStatus(rc, stage.value, detail.value)

    def query_async(self, task: int) -> tuple[int, PrometheusAsyncStatus]:
        st = PrometheusAsyncStatus()
        rc = self.lib.prometheus_reactor_runtime_sgemm_query_async(self.handle, task, C.byref(st))
        return rc, st

    def consume_async(self, task: int, c: np.ndarray) -> CallStatus:
        _f32(c, "c")
        stage, detail = C.c_uint32(), C.c_int()
        rc = self.lib.prometheus_reactor_runtime_sgemm_consume_async(self.handle, task, _ptr(c), c.size,
                                                                     C.byref(stage), C.byref(detail))
        return CallStatus(rc, stage.value, detail.value)

    def abandon_async(self, task: int) -> int:
        return self.lib.prometheus_reactor_runtime_sgemm_abandon_async(self.handle, task)

    # -- reductions
    def reduction(self, x: np.ndarray, operation: int, *, flags: int = 0,
                  out: Optional[np.ndarray] = None) -> tuple[Optional[np.ndarray], PrometheusReductionExecutionResult]:
        _f32(x, "x")
        rows, width = x.shape
        n_out = x.size if operation == OP_SOFTMAX else rows
        y = out if out is not None else np.empty(n_out, dtype=np.float32)
        req = make_reduction_request(x, y, rows, width, operation, flags)
        res = PrometheusReductionExecutionResult()
        rc = self.lib.prometheus_reactor_runtime_reduction(self.handle, C.byref(req), C.byref(res))
        return (y if rc == PROM_OK else None), res

    def row_wise_softmax(self, x: np.ndarray, out: Optional[np.ndarray] = None
                         ) -> tuple[int, Optional[np.ndarray], PrometheusRowWiseSoftmaxResult]:
        rows, width = x.shape
        y = out if out is not None else np.empty_like(x)
        req = PrometheusRowWiseSoftmaxRequest()
        req.struct_size = C.sizeof(req)
        req.input, req.output = _ptr(x), _ptr(y)
        req.row_count, req.elements_per_row = rows, width
        req.input_element_count = req.output_element_count = rows * width
        res = PrometheusRowWiseSoftmaxResult()
        rc = self.lib.prometheus_reactor_runtime_row_wise_softmax(self.handle, C.byref(req), C.byref(res))
        return rc, (y if rc == PROM_OK else None), res

    def next_weight_generation(self) -> int:
        """A fresh weight generation for this handle: the M1 entries require each weight
        preparation to carry a generation above the last one committed (as Go's lane does,
        gemma4e2b_m1_rtx.go:268-545)."""
        self._generation = getattr(self, "_generation", 0) + 1
        return self._generation

    def rmsnorm(self, x: np.ndarray, weight: np.ndarray, eps: float, *, head: bool = False,
                mode: str = "input", stride: Optional[int] = None, width: Optional[int] = None,
                rows: Optional[int] = None
                ) -> tuple[int, Optional[np.ndarray], Optional[np.ndarray], PrometheusGemma4E2BM1InputRmsNormResult]:
        """The M46 RMSNorm family over host rows: mode "input" (fp32), "projection" (BF16
        output), "head" (BF16 input and output; also selected by head=True).  x may be 1-D
        with explicit rows / width / stride (row stride >= width), else [rows, width]."""
        _f32(x, "x")
        _f32(weight, "weight")
        if head:
            mode = "head"
        if x.ndim == 2 and rows is None:
            rows, width = x.shape
            stride = width
        width = width or weight.size
        stride = stride or width
        rows = rows if rows is not None else x.size // stride
        y = np.empty((rows, width), dtype=np.float32)
        inv = np.empty(rows, dtype=np.float32)
        req = PrometheusGemma4E2BM1InputRmsNormRequest()
        req.struct_size = C.sizeof(req)
        req.input, req.weight, req.output, req.inv_rms_output = _ptr(x), _ptr(weight), _ptr(y), _ptr(inv)
        req.input_element_count = x.size
        req.weight_element_count = weight.size
        req.output_element_count = y.size
        req.inv_rms_output_element_count = rows
        req.tokens, req.model_width, req.input_row_stride = rows, width, stride
        req.epsilon = eps
        req.input_generation = req.exact_source_hash = 1
        req.weight_generation = self.next_weight_generation()
        res = PrometheusGemma4E2BM1InputRmsNormResult()
        fn = {"input": self.lib.prometheus_reactor_runtime_gemma4e2b_m1_input_rmsnorm,
              "projection": self.lib.prometheus_reactor_runtime_gemma4e2b_m1_projection_activation_rmsnorm,
              "head": self.lib.prometheus_reactor_runtime_gemma4e2b_m1_head_rmsnorm}[mode]
        rc = fn(self.handle, C.byref(req), C.byref(res))
        ok = rc == PROM_OK
        return rc, (y if ok else None), (inv if ok else None), res

    # -- Gemma M1 positional / score boundary (bridge.go:493-515)
    def gemma_rope(self, source: np.ndarray, cosine: np.ndarray, sine: np.ndarray, tokens: int, heads: int,
                   head_width: int, out: Optional[np.ndarray] = None
                   ) -> tuple[int, np.ndarray, PrometheusGemma4E2BM1RopeResult]:
        for t, nm in ((source, "source"), (cosine, "cosine"), (sine, "sine")):
            _f32(t, nm)
        y = np.empty(source.size, dtype=np.float32) if out is None else out
        req = PrometheusGemma4E2BM1RopeRequest()
        req.struct_size = C.sizeof(req)
        req.source, req.cosine, req.sine, req.output = _ptr(source), _ptr(cosine), _ptr(sine), _ptr(y)
        req.source_element_count, req.cosine_element_count = source.size, cosine.size
        req.sine_element_count, req.output_element_count = sine.size, y.size
        req.tokens, req.heads, req.head_width = tokens, heads, head_width
        req.source_generation = req.table_generation = 1
        res = PrometheusGemma4E2BM1RopeResult()
        rc = self.lib.prometheus_reactor_runtime_gemma4e2b_m1_rope(self.handle, C.byref(req), C.byref(res))
        return rc, y, res

    def gemma_head_rmsnorm_rope(self, x: np.ndarray, weight: np.ndarray, cosine: np.ndarray, sine: np.ndarray,
                                tokens: int, heads: int, head_width: int, eps: float = 1e-6,
                                read_back: bool = True, weight_generation: Optional[int] = None
                                ) -> tuple[int, Optional[np.ndarray], PrometheusGemma4E2BM1HeadRmsNormRopeResult]:
        for t, nm in ((x, "x"), (weight, "weight"), (cosine, "cosine"), (sine, "sine")):
            _f32(t, nm)
        y = np.empty(x.size, dtype=np.float32) if read_back else None
        req = PrometheusGemma4E2BM1HeadRmsNormRopeRequest()
        req.struct_size = C.sizeof(req)
        req.input, req.weight, req.cosine, req.sine = _ptr(x), _ptr(weight), _ptr(cosine), _ptr(sine)
        req.output = _ptr(y) if y is not None else None
        req.input_element_count, req.weight_element_count = x.size, weight.size
        req.cosine_element_count, req.sine_element_count = cosine.size, sine.size
        req.output_element_count = y.size if y is not None else 0
        req.tokens, req.heads, req.head_width, req.epsilon = tokens, heads, head_width, eps
        req.input_generation = req.table_generation = req.exact_source_hash = 1
        req.weight_generation = weight_generation or self.next_weight_generation()
        res = PrometheusGemma4E2BM1HeadRmsNormRopeResult()
        rc = self.lib.prometheus_reactor_runtime_gemma4e2b_m1_head_rmsnorm_rope(self.handle, C.byref(req),
                                                                                C.byref(res))
        return rc, (y if rc == PROM_OK else None), res

    def gemma_attention_scores(self, q: np.ndarray, k: np.ndarray, q_weight: np.ndarray, k_weight: np.ndarray,
                               cosine: np.ndarray, sine: np.ndarray, tokens: int, query_heads: int,
                               head_width: int, scale: float, order: int = 0, eps: float = 1e-6,
                               out: Optional[np.ndarray] = None
                               ) -> tuple[int, np.ndarray, PrometheusGemma4E2BM1AttentionScoresResult]:
        for t, nm in ((q, "q"), (k, "k"), (q_weight, "q_weight"), (k_weight, "k_weight"), (cosine, "cosine"),
                      (sine, "sine")):
            _f32(t, nm)
        s = np.empty(query_heads * tokens * tokens, dtype=np.float32) if out is None else out
        req = PrometheusGemma4E2BM1AttentionScoresRequest()
        req.struct_size = C.sizeof(req)
        req.query_input, req.key_input = _ptr(q), _ptr(k)
        req.query_weight, req.key_weight = _ptr(q_weight), _ptr(k_weight)
        req.cosine, req.sine, req.scores = _ptr(cosine), _ptr(sine), _ptr(s)
        req.query_input_element_count, req.key_input_element_count = q.size, k.size
        req.query_weight_element_count, req.key_weight_element_count = q_weight.size, k_weight.size
        req.cosine_element_count, req.sine_element_count, req.score_element_count = cosine.size, sine.size, s.size
        req.tokens, req.query_heads, req.key_heads, req.head_width = tokens, query_heads, 1, head_width
        req.epsilon, req.scale, req.preparation_order = eps, scale, order
        req.query_input_generation, req.key_input_generation, req.table_generation = 1, 2, 1
        first, second = self.next_weight_generation(), self.next_weight_generation()
        # weights are prepared in preparation order, each with a fresh generation
        req.query_weight_generation, req.key_weight_generation = (first, second) if order == 0 else (second, first)
        req.query_exact_source_hash, req.key_exact_source_hash = 11, 12
        res = PrometheusGemma4E2BM1AttentionScoresResult()
        rc = self.lib.prometheus_reactor_runtime_gemma4e2b_m1_attention_scores(self.handle, C.byref(req),
                                                                               C.byref(res))
        return rc, s, res

    # -- FFT (fft.go:21-44 binds fft64; the batched fp32 entry is native-only)
    def fft64(self, x: np.ndarray, out: Optional[np.ndarray] = None) -> tuple[Optional[np.ndarray], CallStatus]:
        """Forward unnormalised binary64 FFT of a complex128 vector (Go's fftBackend.Transform)."""
        x = np.ascontiguousarray(x, dtype=np.complex128)
        y = np.empty_like(x) if out is None else out
        st, d = C.c_uint32(), C.c_int()
        rc = self.lib.prometheus_reactor_runtime_fft64(self.handle, x.ctypes.data, y.ctypes.data, x.size,
                                                        C.byref(st), C.byref(d))
        return (y if rc == PROM_OK else None), CallStatus(rc, st.value, d.value)

    def fft(self, x: np.ndarray, n: int, batch: int = 1, stride: int = 0, flags: int = 0,
            out: Optional[np.ndarray] = None) -> tuple[np.ndarray, CallStatus]:
        """Batched fp32 FFT of complex64 data laid out `stride` (0: n) elements per batch item."""
        x = np.ascontiguousarray(x, dtype=np.complex64)
        y = np.zeros_like(x) if out is None else out
        req = PrometheusFftRequest()
        req.struct_size = C.sizeof(req)
        req.input, req.output = x.ctypes.data, y.ctypes.data
        req.element_count, req.batch_count, req.stride_elements, req.flags = n, batch, stride, flags
        st, d = C.c_uint32(), C.c_int()
        rc = self.lib.prometheus_reactor_runtime_fft(self.handle, C.byref(req), C.byref(st), C.byref(d))
        return y, CallStatus(rc, st.value, d.value)

    def fft_diagnostics(self) -> PrometheusFftDiagnostics:
        diag = PrometheusFftDiagnostics()
        rc = self.lib.prometheus_reactor_runtime_fft_diagnostics(self.handle, C.byref(diag))
        if rc != PROM_OK:
            raise RuntimeError(f"fft diagnostics rc={rc}")
        return diag

    # -- device-resident extensions (torch tensors or raw device addresses)
    def sgemm_device(self, a, b, c, m: int, n: int, k: int, variant: int = SGEMM_AUTO, stream=None,
                     lda: Optional[int] = None, ldb: Optional[int] = None, ldc: Optional[int] = None) -> None:
        detail = C.c_int()
        rc = self.lib.oct_b200_sgemm_device_ld(self.handle, _ptr(a), lda or k, _ptr(b), ldb or n, _ptr(c), ldc or n,
                                               m, n, k, variant, _stream_ptr(stream), C.byref(detail))
        if rc != PROM_OK:
            raise ReactorIssue(ReactorIssue.SGEMM_FAILED, f"device sgemm rc={rc} detail={detail.value}",
                               detail=detail.value)

    def sgemm_batched_device(self, a, lda: int, stride_a: int, b, ldb: int, stride_b: int, b_trans: bool, c,
                             ldc: int, stride_c: int, batch: int, m: int, n: int, k: int,
                             variant: int = SGEMM_AUTO, stream=None) -> None:
        detail = C.c_int()
        rc = self.lib.oct_b200_sgemm_batched_device(self.handle, _ptr(a), lda, stride_a, _ptr(b), ldb, stride_b,
                                                    1 if b_trans else 0, _ptr(c), ldc, stride_c, batch, m, n, k,
                                                    variant, _stream_ptr(stream), C.byref(detail))
        if rc != PROM_OK:
            raise ReactorIssue(ReactorIssue.SGEMM_FAILED, f"batched sgemm rc={rc} detail={detail.value}",
                               detail=detail.value)

    def reduction_device(self, x, y, rows: int, width: int, operation: int, stream=None) -> None:
        detail = C.c_int()
        rc = self.lib.oct_b200_reduction_device(self.handle, _ptr(x), _ptr(y), rows, width, operation,
                                                _stream_ptr(stream), C.byref(detail))
        if rc != PROM_OK:
            raise RuntimeError(f"device reduction rc={rc} detail={detail.value}")

    def rmsnorm_device(self, x, w, y, inv, rows: int, width: int, eps: float, stream=None) -> None:
        detail = C.c_int()
        rc = self.lib.oct_b200_rmsnorm_device(self.handle, _ptr(x), _ptr(w), _ptr(y), _ptr(inv), rows, width, eps,
                                              _stream_ptr(stream), C.byref(detail))
        if rc != PROM_OK:
            raise RuntimeError(f"device rmsnorm rc={rc} detail={detail.value}")

    def attention_device(self, q, k, v, out, items: int, seq: int, heads: int, head_dim: int,
                         scale: Optional[float] = None, stream=None) -> None:
        """Fused exact attention; q, k, v, out: [items*seq][heads*head_dim] on the device."""
        if scale is None:
            scale = float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))
        detail = C.c_int()
        rc = self.lib.oct_b200_attention_device(self.handle, _ptr(q), _ptr(k), _ptr(v), _ptr(out), items, seq, heads,
                                                head_dim, scale, _stream_ptr(stream), C.byref(detail))
        if rc != PROM_OK:
            raise RuntimeError(f"device attention rc={rc} detail={detail.value}")

    def selftest_wait_timeout(self, budget_ns: int) -> CallStatus:
        """Test-only: a bounded in-kernel wait on a flag nothing sets must report a timeout."""
        detail = C.c_int()
        rc = self.lib.oct_b200_selftest_wait_timeout(self.handle, budget_ns, C.byref(detail))
        return CallStatus(rc, 0, detail.value)

    def sync_status(self, stream=None) -> CallStatus:
        detail = C.c_int()
        rc = self.lib.oct_b200_sync_status(self.handle, _stream_ptr(stream), C.byref(detail))
        return CallStatus(rc, 0, detail.value)


    def set_kernel_timing(self, enable: bool) -> None:
        self.lib.oct_b200_set_kernel_timing(self.handle, 1 if enable else 0)

    def read_kernel_timing(self) -> tuple[float, float, int]:
        """(split_ms_total, main_ms_total, launches) since the last read."""
        s, m, n = C.c_double(), C.c_double(), C.c_uint32()
        rc = self.lib.oct_b200_read_kernel_timing(self.handle, C.byref(s), C.byref(m), C.byref(n))
        if rc != PROM_OK:
            raise RuntimeError(f"kernel timing read failed rc={rc}")
        return s.value, m.value, n.value


    # -- transformer block
    def block(self, family: int, *, hidden: int, heads: int, kv_heads: int, head_dim: int, ffn: int, seq_len: int,
              max_batch: int, eps: float, rope_base: float, grid_w: int = 0, rope_frame: int = 0, tp_rank: int = 0,
              tp_world: int = 1, nccl_id: bytes = b"") -> "Block":
        return Block(self, family, hidden=hidden, heads=heads, kv_heads=kv_heads, head_dim=head_dim, ffn=ffn,
                     seq_len=seq_len, max_batch=max_batch, eps=eps, rope_base=rope_base, grid_w=grid_w,
                     rope_frame=rope_frame, tp_rank=tp_rank, tp_world=tp_world, nccl_id=nccl_id)


    def tp_sgemm(self, rank: int, world: int, max_m: int, max_n: int, nccl_id: bytes = b"",
                 collective: int = 0) -> "TpSgemm":
        return TpSgemm(self, rank, world, max_m, max_n, nccl_id, collective)


def nccl_unique_id(lib) -> bytes:
    buf = (C.c_uint8 * 128)()
    if lib.oct_b200_nccl_unique_id(C.cast(buf, C.c_void_p)) != PROM_OK:
        raise RuntimeError("ncclGetUniqueId failed (libnccl.so.2 not loadable?)")
    return bytes(buf)


class Block:
    """A transformer block on one reactor handle (oct_b200_block_*)."""

    def __init__(self, rt: Runtime, family: int, **cfg):
        self.rt, self.lib = rt, rt.lib
        c = OctB200BlockConfig()
        c.struct_size = C.sizeof(c)
        c.family = family
        for key in ("hidden", "heads", "kv_heads", "head_dim", "ffn", "seq_len", "max_batch", "grid_w", "rope_frame",
                    "tp_rank", "tp_world"):
            setattr(c, key, int(cfg[key]))
        c.eps, c.rope_base = float(cfg["eps"]), float(cfg["rope_base"])
        nid = cfg.get("nccl_id") or b""
        for i, v in enumerate(nid[:128]):
            c.nccl_id[i] = v
        self.config = c
        self.family = family
        bid, detail = C.c_uint64(), C.c_int()
        rc = self.lib.oct_b200_block_create(rt.handle, C.byref(c), C.byref(bid), C.byref(detail))
        if rc != PROM_OK:
            raise RuntimeError(f"block create rc={rc} detail={detail.value}")
        self.id = bid.value

    def set_weights(self, weights: dict) -> None:
        slots = GEMMA_SLOTS if self.family == BLOCK_GEMMA else DIT_SLOTS
        for name, arr in weights.items():
            if hasattr(arr, "data_ptr"):
                ptr, count, on_dev = arr.data_ptr(), arr.numel(), 1 if arr.is_cuda else 0
            else:
                arr = np.ascontiguousarray(arr, dtype=np.float32)
                ptr, count, on_dev = arr.ctypes.data, arr.size, 0
            rc = self.lib.oct_b200_block_set_weight(self.rt.handle, self.id, slots[name], ptr, count, on_dev)
            if rc != PROM_OK:
                raise RuntimeError(f"set_weight {name} rc={rc}")

    def forward_device(self, x, y, batch: int, timesteps=None, stream=None) -> None:
        ts = None if timesteps is None else np.ascontiguousarray(timesteps, dtype=np.float32)
        detail = C.c_int()
        rc = self.lib.oct_b200_block_forward_device(self.rt.handle, self.id, _ptr(x), _ptr(y), batch,
                                                    None if ts is None else ts.ctypes.data, _stream_ptr(stream),
                                                    C.byref(detail))
        if rc != PROM_OK:
            raise RuntimeError(f"block forward rc={rc} detail={detail.value}")

    def forward(self, x: np.ndarray, batch: int, timesteps=None) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty_like(x)
        ts = None if timesteps is None else np.ascontiguousarray(timesteps, dtype=np.float32)
        detail = C.c_int()
        rc = self.lib.oct_b200_block_forward(self.rt.handle, self.id, x.ctypes.data, y.ctypes.data, batch,
                                             None if ts is None else ts.ctypes.data, C.byref(detail))
        if rc != PROM_OK:
            raise RuntimeError(f"block forward rc={rc} detail={detail.value}")
        return y

    def close(self) -> None:
        if getattr(self, "id", None) is not None:
            self.lib.oct_b200_block_destroy(self.rt.handle, self.id)
            self.id = None


class TpSgemm:
    """Column-parallel SGEMM over tensor-parallel ranks (oct_b200_tp_sgemm_*): every
    rank passes the same A and its column shard of B (oct_b200.tp.shard_columns) and
    receives all of C."""

    def __init__(self, rt: Runtime, rank: int, world: int, max_m: int, max_n: int, nccl_id: bytes = b"",
                 collective: int = TP_COLLECTIVE_AUTO):
        self.rt, self.lib = rt, rt.lib
        c = OctB200TpSgemmConfig()
        c.struct_size = C.sizeof(c)
        c.rank, c.world, c.max_m, c.max_n, c.collective = rank, world, max_m, max_n, collective
        for i, v in enumerate((nccl_id or b"")[:128]):
            c.nccl_id[i] = v
        tid, detail = C.c_uint64(), C.c_int()
        rc = self.lib.oct_b200_tp_sgemm_create(rt.handle, C.byref(c), C.byref(tid), C.byref(detail))
        if rc != PROM_OK:
            raise RuntimeError(f"tp sgemm create rc={rc} detail={detail.value}")
        self.id, self.rank, self.world = tid.value, rank, world

    @property
    def collective(self) -> int:
        out = C.c_uint32()
        if self.lib.oct_b200_tp_sgemm_collective(self.rt.handle, self.id, C.byref(out)) != PROM_OK:
            raise RuntimeError("tp sgemm collective query failed")
        return out.value

    def run_device(self, a, b_shard, c, m: int, n: int, k: int, stream=None, lda: int = 0, ldb: int = 0,
                   ldc: int = 0) -> int:
        """Enqueue C = A * B; returns the device address of the library's copy of C (ld n)."""
        res, detail = C.c_void_p(), C.c_int()
        rc = self.lib.oct_b200_sgemm_tp_device(self.rt.handle, self.id, _ptr(a), lda or k, _ptr(b_shard),
                                               ldb or n // self.world, None if c is None else _ptr(c), ldc or n, m,
                                               n, k, _stream_ptr(stream), C.byref(res), C.byref(detail))
        if rc != PROM_OK:
            raise RuntimeError(f"tp sgemm rc={rc} detail={detail.value}")
        return res.value or 0

    def sync(self, stream=None) -> int:
        """Waits for the stream; 0 or the detail code of a failed earlier call."""
        detail = C.c_int()
        rc = self.lib.oct_b200_tp_sgemm_sync(self.rt.handle, self.id, _stream_ptr(stream), C.byref(detail))
        return 0 if rc == PROM_OK else (detail.value or rc)

    def close(self) -> None:
        if getattr(self, "id", None) is not None:
            self.lib.oct_b200_tp_sgemm_destroy(self.rt.handle, self.id)
            self.id = None


def _stream_ptr(stream) -> int:
    if stream is None:
        return 0
    if hasattr(stream, "cuda_stream"):
        return int(stream.cuda_stream)
    return int(stream)


def make_reduction_request(x, y, rows: int, width: int, operation: int, flags: int = 0
                           ) -> PrometheusReductionRequest:
    req = PrometheusReductionRequest()
    req.struct_size = C.sizeof(req)
    req.input, req.output = _ptr(x), _ptr(y)
    req.row_count, req.elements_per_row = rows, width
    req.input_element_count = rows * width
    req.output_element_count = rows * width if operation == OP_SOFTMAX else rows
    req.operation = operation
    req.finalization = FINALIZATION_STABLE_SOFTMAX if operation == OP_SOFTMAX else FINALIZATION_NONE
    req.flags = flags
    return req


def reduction_plan(lib: C.CDLL, rows: int, width: int, operation: int, flags: int = 0
                   ) -> tuple[int, PrometheusReductionPlan]:
    """prometheus_reactor_reduction_plan: host-only, needs no device."""
    dummy = np.zeros(1, dtype=np.float32)
    req = make_reduction_request(dummy, dummy, rows, width, operation, flags)
    plan = PrometheusReductionPlan()
    rc = lib.prometheus_reactor_reduction_plan(C.byref(req), C.byref(plan))
    return rc, plan


# ---- Z-Image model-block executors (reactor_api.h:2713-2784) --------------------------------
def weight_uploads(payloads: list) -> tuple:
    """PrometheusModelBlockWeightUpload[] for binary16 payloads in binding order; the
    identities are FNV-1a of each payload's bytes and shape (any non-zero values serve)."""
    arr = (PrometheusModelBlockWeightUpload * len(payloads))()
    for i, p in enumerate(payloads):
        p = np.ascontiguousarray(p)
        arr[i].binding_index = i
        arr[i].bytes = p.ctypes.data
        arr[i].byte_count = p.nbytes
        arr[i].content_identity = _fnv64(p.tobytes()[:4096]) ^ (i + 1)
        arr[i].layout_identity = _fnv64(repr(p.shape).encode()) | 1
    return arr


def _fnv64(data: bytes) -> int:
    h = 1469598103934665603
    for b in data:
        h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h or 1


class ModelBlock:
    """The handle's one Z-Image model block, driven the way Go's compiled-model
    adapter drives the reference (create -> upload -> execute -> audit / rebind)."""

    def __init__(self, rt: "Runtime"):
        self.rt = rt
        self.lib = rt.lib
        self.id = 0
        self.evidence = PrometheusModelBlockEvidence()

    def create_noise_refiner(self, payloads: list, parameter_set: int = 1,
                             memory_ceiling: int = 1 << 31) -> tuple[int, PrometheusModelBlockEvidence]:
        req = PrometheusModelBlockCreateRequest()
        req.struct_size = C.sizeof(req)
        req.assembly_family, req.parameter_set = NOISE_REFINER_FAMILY, parameter_set
        req.parameter_set_aggregate_identity = ZIMAGE_NOISE_AGGREGATES[parameter_set - 1]
        req.model_contract_identity = req.weight_identity = ZIMAGE_LOCK_ID
        req.shader_portfolio_identity = req.precision_policy_identity = req.capability_route_identity = ZIMAGE_LOCK_ID
        req.memory_ceiling_bytes = memory_ceiling
        req.external_input_bytes = 2 * 1024 * 3840
        req.audit_bytes = ZIMAGE_AUDIT_ARENA_BYTES
        req.shader_id = 24
        req.weight_count = len(payloads)
        ups = weight_uploads(payloads)
        for i in range(len(payloads)):
            req.weights[i].content_identity = ups[i].content_identity
            req.weights[i].layout_identity = ups[i].layout_identity
            req.weights[i].byte_count = ups[i].byte_count
        req.step_count = MODEL_BLOCK_MAX_STEPS
        for i in range(MODEL_BLOCK_MAX_STEPS):
            req.steps[i] = i + 1
        bid = C.c_uint64()
        rc = self.lib.prometheus_reactor_runtime_model_block_create(self.rt.handle, C.byref(req), C.byref(bid),
                                                                    C.byref(self.evidence))
        if rc != PROM_OK:
            return rc, self.evidence
        self.id = bid.value
        rc = self.lib.prometheus_reactor_runtime_model_block_upload_weights(self.rt.handle, self.id, ups, len(ups),
                                                                            C.byref(self.evidence))
        return rc, self.evidence

    def create_context_refiner(self, payloads: list) -> tuple[int, PrometheusModelBlockEvidence]:
        ups = weight_uploads(payloads)
        req = PrometheusContextRefinerCreateRequest()
        req.struct_size = C.sizeof(req)
        req.model_local_block_id, req.lock_identity = 0, ZIMAGE_LOCK_ID
        req.upload_count, req.uploads = len(ups), ups
        bid = C.c_uint64()
        rc = self.lib.prometheus_reactor_runtime_context_refiner_create(self.rt.handle, C.byref(req), C.byref(bid),
                                                                        C.byref(self.evidence))
        self.id = bid.value
        return rc, self.evidence

    def rebind(self, payloads: list, context: bool = False) -> tuple[int, PrometheusModelBlockEvidence]:
        ups = weight_uploads(payloads)
        req = PrometheusNoiseRefinerRebindRequest()
        req.struct_size = C.sizeof(req)
        req.model_local_block_id, req.lock_identity = 1, ZIMAGE_LOCK_ID
        req.upload_count, req.uploads = len(ups), ups
        fn = (self.lib.prometheus_reactor_runtime_context_refiner_rebind if context
              else self.lib.prometheus_reactor_runtime_noise_refiner_rebind)
        rc = fn(self.rt.handle, self.id, C.byref(req), C.byref(self.evidence))
        return rc, self.evidence

    def noise_execute(self, image_bf16: np.ndarray, timestep_bf16: np.ndarray, block: int = 0
                      ) -> tuple[int, PrometheusModelBlockEvidence]:
        req = PrometheusNoiseRefiner0ExecuteRequest()
        req.struct_size = C.sizeof(req)
        req.model_input_bf16, req.timestep_bf16 = image_bf16.ctypes.data, timestep_bf16.ctypes.data
        req.model_input_bytes, req.timestep_bytes = image_bf16.nbytes, timestep_bf16.nbytes
        req.input_identity = req.timestep_identity = req.output_identity = 7
        fn = (self.lib.prometheus_reactor_runtime_noise_refiner1_execute if block == 1
              else self.lib.prometheus_reactor_runtime_noise_refiner0_execute)
        rc = fn(self.rt.handle, self.id, C.byref(req), C.byref(self.evidence))
        return rc, self.evidence

    def context_execute(self, x: np.ndarray) -> tuple[int, PrometheusModelBlockEvidence]:
        req = PrometheusContextRefiner0ExecuteRequest()
        req.struct_size = C.sizeof(req)
        req.context_input, req.context_input_bytes = x.ctypes.data, x.nbytes
        req.input_identity = req.output_identity = 9
        rc = self.lib.prometheus_reactor_runtime_context_refiner0_execute(self.rt.handle, self.id, C.byref(req),
                                                                          C.byref(self.evidence))
        return rc, self.evidence

    def execute_resident(self, input_generation: int, context: bool = False
                         ) -> tuple[int, PrometheusModelBlockEvidence]:
        if context:
            req = PrometheusContextRefinerResidentExecuteRequest()
            fn = self.lib.prometheus_reactor_runtime_context_refiner_execute_resident
        else:
            req = PrometheusNoiseRefinerResidentExecuteRequest()
            fn = self.lib.prometheus_reactor_runtime_noise_refiner_execute_resident
        req.struct_size = C.sizeof(req)
        req.input_generation, req.output_identity = input_generation, 11
        rc = fn(self.rt.handle, self.id, C.byref(req), C.byref(self.evidence))
        return rc, self.evidence

    def audit_final(self, tokens: int, generation: int, context: bool = False
                    ) -> tuple[int, Optional[np.ndarray], PrometheusModelBlockEvidence]:
        out = np.empty((tokens, 3840), dtype=np.float32)
        req = PrometheusNoiseRefinerFinalAuditRequest()
        req.struct_size = C.sizeof(req)
        req.required_output_generation, req.output_identity = generation, 13
        req.output, req.output_element_capacity = out.ctypes.data, out.size
        fn = (self.lib.prometheus_reactor_runtime_context_refiner_audit_final if context
              else self.lib.prometheus_reactor_runtime_noise_refiner_audit_final)
        rc = fn(self.rt.handle, self.id, C.byref(req), C.byref(self.evidence))
        return rc, (out if rc == PROM_OK else None), self.evidence

    def destroy(self) -> int:
        rc = self.lib.prometheus_reactor_runtime_model_block_destroy(self.rt.handle, self.id)
        self.id = 0
        return rc
