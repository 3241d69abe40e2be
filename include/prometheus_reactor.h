/*
 * prometheus_reactor.h -- C ABI (version 1) of the B200-native Prometheus reactor.
 *
 * This library is a drop-in replacement for Oct's `libprometheus_reactor.so` on
 * the fp32 dense compute path: SGEMM, row reductions (sum / max / stable
 * softmax), RMSNorm, and the transformer-block pieces built on them.  Oct's Go
 * host resolves these symbols with dlopen/dlsym and calls them through cgo; no
 * Go-side change is needed.  Every declaration below names the reference
 * declaration it replaces (paths are relative to the Oct repository root).
 *
 * Conventions shared by every entry point:
 *   - Return PROM_OK / PROM_ERROR / PROM_INVALID_HANDLE / PROM_INTERNAL_ERROR.
 *   - `out_stage` reports the pipeline stage that finished last (or failed) and
 *     `out_detail_code` a signed detail: negative = failure class, positive =
 *     executed-path identity.
 *   - All host pointers are borrowed for the duration of the call only.
 *   - No C++ exception ever crosses this boundary.
 *   - Handles are validated against a locked registry on every call; calls on
 *     one handle are serialised inside the library.
 *
 * Struct layouts are byte-compatible with the reference because the Go side
 * passes these structs through cgo unchanged.
 *
 * Entry points prefixed `oct_b200_` are extensions with no counterpart in the
 * reference.  They take DEVICE pointers and a CUDA stream, for callers whose
 * data is already resident in HBM (benchmarks, tensor-parallel drivers).
 */
#ifndef OCT_B200_PROMETHEUS_REACTOR_H
#define OCT_B200_PROMETHEUS_REACTOR_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PROM_REACTOR_API __attribute__((visibility("default")))
#else
#define PROM_REACTOR_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- versioning, status, backend (internal/prometheus/native/reactor_api.h:22-83) ---- */
enum { PROM_REACTOR_ABI_V1 = 1u };

enum {
  PROM_OK = 0,
  PROM_ERROR = 1,
  PROM_INVALID_HANDLE = 2,
  PROM_INTERNAL_ERROR = 3,
};

/* backend_type 2 is what Oct's strict `prometheus { }` path demands
   (internal/prometheus/fft.go:50-55); this library reports it for its CUDA
   device backend so the Go host admits it unchanged. */
enum {
  PROM_BACKEND_UNKNOWN = 0,
  PROM_BACKEND_STUB = 1,
  PROM_BACKEND_VULKAN = 2,
  PROM_BACKEND_VULKAN_SOFTWARE = 3,
};

enum {
  PROM_REASON_NONE = 0,
  PROM_REASON_STUB_UNAVAILABLE = 1,
  PROM_REASON_VULKAN_UNAVAILABLE = 2, /* reused: no usable sm_100 CUDA device */
};

enum {
  PROM_STAGE_NONE = 0,
  PROM_STAGE_INIT = 1,
  PROM_STAGE_TRANSFER_IN = 2,
  PROM_STAGE_SUBMIT = 3,
  PROM_STAGE_TRANSFER_OUT = 4,
  PROM_STAGE_CLEANUP = 5,
};

/* ---- async lifecycle (reactor_api.h:85-103) ---- */
enum {
  PROM_ASYNC_STATE_IDLE = 0,
  PROM_ASYNC_STATE_SUBMITTED = 1,
  PROM_ASYNC_STATE_READY = 2,
  PROM_ASYNC_STATE_FAILED = 3,
  PROM_ASYNC_STATE_CONSUMED = 4,
};

enum {
  PROM_ASYNC_FAILURE_NONE = 0,
  PROM_ASYNC_FAILURE_PRE_SUBMIT = 1,
  PROM_ASYNC_FAILURE_OBSERVATION = 2,
  PROM_ASYNC_FAILURE_QUERY = 3,
  PROM_ASYNC_FAILURE_SUBMISSION = 4,
  PROM_ASYNC_FAILURE_DEVICE_LOST = 5,
};

/* ---- host-side fault injection (reactor_api.h:132-159, 194-202) ----
   Only the bits this library honours are listed.  Every injected failure is
   raised on the host before or after a device call; none makes a kernel fault. */
enum {
  PROM_TESTCFG_FAIL_DEVICE_CREATE = 1u << 0,
  PROM_TESTCFG_FAIL_BUFFER_ALLOC = 1u << 2,
  PROM_TESTCFG_FAIL_UPLOAD = 1u << 3,
  PROM_TESTCFG_FAIL_DISPATCH = 1u << 4,
  PROM_TESTCFG_FAIL_DOWNLOAD = 1u << 5,
  PROM_TESTCFG_FAIL_ASYNC_POLL = 1u << 15,
  PROM_TESTCFG_FORCE_STRICT_FP32 = 1u << 17, /* selects the FP32-FMA SGEMM control */
};

enum {
  PROM_REDUCTION_TESTCFG_FAIL_COMMAND_RECORD = 1u << 0,
  PROM_REDUCTION_TESTCFG_FAIL_QUEUE_SUBMIT = 1u << 1,
  PROM_REDUCTION_TESTCFG_FAIL_COMPLETION_OBSERVATION = 1u << 2,
};

/* ---- SGEMM detail codes (reactor_api.h:204-260) ---- */
enum {
  PROM_DETAIL_INJECTED_UPLOAD_FAILURE = -6001,
  PROM_DETAIL_INJECTED_DISPATCH_FAILURE = -6002,
  PROM_DETAIL_INJECTED_DOWNLOAD_FAILURE = -6003,
  PROM_DETAIL_SIZE_OVERFLOW = -6004,
  PROM_DETAIL_REUSE_IN_FLIGHT = -6005,
  PROM_DETAIL_CAPABILITY_MISMATCH = -6006,
  PROM_DETAIL_PATH_DIRECT = 6101,
  PROM_DETAIL_PATH_STAGED_UPLOAD_TILED = 6106,
  PROM_DETAIL_ASYNC_NOT_READY = -6108,
  PROM_DETAIL_ASYNC_NO_TASK = -6109,
  PROM_DETAIL_ASYNC_ALREADY_CONSUMED = -6110,
  PROM_DETAIL_ASYNC_INVALID_TASK = -6111,
  PROM_DETAIL_ASYNC_SUBMIT_REJECTED = -6112,
  PROM_DETAIL_ASYNC_FAILED = -6114,
  PROM_DETAIL_ASYNC_UNCONSUMED = -6115,
  PROM_DETAIL_INJECTED_ASYNC_POLL_FAILURE = -6116,
  PROM_DETAIL_ASYNC_QUEUE_FULL = -6117,
};

/* SGEMM batch detail codes (reactor_api.h:282-295). */
enum {
  PROM_DETAIL_BATCH_PLAN_INVALID = -6602,
  PROM_DETAIL_BATCH_EXECUTION_FAILED = -6604,
  PROM_DETAIL_BATCH_UNSUPPORTED_OPTION = -6613,
};

/* SGEMM batch flags (reactor_api.h:1449-1451).  Bits 0..7 request a number of
   concurrent workers (0 = 1, at most 8); bit 8 selects contiguous instead of
   round-robin assignment of entries to workers.  Every other bit is rejected
   with PROM_DETAIL_BATCH_UNSUPPORTED_OPTION. */
enum {
  PROM_BATCH_FLAG_PARTITION_CONTIGUOUS = 1u << 8,
};

/* Resident SGEMM benchmark modes and flags (reactor_api.h:1561-1580). */
enum {
  PROM_SGEMM_GPU_TIMING_FAILURE_NONE = 0u,
};
enum {
  PROM_SGEMM_RESIDENT_MODE_PRODUCTION_SELECTOR = 0u,
  PROM_SGEMM_RESIDENT_MODE_EXPLICIT_VARIANT = 1u,
};
enum {
  PROM_SGEMM_RESIDENT_FLAG_VALIDATE_READBACK = 1u << 0,
  PROM_SGEMM_RESIDENT_FLAG_M29_SUBMISSION_RING = 1u << 1,
};

/* RMSNorm / RoPE / score detail codes (internal/prometheus/native/reactor_vulkan.h:1870-1888). */
enum {
  PROM_M46_DETAIL_INVALID_REQUEST = -7401,
  PROM_M46_DETAIL_SHAPE = -7403,
  PROM_M46_DETAIL_STRIDE = -7404,
  PROM_M46_DETAIL_STALE_WEIGHT_GENERATION = -7406,
  PROM_M46_DETAIL_EPSILON = -7407,
  PROM_M46_DETAIL_SIZE_OVERFLOW = -7409,
  PROM_M46_DETAIL_RESOURCE = -7411,
  PROM_M46_DETAIL_COMMAND = -7412,
  PROM_M46_DETAIL_SUBMIT = -7413,
  PROM_M46_DETAIL_COMPLETION_UNCERTAIN = -7414,
  PROM_M46_DETAIL_READBACK = -7416,
  PROM_M46_DETAIL_NONFINITE_INPUT = -7418,
};

/* Details with no reference counterpart (this library's device layer). */
enum {
  OCT_B200_DETAIL_CUDA_ERROR = -7001,        /* a CUDA runtime call failed */
  OCT_B200_DETAIL_DEVICE_TIMEOUT = -7002,    /* a bounded in-kernel wait gave up */
  OCT_B200_DETAIL_OUT_OF_MEMORY = -7003,     /* device allocation failed */
  OCT_B200_DETAIL_BAD_VARIANT = -7004,       /* unknown kernel variant id */
  OCT_B200_DETAIL_UNALIGNED = -7005,         /* device pointer not 16-byte aligned */
  OCT_B200_DETAIL_NOALLOC_TOO_LARGE = -7006, /* product needs more than the fixed no-alloc scratch */
  OCT_B200_DETAIL_UNSUPPORTED_SHAPE = -7007, /* shape outside a fused kernel's envelope */
  OCT_B200_DETAIL_INVALID_ARGUMENT = -7008,  /* null pointer, short leading dimension or out-of-range argument */
  OCT_B200_DETAIL_BLOCK_INVALID = -7010,     /* block configuration / slot / count rejected */
  OCT_B200_DETAIL_BLOCK_ALLOC = -7011,       /* block weights or workspaces could not be allocated */
  OCT_B200_DETAIL_BLOCK_NCCL = -7012,        /* tensor-parallel communicator unavailable */
  OCT_B200_DETAIL_BLOCK_NOT_FOUND = -7013,   /* unknown block id */
  OCT_B200_DETAIL_BLOCK_EXEC = -7014,        /* a block kernel or collective failed */
  OCT_B200_DETAIL_TP_INVALID = -7020,        /* tensor-parallel SGEMM configuration or call rejected */
  OCT_B200_DETAIL_TP_ALLOC = -7021,          /* its output / exchange buffers could not be allocated */
  OCT_B200_DETAIL_TP_NCCL = -7022,           /* communicator or peer-memory setup failed */
  OCT_B200_DETAIL_TP_NOT_FOUND = -7023,      /* unknown tensor-parallel SGEMM id */
  OCT_B200_DETAIL_TP_EXEC = -7024,           /* a kernel, copy or collective of the call failed */
};

/* ---- reductions (reactor_api.h:375-581) ---- */
enum {
  PROM_REDUCTION_OPERATION_SUM = 1u,
  PROM_REDUCTION_OPERATION_MAX = 2u,
  PROM_REDUCTION_OPERATION_SOFTMAX = 3u,
};

enum {
  PROM_REDUCTION_FINALIZATION_NONE = 0u,
  PROM_REDUCTION_FINALIZATION_STABLE_SOFTMAX = 1u,
};

enum {
  PROM_REDUCTION_STRATEGY_AUTO = 0u,
  PROM_REDUCTION_STRATEGY_FUSED_SINGLE_WORKGROUP = 1u,
  PROM_REDUCTION_STRATEGY_COMPOSED = 2u,
  PROM_REDUCTION_STRATEGY_PACKED_SHORT_ROWS = 3u,
};

enum {
  PROM_REDUCTION_STAGE_ROW_SUM = 1u,
  PROM_REDUCTION_STAGE_ROW_MAX = 2u,
  PROM_REDUCTION_STAGE_SOFTMAX_EXP_SUM = 3u,
  PROM_REDUCTION_STAGE_SOFTMAX_NORMALIZE = 4u,
  PROM_REDUCTION_STAGE_SOFTMAX_FUSED = 5u,
  PROM_REDUCTION_STAGE_ROW_SUM_PACKED_SHORT = 6u,
  PROM_REDUCTION_STAGE_SOFTMAX_PACKED_SHORT = 7u,
};

enum {
  PROM_REDUCTION_TEMPORARY_NONE = 0u,
  PROM_REDUCTION_TEMPORARY_PARTIALS = 1u,
  PROM_REDUCTION_TEMPORARY_ROW_MAX = 2u,
  PROM_REDUCTION_TEMPORARY_ROW_SUM = 3u,
};

enum {
  PROM_REDUCTION_FLAG_FORCE_FUSED = 1u << 0u,
  PROM_REDUCTION_FLAG_FORCE_COMPOSED = 1u << 1u,
};

enum {
  PROM_REDUCTION_DETAIL_INVALID_REQUEST = -6801,
  PROM_REDUCTION_DETAIL_NULL_INPUT = -6802,
  PROM_REDUCTION_DETAIL_NULL_OUTPUT = -6803,
  PROM_REDUCTION_DETAIL_ZERO_ROW_COUNT = -6804,
  PROM_REDUCTION_DETAIL_ZERO_ROW_WIDTH = -6805,
  PROM_REDUCTION_DETAIL_UNSUPPORTED_OPERATION = -6806,
  PROM_REDUCTION_DETAIL_INVALID_FINALIZATION = -6807,
  PROM_REDUCTION_DETAIL_SIZE_OVERFLOW = -6808,
  PROM_REDUCTION_DETAIL_INPUT_SIZE_MISMATCH = -6809,
  PROM_REDUCTION_DETAIL_OUTPUT_SIZE_MISMATCH = -6810,
  PROM_REDUCTION_DETAIL_ROW_LIMIT = -6811,
  PROM_REDUCTION_DETAIL_WIDTH_LIMIT = -6812,
  PROM_REDUCTION_DETAIL_ELEMENT_LIMIT = -6813,
  PROM_REDUCTION_DETAIL_NONFINITE_INPUT = -6814,
  PROM_REDUCTION_DETAIL_UNSUPPORTED_STRATEGY = -6815,
  PROM_REDUCTION_DETAIL_MALFORMED_PLAN = -6816,
  PROM_REDUCTION_DETAIL_TEMPORARY_UNDERSIZED = -6817,
  PROM_REDUCTION_DETAIL_RESOURCE_CREATE_FAILED = -6818,
  PROM_REDUCTION_DETAIL_PIPELINE_CREATE_FAILED = -6819,
  PROM_REDUCTION_DETAIL_COMMAND_RECORD_FAILED = -6820,
  PROM_REDUCTION_DETAIL_QUEUE_SUBMIT_FAILED = -6821,
  PROM_REDUCTION_DETAIL_COMPLETION_UNCERTAIN = -6822,
  PROM_REDUCTION_DETAIL_QUERY_FAILED = -6823,
  PROM_REDUCTION_DETAIL_READBACK_FAILED = -6824,
  PROM_REDUCTION_DETAIL_RUNTIME_UNAVAILABLE = -6825,
};

enum {
  PROM_SOFTMAX_DETAIL_INVALID_REQUEST = -6851,
  PROM_SOFTMAX_DETAIL_NULL_INPUT = -6852,
  PROM_SOFTMAX_DETAIL_NULL_OUTPUT = -6853,
  PROM_SOFTMAX_DETAIL_COUNT_MISMATCH = -6854,
  PROM_SOFTMAX_DETAIL_SIZE_OVERFLOW = -6855,
  PROM_SOFTMAX_DETAIL_ROW_LIMIT = -6856,
  PROM_SOFTMAX_DETAIL_WIDTH_LIMIT = -6857,
  PROM_SOFTMAX_DETAIL_ELEMENT_LIMIT = -6858,
  PROM_SOFTMAX_DETAIL_PARTIAL_ALIAS = -6859,
  PROM_SOFTMAX_DETAIL_NONFINITE_INPUT = -6860,
  PROM_SOFTMAX_DETAIL_RUNTIME_UNAVAILABLE = -6861,
};

/* Kernel identities reported in a plan.  The reference numbers its Vulkan
   shaders 16-22 (reactor_api.h:480-488); the CUDA kernels here keep those ids
   for the stage roles they fulfil so that plan replay ids stay comparable. */
enum {
  PROM_REDUCTION_SHADER_ROW_SUM = 16u,
  PROM_REDUCTION_SHADER_ROW_MAX = 17u,
  PROM_REDUCTION_SHADER_SOFTMAX_EXP_SUM = 18u,
  PROM_REDUCTION_SHADER_SOFTMAX_NORMALIZE = 19u,
  PROM_REDUCTION_SHADER_SOFTMAX_FUSED = 20u,
  PROM_REDUCTION_SHADER_ROW_SUM_PACKED_SHORT = 21u,
  PROM_REDUCTION_SHADER_SOFTMAX_PACKED_SHORT = 22u,
};

enum {
  PROM_REDUCTION_IMPLEMENTATION_ROW_SUM = 1001u,
  PROM_REDUCTION_IMPLEMENTATION_ROW_MAX = 1002u,
  PROM_REDUCTION_IMPLEMENTATION_SOFTMAX_EXP_SUM = 1003u,
  PROM_REDUCTION_IMPLEMENTATION_SOFTMAX_NORMALIZE = 1004u,
  PROM_REDUCTION_IMPLEMENTATION_SOFTMAX_FUSED = 1005u,
  PROM_REDUCTION_IMPLEMENTATION_ROW_SUM_PACKED_SHORT = 1006u,
  PROM_REDUCTION_IMPLEMENTATION_SOFTMAX_PACKED_SHORT = 1007u,
};

#define PROM_REDUCTION_MAX_STAGES 8u
/* Reference envelope (reactors/PrometheusReduction.concept:66-75).  This
   library WIDENS it deliberately: rows up to OCT_B200_REDUCTION_MAX_ROWS and
   totals up to OCT_B200_REDUCTION_MAX_TOTAL_ELEMENTS are admitted under the
   same symbols; the in-envelope detail codes are unchanged. */
#define PROM_REDUCTION_MAX_ROWS 1024u
#define PROM_REDUCTION_MAX_ELEMENTS_PER_ROW 1048576u
#define PROM_REDUCTION_MAX_TOTAL_ELEMENTS 16777216u
#define PROM_REDUCTION_LOCAL_SIZE 256u
#define PROM_REDUCTION_ELEMENTS_PER_PARTIAL 1024u
#define PROM_REDUCTION_SINGLE_STAGE_THRESHOLD 1024u
#define PROM_REDUCTION_FORCE_FUSED_MAX_ELEMENTS_PER_ROW 1056u
#define PROM_REDUCTION_PACKED_SHORT_WIDTH_MAX 128u
#define PROM_REDUCTION_PACKED_SHORT_SUM_MIN_ROWS 512u
#define PROM_REDUCTION_PACKED_SHORT_SUM_WIDE_MIN_ROWS 1024u
#define PROM_REDUCTION_PACKED_SHORT_ROWS_PER_GROUP 8u
#define PROM_REDUCTION_PACKED_SHORT_LANES_PER_ROW 32u

#define OCT_B200_REDUCTION_MAX_ROWS 16777216u
#define OCT_B200_REDUCTION_MAX_TOTAL_ELEMENTS (1ull << 34)

#define PROM_ROW_WISE_SOFTMAX_MAX_ROWS PROM_REDUCTION_MAX_ROWS
#define PROM_ROW_WISE_SOFTMAX_MAX_ELEMENTS_PER_ROW PROM_REDUCTION_FORCE_FUSED_MAX_ELEMENTS_PER_ROW
#define PROM_ROW_WISE_SOFTMAX_MAX_TOTAL_ELEMENTS PROM_REDUCTION_MAX_TOTAL_ELEMENTS

/* ---- structs (layouts as reactor_api.h:509-664, 1582-1586, 1751-1779) ---- */
typedef struct PrometheusRowWiseSoftmaxRequest {
  uint32_t struct_size;
  const float* input;
  float* output;
  uint32_t row_count;
  uint32_t elements_per_row;
  uint64_t input_element_count;
  uint64_t output_element_count;
} PrometheusRowWiseSoftmaxRequest;

typedef struct PrometheusRowWiseSoftmaxResult {
  uint32_t struct_size;
  uint32_t stage;
  int32_t detail_code;
  uint32_t output_written;
  uint32_t physical_dispatch_count;
  uint32_t physical_submission_count;
  uint32_t gpu_timestamp_valid;
  uint64_t gpu_duration_ns;
  uint64_t end_to_end_ns;
  uint64_t first_nonfinite_index;
} PrometheusRowWiseSoftmaxResult;

typedef struct PrometheusReductionRequest {
  uint32_t struct_size;
  const float* input;
  float* output;
  uint32_t row_count;
  uint32_t elements_per_row;
  uint64_t input_element_count;
  uint64_t output_element_count;
  uint32_t operation;
  uint32_t finalization;
  uint32_t flags;
} PrometheusReductionRequest;

typedef struct PrometheusReductionStageDispatch {
  uint32_t stage_role;
  uint32_t shader_id;
  uint32_t implementation_id;
  uint32_t groups_x;
  uint32_t groups_y;
  uint32_t groups_z;
  uint32_t input_elements_per_row;
  uint32_t output_partials_per_row;
  uint32_t temporary_role;
  uint64_t temporary_bytes_written;
} PrometheusReductionStageDispatch;

typedef struct PrometheusReductionPlan {
  uint32_t struct_size;
  uint32_t operation;
  uint32_t row_count;
  uint32_t elements_per_row;
  uint32_t strategy;
  uint32_t local_size;
  uint32_t elements_per_partial;
  uint32_t partial_count;
  uint32_t stage_count;
  uint32_t temporary_alignment_bytes;
  uint64_t temporary_bytes;
  uint64_t replay_id;
  PrometheusReductionStageDispatch stages[PROM_REDUCTION_MAX_STAGES];
} PrometheusReductionPlan;

typedef struct PrometheusReductionExecutionResult {
  uint32_t struct_size;
  uint32_t stage;
  int32_t detail_code;
  uint64_t logical_request_id;
  uint32_t physical_slot_id;
  uint32_t physical_slot_generation;
  uint32_t physical_slot_recyclable;
  uint32_t gpu_timestamp_valid;
  uint64_t gpu_duration_ns;
  uint64_t end_to_end_ns;
  uint64_t first_nonfinite_index;
  uint32_t validation_error_count_before;
  uint32_t validation_error_count_after;
  PrometheusReductionPlan plan;
} PrometheusReductionExecutionResult;

typedef struct PrometheusReductionBenchmarkRequest {
  uint32_t struct_size;
  PrometheusReductionRequest reduction;
  uint32_t warmup_iterations;
  uint32_t measured_iterations;
} PrometheusReductionBenchmarkRequest;

typedef struct PrometheusReductionBenchmarkResult {
  uint32_t struct_size;
  uint32_t completed_iterations;
  uint32_t correctness_passed;
  uint32_t validation_passed;
  uint32_t device_lost;
  uint32_t stage_count;
  uint64_t temporary_bytes;
  uint64_t replay_id;
  uint64_t gpu_min_ns;
  uint64_t gpu_median_ns;
  uint64_t gpu_max_ns;
  uint64_t end_to_end_min_ns;
  uint64_t end_to_end_median_ns;
  uint64_t end_to_end_max_ns;
  uint32_t first_mismatch_row;
  uint32_t first_mismatch_column;
  float first_expected;
  float first_actual;
  float first_absolute_error;
  float first_relative_error;
  int32_t detail_code;
} PrometheusReductionBenchmarkResult;

/* One independent product of a batch (reactor_api.h:1307-1314). */
typedef struct PrometheusSgemmBatchEntry {
  const float* a;
  const float* b;
  float* c;
  uint32_t m;
  uint32_t n;
  uint32_t k;
} PrometheusSgemmBatchEntry;

/* Resident benchmark request / result (reactor_api.h:2034-2095), same layout. */
typedef struct PrometheusSgemmResidentBenchmarkRequest {
  uint32_t struct_size;
  const float* a;
  const float* b;
  float* c;
  uint32_t m;
  uint32_t n;
  uint32_t k;
  uint32_t mode;
  uint32_t requested_variant;
  uint32_t warmup_iterations;
  uint32_t iterations;
  uint32_t diagnostic_batch_depth;
  uint32_t flags;
} PrometheusSgemmResidentBenchmarkRequest;

typedef struct PrometheusSgemmResidentBenchmarkResult {
  uint32_t struct_size;
  uint32_t resident_mode_available;
  uint32_t resident_mode_used;
  uint32_t requested_variant;
  uint32_t production_selected_variant;
  uint32_t executed_variant;
  uint32_t executed_compute_mode;
  uint32_t setup_stage;
  int32_t setup_detail_code;
  uint32_t final_stage;
  int32_t final_detail_code;
  uint32_t iterations;
  uint32_t gpu_timestamp_valid;
  uint32_t gpu_timing_failure_reason;
  uint64_t setup_wall_ns;
  uint64_t upload_once_wall_ns;
  uint64_t total_loop_wall_ns;
  uint64_t kernel_min_ns;
  uint64_t kernel_median_ns;
  uint64_t kernel_p95_ns;
  uint64_t readback_once_wall_ns;
  uint64_t validation_wall_ns;
  uint64_t dispatch_submit_wall_ns_median;
  uint64_t sync_wait_wall_ns_median;
  uint32_t diagnostic_batch_depth;
  uint32_t queue_submissions;
  uint32_t fence_waits;
  uint32_t command_buffer_recordings;
  uint32_t command_buffer_resets;
  uint32_t descriptor_updates;
  uint64_t query_result_wall_ns_median;
  uint32_t configured_ring_depth;
  uint32_t physical_slot_count;
  uint32_t max_in_flight_depth;
  uint64_t ring_poll_count;
  uint64_t ring_forced_wait_count;
  uint64_t ring_query_harvest_count;
  uint64_t ring_full_count;
  uint64_t ring_slot_recycle_count;
  uint64_t ring_failure_count;
  uint32_t ring_final_slot_state[4];
} PrometheusSgemmResidentBenchmarkResult;

typedef struct PrometheusCaps {
  uint32_t available;
  uint32_t backend_type;
  uint32_t reason_code;
} PrometheusCaps;

typedef struct PrometheusReactorConfig {
  uint32_t struct_size;
  uint32_t test_flags;
  uint32_t p15_shadow_disabled;     /* accepted, ignored: no selector shadow here */
  uint32_t async_test_flags;
  uint32_t batch_ring_depth;        /* accepted, ignored */
  uint32_t reduction_test_flags;
  uint32_t reduction_ring_depth;    /* reported by reduction diagnostics; one CUDA stream per handle */
  const char* shader_package_root;  /* accepted, ignored: kernels are linked in */
} PrometheusReactorConfig;

typedef struct PrometheusAsyncStatus {
  uint32_t lifecycle_state;
  uint32_t stage;
  int detail_code;
  uint32_t ready;
  uint32_t failed;
  uint32_t consumed;
  uint32_t outstanding_tasks;
} PrometheusAsyncStatus;

/* Gemma RMSNorm request/result (reactor_api.h:1781-1825).  Generations and the
   source hash must be non-zero; the weight generation must exceed the one the
   handle last committed (the reference's stale-weight rule). */
typedef struct PrometheusGemma4E2BM1InputRmsNormRequest {
  uint32_t struct_size;
  const float* input;
  const float* weight;
  float* output;
  float* inv_rms_output;
  uint64_t input_element_count;
  uint64_t weight_element_count;
  uint64_t output_element_count;
  uint64_t inv_rms_output_element_count;
  uint32_t tokens;
  uint32_t model_width;
  uint32_t input_row_stride;
  float epsilon;
  uint64_t input_generation;
  uint64_t weight_generation;
  uint64_t exact_source_hash;
} PrometheusGemma4E2BM1InputRmsNormRequest;

typedef struct PrometheusGemma4E2BM1InputRmsNormResult {
  uint32_t struct_size;
  uint32_t stage;
  int32_t detail_code;
  uint32_t output_written;
  uint32_t matched_input;
  uint64_t input_hash;
  uint64_t weight_hash;
  uint64_t output_hash;
  uint64_t inv_rms_hash;
  uint32_t submit_count;
  uint32_t final_readback_count;
  uint32_t no_product_intermediate_readback_change;
  uint32_t reserved0;
  uint64_t retained_bytes;
  uint64_t buffer_allocation_count;
  uint64_t buffer_reuse_count;
  uint64_t descriptor_update_count;
  uint64_t pipeline_create_count;
  uint64_t command_buffer_reuse_count;
  uint64_t reduction_gpu_ns;
  uint64_t final_reduction_gpu_ns;
  uint64_t inv_rms_gpu_ns;
  uint64_t apply_gpu_ns;
  uint64_t end_to_end_ns;
} PrometheusGemma4E2BM1InputRmsNormResult;

typedef PrometheusGemma4E2BM1InputRmsNormRequest PrometheusGemma4E2BM1HeadRmsNormRequest;
typedef PrometheusGemma4E2BM1InputRmsNormResult PrometheusGemma4E2BM1HeadRmsNormResult;

/* Half-split RoPE request/result (reactor_api.h:1835-1871): source and output
   [token][head][component], tables [token][component]; the operation rounds
   its products and sums through BF16 as the reference's storage graph does. */
typedef struct PrometheusGemma4E2BM1RopeRequest {
  uint32_t struct_size;
  const float* source;
  const float* cosine;
  const float* sine;
  float* output;
  uint64_t source_element_count;
  uint64_t cosine_element_count;
  uint64_t sine_element_count;
  uint64_t output_element_count;
  uint32_t tokens;
  uint32_t heads;
  uint32_t head_width;
  uint32_t reserved0;
  uint64_t source_generation;
  uint64_t table_generation;
} PrometheusGemma4E2BM1RopeRequest;

typedef struct PrometheusGemma4E2BM1RopeResult {
  uint32_t struct_size;
  uint32_t stage;
  int32_t detail_code;
  uint32_t output_written;
  uint32_t dispatch_count;
  uint64_t source_hash;
  uint64_t cosine_hash;
  uint64_t sine_hash;
  uint64_t output_hash;
  uint64_t buffer_allocation_count;
  uint64_t buffer_reuse_count;
  uint64_t descriptor_update_count;
  uint64_t pipeline_create_count;
  uint64_t command_buffer_reuse_count;
} PrometheusGemma4E2BM1RopeResult;

/* Head RMSNorm followed by RoPE with nothing read back in between
   (reactor_api.h:1873-1922).  `output` may be NULL (output_element_count 0):
   the positioned rows then stay on the device only. */
typedef struct PrometheusGemma4E2BM1HeadRmsNormRopeRequest {
  uint32_t struct_size;
  const float* input;
  const float* weight;
  const float* cosine;
  const float* sine;
  float* output;
  uint64_t input_element_count;
  uint64_t weight_element_count;
  uint64_t cosine_element_count;
  uint64_t sine_element_count;
  uint64_t output_element_count;
  uint32_t tokens;
  uint32_t heads;
  uint32_t head_width;
  uint32_t reserved0;
  float epsilon;
  uint64_t input_generation;
  uint64_t weight_generation;
  uint64_t table_generation;
  uint64_t exact_source_hash;
} PrometheusGemma4E2BM1HeadRmsNormRopeRequest;

typedef struct PrometheusGemma4E2BM1HeadRmsNormRopeResult {
  uint32_t struct_size;
  uint32_t stage;
  int32_t detail_code;
  uint32_t output_written;
  uint32_t dispatch_count;
  uint32_t resident_source_bound;
  uint32_t normalized_readback_count;
  uint64_t source_byte_offset;
  uint64_t source_byte_range;
  uint64_t destination_byte_offset;
  uint64_t destination_byte_range;
  uint64_t input_hash;
  uint64_t weight_hash;
  uint64_t output_hash;
  uint64_t buffer_allocation_count;
  uint64_t buffer_reuse_count;
  uint64_t descriptor_update_count;
  uint64_t pipeline_create_count;
  uint64_t command_buffer_reuse_count;
  uint64_t observed_weight_generation;
  uint64_t requested_weight_generation;
} PrometheusGemma4E2BM1HeadRmsNormRopeResult;

/* Raw pre-mask attention scores (reactor_api.h:1924-1985): Q and K each go
   through head RMSNorm -> RoPE on the device, then
   scores[head][query][key] = q . k * scale, every query head reading KV head 0. */
typedef struct PrometheusGemma4E2BM1AttentionScoresRequest {
  uint32_t struct_size;
  const float* query_input;
  const float* key_input;
  const float* query_weight;
  const float* key_weight;
  const float* cosine;
  const float* sine;
  float* scores;
  uint64_t query_input_element_count;
  uint64_t key_input_element_count;
  uint64_t query_weight_element_count;
  uint64_t key_weight_element_count;
  uint64_t cosine_element_count;
  uint64_t sine_element_count;
  uint64_t score_element_count;
  uint32_t tokens;
  uint32_t query_heads;
  uint32_t key_heads;
  uint32_t head_width;
  float epsilon;
  float scale;
  uint32_t preparation_order; /* 0: Q then K; 1: K then Q */
  uint64_t query_input_generation;
  uint64_t key_input_generation;
  uint64_t query_weight_generation;
  uint64_t key_weight_generation;
  uint64_t table_generation;
  uint64_t query_exact_source_hash;
  uint64_t key_exact_source_hash;
} PrometheusGemma4E2BM1AttentionScoresRequest;

typedef struct PrometheusGemma4E2BM1AttentionScoresResult {
  uint32_t struct_size;
  uint32_t stage;
  int32_t detail_code;
  uint32_t score_written;
  uint32_t positional_dispatch_count;
  uint32_t score_dispatch_count;
  uint32_t score_readback_count;
  uint32_t host_detour_count;
  uint32_t query_slot_id;
  uint32_t query_slot_generation;
  uint32_t key_slot_id;
  uint32_t key_slot_generation;
  uint32_t score_slot_id;
  uint32_t score_slot_generation;
  uint64_t query_byte_range;
  uint64_t key_byte_range;
  uint64_t score_byte_range;
  uint64_t score_hash;
  uint64_t buffer_allocation_count;
  uint64_t buffer_reuse_count;
  uint64_t descriptor_update_count;
  uint64_t pipeline_create_count;
  uint64_t observed_weight_generation;
  uint64_t requested_weight_generation;
} PrometheusGemma4E2BM1AttentionScoresResult;

/* Reduction diagnostics (reactor_api.h:600-633): counters of the handle's
   reduction executor.  CUDA meaning: one "physical slot" per handle (the
   handle's stream), a "queue submit" is one enqueued launch sequence. */
typedef struct PrometheusReductionDiagnostics {
  uint32_t struct_size;
  uint32_t initialized;
  uint32_t production_enabled;
  uint32_t experimental_enabled;
  uint32_t configured_ring_depth;
  uint32_t physical_slot_count;
  uint32_t acquire_cursor;
  uint32_t outstanding_slots;
  uint32_t quarantined_slots;
  uint64_t next_logical_request_id;
  uint64_t total_requests;
  uint64_t successful_requests;
  uint64_t logical_failure_count;
  uint64_t physical_recycle_count;
  uint64_t quarantine_count;
  uint64_t reap_count;
  uint64_t pipeline_create_count;
  uint64_t descriptor_update_count;
  uint64_t command_record_count;
  uint64_t queue_submit_count;
  uint64_t buffer_allocation_count;
  uint64_t buffer_reuse_count;
  uint64_t temporary_capacity_bytes;
  uint64_t last_replay_id;
  uint64_t last_gpu_duration_ns;
  uint64_t last_end_to_end_ns;
  uint32_t last_stage_count;
  uint32_t last_physical_slot_id;
  uint32_t last_physical_slot_generation;
  int32_t last_detail_code;
  uint32_t validation_enabled;
  uint32_t validation_error_count;
} PrometheusReductionDiagnostics;

/* Async SGEMM diagnostics (reactor_api.h:1987-2032).  One physical slot per
   task; quarantine and deferred feedback do not exist on CUDA and stay 0. */
typedef struct PrometheusSgemmAsyncTaskDiagnostics {
  int32_t task_id;
  uint32_t generation;
  uint32_t lifecycle_state;
  uint32_t physical_slot_id;
  uint32_t physical_slot_generation;
  uint64_t submission_sequence;
  uint32_t timing_valid;
  uint64_t gpu_duration_ns;
  uint32_t feedback_pending;
  uint32_t feedback_committed;
  int32_t failure_detail;
  uint32_t failure_class;
  uint32_t abandoned;
  uint32_t physical_slot_state;
  uint32_t quarantined;
  uint32_t physical_completion_confirmed;
  uint32_t reap_pending;
  uint32_t reap_completed;
} PrometheusSgemmAsyncTaskDiagnostics;

typedef struct PrometheusSgemmAsyncDiagnostics {
  uint32_t task_capacity;
  uint32_t active_task_count;
  uint32_t submitted_count;
  uint32_t ready_count;
  uint32_t failed_count;
  uint32_t consumed_count;
  uint32_t abandoned_count;
  uint64_t queue_full_count;
  uint64_t stale_id_rejection_count;
  uint32_t max_in_flight;
  uint32_t feedback_pending_count;
  uint64_t feedback_committed_count;
  uint64_t feedback_skipped_count;
  uint64_t next_feedback_sequence;
  uint32_t quarantined_slot_count;
  uint64_t quarantine_event_count;
  uint64_t reap_poll_count;
  uint64_t reap_success_count;
  uint64_t reap_wait_count;
  uint64_t reap_failure_count;
  uint32_t max_quarantine_depth;
  uint32_t runtime_unsafe_to_reuse;
  PrometheusSgemmAsyncTaskDiagnostics tasks[4];
} PrometheusSgemmAsyncDiagnostics;

/* Envelope of the Gemma M1 entry points.  The reference admits only the M1
   geometry (15 tokens, 8 or 1 heads of 256, internal/prometheus/native/
   reactor_api.c:370-395, 404-441, 507-547; reactor_concept_rmsnorm.cpp:157-212);
   this library widens the ceilings below and keeps the same detail codes for
   requests inside the reference's envelope. */
#define OCT_B200_M1_MAX_TOKENS 65536u
#define OCT_B200_M1_MAX_HEADS 64u
#define OCT_B200_M1_MAX_HEAD_WIDTH 1024u

/* ==== reference ABI entry points ==== */

/* reactor_api.h:2557 -- always returns PROM_REACTOR_ABI_V1 (bridge.go:276-290 checks it). */
PROM_REACTOR_API uint32_t prometheus_reactor_abi_version(void);
/* reactor_api.h:2558 -- config may be NULL; tail fields gated by struct_size. */
PROM_REACTOR_API int prometheus_reactor_runtime_create(void* config, void** out_handle);
/* reactor_api.h:2559 -- requires quiescent callers. */
PROM_REACTOR_API int prometheus_reactor_runtime_destroy(void* handle);
/* reactor_api.h:2560 -- available=1, backend_type=2 on a usable sm_100 device. */
PROM_REACTOR_API int prometheus_reactor_runtime_probe(void* handle, PrometheusCaps* out_caps);

/* reactor_api.h:2587-2595 -- C[m x n] = A[m x k] * B[k x n], row-major fp32 host
   buffers, C overwritten.  Sizes beyond the reference's u32 m*n*k ceiling
   (reactor_sgemm.cpp:4171-4176) are admitted: only host/device capacity
   limits apply.  Success reports stage TRANSFER_OUT and PROM_DETAIL_PATH_DIRECT. */
PROM_REACTOR_API int prometheus_reactor_runtime_sgemm(void* handle, const float* a, const float* b, float* c,
                                                      uint32_t m, uint32_t n, uint32_t k,
                                                      uint32_t* out_stage, int* out_detail_code);

/* reactor_api.h:2623-2643 -- non-blocking SGEMM.  The library owns the result
   until consume copies it into `c` (length-checked) or abandon drops it. */
/* SGEMM with an explicit kernel variant (reactor_api.h:2596-2605).  The
   reference's variant ids name its Vulkan shaders; here they name this
   library's kernels: 0 = production selector (as prometheus_reactor_runtime_sgemm),
   else one of OCT_B200_SGEMM_* below.  Any other id: PROM_ERROR, stage INIT,
   OCT_B200_DETAIL_BAD_VARIANT. */
PROM_REACTOR_API int prometheus_reactor_runtime_sgemm_benchmark_variant(void* handle, const float* a, const float* b,
                                                                        float* c, uint32_t m, uint32_t n, uint32_t k,
                                                                        uint32_t requested_variant,
                                                                        uint32_t* out_stage, int* out_detail_code);
/* Resident benchmark (reactor_api.h:2606-2609; reactor_sgemm.cpp:5629-5978):
   A and B are uploaded once, one setup product runs, then warmup + iterations
   products run on the resident buffers, each timed with CUDA events (kernel
   min / median / p95 in ns).  With the M29 ring flag up to
   diagnostic_batch_depth (1..4, default 2) products stay in flight.  With
   VALIDATE_READBACK, C is copied to request->c once at the end. */
PROM_REACTOR_API int prometheus_reactor_runtime_sgemm_resident_benchmark(
    void* handle, const PrometheusSgemmResidentBenchmarkRequest* request,
    PrometheusSgemmResidentBenchmarkResult* out_result);
/* Independent host-buffer products (reactor_api.h:2610-2615; reactor_batch.c:244-520):
   entries run concurrently on up to 8 CUDA streams, and every C is written,
   in entry order, only after all entries succeeded (stage TRANSFER_OUT,
   detail 0); on failure no caller output is touched. */
PROM_REACTOR_API int prometheus_reactor_runtime_sgemm_batch(void* handle, const PrometheusSgemmBatchEntry* entries,
                                                            uint32_t entry_count, uint32_t flags,
                                                            uint32_t* out_stage, int* out_detail_code);
PROM_REACTOR_API int prometheus_reactor_runtime_sgemm_submit_async(void* handle, const float* a, const float* b,
                                                                   uint32_t m, uint32_t n, uint32_t k,
                                                                   int* out_task_id, uint32_t* out_stage,
                                                                   int* out_detail_code);
PROM_REACTOR_API int prometheus_reactor_runtime_sgemm_query_async(void* handle, int task_id,
                                                                  PrometheusAsyncStatus* out_status);
PROM_REACTOR_API int prometheus_reactor_runtime_sgemm_consume_async(void* handle, int task_id, float* c,
                                                                    uint32_t c_len, uint32_t* out_stage,
                                                                    int* out_detail_code);
PROM_REACTOR_API int prometheus_reactor_runtime_sgemm_abandon_async(void* handle, int task_id);
/* reactor_api.h:2635-2636 -- task table and lifecycle counters of the async SGEMM queue. */
PROM_REACTOR_API int prometheus_reactor_runtime_sgemm_async_diagnostics(void* handle,
                                                                         PrometheusSgemmAsyncDiagnostics* out_diag);

/* reactor_api.h:2671-2672 -- host-only planner; same stage roles as the
   reference schedule (reactors/PrometheusReduction.concept:128-164). */
PROM_REACTOR_API int prometheus_reactor_reduction_plan(const PrometheusReductionRequest* request,
                                                        PrometheusReductionPlan* out_plan);
/* reactor_api.h:2673-2675 -- row SUM / MAX / stable SOFTMAX over host buffers. */
PROM_REACTOR_API int prometheus_reactor_runtime_reduction(void* handle, const PrometheusReductionRequest* request,
                                                          PrometheusReductionExecutionResult* out_result);
/* reactor_api.h:2676-2677 -- counters of the handle's reduction executor. */
PROM_REACTOR_API int prometheus_reactor_runtime_reduction_diagnostics(void* handle,
                                                                      PrometheusReductionDiagnostics* out_diag);
/* reactor_api.h:2678-2681 -- warm-up and measured executions of one reduction
   request, then a correctness check of the last output (reactor_vulkan_fused_
   reduction.c:1122-1206).  The check runs on the device: an independent
   recomputation and the reference comparator's tolerances. */
PROM_REACTOR_API int prometheus_reactor_runtime_reduction_benchmark(void* handle,
                                                                    const PrometheusReductionBenchmarkRequest* request,
                                                                    PrometheusReductionBenchmarkResult* out_result);
/* reactor_api.h:2682-2685 -- forced fused softmax; rejects partial aliasing and
   non-finite input like reactor_vulkan_fused_reduction.c:892-994. */
PROM_REACTOR_API int prometheus_reactor_runtime_row_wise_softmax(void* handle,
                                                                 const PrometheusRowWiseSoftmaxRequest* request,
                                                                 PrometheusRowWiseSoftmaxResult* out_result);
/* reactor_api.h:2686-2691 -- RMSNorm y = x / sqrt(mean(x^2) + eps) * weight per
   token row; inv_rms_output receives the per-row scale. */
PROM_REACTOR_API int prometheus_reactor_runtime_gemma4e2b_m1_input_rmsnorm(
    void* handle, const PrometheusGemma4E2BM1InputRmsNormRequest* request,
    PrometheusGemma4E2BM1InputRmsNormResult* out_result);
/* reactor_api.h:2692-2695 -- the same RMSNorm with its output rounded to BF16
   (the Q/K/V projections' activation storage boundary, reactor_api.c:362-368). */
PROM_REACTOR_API int prometheus_reactor_runtime_gemma4e2b_m1_projection_activation_rmsnorm(
    void* handle, const PrometheusGemma4E2BM1InputRmsNormRequest* request,
    PrometheusGemma4E2BM1InputRmsNormResult* out_result);
/* reactor_api.h:2696-2699 -- the same primitive over [token, head, channel] rows,
   input and output rounded to BF16, epsilon 1e-6, row stride = width
   (reactor_api.c:370-395; the reference's 120-row / 256-wide ceilings are widened). */
PROM_REACTOR_API int prometheus_reactor_runtime_gemma4e2b_m1_head_rmsnorm(
    void* handle, const PrometheusGemma4E2BM1HeadRmsNormRequest* request,
    PrometheusGemma4E2BM1HeadRmsNormResult* out_result);
/* reactor_api.h:2700-2703 -- half-split RoPE with BF16 products and sums
   (cpuGemma4e2bRope, gemma4e2b_m1_rtx.go:834-861). */
PROM_REACTOR_API int prometheus_reactor_runtime_gemma4e2b_m1_rope(
    void* handle, const PrometheusGemma4E2BM1RopeRequest* request, PrometheusGemma4E2BM1RopeResult* out_result);
/* reactor_api.h:2704-2707 -- head RMSNorm then RoPE in one device pass (reactor_api.c:404-505). */
PROM_REACTOR_API int prometheus_reactor_runtime_gemma4e2b_m1_head_rmsnorm_rope(
    void* handle, const PrometheusGemma4E2BM1HeadRmsNormRopeRequest* request,
    PrometheusGemma4E2BM1HeadRmsNormRopeResult* out_result);
/* reactor_api.h:2708-2711 -- both positional preparations, then the raw scores
   (reactor_api.c:507-586; cpuGemma4e2bRawScores, gemma4e2b_m1_rtx.go:863-883). */
PROM_REACTOR_API int prometheus_reactor_runtime_gemma4e2b_m1_attention_scores(
    void* handle, const PrometheusGemma4E2BM1AttentionScoresRequest* request,
    PrometheusGemma4E2BM1AttentionScoresResult* out_result);

/* ==== FFT (reactor_api.h:327-380, 1251-1305, 2654-2669) ====
   Radix-2 decimation-in-time complex transforms of N = 2^k <= 2^20 points.
   fft64 (the entry Go's FFT engine binds, internal/prometheus/fft.go:21-44):
   one forward unnormalised transform of interleaved binary64 (re, im) pairs;
   twiddles are computed in binary64 on the host, as the reference does
   (reactor_concept_fft.cpp:51-58), and the butterflies run the reference's
   arithmetic exactly (shaders/sdslv/production/fft/radix2_fp64.sdslv).
   fft: batches of interleaved fp32 pairs, stride_elements apart (0 = N),
   forward or inverse, optionally normalised by 1/N; fp32 twiddles from the
   per-pass angle (radix2_butterfly.sdslv).  Only each batch's N outputs are
   written; the caller's elements between batches are left untouched. */
typedef struct PrometheusComplex32 {
  float real;
  float imag;
} PrometheusComplex32;

enum {
  PROM_FFT_FLAG_FORWARD = 1u << 0,
  PROM_FFT_FLAG_INVERSE = 1u << 1,
  PROM_FFT_FLAG_INVERSE_NORMALIZE = 1u << 2,
  PROM_FFT_FLAG_BENCHMARK_ALLOW_NON_PRODUCTION_PATH = 1u << 3,
};

enum {
  PROM_FFT_PATH_NONE = 0,
  PROM_FFT_PATH_UNAVAILABLE = 1,
  PROM_FFT_PATH_CPU_ORACLE_RESERVED = 2,
  PROM_FFT_PATH_VULKAN_RADIX2_RESERVED = 3, /* the radix-2 device route (here: CUDA) */
};

enum {
  PROM_FFT_PATH_STATUS_UNAVAILABLE = 0,
  PROM_FFT_PATH_STATUS_REGISTERED = 1,
  PROM_FFT_PATH_STATUS_BENCHMARK_ENABLED = 2,
  PROM_FFT_PATH_STATUS_PRODUCTION_ENABLED = 3,
};

enum {
  PROM_FFT_BENCHMARK_VARIANT_NONE = 0,
  PROM_FFT_BENCHMARK_VARIANT_RADIX2 = 2,
};

enum {
  PROM_FFT_DETAIL_UNAVAILABLE = -6701,
  PROM_FFT_DETAIL_INVALID_REQUEST = -6702,
  PROM_FFT_DETAIL_NULL_INPUT = -6703,
  PROM_FFT_DETAIL_NULL_OUTPUT = -6704,
  PROM_FFT_DETAIL_ZERO_ELEMENT_COUNT = -6705,
  PROM_FFT_DETAIL_NON_POWER_OF_TWO = -6706,
  PROM_FFT_DETAIL_INVALID_DIRECTION_FLAGS = -6707,
  PROM_FFT_DETAIL_INVALID_STRIDE = -6708,
  PROM_FFT_DETAIL_SIZE_OVERFLOW = -6709,
  PROM_FFT_DETAIL_ZERO_BATCH_COUNT = -6710,
  PROM_FFT_DETAIL_INVERSE_NORMALIZE_REQUIRES_INVERSE = -6711,
  PROM_FFT_DETAIL_VULKAN_UNAVAILABLE = -6712, /* no usable device */
  PROM_FFT_DETAIL_UNSUPPORTED_SIZE = -6713,
  PROM_FFT_DETAIL_ALLOCATION_FAILED = -6714,
  PROM_FFT_DETAIL_UPLOAD_FAILED = -6715,
  PROM_FFT_DETAIL_DISPATCH_FAILED = -6716,
  PROM_FFT_DETAIL_READBACK_FAILED = -6717,
  PROM_FFT_DETAIL_SHADER_UNAVAILABLE = -6718,
  PROM_FFT_DETAIL_PLAN_DISPATCH_DISAGREEMENT = -6719,
  PROM_FFT_DETAIL_FLOAT64_UNAVAILABLE = -6720,
};

typedef struct PrometheusFftRequest {
  uint32_t struct_size;
  const PrometheusComplex32* input;
  PrometheusComplex32* output;
  uint32_t element_count;
  uint32_t batch_count;
  uint32_t stride_elements;
  uint32_t flags;
} PrometheusFftRequest;

typedef struct PrometheusFftDiagnostics {
  uint32_t struct_size;
  uint32_t api_declared;
  uint32_t capability_reported;
  uint32_t production_enabled;
  uint32_t benchmark_enabled;
  uint32_t last_element_count;
  uint32_t last_batch_count;
  uint32_t last_stride_elements;
  uint32_t last_effective_stride_elements;
  uint32_t last_flags;
  uint32_t last_direction;
  uint32_t last_validation_status;
  int32_t last_failure_detail;
  uint32_t requested_path_id;
  uint32_t executed_path_id;
  uint32_t requested_radix;
  uint32_t executed_radix;
  uint32_t fallback_reason;
  uint32_t plan_pass_count;
  uint32_t ping_pong_swap_count;
  uint32_t final_output_role;
  uint64_t ping_arena_reuse_count;
  uint64_t ping_arena_grow_count;
  uint64_t pong_arena_reuse_count;
  uint64_t pong_arena_grow_count;
  uint64_t twiddle_arena_reuse_count;
  uint64_t twiddle_arena_grow_count;
  uint32_t selector_cache_valid;
  uint32_t plan_valid;
  uint32_t plan_element_count;
  uint32_t plan_log2_element_count;
  uint32_t plan_first_span;
  uint32_t plan_last_span;
  uint32_t plan_radix_mask;
  uint32_t plan_bit_reversal_required;
  uint32_t plan_first_source_role;
  uint32_t plan_first_destination_role;
  uint32_t plan_direction;
  uint32_t plan_twiddle_mode;
  uint64_t selector_cache_reuse_count;
  uint64_t selector_cache_recompute_count;
  uint64_t selector_cache_invalidation_count;
  uint64_t selector_cache_last_dependency_mask;
} PrometheusFftDiagnostics;

/* reactor_api.h:2652-2654 -- forward unnormalised binary64 FFT of `count`
   interleaved pairs (reactor_concept_fft.cpp:107-116). */
PROM_REACTOR_API int prometheus_reactor_runtime_fft64(void* handle, const double* input, double* output,
                                                      uint32_t count, uint32_t* stage, int* detail);
/* reactor_api.h:2655-2658 -- batched fp32 FFT; validation order of
   reactor_vulkan_fft.c:59-86, plan bookkeeping of :88-114. */
PROM_REACTOR_API int prometheus_reactor_runtime_fft(void* handle, const PrometheusFftRequest* request,
                                                    uint32_t* out_stage, int* out_detail_code);
/* reactor_api.h:2659-2663 -- the radix-2 variant (2) only. */
PROM_REACTOR_API int prometheus_reactor_runtime_fft_benchmark_variant(void* handle,
                                                                      const PrometheusFftRequest* request,
                                                                      uint32_t requested_variant, uint32_t* out_stage,
                                                                      int* out_detail_code);
/* reactor_api.h:2664-2669 -- the handle's FFT diagnostics (sized: copy out_size bytes). */
PROM_REACTOR_API int prometheus_reactor_runtime_fft_diagnostics(void* handle, PrometheusFftDiagnostics* out_diag);
PROM_REACTOR_API int prometheus_reactor_runtime_fft_diagnostics_sized(void* handle, PrometheusFftDiagnostics* out_diag,
                                                                      uint32_t out_size);

/* ==== Z-Image model-block executors (reactor_api.h:666-1250, 2713-2784) ====
   One closed model block per handle, as in the reference (one model_block
   state per runtime, reactor_vulkan_model_block.c:1603-1780):
     family 0, shader 23        the resident identity proof: output = input;
     noise refiner (family 1)   Z-Image Turbo noise_refiner.{0,1}: BF16 image
                                tokens [1024][3840] and a BF16 256-d timestep
                                embedding in, the FP32 block output resident;
     context refiner (family 2) context_refiner.{0,1}: FP32 caption tokens
                                [32][3840], unmodulated, output resident.
   Weights are uploaded as the reference's cache payloads: IEEE binary16, linear
   weights row-major [in][out], in the cache manifest's lexical order (the byte
   counts below).  The block runs on the library's DiT block (tcgen05 3xTF32
   products, fused attention, fused norm / modulation / gated residuals); the
   FP16 weights are widened exactly to fp32 and held pre-split for the tensor
   cores, so a block holds about four times the declared weight bytes on the
   device.  The staged M1B / M1C / M1D audit executes, static audits, the
   30-layer main transformer and compiled-model sessions are not provided. */
#define PROM_MODEL_BLOCK_MAX_WEIGHTS 13u
#define PROM_MODEL_BLOCK_MAX_STEPS 7u
#define PROM_MODEL_BLOCK_MAX_AUDIT_POINTS 1u
#define PROM_MODEL_BLOCK_M1B_PIPELINE_COUNT 6u
#define PROM_MODEL_BLOCK_MAIN_STAGE_COUNT 13u

enum {
  PROM_MODEL_BLOCK_STEP_BIND_PIPELINE = 1u,
  PROM_MODEL_BLOCK_STEP_BIND_RESOURCES = 2u,
  PROM_MODEL_BLOCK_STEP_PUSH_CONSTANTS = 3u,
  PROM_MODEL_BLOCK_STEP_DISPATCH = 4u,
  PROM_MODEL_BLOCK_STEP_BARRIER = 5u,
  PROM_MODEL_BLOCK_STEP_AUDIT_COPY = 6u,
  PROM_MODEL_BLOCK_STEP_OUTPUT_COPY = 7u,
};

enum {
  PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST = -6901,
  PROM_MODEL_BLOCK_DETAIL_NOT_FOUND = -6902,
  PROM_MODEL_BLOCK_DETAIL_ALREADY_CREATED = -6903,
  PROM_MODEL_BLOCK_DETAIL_WEIGHT_MISMATCH = -6904,
  PROM_MODEL_BLOCK_DETAIL_RESOURCE_CREATE_FAILED = -6905,
  PROM_MODEL_BLOCK_DETAIL_PIPELINE_CREATE_FAILED = -6906,
  PROM_MODEL_BLOCK_DETAIL_UPLOAD_FAILED = -6907,
  PROM_MODEL_BLOCK_DETAIL_COMMAND_RECORD_FAILED = -6908,
  PROM_MODEL_BLOCK_DETAIL_QUEUE_SUBMIT_FAILED = -6909,
  PROM_MODEL_BLOCK_DETAIL_COMPLETION_UNCERTAIN = -6910,
  PROM_MODEL_BLOCK_DETAIL_AUDIT_FAILED = -6911,
  PROM_MODEL_BLOCK_DETAIL_STALE_OUTPUT = -6912,
  PROM_MODEL_BLOCK_DETAIL_INGRESS_PIPELINE_CREATE_FAILED = -6913,
  PROM_MODEL_BLOCK_DETAIL_INGRESS_DISPATCH_FAILED = -6914,
  PROM_MODEL_BLOCK_DETAIL_INGRESS_AUDIT_MISMATCH = -6915,
  PROM_MODEL_BLOCK_DETAIL_INGRESS_INPUT_SIZE_MISMATCH = -6916,
  PROM_MODEL_BLOCK_DETAIL_INGRESS_TIMESTEP_SIZE_MISMATCH = -6917,
  PROM_MODEL_BLOCK_DETAIL_M1C_SOFTMAX_INVALID = -6918,
  PROM_MODEL_BLOCK_DETAIL_M1D_NONFINITE = -6919,
  PROM_MODEL_BLOCK_DETAIL_PARAMETER_SET_MISMATCH = -6920,
  PROM_MODEL_BLOCK_DETAIL_REBIND_FAILED = -6921,
  PROM_MODEL_BLOCK_DETAIL_DESCRIPTOR_UPDATE_FAILED = -6922,
};

enum {
  PROM_NOISE_REFINER_FAMILY_Z_IMAGE_TURBO = 1u,
  PROM_NOISE_REFINER_PARAMETER_SET_0 = 1u,
  PROM_NOISE_REFINER_PARAMETER_SET_1 = 2u,
  PROM_CONTEXT_REFINER_FAMILY_Z_IMAGE_TURBO = 2u,
  PROM_CONTEXT_REFINER_PARAMETER_SET_0 = 1u,
  PROM_CONTEXT_REFINER_PARAMETER_SET_1 = 2u,
  PROM_MAIN_TRANSFORMER_FAMILY_Z_IMAGE_TURBO = 3u,
  PROM_MAIN_TRANSFORMER_PARAMETER_SET_0 = 1u,
};

enum {
  PROM_NOISE_REFINER_BINDING_BOUND = 1u,
  PROM_NOISE_REFINER_BINDING_VALIDATING = 2u,
  PROM_NOISE_REFINER_BINDING_UPLOADING = 3u,
  PROM_NOISE_REFINER_BINDING_UPDATING_DESCRIPTORS = 4u,
  PROM_NOISE_REFINER_BINDING_READY_TO_COMMIT = 5u,
  PROM_NOISE_REFINER_BINDING_COMMITTED = 6u,
  PROM_NOISE_REFINER_BINDING_FAILED_BEFORE_COMMIT = 7u,
  PROM_NOISE_REFINER_BINDING_COMPLETION_UNCERTAIN = 8u,
  PROM_NOISE_REFINER_BINDING_QUARANTINED = 9u,
};

enum {
  PROM_NOISE_REFINER_AUDIT_NONE = 0u,
  PROM_NOISE_REFINER_AUDIT_M1B = 1u,
  PROM_NOISE_REFINER_AUDIT_M1C = 2u,
  PROM_NOISE_REFINER_AUDIT_M1D = 3u,
};

/* The Z-Image Turbo model lock's identities the closed families are checked
   against (internal/prometheus/models/zimage-turbo/resolved_descriptor.h:5-15,
   resolved_audit_schedule.h:6). */
#define OCT_B200_ZIMAGE_TURBO_LOCK_ID 0x71ef202b4e34b562ull
#define OCT_B200_ZIMAGE_NOISE_REFINER0_AGGREGATE 0xa1ba526898a2a752ull
#define OCT_B200_ZIMAGE_NOISE_REFINER1_AGGREGATE 0x80c0cd75f44cc434ull
#define OCT_B200_ZIMAGE_CONTEXT_REFINER0_AGGREGATE 0xc08b908a921a80e1ull
#define OCT_B200_ZIMAGE_CONTEXT_REFINER1_AGGREGATE 0x30268c3b0d7a6fafull
#define OCT_B200_ZIMAGE_CONTEXT_MEMORY_PLAN_BYTES 536870912ull
#define OCT_B200_ZIMAGE_AUDIT_ARENA_BYTES 47186176u

typedef struct PrometheusModelBlockWeightDeclaration {
  uint64_t content_identity;
  uint64_t layout_identity;
  uint64_t byte_count;
} PrometheusModelBlockWeightDeclaration;

typedef struct PrometheusModelBlockCreateRequest {
  uint32_t struct_size;
  uint32_t assembly_family;
  uint32_t parameter_set;
  uint64_t parameter_set_aggregate_identity;
  uint64_t model_contract_identity;
  uint64_t weight_identity;
  uint64_t shader_portfolio_identity;
  uint64_t precision_policy_identity;
  uint64_t capability_route_identity;
  uint64_t memory_ceiling_bytes;
  uint64_t external_input_bytes;
  uint64_t external_output_bytes;
  uint64_t audit_bytes;
  uint32_t shader_id;
  uint32_t weight_count;
  PrometheusModelBlockWeightDeclaration weights[PROM_MODEL_BLOCK_MAX_WEIGHTS];
  uint32_t step_count;
  uint32_t steps[PROM_MODEL_BLOCK_MAX_STEPS];
} PrometheusModelBlockCreateRequest;

typedef struct PrometheusModelBlockWeightUpload {
  uint32_t binding_index;
  const void* bytes;
  uint64_t byte_count;
  uint64_t content_identity;
  uint64_t layout_identity;
} PrometheusModelBlockWeightUpload;

typedef struct PrometheusNoiseRefinerRebindRequest {
  uint32_t struct_size;
  uint32_t model_local_block_id;
  uint64_t lock_identity;
  uint32_t upload_count;
  const PrometheusModelBlockWeightUpload* uploads;
} PrometheusNoiseRefinerRebindRequest;

typedef struct PrometheusContextRefinerCreateRequest {
  uint32_t struct_size;
  uint32_t model_local_block_id;
  uint64_t lock_identity;
  uint32_t upload_count;
  const PrometheusModelBlockWeightUpload* uploads;
} PrometheusContextRefinerCreateRequest;

typedef PrometheusContextRefinerCreateRequest PrometheusContextRefinerRebindRequest;

typedef struct PrometheusModelBlockExecuteRequest {
  uint32_t struct_size;
  const float* input;
  float* output;
  uint64_t element_count;
  uint64_t input_identity;
  uint32_t audit_enabled;
  float* audit_output;
  uint64_t audit_element_capacity;
} PrometheusModelBlockExecuteRequest;

typedef struct PrometheusNoiseRefiner0ExecuteRequest {
  uint32_t struct_size;
  const void* model_input_bf16;
  const void* timestep_bf16;
  uint64_t model_input_bytes;
  uint64_t timestep_bytes;
  uint64_t input_identity;
  uint64_t timestep_identity;
  uint64_t output_identity;
  uint32_t audit_enabled;
} PrometheusNoiseRefiner0ExecuteRequest;

typedef PrometheusNoiseRefiner0ExecuteRequest PrometheusNoiseRefiner1ExecuteRequest;

typedef struct PrometheusNoiseRefinerResidentExecuteRequest {
  uint32_t struct_size;
  uint64_t input_generation;
  uint64_t output_identity;
  uint32_t audit_enabled;
  uint32_t audit_family;
  uint32_t audit_stage;
  float* audit_output;
  uint64_t audit_element_capacity;
} PrometheusNoiseRefinerResidentExecuteRequest;

typedef struct PrometheusContextRefiner0ExecuteRequest {
  uint32_t struct_size;
  const float* context_input;
  uint64_t context_input_bytes;
  uint64_t input_identity;
  uint64_t output_identity;
  uint32_t audit_enabled;
} PrometheusContextRefiner0ExecuteRequest;

typedef struct PrometheusContextRefinerResidentExecuteRequest {
  uint32_t struct_size;
  uint64_t input_generation;
  uint64_t output_identity;
  uint32_t audit_enabled;
} PrometheusContextRefinerResidentExecuteRequest;

typedef struct PrometheusNoiseRefinerFinalAuditRequest {
  uint32_t struct_size;
  uint64_t required_output_generation;
  uint64_t output_identity;
  float* output;
  uint64_t output_element_capacity;
} PrometheusNoiseRefinerFinalAuditRequest;

typedef PrometheusNoiseRefinerFinalAuditRequest PrometheusContextRefinerFinalAuditRequest;

/* Evidence of the model block (reactor_api.h:1105-1183).  CUDA meaning of the
   counters: a "pipeline" is a kernel the block launches, a "queue submit" one
   enqueued forward; the vk_* counters stay 0. */
typedef struct PrometheusModelBlockEvidence {
  uint32_t struct_size;
  int32_t detail_code;
  uint32_t created;
  uint32_t weights_uploaded;
  uint32_t quarantined;
  uint32_t output_valid;
  uint32_t audit_valid;
  uint32_t fixed_step_count;
  uint32_t weight_count;
  uint64_t persistent_bytes;
  uint64_t reusable_bytes;
  uint64_t audit_bytes;
  uint64_t external_bytes;
  uint64_t total_committed_bytes;
  uint64_t peak_plan_bytes;
  uint64_t cold_buffer_allocation_count;
  uint64_t warm_buffer_allocation_count;
  uint64_t pipeline_create_count;
  uint64_t descriptor_set_count;
  uint64_t weight_upload_count;
  uint64_t execution_count;
  uint64_t last_execution_ns;
  uint64_t execution_plan_identity;
  uint64_t replay_identity;
  uint32_t assembly_family;
  uint32_t parameter_set;
  uint32_t binding_state;
  uint32_t active_weight_window;
  uint64_t parameter_set_aggregate_identity;
  uint64_t binding_generation;
  uint64_t output_generation;
  uint64_t descriptor_generation;
  uint64_t m1b_boundary_gpu_ns[PROM_MODEL_BLOCK_M1B_PIPELINE_COUNT];
  uint64_t gpu_total_begin_tick;
  uint64_t gpu_total_end_tick;
  uint64_t gpu_total_ns;
  uint64_t gpu_compute_begin_tick;
  uint64_t gpu_compute_end_tick;
  uint64_t gpu_compute_ns;
  uint64_t gpu_ingress_transfer_ns;
  uint64_t gpu_joint_copy_ns;
  uint64_t gpu_readback_ns;
  uint64_t main_stage_gpu_begin_tick[PROM_MODEL_BLOCK_MAIN_STAGE_COUNT];
  uint64_t main_stage_gpu_end_tick[PROM_MODEL_BLOCK_MAIN_STAGE_COUNT];
  uint64_t main_stage_gpu_ns[PROM_MODEL_BLOCK_MAIN_STAGE_COUNT];
  uint64_t last_active_target_validation_ns;
  uint64_t last_command_reset_ns;
  uint64_t last_command_begin_ns;
  uint64_t last_command_record_ns;
  uint64_t last_command_end_ns;
  uint64_t last_queue_submit_ns;
  uint64_t last_fence_wait_ns;
  uint64_t last_descriptor_update_ns;
  uint64_t last_staging_memcpy_ns;
  uint64_t last_output_readback_ns;
  uint64_t vk_create_buffer_count;
  uint64_t vk_destroy_buffer_count;
  uint64_t vk_allocate_memory_count;
  uint64_t vk_free_memory_count;
  uint64_t vk_create_shader_module_count;
  uint64_t vk_destroy_shader_module_count;
  uint64_t vk_create_compute_pipelines_count;
  uint64_t vk_allocate_descriptor_sets_count;
  uint64_t vk_update_descriptor_sets_count;
  uint64_t vk_create_command_pool_count;
  uint64_t vk_allocate_command_buffers_count;
  uint64_t vk_reset_command_buffer_count;
  uint64_t vk_queue_submit_count;
  uint64_t vk_fence_wait_count;
  uint64_t vk_timeline_wait_count;
  uint64_t vk_map_memory_count;
  uint64_t vk_unmap_memory_count;
  uint64_t vk_flush_count;
  uint64_t vk_invalidate_count;
  uint64_t m6a_activation_pack_gpu_ns;
  uint64_t m6a_cooperative_execute_gpu_ns;
  uint64_t m6a_w3_segment_repack_gpu_ns;
} PrometheusModelBlockEvidence;

/* reactor_api.h:2713-2715 -- create the handle's one model block
   (validation: reactor_vulkan_model_block.c:393-477). */
PROM_REACTOR_API int prometheus_reactor_runtime_model_block_create(
    void* handle, const PrometheusModelBlockCreateRequest* request, uint64_t* out_block_id,
    PrometheusModelBlockEvidence* out_evidence);
/* reactor_api.h:2716-2718 -- the declared weights, once, in binding order (:1781-1829). */
PROM_REACTOR_API int prometheus_reactor_runtime_model_block_upload_weights(
    void* handle, uint64_t block_id, const PrometheusModelBlockWeightUpload* uploads, uint32_t upload_count,
    PrometheusModelBlockEvidence* out_evidence);
/* reactor_api.h:2719-2721 -- the family-0 resident identity block: output = input,
   audit = the first audit elements (:1884-1953; resident_identity.sdslv). */
PROM_REACTOR_API int prometheus_reactor_runtime_model_block_execute(
    void* handle, uint64_t block_id, const PrometheusModelBlockExecuteRequest* request,
    PrometheusModelBlockEvidence* out_evidence);
/* reactor_api.h:2731-2736 -- noise_refiner.0 / .1 from external BF16 ingress;
   the FP32 output stays resident (:2204-2303; runCanonicalNoiseRefiner0,
   canonical_reference.go:315-480).  audit_enabled must be 0. */
PROM_REACTOR_API int prometheus_reactor_runtime_noise_refiner0_execute(
    void* handle, uint64_t block_id, const PrometheusNoiseRefiner0ExecuteRequest* request,
    PrometheusModelBlockEvidence* out_evidence);
PROM_REACTOR_API int prometheus_reactor_runtime_noise_refiner1_execute(
    void* handle, uint64_t block_id, const PrometheusNoiseRefiner1ExecuteRequest* request,
    PrometheusModelBlockEvidence* out_evidence);
/* reactor_api.h:2737-2739 -- replace block 0's weights with block 1's (:1831-1882). */
PROM_REACTOR_API int prometheus_reactor_runtime_noise_refiner_rebind(
    void* handle, uint64_t block_id, const PrometheusNoiseRefinerRebindRequest* request,
    PrometheusModelBlockEvidence* out_evidence);
/* reactor_api.h:2740-2742 -- noise_refiner.1 on the resident predecessor output
   (:3274-3396).  Only audit_enabled = 0 is provided. */
PROM_REACTOR_API int prometheus_reactor_runtime_noise_refiner_execute_resident(
    void* handle, uint64_t block_id, const PrometheusNoiseRefinerResidentExecuteRequest* request,
    PrometheusModelBlockEvidence* out_evidence);
/* reactor_api.h:2746-2748 -- read back the resident final output (:3402-3459). */
PROM_REACTOR_API int prometheus_reactor_runtime_noise_refiner_audit_final(
    void* handle, uint64_t block_id, const PrometheusNoiseRefinerFinalAuditRequest* request,
    PrometheusModelBlockEvidence* out_evidence);
/* reactor_api.h:2749-2763 -- the context refiner family: create (+ upload), rebind
   to block 1, execute on FP32 ingress or on the resident output, read back
   (reactor_vulkan_model_block.c:2305-2367, 2464-2669). */
PROM_REACTOR_API int prometheus_reactor_runtime_context_refiner_create(
    void* handle, const PrometheusContextRefinerCreateRequest* request, uint64_t* out_block_id,
    PrometheusModelBlockEvidence* out_evidence);
PROM_REACTOR_API int prometheus_reactor_runtime_context_refiner_rebind(
    void* handle, uint64_t block_id, const PrometheusContextRefinerRebindRequest* request,
    PrometheusModelBlockEvidence* out_evidence);
PROM_REACTOR_API int prometheus_reactor_runtime_context_refiner0_execute(
    void* handle, uint64_t block_id, const PrometheusContextRefiner0ExecuteRequest* request,
    PrometheusModelBlockEvidence* out_evidence);
PROM_REACTOR_API int prometheus_reactor_runtime_context_refiner_execute_resident(
    void* handle, uint64_t block_id, const PrometheusContextRefinerResidentExecuteRequest* request,
    PrometheusModelBlockEvidence* out_evidence);
PROM_REACTOR_API int prometheus_reactor_runtime_context_refiner_audit_final(
    void* handle, uint64_t block_id, const PrometheusContextRefinerFinalAuditRequest* request,
    PrometheusModelBlockEvidence* out_evidence);
/* reactor_api.h:2776-2779 -- evidence and teardown (:3503-3522). */
PROM_REACTOR_API int prometheus_reactor_runtime_model_block_get_evidence(void* handle, uint64_t block_id,
                                                                         PrometheusModelBlockEvidence* out_evidence);
PROM_REACTOR_API int prometheus_reactor_runtime_model_block_destroy(void* handle, uint64_t block_id);

/* reactor_api.h:2823-2826 -- aliases kept by the reference for older drafts. */
PROM_REACTOR_API int prometheus_runtime_create(void* config, void** out_handle);
PROM_REACTOR_API int prometheus_runtime_destroy(void* handle);
PROM_REACTOR_API int prometheus_runtime_probe(void* handle, PrometheusCaps* out_caps);

/* ==== extensions: device-resident entry points (no reference counterpart) ==== */

/* SGEMM kernel variants. */
enum {
  OCT_B200_SGEMM_AUTO = 0u,       /* small-M kernel for m <= 16; FMA for tiny products; the CTA pair with 32-deep
                                     stages (232) for m, n >= 2048; else 3xTF32 tcgen05 (1) */
  OCT_B200_SGEMM_TC3XTF32 = 1u,   /* tcgen05/TMEM tensor cores, split-TF32 x3 */
  OCT_B200_SGEMM_FMA = 2u,        /* plain FP32 FMA on the CUDA cores (control) */
  OCT_B200_SGEMM_SMALLM = 3u,     /* m <= 16: HBM-bound CUDA-core kernel, split-K, ordered reduction */
  OCT_B200_SGEMM_SMALLM_TC = 4u,  /* m <= 16: tcgen05 3xTF32 with the TF32 split inside the kernel (C^T = B^T A^T,
                                     A and B read in place: 16-byte aligned, lda / ldb multiples of 4, else
                                     runs as OCT_B200_SGEMM_SMALLM), split-K, ordered reduction */
  OCT_B200_SGEMM_TC_BK16 = 16u,   /* tensor cores, one CTA per 128x256 tile, 16-deep K stages */
  OCT_B200_SGEMM_TC_BK32 = 32u,   /* tensor cores, one CTA per 128x256 tile, 32-deep K stages */
  OCT_B200_SGEMM_TC_PAIR16 = 216u, /* tensor cores, CTA pair (cta_group::2) per 256x256 tile, 16-deep */
  OCT_B200_SGEMM_TC_PAIR32 = 232u, /* CTA pair, 32-deep K stages */
  OCT_B200_SGEMM_TC_INSM16 = 316u, /* CTA pair, TF32 split inside the kernel from A and B in place (no split
                                      pass); needs 16-byte aligned A / B and lda, ldb multiples of 4, else
                                      runs as OCT_B200_SGEMM_TC_PAIR16 */
  OCT_B200_SGEMM_TC_INSM32 = 332u, /* the same with 32-deep K stages (else as OCT_B200_SGEMM_TC_PAIR32) */
};

/* C = A * B on device pointers (row-major, ld = k / n / n), enqueued on
   `stream` (a cudaStream_t; NULL = the CUDA default stream).  Returns right
   after the enqueue.  The TF32 split scratch lives in the handle and is shared
   by every call on it: calls on one handle from different streams must be
   ordered by the caller. */
PROM_REACTOR_API int oct_b200_sgemm_device(void* handle, const float* d_a, const float* d_b, float* d_c,
                                           uint32_t m, uint32_t n, uint32_t k, uint32_t variant,
                                           void* stream, int* out_detail_code);

/* Same as above with explicit leading dimensions (elements) for A, B and C, so
   a caller can address a column shard of a wider matrix.  lda >= k, ldb >= n,
   ldc >= n. */
PROM_REACTOR_API int oct_b200_sgemm_device_ld(void* handle, const float* d_a, uint64_t lda, const float* d_b,
                                              uint64_t ldb, float* d_c, uint64_t ldc, uint32_t m, uint32_t n,
                                              uint32_t k, uint32_t variant, void* stream, int* out_detail_code);

/* Strided batch of products C_i = A_i * op(B_i) for i < batch, X_i = X + i *
   stride_x (element strides; 0 shares an operand across the batch).  With
   b_trans != 0, B_i is [n][k] row-major (ldb >= k) and op(B_i) = B_i^T;
   otherwise B_i is [k][n] (ldb >= n).  The attention score (Q K^T) and
   aggregation (P V) products of the transformer block use this. */
PROM_REACTOR_API int oct_b200_sgemm_batched_device(void* handle, const float* d_a, uint64_t lda, uint64_t stride_a,
                                                   const float* d_b, uint64_t ldb, uint64_t stride_b, uint32_t b_trans,
                                                   float* d_c, uint64_t ldc, uint64_t stride_c, uint32_t batch,
                                                   uint32_t m, uint32_t n, uint32_t k, uint32_t variant, void* stream,
                                                   int* out_detail_code);

/* Row reductions on device pointers.  operation: PROM_REDUCTION_OPERATION_*.
   SUM/MAX write `rows` floats, SOFTMAX writes rows*width floats. */
PROM_REACTOR_API int oct_b200_reduction_device(void* handle, const float* d_in, float* d_out, uint32_t rows,
                                               uint32_t width, uint32_t operation, void* stream,
                                               int* out_detail_code);

/* RMSNorm on device pointers: out[r, :] = in[r, :] * inv_rms[r] * weight[:],
   inv_rms[r] = 1 / sqrt(mean(in[r, :]^2) + eps).  d_inv_rms may be NULL. */
PROM_REACTOR_API int oct_b200_rmsnorm_device(void* handle, const float* d_in, const float* d_weight, float* d_out,
                                             float* d_inv_rms, uint32_t rows, uint32_t width, float epsilon,
                                             void* stream, int* out_detail_code);

/* No counterpart in the reference's C ABI: the exact attention of the Z-Image
   block (`canonicalAttention`, internal/prometheus/zimage/canonical_reference.go:241-289)
   on device pointers, as one fused tcgen05 3xTF32 kernel.
   q, k, v, out: [items * seq][heads * head_dim] row-major fp32, token-major
   with head h in columns h*head_dim .. (the reference's
   [(token*heads + head)*head_dim + c] layout); out = softmax(q k^T * scale) v
   per item and head, bidirectional.  head_dim must be 128 and seq a multiple
   of 128 (else PROM_ERROR with OCT_B200_DETAIL_UNSUPPORTED_SHAPE).  The TF32
   split copies of q, k and v^T go to the handle's scratch. */
PROM_REACTOR_API int oct_b200_attention_device(void* handle, const float* d_q, const float* d_k, const float* d_v,
                                               float* d_out, uint32_t items, uint32_t seq, uint32_t heads,
                                               uint32_t head_dim, float scale, void* stream, int* out_detail_code);

/* Test-only, no reference counterpart: runs the tensor-parallel peer-wait
   kernel against a flag that nothing sets, with a wall-clock budget of
   budget_ns (1 ms .. 1 s).  The wait must give up, record its error bit and
   return: PROM_ERROR with OCT_B200_DETAIL_DEVICE_TIMEOUT, the handle still
   usable.  Failure detection is exercised without faulting or hanging a GPU. */
PROM_REACTOR_API int oct_b200_selftest_wait_timeout(void* handle, uint64_t budget_ns, int* out_detail_code);

/* Waits for `stream` (NULL: the CUDA default stream), then reads and
   clears the device status words the kernels write: returns PROM_ERROR with
   OCT_B200_DETAIL_DEVICE_TIMEOUT if a bounded in-kernel wait gave up, or
   PROM_REDUCTION_DETAIL_NONFINITE_INPUT if a reduction saw NaN/Inf. */
PROM_REACTOR_API int oct_b200_sync_status(void* handle, void* stream, int* out_detail_code);

/* No counterpart in the reference.  C = A * B on device pointers (row-major,
   leading dimensions lda >= k, ldb >= n, ldc >= n) with the tcgen05 3xTF32
   kernel, for callers that cannot allocate device memory: it needs no handle
   and calls no cudaMalloc, cudaFree or allocating library routine.  The TF32
   split scratch and the kernel status word live in one fixed 64 MiB device
   array that every GPU loading the library holds until the process exits.
   Limit: 8 * (roundup(m,256) + roundup(n,256)) * roundup(k,32) bytes must fit
   in 64 MiB (any m, n, k <= 2048 does); larger products are rejected with
   PROM_ERROR and OCT_B200_DETAIL_NOALLOC_TOO_LARGE, and C is left untouched.
   The first call on each device looks up the array's device address, so make
   that first call before any stream capture.  The address is looked up in,
   and cached for, the device's primary context (the one the CUDA runtime
   uses); a process that resets the device (cudaDeviceReset) or drives the
   GPU through another context must not call this entry point afterwards.
   Null pointers or short leading dimensions fail with
   OCT_B200_DETAIL_INVALID_ARGUMENT.  The call waits on `stream` (NULL
   = the CUDA default stream) until the product is done and reports an
   in-kernel timeout as OCT_B200_DETAIL_DEVICE_TIMEOUT.  Every call shares the
   one array, so calls whose work overlaps on the GPU (from several host
   threads or streams) race and must be serialised by the caller. */
PROM_REACTOR_API int oct_b200_sgemm_device_noalloc(const float* d_a, uint64_t lda, const float* d_b, uint64_t ldb,
                                                   float* d_c, uint64_t ldc, uint32_t m, uint32_t n, uint32_t k,
                                                   void* stream, int* out_detail_code);

/* Per-launch timing of the tensor-core SGEMM: when enabled, CUDA events are
   recorded on the launch stream around the TF32 split pass and the main
   kernel of every launch; read returns the summed milliseconds of the
   launches since the last read (waiting for them) and resets the count. */
PROM_REACTOR_API int oct_b200_set_kernel_timing(void* handle, int enable);
PROM_REACTOR_API int oct_b200_read_kernel_timing(void* handle, double* split_ms_total, double* main_ms_total,
                                                 uint32_t* launches);

/* ---- transformer block (extension; the reference's closest counterpart is the
   model-block lifecycle create -> upload_weights -> execute -> destroy,
   reactor_api.h:2713-2784, which is specific to Z-Image checkpoints) ---- */
enum { OCT_B200_BLOCK_GEMMA = 1u, OCT_B200_BLOCK_DIT = 2u };

/* Weight slots.  Matrices are [in][out] row-major fp32 (canonicalLinear's
   layout, canonical_reference.go:156-175); gains and biases are vectors.
   Gemma: WQKV = [hidden][(heads + 2*kv_heads) * head_dim] (q heads | k | v);
          WGU = [hidden][2*ffn] (gate | up); WO = [heads*head_dim][hidden];
          WD = [ffn][hidden].
   DiT:   ADA_W = [256][6*hidden] (scale_a | gate_a | scale_m | gate_m | shift_a | shift_m),
          ADA_B = [6*hidden]; WQKV = [hidden][3*heads*128]; W13 = [hidden][2*ffn]
          (w1 | w3); W2 = [ffn][hidden]; Q_NORM, K_NORM = [128]. */
enum {
  OCT_B200_GEMMA_NORM1 = 0, OCT_B200_GEMMA_WQKV = 1, OCT_B200_GEMMA_WO = 2, OCT_B200_GEMMA_NORM2 = 3,
  OCT_B200_GEMMA_WGU = 4, OCT_B200_GEMMA_WD = 5,
};
enum {
  OCT_B200_DIT_ADA_W = 0, OCT_B200_DIT_ADA_B = 1, OCT_B200_DIT_ATTN_NORM1 = 2, OCT_B200_DIT_WQKV = 3,
  OCT_B200_DIT_Q_NORM = 4, OCT_B200_DIT_K_NORM = 5, OCT_B200_DIT_WO = 6, OCT_B200_DIT_ATTN_NORM2 = 7,
  OCT_B200_DIT_FFN_NORM1 = 8, OCT_B200_DIT_W13 = 9, OCT_B200_DIT_W2 = 10, OCT_B200_DIT_FFN_NORM2 = 11,
};

/* heads and ffn are THIS rank's share under tensor parallelism (tp_world > 1):
   the caller passes column shards of WQKV / WGU (W13) and row shards of WO /
   WD (W2); the two row-parallel products are all-reduced over NCCL inside
   the forward.  Gemma requires kv_heads == 1 (MQA; the KV head is replicated
   on every rank).  DiT requires head_dim == 128 and rope axes (32, 48, 48). */
typedef struct OctB200BlockConfig {
  uint32_t struct_size;
  uint32_t family;
  uint32_t hidden;
  uint32_t heads;
  uint32_t kv_heads;
  uint32_t head_dim;
  uint32_t ffn;
  uint32_t seq_len;    /* tokens per sequence (Gemma) or per image (DiT) */
  uint32_t max_batch;  /* sequences / images per forward the workspaces are sized for */
  float eps;           /* block RMSNorm epsilon (Gemma 1e-6, DiT 1e-5) */
  float rope_base;     /* Gemma base (10000), DiT theta (256) */
  uint32_t grid_w;     /* DiT: image tokens per grid row */
  uint32_t rope_frame; /* DiT: frame coordinate of the image tokens */
  uint32_t tp_rank;
  uint32_t tp_world;
  uint8_t nccl_id[128]; /* tp_world > 1: the same oct_b200_nccl_unique_id bytes on every rank */
} OctB200BlockConfig;

/* ncclGetUniqueId (NCCL is dlopen'ed; nothing links it).  Rank 0 calls this
   and shares the 128 bytes with the other ranks.  One id seeds exactly one
   communicator: create a fresh id for every tensor-parallel block. */
PROM_REACTOR_API int oct_b200_nccl_unique_id(uint8_t* out_128_bytes);
PROM_REACTOR_API int oct_b200_block_create(void* handle, const OctB200BlockConfig* config, uint64_t* out_block_id,
                                           int* out_detail_code);
PROM_REACTOR_API int oct_b200_block_set_weight(void* handle, uint64_t block_id, uint32_t slot, const float* data,
                                               uint64_t element_count, uint32_t data_on_device);
/* y = block(x), x and y device buffers [batch * seq_len][hidden]; timesteps
   (DiT only) is a HOST array of `batch` floats.  Enqueued on `stream` (NULL =
   CUDA default stream). */
PROM_REACTOR_API int oct_b200_block_forward_device(void* handle, uint64_t block_id, const float* d_x, float* d_y,
                                                   uint32_t batch, const float* timesteps, void* stream,
                                                   int* out_detail_code);
/* Same with host buffers: copies x in and y out, returns when y is written. */
PROM_REACTOR_API int oct_b200_block_forward(void* handle, uint64_t block_id, const float* x, float* y, uint32_t batch,
                                            const float* timesteps, int* out_detail_code);
PROM_REACTOR_API int oct_b200_block_destroy(void* handle, uint64_t block_id);

/* ---- column-parallel SGEMM over tensor-parallel ranks (extension: the
   reference drives one device per handle, prometheus_reactor_runtime_sgemm,
   reactor_api.h:2587-2595; this is its multi-GPU form, one process per GPU).
   C = A * B for A [m][k] (the same on every rank) and B [k][n] column-sharded:
   rank r passes B[:, r*n/world .. (r+1)*n/world) as d_b_shard ([k][n/world],
   leading dimension ldb).  Every rank receives all of C [m][n], row-major.
   Every rank makes the same calls in the same order with the same m, n, k;
   n must be a multiple of 4 * world, m <= max_m, n <= max_n.
   Collective AUTO takes the peer-store path when every rank runs on its own
   GPU: the GEMM epilogue stores each finished tile into every rank's output
   buffer over NVLink (no TMA or bulk copy reads or writes peer memory), then a
   bounded flag wait publishes completion.  NCCL: the GEMM writes this rank's
   slab, ncclAllGather fills the rest, a repack kernel makes row-major C. ---- */
enum {
  OCT_B200_TP_COLLECTIVE_AUTO = 0u, /* peer stores when possible, else NCCL */
  OCT_B200_TP_COLLECTIVE_PEER = 1u, /* peer stores; creation fails when not possible */
  OCT_B200_TP_COLLECTIVE_NCCL = 2u, /* NCCL all-gather + repack */
};
typedef struct OctB200TpSgemmConfig {
  uint32_t struct_size;
  uint32_t rank;
  uint32_t world;
  uint32_t max_m;      /* largest m of any call */
  uint32_t max_n;      /* largest full n of any call (multiple of 4 * world) */
  uint32_t collective; /* OCT_B200_TP_COLLECTIVE_* */
  uint8_t nccl_id[128]; /* world > 1: the same oct_b200_nccl_unique_id bytes on every rank */
} OctB200TpSgemmConfig;
/* Collective: every rank calls it with the same world, max_m, max_n, id. */
PROM_REACTOR_API int oct_b200_tp_sgemm_create(void* handle, const OctB200TpSgemmConfig* config, uint64_t* out_id,
                                              int* out_detail_code);
/* Enqueue one product on `stream` (NULL = CUDA default stream).  d_c
   (optional, leading dimension ldc >= n) receives C; *out_result (optional)
   receives the library's own copy of C (leading dimension n), valid until this
   rank's next call on the same id (reads must finish, or be ordered on
   `stream`, before that call).  At least one of d_c, out_result is given. */
PROM_REACTOR_API int oct_b200_sgemm_tp_device(void* handle, uint64_t id, const float* d_a, uint64_t lda,
                                              const float* d_b_shard, uint64_t ldb, float* d_c, uint64_t ldc,
                                              uint32_t m, uint32_t n, uint32_t k, void* stream, float** out_result,
                                              int* out_detail_code);
/* Waits for `stream`; PROM_ERROR with OCT_B200_DETAIL_DEVICE_TIMEOUT when a
   bounded wait of an earlier call gave up (a peer never signalled). */
PROM_REACTOR_API int oct_b200_tp_sgemm_sync(void* handle, uint64_t id, void* stream, int* out_detail_code);
/* The collective the object took: OCT_B200_TP_COLLECTIVE_PEER or _NCCL (AUTO for world 1). */
PROM_REACTOR_API int oct_b200_tp_sgemm_collective(void* handle, uint64_t id, uint32_t* out_collective);
/* Collective: every rank destroys its object (a bounded barrier keeps peers'
   buffers mapped until no rank can still write them). */
PROM_REACTOR_API int oct_b200_tp_sgemm_destroy(void* handle, uint64_t id);

/* Library build identity, for diagnostics. */
PROM_REACTOR_API const char* oct_b200_build_info(void);

#ifdef __cplusplus
}
#endif

#endif /* OCT_B200_PROMETHEUS_REACTOR_H */
