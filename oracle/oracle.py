"""ctypes + numpy front end of the CPU oracle (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use this
module, always as the checker or the timed CPU baseline, never as the product.
The C functions restate Oct's CPU code (see oracle.c for the file:line of each);
this file adds the input generators of Oct's own tests and an fp64 GEMM.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB = ORACLE_DIR / "_build" / "liboct_oracle.so"

_lib = None


def build() -> Path:
    """Compile oracle.c (make) if its shared object is missing or stale."""
    if not LIB.exists() or LIB.stat().st_mtime < (ORACLE_DIR / "oracle.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
    return LIB


class Correctness(C.Structure):
    _fields_ = [("pass_", C.c_int32), ("failing_count", C.c_int32), ("first_failing_index", C.c_int64),
                ("max_abs_error", C.c_double), ("max_rel_error", C.c_double),
                ("first_expected", C.c_float), ("first_actual", C.c_float)]


class Mismatch(C.Structure):
    _fields_ = [("row", C.c_int64), ("column", C.c_int64), ("expected", C.c_float), ("actual", C.c_float),
                ("abs_error", C.c_float), ("rel_error", C.c_float)]


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(str(LIB))
        i64, vp, i32 = C.c_int64, C.c_void_p, C.c_int
        L.oracle_cpu_sgemm_f32_rows.argtypes = [i64, i64, i64, vp, vp, vp, i64, i64]
        L.oracle_cpu_sgemm_f32.argtypes = [i64, i64, i64, vp, vp, vp]
        L.oracle_cpu_sgemm_f32_mt.argtypes = [i64, i64, i64, vp, vp, vp, i64, i64, i32]
        L.oracle_oct_matmul_f64_rows.argtypes = [i64, i64, i64, vp, vp, vp, i64, i64]
        L.oracle_sgemm_f64_rows.argtypes = [i64, i64, i64, vp, vp, vp, i64, i64, i32]
        L.oracle_compare_against_oracle.argtypes = [vp, vp, i64, C.c_double, C.c_double, C.POINTER(Correctness)]
        L.oracle_find_nonfinite.argtypes = [vp, i64]
        L.oracle_find_nonfinite.restype = i64
        L.oracle_reduction_cpu_reference.argtypes = [i64, i64, i32, vp, vp, i32]
        L.oracle_reduction_cpu_reference.restype = i32
        L.oracle_reduction_compare.argtypes = [i64, i64, i32, vp, vp, C.POINTER(Mismatch)]
        L.oracle_reduction_compare.restype = i32
        L.oracle_rmsnorm_f32.argtypes = [i64, i64, i64, vp, vp, C.c_float, vp, vp, i32, i32]
        L.oracle_rmsnorm_f64.argtypes = [i64, i64, i64, vp, vp, C.c_double, vp, vp, i32]
        L.oracle_bf16_round.argtypes = [i64, vp, vp]
        L.oracle_m1_rmsnorm.argtypes = [i64, i64, i64, vp, vp, C.c_float, i32, i32, vp, vp]
        L.oracle_m1_rope.argtypes = [i64, i64, i64, vp, vp, vp, vp]
        L.oracle_m1_scores.argtypes = [i64, i64, i64, vp, vp, C.c_double, i32, vp]
        L.oracle_fft64.argtypes = [i64, vp, vp, vp]
        L.oracle_fft32.argtypes = [i64, i64, i64, i32, i32, vp, vp]
        L.oracle_max_threads.restype = i32
        _lib = L
    return _lib


def _p(x: np.ndarray) -> int:
    assert x.flags.c_contiguous
    return x.ctypes.data


def max_threads() -> int:
    return int(lib().oracle_max_threads())


# ------------------------------------------------------------------ SGEMM
def cpu_sgemm_f32(a: np.ndarray, b: np.ndarray, m: int, n: int, k: int, rows: slice | None = None,
                  threads: int = 1) -> np.ndarray:
    """Oct's cpuSGEMM (runtime.go:319-331) over rows[start:stop]."""
    r0, r1 = (0, m) if rows is None else (rows.start or 0, rows.stop if rows.stop is not None else m)
    out = np.empty((r1 - r0) * n, dtype=np.float32)
    if threads == 1:
        lib().oracle_cpu_sgemm_f32_rows(m, n, k, _p(a), _p(b), _p(out), r0, r1 - r0)
    else:
        lib().oracle_cpu_sgemm_f32_mt(m, n, k, _p(a), _p(b), _p(out), r0, r1 - r0, threads)
    return out


def oct_matmul_f64(a64: np.ndarray, b64: np.ndarray, m: int, n: int, k: int, rows: slice | None = None) -> np.ndarray:
    """Oct's compiled `@` __octMatMulMM[float64] (emit_go_runtime.go:168-200)."""
    r0, r1 = (0, m) if rows is None else (rows.start or 0, rows.stop if rows.stop is not None else m)
    out = np.empty((r1 - r0) * n, dtype=np.float64)
    lib().oracle_oct_matmul_f64_rows(m, n, k, _p(a64), _p(b64), _p(out), r0, r1 - r0)
    return out


def sgemm_f64(a: np.ndarray, b: np.ndarray, m: int, n: int, k: int, rows: slice | None = None,
              threads: int | None = None) -> np.ndarray:
    """Binary64-accumulated product of fp32 inputs (Marionette CheckProduct)."""
    r0, r1 = (0, m) if rows is None else (rows.start or 0, rows.stop if rows.stop is not None else m)
    out = np.empty((r1 - r0) * n, dtype=np.float64)
    lib().oracle_sgemm_f64_rows(m, n, k, _p(a), _p(b), _p(out), r0, r1 - r0, threads or max_threads())
    return out


def compare_against_oracle(expected: np.ndarray, actual: np.ndarray, abs_tol: float = 1e-4,
                           rel_tol: float = 1e-4) -> Correctness:
    """compareAgainstOracle (runtime.go:339-383); defaults are runtime.go:12-15."""
    e = np.ascontiguousarray(expected, dtype=np.float32).ravel()
    a = np.ascontiguousarray(actual, dtype=np.float32).ravel()
    res = Correctness()
    lib().oracle_compare_against_oracle(_p(e), _p(a), e.size, abs_tol, rel_tol, C.byref(res))
    return res


# ------------------------------------------------------------------ reductions
def reduction_cpu_reference(x: np.ndarray, op: int, threads: int = 1) -> tuple[int, np.ndarray]:
    rows, width = x.shape
    out = np.empty(x.size if op == 3 else rows, dtype=np.float32)
    rc = lib().oracle_reduction_cpu_reference(rows, width, op, _p(x), _p(out), threads)
    return rc, out


def reduction_compare(rows: int, width: int, op: int, expected: np.ndarray, actual: np.ndarray
                      ) -> tuple[int, Mismatch]:
    mm = Mismatch()
    e = np.ascontiguousarray(expected, dtype=np.float32)
    a = np.ascontiguousarray(actual, dtype=np.float32)
    rc = lib().oracle_reduction_compare(rows, width, op, _p(e), _p(a), C.byref(mm))
    return rc, mm


def find_nonfinite(x: np.ndarray) -> int:
    return int(lib().oracle_find_nonfinite(_p(np.ascontiguousarray(x, dtype=np.float32)), x.size))


def rmsnorm_f32(x: np.ndarray, w: np.ndarray, eps: float, threads: int = 1, form: str = "head"
                ) -> tuple[np.ndarray, np.ndarray]:
    """fp32 RMSNorm as Oct's CPU code evaluates it: form "head" is cpuHeadRMSNorm
    (gemma4e2b_m1_rtx.go:811-832, Gemma), "canonical" is CanonicalRMSNorm
    (zimage/canonical_contract.go:91-105, the Z-Image / DiT path)."""
    rows, width = x.shape
    out = np.empty_like(x)
    inv = np.empty(rows, dtype=np.float32)
    lib().oracle_rmsnorm_f32(rows, width, width, _p(x), _p(w), eps, _p(out), _p(inv), threads,
                             {"head": 0, "canonical": 1}[form])
    return out, inv


def rmsnorm_f64(x: np.ndarray, w: np.ndarray, eps: float, threads: int | None = None
                ) -> tuple[np.ndarray, np.ndarray]:
    rows, width = x.shape
    out = np.empty(x.shape, dtype=np.float64)
    inv = np.empty(rows, dtype=np.float64)
    lib().oracle_rmsnorm_f64(rows, width, width, _p(x), _p(w), float(np.float32(eps)), _p(out), _p(inv),
                             threads or max_threads())
    return out, inv


# ------------------------------------------------------------------ inputs of Oct's own tests
def deterministic_matrix(rows: int, cols: int) -> np.ndarray:
    """deterministicMatrix (runtime.go:242-249): ((i % 23) - 11) / 7 as float32."""
    i = np.arange(rows * cols, dtype=np.int64)
    return (((i % 23) - 11).astype(np.float32) / np.float32(7.0)).astype(np.float32)


def marionette_matrix(count: int, seed: int) -> np.ndarray:
    """Matrix(count, seed) of reactor_concept_sgemm_tests.cpp:14-19: ((i*7+seed)%23 - 11) / 8."""
    i = np.arange(count, dtype=np.int64)
    return ((((i * 7 + seed) % 23) - 11).astype(np.float32) / np.float32(8.0)).astype(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32ToBF16 -> bf16ToFloat32 (gemma4e2b_m1_rtx.go:1005-1014): round to nearest even."""
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) >> 16) & 0xFFFF
    return (rounded.astype(np.uint32) << 16).view(np.float32)


def gemma_corpus_a(count: int) -> np.ndarray:
    """deterministicCorpusFP32 (gemma4e2b_sgemm_corpus_test.go:107-113)."""
    i = np.arange(count, dtype=np.int64)
    return (((i * 17) % 101 - 50).astype(np.float32) / np.float32(31.0)).astype(np.float32)


def gemma_corpus_b(count: int) -> np.ndarray:
    """deterministicCorpusBF16 (gemma4e2b_sgemm_corpus_test.go:115-122)."""
    i = np.arange(count, dtype=np.int64)
    return bf16_round((((i * 29) % 127 - 63).astype(np.float32) / np.float32(37.0)).astype(np.float32))


def reduction_input(rows: int, width: int, distribution: str = "deterministic", bias: float = 0.0) -> np.ndarray:
    """deterministic_input / fr_m0_input of reactor_reduction_tests.cpp:77-114."""
    r = np.arange(rows, dtype=np.int64)[:, None]
    c = np.arange(width, dtype=np.int64)[None, :]
    centered = ((r * 29 + c * 17) % 101) - 50
    x = (np.float32(bias) + centered.astype(np.float32) / np.float32(16.0)).astype(np.float32)
    if distribution == "constant":
        x[:] = np.float32(3.25)
    elif distribution == "positive-extreme":
        x = np.broadcast_to(np.float32(10000.0) + ((c % 17) - 8).astype(np.float32), (rows, width)).copy()
    elif distribution == "negative-extreme":
        x = np.broadcast_to(np.float32(-10000.0) + ((c % 17) - 8).astype(np.float32), (rows, width)).copy()
    elif distribution == "heterogeneous":
        mode = (r % 4) * np.ones_like(c)
        v0 = np.full((rows, width), 2.0, dtype=np.float32)
        v1 = np.broadcast_to(((c % 101) - 50).astype(np.float32) / np.float32(8.0), (rows, width))
        v2 = np.broadcast_to(np.float32(10000.0) + ((c % 17) - 8).astype(np.float32), (rows, width))
        v3 = np.broadcast_to(np.float32(-10000.0) + ((c % 17) - 8).astype(np.float32), (rows, width))
        x = np.where(mode == 0, v0, np.where(mode == 1, v1, np.where(mode == 2, v2, v3))).astype(np.float32)
    return np.ascontiguousarray(x, dtype=np.float32)


def uniform_matrix(rows: int, cols: int, seed: int) -> np.ndarray:
    """Seeded U[-1, 1) fp32 matrix (PCG64): the SGEMM benchmark input distribution."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return (rng.random((rows, cols), dtype=np.float32) * np.float32(2.0) - np.float32(1.0)).astype(np.float32)


def normal_matrix(rows: int, cols: int, seed: int) -> np.ndarray:
    """Seeded N(0, 1) fp32 matrix (PCG64): the reduction benchmark input distribution."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.standard_normal((rows, cols), dtype=np.float32)


# ------------------------------------------------------------------ Gemma M1 BF16 boundary
def _f32c(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32ToBF16 then bf16ToFloat32 (gemma4e2b_m1_rtx.go:1005-1014)."""
    x = _f32c(x)
    out = np.empty_like(x)
    lib().oracle_bf16_round(x.size, _p(x), _p(out))
    return out


def m1_rmsnorm(x: np.ndarray, w: np.ndarray, eps: float, round_in: bool, round_out: bool,
               stride: int | None = None, rows: int | None = None, width: int | None = None
               ) -> tuple[np.ndarray, np.ndarray]:
    """The M46 RMSNorm family's arithmetic (reference oracle, reactor_concept_rmsnorm_tests.cpp:17-35)."""
    x, w = _f32c(x), _f32c(w)
    width = width or w.size
    stride = stride or width
    rows = rows if rows is not None else x.size // stride
    out = np.empty(rows * width, dtype=np.float32)
    inv = np.empty(rows, dtype=np.float32)
    lib().oracle_m1_rmsnorm(rows, width, stride, _p(x), _p(w), eps, int(round_in), int(round_out), _p(out), _p(inv))
    return out, inv


def m1_rope(src: np.ndarray, cos: np.ndarray, sin: np.ndarray, tokens: int, heads: int, hw: int) -> np.ndarray:
    """cpuGemma4e2bRope (gemma4e2b_m1_rtx.go:834-861)."""
    src, cos, sin = _f32c(src), _f32c(cos), _f32c(sin)
    out = np.empty(tokens * heads * hw, dtype=np.float32)
    lib().oracle_m1_rope(tokens, heads, hw, _p(src), _p(cos), _p(sin), _p(out))
    return out


def m1_head_rmsnorm_rope(x, w, cos, sin, tokens: int, heads: int, hw: int, eps: float = 1e-6) -> np.ndarray:
    """BF16 head RMSNorm then RoPE (reactor_api.c:404-505; the test oracle `positional`,
    reactor_concept_rmsnorm_tests.cpp:59-70)."""
    normed, _ = m1_rmsnorm(x, w, eps, True, True, stride=hw, rows=tokens * heads, width=hw)
    return m1_rope(normed, cos, sin, tokens, heads, hw)


def m1_scores(q: np.ndarray, k: np.ndarray, tokens: int, qheads: int, hw: int, scale: float,
              form: str = "f64") -> np.ndarray:
    """Raw scores [qheads][tokens][tokens]; form "f64" is the reference test's binary64 chain,
    "go" is cpuGemma4e2bRawScores' fp32 loop (gemma4e2b_m1_rtx.go:863-883)."""
    q, k = _f32c(q), _f32c(k)
    out = np.empty(qheads * tokens * tokens, dtype=np.float32)
    lib().oracle_m1_scores(tokens, qheads, hw, _p(q), _p(k), float(scale), {"f64": 0, "go": 1}[form], _p(out))
    return out


# ------------------------------------------------------------------ FFT
def fft64(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """The reference's binary64 radix-2 network on complex128 input (oracle.c
    oracle_fft64); returns (spectrum, the n-double twiddle table)."""
    x = np.ascontiguousarray(x, dtype=np.complex128)
    n = x.size
    out = np.empty(n, dtype=np.complex128)
    tw = np.empty(max(n, 2), dtype=np.float64)
    lib().oracle_fft64(n, _p(x), _p(out), _p(tw))
    return out, tw


def fft32(x: np.ndarray, n: int, batch: int = 1, stride: int | None = None, inverse: bool = False,
          normalize: bool = False) -> np.ndarray:
    """The fp32 radix-2 network (oracle.c oracle_fft32) on complex64 input laid out
    `stride` elements per batch item."""
    stride = stride or n
    x = np.ascontiguousarray(x, dtype=np.complex64)
    out = np.zeros_like(x)
    lib().oracle_fft32(n, batch, stride, int(inverse), int(normalize), _p(x), _p(out))
    return out
