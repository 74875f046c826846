"""numpy interface to the CPU oracle (oracle/orc.c).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and the CPU legs
of bench.py as the checker / CPU baseline; never by the product path.

Arrays of fp16 values are passed as numpy float16 (same bits as the C side's uint16).
Every function cites the reference code it restates in orc.c.
"""
import ctypes
import os

import numpy as np

from . import build as _build

_lib = None

_i64 = ctypes.c_int64
_p = ctypes.c_void_p


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        L = ctypes.CDLL(path)
        L.orc_h2f.restype = ctypes.c_float
        L.orc_h2f.argtypes = [ctypes.c_uint16]
        L.orc_f2h.restype = ctypes.c_uint16
        L.orc_f2h.argtypes = [ctypes.c_float]
        L.orc_f2h_array.argtypes = [_p, _p, _i64]
        L.orc_h2f_array.argtypes = [_p, _p, _i64]
        L.orc_uniform_f16_at.restype = ctypes.c_uint16
        L.orc_uniform_f16_at.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        L.orc_fill_uniform_f16.argtypes = [_p, _i64, ctypes.c_uint64, ctypes.c_uint64]
        L.orc_gemm_f32_seq.argtypes = [_p, _p, _p] + [_i64] * 8
        L.orc_gemm_f64.restype = ctypes.c_int
        L.orc_gemm_f64.argtypes = [_p, _p, _p] + [_i64] * 8 + [ctypes.c_int]
        L.orc_contract5d_f64.restype = ctypes.c_int
        L.orc_contract5d_f64.argtypes = [_p, _p, _p, _p, _p, _p, _p, _p, ctypes.c_int]
        L.orc_widen_b.argtypes = [_p, _p, _i64, _i64, _i64]
        L.orc_widen_b_mt.argtypes = [_p, _p, _i64, _i64, _i64, ctypes.c_int]
        L.orc_gemm_f32_blocked.restype = ctypes.c_int
        L.orc_gemm_f32_blocked.argtypes = [_p, _p, _p, _p] + [_i64] * 8 + [ctypes.c_int]
        L.orc_simd_level.restype = ctypes.c_int
        L.orc_typed_to_f32.argtypes = [_p, ctypes.c_int, _p, _i64]
        L.orc_f32_to_typed.argtypes = [_p, ctypes.c_int, _p, _i64]
        L.orc_fill_uniform.argtypes = [_p, _i64, ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64]
        L.orc_gemm_f64_f32in.restype = ctypes.c_int
        L.orc_gemm_f64_f32in.argtypes = [_p, _p, _p] + [_i64] * 8 + [ctypes.c_int]
        L.orc_check_tolerance.restype = _i64
        L.orc_check_tolerance.argtypes = [_p, _i64, _p, _i64, _i64, _i64, _i64, ctypes.c_double,
                                          ctypes.c_double, _p, _p, _p]
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def nthreads():
    return max(1, len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count() or 1)


def f2h(x):
    """fp32 -> fp16, round to nearest even (bit-level restatement)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f2h_array(_ptr(x), _ptr(out), x.size)
    return out.view(np.float16)


def h2f(h):
    h = np.ascontiguousarray(h, dtype=np.float16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().orc_h2f_array(_ptr(h), _ptr(out), h.size)
    return out


def uniform_f16(shape, seed, offset=0):
    """Seeded U[-1,1] fp16 (the generator b2g_fill_uniform_f16 reproduces on the GPU).
    Replaces randomMatrix, mmm.cpp:1409-1414."""
    n = int(np.prod(shape)) if len(shape) else 1
    out = np.empty(n, dtype=np.uint16)
    lib().orc_fill_uniform_f16(_ptr(out), n, seed, offset)
    return out.view(np.float16).reshape(shape)


def gemm_f32_seq(A, B, rows=None):
    """GEMM_Naive, mmm.cpp:52-62: fp32 accumulate, k ascending.  Rows [r0, r1) of C."""
    A = np.ascontiguousarray(A, dtype=np.float16)
    B = np.ascontiguousarray(B, dtype=np.float16)
    M, K = A.shape
    K2, N = B.shape
    assert K == K2
    r0, r1 = rows if rows is not None else (0, M)
    C = np.empty((r1 - r0, N), dtype=np.float32)
    # orc_gemm_f32_seq writes C[r*ldc + c] for absolute r; offset the base pointer
    base = C.ctypes.data - r0 * N * 4
    lib().orc_gemm_f32_seq(_ptr(A), _ptr(B), ctypes.c_void_p(base), M, N, K, K, N, N, r0, r1)
    return C


def gemm_f64(A, B, rows=None, threads=None):
    """FP64-accumulated reference GEMM, rows [r0, r1)."""
    A = np.ascontiguousarray(A, dtype=np.float16)
    B = np.ascontiguousarray(B, dtype=np.float16)
    M, K = A.shape
    K2, N = B.shape
    assert K == K2
    r0, r1 = rows if rows is not None else (0, M)
    C = np.empty((r1 - r0, N), dtype=np.float64)
    rc = lib().orc_gemm_f64(_ptr(A), _ptr(B), _ptr(C), M, N, K, K, N, N, r0, r1,
                            threads or nthreads())
    assert rc == 0
    return C


def widen_b(B, threads=None):
    """B (fp16) widened to fp32 once, shared by every row panel of the CPU baseline."""
    B = np.ascontiguousarray(B, dtype=np.float16)
    K, N = B.shape
    Bf = np.empty((K, N), dtype=np.float32)
    lib().orc_widen_b_mt(_ptr(B), _ptr(Bf), K, N, N, threads or nthreads())
    return Bf


def gemm_f32_blocked(A, B, rows=None, threads=None, Bf=None):
    """Blocked multithreaded GEMM with GEMM_Naive's arithmetic (the CPU baseline)."""
    A = np.ascontiguousarray(A, dtype=np.float16)
    B = np.ascontiguousarray(B, dtype=np.float16)
    M, K = A.shape
    K2, N = B.shape
    assert K == K2
    r0, r1 = rows if rows is not None else (0, M)
    C = np.empty((r1 - r0, N), dtype=np.float32)
    bf = _ptr(Bf) if Bf is not None else None
    rc = lib().orc_gemm_f32_blocked(_ptr(A), _ptr(B), bf, _ptr(C), M, N, K, K, N, N, r0, r1,
                                    threads or nthreads())
    assert rc == 0
    return C


def contract5d_f64(A, a_shape, a_stride, B, b_shape, b_stride, c_shape, c_stride, c_size=None,
                   threads=None):
    """C[a,b,i,n] = sum_{j,k} A[a,b,i,j,k] B[j,k,n] over element strides (FP64 accumulate).
    A, B: flat fp16 buffers; returns a flat fp64 buffer of c_size elements laid out by
    c_stride (mmmTensor.cpp:329-340 pack + 246-252 remap, in index form)."""
    A = np.ascontiguousarray(A, dtype=np.float16).ravel()
    B = np.ascontiguousarray(B, dtype=np.float16).ravel()
    a_shape = np.asarray(a_shape, dtype=np.int64)
    a_stride = np.asarray(a_stride, dtype=np.int64)
    b_shape = np.asarray(b_shape, dtype=np.int64)
    b_stride = np.asarray(b_stride, dtype=np.int64)
    c_stride = np.asarray(c_stride, dtype=np.int64)
    if c_size is None:
        c_size = int(sum((int(s) - 1) * int(st) for s, st in zip(c_shape, c_stride))) + 1
    C = np.zeros(c_size, dtype=np.float64)
    rc = lib().orc_contract5d_f64(_ptr(A), _ptr(a_shape), _ptr(a_stride), _ptr(B), _ptr(b_shape),
                                  _ptr(b_stride), _ptr(C), _ptr(c_stride), threads or nthreads())
    assert rc == 0
    return C


def tolerance(K, max_a, max_b):
    """Absolute part of the acceptance bound: 1e-3*sqrt(K)*max|a|*max|b|."""
    return 1e-3 * np.sqrt(max(K, 1)) * max_a * max_b


def check(got, ref, K, max_a, max_b):
    """|got - ref| <= 1e-3*sqrt(K)*max|a|*max|b| + 1e-3*|ref| elementwise.
    Returns (n_bad, max_abs, max_rel, first_bad_flat_index)."""
    got = np.ascontiguousarray(got, dtype=np.float32)
    ref = np.ascontiguousarray(ref, dtype=np.float64)
    assert got.shape == ref.shape
    g2 = got.reshape(-1, got.shape[-1]) if got.ndim > 1 else got.reshape(1, -1)
    r2 = ref.reshape(g2.shape)
    ma = ctypes.c_double()
    mr = ctypes.c_double()
    fb = ctypes.c_int64()
    bad = lib().orc_check_tolerance(_ptr(g2), g2.shape[1], _ptr(r2), r2.shape[1], g2.shape[0],
                                    g2.shape[1], K, float(max_a), float(max_b), ctypes.byref(ma),
                                    ctypes.byref(mr), ctypes.byref(fb))
    return int(bad), ma.value, mr.value, int(fb.value)


# ---- operand types other than fp16 (codes of b2g_gemm.h): raw bits as uint16 / uint8 arrays
F16, BF16, E4M3, E5M2 = 0, 1, 2, 3
_BITS = {F16: np.uint16, BF16: np.uint16, E4M3: np.uint8, E5M2: np.uint8}


def uniform(shape, seed, dtype, offset=0):
    """The seeded U[-1,1] sequence rounded (nearest even) into `dtype`; raw bits."""
    n = int(np.prod(shape)) if len(shape) else 1
    out = np.empty(n, dtype=_BITS[dtype])
    lib().orc_fill_uniform(_ptr(out), n, dtype, seed, offset)
    return out.reshape(shape)


def to_f32(bits, dtype):
    """Exact fp32 values of `dtype` bits."""
    bits = np.ascontiguousarray(bits, dtype=_BITS[dtype])
    out = np.empty(bits.shape, dtype=np.float32)
    lib().orc_typed_to_f32(_ptr(bits), dtype, _ptr(out), bits.size)
    return out


def from_f32(x, dtype):
    """fp32 -> `dtype` bits, round to nearest even (fp8: saturating)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=_BITS[dtype])
    lib().orc_f32_to_typed(_ptr(x), dtype, _ptr(out), x.size)
    return out


def gemm_f64_typed(A_bits, B_bits, dtype, rows=None, threads=None):
    """FP64-accumulated GEMM of two `dtype` matrices given as raw bits, rows [r0, r1)."""
    A = to_f32(A_bits, dtype)
    B = to_f32(B_bits, dtype)
    M, K = A.shape
    K2, N = B.shape
    assert K == K2
    r0, r1 = rows if rows is not None else (0, M)
    C = np.empty((r1 - r0, N), dtype=np.float64)
    lib().orc_gemm_f64_f32in(_ptr(A), _ptr(B), _ptr(C), M, N, K, K, N, N, r0, r1,
                             threads or nthreads())
    return C
