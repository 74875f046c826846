"""ctypes binding of libb2g_gemm.so, the C ABI declared in include/b2g_gemm.h.

This is the Python mirror of the reference's drop-in surface: GEMM(A, B, C, M, N, K) for
the kernel launch of mmm.cpp:1496 and contract5d(...) for the G pack + contraction launch
of mmmTensor.cpp:329-369.  Operands are device pointers (ints) or objects exposing
``data_ptr()`` (e.g. torch CUDA tensors, used only as device-memory plumbing).

The binding never computes anything itself: if the shared library is missing it raises,
and every call goes to the CUDA kernels.
"""
import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libb2g_gemm.so")
HEADER = os.path.join(ROOT, "include", "b2g_gemm.h")

OK = 0
ERR_INVALID_ARG = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_TIMEOUT = 4
ERR_NCCL = 5

DTYPE_F16, DTYPE_BF16, DTYPE_E4M3, DTYPE_E5M2, DTYPE_F32 = 0, 1, 2, 3, 4

PATH_NONE, PATH_TC_1CTA, PATH_TC_2CTA, PATH_GENERIC, PATH_ZERO, PATH_EMPTY = range(6)
PATH_NAMES = {0: "none", 1: "tc_1cta", 2: "tc_2cta", 3: "generic", 4: "zero", 5: "empty"}


class B2GError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__("b2g error %d: %s" % (code, msg))
        self.code = code


_lib = None


def load(path=None):
    """Load libb2g_gemm.so (built by build.py).  Raises if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise FileNotFoundError(
            "libb2g_gemm.so not found at %s; build it with python rdna4-gemm-wmma_b200/build.py" % p)
    L = ctypes.CDLL(p)
    i64, vp = ctypes.c_int64, ctypes.c_void_p
    i64p = ctypes.POINTER(ctypes.c_int64)
    L.b2g_gemm_f16_f32.restype = ctypes.c_int
    L.b2g_gemm_f16_f32.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, vp]
    L.b2g_gemm_ex.restype = ctypes.c_int
    L.b2g_gemm_ex.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, ctypes.c_float,
                              ctypes.c_float, vp]
    L.b2g_contract5d_ex.restype = ctypes.c_int
    L.b2g_contract5d_ex.argtypes = [vp, i64p, i64p, vp, i64p, i64p, vp, i64p, i64p,
                                    ctypes.c_float, ctypes.c_float, vp]
    L.b2g_gemm.restype = ctypes.c_int
    L.b2g_gemm.argtypes = [vp, vp, vp, i64, i64, i64]
    L.b2g_gemm_typed.restype = ctypes.c_int
    L.b2g_gemm_typed.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, ctypes.c_int,
                                 ctypes.c_float, ctypes.c_float, vp]
    L.b2g_contract5d_typed.restype = ctypes.c_int
    L.b2g_contract5d_typed.argtypes = [vp, i64p, i64p, vp, i64p, i64p, vp, i64p, i64p,
                                       ctypes.c_int, ctypes.c_float, ctypes.c_float, vp]
    L.b2g_fill_uniform.restype = ctypes.c_int
    L.b2g_fill_uniform.argtypes = [vp, i64, ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64, vp]
    L.b2g_gemm_f16_f32_noalloc.restype = ctypes.c_int
    L.b2g_gemm_f16_f32_noalloc.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, vp]
    L.b2g_contract5d_f16_f32.restype = ctypes.c_int
    L.b2g_contract5d_f16_f32.argtypes = [vp, i64p, i64p, vp, i64p, i64p, vp, i64p, i64p, vp]
    L.b2g_fill_uniform_f16.restype = ctypes.c_int
    L.b2g_fill_uniform_f16.argtypes = [vp, i64, ctypes.c_uint64, ctypes.c_uint64, vp]
    L.b2g_last_error_string.restype = ctypes.c_char_p
    L.b2g_last_error_string.argtypes = []
    L.b2g_last_path.restype = ctypes.c_int
    L.b2g_device_status.restype = ctypes.c_int
    L.b2g_device_status.argtypes = [ctypes.c_int]
    L.b2g_set_option.restype = ctypes.c_int
    L.b2g_set_option.argtypes = [ctypes.c_char_p, i64]
    L.b2g_get_option.restype = i64
    L.b2g_get_option.argtypes = [ctypes.c_char_p]
    L.b2g_tile_coord.restype = None
    L.b2g_tile_coord.argtypes = [ctypes.c_int] * 4 + [ctypes.POINTER(ctypes.c_int)] * 2
    L.b2g_version.restype = ctypes.c_char_p
    L.b2g_gemm_sharded.restype = ctypes.c_int
    L.b2g_gemm_sharded.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, vp, ctypes.c_int,
                                   ctypes.c_int, vp]
    L.b2g_gemm_sharded_k.restype = ctypes.c_int
    L.b2g_gemm_sharded_k.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, vp, vp]
    L.b2g_gemm_sharded_n.restype = ctypes.c_int
    L.b2g_gemm_sharded_n.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, vp, ctypes.c_int,
                                     ctypes.c_int, vp, vp]
    L.b2g_rs_plan_create.restype = ctypes.c_int
    L.b2g_rs_plan_create.argtypes = [vp, i64, i64, ctypes.POINTER(ctypes.c_void_p)]
    L.b2g_rs_plan_destroy.restype = ctypes.c_int
    L.b2g_rs_plan_destroy.argtypes = [vp]
    L.b2g_gemm_sharded_k_p2p.restype = ctypes.c_int
    L.b2g_gemm_sharded_k_p2p.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, vp]
    L.b2g_gemm_sum_slots.restype = ctypes.c_int
    L.b2g_gemm_sum_slots.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, vp, i64,
                                     ctypes.c_int, ctypes.c_int, vp, ctypes.c_uint32, vp]
    L.b2g_chain_plan_create.restype = ctypes.c_int
    L.b2g_chain_plan_create.argtypes = [vp, vp, i64, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]
    L.b2g_chain_plan_destroy.restype = ctypes.c_int
    L.b2g_chain_plan_destroy.argtypes = [vp]
    L.b2g_gemm_sharded_chain.restype = ctypes.c_int
    L.b2g_gemm_sharded_chain.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, ctypes.c_int, vp]
    L.b2g_chain_broadcast.restype = ctypes.c_int
    L.b2g_chain_broadcast.argtypes = [vp, i64, ctypes.c_int, vp]
    L.b2g_plan_preview.restype = ctypes.c_int
    L.b2g_plan_preview.argtypes = [i64, i64, i64, ctypes.c_int, ctypes.c_int] + \
        [ctypes.POINTER(ctypes.c_int)] * 5
    L.b2g_gemm_sharded_n_chain.restype = ctypes.c_int
    L.b2g_gemm_sharded_n_chain.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, ctypes.c_int, vp]
    L.b2g_gemm_epilogue.restype = ctypes.c_int
    L.b2g_gemm_epilogue.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, ctypes.c_int,
                                    ctypes.c_float, ctypes.c_float, vp, ctypes.c_int, vp]
    L.b2g_contract5d_epilogue.restype = ctypes.c_int
    L.b2g_contract5d_epilogue.argtypes = [vp, i64p, i64p, vp, i64p, i64p, vp, i64p, i64p,
                                          ctypes.c_int, ctypes.c_float, ctypes.c_float, vp,
                                          ctypes.c_int, vp]
    L.b2g_contract5d_batched.restype = ctypes.c_int
    L.b2g_contract5d_batched.argtypes = [vp, i64p, i64p, vp, i64p, i64p, i64, vp, i64p, i64p,
                                         ctypes.c_int, ctypes.c_float, ctypes.c_float, vp]
    L.b2g_gemm_batched.restype = ctypes.c_int
    L.b2g_gemm_batched.argtypes = [vp, vp, vp] + [i64] * 10 + [vp]
    L.b2g_slab_rows.restype = ctypes.c_int
    L.b2g_slab_rows.argtypes = [i64, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int64),
                                ctypes.POINTER(ctypes.c_int64)]
    L.b2g_comm_unique_id.restype = ctypes.c_int
    L.b2g_comm_unique_id.argtypes = [vp]
    L.b2g_comm_init.restype = ctypes.c_int
    L.b2g_comm_init.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int, vp]
    L.b2g_comm_destroy.restype = ctypes.c_int
    L.b2g_comm_destroy.argtypes = [vp]
    L.b2g_comm_check.restype = ctypes.c_int
    L.b2g_comm_check.argtypes = [vp, i64, vp]
    if path is None:
        _lib = L
    return L


def declared_symbols(header=HEADER):
    """Names of the functions include/b2g_gemm.h declares."""
    txt = open(header).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(b2g_[a-z0-9_]+)\s*\(", txt)))


def _ptr(x):
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    raise TypeError("expected a device pointer (int) or an object with data_ptr()")


def _stream(s):
    if s is None:
        try:
            import torch  # plumbing only: the caller's current stream
            if torch.cuda.is_available():
                return torch.cuda.current_stream().cuda_stream
        except ImportError:
            pass
        return None
    if isinstance(s, int):
        return s
    return s.cuda_stream


def _check(rc):
    if rc != OK:
        raise B2GError(rc, load().b2g_last_error_string().decode())


def gemm(A, B, C, M, N, K, lda=None, ldb=None, ldc=None, stream=None):
    """C[M,N] = A[M,K] . B[K,N] (fp16 in, fp32 out, row-major)."""
    L = load()
    _check(L.b2g_gemm_f16_f32(_ptr(A), _ptr(B), _ptr(C), M, N, K,
                              K if lda is None else lda, N if ldb is None else ldb,
                              N if ldc is None else ldc, _stream(stream)))


def gemm_ex(A, B, C, M, N, K, alpha=1.0, beta=0.0, lda=None, ldb=None, ldc=None, stream=None):
    """C = alpha * A[M,K].B[K,N] + beta * C."""
    L = load()
    _check(L.b2g_gemm_ex(_ptr(A), _ptr(B), _ptr(C), M, N, K, K if lda is None else lda,
                         N if ldb is None else ldb, N if ldc is None else ldc, float(alpha),
                         float(beta), _stream(stream)))


def GEMM(A, B, C, M, N, K):
    """The reference's drop-in form (contiguous, default stream)."""
    _check(load().b2g_gemm(_ptr(A), _ptr(B), _ptr(C), M, N, K))


def _arr(vals, n):
    vals = [int(v) for v in vals]
    assert len(vals) == n
    return (ctypes.c_int64 * n)(*vals)


def contract5d(A, a_shape, a_stride, B, b_shape, b_stride, C, c_shape, c_stride, stream=None):
    """C[a,b,i,n] = sum_{j,k} A[a,b,i,j,k] B[j,k,n]; shapes/strides in elements."""
    L = load()
    _check(L.b2g_contract5d_f16_f32(_ptr(A), _arr(a_shape, 5), _arr(a_stride, 5), _ptr(B),
                                    _arr(b_shape, 3), _arr(b_stride, 3), _ptr(C), _arr(c_shape, 4),
                                    _arr(c_stride, 4), _stream(stream)))


def contract5d_ex(A, a_shape, a_stride, B, b_shape, b_stride, C, c_shape, c_stride, alpha=1.0,
                  beta=0.0, stream=None):
    L = load()
    _check(L.b2g_contract5d_ex(_ptr(A), _arr(a_shape, 5), _arr(a_stride, 5), _ptr(B),
                               _arr(b_shape, 3), _arr(b_stride, 3), _ptr(C), _arr(c_shape, 4),
                               _arr(c_stride, 4), float(alpha), float(beta), _stream(stream)))


def fill_uniform(dst, n, seed, offset=0, stream=None, dtype=DTYPE_F16):
    """n elements of the seeded U[-1,1] sequence (element offset `offset`) in `dtype`."""
    _check(load().b2g_fill_uniform(_ptr(dst), n, dtype, seed, offset, _stream(stream)))


def gemm_typed(A, B, C, M, N, K, dtype, alpha=1.0, beta=0.0, lda=None, ldb=None, ldc=None,
               stream=None):
    """C = alpha * A.B + beta * C with A, B of operand type `dtype` (DTYPE_*)."""
    _check(load().b2g_gemm_typed(_ptr(A), _ptr(B), _ptr(C), M, N, K, K if lda is None else lda,
                                 N if ldb is None else ldb, N if ldc is None else ldc, dtype,
                                 float(alpha), float(beta), _stream(stream)))


def last_path():
    return load().b2g_last_path()


def device_status(clear=True):
    return load().b2g_device_status(1 if clear else 0)


def set_option(key, value):
    rc = load().b2g_set_option(key.encode(), int(value))
    if rc != OK:
        raise B2GError(rc, "bad option %s=%r" % (key, value))


def get_option(key):
    return load().b2g_get_option(key.encode())


def tile_coord(t, num_m, num_n, group):
    tm, tn = ctypes.c_int(), ctypes.c_int()
    load().b2g_tile_coord(t, num_m, num_n, group, ctypes.byref(tm), ctypes.byref(tn))
    return tm.value, tn.value


def slab_rows(M, world, rank):
    """(row0, rows) of rank's M-row slab (balanced contiguous partition)."""
    r0, n = ctypes.c_int64(), ctypes.c_int64()
    _check(load().b2g_slab_rows(M, world, rank, ctypes.byref(r0), ctypes.byref(n)))
    return r0.value, n.value


def comm_unique_id():
    """128-byte NCCL unique id (bytes) for b2g_comm_init."""
    buf = ctypes.create_string_buffer(128)
    _check(load().b2g_comm_unique_id(buf))
    return buf.raw


def comm_init(world, rank, uid):
    comm = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(bytes(uid), 128)
    _check(load().b2g_comm_init(ctypes.byref(comm), world, rank, buf))
    return comm.value


def comm_destroy(comm):
    _check(load().b2g_comm_destroy(comm))


def comm_check(comm, timeout_ms=5000, stream=None):
    """Liveness check between steps: B2G_OK if every rank answered within timeout_ms, else the
    communicator is aborted and B2GError (ERR_TIMEOUT) is raised."""
    _check(load().b2g_comm_check(comm, int(timeout_ms), None if stream is None else _stream(stream)))


def gemm_sharded(A_slab, B, C_slab, M, N, K, comm, root=0, k_panels=4, lda=None, ldb=None,
                 ldc=None, stream=None):
    """This rank's part of the M-row-slab sharded GEMM; B is broadcast from root in K panels."""
    _check(load().b2g_gemm_sharded(_ptr(A_slab), _ptr(B), _ptr(C_slab), M, N, K,
                                   K if lda is None else lda, N if ldb is None else ldb,
                                   N if ldc is None else ldc, comm, root, k_panels,
                                   _stream(stream)))


def _ld(x, given, what):
    if given is not None:
        return given
    if hasattr(x, "stride"):
        return max(1, x.stride(0))
    raise ValueError(what + " is required for a raw pointer")


def gemm_sharded_k(A_kslab, B_kslab, C_slab, M, N, K, comm, lda=None, ldb=None, ldc=None,
                   stream=None):
    """K-split GEMM + reduce-scatter: this rank holds K slab slab_rows(K, world, rank) of A and
    B and receives rows [rank*M/world, (rank+1)*M/world) of C.  Leading dimensions default to
    the tensors' row strides."""
    _check(load().b2g_gemm_sharded_k(_ptr(A_kslab), _ptr(B_kslab), _ptr(C_slab), M, N, K,
                                     _ld(A_kslab, lda, "lda"), _ld(B_kslab, ldb, "ldb"),
                                     _ld(C_slab, ldc, "ldc"), comm, _stream(stream)))


def gemm_sharded_n(A, B_nslab, C_nslab, M, N, K, comm, root=0, m_panels=4, C_full=None,
                   lda=None, ldb=None, ldc=None, stream=None):
    """N-slab GEMM: A broadcast from root in row panels, this rank's column slab of C
    computed locally; with C_full, every rank also receives the whole C (all-gather)."""
    _check(load().b2g_gemm_sharded_n(_ptr(A), _ptr(B_nslab), _ptr(C_nslab), M, N, K,
                                     _ld(A, lda, "lda"), _ld(B_nslab, ldb, "ldb"),
                                     _ld(C_nslab, ldc, "ldc"), comm, root, m_panels,
                                     _ptr(C_full), _stream(stream)))


def rs_plan_create(comm, M, N):
    """Collective: receive slots for the peer-memory reduce-scatter of an M x N product."""
    plan = ctypes.c_void_p()
    _check(load().b2g_rs_plan_create(comm, M, N, ctypes.byref(plan)))
    return plan.value


def rs_plan_destroy(plan):
    _check(load().b2g_rs_plan_destroy(plan))


def gemm_sharded_k_p2p(plan, A_kslab, B_kslab, C_slab, M, N, K, lda=None, ldb=None, ldc=None,
                       stream=None):
    """gemm_sharded_k with the reduce-scatter fused into the GEMMs over peer memory."""
    _check(load().b2g_gemm_sharded_k_p2p(plan, _ptr(A_kslab), _ptr(B_kslab), _ptr(C_slab), M, N, K,
                                         _ld(A_kslab, lda, "lda"), _ld(B_kslab, ldb, "ldb"),
                                         _ld(C_slab, ldc, "ldc"), _stream(stream)))


def gemm_sum_slots(A, B, C, M, N, K, slots, slot_stride, count, self_index, status=None,
                   epoch=0, lda=None, ldb=None, ldc=None, stream=None):
    """C = sum over s < count, in order, of term s: A.B for s == self_index, else the fp32
    M x N block at slots + s * slot_stride (the peer-memory K-split's epilogue on its own)."""
    _check(load().b2g_gemm_sum_slots(_ptr(A), _ptr(B), _ptr(C), M, N, K,
                                     K if lda is None else lda, N if ldb is None else ldb,
                                     N if ldc is None else ldc,
                                     None if slots is None else _ptr(slots), slot_stride, count,
                                     self_index, None if status is None else _ptr(status),
                                     epoch, _stream(stream)))


def chain_plan_create(comm, B, nbytes, root=0):
    """Collective: copy-engine broadcast chain over `comm` for this rank's B buffer."""
    plan = ctypes.c_void_p()
    _check(load().b2g_chain_plan_create(comm, _ptr(B), nbytes, root, ctypes.byref(plan)))
    return plan.value


def chain_plan_destroy(plan):
    _check(load().b2g_chain_plan_destroy(plan))


def gemm_sharded_chain(plan, A_slab, C_slab, M, N, K, k_panels=8, lda=None, ldb=None, ldc=None,
                       stream=None):
    """This rank's part of the M-row-slab GEMM with B arriving through the chain plan."""
    _check(load().b2g_gemm_sharded_chain(plan, _ptr(A_slab), _ptr(C_slab), M, N, K,
                                         K if lda is None else lda, N if ldb is None else ldb,
                                         N if ldc is None else ldc, k_panels, _stream(stream)))


def chain_broadcast(plan, nbytes, panels=8, stream=None):
    """The plan's buffer (first nbytes) from the root to every rank along the chain."""
    _check(load().b2g_chain_broadcast(plan, nbytes, panels, _stream(stream)))


def plan_preview(M, N, K, dtype=0, sm_count=148, rows=False):
    """(cta_group, tile_n, k_splits, num_full) the library would choose (no GPU needed); with
    rows=True also the A rows per CTA (128, or 64 for half-height pair tiles)."""
    out = [ctypes.c_int() for _ in range(5)]
    _check(load().b2g_plan_preview(M, N, K, dtype, sm_count, *[ctypes.byref(x) for x in out]))
    vals = tuple(x.value for x in out)
    return vals if rows else vals[:4]


def gemm_sharded_n_chain(plan, B_nslab, C_nslab, M, N, K, m_panels=4, lda=None, ldb=None,
                         ldc=None, stream=None):
    """N-slab GEMM with A (the plan's buffer) arriving in row panels through the chain."""
    _check(load().b2g_gemm_sharded_n_chain(plan, _ptr(B_nslab), _ptr(C_nslab), M, N, K,
                                           K if lda is None else lda, _ld(B_nslab, ldb, "ldb"),
                                           _ld(C_nslab, ldc, "ldc"), m_panels, _stream(stream)))


def gemm_epilogue(A, B, C, M, N, K, dtype=0, alpha=1.0, beta=0.0, bias=None, c_dtype=4,
                  lda=None, ldb=None, ldc=None, stream=None):
    """C = alpha*A.B + beta*C + bias with C of type c_dtype (DTYPE_F32 / DTYPE_F16 / DTYPE_BF16)."""
    _check(load().b2g_gemm_epilogue(_ptr(A), _ptr(B), _ptr(C), M, N, K, K if lda is None else lda,
                                    N if ldb is None else ldb, N if ldc is None else ldc, dtype,
                                    float(alpha), float(beta), _ptr(bias), c_dtype,
                                    _stream(stream)))


def contract5d_epilogue(A, a_shape, a_stride, B, b_shape, b_stride, C, c_shape, c_stride, dtype=0,
                        alpha=1.0, beta=0.0, bias=None, c_dtype=4, stream=None):
    _check(load().b2g_contract5d_epilogue(_ptr(A), _arr(a_shape, 5), _arr(a_stride, 5), _ptr(B),
                                          _arr(b_shape, 3), _arr(b_stride, 3), _ptr(C),
                                          _arr(c_shape, 4), _arr(c_stride, 4), dtype, float(alpha),
                                          float(beta), _ptr(bias), c_dtype, _stream(stream)))


def gemm_batched(A, B, C, L, M, N, K, stride_a, stride_b, stride_c, lda=None, ldb=None,
                 ldc=None, stream=None):
    """C[l] = A[l].B[l] for l < L (batch strides in elements)."""
    _check(load().b2g_gemm_batched(_ptr(A), _ptr(B), _ptr(C), L, M, N, K,
                                   K if lda is None else lda, N if ldb is None else ldb,
                                   N if ldc is None else ldc, stride_a, stride_b, stride_c,
                                   _stream(stream)))


def contract5d_batched(A, a_shape, a_stride, B, b_shape, b_stride, b_batch_stride, C, c_shape,
                       c_stride, dtype=0, alpha=1.0, beta=0.0, stream=None):
    """C[a,b,i,n] = alpha*sum_{j,k} A[a,b,i,j,k] B[a,j,k,n] + beta*C (mode a is a batch mode)."""
    _check(load().b2g_contract5d_batched(_ptr(A), _arr(a_shape, 5), _arr(a_stride, 5), _ptr(B),
                                         _arr(b_shape, 3), _arr(b_stride, 3), b_batch_stride,
                                         _ptr(C), _arr(c_shape, 4), _arr(c_stride, 4), dtype,
                                         float(alpha), float(beta), _stream(stream)))


def version():
    return load().b2g_version().decode()
