"""b2g_gemm_f16_f32_noalloc: the GEMM entry point that allocates nothing.

Some callers can't call cudaMalloc -- for example a host runtime that has handed all device
memory to its own pool allocator up front, or a serving loop that must not allocate on every
call.  When the library splits K (too few output tiles to fill the GPU) and the partial tiles
go through global memory, the ordinary entry point takes that workspace from cudaMallocAsync;
this one uses a fixed 32 MiB array compiled into the library instead.  (Splits reduced through
distributed shared memory need no workspace at all, so the comparison turns that fix-up off to
keep the array in use.)  These tests call it through the C ABI and check its result against
the ordinary entry point's on two calls in a row -- the array keeps the previous call's
contents, so the second call shows that nothing stale is read -- and check that a request
needing more scratch than the array holds is refused with a clear error, and that a split the
default plan only adds for the tail wave is dropped (not refused) when it does not fit.
Results are also checked against the FP64 oracle on sampled rows.  This file is collected
last.
"""
import ctypes

import numpy as np
import pytest

from gpu_util import assert_close, options

pytestmark = pytest.mark.gpu


def _stream(torch):
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_allocating_entry_point_twice(b2g, cuda, orc):
    torch = cuda
    L = b2g.load()
    L.b2g_gemm_f16_f32_noalloc.restype = ctypes.c_int
    L.b2g_gemm_f16_f32_noalloc.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 6 + \
        [ctypes.c_void_p]
    # one 128-row tile row over 4096 columns: 16 tiles of 128 x 256, so the library splits K 8
    # ways; with the global-memory fix-up the 16 MiB of partial tiles live in the scratch array
    M, N, K = 128, 4096, 8192
    assert b2g.plan_preview(M, N, K)[2] > 1
    dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
    dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
    b2g.fill_uniform(dA, M * K, 71)
    b2g.fill_uniform(dB, K * N, 72)
    with options(b2g, cluster_fixup=0):
        ref = torch.empty((M, N), dtype=torch.float32, device="cuda")
        b2g.gemm(dA, dB, ref, M, N, K)  # the ordinary (allocating) entry point
        torch.cuda.synchronize()
        ref_h = ref.cpu().numpy().astype(np.float64)
        for call in range(2):
            out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
            rc = L.b2g_gemm_f16_f32_noalloc(dA.data_ptr(), dB.data_ptr(), out.data_ptr(), M, N,
                                            K, K, N, N, _stream(torch))
            assert rc == b2g.OK, L.b2g_last_error_string()
            torch.cuda.synchronize()
            assert b2g.device_status() == 0
            assert_close(orc, out.cpu().numpy(), ref_h, K, what="no-alloc call %d" % call)
    # the 8 partials of a tile are summed in the same order either way: identical bits
    assert torch.equal(out, ref)
    # and against the FP64 oracle on sampled rows (the same seeded operands, made on the host)
    B = orc.uniform_f16((K, N), 72)
    for r in (0, 1, 63, 64, 100, 127):
        a = orc.uniform_f16((1, K), 71, r * K)
        assert_close(orc, out[r:r + 1].cpu().numpy(), orc.gemm_f64(a, B), K, what="row %d" % r)


def test_noalloc_drops_a_tail_split_that_does_not_fit(b2g, cuda, orc):
    """Under the default plan a grid of whole waves plus a partial one splits only the partial
    wave's tiles; with 512-wide CTA-pair tiles those partials can need more than the 32 MiB
    array.  The no-alloc entry point then runs the tail unsplit instead of refusing: it must
    return B2G_OK with a correct result.  (Its bits may differ from the allocating call's,
    which keeps the split.)  The shape is found on the device: the first candidate whose
    allocating call keeps more than 32 MiB of partials."""
    torch = cuda
    L = b2g.load()
    L.b2g_gemm_f16_f32_noalloc.restype = ctypes.c_int
    L.b2g_gemm_f16_f32_noalloc.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 6 + \
        [ctypes.c_void_p]
    K = 4096
    found = None
    for m_t, n_t in [(15, 11), (16, 10), (17, 10), (13, 13), (18, 9), (14, 12), (19, 9)]:
        M, N = 256 * m_t, 512 * n_t
        dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
        dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
        b2g.fill_uniform(dA, M * K, 73)
        b2g.fill_uniform(dB, K * N, 74)
        ref = torch.empty((M, N), dtype=torch.float32, device="cuda")
        b2g.gemm(dA, dB, ref, M, N, K)
        torch.cuda.synchronize()
        if b2g.get_option("last_split_ws_bytes") > (32 << 20):
            found = (M, N, dA, dB, ref)
            break
    if found is None:
        pytest.skip("no candidate shape needs more than 32 MiB of tail-split partials here")
    M, N, dA, dB, ref = found
    out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    rc = L.b2g_gemm_f16_f32_noalloc(dA.data_ptr(), dB.data_ptr(), out.data_ptr(), M, N, K, K, N,
                                    N, _stream(torch))
    assert rc == b2g.OK, L.b2g_last_error_string()
    assert b2g.get_option("last_split_ws_bytes") == 0  # the tail ran unsplit
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    assert not torch.isnan(out).any()
    assert_close(orc, out.cpu().numpy(), ref.cpu().numpy().astype(np.float64), K,
                 what="against the allocating entry point")
    B = orc.uniform_f16((K, N), 74)
    for r in (0, M // 2, M - 1):
        a = orc.uniform_f16((1, K), 73, r * K)
        assert_close(orc, out[r:r + 1].cpu().numpy(), orc.gemm_f64(a, B), K, what="row %d" % r)


def test_noalloc_refuses_scratch_beyond_its_maximum(b2g, cuda):
    torch = cuda
    L = b2g.load()
    L.b2g_gemm_f16_f32_noalloc.restype = ctypes.c_int
    L.b2g_gemm_f16_f32_noalloc.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 6 + \
        [ctypes.c_void_p]
    M = N = 2048
    K = 8192
    dA = torch.zeros((M, K), dtype=torch.float16, device="cuda")
    dC = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    with options(b2g, split_k=64):  # 64-way split of every tile: far more than 32 MiB
        rc = L.b2g_gemm_f16_f32_noalloc(dA.data_ptr(), dA.data_ptr(), dC.data_ptr(), M, N, K,
                                        K, N, N, _stream(torch))
    assert rc == b2g.ERR_INVALID_ARG
    assert b"exceeds" in L.b2g_last_error_string()
