"""GPU parity of the typed entry points (b2g_gemm_typed, b2g_contract5d_typed,
b2g_fill_uniform) for bf16 and the fp8 types, against the FP64 oracle.

fp16 is the reference's operand type; bf16 (tcgen05 kind::f16, format BF16) and e4m3 / e5m2
(kind::f8f6f4) run on the same pipeline.  Products of any of these types are exact in fp32.
Tolerance: |C - R| <= 1e-3*sqrt(K)*max|a|*max|b| + 1e-3*|R| against the FP64 reference R of
the exact operand values.
"""
import numpy as np
import pytest

from gpu_util import VARIANT_H_IDS, VARIANTS_H, assert_close, options, to_dev

pytestmark = pytest.mark.gpu

DTYPES = [1, 2, 3]
DT_IDS = ["bf16", "e4m3", "e5m2"]


def _typed(b2g, torch, orc, M, N, K, dt, lda=None, ldb=None, ldc=None, seed=91, **opt):
    lda, ldb, ldc = lda or K, ldb or N, ldc or N
    A = orc.uniform((M, lda), seed, dt)
    B = orc.uniform((K, ldb), seed + 1, dt)
    dC = torch.full((M, ldc), float("nan"), dtype=torch.float32, device="cuda")
    dA, dB = to_dev(torch, A), to_dev(torch, B)  # keep the buffers alive across the call
    with options(b2g, **opt):
        b2g.gemm_typed(dA, dB, dC, M, N, K, dt, lda=lda, ldb=ldb, ldc=ldc)
        torch.cuda.synchronize()
        path = b2g.last_path()
    assert b2g.device_status() == 0
    return A[:, :K], B[:, :N], dC.cpu().numpy()[:, :N], path


@pytest.mark.parametrize("dt", DTYPES, ids=DT_IDS)
def test_fill_uniform_typed_matches_oracle(b2g, cuda, orc, dt):
    torch = cuda
    n = 1 << 18
    esz = 1 if dt >= 2 else 2
    d = torch.empty(n * esz, dtype=torch.uint8, device="cuda")
    L = b2g.load()
    rc = L.b2g_fill_uniform(d.data_ptr(), n, dt, 5, 777, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    host = orc.uniform((n,), 5, dt, offset=777)
    assert np.array_equal(d.cpu().numpy().view(host.dtype), host)


@pytest.mark.parametrize("cg,tn", VARIANTS_H, ids=VARIANT_H_IDS)
@pytest.mark.parametrize("dt", DTYPES, ids=DT_IDS)
@pytest.mark.parametrize("MNK", [(256, 512, 512), (384, 1024, 1152), (200, 272, 208)])
def test_gemm_typed(b2g, cuda, orc, cg, tn, dt, MNK):
    M, N, K = MNK
    r16 = lambda x: (x + 15) // 16 * 16
    A, B, C, path = _typed(b2g, cuda, orc, M, N, K, dt, lda=r16(K), ldb=r16(N), ldc=r16(N),
                           cta_group=cg, tile_n=tn)
    assert path in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)
    Af, Bf = orc.to_f32(A, dt), orc.to_f32(B, dt)
    ref = orc.gemm_f64_typed(A, B, dt)
    assert_close(orc, C, ref, K, float(np.abs(Af).max()), float(np.abs(Bf).max()),
                 what="dtype %d %s" % (dt, MNK))


@pytest.mark.parametrize("dt", DTYPES, ids=DT_IDS)
def test_gemm_typed_generic_bit_exact(b2g, cuda, orc, dt):
    """Unaligned pitches: the generic kernel accumulates exact products in fp32 with K
    ascending, so C equals the same sequential fp32 sum computed on the host."""
    M, N, K = 17, 13, 37
    A, B, C, path = _typed(b2g, cuda, orc, M, N, K, dt)
    assert path == b2g.PATH_GENERIC
    Af, Bf = orc.to_f32(A, dt), orc.to_f32(B, dt)
    acc = np.zeros((M, N), dtype=np.float32)
    for k in range(K):
        acc = acc + Af[:, k:k + 1] * Bf[k:k + 1, :]  # exact products, fp32 sums, k ascending
    assert np.array_equal(C.view(np.uint32), acc.view(np.uint32))


@pytest.mark.parametrize("dt", DTYPES, ids=DT_IDS)
def test_contract_reference_form_typed(b2g, cuda, orc, dt):
    """The reference's contraction layout (K-major B, M-contiguous output) for each type."""
    import ctypes
    torch = cuda
    mt, rt, nt, rt_l, bt = 8, 32, 2, 128, 256
    G = orc.uniform((rt * nt * mt * rt_l,), 93, dt)
    In = orc.uniform((bt * nt * rt_l,), 94, dt)
    a_shape, a_st = (mt, 1, rt, nt, rt_l), (rt_l, 0, nt * mt * rt_l, mt * rt_l, 1)
    b_shape, b_st = (nt, rt_l, bt), (rt_l, 1, nt * rt_l)
    c_shape, c_st = (mt, 1, rt, bt), (bt * rt, 0, 1, rt)
    dOut = torch.full((mt * bt * rt,), float("nan"), dtype=torch.float32, device="cuda")
    arr = lambda v: (ctypes.c_int64 * len(v))(*v)
    L = b2g.load()
    dG, dIn = to_dev(torch, G), to_dev(torch, In)  # keep the buffers alive across the call
    rc = L.b2g_contract5d_typed(dG.data_ptr(), arr(a_shape), arr(a_st),
                                dIn.data_ptr(), arr(b_shape), arr(b_st),
                                dOut.data_ptr(), arr(c_shape), arr(c_st), dt, ctypes.c_float(1.0),
                                ctypes.c_float(0.0), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.b2g_last_error_string()
    torch.cuda.synchronize()
    assert b2g.last_path() in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)
    # FP64 reference through the packed-GEMM view of the exact operand values
    Gf = orc.to_f32(G, dt).reshape(rt, nt, mt, rt_l)
    Inf = orc.to_f32(In, dt).reshape(bt, nt, rt_l)
    want = np.einsum("rnmk,bnk->mbr", Gf.astype(np.float64), Inf.astype(np.float64))
    assert_close(orc, dOut.cpu().numpy(), want.reshape(-1), nt * rt_l,
                 float(np.abs(Gf).max()), float(np.abs(Inf).max()))
