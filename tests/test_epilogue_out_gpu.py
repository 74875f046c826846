"""GPU tests of the fused epilogue variants (b2g_gemm_epilogue, b2g_contract5d_epilogue):
a per-column fp32 bias, and fp16 / bf16 output, against the FP64 oracle.

C = alpha*A.B + beta*C + bias.  The bias is added exactly once per element, also when K is
split (partials are fp32; the final store adds it).  A 16-bit C is the fp32 result rounded to
nearest even, so its tolerance adds the output type's unit roundoff u to the relative term:
|C - R| <= 1e-3*sqrt(K)*max|a|*max|b|*|alpha| + (1e-3 + u)*|R|  (u = 2^-11 fp16, 2^-8 bf16;
0 for fp32 C).  The pad columns of C must stay untouched.
"""
import numpy as np
import pytest

from gpu_util import VARIANT_H_IDS, VARIANTS_H, options, to_dev

pytestmark = pytest.mark.gpu

F32, F16, BF16 = 4, 0, 1
UROUND = {F32: 0.0, F16: 2.0 ** -11, BF16: 2.0 ** -8}
OUT_IDS = {F32: "f32", F16: "f16", BF16: "bf16"}


def _alloc_c(torch, M, ldc, c_dtype):
    if c_dtype == F32:
        return torch.full((M, ldc), float("nan"), dtype=torch.float32, device="cuda")
    dt = torch.float16 if c_dtype == F16 else torch.bfloat16
    return torch.full((M, ldc), float("nan"), dtype=dt, device="cuda")


def _host_f64(orc, dC, c_dtype):
    if c_dtype == F32:
        return dC.cpu().numpy().astype(np.float64)
    bits = dC.cpu().view(torch_int16()).numpy().view(np.uint16)
    return orc.to_f32(bits, c_dtype).astype(np.float64)


def torch_int16():
    import torch
    return torch.int16


def _check(orc, got, ref, K, alpha, c_dtype, what):
    tol = 1e-3 * np.sqrt(max(K, 1)) * abs(alpha) + (1e-3 + UROUND[c_dtype]) * np.abs(ref)
    err = np.abs(got - ref)
    bad = ~(err <= tol)
    assert not bad.any(), "%s: %d bad, max err %.3g, first %r" % (
        what, int(bad.sum()), float(np.nanmax(err)), np.argwhere(bad)[0].tolist())


@pytest.mark.parametrize("cg,tn", VARIANTS_H, ids=VARIANT_H_IDS)
@pytest.mark.parametrize("c_dtype", [F32, F16, BF16], ids=["f32", "f16", "bf16"])
def test_bias_and_output_type(b2g, cuda, orc, cg, tn, c_dtype):
    torch = cuda
    M, N, K = 384, 600, 320  # N not a multiple of 32: the last chunk is ragged
    ldc = 608
    A = orc.uniform_f16((M, K), 51)
    B = orc.uniform_f16((K, 608), 52)
    bias = orc.uniform_f16((N,), 53).astype(np.float32) * 4
    dC = _alloc_c(torch, M, ldc, c_dtype)
    alpha = -1.5
    with options(b2g, cta_group=cg, tile_n=tn):
        b2g.gemm_epilogue(to_dev(torch, A), to_dev(torch, B), dC, M, N, K, 0, alpha, 0.0,
                          to_dev(torch, bias), c_dtype, ldb=608, ldc=ldc)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    assert b2g.last_path() in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)
    got = _host_f64(orc, dC, c_dtype)
    ref = alpha * orc.gemm_f64(A, B[:, :N]) + bias.astype(np.float64)[None, :]
    _check(orc, got[:, :N], ref, K, alpha, c_dtype, "variant %s out %s" % ((cg, tn), c_dtype))
    assert np.isnan(got[:, N:]).all()


@pytest.mark.parametrize("c_dtype", [F32, F16, BF16], ids=["f32", "f16", "bf16"])
@pytest.mark.parametrize("cluster_fixup", [1, 0])
def test_bias_once_under_split_k(b2g, cuda, orc, c_dtype, cluster_fixup):
    """The bias is added by the final store only, whichever fix-up reduces the partials."""
    torch = cuda
    M, N, K = 128, 1024, 4096
    A = orc.uniform_f16((M, K), 54)
    B = orc.uniform_f16((K, N), 55)
    bias = np.linspace(-3, 3, N).astype(np.float32)
    dC = _alloc_c(torch, M, N, c_dtype)
    with options(b2g, split_k=4, cta_group=1, tile_n=256, cluster_fixup=cluster_fixup):
        b2g.gemm_epilogue(to_dev(torch, A), to_dev(torch, B), dC, M, N, K, 0, 1.0, 0.0,
                          to_dev(torch, bias), c_dtype)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    ref = orc.gemm_f64(A, B) + bias.astype(np.float64)[None, :]
    _check(orc, _host_f64(orc, dC, c_dtype), ref, K, 1.0, c_dtype, "split")


def test_bias_with_beta_fp32(b2g, cuda, orc):
    """fp32 C with beta = 1 (TMA reduce-add) and beta = 0.5 (scaled first): bias added once."""
    torch = cuda
    M, N, K = 256, 512, 512
    A = orc.uniform_f16((M, K), 56)
    B = orc.uniform_f16((K, N), 57)
    C0 = orc.uniform_f16((M, N), 58).astype(np.float32)
    bias = orc.uniform_f16((N,), 59).astype(np.float32)
    for beta in (1.0, 0.5):
        dC = to_dev(torch, C0)
        b2g.gemm_epilogue(to_dev(torch, A), to_dev(torch, B), dC, M, N, K, 0, 2.0, beta,
                          to_dev(torch, bias), F32)
        torch.cuda.synchronize()
        ref = 2.0 * orc.gemm_f64(A, B) + beta * C0.astype(np.float64) + bias[None, :]
        _check(orc, dC.cpu().numpy().astype(np.float64), ref, K, 2.0, F32, "beta %g" % beta)


@pytest.mark.parametrize("c_dtype", [F32, F16, BF16], ids=["f32", "f16", "bf16"])
def test_generic_path_bias_and_output_type(b2g, cuda, orc, c_dtype):
    torch = cuda
    M, N, K = 33, 19, 45  # unaligned pitches: the generic kernel
    A = orc.uniform_f16((M, K), 60)
    B = orc.uniform_f16((K, N), 61)
    bias = orc.uniform_f16((N,), 62).astype(np.float32)
    dC = _alloc_c(torch, M, N, c_dtype)
    b2g.gemm_epilogue(to_dev(torch, A), to_dev(torch, B), dC, M, N, K, 0, 0.5, 0.0,
                      to_dev(torch, bias), c_dtype)
    torch.cuda.synchronize()
    assert b2g.last_path() == b2g.PATH_GENERIC
    ref = 0.5 * orc.gemm_f64(A, B) + bias[None, :]
    _check(orc, _host_f64(orc, dC, c_dtype), ref, K, 0.5, c_dtype, "generic")


def test_typed_inputs_bf16_out(b2g, cuda, orc):
    """bf16 and e4m3 operands with a bf16 C and a bias."""
    torch = cuda
    M, N, K = 256, 512, 384
    for dt in (1, 2):
        A = orc.uniform((M, K), 63, dt)
        B = orc.uniform((K, N), 64, dt)
        bias = np.full(N, 0.75, np.float32)
        dC = _alloc_c(torch, M, N, BF16)
        b2g.gemm_epilogue(to_dev(torch, A), to_dev(torch, B), dC, M, N, K, dt, 1.0, 0.0,
                          to_dev(torch, bias), BF16)
        torch.cuda.synchronize()
        ref = orc.gemm_f64_typed(A, B, dt) + 0.75
        _check(orc, _host_f64(orc, dC, BF16), ref, K, 1.0, BF16, "dtype %d" % dt)


def test_reference_form_contraction_with_bias_bf16(b2g, cuda, orc):
    """The reference's [m][b][r] output layout (M-contiguous: generic kernel for a 16-bit C)
    and a contiguous contraction (tensor-core path), both with a bias over n."""
    torch = cuda
    mt, rt, nt, rt_l, bt = 4, 32, 2, 64, 256
    G = orc.uniform_f16((rt * nt * mt * rt_l,), 65)
    In = orc.uniform_f16((bt * nt * rt_l,), 66)
    bias = orc.uniform_f16((bt,), 67).astype(np.float32)
    a_shape, a_st = (mt, 1, rt, nt, rt_l), (rt_l, 0, nt * mt * rt_l, mt * rt_l, 1)
    b_shape, b_st = (nt, rt_l, bt), (rt_l, 1, nt * rt_l)
    c_shape, c_st = (mt, 1, rt, bt), (bt * rt, 0, 1, rt)
    dOut = torch.full((mt * bt * rt,), float("nan"), dtype=torch.bfloat16, device="cuda")
    b2g.contract5d_epilogue(to_dev(torch, G), a_shape, a_st, to_dev(torch, In), b_shape, b_st,
                            dOut, c_shape, c_st, 0, 1.0, 0.0, to_dev(torch, bias), BF16)
    torch.cuda.synchronize()
    ref = orc.contract5d_f64(G, a_shape, a_st, In, b_shape, b_st, c_shape, c_st,
                             c_size=mt * bt * rt).reshape(mt, bt, rt)
    ref = ref + bias.astype(np.float64)[None, :, None]
    got = _host_f64(orc, dOut, BF16).reshape(mt, bt, rt)
    _check(orc, got, ref, nt * rt_l, 1.0, BF16, "reference form")
    # contiguous operands: C[a,b,i,n] row-major, tensor-core path
    a, b, i, j, k, n = 2, 4, 32, 4, 64, 256
    A = orc.uniform_f16((a * b * i * j * k,), 68)
    Bm = orc.uniform_f16((j * k * n,), 69)
    st = lambda sh: [int(np.prod(sh[d + 1:])) for d in range(len(sh))]
    dC = torch.full((a * b * i * n,), float("nan"), dtype=torch.float16, device="cuda")
    b2g.contract5d_epilogue(to_dev(torch, A), (a, b, i, j, k), st((a, b, i, j, k)),
                            to_dev(torch, Bm), (j, k, n), st((j, k, n)), dC, (a, b, i, n),
                            st((a, b, i, n)), 0, 1.0, 0.0, to_dev(torch, bias[:n]), F16)
    torch.cuda.synchronize()
    assert b2g.last_path() in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)
    ref = orc.gemm_f64(A.reshape(a * b * i, j * k), Bm.reshape(j * k, n)) + bias[None, :n]
    _check(orc, _host_f64(orc, dC, F16).reshape(a * b * i, n), ref, j * k, 1.0, F16, "contiguous")


def test_16bit_output_rejects_beta(b2g, cuda):
    torch = cuda
    d = torch.zeros((128, 128), dtype=torch.float16, device="cuda")
    with pytest.raises(b2g.B2GError):
        b2g.gemm_epilogue(d, d, d, 128, 128, 128, 0, 1.0, 1.0, None, F16)
    with pytest.raises(b2g.B2GError):
        b2g.gemm_epilogue(d, d, d, 128, 128, 128, 0, 1.0, 0.0, None, 2)  # e4m3 C: unsupported
