"""Seeded randomized parity tests against the FP64 oracle.

GEMM: random ragged M, N, K, row pitches padded or not (pitches that break TMA's 16-byte rules
take the generic kernel), alpha/beta, and a random kernel variant / split-K / fix-up choice;
the pad columns of C must stay untouched.  Contraction: random 5-D extents with each operand
stored in a random order of its modes (so the tensor maps see permuted strides), checked
through b2g_contract5d_ex.
Tolerance: |C - R| <= 1e-3*sqrt(K)*max|a|*max|b|*|alpha| + 1e-3*|R|.
"""
import itertools
import random

import numpy as np
import pytest

from gpu_util import VARIANTS, assert_close, options, to_dev

pytestmark = pytest.mark.gpu


def _gemm_case(rng):
    M = rng.choice([1, 7, 100, 128, 129, 255, 384, 600])
    N = rng.choice([1, 8, 56, 256, 300, 512, 700])
    K = rng.choice([1, 8, 63, 64, 65, 320, 1000, 1300])
    pad = lambda x: x + rng.choice([0, 0, 8, 13])
    opts = {}
    v = rng.choice([None] + VARIANTS)
    if v is not None:
        opts.update(cta_group=v[0], tile_n=v[1])
    opts["split_k"] = rng.choice([0, 0, 2, 3])
    opts["cluster_fixup"] = rng.choice([0, 1])
    alpha = rng.choice([1.0, 0.5, -2.0])
    beta = rng.choice([0.0, 0.0, 1.0, 0.25])
    return M, N, K, pad(K), pad(N), pad(N), alpha, beta, opts


@pytest.mark.parametrize("case", range(80))
def test_gemm_fuzz(b2g, cuda, orc, case):
    torch = cuda
    rng = random.Random(1000 + case)
    M, N, K, lda, ldb, ldc, alpha, beta, opts = _gemm_case(rng)
    seed = 3 * case + 11
    A = orc.uniform_f16((M, K), seed)
    B = orc.uniform_f16((K, N), seed + 1)
    Ap = orc.uniform_f16((M, lda), seed + 7)
    Ap[:, :K] = A
    Bp = orc.uniform_f16((K, ldb), seed + 8)
    Bp[:, :N] = B
    C0 = orc.uniform_f16((M, N), seed + 2).astype(np.float32)
    Cp = np.full((M, ldc), np.nan, np.float32)
    Cp[:, :N] = C0
    dC = to_dev(torch, Cp)
    with options(b2g, **opts):
        b2g.gemm_ex(to_dev(torch, Ap), to_dev(torch, Bp), dC, M, N, K, alpha, beta, lda=lda,
                    ldb=ldb, ldc=ldc)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    out = dC.cpu().numpy()
    ref = alpha * orc.gemm_f64(A, B) + beta * C0.astype(np.float64)
    what = "case %d: %dx%dx%d ld=(%d,%d,%d) a=%g b=%g %r path=%d" % (
        case, M, N, K, lda, ldb, ldc, alpha, beta, opts, b2g.last_path())
    assert_close(orc, out[:, :N], ref, K, abs(alpha), 1.0, what=what)
    assert np.isnan(out[:, N:]).all(), what  # pad columns untouched


def _strides(shape, order):
    """Element strides of a dense tensor of `shape` stored with its modes in `order`
    (outermost first)."""
    st = [0] * len(shape)
    s = 1
    for d in reversed(order):
        st[d] = s
        s *= shape[d]
    return st, s


@pytest.mark.parametrize("case", range(24))
def test_contraction_fuzz(b2g, cuda, orc, case):
    torch = cuda
    rng = random.Random(5000 + case)
    a, b, i = rng.choice([1, 2, 3]), rng.choice([1, 2, 4]), rng.choice([8, 16, 33, 64])
    j, k, n = rng.choice([1, 2, 3]), rng.choice([8, 64, 72, 128]), rng.choice([8, 40, 256, 264])
    a_shape, b_shape, c_shape = (a, b, i, j, k), (j, k, n), (a, b, i, n)
    perms = lambda r: list(itertools.permutations(range(r)))
    # half the cases keep each operand in its natural order (the fast path); the others
    # permute every operand's storage order
    if case % 2 == 0:
        a_ord, b_ord, c_ord = (0, 1, 2, 3, 4), (0, 1, 2), (0, 1, 2, 3)
    else:
        a_ord, b_ord, c_ord = rng.choice(perms(5)), rng.choice(perms(3)), rng.choice(perms(4))
    a_st, a_n = _strides(a_shape, a_ord)
    b_st, b_n = _strides(b_shape, b_ord)
    c_st, c_n = _strides(c_shape, c_ord)
    A = orc.uniform_f16((a_n,), 40 + case)
    B = orc.uniform_f16((b_n,), 80 + case)
    alpha = rng.choice([1.0, -0.5])
    dC = torch.full((c_n,), float("nan"), dtype=torch.float32, device="cuda")
    b2g.contract5d_ex(to_dev(torch, A), a_shape, a_st, to_dev(torch, B), b_shape, b_st, dC,
                      c_shape, c_st, alpha, 0.0)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    ref = alpha * orc.contract5d_f64(A, a_shape, a_st, B, b_shape, b_st, c_shape, c_st,
                                     c_size=c_n)
    assert_close(orc, dC.cpu().numpy(), ref, j * k, abs(alpha), 1.0,
                 what="case %d: A%r%r B%r%r C%r%r path=%d" % (case, a_shape, a_ord, b_shape, b_ord,
                                                             c_shape, c_ord, b2g.last_path()))


@pytest.mark.parametrize("case", range(24))
def test_typed_gemm_fuzz(b2g, cuda, orc, case):
    """bf16 / e4m3 / e5m2 operands on random ragged shapes, pitches, alpha/beta and kernel
    choices (8-bit pitches that are not multiples of 16 bytes take the generic kernel)."""
    torch = cuda
    rng = random.Random(9000 + case)
    dt = (1, 2, 3)[case % 3]
    M = rng.choice([1, 100, 128, 300, 512])
    N = rng.choice([16, 200, 256, 528])
    K = rng.choice([16, 64, 200, 512, 1040])
    pad = lambda x: x + rng.choice([0, 0, 16, 7])
    lda, ldb, ldc = pad(K), pad(N), pad(N)
    opts = {}
    v = rng.choice([None] + VARIANTS)
    if v is not None:
        opts.update(cta_group=v[0], tile_n=v[1])
    opts["split_k"] = rng.choice([0, 0, 2])
    alpha, beta = rng.choice([1.0, -0.5]), rng.choice([0.0, 1.0])
    A = orc.uniform((M, lda), 300 + case, dt)
    B = orc.uniform((K, ldb), 400 + case, dt)
    C0 = orc.uniform_f16((M, N), 500 + case).astype(np.float32)
    Cp = np.full((M, ldc), np.nan, np.float32)
    Cp[:, :N] = C0
    dA, dB, dC = to_dev(torch, A), to_dev(torch, B), to_dev(torch, Cp)
    with options(b2g, **opts):
        b2g.gemm_typed(dA, dB, dC, M, N, K, dt, alpha, beta, lda=lda, ldb=ldb, ldc=ldc)
        torch.cuda.synchronize()
        path = b2g.last_path()
    assert b2g.device_status() == 0
    A, B = A[:, :K], B[:, :N]
    Af, Bf = orc.to_f32(A, dt), orc.to_f32(B, dt)
    ref = alpha * orc.gemm_f64_typed(A, B, dt) + beta * C0.astype(np.float64)
    out = dC.cpu().numpy()
    what = "case %d dtype %d: %dx%dx%d ld=(%d,%d,%d) a=%g b=%g %r path=%d" % (
        case, dt, M, N, K, lda, ldb, ldc, alpha, beta, opts, path)
    assert_close(orc, out[:, :N], ref, K, abs(alpha) * float(np.abs(Af).max()),
                 float(np.abs(Bf).max()), what=what)
    assert np.isnan(out[:, N:]).all(), what
