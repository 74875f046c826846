"""CPU tests of the oracle (oracle/orc.c), pinned against golden fixtures produced by the
reference's own code (tests/golden/gen_golden.py: GEMM_Naive mmm.cpp:52-62, G pack
mmmTensor.cpp:329-340, validateResults mmmTensor.cpp:278-306)."""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _gemm_cases():
    z = np.load(os.path.join(GOLDEN, "gemm_naive.npz"))
    for i in range(int(z["n_cases"])):
        A = z["c%d_A" % i].view(np.float16)
        B = z["c%d_B" % i].view(np.float16)
        yield i, A, B, z["c%d_C" % i], str(z["c%d_dist" % i])


def test_fp16_conversions_exhaustive(orc):
    allh = np.arange(65536, dtype=np.uint16).view(np.float16)
    f = orc.h2f(allh)
    ref = allh.astype(np.float32)
    same = (f.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(f) & np.isnan(ref))
    assert same.all()
    rng = np.random.default_rng(0)
    x = np.concatenate([
        (rng.standard_normal(200000) * 300).astype(np.float32),
        (rng.standard_normal(200000) * 1e-5).astype(np.float32),
        np.array([65504, 65519.996, 65520, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26, 0.0, -0.0],
                 dtype=np.float32)])
    with np.errstate(over="ignore"):
        want = x.astype(np.float16)
    assert np.array_equal(orc.f2h(x).view(np.uint16), want.view(np.uint16))


def test_uniform_generator(orc):
    u = orc.uniform_f16((1 << 20,), 1)
    v = u.astype(np.float64)
    assert v.min() >= -1.0 and v.max() <= 1.0
    assert abs(v.mean()) < 5e-3 and abs(v.var() - 1.0 / 3.0) < 5e-3
    # deterministic, and offsets address the same stream
    assert np.array_equal(u.view(np.uint16), orc.uniform_f16((1 << 20,), 1).view(np.uint16))
    tail = orc.uniform_f16((1000,), 1, offset=5000)
    assert np.array_equal(tail.view(np.uint16), u[5000:6000].view(np.uint16))
    assert not np.array_equal(u[:1000].view(np.uint16), orc.uniform_f16((1000,), 2).view(np.uint16))


def test_sequential_gemm_bit_exact_vs_reference_gemm_naive(orc):
    for i, A, B, C, _ in _gemm_cases():
        got = orc.gemm_f32_seq(A, B)
        assert np.array_equal(got.view(np.uint32), C.view(np.uint32)), "case %d" % i


def test_blocked_cpu_baseline_bit_exact_vs_reference_gemm_naive(orc):
    for i, A, B, C, _ in _gemm_cases():
        for threads in (1, 3):
            got = orc.gemm_f32_blocked(A, B, threads=threads)
            assert np.array_equal(got.view(np.uint32), C.view(np.uint32)), "case %d" % i


def test_blocked_cpu_baseline_bit_exact_vs_sequential_random(orc):
    """Random ragged shapes, row ranges, thread counts and a shared widened B: the blocked
    baseline keeps GEMM_Naive's arithmetic (fp32, k ascending) bit for bit."""
    from hypothesis import given, settings, strategies as st

    @settings(max_examples=60, deadline=None)
    @given(M=st.integers(1, 70), N=st.integers(1, 140), K=st.integers(1, 300),
           seed=st.integers(0, 2**31), threads=st.integers(1, 5), data=st.data())
    def check(M, N, K, seed, threads, data):
        r0 = data.draw(st.integers(0, M - 1))
        r1 = data.draw(st.integers(r0 + 1, M))
        A = orc.uniform_f16((M, K), seed)
        B = orc.uniform_f16((K, N), seed + 1)
        ref = orc.gemm_f32_seq(A, B, rows=(r0, r1))
        Bf = orc.widen_b(B, threads=threads) if seed % 2 else None
        got = orc.gemm_f32_blocked(A, B, rows=(r0, r1), threads=threads, Bf=Bf)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))

    check()


def test_fp64_oracle_within_tolerance_of_reference(orc):
    for i, A, B, C, _ in _gemm_cases():
        K = A.shape[1]
        ref = orc.gemm_f64(A, B)
        bad, ma, mr, _ = orc.check(C, ref, K, 1.0, 1.0)
        assert bad == 0, "case %d" % i
        # and agrees with numpy's own float64 product
        assert np.allclose(ref, A.astype(np.float64) @ B.astype(np.float64), rtol=0, atol=1e-12)


def test_row_ranges(orc):
    i, A, B, C, _ = list(_gemm_cases())[5]
    rows = (17, 60)
    assert np.array_equal(orc.gemm_f32_seq(A, B, rows=rows).view(np.uint32),
                          C[rows[0]:rows[1]].view(np.uint32))
    assert np.array_equal(orc.gemm_f32_blocked(A, B, rows=rows).view(np.uint32),
                          C[rows[0]:rows[1]].view(np.uint32))
    ref = orc.gemm_f64(A, B, rows=rows)
    assert np.allclose(ref, orc.gemm_f64(A, B)[rows[0]:rows[1]], rtol=0, atol=0)


def _ref_form():
    z = np.load(os.path.join(GOLDEN, "contraction_ref.npz"))
    mt, rt, nt, rt_l, bt = (int(x) for x in z["dims"])
    return z, mt, rt, nt, rt_l, bt


def test_reference_form_strides_reproduce_reference_pack(orc):
    """The stride description of G used by b2g_contract5d (a_shape=(mt,1,rt,nt,rt_l),
    a_stride=(rt_l,0,nt*mt*rt_l,mt*rt_l,1)) addresses exactly the reference's packed A."""
    z, mt, rt, nt, rt_l, bt = _ref_form()
    G = z["G"]
    Ap = z["A_packed"].reshape(mt * rt, nt * rt_l)
    m, r, n, k = np.meshgrid(np.arange(mt), np.arange(rt), np.arange(nt), np.arange(rt_l), indexing="ij")
    idx = m * rt_l + r * nt * mt * rt_l + n * mt * rt_l + k
    view = np.empty_like(Ap)
    view[(m * rt + r).ravel(), (n * rt_l + k).ravel()] = G[idx.ravel()]
    assert np.array_equal(view, Ap)


def test_contraction_oracle_vs_reference_fixture(orc):
    z, mt, rt, nt, rt_l, bt = _ref_form()
    G = z["G"].view(np.float16)
    In = z["In"].view(np.float16)
    ref = orc.contract5d_f64(G, (mt, 1, rt, nt, rt_l), (rt_l, 0, nt * mt * rt_l, mt * rt_l, 1),
                             In, (nt, rt_l, bt), (rt_l, 1, nt * rt_l), (mt, 1, rt, bt),
                             (bt * rt, 0, 1, rt), c_size=mt * bt * rt)
    bad, ma, mr, _ = orc.check(z["Out"], ref, nt * rt_l, 1.0, 1.0)
    assert bad == 0
    # the packed-GEMM view of the same numbers
    Ap = z["A_packed"].view(np.float16).reshape(mt * rt, nt * rt_l)
    Bt = np.ascontiguousarray(In.reshape(bt, nt * rt_l).T)
    assert np.array_equal(orc.gemm_f32_seq(Ap, Bt).view(np.uint32), z["C_rowmajor"].view(np.uint32))


def test_known_answers(orc):
    K = 96
    ones = np.ones((8, K), np.float16)
    assert (orc.gemm_f32_seq(ones, ones.T.copy()) == K).all()
    A = orc.uniform_f16((8, K), 3)
    eye = np.eye(K, dtype=np.float16)
    assert np.array_equal(orc.gemm_f32_seq(A, eye), A.astype(np.float32))
    Ai = (np.arange(8 * K) % 7 - 3).astype(np.float16).reshape(8, K)
    Bi = (np.arange(K * 5) % 5 - 2).astype(np.float16).reshape(K, 5)
    assert np.array_equal(orc.gemm_f64(Ai, Bi), Ai.astype(np.int64) @ Bi.astype(np.int64))


def test_tolerance_check_catches_planted_error(orc):
    i, A, B, C, _ = list(_gemm_cases())[4]
    K = A.shape[1]
    ref = orc.gemm_f64(A, B)
    bad = C.copy()
    bad[3, 5] += np.float32(2 * orc.tolerance(K, 1, 1) + 1e-3 * abs(ref[3, 5]))
    n, ma, mr, first = orc.check(bad, ref, K, 1.0, 1.0)
    assert n == 1 and first == 3 * C.shape[1] + 5
    nan = C.copy()
    nan[0, 0] = np.nan
    assert orc.check(nan, ref, K, 1.0, 1.0)[0] == 1


@pytest.mark.parametrize("shape", [(2, 3, 4, 5, 6), (1, 1, 7, 2, 9)])
def test_contraction_oracle_matches_numpy_einsum(orc, shape):
    a, b, i, j, k = shape
    n = 11
    A = orc.uniform_f16((a, b, i, j, k), 5)
    B = orc.uniform_f16((j, k, n), 6)
    st = lambda s: [int(np.prod(s[d + 1:])) for d in range(len(s))]
    ref = orc.contract5d_f64(A, shape, st(shape), B, (j, k, n), st((j, k, n)), (a, b, i, n),
                             st((a, b, i, n)))
    want = np.einsum("abijk,jkn->abin", A.astype(np.float64), B.astype(np.float64))
    assert np.allclose(ref.reshape(a, b, i, n), want, rtol=1e-13, atol=1e-13)


@pytest.mark.parametrize("dt,tname", [(2, "float8_e4m3fn"), (3, "float8_e5m2")])
def test_fp8_conversions_match_torch(orc, dt, tname):
    """Decode of all 256 codes and round-to-nearest-even encode of random and tie values agree
    with torch's independent float8 implementation (in range; both saturate differently out of
    range, where torch gives NaN)."""
    torch = pytest.importorskip("torch")
    tdt = getattr(torch, tname)
    codes = np.arange(256, dtype=np.uint8)
    mine = orc.to_f32(codes, dt)
    ref = torch.from_numpy(codes).view(tdt).float().numpy()
    assert ((mine == ref) | (np.isnan(mine) & np.isnan(ref))).all()
    lim = 440.0 if dt == 2 else 57000.0
    x = np.clip(np.random.default_rng(dt).standard_normal(100000) * 4, -lim, lim).astype(np.float32)
    finite = ref[np.isfinite(ref)]
    ties = ((np.sort(finite)[1:] + np.sort(finite)[:-1]) / 2).astype(np.float32)
    x = np.concatenate([x, ties[np.abs(ties) < lim]])
    assert np.array_equal(orc.from_f32(x, dt), torch.from_numpy(x).to(tdt).view(torch.uint8).numpy())


def test_bf16_conversions_match_torch(orc):
    torch = pytest.importorskip("torch")
    allb = np.arange(65536, dtype=np.uint16)
    m = orc.to_f32(allb, orc.BF16)
    r = torch.from_numpy(allb.view(np.int16)).view(torch.bfloat16).float().numpy()
    assert ((m == r) | (np.isnan(m) & np.isnan(r))).all()
    x = (np.random.default_rng(5).standard_normal(100000) * 100).astype(np.float32)
    assert np.array_equal(orc.from_f32(x, orc.BF16),
                          torch.from_numpy(x).to(torch.bfloat16).view(torch.uint16).numpy())


def test_typed_uniform_is_the_fp16_sequence_rounded(orc):
    """Every operand type draws the same fp32 values; fp16 matches uniform_f16 bit for bit."""
    assert np.array_equal(orc.uniform((4096,), 9, orc.F16), orc.uniform_f16((4096,), 9).view(np.uint16))
    for dt in (orc.BF16, orc.E4M3, orc.E5M2):
        v = orc.to_f32(orc.uniform((4096,), 9, dt), dt)
        assert np.abs(v).max() <= 1.0 and np.abs(v - orc.uniform_f16((4096,), 9).astype(np.float32)).max() < 0.07
