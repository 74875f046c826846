"""Generate the golden fixtures in tests/golden/ from the reference's own code.

    python tests/golden/gen_golden.py

Needs the reference checkout (B2G_REFERENCE_DIR, or a `reference` directory beside the
repository; see oracle/build_ref.py):
oracle/build_ref.py compiles the reference's GEMM_Naive (mmm.cpp:52-62), its two
validateResults (mmm.cpp:1387-1407, mmmTensor.cpp:278-306) and its G pack loop
(mmmTensor.cpp:329-340) for the CPU.  Inputs come from the seeded generator of the oracle,
so the fixtures hold (inputs, reference outputs) pairs that tests/test_oracle.py and the GPU
tests replay without the reference present.

Files written:
  gemm_naive.npz        cases c<i>_{A,B,C}: A, B fp16 bits (uint16), C = GEMM_Naive(A, B)
                        (fp32), over ragged and tile-sized shapes, U[-1,1] and U[0,1] inputs.
  contraction_ref.npz   the reference's contraction at a small size: G, In (fp16 bits),
                        A_packed = the reference pack of G, C_rowmajor = GEMM_Naive(A_packed,
                        In^T), Out = C_rowmajor remapped to [m][b][r]; checked with the
                        reference's validateResults (mmmTensor.cpp:278-306), which must accept
                        Out and reject a perturbed copy.
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import build_ref, orc  # noqa: E402

GEMM_CASES = [
    # (M, N, K, seed, distribution)
    (1, 1, 1, 101, "pm1"),
    (5, 7, 3, 102, "pm1"),
    (16, 16, 16, 103, "pm1"),
    (33, 17, 50, 104, "pm1"),
    (64, 80, 96, 105, "pm1"),
    (127, 129, 64, 106, "pm1"),
    (128, 256, 64, 107, "pm1"),
    (96, 64, 520, 108, "pm1"),
    (40, 48, 256, 109, "u01"),   # the reference's own input distribution (mmm.cpp:1409-1414)
]

# reference contraction, reduced sizes (reference: mt=128, rt=64, nt=64, rt_l=128, bt=8192)
CON = dict(mt=5, rt=4, nt=3, rt_l=8, bt=24)


def _inputs(shape, seed, dist):
    x = orc.uniform_f16(shape, seed)
    if dist == "u01":
        x = np.abs(x)
    return x


def main():
    lib = ctypes.CDLL(build_ref.build(force=True))
    vp, i = ctypes.c_void_p, ctypes.c_int
    lib.ref_gemm_naive.argtypes = [vp, vp, vp, i, i, i]
    lib.ref_validate_tensor.argtypes = [vp, vp, i, i, i]
    lib.ref_validate_tensor.restype = i
    lib.ref_validate_gemm.argtypes = [vp, vp, i]
    lib.ref_validate_gemm.restype = i
    lib.ref_pack_g.argtypes = [vp, vp, i, i, i, i]
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)

    out = {}
    for idx, (M, N, K, seed, dist) in enumerate(GEMM_CASES):
        A = np.ascontiguousarray(_inputs((M, K), seed, dist))
        B = np.ascontiguousarray(_inputs((K, N), seed + 7, dist))
        C = np.empty((M, N), dtype=np.float32)
        lib.ref_gemm_naive(P(A), P(B), P(C), M, N, K)
        assert lib.ref_validate_gemm(P(C), P(C), M * N) == 1
        out["c%d_A" % idx] = A.view(np.uint16)
        out["c%d_B" % idx] = B.view(np.uint16)
        out["c%d_C" % idx] = C
        out["c%d_dist" % idx] = np.array(dist)
    out["n_cases"] = np.array(len(GEMM_CASES))
    np.savez_compressed(os.path.join(HERE, "gemm_naive.npz"), **out)

    mt, rt, nt, rt_l, bt = CON["mt"], CON["rt"], CON["nt"], CON["rt_l"], CON["bt"]
    M, K, N = mt * rt, nt * rt_l, bt
    G = np.ascontiguousarray(orc.uniform_f16((rt * nt * mt * rt_l,), 201))
    In = np.ascontiguousarray(orc.uniform_f16((bt * nt * rt_l,), 202))
    Ap = np.zeros((M, K), dtype=np.float16)
    lib.ref_pack_g(P(G), P(Ap), rt, nt, mt, rt_l)
    Bt = np.ascontiguousarray(In.reshape(bt, K).T)  # Input is K-major: In[b][n*rt_l+k]
    Crm = np.empty((M, N), dtype=np.float32)
    lib.ref_gemm_naive(P(Ap), P(Bt), P(Crm), M, N, K)
    Out = np.empty(mt * bt * rt, dtype=np.float32)
    for m in range(mt):
        for b in range(bt):
            for r in range(rt):
                Out[m * (bt * rt) + b * rt + r] = Crm[m * rt + r, b]
    assert lib.ref_validate_tensor(P(Out), P(Crm), mt, bt, rt) == 1
    bad = Out.copy()
    bad[7] += 1.0
    assert lib.ref_validate_tensor(P(bad), P(Crm), mt, bt, rt) == 0
    np.savez_compressed(os.path.join(HERE, "contraction_ref.npz"), G=G.view(np.uint16),
                        In=In.view(np.uint16), A_packed=Ap.view(np.uint16), C_rowmajor=Crm,
                        Out=Out, dims=np.array([mt, rt, nt, rt_l, bt]))
    print("wrote gemm_naive.npz (%d cases) and contraction_ref.npz" % len(GEMM_CASES))


if __name__ == "__main__":
    main()
