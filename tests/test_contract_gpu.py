"""GPU parity tests of the 5-D contraction entry point against the CPU oracle.

C[a,b,i,n] = sum_{j,k} A[a,b,i,j,k] * B[j,k,n] read in place through tensor maps on the
caller's strides.  Two families:
  * the BASELINE form (contiguous [a][b][i][j][k] x [j][k][n] -> [a][b][i][n]) and
    permuted-memory variants of it that cannot be coalesced into a 2-D GEMM;
  * the reference's own form (mmmTensor.cpp): Out[m,b,r] = sum_{n,k} G[r,n,m,k] In[b,n,k]
    (G pack 329-340, K-major Input read 168, Output remap 246-252), i.e. K-major B and an
    M-contiguous output.
Tolerance: |C - R| <= 1e-3*sqrt(K)*max|a|*max|b| + 1e-3*|R| against the FP64 oracle.
"""
import numpy as np
import pytest

from gpu_util import VARIANT_H_IDS, VARIANTS_H, assert_close, options, to_dev

pytestmark = pytest.mark.gpu


def _dense_strides(shape, order):
    """Element strides of `shape` stored with dims in memory order `order` (outer first)."""
    st = [0] * len(shape)
    acc = 1
    for d in reversed(order):
        st[d] = acc
        acc *= shape[d]
    return st, acc


def _contract(b2g, torch, orc, a_shape, a_order, n, c_order, b_kmajor=False, seed=3):
    a, b, i, j, k = a_shape
    a_st, a_size = _dense_strides(a_shape, a_order)
    b_shape = (j, k, n)
    b_st, b_size = _dense_strides(b_shape, (2, 0, 1) if b_kmajor else (0, 1, 2))
    c_shape = (a, b, i, n)
    c_st, c_size = _dense_strides(c_shape, c_order)
    A = orc.uniform_f16((a_size,), seed)
    B = orc.uniform_f16((b_size,), seed + 1)
    dA, dB = to_dev(torch, A), to_dev(torch, B)
    dC = torch.full((c_size,), float("nan"), dtype=torch.float32, device="cuda")
    b2g.contract5d(dA, a_shape, a_st, dB, b_shape, b_st, dC, c_shape, c_st)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    path = b2g.last_path()
    ref = orc.contract5d_f64(A, a_shape, a_st, B, b_shape, b_st, c_shape, c_st, c_size=c_size)
    assert_close(orc, dC.cpu().numpy(), ref, j * k, what="contract %s" % (a_shape,))
    return path


@pytest.mark.parametrize("cg,tn", VARIANTS_H, ids=VARIANT_H_IDS)
def test_contract_baseline_form_small(b2g, cuda, orc, cg, tn):
    """BASELINE configs[2] layout at reduced size: coalesces to a plain 2-D GEMM view."""
    with options(b2g, cta_group=cg, tile_n=tn):
        path = _contract(b2g, cuda, orc, (2, 4, 32, 4, 64), (0, 1, 2, 3, 4), 256, (0, 1, 2, 3))
    assert path in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)


@pytest.mark.parametrize("cg,tn", VARIANTS_H, ids=VARIANT_H_IDS)
def test_contract_permuted_memory_not_coalescible(b2g, cuda, orc, cg, tn):
    """A stored as [b][a][i][j][k] and C as [b][a][i][n]: the M modes cannot be merged, so the
    load box spans (i, b, a) of a rank-5 tensor map and the store box spans three modes."""
    with options(b2g, cta_group=cg, tile_n=tn):
        path = _contract(b2g, cuda, orc, (2, 4, 16, 2, 64), (1, 0, 2, 3, 4), 192, (1, 0, 2, 3))
    assert path in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)


@pytest.mark.parametrize("cg,tn", VARIANTS_H, ids=VARIANT_H_IDS)
def test_contract_ragged_k_mode(b2g, cuda, orc, cg, tn):
    """A stored [b][a][j][i][k], so neither the K modes (j, k) nor the M modes (b, i) merge;
    k = 96 is not a multiple of the 64-wide K block: each j visits two K blocks, the second
    half zero-filled by TMA; i = 100 does not divide the 128-row tile (28 rows zero-filled,
    clipped at the store)."""
    with options(b2g, cta_group=cg, tile_n=tn):
        path = _contract(b2g, cuda, orc, (1, 3, 100, 3, 96), (1, 0, 3, 2, 4), 136, (1, 0, 2, 3))
    assert path in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)


def _reference_form(b2g, torch, orc, mt, rt, nt, rt_l, bt, seed=9):
    """The reference's contraction: G[r][n][m][k], In[b][n*rt_l+k], Out[m][b][r]."""
    G = orc.uniform_f16((rt * nt * mt * rt_l,), seed)
    In = orc.uniform_f16((bt * nt * rt_l,), seed + 1)
    a_shape = (mt, 1, rt, nt, rt_l)
    a_st = (rt_l, 0, nt * mt * rt_l, mt * rt_l, 1)
    b_shape = (nt, rt_l, bt)
    b_st = (rt_l, 1, nt * rt_l)
    c_shape = (mt, 1, rt, bt)
    c_st = (bt * rt, 0, 1, rt)
    dG, dIn = to_dev(torch, G), to_dev(torch, In)
    dOut = torch.full((mt * bt * rt,), float("nan"), dtype=torch.float32, device="cuda")
    b2g.contract5d(dG, a_shape, a_st, dIn, b_shape, b_st, dOut, c_shape, c_st)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    path = b2g.last_path()
    ref = orc.contract5d_f64(G, a_shape, a_st, In, b_shape, b_st, c_shape, c_st,
                             c_size=mt * bt * rt)
    assert_close(orc, dOut.cpu().numpy(), ref, nt * rt_l, what="reference form")
    return path


@pytest.mark.parametrize("cg,tn", VARIANTS_H, ids=VARIANT_H_IDS)
def test_contract_reference_form_small(b2g, cuda, orc, cg, tn):
    """rt=8, mt=16, nt=4, rt_l=64, bt=256: K-major B and an M-contiguous output (8-row
    store boxes)."""
    with options(b2g, cta_group=cg, tile_n=tn):
        path = _reference_form(b2g, cuda, orc, mt=16, rt=8, nt=4, rt_l=64, bt=256)
    assert path in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)


def test_contract_reference_form_medium(b2g, cuda, orc):
    """rt=64 as in the reference (mmmTensor.cpp:22), smaller mt/bt so the FP64 oracle is quick."""
    path = _reference_form(b2g, cuda, orc, mt=16, rt=64, nt=8, rt_l=128, bt=512)
    assert path in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)
